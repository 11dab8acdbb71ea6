"""Generate golden vectors by running the reference's own PyTorch forward.

Runs ``demo_e2e.Qwen3Model(..., Backend.TORCH)`` from a MegaQwen checkout
(path given by ``--reference`` or ``$MEGAQWEN_REF``) on CPU in fp32, on the
seeded synthetic weights of ``megaqwen_b200.weights``, and stores the results
under ``tests/golden/``.  The reference cannot travel to the GPU hosts, so the
outputs are committed; this script is how they were made.

Cases
-----
``config1_l28``  BASELINE config 1: 28 layers, 8-token prompt of uniform ids
                 (seed 0), prefill, then 32 greedy decode steps.
``long_l2``      2 layers, 200-token prompt (seed 1), prefill, then 16 greedy
                 decode steps: attention over longer caches.

For each step the file keeps the greedy token, the top-256 logits (values and
ids, fp32), the logit sum / sum of squares / max, and for a few steps the full
logit vector in fp16.  It also keeps the bf16 K/V cache rows (as int16 bit patterns) of selected
positions.
"""
from __future__ import annotations

import argparse
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from megaqwen_b200.weights import make_weights, seeded_prompt  # noqa: E402

TOPK = 256


class _StateDictShim:
    """Minimal stand-in for a Hugging Face model: ``Qwen3Model.__init__`` only
    calls ``.parameters()`` (for the device) and ``.state_dict()``
    (demo_e2e.py:370-379)."""

    def __init__(self, sd):
        self._sd = sd

    def state_dict(self):
        return self._sd

    def parameters(self):
        return iter(self._sd.values())


def run_case(demo, name, num_layers, prompt_len, prompt_seed, steps, full_steps):
    w = make_weights(num_layers)
    sd = {k: v.float() for k, v in w.state_dict().items()}
    cfg = demo.Qwen3Config(num_hidden_layers=num_layers)
    cfg.max_position_embeddings = 4096
    model = demo.Qwen3Model(_StateDictShim(sd), cfg, demo.Backend.TORCH)
    model.dtype = torch.bfloat16
    prompt = seeded_prompt(prompt_len, seed=prompt_seed).long().view(1, -1)
    t0 = time.time()
    with torch.no_grad():
        logits, kv, cache_len = model.prefill(prompt)
        step_logits = [logits[0, -1].clone()]
        tok = int(torch.argmax(step_logits[-1]))
        toks = [tok]
        for i in range(steps):
            lg, kv = model.decode_step(torch.tensor([[tok]]), kv, cache_len + i)
            step_logits.append(lg[0, -1].clone())
            tok = int(torch.argmax(step_logits[-1]))
            toks.append(tok)
    dt = time.time() - t0
    L = torch.stack(step_logits)                          # [steps+1, V]
    top = torch.topk(L, TOPK, dim=-1)
    # K/V rows of a few positions in the reference megakernel layout [L,8,S,128].
    sel_pos = sorted({0, prompt_len - 1, prompt_len, prompt_len + steps - 1})
    kc = torch.stack([kv[li][0][0, :, sel_pos] for li in range(num_layers)])   # [L,8,P,128]
    vc = torch.stack([kv[li][1][0, :, sel_pos] for li in range(num_layers)])
    out = {
        "prompt": prompt.view(-1).numpy().astype(np.int32),
        "tokens": np.array(toks, dtype=np.int32),
        "top_vals": top.values.numpy().astype(np.float32),
        "top_ids": top.indices.numpy().astype(np.int32),
        "logit_sum": L.sum(-1).numpy().astype(np.float64),
        "logit_sumsq": (L.double() ** 2).sum(-1).numpy(),
        "logit_max": L.max(-1).values.numpy().astype(np.float32),
        "full_steps": np.array(full_steps, dtype=np.int32),
        "full_logits_f16": L[full_steps].numpy().astype(np.float16),
        "kv_positions": np.array(sel_pos, dtype=np.int32),
        "k_rows_bf16": kc.to(torch.bfloat16).view(torch.int16).numpy(),
        "v_rows_bf16": vc.to(torch.bfloat16).view(torch.int16).numpy(),
        "num_layers": np.int32(num_layers),
    }
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"{name}: {num_layers} layers, prompt {prompt_len}, {steps} steps in {dt:.1f}s; tokens {toks[:8]}...")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MEGAQWEN_REF", ""))
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <MegaQwen checkout> or set MEGAQWEN_REF")
    sys.path.insert(0, args.reference)
    torch.set_num_threads(os.cpu_count() or 1)
    import demo_e2e as demo  # the reference's own forward

    run_case(demo, "config1_l28", 28, 8, 0, 32, [0, 1, 32])
    run_case(demo, "long_l2", 2, 200, 1, 16, [0, 16])


if __name__ == "__main__":
    main()
