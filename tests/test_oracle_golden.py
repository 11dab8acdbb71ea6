"""The CPU oracle against golden vectors produced by the reference's own
PyTorch forward (demo_e2e.Qwen3Model, Backend.TORCH; see tests/golden/make_golden.py).

Tolerances: the north-star bar for logits (max-abs 3e-2, cosine >= 0.9995);
the oracle is in fact within ~2e-3 of the reference because both are fp32 and
differ only in summation order.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from megaqwen_b200.weights import make_weights
from oracle.qwen3_cpu import Qwen3CpuOracle

LOGIT_MAX_ABS = 3e-2
COSINE_MIN = 0.9995


def _load(golden_dir, name):
    return dict(np.load(golden_dir / f"{name}.npz"))


@pytest.mark.parametrize("name", ["long_l2", "config1_l28"])
def test_oracle_matches_reference_forward(golden_dir, name):
    g = _load(golden_dir, name)
    w = make_weights(int(g["num_layers"]))
    o = Qwen3CpuOracle(w, max_seq_len=512)
    steps = len(g["tokens"]) - 1
    toks, logits = o.greedy(g["prompt"], steps)
    assert toks == [int(t) for t in g["tokens"]]
    L = torch.stack(logits)
    top_ids = torch.from_numpy(g["top_ids"]).long()
    mine = torch.gather(L, 1, top_ids)
    assert (mine - torch.from_numpy(g["top_vals"])).abs().max().item() < 5e-3
    full = torch.from_numpy(g["full_logits_f16"].astype(np.float32))
    ours = L[torch.from_numpy(g["full_steps"]).long()]
    assert (ours - full).abs().max().item() < LOGIT_MAX_ABS
    cos = torch.nn.functional.cosine_similarity(ours, full, dim=-1)
    assert cos.min().item() > COSINE_MIN
    np.testing.assert_allclose(L.double().sum(-1).numpy(), g["logit_sum"], rtol=0, atol=0.5)
    np.testing.assert_allclose((L.double() ** 2).sum(-1).numpy(), g["logit_sumsq"], rtol=1e-4)
    # bf16 K/V cache rows: identical except rare 1-ulp rounding flips.
    pos = torch.from_numpy(g["kv_positions"]).long()
    for key, cache in (("k_rows_bf16", o.k_cache), ("v_rows_bf16", o.v_cache)):
        ref = torch.from_numpy(g[key]).view(torch.bfloat16)
        got = cache[:, :, pos]
        assert (got == ref).float().mean().item() > 0.9
        assert (got.float() - ref.float()).abs().max().item() <= 0.0625


def test_decode_only_prompt_matches_prefill_tokens(golden_dir):
    """Running the prompt through decode (MegakernelGenerator's way) gives the
    same greedy continuation on the short-prompt case."""
    g = _load(golden_dir, "long_l2")
    w = make_weights(2)
    o = Qwen3CpuOracle(w, max_seq_len=512)
    toks, _ = o.greedy(g["prompt"][:32], 4, use_prefill=False)
    toks2, _ = o.greedy(g["prompt"][:32], 4, use_prefill=True)
    assert toks == toks2
