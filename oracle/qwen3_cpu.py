"""CPU oracle for the Qwen3-0.6B decode/prefill hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker or the timed CPU baseline.  The product path
(``megaqwen_b200``) never imports it and has no CPU fallback.

What it restates: the reference's pure-PyTorch forward, ``demo_e2e.py``
``Qwen3Model`` with ``Backend.TORCH`` on fp32 weights, which is the correctness
standard the decode megakernel is measured against.  Numerics contract of that
path (fp32 weights on CPU):

* activations, residual stream, norms, projections, softmax and MLP in fp32;
* K/V caches in bf16 (``demo_e2e.py:371,395-398``), so decode attention reads
  bf16-rounded K/V for *every* position including the current one
  (``demo_e2e.py:298-300`` writes the row, then ``:300`` attends over the cache);
* prefill attention uses the unrounded fp32 K/V of the prompt
  (``demo_e2e.py:282-294``) and writes bf16 copies into the cache;
* RoPE tables in bf16 (``demo_e2e.py:169-177``), applied rotate-half in fp32
  (``demo_e2e.py:180-195``);
* RMSNorm ``x * rsqrt(mean(x^2) + eps) * w`` in fp32 (``demo_e2e.py:37-53``);
  the reference sums the squares sequentially in a Python loop; this
  restatement uses a vectorised fp32 sum (differences are in the last ulp);
* logits ``= final_norm(h) @ embed^T`` (tied head, ``demo_e2e.py:375,402,413``).

Parity pin: ``tests/golden/`` holds outputs of the reference's own
``demo_e2e.Qwen3Model(Backend.TORCH)`` run on the same seeded weights
(``tests/golden/make_golden.py`` imported the reference to make them), and
``tests/test_oracle_golden.py`` checks this module against them.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from megaqwen_b200.weights import (
    HEAD_DIM, HIDDEN_SIZE, NUM_KV_HEADS, NUM_Q_HEADS, RMS_NORM_EPS, Qwen3Weights, rope_tables,
)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = RMS_NORM_EPS) -> torch.Tensor:
    """demo_e2e.py:37-53 (torch_rms_norm_sequential), fp32."""
    var = (x * x).mean(dim=-1, keepdim=True)
    return x * torch.rsqrt(var + eps) * w


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE (demo_e2e.py:180-195).  ``cos``/``sin``: bf16 rows
    broadcastable to ``x[..., :]``; math in fp32."""
    half = x.shape[-1] // 2
    c = cos.float()[..., :half]
    s = sin.float()[..., :half]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


class Qwen3CpuOracle:
    """fp32 CPU restatement of ``demo_e2e.Qwen3Model`` (Backend.TORCH).

    Keeps its own bf16 KV caches in the reference megakernel's layout
    ``[num_layers, 8, max_seq_len, 128]`` so tests can compare them with the
    device caches directly.
    """

    def __init__(self, weights: Qwen3Weights, max_seq_len: int = 2048, num_threads: Optional[int] = None):
        if num_threads is not None:
            torch.set_num_threads(num_threads)
        self.num_layers = weights.num_layers
        self.max_seq_len = max_seq_len
        self.embed = weights.embed.float()
        self.final_norm = weights.final_norm.float()
        self.layers = [{k: v.float() for k, v in layer.items()} for layer in weights.layers]
        self.cos, self.sin = rope_tables(max_seq_len)
        self.k_cache = torch.zeros(self.num_layers, NUM_KV_HEADS, max_seq_len, HEAD_DIM, dtype=torch.bfloat16)
        self.v_cache = torch.zeros_like(self.k_cache)
        self.scale = 1.0 / math.sqrt(HEAD_DIM)
        self.last_hidden = None

    def reset(self):
        self.k_cache.zero_()
        self.v_cache.zero_()

    # -- one transformer layer (demo_e2e.py:351-362, :266-304, :324-328) --------
    def _layer(self, li: int, h: torch.Tensor, positions: torch.Tensor, prefill: bool) -> torch.Tensor:
        w = self.layers[li]
        S = h.shape[0]
        x = rms_norm(h, w["input_layernorm"])
        q = (x @ w["q_proj"].T).view(S, NUM_Q_HEADS, HEAD_DIM).transpose(0, 1)      # [16,S,128]
        k = (x @ w["k_proj"].T).view(S, NUM_KV_HEADS, HEAD_DIM).transpose(0, 1)     # [8,S,128]
        v = (x @ w["v_proj"].T).view(S, NUM_KV_HEADS, HEAD_DIM).transpose(0, 1)
        q = rms_norm(q, w["q_norm"])
        k = rms_norm(k, w["k_norm"])
        cos = self.cos[positions].unsqueeze(0)
        sin = self.sin[positions].unsqueeze(0)
        q = rope(q, cos, sin)
        k = rope(k, cos, sin)
        groups = NUM_Q_HEADS // NUM_KV_HEADS
        if prefill:
            # demo_e2e.py:282-297: causal attention on the fp32 K/V, then cache write.
            kk = k.repeat_interleave(groups, dim=0)
            vv = v.repeat_interleave(groups, dim=0)
            scores = (q @ kk.transpose(-1, -2)) * self.scale
            mask = torch.triu(torch.ones(S, S, dtype=torch.bool), diagonal=1)
            scores = scores.masked_fill(mask, float("-inf"))
            attn = torch.softmax(scores, dim=-1) @ vv                                  # [16,S,128]
            p0 = int(positions[0])
            self.k_cache[li, :, p0:p0 + S] = k.to(torch.bfloat16)
            self.v_cache[li, :, p0:p0 + S] = v.to(torch.bfloat16)
        else:
            # demo_e2e.py:298-300 + :198-211: write bf16 row, attend over bf16 cache.
            p = int(positions[0])
            self.k_cache[li, :, p] = k[:, 0].to(torch.bfloat16)
            self.v_cache[li, :, p] = v[:, 0].to(torch.bfloat16)
            kc = self.k_cache[li, :, : p + 1].float().repeat_interleave(groups, dim=0)   # [16,L,128]
            vc = self.v_cache[li, :, : p + 1].float().repeat_interleave(groups, dim=0)
            scores = (q @ kc.transpose(-1, -2)) * self.scale
            attn = torch.softmax(scores, dim=-1) @ vc
        attn = attn.transpose(0, 1).reshape(S, NUM_Q_HEADS * HEAD_DIM)
        h = h + attn @ w["o_proj"].T
        x = rms_norm(h, w["post_attention_layernorm"])
        gate = x @ w["gate_proj"].T
        up = x @ w["up_proj"].T
        h = h + (F.silu(gate) * up) @ w["down_proj"].T
        return h

    @torch.no_grad()
    def forward(self, token_ids, start_pos: int, prefill: bool, all_logits: bool = False) -> torch.Tensor:
        ids = torch.as_tensor(token_ids, dtype=torch.long).view(-1)
        S = ids.numel()
        if start_pos + S > self.max_seq_len:
            raise ValueError("position exceeds max_seq_len")
        h = self.embed[ids]
        positions = torch.arange(start_pos, start_pos + S)
        for li in range(self.num_layers):
            if prefill:
                h = self._layer(li, h, positions, True)
            else:
                rows = [self._layer(li, h[i:i + 1], positions[i:i + 1], False) for i in range(S)]
                h = torch.cat(rows, 0)
        self.last_hidden = h[-1].clone()
        x = rms_norm(h if all_logits else h[-1:], self.final_norm)
        return x @ self.embed.T                                                        # fp32 logits

    def prefill(self, token_ids, all_logits: bool = False) -> torch.Tensor:
        """``Qwen3Model.prefill`` (demo_e2e.py:390-403): positions ``0..S-1``."""
        return self.forward(token_ids, 0, True, all_logits)

    def decode_step(self, token_id: int, position: int) -> torch.Tensor:
        """``Qwen3Model.decode_step`` (demo_e2e.py:405-415): one token at ``position``."""
        return self.forward([int(token_id)], position, False)[0]

    def greedy(self, prompt, steps: int, use_prefill: bool = True):
        """Prompt then ``steps`` greedy tokens; returns (tokens, per-step logits list).

        ``use_prefill=False`` runs the prompt token by token through decode,
        the way ``MegakernelGenerator.generate`` does (megakernel_decode.py:1166-1167).
        """
        prompt = [int(t) for t in prompt]
        self.reset()
        if use_prefill:
            logits = self.prefill(prompt)[-1]
        else:
            for i, t in enumerate(prompt):
                logits = self.decode_step(t, i)
        pos = len(prompt)
        out_tokens, out_logits = [], [logits]
        tok = int(torch.argmax(logits))
        out_tokens.append(tok)
        for _ in range(steps):
            logits = self.decode_step(tok, pos)
            pos += 1
            out_logits.append(logits)
            tok = int(torch.argmax(logits))
            out_tokens.append(tok)
        return out_tokens, out_logits
