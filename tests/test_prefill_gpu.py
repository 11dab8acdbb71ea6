"""Tensor-core prefill (tcgen05 GEMMs + flash attention) against the CPU
oracle's prefill (the reference PyTorch forward, demo_e2e.py:390-403).

The prefill rounds GEMM and attention operands to bf16 (the reference's own
cuBLAS prefill keeps every intermediate in bf16, fused_prefill.cu:601-867);
the oracle is fp32.  Bar: last-position logits max-abs <= 3e-2 and cosine
>= 0.9995 (the north-star logits tolerance); greedy token equal unless the
oracle's top-2 gap is below the observed error; K/V cache rows within bf16
rounding of the oracle's."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tests.test_decode_gpu import (COSINE_MIN, LOGIT_MAX_ABS, assert_logits_close, assert_token_consistent,
                                   dev_weights, make_decoder, make_oracle)

pytestmark = pytest.mark.gpu


def _cache_rel_err(dev_cache, ref_cache, upto):
    got = dev_cache[:, :, :upto].float().cpu()
    ref = ref_cache[:, :, :upto].float()
    return ((got - ref).abs().max() / ref.abs().max().clamp_min(1e-6)).item()


@pytest.mark.parametrize("num_layers,S", [(2, 1), (2, 8), (2, 200), (1, 2048), (28, 64)])
def test_prefill_matches_oracle(num_layers, S):
    from megaqwen_b200.weights import seeded_prompt
    ids = seeded_prompt(S, seed=5)
    dec = make_decoder(num_layers, S + 16, cls="MegakernelPrefillDecoder", max_prefill_len=S)
    o = make_oracle(num_layers, S + 16)
    tok, logits = dec.prefill_step_with_logits(ids)
    ref = o.prefill(ids.tolist())[-1]
    assert_logits_close(logits, ref, f"L={num_layers} S={S}")
    assert_token_consistent(tok, logits, ref, "prefill token")
    assert dec.position() == S
    assert _cache_rel_err(dec.get_k_cache(), o.k_cache, S) < 0.05
    assert _cache_rel_err(dec.get_v_cache(), o.v_cache, S) < 0.05
    # decode continues from the prefilled cache
    t2, lg2 = dec.decode_step_with_logits(tok)
    ref2 = o.decode_step(tok, S)
    assert_logits_close(lg2, ref2, "decode after prefill")


def test_prefill_batch_matches_single_sequences():
    import megaqwen_b200
    from megaqwen_b200.weights import rope_tables, seeded_prompt
    L, S, B, MS = 2, 96, 3, 128
    _, wd = dev_weights(L)
    cos, sin = rope_tables(MS, device="cuda")
    ids = torch.stack([seeded_prompt(S, seed=10 + b) for b in range(B)]).cuda()
    kc = torch.zeros(B, L, 8, MS, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    logits = torch.empty(B, 151936, device="cuda")
    toks = megaqwen_b200._C.prefill_batch(wd.embed, wd.layer_weights_flat(), wd.final_norm, wd.lm_head, cos, sin,
                                          ids, kc, vc, logits).cpu().tolist()
    for b in range(B):
        dec = make_decoder(L, MS, cls="MegakernelPrefillDecoder", max_prefill_len=S)
        tok, lg = dec.prefill_step_with_logits(ids[b].cpu())
        assert tok == toks[b]
        assert (lg - logits[b]).abs().max().item() < 1e-3
        assert torch.equal(dec.get_k_cache()[:, :, :S], kc[b, :, :, :S])


def test_prefill_batch_above_128_sequences():
    """Batches above 128 sequences take the fp32-logits LM-head GEMM and the
    two-stage argmax (64 blocks per sequence, then one reduction block); up to
    128 the small-batch GEMM with the argmax fused.  A 130-sequence batch
    against the same prompts in batches of 128 and 2: logits agree, and each
    path's tokens are the first index of its own row maximum."""
    import megaqwen_b200
    from megaqwen_b200.weights import rope_tables, seeded_prompt
    L, S, B, MS = 1, 16, 130, 32
    _, wd = dev_weights(L)
    cos, sin = rope_tables(MS, device="cuda")
    ids = torch.stack([seeded_prompt(S, seed=300 + b) for b in range(B)]).cuda()

    def run(rows):
        n = len(rows)
        kc = torch.zeros(n, L, 8, MS, 128, dtype=torch.bfloat16, device="cuda")
        vc = torch.zeros_like(kc)
        lg = torch.empty(n, 151936, device="cuda")
        tk = megaqwen_b200._C.prefill_batch(wd.embed, wd.layer_weights_flat(), wd.final_norm, wd.lm_head, cos, sin,
                                            ids[rows].contiguous(), kc, vc, lg)
        torch.cuda.synchronize()
        return tk.cpu(), lg

    big_t, big_l = run(list(range(B)))
    small = [run(list(range(128))), run([128, 129])]
    small_t = torch.cat([t for t, _ in small])
    small_l = torch.cat([lg for _, lg in small])
    assert (big_l - small_l).abs().max().item() < 1e-3
    assert torch.equal(big_t, torch.argmax(big_l, dim=1).cpu().to(big_t.dtype))
    assert torch.equal(small_t, torch.argmax(small_l, dim=1).cpu().to(small_t.dtype))
    top2 = torch.topk(small_l, 2, dim=1).values
    clear = (top2[:, 0] - top2[:, 1]).cpu() > 1e-3
    assert torch.equal(big_t[clear], small_t[clear])


def test_config4_shape_batch8():
    """BASELINE config 4 shape on 2 layers: batch 8, prompt 2048, then decode."""
    import megaqwen_b200
    from megaqwen_b200.weights import rope_tables, seeded_prompt
    L, S, B, MS = 2, 2048, 8, 2048 + 32
    _, wd = dev_weights(L)
    cos, sin = rope_tables(MS, device="cuda")
    ids = torch.stack([seeded_prompt(S, seed=100 + b) for b in range(B)]).cuda()
    kc = torch.zeros(B, L, 8, MS, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    logits = torch.empty(B, 151936, device="cuda")
    toks = megaqwen_b200._C.prefill_batch(wd.embed, wd.layer_weights_flat(), wd.final_norm, wd.lm_head, cos, sin,
                                          ids, kc, vc, logits).cpu().tolist()
    o = make_oracle(L, MS)
    for b in (0, 7):
        ref = o.prefill(ids[b].cpu().tolist())[-1]
        assert_logits_close(logits[b], ref, f"seq {b}")
        assert_token_consistent(toks[b], logits[b], ref, f"seq {b}")


def test_reference_launch_prefill_float_abi():
    """launch_prefill_float (the reference's prefill launcher signature, host
    layer array, ignored scratch and cuBLAS handle) through the C ABI."""
    from megaqwen_b200.build import LIB
    from megaqwen_b200.weights import LAYER_KEYS, rope_tables, seeded_prompt
    lib = ctypes.CDLL(str(LIB))
    L, S, MS = 2, 40, 64
    _, wd = dev_weights(L)
    cos, sin = rope_tables(MS, device="cuda")
    ids = seeded_prompt(S, seed=3).cuda()
    table = (ctypes.c_void_p * (11 * L))(*[wd.layers[i][k].data_ptr() for i in range(L) for k in LAYER_KEYS])
    kc = torch.zeros(L, 8, MS, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    V = ctypes.c_void_p
    lib.launch_prefill_float.argtypes = [V, V, ctypes.c_int, V, V, V, V, V, V, V, V] + [V] * 17 + \
        [ctypes.c_int, ctypes.c_int, ctypes.c_float, V, V]
    lib.launch_prefill_float(ids.data_ptr(), out.data_ptr(), S, wd.embed.data_ptr(), ctypes.cast(table, V),
                             wd.final_norm.data_ptr(), wd.lm_head.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                             kc.data_ptr(), vc.data_ptr(), *([None] * 17), L, MS, 128 ** -0.5, None,
                             torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert lib.mq_prefill_get_last_error() == 0
    dec = make_decoder(L, MS, cls="MegakernelPrefillDecoder", max_prefill_len=S)
    assert int(out.item()) == dec.prefill_step(ids.cpu())
    assert torch.equal(kc[:, :, :S], dec.get_k_cache()[:, :, :S])


def test_reference_launch_prefill_megakernel_abi():
    """launch_prefill_megakernel (the reference's short-prompt launcher: DEVICE
    layer table, fp32 scratch accepted and ignored) gives the prefill
    decoder's token and cache rows."""
    from megaqwen_b200.build import LIB
    from megaqwen_b200.weights import LAYER_KEYS, rope_tables, seeded_prompt
    lib = ctypes.CDLL(str(LIB))
    L, S, MS = 2, 48, 64
    _, wd = dev_weights(L)
    cos, sin = rope_tables(MS, device="cuda")
    ids = seeded_prompt(S, seed=8).cuda()
    table = torch.tensor([wd.layers[i][k].data_ptr() for i in range(L) for k in LAYER_KEYS], dtype=torch.int64,
                         device="cuda")
    kc = torch.zeros(L, 8, MS, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    out = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    V = ctypes.c_void_p
    lib.launch_prefill_megakernel.argtypes = [V, V, ctypes.c_int] + [V] * 8 + [V] * 12 + \
        [ctypes.c_int, ctypes.c_int, ctypes.c_float, V]
    lib.launch_prefill_megakernel(ids.data_ptr(), out.data_ptr(), S, wd.embed.data_ptr(), table.data_ptr(),
                                  wd.final_norm.data_ptr(), wd.lm_head.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                  kc.data_ptr(), vc.data_ptr(), *([None] * 12), L, MS, 128 ** -0.5,
                                  torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert lib.mq_prefill_get_last_error() == 0
    dec = make_decoder(L, MS, cls="MegakernelFusedPrefillDecoder", max_prefill_len=S)
    assert int(out.item()) == dec.prefill_step(ids.cpu())
    assert torch.equal(kc[:, :, :S], dec.get_k_cache()[:, :, :S])
    assert torch.equal(vc[:, :, :S], dec.get_v_cache()[:, :, :S])
