"""mq_decode_noalloc: the decode step for callers that cannot allocate device
memory (code running under an allocator or memory pool that owns all device
memory, or with a fixed workspace budget), checked through the C ABI against
mq_decode with a caller-allocated workspace, on two consecutive steps.

This file is collected last on purpose: the entry point keeps its scratch in a
static device array shared by all calls, and the test must pass both alone in
a fresh process and after every other test.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

LOGIT_MAX_ABS = 1e-3      # same engine, same inputs: only summation order may differ


class LayerWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "input_layernorm_weight", "q_proj_weight", "k_proj_weight", "v_proj_weight", "q_norm_weight",
        "k_norm_weight", "o_proj_weight", "post_attn_layernorm_weight", "gate_proj_weight", "up_proj_weight",
        "down_proj_weight")]


class DecodeParams(ctypes.Structure):
    _fields_ = [
        ("input_token", ctypes.c_int), ("input_token_ptr", ctypes.c_void_p), ("output_token", ctypes.c_void_p),
        ("logits", ctypes.c_void_p), ("embed", ctypes.c_void_p), ("layers", ctypes.c_void_p),
        ("final_norm", ctypes.c_void_p), ("lm_head", ctypes.c_void_p), ("cos_table", ctypes.c_void_p),
        ("sin_table", ctypes.c_void_p), ("k_cache", ctypes.c_void_p), ("v_cache", ctypes.c_void_p),
        ("hidden_out", ctypes.c_void_p), ("normalized_out", ctypes.c_void_p), ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t), ("num_layers", ctypes.c_int), ("position", ctypes.c_int),
        ("position_ptr", ctypes.c_void_p), ("max_seq_len", ctypes.c_int), ("attn_scale", ctypes.c_float),
        ("num_ctas", ctypes.c_int), ("attn_chunk", ctypes.c_int), ("timeout_ns", ctypes.c_longlong),
        ("inject_skip_cta", ctypes.c_int), ("trace", ctypes.c_void_p), ("host_result", ctypes.c_void_p),
        ("host_seq", ctypes.c_uint), ("tp_rank", ctypes.c_int), ("tp_size", ctypes.c_int),
        ("peer_workspaces", ctypes.c_void_p),
    ]


def _lib():
    from megaqwen_b200.build import LIB
    lib = ctypes.CDLL(str(LIB))
    for name in ("mq_decode", "mq_decode_noalloc"):
        getattr(lib, name).argtypes = [ctypes.POINTER(DecodeParams), ctypes.c_void_p]
        getattr(lib, name).restype = ctypes.c_int
    lib.mq_decode_noalloc_reset.argtypes = [ctypes.c_void_p]
    lib.mq_decode_noalloc_fetch.argtypes = [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_uint32),
                                            ctypes.POINTER(ctypes.c_uint32), ctypes.c_void_p]
    lib.mq_decode_workspace_bytes.restype = ctypes.c_size_t
    lib.mq_last_error_detail.restype = ctypes.c_char_p
    return lib


def test_noalloc_matches_allocating_entry_point():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    from megaqwen_b200.weights import make_weights, rope_tables

    lib = _lib()
    L, S = 2, 64
    w = make_weights(L).to("cuda")
    cos, sin = rope_tables(S, device="cuda")
    table = (LayerWeights * L)()
    for i, layer in enumerate(w.layers):
        table[i] = LayerWeights(*[layer[k].data_ptr() for k in (
            "input_layernorm", "q_proj", "k_proj", "v_proj", "q_norm", "k_norm", "o_proj",
            "post_attention_layernorm", "gate_proj", "up_proj", "down_proj")])
    d_table = torch.frombuffer(bytearray(bytes(table)), dtype=torch.uint8).to("cuda")

    def buffers():
        kc = torch.zeros(L, 8, S, 128, dtype=torch.bfloat16, device="cuda")
        return {"k": kc, "v": torch.zeros_like(kc), "tok": torch.full((1,), -1, dtype=torch.int32, device="cuda"),
                "logits": torch.empty(151936, dtype=torch.float32, device="cuda")}

    def params(buf, token, position, workspace=None, ws_bytes=0):
        p = DecodeParams()
        p.input_token = token
        p.output_token = buf["tok"].data_ptr()
        p.logits = buf["logits"].data_ptr()
        p.embed = w.embed.data_ptr()
        p.layers = d_table.data_ptr()
        p.final_norm = w.final_norm.data_ptr()
        p.lm_head = w.lm_head.data_ptr()
        p.cos_table = cos.data_ptr()
        p.sin_table = sin.data_ptr()
        p.k_cache = buf["k"].data_ptr()
        p.v_cache = buf["v"].data_ptr()
        p.workspace = workspace
        p.workspace_bytes = ws_bytes
        p.num_layers = L
        p.position = position
        p.max_seq_len = S
        p.attn_scale = 128 ** -0.5
        return p

    stream = torch.cuda.current_stream().cuda_stream
    ws = torch.zeros(lib.mq_decode_workspace_bytes(), dtype=torch.uint8, device="cuda")
    ref, new = buffers(), buffers()
    for position, token in enumerate([17, 4242]):           # two calls in a row
        rc = lib.mq_decode(ctypes.byref(params(ref, token, position, ws.data_ptr(), ws.numel())), stream)
        assert rc == 0, lib.mq_last_error_detail()
        rc = lib.mq_decode_noalloc(ctypes.byref(params(new, token, position)), stream)
        assert rc == 0, lib.mq_last_error_detail()
        torch.cuda.synchronize()
        assert int(new["tok"].item()) == int(ref["tok"].item()) >= 0
        err = (new["logits"] - ref["logits"]).abs().max().item()
        assert err <= LOGIT_MAX_ABS, f"step {position}: logits max-abs {err}"
        assert torch.equal(new["k"][:, :, position], ref["k"][:, :, position])

    # sizes beyond the static scratch are refused on the host
    bad = params(new, 1, 2)
    bad.num_ctas = 1000
    assert lib.mq_decode_noalloc(ctypes.byref(bad), stream) == 1
    assert b"static scratch" in lib.mq_last_error_detail()

    # A device-side input error (token read from device memory, out of range)
    # is recorded in the static scratch and blocks later steps until the
    # caller clears it with mq_decode_noalloc_reset; then a step succeeds and
    # still matches the allocating entry point.
    tok_err, err, info = ctypes.c_int(0), ctypes.c_uint32(0), ctypes.c_uint32(0)
    bad_tok = torch.full((1,), -5, dtype=torch.int32, device="cuda")
    p = params(new, 0, 2)
    p.input_token_ptr = bad_tok.data_ptr()
    assert lib.mq_decode_noalloc(ctypes.byref(p), stream) == 0
    assert lib.mq_decode_noalloc_fetch(ctypes.byref(tok_err), ctypes.byref(err), ctypes.byref(info), stream) == 0
    assert err.value == 4 and ctypes.c_int32(info.value).value == -5       # MQ_ERR_BAD_TOKEN, the token
    assert lib.mq_decode_noalloc_reset(stream) == 0
    rc = lib.mq_decode(ctypes.byref(params(ref, 99, 2, ws.data_ptr(), ws.numel())), stream)
    assert rc == 0, lib.mq_last_error_detail()
    assert lib.mq_decode_noalloc(ctypes.byref(params(new, 99, 2)), stream) == 0
    assert lib.mq_decode_noalloc_fetch(ctypes.byref(tok_err), ctypes.byref(err), ctypes.byref(info), stream) == 0
    torch.cuda.synchronize()
    assert err.value == 0
    assert tok_err.value == int(new["tok"].item()) == int(ref["tok"].item())
    assert (new["logits"] - ref["logits"]).abs().max().item() <= LOGIT_MAX_ABS
