"""CPU-side checks of the boundary: the C-ABI library loads and exports every
function include/megaqwen_b200.h declares; host-side argument checks of the
torch extension; the reference-module mirror; weight/RoPE generation."""
from __future__ import annotations

import ctypes
import math
import re
from pathlib import Path

import pytest
import torch

import megaqwen_b200
from megaqwen_b200 import megakernel_decode as mkd
from megaqwen_b200 import weights as W
from megaqwen_b200.build import LIB

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "megaqwen_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(\w+)\s*\(", text, flags=re.M)
    return sorted({n for n in names if n not in ("if", "sizeof")})


def test_header_declares_reference_entry_points():
    names = declared_functions()
    for n in ("launch_ldg_decode", "launch_ldg_decode_with_logits", "mq_decode", "mq_decode_workspace_bytes",
              "mq_decode_workspace_init", "mq_decode_fetch", "mq_get_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(LIB))
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_library_host_only_calls():
    lib = ctypes.CDLL(str(LIB))
    lib.mq_decode_workspace_bytes.restype = ctypes.c_size_t
    assert lib.mq_decode_workspace_bytes() >= 256 + 2 * 8 * (4096 + 2048 + 1024 + 3072 + 1024)
    lib.mq_error_string.restype = ctypes.c_char_p
    assert lib.mq_error_string(2) == b"inter-CTA handoff wait timed out"
    lib.mq_version.restype = ctypes.c_char_p
    assert lib.mq_version().startswith(b"megaqwen_b200")
    # A null parameter block is rejected on the host, before any CUDA call.
    assert lib.mq_decode(None, None) == 1
    assert lib.mq_decode_workspace_init(None, ctypes.c_size_t(0), None) == 7


def test_struct_layout_matches_reference():
    # LDGLayerWeights: eleven pointers in the reference order (fused_decode_ldg.cu:24-36).
    text = HEADER.read_text()
    body = re.search(r"typedef struct LDGLayerWeights \{(.*?)\} LDGLayerWeights;", text, re.S).group(1)
    fields = re.findall(r"const void\* (\w+);", body)
    assert fields == ["input_layernorm_weight", "q_proj_weight", "k_proj_weight", "v_proj_weight",
                      "q_norm_weight", "k_norm_weight", "o_proj_weight", "post_attn_layernorm_weight",
                      "gate_proj_weight", "up_proj_weight", "down_proj_weight"]


def test_extension_rejects_cpu_tensors():
    w = W.make_weights(1)
    cos, sin = W.rope_tables(64)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        megaqwen_b200.MegakernelDecoder(w.embed, w.layer_weights_flat(), w.final_norm, w.lm_head, cos, sin, 1, 64)
    with pytest.raises(RuntimeError, match="num_layers"):
        megaqwen_b200.MegakernelDecoder(w.embed, [], w.final_norm, w.lm_head, cos, sin, 0, 64)
    with pytest.raises(RuntimeError, match="init_ldg"):
        megaqwen_b200.decode_ldg(1, w.final_norm, w.lm_head, cos, sin, cos, cos, cos, cos, cos, cos, cos, cos, cos,
                                 cos, cos, cos, cos, 1, 0, 1, 64)


def test_weights_prefix_and_determinism():
    a = W.make_weights(2, cache=False)
    b = W.make_weights(1, cache=False)
    assert torch.equal(a.embed, b.embed)
    for k in W.LAYER_KEYS:
        assert torch.equal(a.layers[0][k], b.layers[0][k])
    assert a.layers[0]["q_proj"].dtype == torch.bfloat16
    assert torch.all(a.layers[1]["q_norm"] == 1)
    std = a.layers[1]["down_proj"].float().std().item()
    assert abs(std - 0.02) < 1e-3
    flat = a.layer_weights_flat()
    assert len(flat) == 22 and flat[11] is a.layers[1]["input_layernorm"]
    lists = a.layer_weight_lists()
    assert len(lists) == 11 and lists[1][1] is a.layers[1]["q_proj"]


def test_rope_tables_match_reference_formula():
    cos, sin = W.rope_tables(100)
    p, i = 37, 5
    ang = p * (1.0 / (1e6 ** (2 * i / 128)))
    assert abs(cos[p, i].item() - math.cos(ang)) < 1e-2
    assert torch.equal(cos[:, :64], cos[:, 64:])
    assert sin.dtype == torch.bfloat16 and sin.shape == (100, 128)


def test_seeded_prompt():
    p = W.seeded_prompt(8)
    assert p.dtype == torch.int32 and p.shape == (8,)
    assert torch.equal(p, W.seeded_prompt(8))
    assert int(p.min()) >= 0 and int(p.max()) < W.VOCAB_SIZE


def test_reference_module_mirror():
    for fn in (mkd._compile_decode_kernel, mkd._compile_prefill_kernel, mkd._compile_fused_prefill_kernel):
        m = fn()
        assert hasattr(m, "MegakernelDecoder") and hasattr(m, "MegakernelPrefillDecoder")
    assert mkd.HIDDEN_SIZE == 1024 and mkd.VOCAB_SIZE == 151936
    wd = mkd.load_qwen3_weights(num_layers=1, max_seq_len=16, device="cpu")
    assert set(wd) >= {"embed_weight", "layer_weights", "final_norm_weight", "lm_head_weight", "cos_table",
                       "sin_table", "tokenizer"}
    assert len(wd["layer_weights"]) == 11
