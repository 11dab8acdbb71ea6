"""ctypes driver for the reference decode megakernel built for sm_100a.

TEST AND BENCHMARK INFRASTRUCTURE ONLY (the comparator, never the product).
Loads ``oracle/_ref/libref_ldg_decode.so`` (made by ``oracle/build_ref.py``
from the reference's unchanged ``csrc/megakernel/fused_decode_ldg.cu``) and
drives it through its own launcher ``launch_ldg_decode``
(fused_decode_ldg.cu:893-969): the cooperative 82 x 256 grid.sync kernel, then
``ldg_lm_head_phase1`` (1184 blocks) and ``ldg_lm_head_phase2``.  Buffers follow
the reference's own allocation (megakernel_decode.py:137-159): bf16 caches
``[L, 8, max_seq, 128]``, bf16 hidden buffer, fp32 scratch vectors and the
1184-entry argmax scratch.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

LIB = Path(__file__).resolve().parent / "_ref" / "libref_ldg_decode.so"
LAYER_KEYS = ("input_layernorm", "q_proj", "k_proj", "v_proj", "q_norm", "k_norm", "o_proj",
              "post_attention_layernorm", "gate_proj", "up_proj", "down_proj")


class _LayerWeights(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in (
        "input_layernorm_weight", "q_proj_weight", "k_proj_weight", "v_proj_weight", "q_norm_weight",
        "k_norm_weight", "o_proj_weight", "post_attn_layernorm_weight", "gate_proj_weight", "up_proj_weight",
        "down_proj_weight")]


class RefLdgDecoder:
    """The reference's decode step on device-resident weights (``Qwen3Weights``
    already on the GPU) with its own caches and scratch."""

    def __init__(self, wd, cos, sin, num_layers: int, max_seq_len: int):
        if not LIB.exists():
            raise FileNotFoundError(f"{LIB} is not built (oracle/build_ref.py)")
        self.lib = ctypes.CDLL(str(LIB))
        self.lib.launch_ldg_decode.restype = None
        self.lib.launch_ldg_decode.argtypes = (
            [ctypes.c_int, ctypes.c_void_p] + [ctypes.c_void_p] * 19 + [ctypes.c_int] * 4 +
            [ctypes.c_float, ctypes.c_void_p])
        dev = wd.embed.device
        self.wd, self.cos, self.sin = wd, cos, sin
        self.L, self.S = num_layers, max_seq_len
        table = (_LayerWeights * num_layers)()
        for i in range(num_layers):
            table[i] = _LayerWeights(*[wd.layers[i][k].data_ptr() for k in LAYER_KEYS])
        self.d_table = torch.frombuffer(bytearray(bytes(table)), dtype=torch.uint8).to(dev)
        self.k_cache = torch.zeros(num_layers, 8, max_seq_len, 128, dtype=torch.bfloat16, device=dev)
        self.v_cache = torch.zeros_like(self.k_cache)
        f32 = lambda n: torch.zeros(n, dtype=torch.float32, device=dev)  # noqa: E731
        self.hidden = torch.zeros(1024, dtype=torch.bfloat16, device=dev)
        self.scratch = [f32(1024), f32(1024), f32(2048), f32(1024), f32(1024), f32(2048), f32(3072), f32(1024)]
        self.block_vals = f32(1184)
        self.block_idxs = torch.zeros(1184, dtype=torch.int32, device=dev)
        self.out = torch.zeros(1, dtype=torch.int32, device=dev)

    def launch(self, token: int, position: int, stream: int):
        s = self.scratch
        self.lib.launch_ldg_decode(
            int(token), self.out.data_ptr(), self.wd.embed.data_ptr(), self.d_table.data_ptr(),
            self.wd.final_norm.data_ptr(), self.wd.lm_head.data_ptr(), self.cos.data_ptr(), self.sin.data_ptr(),
            self.k_cache.data_ptr(), self.v_cache.data_ptr(), self.hidden.data_ptr(),
            s[0].data_ptr(), s[1].data_ptr(), s[2].data_ptr(), s[3].data_ptr(), s[4].data_ptr(), s[5].data_ptr(),
            s[6].data_ptr(), s[7].data_ptr(), self.block_vals.data_ptr(), self.block_idxs.data_ptr(),
            self.L, int(position), int(position) + 1, self.S, float(128 ** -0.5), stream)

    def decode_step(self, token: int, position: int) -> int:
        """One step with the token read back (the reference's ``.item()`` per
        token, megakernel_decode.py:195-200)."""
        self.launch(token, position, torch.cuda.current_stream().cuda_stream)
        return int(self.out.item())
