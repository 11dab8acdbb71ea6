"""Kernel-selection surface of the reference ``chat.py`` (chat.py:11-62).

The reference JIT-compiles one of three decode-kernel variants
(``baseline``, ``fastmath``, ``blocks128_fastmath``) with ``load_inline`` and
picks one per request by generation length.  Here every variant name maps to
the single prebuilt sm_100a decode kernel: ``compile_kernel(variant)``
validates the name exactly as the reference does and returns the extension
module, which exposes the same four chat functions
(``init_ldg_layer_weights``, ``init_ldg_embed_weight``, ``decode_ldg``,
``decode_ldg_with_logits``; reference chat.py:147-323).  A chat.py user swaps
``from chat import compile_kernel`` for
``from megaqwen_b200.chat import compile_kernel`` and changes nothing else.

The interactive REPL, the Hugging Face tokenizer and checkpoint loading of the
reference file are not part of the decode path and are not provided.
"""
from __future__ import annotations

import torch

from .weights import HEAD_DIM, HIDDEN_SIZE, INTERMEDIATE_SIZE, NUM_KV_HEADS, NUM_LAYERS  # noqa: F401

MAX_SEQ_LEN = 512                                         # chat.py:15

SUPPORTED_DECODE_KERNEL_VARIANTS = ("baseline", "fastmath", "blocks128_fastmath")   # chat.py:17
AUTO_KERNEL_VARIANT = "auto"                              # chat.py:18
SHORT_DECODE_TOKEN_THRESHOLD = 128                        # chat.py:19


def select_optimal_kernel_variant(max_new_tokens: int) -> str:
    """Variant name for a generation length (chat.py:22-29): ``fastmath`` up
    to ``SHORT_DECODE_TOKEN_THRESHOLD`` new tokens, ``blocks128_fastmath``
    beyond.  Raises ``ValueError`` for a non-positive length.  All names run
    the same kernel here; the policy is kept so callers see the same names."""
    if max_new_tokens <= 0:
        raise ValueError("max_new_tokens must be positive")
    if max_new_tokens <= SHORT_DECODE_TOKEN_THRESHOLD:
        return "fastmath"
    return "blocks128_fastmath"


def compile_kernel(variant: str = "baseline"):
    """The chat decode module for ``variant`` (chat.py:59-343).

    Raises ``ValueError`` with the reference's message for an unknown name.
    Nothing is compiled at run time: the module is the prebuilt extension,
    shared by every variant name (built by ``megaqwen_b200/build.py``)."""
    if variant not in SUPPORTED_DECODE_KERNEL_VARIANTS:
        supported = ", ".join(SUPPORTED_DECODE_KERNEL_VARIANTS)
        raise ValueError(f"unsupported kernel variant '{variant}', expected one of: {supported}")
    from . import _C
    return _C


def precompute_rope_freqs(head_dim: int, max_seq_len: int, theta: float = 1000000.0, device="cuda"):
    """bf16 cos/sin tables ``[max_seq_len, head_dim]`` (chat.py:48-56)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim))
    t = torch.arange(max_seq_len, device=device, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    cos = freqs.cos().to(torch.bfloat16)
    sin = freqs.sin().to(torch.bfloat16)
    return torch.cat([cos, cos], dim=-1), torch.cat([sin, sin], dim=-1)
