"""megaqwen_b200: a B200 (sm_100a) Qwen3-0.6B decode engine behind the
reference MegaQwen torch-extension API.

The native parts are built in-tree by ``megaqwen_b200.build`` (see
``__graft_entry__.build()``).  The torch extension ``_C`` (and through it
``lib/libmegaqwen_b200.so``) is loaded on first use of a native name
(``megaqwen_b200.MegakernelDecoder``, ``megaqwen_b200._C`` ...), so the pure
host-side modules (``megaqwen_b200.weights``) import without mapping any native
library.  Using a native name without the built extension raises ImportError:
there is no CPU or pure-PyTorch fallback.
"""
from __future__ import annotations

import importlib

from . import weights  # noqa: F401  (pure torch/CPU: seeded weights, RoPE tables, prompts)

_NATIVE = (
    "MegakernelDecoder",
    "MegakernelPrefillDecoder",
    "MegakernelFusedPrefillDecoder",
    "MegakernelBatchDecoder",
    "MegakernelTPDecoder",
    "init_ldg_layer_weights",
    "init_ldg_embed_weight",
    "decode_ldg",
    "decode_ldg_with_logits",
)


def _load_native():
    import torch  # noqa: F401  (loads libtorch before the extension)
    try:
        return importlib.import_module("._C", __name__)
    except ImportError as exc:
        raise ImportError(
            "megaqwen_b200 native extension is not built; run `python megaqwen_b200/build.py`"
        ) from exc


def __getattr__(name):
    if name == "_C":
        return _load_native()
    if name in _NATIVE:
        return getattr(_load_native(), name)
    if name in ("megakernel_decode", "chat"):
        return importlib.import_module("." + name, __name__)
    raise AttributeError(f"module 'megaqwen_b200' has no attribute {name!r}")


__all__ = list(_NATIVE) + ["weights"]
