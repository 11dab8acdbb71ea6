"""megaqwen_b200: a B200 (sm_100a) Qwen3-0.6B decode engine behind the
reference MegaQwen torch-extension API.

The native parts are built in-tree by ``megaqwen_b200.build`` (see
``__graft_entry__.build()``).  Importing this package without them raises
ImportError: there is no CPU or pure-PyTorch fallback.
"""
from __future__ import annotations

import torch  # noqa: F401  (loads libtorch before the extension)

from . import weights  # noqa: F401

try:
    from . import _C  # type: ignore[attr-defined]
except ImportError as exc:  # pragma: no cover - exercised only on broken installs
    raise ImportError(
        "megaqwen_b200 native extension is not built; run `python megaqwen_b200/build.py`"
    ) from exc

MegakernelDecoder = _C.MegakernelDecoder
MegakernelPrefillDecoder = _C.MegakernelPrefillDecoder
MegakernelFusedPrefillDecoder = _C.MegakernelFusedPrefillDecoder
MegakernelBatchDecoder = _C.MegakernelBatchDecoder
init_ldg_layer_weights = _C.init_ldg_layer_weights
init_ldg_embed_weight = _C.init_ldg_embed_weight
decode_ldg = _C.decode_ldg
decode_ldg_with_logits = _C.decode_ldg_with_logits

__all__ = [
    "MegakernelDecoder",
    "MegakernelPrefillDecoder",
    "MegakernelFusedPrefillDecoder",
    "MegakernelBatchDecoder",
    "init_ldg_layer_weights",
    "init_ldg_embed_weight",
    "decode_ldg",
    "decode_ldg_with_logits",
    "weights",
]
