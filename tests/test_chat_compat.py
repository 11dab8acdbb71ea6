"""chat.py kernel-selection surface (reference chat.py:17-29, 59-62) and the
package's lazy native loading.  Mirrors the reference's
tests/test_chat_kernel_selection.py; CPU only."""
from __future__ import annotations

import subprocess
import sys

import pytest

from megaqwen_b200.chat import (
    AUTO_KERNEL_VARIANT,
    SHORT_DECODE_TOKEN_THRESHOLD,
    SUPPORTED_DECODE_KERNEL_VARIANTS,
    compile_kernel,
    precompute_rope_freqs,
    select_optimal_kernel_variant,
)
from conftest import ROOT


def test_short_decode_prefers_fastmath() -> None:
    assert select_optimal_kernel_variant(1) == "fastmath"
    assert select_optimal_kernel_variant(SHORT_DECODE_TOKEN_THRESHOLD) == "fastmath"


def test_medium_and_long_decode_prefers_blocks128_fastmath() -> None:
    assert select_optimal_kernel_variant(SHORT_DECODE_TOKEN_THRESHOLD + 1) == "blocks128_fastmath"
    assert select_optimal_kernel_variant(500) == "blocks128_fastmath"


def test_kernel_selection_rejects_non_positive_decode_length() -> None:
    with pytest.raises(ValueError, match="max_new_tokens must be positive"):
        select_optimal_kernel_variant(0)
    with pytest.raises(ValueError, match="max_new_tokens must be positive"):
        select_optimal_kernel_variant(-1)


def test_supported_kernel_variants_include_auto_and_tuned_options() -> None:
    assert AUTO_KERNEL_VARIANT == "auto"
    assert SUPPORTED_DECODE_KERNEL_VARIANTS == ("baseline", "fastmath", "blocks128_fastmath")


def test_compile_kernel_maps_every_variant_to_the_chat_module() -> None:
    mods = {v: compile_kernel(v) for v in SUPPORTED_DECODE_KERNEL_VARIANTS}
    assert len({id(m) for m in mods.values()}) == 1
    m = compile_kernel()
    for name in ("init_ldg_layer_weights", "init_ldg_embed_weight", "decode_ldg", "decode_ldg_with_logits"):
        assert callable(getattr(m, name))


def test_compile_kernel_rejects_unknown_variant() -> None:
    with pytest.raises(ValueError, match="unsupported kernel variant 'turbo', expected one of: "
                                         "baseline, fastmath, blocks128_fastmath"):
        compile_kernel("turbo")
    with pytest.raises(ValueError, match="unsupported kernel variant"):
        compile_kernel(AUTO_KERNEL_VARIANT)   # "auto" is resolved by the caller, as in chat.py:446-450


def test_precompute_rope_freqs_matches_package_tables() -> None:
    from megaqwen_b200.weights import rope_tables
    c, s = precompute_rope_freqs(128, 64, device="cpu")
    c2, s2 = rope_tables(64)
    assert c.dtype == c2.dtype and bool((c == c2).all()) and bool((s == s2).all())


def test_weights_import_maps_no_native_library() -> None:
    """The CPU reference arm imports megaqwen_b200.weights; that must not load
    the product's extension or library."""
    code = ("import megaqwen_b200.weights, oracle.qwen3_cpu, sys\n"
            "maps = open('/proc/self/maps').read()\n"
            "bad = [m for m in ('libmegaqwen_b200', 'megaqwen_b200/_C') if m in maps]\n"
            "print('MAPPED', bad)\n"
            "sys.exit(1 if bad else 0)\n")
    r = subprocess.run([sys.executable, "-c", code], cwd=str(ROOT), capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
