"""Python surface of the reference module ``csrc/megakernel/megakernel_decode.py``.

Same names and call shapes, backed by the prebuilt sm_100a extension instead
of ``load_inline`` JIT builds:

* ``_compile_decode_kernel`` / ``_compile_prefill_kernel`` /
  ``_compile_fused_prefill_kernel`` (reference :33-262, :265-682, :685-1074)
  return the extension module that holds ``MegakernelDecoder``,
  ``MegakernelPrefillDecoder`` and ``MegakernelFusedPrefillDecoder``;
* ``load_qwen3_weights`` (reference :1077-1133) returns the same dict keys;
  with no checkpoint available offline it serves the seeded synthetic weights
  of :mod:`megaqwen_b200.weights` (RoPE theta 1e6, the Qwen3 value);
* ``MegakernelGenerator`` / ``MegakernelPrefillGenerator`` /
  ``MegakernelFusedPrefillGenerator`` (reference :1136-1407) run greedy
  generation on token ids.  Text prompts need a tokenizer object with
  ``encode``/``decode``; none is bundled.
"""
from __future__ import annotations

from typing import Iterable, List, Optional, Sequence, Union

import torch

from . import _C
from .weights import (  # noqa: F401  (constants re-exported like the reference module)
    HEAD_DIM, HIDDEN_SIZE, INTERMEDIATE_SIZE, KV_SIZE, NUM_KV_HEADS, NUM_LAYERS, NUM_Q_HEADS, Q_SIZE, VOCAB_SIZE,
    make_weights, rope_tables,
)


def _compile_decode_kernel():
    return _C


def _compile_prefill_kernel():
    return _C


def _compile_fused_prefill_kernel():
    return _C


def load_qwen3_weights(model_name: str = "Qwen/Qwen3-0.6B", max_seq_len: int = 2048, num_layers: int = NUM_LAYERS,
                       seed: int = 0, device: Union[str, torch.device] = "cuda"):
    """Weights dict in the reference's format (megakernel_decode.py:1123-1130).

    ``model_name`` is accepted for signature compatibility; the weights are the
    seeded N(0, 0.02) synthetic ones.  ``tokenizer`` is None.
    """
    w = make_weights(num_layers, seed=seed).to(device)
    cos, sin = rope_tables(max_seq_len, device=device)
    return {
        "embed_weight": w.embed,
        "layer_weights": w.layer_weights_flat(),
        "final_norm_weight": w.final_norm,
        "lm_head_weight": w.lm_head,
        "cos_table": cos,
        "sin_table": sin,
        "tokenizer": None,
        "num_layers": num_layers,
    }


PromptT = Union[str, Sequence[int], torch.Tensor]


class _GeneratorBase:
    decoder_cls = None
    default_max_prefill_len: Optional[int] = None

    def __init__(self, model_name: str = "Qwen/Qwen3-0.6B", max_seq_len: int = 2048,
                 max_prefill_len: Optional[int] = None, weights: Optional[dict] = None, tokenizer=None):
        weights = weights or load_qwen3_weights(model_name, max_seq_len)
        args = [weights["embed_weight"], weights["layer_weights"], weights["final_norm_weight"],
                weights["lm_head_weight"], weights["cos_table"], weights["sin_table"],
                weights.get("num_layers", NUM_LAYERS), max_seq_len]
        if self.default_max_prefill_len is not None:
            self.max_prefill_len = max_prefill_len or self.default_max_prefill_len
            args.append(self.max_prefill_len)
        self.decoder = self.decoder_cls(*args)
        self.tokenizer = tokenizer or weights.get("tokenizer")
        self.max_seq_len = max_seq_len
        self._weights = weights

    def _ids(self, prompt: PromptT) -> List[int]:
        if isinstance(prompt, str):
            if self.tokenizer is None:
                raise ValueError("text prompts need a tokenizer; pass token ids instead")
            return list(self.tokenizer.encode(prompt, add_special_tokens=True))
        if isinstance(prompt, torch.Tensor):
            return [int(t) for t in prompt.view(-1).tolist()]
        return [int(t) for t in prompt]

    def _out(self, ids: List[int]):
        if self.tokenizer is not None:
            return self.tokenizer.decode(ids, skip_special_tokens=True)
        return ids

    def _stop(self, stop_tokens):
        if stop_tokens is not None:
            return set(stop_tokens)
        eos = getattr(self.tokenizer, "eos_token_id", None)
        return {eos} if eos is not None else set()


class MegakernelGenerator(_GeneratorBase):
    """Decode-only generator: the prompt runs token by token through decode
    (reference megakernel_decode.py:1158-1187)."""

    decoder_cls = _C.MegakernelDecoder

    def generate(self, prompt: PromptT, max_new_tokens: int = 100, temperature: float = 1.0,
                 stop_tokens: Optional[Iterable[int]] = None):
        return self._out(list(self.generate_stream(prompt, max_new_tokens, stop_tokens, _raw=True)))

    def generate_stream(self, prompt: PromptT, max_new_tokens: int = 100, stop_tokens=None, _raw: bool = False):
        if max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be positive")
        self.decoder.reset()
        ids = self._ids(prompt)
        if not ids:
            raise ValueError("empty prompt")
        for t in ids[:-1]:
            self.decoder.decode_step(t)
        cur = ids[-1]
        stop = self._stop(stop_tokens)
        for _ in range(max_new_tokens):
            nxt = self.decoder.decode_step(cur)
            if nxt in stop:
                break
            yield nxt if (_raw or self.tokenizer is None) else self.tokenizer.decode([nxt])
            cur = nxt
            if self.decoder.position() >= self.max_seq_len - 1:
                break


class MegakernelPrefillGenerator(_GeneratorBase):
    """Prefill + decode generator (reference megakernel_decode.py:1214-1307)."""

    decoder_cls = _C.MegakernelPrefillDecoder
    default_max_prefill_len = 512

    def _prefill(self, prompt: PromptT) -> int:
        self.decoder.reset()
        ids = self._ids(prompt)
        if len(ids) > self.max_prefill_len:
            raise ValueError(f"Prompt length {len(ids)} exceeds max prefill length {self.max_prefill_len}")
        return self.decoder.prefill_step(torch.tensor(ids, dtype=torch.int32))

    def generate(self, prompt: PromptT, max_new_tokens: int = 100, stop_tokens=None):
        return self._out(list(self.generate_stream(prompt, max_new_tokens, stop_tokens, _raw=True)))

    def generate_stream(self, prompt: PromptT, max_new_tokens: int = 100, stop_tokens=None, _raw: bool = False):
        nxt = self._prefill(prompt)
        stop = self._stop(stop_tokens)
        for _ in range(max_new_tokens):
            if nxt in stop:
                break
            yield nxt if (_raw or self.tokenizer is None) else self.tokenizer.decode([nxt])
            if self.decoder.position() >= self.max_seq_len - 1:
                break
            nxt = self.decoder.decode_step(nxt)

    def prefill_only(self, prompt: PromptT):
        nxt = self._prefill(prompt)
        return nxt, self.decoder.position()


class MegakernelFusedPrefillGenerator(MegakernelPrefillGenerator):
    """Short-prompt prefill generator (reference megakernel_decode.py:1310-1407)."""

    decoder_cls = _C.MegakernelFusedPrefillDecoder
    default_max_prefill_len = 64
