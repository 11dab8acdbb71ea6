"""Seeded synthetic Qwen3-0.6B weights in the reference's weight layout.

There is no network on the build or GPU hosts, so Hugging Face checkpoints are
unavailable.  Every benchmark and parity test therefore runs on random-init
weights drawn the same way everywhere:

* one ``torch.Generator`` seeded with 0, consumed in a fixed key order:
  ``embed_tokens``, then for each layer the eleven per-layer tensors in the
  order the reference flattens them (``csrc/megakernel/megakernel_decode.py:1108-1120``),
  then the final norm;
* projection matrices and the embedding are N(0, 0.02); RMSNorm weights are
  1.0 and draw nothing from the generator;
* every tensor is rounded to bf16 once; the CPU oracle upcasts those same bf16
  values to fp32, so both sides see identical weights;
* ``lm_head`` is the embedding (Qwen3-0.6B ties them).

Shapes follow Hugging Face ``nn.Linear`` (row-major ``[out_features, in_features]``),
which is what the reference kernels index (``fused_decode_ldg.cu:24-36``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List, Optional

import torch

HIDDEN_SIZE = 1024
INTERMEDIATE_SIZE = 3072
NUM_Q_HEADS = 16
NUM_KV_HEADS = 8
HEAD_DIM = 128
Q_SIZE = NUM_Q_HEADS * HEAD_DIM
KV_SIZE = NUM_KV_HEADS * HEAD_DIM
NUM_LAYERS = 28
VOCAB_SIZE = 151936
RMS_NORM_EPS = 1e-6
ROPE_THETA = 1_000_000.0
INIT_STD = 0.02

# Names of the eleven per-layer tensors, in the reference's flattening order
# (megakernel_decode.py:1108-1120 and the LDGLayerWeights struct fields).
LAYER_KEYS = (
    "input_layernorm",
    "q_proj",
    "k_proj",
    "v_proj",
    "q_norm",
    "k_norm",
    "o_proj",
    "post_attention_layernorm",
    "gate_proj",
    "up_proj",
    "down_proj",
)

LAYER_SHAPES = {
    "input_layernorm": (HIDDEN_SIZE,),
    "q_proj": (Q_SIZE, HIDDEN_SIZE),
    "k_proj": (KV_SIZE, HIDDEN_SIZE),
    "v_proj": (KV_SIZE, HIDDEN_SIZE),
    "q_norm": (HEAD_DIM,),
    "k_norm": (HEAD_DIM,),
    "o_proj": (HIDDEN_SIZE, Q_SIZE),
    "post_attention_layernorm": (HIDDEN_SIZE,),
    "gate_proj": (INTERMEDIATE_SIZE, HIDDEN_SIZE),
    "up_proj": (INTERMEDIATE_SIZE, HIDDEN_SIZE),
    "down_proj": (HIDDEN_SIZE, INTERMEDIATE_SIZE),
}

# Hugging Face state-dict names of the per-layer tensors.
HF_LAYER_NAMES = {
    "input_layernorm": "input_layernorm.weight",
    "q_proj": "self_attn.q_proj.weight",
    "k_proj": "self_attn.k_proj.weight",
    "v_proj": "self_attn.v_proj.weight",
    "q_norm": "self_attn.q_norm.weight",
    "k_norm": "self_attn.k_norm.weight",
    "o_proj": "self_attn.o_proj.weight",
    "post_attention_layernorm": "post_attention_layernorm.weight",
    "gate_proj": "mlp.gate_proj.weight",
    "up_proj": "mlp.up_proj.weight",
    "down_proj": "mlp.down_proj.weight",
}


def _is_norm(key: str) -> bool:
    return key.endswith("norm") or key.endswith("layernorm")


@dataclass
class Qwen3Weights:
    """bf16 weights of one model instance (CPU or device tensors)."""

    embed: torch.Tensor                      # [VOCAB, HIDDEN]
    layers: List[dict]                       # per layer: key -> tensor
    final_norm: torch.Tensor                 # [HIDDEN]
    seed: int = 0
    num_layers: int = NUM_LAYERS
    _flat: Optional[List[torch.Tensor]] = field(default=None, repr=False)

    @property
    def lm_head(self) -> torch.Tensor:
        return self.embed

    def layer_weights_flat(self) -> List[torch.Tensor]:
        """The reference's flat ``28*11`` list (megakernel_decode.py:1106-1120)."""
        out = []
        for layer in self.layers:
            out.extend(layer[k] for k in LAYER_KEYS)
        return out

    def layer_weight_lists(self) -> List[List[torch.Tensor]]:
        """chat.py's eleven per-kind lists (``init_ldg_layer_weights``, chat.py:151-163)."""
        return [[layer[k] for layer in self.layers] for k in LAYER_KEYS]

    def to(self, device) -> "Qwen3Weights":
        return Qwen3Weights(
            embed=self.embed.to(device).contiguous(),
            layers=[{k: v.to(device).contiguous() for k, v in layer.items()} for layer in self.layers],
            final_norm=self.final_norm.to(device).contiguous(),
            seed=self.seed,
            num_layers=self.num_layers,
        )

    def state_dict(self) -> dict:
        """Hugging Face-style names (the layout ``load_qwen3_weights`` reads)."""
        sd = {"model.embed_tokens.weight": self.embed, "model.norm.weight": self.final_norm,
              "lm_head.weight": self.embed}
        for i, layer in enumerate(self.layers):
            for k in LAYER_KEYS:
                sd[f"model.layers.{i}.{HF_LAYER_NAMES[k]}"] = layer[k]
        return sd


_CACHE: dict = {}


def make_weights(num_layers: int = NUM_LAYERS, seed: int = 0, std: float = INIT_STD,
                 cache: bool = True) -> Qwen3Weights:
    """Draw the seeded bf16 weights on the CPU.

    A model with fewer layers is a prefix of the full model's draw: the
    embedding and layers ``0..num_layers-1`` hold the same values as in the
    28-layer model.  The final norm is all ones and draws nothing.
    """
    key = (num_layers, seed, std)
    if cache and key in _CACHE:
        return _CACHE[key]
    # Reuse a longer cached draw when there is one (prefix property).
    if cache:
        for (nl, sd, st), w in _CACHE.items():
            if sd == seed and st == std and nl >= num_layers:
                res = Qwen3Weights(embed=w.embed, layers=w.layers[:num_layers],
                                   final_norm=w.final_norm, seed=seed, num_layers=num_layers)
                _CACHE[key] = res
                return res
    g = torch.Generator().manual_seed(seed)

    def draw(shape):
        return (torch.randn(*shape, generator=g, dtype=torch.float32) * std).to(torch.bfloat16)

    embed = draw((VOCAB_SIZE, HIDDEN_SIZE))
    layers = []
    for _ in range(num_layers):
        layer = {}
        for k in LAYER_KEYS:
            shape = LAYER_SHAPES[k]
            if _is_norm(k):
                layer[k] = torch.ones(*shape, dtype=torch.bfloat16)
            else:
                layer[k] = draw(shape)
        layers.append(layer)
    final_norm = torch.ones(HIDDEN_SIZE, dtype=torch.bfloat16)
    w = Qwen3Weights(embed=embed, layers=layers, final_norm=final_norm, seed=seed, num_layers=num_layers)
    if cache:
        _CACHE[key] = w
    return w


def rope_tables(max_seq_len: int, theta: float = ROPE_THETA, device="cpu"):
    """bf16 ``cos``/``sin`` tables ``[max_seq_len, HEAD_DIM]``.

    Same construction as the reference (chat.py:48-56 and demo_e2e.py:169-177):
    ``inv_freq = theta^(-2i/128)``, angles ``t * inv_freq`` in fp32, cos/sin
    rounded to bf16 and the 64 columns repeated twice.
    """
    inv_freq = 1.0 / (theta ** (torch.arange(0, HEAD_DIM, 2, dtype=torch.float32) / HEAD_DIM))
    t = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    cos = freqs.cos().to(torch.bfloat16)
    sin = freqs.sin().to(torch.bfloat16)
    cos = torch.cat([cos, cos], dim=-1).contiguous()
    sin = torch.cat([sin, sin], dim=-1).contiguous()
    return cos.to(device), sin.to(device)


def seeded_prompt(length: int, seed: int = 0, vocab: int = VOCAB_SIZE) -> torch.Tensor:
    """Uniform token ids in ``[0, vocab)`` from a seed-``seed`` generator (int32)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (length,), generator=g, dtype=torch.int64).to(torch.int32)


ATTN_SCALE = 1.0 / math.sqrt(HEAD_DIM)
