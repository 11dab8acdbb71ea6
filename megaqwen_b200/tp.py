"""KV-head tensor-parallel batch-1 decode across GPUs (one rank per GPU).

``MegakernelTPDecoder`` (the torch extension) runs one decode step of a
rank's share of the model; the kernel exchanges the per-layer O and down
projection partials and the argmax keys with the other ranks itself, by
plain peer stores over NVLink into every rank's workspace.  This module holds
the host-side pieces around it:

* ``tp_partition(rank, tp)``: which rows and columns of each weight a rank
  reads (the same split the kernel computes);
* ``make_tp_decoder(...)``: builds the rank's decoder and connects the ranks'
  workspaces by exchanging CUDA IPC handles over ``torch.distributed``.

There is no counterpart in the reference (it decodes on one GPU); the
partition follows the usual Megatron split for GQA: q/k/v rows and attention
by kv head, O and down row-parallel (each rank multiplies its own input
columns and the partial outputs are summed), gate/up column-parallel, LM head
split over the vocabulary.
"""
from __future__ import annotations

from dataclasses import dataclass

from .weights import HEAD_DIM, HIDDEN_SIZE, INTERMEDIATE_SIZE, NUM_KV_HEADS, NUM_Q_HEADS, VOCAB_SIZE

TP_SIZES = (1, 2, 4, 8)


@dataclass(frozen=True)
class TpSlice:
    """Half-open ranges owned by one rank."""

    kv_heads: tuple       # kv heads (attention, k/v rows, cache rows)
    q_rows: tuple         # rows of q_proj (= columns of o_proj)
    kv_rows: tuple        # rows of k_proj and v_proj
    act_rows: tuple       # rows of gate_proj/up_proj (= columns of down_proj)
    vocab_rows: tuple     # rows of the LM head


def tp_partition(rank: int, tp: int) -> TpSlice:
    if tp not in TP_SIZES:
        raise ValueError(f"tp must be one of {TP_SIZES}")
    if not 0 <= rank < tp:
        raise ValueError("rank out of range")
    nh = NUM_KV_HEADS // tp
    qh = NUM_Q_HEADS // NUM_KV_HEADS
    ia = INTERMEDIATE_SIZE // tp
    return TpSlice(
        kv_heads=(nh * rank, nh * (rank + 1)),
        q_rows=(nh * qh * HEAD_DIM * rank, nh * qh * HEAD_DIM * (rank + 1)),
        kv_rows=(nh * HEAD_DIM * rank, nh * HEAD_DIM * (rank + 1)),
        act_rows=(ia * rank, ia * (rank + 1)),
        vocab_rows=(VOCAB_SIZE * rank // tp, VOCAB_SIZE * (rank + 1) // tp),
    )


def make_tp_decoder(weights, cos, sin, num_layers: int, max_seq_len: int, group=None):
    """The calling rank's ``MegakernelTPDecoder``, connected to the others.

    ``weights``: this rank's device copy of the full weights (a
    ``Qwen3Weights``); every rank of ``group`` (default: the world) must call
    this together, one process per GPU.  Collective: exchanges the ranks'
    workspace IPC handles with ``all_gather_object``.
    """
    import torch.distributed as dist
    from . import _C
    rank = dist.get_rank(group)
    tp = dist.get_world_size(group)
    dec = _C.MegakernelTPDecoder(weights.embed, weights.layer_weights_flat(), weights.final_norm, weights.lm_head,
                                 cos, sin, num_layers, max_seq_len, rank, tp)
    handles = [None] * tp
    dist.all_gather_object(handles, dec.ipc_handle(), group=group)
    dec.connect(handles)
    dist.barrier(group)
    return dec


__all__ = ["TpSlice", "tp_partition", "make_tp_decoder", "TP_SIZES", "HIDDEN_SIZE"]
