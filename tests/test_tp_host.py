"""Tensor-parallel decode, host side (CPU only): the partition of the weights
over ranks, and -- on two gloo ranks -- one decode layer and the LM-head argmax
computed the way the kernel splits them (q/k/v and attention by kv head, O and
down row-parallel with partials added in rank order, gate/up and the
vocabulary split), checked against the unsharded oracle layer."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from megaqwen_b200.tp import TP_SIZES, tp_partition
from megaqwen_b200.weights import HEAD_DIM, NUM_KV_HEADS, NUM_Q_HEADS, VOCAB_SIZE


@pytest.mark.parametrize("tp", TP_SIZES)
def test_partition_covers_every_row_once(tp):
    parts = [tp_partition(r, tp) for r in range(tp)]
    for field, total in (("kv_heads", NUM_KV_HEADS), ("q_rows", NUM_Q_HEADS * HEAD_DIM),
                         ("kv_rows", NUM_KV_HEADS * HEAD_DIM), ("act_rows", 3072), ("vocab_rows", VOCAB_SIZE)):
        spans = [getattr(p, field) for p in parts]
        assert spans[0][0] == 0 and spans[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    for p in parts:
        h0, h1 = p.kv_heads
        assert p.q_rows == (h0 * 2 * HEAD_DIM, h1 * 2 * HEAD_DIM)      # both q heads of each kv head
        assert p.kv_rows == (h0 * HEAD_DIM, h1 * HEAD_DIM)


def test_partition_rejects_bad_sizes():
    with pytest.raises(ValueError):
        tp_partition(0, 3)
    with pytest.raises(ValueError):
        tp_partition(2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import torch.distributed as dist
    import torch.nn.functional as F
    from megaqwen_b200.weights import make_weights
    from oracle.qwen3_cpu import Qwen3CpuOracle, rms_norm, rope

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.manual_seed(0)
    w = make_weights(1)
    o = Qwen3CpuOracle(w, max_seq_len=16)
    L = o.layers[0]
    pos = 5
    g = torch.Generator().manual_seed(1)
    h = torch.randn(1, 1024, generator=g)
    kc = torch.randn(NUM_KV_HEADS, pos, HEAD_DIM, generator=g).to(torch.bfloat16)
    vc = torch.randn(NUM_KV_HEADS, pos, HEAD_DIM, generator=g).to(torch.bfloat16)
    o.k_cache[0, :, :pos] = kc
    o.v_cache[0, :, :pos] = vc
    ref = o._layer(0, h, torch.tensor([pos]), False)

    p = tp_partition(rank, world)
    q0, q1 = p.q_rows
    k0, k1 = p.kv_rows
    a0, a1 = p.act_rows
    x = rms_norm(h, L["input_layernorm"])
    nh = p.kv_heads[1] - p.kv_heads[0]
    q = (x @ L["q_proj"][q0:q1].T).view(1, 2 * nh, HEAD_DIM).transpose(0, 1)
    k = (x @ L["k_proj"][k0:k1].T).view(1, nh, HEAD_DIM).transpose(0, 1)
    v = (x @ L["v_proj"][k0:k1].T).view(1, nh, HEAD_DIM).transpose(0, 1)
    q = rope(rms_norm(q, L["q_norm"]), o.cos[pos], o.sin[pos])
    k = rope(rms_norm(k, L["k_norm"]), o.cos[pos], o.sin[pos])
    kk = torch.cat([kc[p.kv_heads[0]:p.kv_heads[1]].float(), k.to(torch.bfloat16).float()], 1)
    vv = torch.cat([vc[p.kv_heads[0]:p.kv_heads[1]].float(), v.to(torch.bfloat16).float()], 1)
    kk = kk.repeat_interleave(2, 0)
    vv = vv.repeat_interleave(2, 0)
    att = torch.softmax((q @ kk.transpose(-1, -2)) * o.scale, -1) @ vv            # [2nh, 1, 128]
    att = att.transpose(0, 1).reshape(1, -1)

    def gather_sum(base, part):
        parts = [torch.zeros_like(part) for _ in range(world)]
        dist.all_gather(parts, part)
        for t in parts:                       # rank order, as the kernel adds them
            base = base + t
        return base

    hmid = gather_sum(h, att @ L["o_proj"][:, q0:q1].T)                          # row-parallel O
    x2 = rms_norm(hmid, L["post_attention_layernorm"])
    act = F.silu(x2 @ L["gate_proj"][a0:a1].T) * (x2 @ L["up_proj"][a0:a1].T)
    hout = gather_sum(hmid, act @ L["down_proj"][:, a0:a1].T)                    # row-parallel down
    err = (hout - ref).abs().max().item()

    # vocabulary-split LM head: each rank's best (value, index), max over ranks
    xf = rms_norm(hout, o.final_norm)
    v0, v1 = p.vocab_rows
    lg = (xf @ o.embed[v0:v1].T)[0]
    i = int(torch.argmax(lg))
    keys = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
    dist.all_gather(keys, torch.tensor([float(lg[i]), float(v0 + i)], dtype=torch.float64))
    best = max(keys, key=lambda t: (t[0].item(), -t[1].item()))
    full = int(torch.argmax((xf @ o.embed.T)[0]))
    out[rank] = (err, int(best[1].item()), full)
    dist.destroy_process_group()


def test_tp2_layer_and_argmax_match_unsharded_oracle():
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    mp.start_processes(_rank_main, args=(2, _free_port(), out), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        err, tok, full = out[r]
        assert err < 1e-4, f"rank {r}: layer output max-abs {err}"
        assert tok == full
