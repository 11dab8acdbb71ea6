"""Batched decode (mq_decode_batch through MegakernelBatchDecoder) against
the CPU oracle and the single-sequence decode engine.

Each sequence of the batch has its own cache and position (ragged
contexts).  The batch path rounds GEMM operands to bf16 (the single-sequence
engine keeps fp32 activations), so the bar is the north-star logits bar:
max-abs <= 3e-2 and cosine >= 0.9995 against the oracle, tokens equal unless
the oracle's top-2 gap is within the observed error.  Each sequence is driven
with the batch's own token so near-ties cannot make the runs diverge."""
from __future__ import annotations

import pytest
import torch

from tests.test_decode_gpu import assert_logits_close, assert_token_consistent, dev_weights, make_oracle

pytestmark = pytest.mark.gpu


def make_batch(num_layers, max_seq_len, batch, use_graph=True):
    import megaqwen_b200
    from megaqwen_b200.weights import rope_tables
    _, wd = dev_weights(num_layers)
    cos, sin = rope_tables(max_seq_len, device="cuda")
    return megaqwen_b200._C.MegakernelBatchDecoder(wd.embed, wd.layer_weights_flat(), wd.final_norm, wd.lm_head,
                                                   cos, sin, num_layers, max_seq_len, batch, use_graph)


def _fill_from_oracle(bd, o_list, prompts):
    """Runs each prompt through its oracle and copies the bf16 caches into
    the batch decoder's sequence slots."""
    kc, vc = bd.get_k_cache(), bd.get_v_cache()
    for b, (o, pr) in enumerate(zip(o_list, prompts)):
        if len(pr) > 1:
            o.prefill(pr[:-1])
        n = len(pr) - 1
        kc[b, :, :, :n].copy_(o.k_cache[:, :, :n].to(kc.device))
        vc[b, :, :, :n].copy_(o.v_cache[:, :, :n].to(vc.device))


@pytest.mark.parametrize("batch,lens", [(3, [1, 5, 40]), (17, None)])
def test_batch_decode_matches_oracle(batch, lens):
    L, MS = 1, 320
    g = torch.Generator().manual_seed(batch)
    if lens is None:
        lens = [int(x) for x in torch.randint(1, 300, (batch,), generator=g)]
    prompts = [torch.randint(0, 151936, (n,), generator=g).tolist() for n in lens]
    oracles = [make_oracle(L, MS) for _ in range(batch)]
    bd = make_batch(L, MS, batch, use_graph=False)
    _fill_from_oracle(bd, oracles, prompts)
    bd.set_state(torch.tensor([p[-1] for p in prompts]), torch.tensor([len(p) - 1 for p in prompts]))
    pos = [len(p) - 1 for p in prompts]
    toks = [p[-1] for p in prompts]
    check = range(batch) if batch <= 4 else (0, 7, batch - 1)
    for step in range(3):
        bd.step(True)
        bd.check()
        logits = bd.logits().cpu()
        out = bd.tokens().cpu().tolist()
        assert bd.positions().cpu().tolist() == [p + 1 for p in pos]
        for b in check:
            ref = oracles[b].decode_step(toks[b], pos[b])
            assert_logits_close(logits[b], ref, f"step {step} seq {b} pos {pos[b]}")
            assert_token_consistent(out[b], logits[b], ref, f"step {step} seq {b}")
            assert out[b] == int(torch.argmax(logits[b]).item())
        toks = out
        pos = [p + 1 for p in pos]


@pytest.mark.parametrize("batch", [16, 64, 128])
def test_batch_decode_matches_single_engine(batch):
    """Full 28-layer model, padded batch sizes 16/64/128, against the
    single-sequence engine (itself pinned to the oracle) on a few sequences."""
    from tests.test_decode_gpu import make_decoder
    L, MS, steps = 28, 64, 4
    bd = make_batch(L, MS, batch, use_graph=False)
    g = torch.Generator().manual_seed(100 + batch)
    start = torch.randint(0, 151936, (batch,), generator=g)
    bd.set_state(start, torch.zeros(batch, dtype=torch.int32))
    picks = (0, batch // 2, batch - 1)
    singles = {b: make_decoder(L, MS) for b in picks}
    toks = start.tolist()
    for step in range(steps):
        bd.step(True)
        bd.check()
        logits = bd.logits().cpu()
        out = bd.tokens().cpu().tolist()
        for b in picks:
            _, lg = singles[b].decode_step_with_logits(toks[b])
            assert_logits_close(logits[b], lg, f"B={batch} step {step} seq {b}")
            assert_token_consistent(out[b], logits[b], lg.cpu(), f"B={batch} step {step} seq {b}")
        toks = out
    # every sequence's caches hold exactly `steps` rows
    kc = bd.get_k_cache()
    assert kc[:, :, :, :steps].abs().sum().item() > 0
    assert kc[:, :, :, steps:].abs().sum().item() == 0


def test_batch_graph_replay_matches_eager():
    """The CUDA-graph replay (one capture per context bucket, re-captured
    when the context crosses 256 positions) against the eager launch path.
    The step is deterministic (split-K partials are summed in a fixed order
    through distributed shared memory, no atomics), so tokens and K/V caches
    are bit-identical."""
    L, MS, B, steps = 2, 600, 16, 300
    g = torch.Generator().manual_seed(9)
    start = torch.randint(0, 151936, (B,), generator=g)
    pos0 = torch.randint(0, 10, (B,), generator=g)
    runs, caches = [], []
    for use_graph in (False, True):
        bd = make_batch(L, MS, B, use_graph=use_graph)
        bd.set_state(start, pos0)
        out = bd.generate(steps)
        bd.check()
        runs.append(out.cpu())
        caches.append(bd.get_k_cache().clone())
        assert bd.positions().cpu().tolist() == (pos0 + steps).tolist()
    assert torch.equal(runs[0], runs[1])
    assert torch.equal(caches[0], caches[1])


def test_batch_step_is_deterministic():
    L, MS, B = 2, 128, 64
    outs = []
    for _ in range(2):
        bd = make_batch(L, MS, B, use_graph=False)
        bd.set_state(torch.arange(B) * 7, torch.arange(B) % 5)
        bd.step(True)
        outs.append((bd.tokens().cpu(), bd.logits().cpu()))
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])


def test_batch_rejects_bad_state():
    bd = make_batch(1, 32, 4, use_graph=False)
    with pytest.raises(RuntimeError):
        bd.set_state(torch.tensor([1, 2, 3, 151936]), torch.zeros(4))
    with pytest.raises(RuntimeError):
        bd.set_state(torch.tensor([1, 2, 3, 4]), torch.tensor([0, 0, 0, 32]))
    with pytest.raises(RuntimeError):
        bd.set_state(torch.tensor([1, 2]), torch.zeros(2))


def test_decode_step_batched_entrypoint():
    """decode_step_batched(tokens) -> next tokens, the additive batch
    entrypoint, equals set_state + step on a second decoder."""
    L, MS, B = 2, 64, 16
    a = make_batch(L, MS, B, use_graph=True)
    b = make_batch(L, MS, B, use_graph=False)
    toks = torch.arange(B, dtype=torch.int32) * 1000 + 3
    a.set_state(toks, torch.zeros(B))
    b.set_state(toks, torch.zeros(B))
    for step in range(5):
        out_a = a.decode_step_batched(toks.cuda())
        b.set_state(toks, torch.full((B,), step))
        out_b = b.step(False).clone()
        assert torch.equal(out_a.cpu(), out_b.cpu())
        toks = out_a.cpu()
    assert a.positions().cpu().tolist() == [5] * B


@pytest.mark.parametrize("batch,length", [(16, 1600), (64, 1200)])
def test_batch_long_context_units_match_oracle(batch, length):
    """Long contexts select 512- and 1024-position attention units (and their
    multi-unit merge); checked sequences follow the oracle, the others carry
    random caches at long positions so the grid is full."""
    L, MS = 1, 2048
    g = torch.Generator().manual_seed(batch + length)
    checked = (0, batch // 2, batch - 1)
    oracles = {b: make_oracle(L, MS) for b in checked}
    prompts = {b: torch.randint(0, 151936, (length - 37 * i,), generator=g).tolist() for i, b in enumerate(checked)}
    bd = make_batch(L, MS, batch, use_graph=False)
    kc, vc = bd.get_k_cache(), bd.get_v_cache()
    kc.normal_()
    vc.normal_()
    pos = torch.randint(length - 200, length, (batch,), generator=g)
    toks = torch.randint(0, 151936, (batch,), generator=g)
    for b in checked:
        pr = prompts[b]
        oracles[b].prefill(pr[:-1])
        n = len(pr) - 1
        kc[b, :, :, :n].copy_(oracles[b].k_cache[:, :, :n].to(kc.device))
        vc[b, :, :, :n].copy_(oracles[b].v_cache[:, :, :n].to(vc.device))
        pos[b] = n
        toks[b] = pr[-1]
    bd.set_state(toks, pos)
    for step in range(2):
        bd.step(True)
        bd.check()
        logits = bd.logits().cpu()
        out = bd.tokens().cpu().tolist()
        for b in checked:
            ref = oracles[b].decode_step(int(toks[b]), int(pos[b]))
            assert_logits_close(logits[b], ref, f"B={batch} seq {b} pos {int(pos[b])}")
            assert_token_consistent(out[b], logits[b], ref, f"B={batch} seq {b}")
        toks = torch.tensor(out)
        pos = pos + 1
