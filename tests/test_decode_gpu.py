"""Parity of the sm_100a decode engine against the CPU oracle and the golden
vectors of the reference's PyTorch forward.  Every test calls the engine
through the reference-compatible extension, which calls the C ABI.

Tolerances: per-step logits max-abs <= 3e-2 and cosine
>= 0.9995 against the oracle; greedy tokens identical.  bf16 K/V cache rows
written by the engine match the oracle's bf16 rows except for rare 1-ulp
rounding flips (both round fp32 values that differ in summation order).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LOGIT_MAX_ABS = 3e-2
COSINE_MIN = 0.9995


def _engine():
    import megaqwen_b200
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return megaqwen_b200


_DEV_WEIGHTS = {}


def dev_weights(num_layers):
    from megaqwen_b200.weights import make_weights
    if num_layers not in _DEV_WEIGHTS:
        _DEV_WEIGHTS.clear()
        torch.cuda.empty_cache()
        _DEV_WEIGHTS[num_layers] = (make_weights(num_layers), make_weights(num_layers).to("cuda"))
    return _DEV_WEIGHTS[num_layers]


def make_decoder(num_layers, max_seq_len, cls="MegakernelDecoder", **kw):
    from megaqwen_b200.weights import rope_tables
    m = _engine()
    _, wd = dev_weights(num_layers)
    cos, sin = rope_tables(max_seq_len, device="cuda")
    args = [wd.embed, wd.layer_weights_flat(), wd.final_norm, wd.lm_head, cos, sin, num_layers, max_seq_len]
    if cls != "MegakernelDecoder":
        args.append(kw.pop("max_prefill_len", 512))
    return getattr(m, cls)(*args)


def make_oracle(num_layers, max_seq_len):
    from oracle.qwen3_cpu import Qwen3CpuOracle
    wc, _ = dev_weights(num_layers)
    return Qwen3CpuOracle(wc, max_seq_len=max_seq_len)


def assert_logits_close(got, ref, what=""):
    got = got.detach().float().cpu()
    ref = ref.detach().float().cpu()
    err = (got - ref).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(got.view(1, -1), ref.view(1, -1)).item()
    assert err <= LOGIT_MAX_ABS, f"{what}: max-abs {err}"
    assert cos >= COSINE_MIN, f"{what}: cosine {cos}"
    return err


def assert_token_consistent(tok, logits, ref, what=""):
    """Greedy tokens must agree unless the oracle's top-2 gap is below the
    logit tolerance actually observed (a genuine near-tie)."""
    ref_tok = int(torch.argmax(ref).item())
    if tok == ref_tok:
        return
    top2 = torch.topk(ref.float(), 2).values
    gap = (top2[0] - top2[1]).item()
    err = (logits.float().cpu() - ref.float()).abs().max().item()
    assert gap <= 2 * err, f"{what}: token {tok} vs {ref_tok}, top-2 gap {gap}, logits max-abs {err}"


def assert_cache_close(dec_cache, ref_cache, upto):
    got = dec_cache[:, :, :upto].cpu()
    ref = ref_cache[:, :, :upto]
    eq = (got == ref).float().mean().item()
    diff = (got.float() - ref.float()).abs().max().item()
    assert eq > 0.97, f"bf16 K/V rows equal fraction {eq}"
    scale = ref.float().abs().max().item()
    assert diff <= 0.02 * max(scale, 1.0), f"K/V max diff {diff}"


@pytest.mark.parametrize("num_layers", [1, 2])
def test_decode_steps_match_oracle_small(num_layers):
    dec = make_decoder(num_layers, 256)
    o = make_oracle(num_layers, 256)
    toks = [11, 151935, 0, 7, 4242, 99999, 5, 123]
    for p, t in enumerate(toks):
        tok, logits = dec.decode_step_with_logits(t)
        ref = o.decode_step(t, p)
        assert_logits_close(logits, ref, f"L={num_layers} pos={p}")
        assert tok == int(torch.argmax(logits).item())
        assert tok == int(torch.argmax(ref).item())
    assert dec.position() == len(toks)
    assert_cache_close(dec.get_k_cache(), o.k_cache, len(toks))
    assert_cache_close(dec.get_v_cache(), o.v_cache, len(toks))
    # final hidden and normalized outputs (reference ABI side outputs)
    hid = dec.get_hidden_buffer().float().cpu()
    assert (hid - o.last_hidden).abs().max().item() < 2e-2 * max(1.0, o.last_hidden.abs().max().item())


def test_split_k_attention_matches_oracle():
    """Small attention chunks force several work units per kv head (up to 18,
    so the combiner's warps poll more than one unit each) and the fixed
    combiner's merge, at positions where one unit would also do."""
    dec = make_decoder(2, 512)
    o = make_oracle(2, 512)
    dec.set_attn_chunk(8)
    g = torch.Generator().manual_seed(3)
    toks = torch.randint(0, 151936, (150,), generator=g).tolist()
    for p, t in enumerate(toks):
        tok, logits = dec.decode_step_with_logits(t)
        ref = o.decode_step(t, p)
        assert_logits_close(logits, ref, f"pos={p}")
        assert_token_consistent(tok, logits, ref, f"pos={p}")
    assert_cache_close(dec.get_k_cache(), o.k_cache, len(toks))


@pytest.mark.parametrize("ctas", [8, 64, 131])
def test_cta_count_does_not_change_results(ctas):
    dec = make_decoder(2, 128)
    ref = make_decoder(2, 128)
    dec.set_num_ctas(ctas)
    for t in [5, 17, 29, 31000]:
        a, la = dec.decode_step_with_logits(t)
        b, lb = ref.decode_step_with_logits(t)
        assert a == b
        assert (la - lb).abs().max().item() < 1e-3


def test_config1_28_layers_matches_golden(golden_dir):
    """BASELINE config 1 on the GPU: 8-token prompt, 32 greedy steps, against the
    reference forward's own outputs."""
    g = dict(np.load(golden_dir / "config1_l28.npz"))
    dec = make_decoder(28, 512, cls="MegakernelPrefillDecoder")
    tok = dec.prefill_step(torch.from_numpy(g["prompt"]))
    assert dec.position() == len(g["prompt"])
    tokens = [tok]
    logits_steps = []
    for _ in range(len(g["tokens"]) - 1):
        t, lg = dec.decode_step_with_logits(tokens[-1])
        tokens.append(t)
        logits_steps.append(lg.cpu())
    assert tokens == [int(x) for x in g["tokens"]]
    top_ids = torch.from_numpy(g["top_ids"]).long()[1:]
    mine = torch.gather(torch.stack(logits_steps), 1, top_ids)
    assert (mine - torch.from_numpy(g["top_vals"][1:])).abs().max().item() < LOGIT_MAX_ABS
    full = torch.from_numpy(g["full_logits_f16"].astype(np.float32))
    for row, s in enumerate(g["full_steps"]):
        if s >= 1:
            assert_logits_close(logits_steps[s - 1], full[row], f"golden step {s}")


def test_greedy_256_steps_match_oracle():
    """North-star parity: 16-token seeded prompt, 256 greedy steps on the full
    model; tokens identical to the oracle and logits within tolerance."""
    from megaqwen_b200.weights import seeded_prompt
    prompt = seeded_prompt(16).tolist()
    dec = make_decoder(28, 512)
    o = make_oracle(28, 512)
    ref_tokens, ref_logits = o.greedy(prompt, 256, use_prefill=False)
    for t in prompt[:-1]:
        dec.decode_step(t)
    dev_tokens = dec.generate_greedy(prompt[-1], 257).cpu().tolist()
    assert dev_tokens == ref_tokens
    # teacher-forced logits spot checks on a fresh decoder
    dec2 = make_decoder(28, 512)
    for t in prompt[:-1]:
        dec2.decode_step(t)
    cur = prompt[-1]
    for i in range(12):
        _, lg = dec2.decode_step_with_logits(cur)
        assert_logits_close(lg, ref_logits[i], f"step {i}")
        cur = ref_tokens[i]


def test_prefill_classes_and_position_semantics():
    dec = make_decoder(2, 64, cls="MegakernelFusedPrefillDecoder", max_prefill_len=16)
    assert dec.max_prefill_len() == 16
    with pytest.raises(RuntimeError, match="Empty"):
        dec.prefill_step(torch.zeros(0, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="exceeds maximum"):
        dec.prefill_step(torch.zeros(17, dtype=torch.int32))
    o = make_oracle(2, 64)
    ids = [3, 1, 4, 1, 5, 9, 2, 6]
    tok = dec.prefill_step(torch.tensor(ids, dtype=torch.int32))
    ref = o.prefill(ids)[-1]
    assert tok == int(torch.argmax(ref))
    assert dec.position() == len(ids)
    t2 = dec.decode_step(tok)
    assert t2 == int(torch.argmax(o.decode_step(tok, len(ids))))
    dec.reset()
    assert dec.position() == 0 and int(dec.get_k_cache().abs().sum().item()) == 0


def test_step_counter_wrap_does_not_change_tokens():
    """The handoff words carry the step counter (25 bits, wraps to 0); steps
    run across the wrap give the same greedy tokens as steps far from it."""
    from megaqwen_b200.weights import seeded_prompt
    prompt = seeded_prompt(8).tolist()

    def run(epoch):
        dec = make_decoder(28, 64)
        if epoch is not None:
            dec.set_step_epoch(epoch)
        out, cur = [], prompt[0]
        for i in range(len(prompt) + 8):
            tok = dec.decode_step(cur)
            out.append(tok)
            cur = prompt[i + 1] if i + 1 < len(prompt) else tok
        return out

    ref = run(None)
    assert run((1 << 25) - 5) == ref


def test_position_and_token_bounds():
    dec = make_decoder(1, 4)
    for t in range(4):
        dec.decode_step(t)
    with pytest.raises(RuntimeError, match="max_seq_len"):
        dec.decode_step(1)
    dec.reset()
    with pytest.raises(RuntimeError, match="token"):
        dec.decode_step(151936)
    with pytest.raises(RuntimeError, match="token"):
        dec.decode_step(-1)


def test_chat_module_abi_matches_decoder():
    """chat.py's module functions (caller-owned caches and scratch, reference
    launchers through the C ABI) give the same tokens and logits."""
    m = _engine()
    from megaqwen_b200.weights import rope_tables
    _, wd = dev_weights(2)
    cos, sin = rope_tables(64, device="cuda")
    m.init_ldg_layer_weights(*wd.layer_weight_lists())
    m.init_ldg_embed_weight(wd.embed)
    kc = torch.zeros(2, 8, 64, 128, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    f = lambda n: torch.empty(n, dtype=torch.float32, device="cuda")  # noqa: E731
    scratch = [torch.empty(1024, dtype=torch.bfloat16, device="cuda"), f(1024), f(1024), f(2048), f(1024), f(1024),
               f(2048), f(3072), f(1024), f(1184), torch.empty(1184, dtype=torch.int32, device="cuda")]
    dec = make_decoder(2, 64)
    toks = [17, 4, 151000, 2]
    for p, t in enumerate(toks):
        a = m.decode_ldg(t, wd.final_norm, wd.lm_head, cos, sin, kc, vc, *scratch, 2, p, p + 1, 64)
        b, lb = dec.decode_step_with_logits(t)
        assert a == b
    kc2 = kc.clone()
    a2, la = m.decode_ldg_with_logits(9, wd.final_norm, wd.lm_head, cos, sin, kc, vc, *scratch, 2, 4, 5, 64)
    b2, lb = dec.decode_step_with_logits(9)
    assert a2 == b2 and (la - lb).abs().max().item() < 1e-3
    assert torch.equal(kc[:, :, :4], kc2[:, :, :4])
    assert torch.equal(kc[:, :, :5], dec.get_k_cache()[:, :, :5])
    with pytest.raises(RuntimeError):
        m.decode_ldg(9, wd.final_norm, wd.lm_head, cos, sin, kc, vc, *scratch, 2, 64, 65, 64)


def test_device_wait_timeout_is_reported_and_recoverable():
    """Failure detection without a GPU fault: one CTA withholds its layer-0
    handoff stores, every other CTA's bounded wait runs out, the engine reports
    the timeout as an error status and the context stays usable."""
    dec = make_decoder(1, 32)
    ref = dec.decode_step(5)
    dec.reset()
    dec.set_timeout_ns(50_000_000)   # 50 ms
    dec.set_inject_skip_cta(1 + 3)   # CTA 3 withholds its QKV rows
    with pytest.raises(RuntimeError, match="timed out"):
        dec.decode_step(5)
    dec.set_inject_skip_cta(0)
    dec.reset()
    assert dec.decode_step(5) == ref
    torch.cuda.synchronize()


def test_long_context_prefilled_cache():
    """BASELINE config 3 shape: caches pre-filled with N(0,1) bf16 K/V, then
    decode steps with split-K attention over thousands of positions."""
    P = 2048
    L = 4
    dec = make_decoder(L, P + 8)
    o = make_oracle(L, P + 8)
    g = torch.Generator().manual_seed(7)
    k = torch.randn(L, 8, P, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(L, 8, P, 128, generator=g).to(torch.bfloat16)
    o.k_cache[:, :, :P] = k
    o.v_cache[:, :, :P] = v
    dec.get_k_cache()[:, :, :P].copy_(k)
    dec.get_v_cache()[:, :, :P].copy_(v)
    dec.set_position(P)
    for i, t in enumerate([77, 1234]):
        tok, lg = dec.decode_step_with_logits(t)
        ref = o.decode_step(t, P + i)
        assert_logits_close(lg, ref, f"pos {P + i}")
        assert tok == int(torch.argmax(ref))
