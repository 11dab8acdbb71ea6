"""Benchmark: batch-1 greedy decode of Qwen3-0.6B on B200 (sm_100a).

Headline: 28 layers, bf16 seeded synthetic weights,
16-token seeded prompt, then greedy decode; one *step* is one decode token.
``value`` is tokens/s over K timed steps with the token fed back on the device
(no host round trip), timed with CUDA events; ``e2e`` is the same metric
through the public ``MegakernelDecoder.decode_step(int) -> int`` call (token
in by value, result read back to the host every step).  Extra keys: decode
tok/s and roofline fraction at positions 1/128/512/2048/8192 (config 3 caches
pre-filled with N(0,1) K/V), prefill tok/s, the CPU oracle baseline.

Multi-GPU (``--gpus N`` under torchrun): independent replicas, one per GPU, no
collective on the data path; ``value`` = all ranks' tokens / max-over-ranks
time.

``--impl reference`` times the reference's PyTorch CPU forward (restated in
``oracle/qwen3_cpu.py``) on this host's cores, same metric and workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import threading
import time

import torch

HBM_FALLBACK_GBS = 6650.0
WEIGHT_BYTES = 1_192_101_888            # 28 layers + lm_head + norms + one embedding row
KV_BYTES_PER_POS = 114_688              # K+V, all layers, one position (bf16)


# DRAM bytes (read + write) of one decode_step_kernel launch at position ~20 from
# one `ncu --set full` capture (profiles/decode_step_kernel_config2.md).  DRAM
# traffic tracks the algorithmic bytes (the same holds at p = 8192,
# profiles/decode_step_kernel_p8192.md), so the bench scales it to its own mean
# position by the algorithmic-bytes ratio.
NCU_TRAFFIC_P20 = 1_194_463_000 + 3_732_736


def bytes_per_token(pos: int) -> int:
    """Algorithmic HBM bytes of one decode token at position ``pos``: every
    weight once, K/V rows 0..pos read, row pos written."""
    return WEIGHT_BYTES + KV_BYTES_PER_POS * (pos + 2)


def prefill_flops(B, S):
    """Dense FLOPs of a B x S prefill: linear layers 2 x 440,401,920 per token,
    causal attention 28 * 16 * 4 * 128 * S(S+1)/2 per sequence, LM head of the
    last token per sequence."""
    return B * (S * 2 * 440_401_920 + 28 * 16 * 4 * 128 * S * (S + 1) / 2 + 2 * 151936 * 1024)


def measured_bf16_tflops():
    here = os.path.dirname(os.path.abspath(__file__))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def measured_hbm_gbs():
    here = os.path.dirname(os.path.abspath(__file__))
    try:
        with open(os.path.join(here, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return HBM_FALLBACK_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=2)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        if torch.cuda.is_available():
            torch.cuda.set_device(0)
    return rank, world, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def cpu_oracle_rate(budget_s: float, num_layers: int = 28, prompt_len: int = 16):
    """Decode tok/s of the CPU oracle (fp32) on this host, bounded to ~budget_s."""
    from megaqwen_b200.weights import make_weights, seeded_prompt
    from oracle.qwen3_cpu import Qwen3CpuOracle
    o = Qwen3CpuOracle(make_weights(num_layers), max_seq_len=prompt_len + 4096)
    prompt = seeded_prompt(prompt_len).tolist()
    logits = o.prefill(prompt)[-1]
    tok = int(torch.argmax(logits))
    pos = prompt_len
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        tok = int(torch.argmax(o.decode_step(tok, pos)))
        pos += 1
        n += 1
    dt = time.perf_counter() - t0
    return n / dt, n, torch.get_num_threads(), pos


def run_reference(args, rank, world):
    if rank != 0:
        return
    steps = args.steps
    from megaqwen_b200.weights import make_weights, seeded_prompt
    from oracle.qwen3_cpu import Qwen3CpuOracle
    torch.set_num_threads(os.cpu_count() or 1)
    o = Qwen3CpuOracle(make_weights(28), max_seq_len=16 + args.warmup + steps + 8)
    prompt = seeded_prompt(16).tolist()
    tok = int(torch.argmax(o.prefill(prompt)[-1]))
    pos = 16
    for _ in range(args.warmup):
        tok = int(torch.argmax(o.decode_step(tok, pos)))
        pos += 1
    t0 = time.perf_counter()
    for _ in range(steps):
        tok = int(torch.argmax(o.decode_step(tok, pos)))
        pos += 1
    dt = time.perf_counter() - t0
    v = steps / dt
    cores = torch.get_num_threads()
    line = {
        "impl": "reference", "metric": "batch-1 decode tok/s", "value": round(v, 3), "unit": "tok/s",
        "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(1000 * dt / steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2 decode on host cores: reference PyTorch forward (demo_e2e Backend.TORCH, "
                               "restated in oracle/qwen3_cpu.py), fp32, 28 layers, 16-token seeded prompt",
                   "positions": f"{16 + args.warmup}..{pos - 1}"},
        "cpu_baseline": {"value": round(v, 3), "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": f"{steps} decode steps at positions {16 + args.warmup}..{pos - 1}"},
        "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def time_device_steps(dec, tok_buf, steps):
    """Decode ``steps`` tokens back to back with device token feedback.
    Returns the total device time (ms) between two CUDA events bracketing all
    steps.  (Events between individual launches are not used: they stall the
    launch pipeline and add ~0.1-0.2 ms per step.)"""
    stream = torch.cuda.current_stream()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    ptr = tok_buf.data_ptr()
    t_start.record(stream)
    for _ in range(steps):
        dec.decode_step_async(ptr, ptr)
    t_end.record(stream)
    torch.cuda.synchronize()
    return t_start.elapsed_time(t_end)


def run_prefill(args, w, cos, sin, dev):
    """Prefill (config 4): batch 1 and 8, 2048-token prompts, tensor-core path."""
    import megaqwen_b200
    from megaqwen_b200.weights import seeded_prompt
    sweep_prefill = {}
    peak_tf, peak_kind = measured_bf16_tflops()
    for B in args.prefill_batches:
        S = 2048
        ids = torch.stack([seeded_prompt(S, seed=4 + b) for b in range(B)]).to(dev)
        kc = torch.zeros(B, 28, 8, S + 8, 128, dtype=torch.bfloat16, device=dev)
        vc = torch.zeros_like(kc)
        wsb = torch.empty(megaqwen_b200._C.prefill_workspace_bytes(B, S), dtype=torch.uint8, device=dev)
        run = lambda: megaqwen_b200._C.prefill_batch(w.embed, w.layer_weights_flat(), w.final_norm, w.lm_head,
                                                     cos, sin, ids, kc, vc, None, wsb)  # noqa: E731
        for _ in range(2):
            run()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = args.prefill_reps
        e0.record()
        for _ in range(reps):
            run()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        flops = prefill_flops(B, S)
        sweep_prefill[f"B{B}_S{S}"] = {"tok_s": round(B * S / (ms / 1000.0), 1), "ms": round(ms, 3),
                                       "tflops": round(flops / (ms / 1000.0) / 1e12, 1),
                                       "frac_of_bf16_peak": round(flops / (ms / 1000.0) / 1e12 / peak_tf, 4),
                                       "peak_tflops": peak_tf, "peak_kind": peak_kind}
        del kc, vc, wsb
        torch.cuda.empty_cache()
    return sweep_prefill


def run_batch(args, w, cos, sin, dev, hbm, world):
    """Batched decode (config 5): per batch size and start position, graph-replayed
    steps over B sequences whose caches are pre-filled with N(0,1) bf16 K/V."""
    import megaqwen_b200
    batch = {}
    g = torch.Generator(device=dev).manual_seed(13)
    for B in args.batch_sizes:
        for P in args.batch_positions:
            MS = P + args.batch_steps + 16
            bd = megaqwen_b200._C.MegakernelBatchDecoder(w.embed, w.layer_weights_flat(), w.final_norm,
                                                         w.lm_head, cos, sin, 28, MS, B, True)
            kc, vc = bd.get_k_cache(), bd.get_v_cache()
            kc[:, :, :, :P].normal_(generator=g)
            vc[:, :, :, :P].normal_(generator=g)
            bd.set_state(torch.arange(B) * 37 + 5, torch.full((B,), P))
            for _ in range(3):
                bd.step(False)
            torch.cuda.synchronize()
            barrier(world)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n = args.batch_steps
            e0.record()
            for _ in range(n):
                bd.step(False)
            e1.record()
            torch.cuda.synchronize()
            bd.check()
            ms = max_over_ranks(e0.elapsed_time(e1), world) / n
            pm = P + 3 + n // 2
            step_bytes = WEIGHT_BYTES + B * KV_BYTES_PER_POS * (pm + 2)
            batch[f"B{B}_pos{P}"] = {
                "tok_s": round(world * B / (ms / 1000.0), 1), "tok_s_per_gpu": round(B / (ms / 1000.0), 1),
                "ms_per_step": round(ms, 4),
                "roofline_frac": round(step_bytes / (ms / 1000.0) / 1e9 / hbm, 4),
                "bytes_per_step": step_bytes}
            del bd, kc, vc
            torch.cuda.empty_cache()
    return batch


def run_ours(args, rank, world, local):
    import megaqwen_b200
    from megaqwen_b200.weights import make_weights, rope_tables, seeded_prompt

    dev = torch.device("cuda", local)
    hbm, hbm_kind = measured_hbm_gbs()
    max_pos = max(args.sweep + [16 + args.warmup + args.steps] +
                  [p + args.batch_steps + 16 for p in args.batch_positions]) + 64
    w = make_weights(28).to(dev)
    cos, sin = rope_tables(max_pos + 8, device=dev)
    dec = megaqwen_b200.MegakernelDecoder(w.embed, w.layer_weights_flat(), w.final_norm, w.lm_head, cos, sin, 28,
                                          max_pos + 8)
    prompt = seeded_prompt(16).tolist()
    if args.only_prefill:
        # profiling entry: only the prefill measurements, one JSON line
        res = run_prefill(args, w, cos, sin, dev)
        if rank == 0:
            print(json.dumps({"prefill": res}), flush=True)
        return
    if args.only_batch:
        # profiling entry: only the batched-decode measurements, one JSON line
        batch = run_batch(args, w, cos, sin, dev, hbm, world)
        if rank == 0:
            print(json.dumps({"batch_decode": batch}), flush=True)
        return

    # --- headline: config 2, device-fed greedy decode after a 16-token prompt ---
    for t in prompt[:-1]:
        dec.decode_step(t)
    tok_buf = torch.tensor([prompt[-1]], dtype=torch.int32, device=dev)
    for _ in range(args.warmup):
        dec.decode_step_async(tok_buf.data_ptr(), tok_buf.data_ptr())
    dec.check()
    p_first = dec.position()
    barrier(world)
    with ClockSampler(local) as clk:
        total_ms = time_device_steps(dec, tok_buf, args.steps)
    dec.check()
    barrier(world)
    total_ms_max = max_over_ranks(total_ms, world)
    ms_step = total_ms_max / args.steps
    value = world * args.steps / (total_ms_max / 1000.0)
    launch_ms = total_ms / args.steps   # back-to-back launches: per-launch average
    p_mid = p_first + args.steps // 2
    achieved = bytes_per_token(p_mid) / (launch_ms / 1000.0) / 1e9

    # --- e2e through the public API: host token in, host token out each step ---
    cur = int(tok_buf.item())
    for _ in range(3):
        cur = dec.decode_step(cur)
    barrier(world)
    t0 = time.perf_counter()
    e2e_steps = args.steps
    for _ in range(e2e_steps):
        cur = dec.decode_step(cur)
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0, world)
    e2e = world * e2e_steps / e2e_s

    # --- position sweep (rank 0 reports) ---
    sweep = {}
    if not args.no_sweep:
        g = torch.Generator(device=dev).manual_seed(11)
        for P in args.sweep:
            dec.reset()
            if P <= 512:
                ids = seeded_prompt(P, seed=2).tolist() if P > 0 else []
                for t in ids:
                    dec.decode_step(t)
            else:
                kc, vc = dec.get_k_cache(), dec.get_v_cache()
                kc[:, :, :P].normal_(generator=g)
                vc[:, :, :P].normal_(generator=g)
                dec.set_position(P)
            buf = torch.tensor([5], dtype=torch.int32, device=dev)
            for _ in range(3):
                dec.decode_step_async(buf.data_ptr(), buf.data_ptr())
            n = args.sweep_steps
            tot = time_device_steps(dec, buf, n)
            dec.check()
            lm = tot / n
            pm = P + 3 + n // 2
            sweep[str(P)] = {"tok_s": round(n / (tot / 1000.0), 1),
                             "roofline_frac": round(bytes_per_token(pm) / (lm / 1000.0) / 1e9 / hbm, 4)}
        sweep_prefill = run_prefill(args, w, cos, sin, dev)
    else:
        sweep_prefill = None

    # --- batched decode (config 5): B independent sequences per GPU, one token each per step ---
    batch = run_batch(args, w, cos, sin, dev, hbm, world) if args.batch_sizes else {}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, n, cores, last = cpu_oracle_rate(args.cpu_budget)
        cpu = {"value": round(rate, 3), "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": f"{n} fp32 decode steps of the 28-layer model at positions 16..{last - 1} "
                         f"(~{args.cpu_budget:.0f} s)"}

    if rank == 0:
        line = {
            "metric": "batch-1 decode tok/s", "value": round(value, 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) weights, seeded prompt)",
            "config": {"workload": "config2: Qwen3-0.6B arch, 28 layers, batch-1 greedy decode after a 16-token "
                                   "seeded prompt, token fed back on device",
                       "positions": f"{p_first}..{p_first + args.steps - 1}", "batch_per_gpu": 1,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": "no flush: weights 1.19 GB streamed per token > 126 MB L2"},
            "gpu_launches": args.steps,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4),
                         "traffic": round(NCU_TRAFFIC_P20 * bytes_per_token(p_mid) / bytes_per_token(20)),
                         "traffic_source": "ncu capture at p~20, scaled by algorithmic bytes",
                         "peak_kind": hbm_kind, "bytes_per_launch": bytes_per_token(p_mid),
                         "launch_ms": round(launch_ms, 5)},
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 16,
                    "d2h_path": "token, error, info, seq written by the kernel to mapped pinned host memory"},
            "clocks": clk.summary(),
            "positions": sweep,
            "prefill": sweep_prefill,
            "batch_decode": batch or None,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=512)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--sweep", type=lambda s: [int(x) for x in s.split(",") if x], default=[1, 128, 512, 2048, 8192, 32768])
    ap.add_argument("--sweep-steps", type=int, default=64)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--batch-sizes", type=lambda s: [int(x) for x in s.split(",") if x], default=[16, 64])
    ap.add_argument("--batch-steps", type=int, default=32)
    ap.add_argument("--batch-positions", type=lambda s: [int(x) for x in s.split(",") if x], default=[16, 1024])
    ap.add_argument("--only-batch", action="store_true", help="run only the batched-decode measurements")
    ap.add_argument("--only-prefill", action="store_true", help="run only the prefill measurements")
    ap.add_argument("--prefill-batches", type=lambda s: [int(x) for x in s.split(",") if x], default=[1, 8])
    ap.add_argument("--prefill-reps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=12.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        world = int(os.environ.get("WORLD_SIZE", "1"))
        run_reference(args, rank, world)
        return
    rank, world, local = dist_setup(args.gpus)
    try:
        run_ours(args, rank, world, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
