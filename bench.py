#!/usr/bin/env python
"""Benchmark of the Foveal Pattention MLP forward (token-routed) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 8b]

One step = one token-routed forward (router + selection + block CSR + gated contraction + additive
stream) over one batch of the configuration's synthetic input (Llama-3-8B MLP shape by default:
x [8, 2048, 4096] bf16, 224 blocks, base 4, top-p 0.8, K in [8, 56]).  With N > 1 (torchrun, one
process per GPU) every rank processes its own batch with replicated weights: tokens are independent,
so there is no collective and the scaling is weak.

Prints one JSON line (rank 0): ``value`` = tokens/s over all ranks with inputs resident in HBM,
timed with CUDA events around exactly K steps (max over ranks); ``e2e`` = the same through the public
``FovealPattentionMLP.forward_host`` with the input copied from pinned host memory and the output
copied back every step (copies overlapped with compute, chunk by chunk); ``roofline`` = the dominant kernel's algorithmic FLOP rate against the measured bf16
peak; ``cpu_baseline`` = the CPU oracle on a token sample (rank 0, N = 1).

``--impl reference`` times the CPU restatement of the reference path (oracle/, all host threads) on a
bounded token sample per step, on rank 0 only.
"""

from __future__ import annotations

import argparse
import datetime
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import torch  # noqa: E402

fsi = importlib.import_module("foveal-sparse-indexer_b200")
configs = fsi.configs

METRIC = "Pattention-MLP fwd tokens/s & % bf16 tensor peak (8B shape), 1/2/4/8 B200 vs host CPU"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
KERNELS_PER_STEP = 4  # route_proj, route (selection + block lists), gateup, down


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="8b", help="8b (default) or 70b for the main measurement")
    ap.add_argument("--mode", choices=["default", "decode", "sweep", "blockshard", "variants"], default="default",
                    help="decode / sweep / variants print one JSON line per point instead of the bench line; "
                         "blockshard (torchrun, >= 2 ranks) times the parameter-block-sharded forward of --config")
    ap.add_argument("--chunks", type=int, default=1, help="blockshard: token chunks whose reduce-scatter "
                    "overlaps the next chunk's compute")
    ap.add_argument("--e2e-steps", type=int, default=0)
    ap.add_argument("--chunk-tokens", type=int, default=4096)
    ap.add_argument("--cpu-sample", type=int, default=8192,
                    help="tokens of the CPU-baseline sample (about 10-30 s of host work over 3 timed calls)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return FALLBACK_PEAKS, "fallback"


def tensor_peak(clk):
    """bf16 tensor peak for this run's fraction: the burst figure of the measured peaks, unless the clock
    record taken during the timed region shows ``sw_power_cap`` (then the sustained, power-capped one).
    Returns (peak TFLOP/s, note, {"burst": ..., "sustained": ...})."""
    peaks, src = load_peaks()
    burst = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    sus = float(peaks.get("bf16_tflops_sustained", burst))
    capped = "sw_power_cap" in (clk or {}).get("reasons", [])
    which = "sustained" if capped else "burst"
    note = (f"{src} bf16 {which} ({'MEASURED_PEAKS.json' if src == 'measured' else 'fallback'}): "
            f"the clock record of the timed region {'shows' if capped else 'does not show'} sw_power_cap "
            f"(median SM {clk.get('sm_mhz') if clk else None} MHz)")
    return (sus if capped else burst), note, {"burst": burst, "sustained": sus}


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def load_traffic():
    path = os.path.join(REPO, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


def config_block(wl, world):
    return {"workload": f"{wl.name}: token-routed Pattention MLP fwd", "model": "Llama-3-8B MLP shape"
            if wl.name == "8b" else wl.name, "tokens_per_rank": wl.tokens, "batch": wl.batch,
            "seq_len": wl.seq_len, "d_model": wl.hidden_dim, "param_tokens": wl.intermediate_dim,
            "blocks": wl.num_blocks, "base_blocks": wl.base_blocks, "top_p": wl.top_p,
            "k_min": wl.min_remote_blocks, "k_max": wl.max_remote_blocks, "routing": "token",
            "global_batch_tokens": wl.tokens * world, "parallelism": f"token-split x{world} (no collective)",
            "l2": "inputs larger than L2: x 134 MB + weights 352 MB + activations 470 MB per step vs 126 MB L2"}


# ------------------------------------------------------------------ clocks
def gpu_smi_id(dev, local: int) -> str:
    """nvidia-smi -i selector for this CUDA device (its UUID; the local index if unavailable)."""
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else f"GPU-{u}"
    except Exception:
        return str(local)


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        load = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ CPU baseline (oracle)
def cpu_oracle_rate(wl, w_cpu, x_cpu, sample: int, reps: int = 3):
    import oracle  # CPU baseline leg only
    torch.set_num_threads(os.cpu_count() or 1)
    xs = x_cpu[:sample].float().contiguous()
    kw = dict(base_blocks=wl.base_blocks, top_p=wl.top_p, min_remote_blocks=wl.min_remote_blocks,
              max_remote_blocks=wl.max_remote_blocks, temperature=wl.temperature)
    oracle.token_forward(xs[:16], w_cpu, **kw)  # warm-up
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        oracle.token_forward(xs, w_cpu, **kw)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": sample / med, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "cpu_model": cpu_model(),
            "sample": f"{sample} tokens of the {wl.name} workload, oracle token_forward (fp32 torch CPU), "
                      f"median of {reps} after 1 warm-up; {med:.2f} s per call"}


# ------------------------------------------------------------------ reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return
    import oracle  # reference arm: the CPU restatement of the reference path
    wl = configs.CONFIGS[args.config]
    torch.set_num_threads(os.cpu_count() or 1)
    w = configs.make_weights(wl)
    x2d = configs.make_x(wl).reshape(-1, wl.hidden_dim)
    kw = dict(base_blocks=wl.base_blocks, top_p=wl.top_p, min_remote_blocks=wl.min_remote_blocks,
              max_remote_blocks=wl.max_remote_blocks, temperature=wl.temperature)
    # size the per-step sample so that warm-up + steps stay within ~3 minutes
    sample = 64
    t0 = time.perf_counter()
    oracle.token_forward(x2d[:sample].contiguous(), w, **kw)
    per_tok = (time.perf_counter() - t0) / sample
    budget = 150.0 / max(1, args.steps + args.warmup)
    sample = int(max(16, min(1024, budget / max(per_tok, 1e-6))))
    xs = x2d[:sample].contiguous()
    for _ in range(args.warmup):
        oracle.token_forward(xs, w, **kw)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.token_forward(xs, w, **kw)
    dt = time.perf_counter() - t0
    value = sample * args.steps / dt
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) x, N(0,0.02) weights)",
        "impl": "reference", "config": config_block(wl, 1),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": f"{sample} tokens per step of the {wl.name} workload (oracle token_forward, "
                                   f"fp32 torch CPU restatement of the reference path)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def run_ours(args):
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    wl = configs.CONFIGS[args.config]
    w = configs.make_weights(wl)
    m = fsi.FovealPattentionMLP(hidden_dim=wl.hidden_dim, intermediate_dim=wl.intermediate_dim,
                                base_blocks=wl.base_blocks, remote_blocks=wl.max_remote_blocks,
                                temperature=wl.temperature, dtype=torch.bfloat16, routing="token", top_p=wl.top_p,
                                min_remote_blocks=wl.min_remote_blocks, max_remote_blocks=wl.max_remote_blocks)
    m.load_state_dict({k: t.to(torch.bfloat16) for k, t in w.state_dict().items()}, strict=False)
    m = m.to(dev).eval()
    x_cpu = configs.make_x(wl, seed=rank).reshape(-1, wl.hidden_dim)
    x = x_cpu.to(dev, torch.bfloat16)
    M, D = x.shape
    kg, ku, v, packed, wq, k16, wout = m._weights()
    kw = dict(base_blocks=wl.base_blocks, top_p=wl.top_p, min_remote=wl.min_remote_blocks,
              max_remote=wl.max_remote_blocks, temperature=wl.temperature, additive=True)

    def step(y_out):
        fsi.kernels.token_forward(x, kg, ku, v, packed, wq, k16, wout, y=y_out, **kw)

    y = torch.empty(M, D, dtype=torch.bfloat16, device=dev)
    with torch.no_grad():
        for _ in range(args.warmup):
            step(y)
        # mean active blocks per token of this workload (for the algorithmic FLOP count)
        _, _, cnt, _ = fsi.kernels.token_forward(x, kg, ku, v, packed, wq, k16, wout, want_routes=True, **kw)
        a_mean = wl.base_blocks + float(cnt.float().mean())
        torch.cuda.synchronize()

        K = args.steps
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(K)]
        for row in ev:
            for e in row:
                e.record()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        clocks = ClockSampler(gpu_smi_id(dev, local))
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        clocks.start()
        time.sleep(0.3)  # let the sampler attach before the timed region
        start.record()
        for k in range(K):
            fsi._lib.set_stage_events(ev[k])
            step(y)
        end.record()
        torch.cuda.synchronize()
        fsi._lib.set_stage_events(None)
        clk = clocks.stop()
        t_ms = start.elapsed_time(end)
        if world > 1:
            t = torch.tensor([t_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_ms = float(t.item())
        stage = [statistics.mean(ev[k][i].elapsed_time(ev[k][i + 1]) for k in range(K)) for i in range(4)]

        err = fsi._lib.device_error(fsi._lib.workspace(dev, 0))

        # e2e through the public API: pinned host input -> forward -> pinned host output, every step
        E = args.e2e_steps or max(10, K // 10)
        x_host = x_cpu.to(torch.bfloat16).pin_memory()
        y_hosts = [torch.empty(M, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        cur = torch.cuda.current_stream(dev)

        def e2e_step(k):
            # pipelined batches: batch k+1's copy-in overlaps batch k's last chunks; the output buffer
            # of batch k is reused by batch k+2 only after batch k's result is complete
            y_host = y_hosts[k % 2]
            if done[k % 2] is not None:
                done[k % 2].synchronize()
            _, done[k % 2] = m.forward_host_async(x_host, out=y_host, chunk_tokens=args.chunk_tokens)

        done = [None, None]
        for k in range(3):
            e2e_step(k)
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        done = [None, None]
        s2.record()
        for k in range(E):
            e2e_step(k)
        for d_ in done:
            if d_ is not None:
                cur.wait_event(d_)
        e2.record()
        torch.cuda.synchronize()
        e2_ms = s2.elapsed_time(e2)
        if world > 1:
            t = torch.tensor([e2_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2_ms = float(t.item())

    value = world * M * K / (t_ms / 1e3)
    ms_step = t_ms / K
    peak, peak_note, peaks_all = tensor_peak(clk)
    gu_flops = 4.0 * D * 64 * a_mean * M
    dn_flops = 2.0 * D * 64 * a_mean * M
    # stage events: 0 start, 1 routed (block lists built in the same kernel), 2 = 1, 3 gate/up, 4 down
    stage = [stage[0] + stage[1], 0.0, stage[2], stage[3]]
    names = ["route", "lists", "gateup", "down"]
    dom = 2 if stage[2] >= stage[3] else 3
    dom_flops = gu_flops if dom == 2 else dn_flops
    achieved = dom_flops / (stage[dom] / 1e3) / 1e12
    traffic = load_traffic().get(f"{wl.name}_{names[dom]}")
    total_flops = gu_flops + dn_flops
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) x, N(0,0.02) weights)",
        "config": config_block(wl, world),
        "tensor_peak_frac": total_flops / (ms_step / 1e3) / 1e12 / peak,
        "tensor_peak_frac_both": {k: total_flops / (ms_step / 1e3) / 1e12 / v for k, v in peaks_all.items()},
        "active_blocks_per_token": a_mean,
        "stages_ms": {n: s for n, s in zip(names, stage) if n != "lists"},
        "roofline": {"bound": "tensor", "kernel": names[dom], "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic, "peak_source": peak_note,
                     "frac_both": {k: achieved / v for k, v in peaks_all.items()},
                     "algorithmic_flops_per_launch": dom_flops},
        "e2e": {"value": world * M * E / (e2_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": M * D * 2, "d2h_bytes_per_step": M * D * 2,
                "path": "FovealPattentionMLP.forward_host_async: pinned host x -> device -> pinned host y, "
                        f"{args.chunk_tokens}-token chunks, copies overlapped with compute, consecutive "
                        "batches pipelined"},
        "gpu_launches": KERNELS_PER_STEP * K,
        "clocks": clk,
        "device_error": err,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_oracle_rate(wl, w, x_cpu, args.cpu_sample)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ extra measurement modes
def _module_for(wl, w, dev):
    m = fsi.FovealPattentionMLP(hidden_dim=wl.hidden_dim, intermediate_dim=wl.intermediate_dim,
                                base_blocks=wl.base_blocks, remote_blocks=wl.max_remote_blocks,
                                temperature=wl.temperature, dtype=torch.bfloat16, routing="token", top_p=wl.top_p,
                                min_remote_blocks=wl.min_remote_blocks, max_remote_blocks=wl.max_remote_blocks)
    m.load_state_dict({k: t.to(torch.bfloat16) for k, t in w.state_dict().items()}, strict=False)
    return m.to(dev).eval()


def _time_calls(fn, n, warm=5):
    for _ in range(warm):
        fn()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    torch.cuda.synchronize()
    for a, b in ev:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    return sorted(a.elapsed_time(b) for a, b in ev)


def run_decode(args):
    """Decode step (64 tokens, 8B shape), K_max in {8, 16, 32}: p50 latency per call and GB/s."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks, src = load_peaks()
    for wl in configs.decode_points():
        w = configs.make_weights(wl)
        m = _module_for(wl, w, dev)
        x = configs.make_x(wl).reshape(-1, wl.hidden_dim).to(dev, torch.bfloat16)
        with torch.no_grad():
            _, info = m(x, return_router_info=True)
            cnt, idx = info["remote_counts"], info["remote_indices"]
            used = torch.zeros(wl.num_blocks, dtype=torch.bool, device=dev)
            used[:wl.base_blocks] = True
            for t in range(x.shape[0]):
                used[idx[t, :int(cnt[t])].long()] = True
            nb = int(used.sum())
            ts = _time_calls(lambda: m(x), 200)
            # the same call captured once in a CUDA graph and replayed (how a decode loop runs it)
            gs = torch.cuda.Stream(dev)
            gs.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(gs):
                for _ in range(3):
                    m(x)
            torch.cuda.current_stream(dev).wait_stream(gs)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                m(x)
            tg = _time_calls(graph.replay, 200)
            del graph
        p50 = ts[len(ts) // 2]
        g50 = tg[len(tg) // 2]
        D = wl.hidden_dim
        alg_bytes = 3 * 64 * D * 2 * nb + 2 * x.numel() * 2          # touched blocks (gate, up, v) + x + y
        moved = (2 * 64 * D * 2 * nb) + wl.intermediate_dim * D * 2 + 2 * x.numel() * 2  # v_t read whole
        print(json.dumps({"mode": "decode", "config": wl.name, "tokens": x.shape[0], "k_max": wl.max_remote_blocks,
                          "p50_ms": p50, "p10_ms": ts[len(ts) // 10], "p90_ms": ts[9 * len(ts) // 10],
                          "graph_p50_ms": g50, "graph_tokens_per_s": x.shape[0] / (g50 / 1e3),
                          "graph_algorithmic_GBps": alg_bytes / (g50 / 1e3) / 1e9,
                          "tokens_per_s": x.shape[0] / (p50 / 1e3), "blocks_touched": nb,
                          "algorithmic_GBps": alg_bytes / (p50 / 1e3) / 1e9,
                          "moved_GBps": moved / (p50 / 1e3) / 1e9, "hbm_peak_GBps": peaks["hbm_gbs"]}), flush=True)


def run_sweep(args):
    """Sparsity sweep (x [4, 4096, 4096], 8B shape): tokens/s per (top_p, K_max) and the speedup over
    the dense SwiGLU equivalent (all 224 blocks, same kernels; and cuBLAS through torch)."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    pts = configs.sweep_points()
    w = configs.make_weights(pts[0])
    x = configs.make_x(pts[0]).reshape(-1, pts[0].hidden_dim).to(dev, torch.bfloat16)
    M = x.shape[0]
    with torch.no_grad():
        m = _module_for(pts[0], w, dev)
        kg, ku, v, packed, wq, k16, wout = m._weights()
        active = torch.arange(pts[0].num_blocks, dtype=torch.int32, device=dev)
        dense_ours = _time_calls(lambda: fsi.kernels.pooled_forward(x, kg, ku, v, packed, active), 10)
        import torch.nn.functional as F
        dense_torch = _time_calls(lambda: F.linear(F.silu(F.linear(x, kg)) * F.linear(x, ku), v.t()), 10)
        d_ours, d_torch = dense_ours[len(dense_ours) // 2], dense_torch[len(dense_torch) // 2]
        for wl in pts:
            mm = _module_for(wl, w, dev)
            _, info = mm(x, return_router_info=True)
            a_mean = wl.base_blocks + float(info["remote_counts"].float().mean())
            ts = _time_calls(lambda: mm(x), 10)
            t = ts[len(ts) // 2]
            print(json.dumps({"mode": "sweep", "top_p": wl.top_p, "k_max": wl.max_remote_blocks,
                              "active_blocks_per_token": a_mean, "active_fraction": a_mean / wl.num_blocks,
                              "ms": t, "tokens_per_s": M / (t / 1e3),
                              "speedup_vs_dense_same_kernels": d_ours / t, "speedup_vs_dense_cublas": d_torch / t,
                              "dense_ms_same_kernels": d_ours, "dense_ms_cublas": d_torch}), flush=True)


def _variant_module(case, dev):
    kind = case["kind"]
    cls = {"bsl": fsi.BlockSparseLinear, "tf": fsi.FovealTokenformerLinear, "ffn": fsi.FovealTokenformerFFN}[kind]
    m = cls(**configs.variant_kwargs(case))
    m.load_state_dict(configs.variant_params(m, 0, "bf16"))
    return m.to(dev, torch.bfloat16).eval()


def run_variants(args):
    """Layers that share the router (bf16, inference): BlockSparseLinear with the 8B MLP's up-projection
    shape at 16384 / 64 / 1 tokens and a Tokenformer FFN at 16384 tokens.  Per point: the routed
    forward (block keys cached; scores, selection, union, contraction; no host synchronisation) and the
    contraction alone, both by CUDA events (median of 20), the union size, useful TFLOP/s (over the
    union) against the measured bf16 peak, the dense equivalent through cuBLAS (torch) and the oracle
    on the host cores for a 64-token sample."""
    import oracle  # CPU baseline only

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peaks, src = load_peaks()
    peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    for name, token_counts in (("bsl_8b", (16384, 64, 1)), ("tf_ffn", (16384,))):
        case = configs.VARIANT_BENCH[name]
        m = _variant_module(case, dev)
        x_all = configs.variant_x(case, 0, "bf16").reshape(-1, case["x_shape"][-1])
        for M in token_counts:
            x = x_all[:M].to(dev, torch.bfloat16).contiguous()
            with torch.no_grad():
                if case["kind"] == "bsl":
                    r = m.forward_kernels(x, fast=True)
                    n_act = int(r["n_active"].item())
                    blocks, n_active, ctx16 = r["blocks"], r["n_active"], r["ctx16"]
                    t_all = _time_calls(lambda: m.forward_kernels(x, fast=True), 20)
                    t_mm = _time_calls(lambda: fsi.kernels.block_sparse_linear(
                        x, m.weight, m.bias, blocks, n_active, ctx16, m.indexer.out_proj.weight), 20)
                    flops = 2.0 * M * case["in_features"] * n_act * 64
                    W = m.weight
                    t_dense = _time_calls(lambda: torch.nn.functional.linear(x, W), 20)
                    union = {"union_blocks": n_act, "total_blocks": m.num_blocks}
                    if M <= 64:
                        # decode-sized batches run from a CUDA graph (no host work per call)
                        gs = torch.cuda.Stream(dev)
                        gs.wait_stream(torch.cuda.current_stream(dev))
                        with torch.cuda.stream(gs):
                            for _ in range(3):
                                m.forward_kernels(x, fast=True)
                        torch.cuda.current_stream(dev).wait_stream(gs)
                        graph = torch.cuda.CUDAGraph()
                        with torch.cuda.graph(graph):
                            m.forward_kernels(x, fast=True)
                        tg = _time_calls(graph.replay, 50)
                        union["graph_ms"] = tg[len(tg) // 2]
                        del graph
                else:
                    t_all = _time_calls(lambda: m.forward_kernels(x), 20)
                    unions, flops = [], 0.0
                    h = x
                    for layer in (m.fc1, m.fc2):
                        r = layer.forward_kernels(h)
                        n_act = int(r["n_active"].item())
                        unions.append(n_act)
                        flops += 2.0 * M * n_act * 64 * (layer.in_features + layer.out_features)
                        h = r["out"]
                    t_mm = None
                    kp1, vp1, kp2, vp2 = m.fc1.k_param, m.fc1.v_param, m.fc2.k_param, m.fc2.v_param

                    def dense():
                        a = torch.nn.functional.gelu(torch.nn.functional.normalize(x @ kp1.t(), dim=-1)) @ vp1
                        return torch.softmax((a @ kp2.t()) / math.sqrt(m.fc2.in_features), dim=-1) @ vp2
                    t_dense = _time_calls(dense, 20)
                    union = {"union_blocks_fc1_fc2": unions, "total_blocks": m.fc1.num_blocks}
            tm = t_all[len(t_all) // 2]
            line = {"mode": "variants", "layer": name, "tokens": M, **union, "ms": tm,
                    "tokens_per_s": M / (tm / 1e3), "useful_tflops": flops / (tm / 1e3) / 1e12,
                    "tensor_peak_frac": flops / (tm / 1e3) / 1e12 / peak, "peak_tflops": peak, "peak_source": src,
                    "dense_torch_cublas_ms": t_dense[len(t_dense) // 2]}
            if t_mm is not None:
                c = t_mm[len(t_mm) // 2]
                line.update({"contraction_ms": c, "contraction_tflops": flops / (c / 1e3) / 1e12})
            print(json.dumps(line), flush=True)
        # CPU baseline: the oracle on a 64-token sample on the host cores
        if not args.no_cpu_baseline:
            xs = x_all[:64].float()
            p = {k: v.detach().float().cpu() for k, v in m.state_dict().items()}
            t0 = time.perf_counter()
            if case["kind"] == "bsl":
                oracle.block_sparse_linear(xs, p["weight"], p.get("bias"), p["indexer.q_proj.weight"],
                                           p["weight_to_k.weight"], p["weight_to_v.weight"],
                                           p["indexer.out_proj.weight"], block_size=64,
                                           base_blocks=case["base_blocks"], top_p=case["top_p"], min_remote_blocks=0,
                                           max_remote_blocks=case["max_remote_blocks"],
                                           remote_capacity=case["remote_capacity"], fast_rule=True)
            else:
                h = xs
                for f, act in (("fc1.", "gelu_l2"), ("fc2.", "softmax")):
                    h = oracle.tokenformer_linear(h, p[f + "k_param"], p[f + "v_param"], p[f + "indexer.q_proj.weight"],
                                                  p[f + "indexer.k_proj.weight"], p[f + "indexer.v_proj.weight"],
                                                  p[f + "indexer.out_proj.weight"], block_size=64,
                                                  base_blocks=case["base_blocks"], top_p=case["top_p"],
                                                  min_remote_blocks=0, max_remote_blocks=case["max_remote_blocks"],
                                                  remote_capacity=4, activation=act)[0]
            dt = time.perf_counter() - t0
            print(json.dumps({"mode": "variants", "layer": name, "cpu_baseline": {
                "value": 64 / dt, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                "sample": "64 tokens, oracle (fp32 torch CPU) incl. block keys"}}), flush=True)


def run_blockshard(args):
    """Parameter-block sharding (strong scaling): every rank holds the same batch, computes the blocks
    b % world == rank, and the fp32 partials are reduce-scattered over token rows chunk by chunk (NCCL on
    a side stream, overlapping the next chunk's compute).  One JSON line: tokens/s of the whole batch
    (max over ranks), and the same forward without the collectives for reference."""
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2:
        raise SystemExit("--mode blockshard needs torchrun with at least 2 ranks")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    wl = configs.CONFIGS[args.config if args.config != "8b" else "70b"]
    w = configs.make_weights(wl)
    m = fsi.FovealPattentionMLP(hidden_dim=wl.hidden_dim, intermediate_dim=wl.intermediate_dim,
                                base_blocks=wl.base_blocks, remote_blocks=wl.max_remote_blocks,
                                temperature=wl.temperature, dtype=torch.bfloat16, routing="token", top_p=wl.top_p,
                                min_remote_blocks=wl.min_remote_blocks, max_remote_blocks=wl.max_remote_blocks)
    m.load_state_dict({k: t.to(torch.bfloat16) for k, t in w.state_dict().items()}, strict=False)
    m = m.to(dev).eval()
    fsi.sharding.shard_parameter_blocks(m)
    x = configs.make_x(wl).reshape(-1, wl.hidden_dim).to(dev, torch.bfloat16)
    M, D = x.shape
    chunks = max(1, args.chunks)

    def step():
        fsi.sharding.sharded_token_forward(m, x, reduce="scatter", chunks=chunks)

    def compute_only():
        fsi.sharding._cuda_partial(m, x, world, rank, rank == 0, False)

    def timed(fn, K):
        dist.barrier()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(K):
            fn()
        s1.record()
        torch.cuda.synchronize()
        t = torch.tensor([s0.elapsed_time(s1) / K], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.no_grad():
        for _ in range(max(3, args.warmup)):
            step()
            compute_only()
        ms = timed(step, args.steps)
        ms_compute = timed(compute_only, args.steps)
    if rank == 0:
        line = {"mode": "blockshard", "metric": METRIC, "value": M / (ms / 1e3), "unit": "tokens/s",
                "n_gpus": world, "steps": args.steps, "ms_per_step": ms, "scaling": "strong",
                "higher_is_better": True, "dtype": "bf16", "data": "synthetic (seeded)",
                "config": {"workload": f"{wl.name}: token-routed forward, parameter blocks sharded b % {world}",
                           "tokens": M, "d_model": D, "blocks": wl.num_blocks, "chunks": chunks,
                           "parallelism": f"block-shard x{world} + NCCL reduce-scatter (fp32 partials)"},
                "compute_only_ms": ms_compute,
                "collective_bytes_per_rank": M * D * 4}
        print(json.dumps(line), flush=True)
    dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "decode":
        run_decode(args)
    elif args.mode == "sweep":
        run_sweep(args)
    elif args.mode == "blockshard":
        run_blockshard(args)
    elif args.mode == "variants":
        run_variants(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
