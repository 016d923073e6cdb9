#!/usr/bin/env python
"""Benchmark of the Foveal Pattention MLP forward (token-routed) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 8b]

One step = one token-routed forward (router + selection + block CSR + gated contraction + additive
stream) over one batch of the configuration's synthetic input (Llama-3-8B MLP shape by default:
x [8, 2048, 4096] bf16, 224 blocks, base 4, top-p 0.8, K in [8, 56]).

N = 1: ``value`` = tokens/s with inputs resident in HBM, CUDA events around exactly K steps; ``e2e`` =
the same through ``FovealPattentionMLP.forward_host_async`` with pinned host input and output every step;
``roofline`` = the dominant kernel's useful FLOP rate against the measured bf16 peak (burst, or sustained
when the clock record of the timed region shows the power cap); ``cpu_baseline`` = the CPU oracle on a
token sample.  Extra keys timed in the same run: ``decode`` (config 3), ``sweep`` (config 5), ``70b``
(config 4 on one GPU) and ``pooled`` (the reference's default pooled routing against its cuBLAS path).

N > 1 (torchrun, one process per GPU, NCCL): one global batch of the configuration, parameter blocks
sharded over the ranks and bf16 partial outputs reduce-scattered over token rows chunk by chunk (strong
scaling, max over ranks); ``token_split`` (every rank its own batch, no collective), ``e2e`` from each
rank's slice of the batch in pinned host memory, and ``blockshard_70b`` (the 70B configuration sharded,
with its 1-GPU time measured by the same processes).

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
# block-sharded step with split routing, per token chunk: route_proj + route of this rank's tokens, the
# routing kernel's block-list pass over the given routes, gateup, down
KERNELS_PER_SHARDED_CHUNK = 5
# the same through peer memory (one piece): those five, the route exchange (two puts, flag, wait), the
# output flag and the combine
KERNELS_PEER_STEP = 11


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default="8b", help="8b (default) or 70b for the main measurement")
    ap.add_argument("--mode", choices=["default", "decode", "sweep", "pooled", "70b", "variants"], default="default",
                    help="decode / sweep / pooled / 70b print one of the N = 1 line's extra keys alone; variants "
                         "prints one JSON line per BlockSparseLinear / Tokenformer point")
    ap.add_argument("--e2e-steps", type=int, default=0)
    ap.add_argument("--chunk-tokens", type=int, default=4096)
    ap.add_argument("--cpu-sample", type=int, default=8192,
                    help="tokens of the CPU-baseline sample (about 10-30 s of host work over 3 timed calls)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the decode / sweep / 70B / pooled keys")
    ap.add_argument("--shard-chunks", type=int, default=1,
                    help="N > 1: token chunks of the device-resident block-sharded step (1: the routes are "
                         "split over the ranks and the whole batch runs as one piece; measured fastest)")
    ap.add_argument("--reduce", choices=["nccl", "peer"], default="peer",
                    help="N > 1: sum of the block shards' partials through peer memory (the down projection "
                         "stores each row's partial on the rank that owns it; measured faster at 2 and 8 GPUs), "
                         "or by the NCCL reduce-scatter")
    ap.add_argument("--e2e-chunks", type=int, default=4,
                    help="N > 1: token chunks of the host-buffer block-sharded step (copies overlap compute)")
    ap.add_argument("--partial-dtype", choices=["bf16", "fp32"], default="bf16",
                    help="N > 1: dtype of the partial outputs the reduce-scatter sums")
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


def config_block(wl, world, parallelism, global_tokens=None):
    return {"workload": f"{wl.name}: token-routed Pattention MLP fwd", "model": "Llama-3-8B MLP shape"
            if wl.name == "8b" else wl.name, "batch": wl.batch,
            "seq_len": wl.seq_len, "d_model": wl.hidden_dim, "param_tokens": wl.intermediate_dim,
            "blocks": wl.num_blocks, "base_blocks": wl.base_blocks, "top_p": wl.top_p,
            "k_min": wl.min_remote_blocks, "k_max": wl.max_remote_blocks, "routing": "token",
            "global_batch_tokens": wl.tokens if global_tokens is None else global_tokens,
            "parallelism": parallelism,
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
        "impl": "reference", "config": config_block(wl, 1, "host CPU (oracle port, all threads)"),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": f"{sample} tokens per step of the {wl.name} workload (oracle token_forward, "
                                   f"fp32 torch CPU restatement of the reference path)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def make_module(wl, w, dev, routing="token", remote_blocks=None):
    """bf16 module of workload ``wl`` on ``dev`` holding the values of ``w`` (CPU or device tensors)."""
    m = fsi.FovealPattentionMLP(hidden_dim=wl.hidden_dim, intermediate_dim=wl.intermediate_dim,
                                base_blocks=wl.base_blocks,
                                remote_blocks=wl.max_remote_blocks if remote_blocks is None else remote_blocks,
                                temperature=wl.temperature, dtype=torch.bfloat16, routing=routing, top_p=wl.top_p,
                                min_remote_blocks=wl.min_remote_blocks, max_remote_blocks=wl.max_remote_blocks,
                                device=dev)
    with torch.no_grad():
        for k, t in w.state_dict().items():
            m.get_parameter(k).copy_(t.to(dev, torch.bfloat16))
    return m.eval()


def set_router(m, wl):
    """Point a token-routed module at another workload's router settings (same weights)."""
    m.top_p, m.min_remote_blocks, m.max_remote_blocks = wl.top_p, wl.min_remote_blocks, wl.max_remote_blocks


def timed_steps(step, K, dev, world, clocks=None):
    """K calls of ``step`` between a barrier + synchronize on both sides; CUDA events on the current stream.
    Returns (ms over the K steps, max over ranks; clock record or None)."""
    import torch.distributed as dist
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.start()
        time.sleep(0.3)  # let the sampler attach before the timed region
    s0.record()
    for _ in range(K):
        step()
    s1.record()
    torch.cuda.synchronize()
    clk = clocks.stop() if clocks is not None else None
    t = s0.elapsed_time(s1)
    if world > 1:
        tt = torch.tensor([t], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t = float(tt.item())
    return t, clk


def mean_active(m, x):
    """Mean active blocks per token (base + remote count) of one forward of ``x``."""
    _, info = m(x, return_router_info=True)
    return m.base_blocks + float(info["remote_counts"].float().mean())


def roofline_block(stage, a_mean, M, D, clk, names=("route", "gateup", "down")):
    """The dominant tensor-core kernel's useful FLOP rate against the bf16 peak."""
    gu_flops = 4.0 * D * 64 * a_mean * M
    dn_flops = 2.0 * D * 64 * a_mean * M
    dom = "gateup" if stage["gateup"] >= stage["down"] else "down"
    dom_flops = gu_flops if dom == "gateup" else dn_flops
    achieved = dom_flops / (stage[dom] / 1e3) / 1e12
    peak, note, peaks_all = tensor_peak(clk)
    return {"bound": "tensor", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak, "traffic": load_traffic().get(f"8b_{dom}"), "peak_source": note,
            "frac_both": {k: achieved / v for k, v in peaks_all.items()},
            "algorithmic_flops_per_launch": dom_flops}, gu_flops + dn_flops, peak, peaks_all


def stage_split(run, K=10):
    """Mean CUDA-event stage times (ms) of ``run`` (one token-routed forward): route, gate/up, down."""
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(K)]
    for row in ev:
        for e in row:
            e.record()
    torch.cuda.synchronize()
    for k in range(K):
        fsi._lib.set_stage_events(ev[k])
        run()
    torch.cuda.synchronize()
    fsi._lib.set_stage_events(None)
    st = [statistics.mean(ev[k][i].elapsed_time(ev[k][i + 1]) for k in range(K)) for i in range(4)]
    return {"route": st[0] + st[1], "gateup": st[2], "down": st[3]}


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
    if world > 1:
        line = run_ours_sharded(args, rank, world, local, dev)
        dist.barrier()
        dist.destroy_process_group()
    else:
        line = run_ours_single(args, local, dev)
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_ours_single(args, local, dev):
    """N = 1: the token-routed forward of --config, device-resident and end to end, plus (unless
    --no-extras) the decode, sparsity-sweep, 70B and pooled-routing figures of the other configurations,
    each timed in this run."""
    wl = configs.CONFIGS[args.config]
    w = configs.make_weights(wl)
    m = make_module(wl, w, dev)
    x_cpu = configs.make_x(wl).reshape(-1, wl.hidden_dim)
    x = x_cpu.to(dev, torch.bfloat16)
    M, D = x.shape
    kg, ku, v, packed, wq, k16, wout = m._weights()
    kw = dict(base_blocks=wl.base_blocks, top_p=wl.top_p, min_remote=wl.min_remote_blocks,
              max_remote=wl.max_remote_blocks, temperature=wl.temperature, additive=True)
    y = torch.empty(M, D, dtype=torch.bfloat16, device=dev)

    def step():
        fsi.kernels.token_forward(x, kg, ku, v, packed, wq, k16, wout, y=y, **kw)

    K = args.steps
    with torch.no_grad():
        for _ in range(args.warmup):
            step()
        a_mean = mean_active(m, x)
        t_ms, clk = timed_steps(step, K, dev, 1, ClockSampler(gpu_smi_id(dev, local)))
        stage = stage_split(step)
        err = fsi._lib.device_error(fsi._lib.workspace(dev, 0))
        e2e = measure_e2e_single(args, m, x_cpu, dev)

    ms_step = t_ms / K
    roof, total_flops, peak, peaks_all = roofline_block(stage, a_mean, M, D, clk)
    line = {
        "metric": METRIC, "value": M * K / (t_ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": K,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) x, N(0,0.02) weights)",
        "config": config_block(wl, 1, "single GPU"),
        "tensor_peak_frac": total_flops / (ms_step / 1e3) / 1e12 / peak,
        "tensor_peak_frac_both": {k: total_flops / (ms_step / 1e3) / 1e12 / p_ for k, p_ in peaks_all.items()},
        "active_blocks_per_token": a_mean,
        "stages_ms": stage,
        "roofline": roof,
        "e2e": e2e,
        "gpu_launches": KERNELS_PER_STEP * K,
        "clocks": clk,
        "device_error": err,
    }
    if not args.no_extras:
        with torch.no_grad():
            line["decode"] = extra_decode(m, x, dev)
            line["sweep"] = extra_sweep(m, x, dev)
            line["pooled"] = extra_pooled(wl, m, x, dev)
            del kg, ku, v, packed, wq, k16, wout
            del m
            fsi._lib.release_workspaces()
            torch.cuda.empty_cache()
            line["70b"] = extra_70b(args, dev)
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_oracle_rate(wl, w, x_cpu, args.cpu_sample)
    return line


def measure_e2e_single(args, m, x_cpu, dev):
    """The same forward through the public API with host buffers: pinned host x -> device -> pinned host y
    every step (FovealPattentionMLP.forward_host_async, consecutive batches pipelined)."""
    M, D = x_cpu.shape
    E = args.e2e_steps or max(10, args.steps // 10)
    x_host = x_cpu.to(torch.bfloat16).pin_memory()
    y_hosts = [torch.empty(M, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    cur = torch.cuda.current_stream(dev)
    done = [None, None]

    def e2e_step(k):
        # batch k+1's copy-in overlaps batch k's last chunks; batch k's output buffer is reused by batch
        # k+2 only after batch k's result is complete
        if done[k % 2] is not None:
            done[k % 2].synchronize()
        _, done[k % 2] = m.forward_host_async(x_host, out=y_hosts[k % 2], chunk_tokens=args.chunk_tokens)

    for k in range(3):
        e2e_step(k)
    torch.cuda.synchronize()
    done = [None, None]
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record()
    for k in range(E):
        e2e_step(k)
    for d_ in done:
        if d_ is not None:
            cur.wait_event(d_)
    e2.record()
    torch.cuda.synchronize()
    e2_ms = s2.elapsed_time(e2)
    return {"value": M * E / (e2_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": M * D * 2,
            "d2h_bytes_per_step": M * D * 2, "steps": E,
            "path": "FovealPattentionMLP.forward_host_async: pinned host x -> device -> pinned host y, "
                    f"{args.chunk_tokens}-token chunks, copies overlapped with compute, consecutive batches "
                    "pipelined"}


# ------------------------------------------------------------------ the other configurations (N = 1)
def extra_decode(m, x8, dev):
    """Config 3: 64 decode tokens (the first 64 rows of the 8B input, the same weights), top-p 0.9,
    K_max 8 / 16 / 32.  p50 per call, eager and replayed from a CUDA graph, and GB/s of the blocks the
    call touches (gate, up and v rows) plus x and y, against the measured HBM copy bandwidth."""
    peaks, _ = load_peaks()
    x = x8[:64].contiguous()
    out = []
    for wl in configs.decode_points():
        set_router(m, wl)
        _, info = m(x, return_router_info=True)
        cnt, idx = info["remote_counts"], info["remote_indices"]
        used = torch.zeros(wl.num_blocks, dtype=torch.bool, device=dev)
        used[:wl.base_blocks] = True
        used[idx.long().masked_fill(torch.arange(idx.shape[1], device=dev)[None] >= cnt[:, None].long(), 0)] = True
        nb = int(used.sum())
        ts = _time_calls(lambda: m(x), 100)
        gs = torch.cuda.Stream(dev)
        gs.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(gs):
            for _ in range(3):
                m(x)
        torch.cuda.current_stream(dev).wait_stream(gs)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            m(x)
        tg = _time_calls(graph.replay, 100)
        del graph
        D = wl.hidden_dim
        alg_bytes = 3 * 64 * D * 2 * nb + 2 * x.numel() * 2
        p50, g50 = ts[len(ts) // 2], tg[len(tg) // 2]
        out.append({"k_max": wl.max_remote_blocks, "p50_ms": round(p50, 5), "graph_p50_ms": round(g50, 5),
                    "blocks_touched": nb, "GBps": round(alg_bytes / (g50 / 1e3) / 1e9, 1),
                    "hbm_frac": round(alg_bytes / (g50 / 1e3) / 1e9 / peaks["hbm_gbs"], 3)})
    set_router(m, configs.CONFIGS["8b"])
    return {"tokens": 64, "top_p": 0.9, "points": out,
            "bytes": "gate, up and v rows of the touched blocks + x + y (graph p50)"}


def extra_sweep(m, x, dev):
    """Config 5 (x [4, 4096, 4096]: the same 16384 rows and weights as the 8B input): tokens/s of the
    token-routed forward at every (top_p, K_max) point and its speed-up over the dense SwiGLU (all 224
    blocks) through this library's kernels and through cuBLAS (torch)."""
    import torch.nn.functional as F
    kg, ku, v, packed, *_ = m._weights()
    active = torch.arange(m.num_blocks, dtype=torch.int32, device=dev)
    d_ours = _median(_time_calls(lambda: fsi.kernels.pooled_forward(x, kg, ku, v, packed, active), 10))
    d_cublas = _median(_time_calls(lambda: F.linear(F.silu(F.linear(x, kg)) * F.linear(x, ku), v.t()), 10))
    pts = []
    for wl in configs.sweep_points():
        set_router(m, wl)
        a = mean_active(m, x)
        t = _median(_time_calls(lambda: m(x), 10))
        pts.append([wl.top_p, wl.max_remote_blocks, round(a, 1), round(x.shape[0] / (t / 1e3) / 1e6, 3),
                    round(d_ours / t, 2), round(d_cublas / t, 2)])
    set_router(m, configs.CONFIGS["8b"])
    return {"columns": ["top_p", "k_max", "active_blocks_per_token", "Mtokens_per_s", "x_dense_same_kernels",
                        "x_dense_cublas"], "points": pts, "dense_ms_same_kernels": round(d_ours, 4),
            "dense_ms_cublas": round(d_cublas, 4)}


def extra_pooled(wl, m_tok, x, dev):
    """The reference's default routing (pooled, eval: one active set of base 4 + 20 remote blocks, cached)
    at the 8B shape, against the reference's own GPU execution of that path restated with torch (the
    cached active rows gathered once, then two cuBLAS projections, SiLU * up, and the cuBLAS down
    projection; foveal_pattention.py:278-288 / :329-335, its Triton SwiGLU replaced by torch
    elementwise)."""
    import torch.nn.functional as F
    mp_ = fsi.FovealPattentionMLP(hidden_dim=wl.hidden_dim, intermediate_dim=wl.intermediate_dim,
                                  base_blocks=4, remote_blocks=20, dtype=torch.bfloat16, device=dev).eval()
    with torch.no_grad():
        for k in ("k_gate", "k_up", "v", "q_proj_16d.weight", "block_keys_16d", "out_proj_16d.weight"):
            mp_.get_parameter(k).copy_(m_tok.get_parameter(k))
    x3 = x.view(8, -1, wl.hidden_dim)
    mp_(x3)  # routes once on the pooled query and caches the active set
    t_ours = _median(_time_calls(lambda: mp_(x3), 20))
    idx = (mp_._cached_active_blocks.long()[:, None] * 64 + torch.arange(64, device=dev)).flatten()
    kg_a, ku_a, v_a = (mp_.k_gate[idx].detach().contiguous(), mp_.k_up[idx].detach().contiguous(),
                       mp_.v[idx].detach().contiguous())
    t_ref = _median(_time_calls(lambda: F.linear(F.silu(F.linear(x, kg_a)) * F.linear(x, ku_a), v_a.t()), 20))
    flops = 6.0 * wl.hidden_dim * 64 * 24 * x.shape[0]
    return {"active_blocks": 24, "tokens": x.shape[0], "ms": round(t_ours, 4), "tflops": round(flops / t_ours / 1e9, 1),
            "reference_gpu_path_ms": round(t_ref, 4), "speedup_vs_reference_gpu_path": round(t_ref / t_ours, 3)}


def extra_70b(args, dev):
    """Config 4 on one GPU: x [4, 4096, 8192], 448 blocks, top-p 0.8, K in [16, 112] (weights and x drawn
    on the device)."""
    wl = configs.CONFIGS["70b"]
    w = configs.make_weights(wl, device=dev)
    m = make_module(wl, w, dev)
    del w
    x = configs.make_x(wl, device=dev).reshape(-1, wl.hidden_dim).to(torch.bfloat16)
    for _ in range(3):
        m(x)
    a = mean_active(m, x)
    t = _median(_time_calls(lambda: m(x), 10, warm=2))
    st = stage_split(lambda: m(x), K=3)
    flops = 6.0 * wl.hidden_dim * 64 * a * x.shape[0]
    peak, _, _ = tensor_peak(None)
    out = {"tokens": x.shape[0], "ms": round(t, 4), "tokens_per_s": x.shape[0] / (t / 1e3),
           "active_blocks_per_token": a, "stages_ms": {k: round(v_, 4) for k, v_ in st.items()},
           "tensor_peak_frac_burst": round(flops / (t / 1e3) / 1e12 / peak, 4)}
    del m
    fsi._lib.release_workspaces()
    torch.cuda.empty_cache()
    return out


def _median(ts):
    return ts[len(ts) // 2]


# ------------------------------------------------------------------ N > 1
def run_ours_sharded(args, rank, world, local, dev):
    """N > 1: the 8B configuration's one global batch of 16384 tokens, parameter blocks sharded over the
    ranks (b % N) and the partials reduce-scattered over token rows with NCCL (bf16 partials, token
    chunks whose collective overlaps the next chunk's compute); strong scaling.  Extra keys: the token
    split (every rank its own batch, no collective), the same block-sharded forward end to end from each
    rank's slice of the batch in host memory, and the 70B configuration block-sharded with its 1-GPU
    time measured by the same processes."""
    import torch.distributed as dist
    wl = configs.CONFIGS[args.config]
    pd = torch.bfloat16 if args.partial_dtype == "bf16" else torch.float32
    w = configs.make_weights(wl)
    m = make_module(wl, w, dev)
    x_cpu = configs.make_x(wl).reshape(-1, wl.hidden_dim)
    x = x_cpu.to(dev, torch.bfloat16)  # replicated on every rank
    M, D = x.shape
    K, ch = args.steps, args.shard_chunks
    with torch.no_grad():
        a_mean = mean_active(m, x)
        # token split: every rank its own batch (drawn on the device), replicated weights, no collective
        x_own = configs.make_x(wl, seed=1000 + rank, device=dev).reshape(-1, wl.hidden_dim).to(torch.bfloat16)
        for _ in range(args.warmup):
            m(x_own)
        t_split, _ = timed_steps(lambda: m(x_own), K, dev, world)
        del x_own
        # block sharding
        peer = args.reduce == "peer"
        fsi.sharding.shard_parameter_blocks(m, partial_dtype=pd, peer_reduce=peer)

        def step():
            fsi.sharding.sharded_token_forward(m, x, reduce="scatter", chunks=ch)

        for _ in range(args.warmup):
            step()
        t_ms, clk = timed_steps(step, K, dev, world, ClockSampler(gpu_smi_id(dev, local)))
        # where the time goes on this rank, for the whole batch in one piece: routing of this rank's
        # tokens, the all-gather of the routes, the shard's kernels from the given routes (block lists and
        # H clears, gate/up, down) and the reduce-scatter alone
        s_rows = M // world
        x_mine = x[rank * s_rows:(rank + 1) * s_rows]
        t_route, _ = timed_steps(lambda: fsi.sharding._cuda_route(m, x_mine), 10, dev, world)
        t_rag, _ = timed_steps(lambda: fsi.sharding._gather_routes(m, x_mine, None, world, rank,
                                                                  fsi.sharding._cuda_route), 10, dev, world)
        ridx, cnt, ctx = fsi.sharding._gather_routes(m, x_mine, None, world, rank, fsi.sharding._cuda_route)
        stage = stage_split(lambda: fsi.sharding._cuda_routed_partial(m, x, world, rank, ridx, cnt, ctx))
        stage["route_own_tokens"] = t_route / 10
        stage["route_and_allgather"] = t_rag / 10
        part = torch.empty(M, D, dtype=pd, device=dev)
        ys = torch.empty(M // world, D, dtype=pd, device=dev)
        t_rs, _ = timed_steps(lambda: dist.reduce_scatter_tensor(ys, part), 10, dev, world)
        peer_state = getattr(m, "_peer_state", None)
        peer_used = peer_state is not None and peer_state.epoch > 0
        if peer_used:
            stage["peer"] = peer_stage_times(m, x, world, rank)
        err = fsi._lib.device_error(fsi._lib.workspace(dev, 0))
        if peer_state is not None:
            err = err or fsi._lib.device_error(peer_state.err) or fsi._lib.device_error(peer_state.err_wait)
        fsi.sharding.release_peer_buffers(m)
        m._peer_reduce = False  # the host-buffer path below reduces with NCCL
        e2e = measure_e2e_sharded(args, m, x_cpu, rank, world, dev)
        del m, x, part, ys
        fsi._lib.release_workspaces()
        torch.cuda.empty_cache()
        bs70 = None if args.no_extras else blockshard_70b(args, rank, world, dev, pd)
    ms_step = t_ms / K
    roof, total_flops, peak, peaks_all = roofline_block(stage, a_mean, M, D, clk)
    roof["note"] = ("per rank: the shard's kernels over all tokens; useful FLOPs = this rank's 1/N share of the "
                    "active-block FLOPs")
    for key in ("achieved", "frac"):
        roof[key] /= world
    roof["frac_both"] = {k: v_ / world for k, v_ in roof["frac_both"].items()}
    roof["algorithmic_flops_per_launch"] /= world
    line = {
        "metric": METRIC, "value": M * K / (t_ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": K,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) x, N(0,0.02) weights)",
        "config": config_block(wl, world, f"parameter blocks sharded b % {world}, routing split over the "
                                          f"ranks (routes all-gathered) + "
                                          + ("peer-memory reduce-scatter (down projection stores each row's "
                                             "partial on its owner over NVLink, then a combine kernel)"
                                             if peer_used else "NCCL reduce-scatter")
                                          + f" of {args.partial_dtype} partials, "
                                          + (f"{ch} token chunks overlapped" if ch > 1 else "one piece"),
                               global_tokens=M),
        "reduce": "peer" if peer_used else "nccl",
        "tensor_peak_frac": total_flops / (ms_step / 1e3) / 1e12 / (peak * world),
        "active_blocks_per_token": a_mean,
        "stages_ms_rank0_unchunked": stage,
        "stages_note": "route = block lists and H clears from the given routes; route_own_tokens = routing of "
                       "this rank's 1/N of the tokens; route_and_allgather = the same plus the all-gather of "
                       "the routes",
        "reduce_scatter_ms": t_rs / 10, "collective_bytes_per_rank": M * D * (2 if pd == torch.bfloat16 else 4),
        "roofline": roof,
        "e2e": e2e,
        "token_split": {"value": world * M * K / (t_split / 1e3), "unit": "tokens/s", "scaling": "weak",
                        "ms_per_step": t_split / K, "tokens_per_rank": M,
                        "parallelism": f"token split x{world} (no collective)"},
        "gpu_launches": (KERNELS_PEER_STEP if peer_used else KERNELS_PER_SHARDED_CHUNK * ch) * K,
        "clocks": clk,
        "device_error": err,
    }
    if bs70 is not None:
        line["blockshard_70b"] = bs70
    return line


def peer_stage_times(m, x, world, rank, K=10):
    """Where the peer-memory step's time goes on this rank (CUDA events, mean of K calls): routing of this
    rank's rows and their exchange through the peer route tables (put, flag, wait for every rank); the
    contraction whose epilogue stores each row on its owner (+ the flag kernel); the combine (including its
    wait for the other ranks' flags)."""
    sh = fsi.sharding
    M, D = x.shape
    s = M // world
    xv = x.view(world, s, D)
    pd = sh._partial_dtype(m)
    kg, ku, v, packed, _, _, wout = m._weights()
    cap = max(int(m.max_remote_blocks), 1)
    pr = sh._peer_state(m, s, D, pd, cap, x.device)
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(K)]
    for k in range(K):
        ev[k][0].record()
        ridx, cnt, ctx = sh._cuda_route(m, xv[rank])
        e = pr.epoch + 1
        par = e & 1
        fsi.kernels.peer_put(ridx.to(torch.int32), [pr.route_ids(par, a) + rank * s * cap * 4 for a in pr.addr])
        fsi.kernels.peer_put(cnt.to(torch.int32), [pr.route_counts(par, a) + rank * s * 4 for a in pr.addr])
        fsi.kernels.peer_signal(pr.route_flags(), e, x.device)
        pr.ctx_full[rank * s:(rank + 1) * s].copy_(ctx)
        fsi.kernels.peer_wait(pr.base + sh.PeerReduce.ROUTE_FLAGS, world, e, pr.err_wait)
        ev[k][1].record()
        fsi.kernels.routed_peer_forward(x, kg, ku, v, packed, wout, pr.route_ids(par), pr.route_counts(par),
                                        pr.ctx_full, base_blocks=m.base_blocks, block_stride=world,
                                        block_offset=rank, peer_out=pr.slots(par), peer_flags=pr.flags(),
                                        rows_per_rank=s, epoch=e, out_f32=pd == torch.float32, capacity=cap)
        pr.epoch = e
        ev[k][2].record()
        fsi.kernels.peer_combine(pr.recv(par), pr.base, world, s, D, in_f32=pd == torch.float32, epoch=e,
                                 out_dtype=pd, err_ws=pr.err)
        ev[k][3].record()
    torch.cuda.synchronize()
    mean = lambda i: statistics.mean(ev[k][i].elapsed_time(ev[k][i + 1]) for k in range(K))  # noqa: E731
    return {"route_and_exchange": mean(0), "contraction_with_peer_stores": mean(1), "combine_incl_wait": mean(2)}


def measure_e2e_sharded(args, m, x_cpu, rank, world, dev):
    """Block-sharded forward end to end: every rank starts from its own slice of the batch in pinned host
    memory and ends with its output rows in pinned host memory (sharding.sharded_forward_host: copy-in,
    NVLink all-gather, shard compute, reduce-scatter, copy-out, chunk by chunk)."""
    M, D = x_cpu.shape
    s = M // world
    x_host = x_cpu[rank * s:(rank + 1) * s].to(torch.bfloat16).pin_memory()
    y_host = torch.empty(s, D, dtype=torch.bfloat16).pin_memory()
    E = args.e2e_steps or max(10, args.steps // 10)
    step = lambda: fsi.sharding.sharded_forward_host(m, x_host, out=y_host, chunks=args.e2e_chunks)  # noqa: E731
    for _ in range(3):
        step()
    t, _ = timed_steps(step, E, dev, world)
    return {"value": M * E / (t / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": M * D * 2,
            "d2h_bytes_per_step": M * D * 2, "steps": E, "bytes_note": "summed over ranks (each copies its slice)",
            "path": "sharding.sharded_forward_host: each rank's slice from pinned host memory, NVLink all-gather, "
                    "shard compute, reduce-scatter, pinned host output slice",
            "chunks": args.e2e_chunks}


def blockshard_70b(args, rank, world, dev, pd):
    """70B configuration (x [4, 4096, 8192], 448 blocks): 1-GPU time (every rank runs the unsharded forward
    on its own GPU at the same time; max over ranks) and the block-sharded time; efficiency =
    t_1 / (N * t_N)."""
    wl = configs.CONFIGS["70b"]
    w = configs.make_weights(wl, device=dev)
    m = make_module(wl, w, dev)
    del w
    x = configs.make_x(wl, device=dev).reshape(-1, wl.hidden_dim).to(torch.bfloat16)
    K = max(5, min(args.steps, 20))
    for _ in range(3):
        m(x)
    t1, _ = timed_steps(lambda: m(x), K, dev, world)
    fsi.sharding.shard_parameter_blocks(m, partial_dtype=pd, peer_reduce=args.reduce == "peer")
    step = lambda: fsi.sharding.sharded_token_forward(m, x, reduce="scatter", chunks=args.shard_chunks)  # noqa: E731
    for _ in range(3):
        step()
    tn, _ = timed_steps(step, K, dev, world)
    M = x.shape[0]
    out = {"tokens": M, "value": M * K / (tn / 1e3), "unit": "tokens/s", "ms_per_step": tn / K,
           "one_gpu_ms_per_step": t1 / K, "efficiency": (t1 / K) / (world * tn / K),
           "speedup": t1 / tn, "reduce": "peer" if getattr(m, "_peer_state", None) is not None else "nccl"}
    fsi.sharding.release_peer_buffers(m)
    del m, x
    fsi._lib.release_workspaces()
    torch.cuda.empty_cache()
    return out


# ------------------------------------------------------------------ extra measurement modes
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


def run_extra_mode(args):
    """--mode decode / sweep / pooled / 70b: one of the N = 1 line's extra keys on its own."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    with torch.no_grad():
        if args.mode == "70b":
            out = extra_70b(args, dev)
        else:
            wl = configs.CONFIGS["8b"]
            m = make_module(wl, configs.make_weights(wl), dev)
            x = configs.make_x(wl).reshape(-1, wl.hidden_dim).to(dev, torch.bfloat16)
            out = {"decode": extra_decode, "sweep": extra_sweep,
                   "pooled": lambda m_, x_, d_: extra_pooled(wl, m_, x_, d_)}[args.mode](m, x, dev)
    print(json.dumps({"mode": args.mode, **out}), flush=True)


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


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.mode in ("decode", "sweep", "pooled", "70b"):
        run_extra_mode(args)
    elif args.mode == "variants":
        run_variants(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
