#!/usr/bin/env python
"""Benchmark of the fused multi-adapter LoRA op on B200 (one process per GPU).

Headline workload (default, cfg2): one bf16 projection 4096 -> 4096, 16 adapters of rank 16,
4096 tokens per GPU whose per-adapter row counts follow Zipf(1.1), packed into 128-row bins by
the scheduler.  With N GPUs the global batch holds N x 4096 tokens; every rank computes the same
packing and takes its rows (weak scaling: fixed work per GPU, no communication in the forward).

Printed by rank 0, one JSON line:
  value        whole-job tokens/s of the forward with inputs resident in HBM, CUDA events around
               each step (routed shrink + fused base GEMM/LoRA expand), L2 flushed (256 MiB write)
               before every step, max over ranks
  e2e          the same through the public host-batch call (b200_ops.fused_lora_forward_host):
               pinned host x in, pinned host y out, timed by the host wall clock from before the
               call to after the stream synchronize, max over ranks
  roofline     the fused GEMM kernel: algorithmic FLOPs / its event-timed duration against the
               measured bf16 peak
  backward     the backward's stages as launches of their own (routed shrinks, grad_x GEMM, dA/dB
               grams), event-timed, and the grams' HBM roofline
  fwd_bwd      forward + backward through the plugin calls (+ the all-reduce of spanning adapters'
               gradients at N > 1)
  workloads    cfg3 (Llama-3-8B projections, 64 mixed-rank adapters) and cfg5 (70B projections,
               256 adapters of rank 64): forward + backward over every projection per step, the
               workload's tokens split over the N GPUs (strong scaling), all-reduce included
  cpu_baseline the CPU oracle (numpy float32 restatement of the reference op) on the host cores,
               rank 0 at N = 1, a bounded sample of the same workload

``--impl reference`` times that CPU restatement of the reference's op instead, on the same global
token count; it imports nothing of this package (the workload shapes are read from the plain file
lorafusion_b200/workloads.py, the layout comes from oracle/scheduler_oracle.py).
"""

from __future__ import annotations

import argparse
import datetime
import importlib.util
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "fused LoRA tokens/sec/GPU fwd & fwd+bwd; % bf16 roofline; 1/2/4/8 GPU"
WORKLOAD = "cfg2_h4096_a16_r16"
EXTRA = "cfg3_llama8b_a64_mixed,cfg5_70b_a256_r64"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 << 20
# bounded CPU samples of the multi-projection workloads: leading rows of the packed global batch
CPU_SAMPLE_ROWS = {"cfg3_llama8b_a64_mixed": 512, "cfg5_70b_a256_r64": 128}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=WORKLOAD)
    ap.add_argument("--extra", default=EXTRA, help="comma-separated fwd+bwd workloads timed after the headline "
                                                   "(all projections, strong scaling); 'none' to skip")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-fwd-bwd", action="store_true")
    ap.add_argument("--separate-launches", action="store_true",
                    help="no cooperative launches (profilers refuse them): shrinks as launches of their own")
    return ap.parse_args()


def load_workloads_module():
    """lorafusion_b200/workloads.py loaded as a plain file (numpy only), not through the package."""
    spec = importlib.util.spec_from_file_location("lf_workload_shapes", os.path.join(REPO, "lorafusion_b200",
                                                                                       "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"])),
                "source": "measured"}
    except (OSError, KeyError, ValueError):
        return dict(FALLBACK_PEAKS, source="fallback")


def load_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from the committed ncu summary, if one covers this kernel/workload."""
    path = os.path.join(REPO, "profiles", "ncu_traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 3 and not line.startswith("#") and parts[0] == kernel and parts[1] == workload:
                return float(parts[2])
    except OSError:
        pass
    return None


def repo_libraries_mapped() -> list[str]:
    """Shared libraries of this repository mapped into the process (evidence of which code ran)."""
    out = set()
    try:
        for line in open("/proc/self/maps"):
            path = line.split()[-1] if len(line.split()) >= 6 else ""
            if path.startswith(REPO) and ".so" in os.path.basename(path):
                out.add(os.path.relpath(path, REPO))
    except OSError:
        pass
    return sorted(out)


class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.dev)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def algorithmic_counts(routes, ranks, K, N, T):
    """Per-launch algorithmic work: routes are (start, end, adapter) triples."""
    R = sum((e - s) * ranks[a] for s, e, a in routes)
    active = sorted({a for s, e, a in routes if e > s})
    rsum = sum(ranks[a] for a in active)
    gemm_flops = 2.0 * T * K * N + 2.0 * R * N
    shrink_flops = 2.0 * R * K
    shrink_bytes = T * K * 2 + rsum * K * 2 + R * 2
    gram_bytes = T * K * 2 + T * N * 2 + 2 * R * 2 + rsum * (K + N) * 4
    return dict(R=R, gemm_flops=gemm_flops, shrink_flops=shrink_flops, shrink_bytes=shrink_bytes,
                gram_bytes=gram_bytes, fwd_flops=gemm_flops + shrink_flops,
                fwdbwd_flops=4.0 * T * K * N + 6.0 * R * (K + N))


# =============================================================================== CPU (oracle) side
def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        if n and n[0]:
            return int(n[0])
    except Exception:  # noqa: BLE001
        pass
    return os.cpu_count() or 1


def use_all_host_cores():
    """BLAS threads = the host's cores (torchrun sets OMP_NUM_THREADS=1 in every rank)."""
    try:
        from threadpoolctl import threadpool_limits
        return threadpool_limits(limits=os.cpu_count() or 1, user_api="blas")
    except Exception:  # noqa: BLE001
        return None


def oracle_layout(wlm, wl, total_rows):
    """The packed global batch's routes from the oracle's scheduler restatement."""
    from oracle.scheduler_oracle import bucket_rows, greedy_bins
    counts = wlm.row_counts(wl, total_rows)
    bins = greedy_bins(bucket_rows([(i, i, c) for i, c in enumerate(counts)]), wl.tile_capacity)
    routes, cur = [], 0
    for entries in bins:
        for a, n in entries:
            routes.append((cur, cur + n, a))
            cur += n
    return routes, cur


def leading_routes(routes, n):
    return [(s, min(e, n), a) for s, e, a in routes if s < n]


class OracleProblem:
    """bf16-rounded float32 inputs of one projection for the numpy oracle (adapters in `routes` only).
    ``tiled_w``: the base weight repeats one random 256-row block (its values do not change the
    oracle's arithmetic work; generating a 28672 x 8192 matrix would dominate a short sample)."""

    def __init__(self, rng, T, K, N, ranks, routes, with_grad, tiled_w=False):
        from oracle import mock_oracle
        r16 = mock_oracle.bf16_round
        self.x = r16(rng.standard_normal((T, K), dtype=np.float32))
        if tiled_w and N > 256:
            blk = r16(rng.standard_normal((256, K), dtype=np.float32) / np.float32(math.sqrt(K)))
            self.w = np.ascontiguousarray(np.tile(blk, (-(-N // 256), 1))[:N])
        else:
            self.w = r16(rng.standard_normal((N, K), dtype=np.float32) / np.float32(math.sqrt(K)))
        ids = sorted({a for _, _, a in routes})
        self.a = {i: r16(rng.standard_normal((ranks[i], K), dtype=np.float32) / np.float32(math.sqrt(K))) for i in ids}
        self.b = {i: r16(np.float32(0.02) * rng.standard_normal((N, ranks[i]), dtype=np.float32)) for i in ids}
        self.g = r16(rng.standard_normal((T, N), dtype=np.float32)) if with_grad else None
        self.sc = {i: 2.0 for i in ids}
        self.routes = routes

    def forward(self):
        from oracle import mock_oracle
        return mock_oracle.fused_lora_forward(self.x, self.w, self.a, self.b, self.sc, self.routes)

    def backward(self):
        from oracle import mock_oracle
        return mock_oracle.fused_lora_backward(self.g, self.x, self.w, self.a, self.b, self.sc, self.routes)


def cpu_headline_sample(wlm, wl, n_gpus, steps=None, budget_s=None, with_grad=False):
    """Times of full forwards of the global batch (N x tokens per GPU) by the numpy oracle."""
    routes, T = oracle_layout(wlm, wl, wl.total_rows * n_gpus)
    _, K, N = wl.projections[0]
    pb = OracleProblem(np.random.default_rng(0), T, K, N, wlm.adapter_ranks(wl), routes, with_grad)
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        pb.forward()
        times.append(time.perf_counter() - t0)
        if steps is not None and len(times) >= steps:
            break
        if steps is None and time.perf_counter() - t_start > budget_s:
            break
    return T, times, pb


def cpu_workload_sample(wlm, wl, steps):
    """Forward + backward over every projection of the leading CPU_SAMPLE_ROWS rows of the packed batch."""
    routes, _ = oracle_layout(wlm, wl, wl.total_rows)
    n = CPU_SAMPLE_ROWS.get(wl.name, 256)
    sroutes = leading_routes(routes, n)
    ranks = wlm.adapter_ranks(wl)
    rng = np.random.default_rng(1)
    probs = [OracleProblem(rng, n, K, N, ranks, sroutes, True, tiled_w=True) for _, K, N in wl.projections]
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        for pb in probs:
            pb.forward()
            pb.backward()
        times.append(time.perf_counter() - t0)
    return n, times


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0  # rank 0 alone times the CPU arm; the other ranks exit without work
    limiter = use_all_host_cores()  # noqa: F841 - keeps the BLAS thread limit in force
    wlm = load_workloads_module()
    wl = wlm.WORKLOADS[args.workload]
    n_gpus = args.gpus
    _, _, _ = cpu_headline_sample(wlm, wl, n_gpus, steps=max(1, args.warmup))
    T, times, pb = cpu_headline_sample(wlm, wl, n_gpus, steps=args.steps, with_grad=not args.no_fwd_bwd)
    ms = 1e3 * statistics.mean(times)
    value = T / (ms / 1e3)
    cores = cpu_threads()
    _, K, N = wl.projections[0]
    fwd_bwd = None
    if not args.no_fwd_bwd:
        fb = []
        for _ in range(2):  # bounded: two full forward + backward steps of the global batch
            t0 = time.perf_counter()
            pb.forward()
            pb.backward()
            fb.append(time.perf_counter() - t0)
        fwd_bwd = {"value": T / statistics.mean(fb), "unit": "tokens/s", "ms_per_step": 1e3 * statistics.mean(fb),
                   "sample": f"2 full forward+backward steps of {T} tokens"}
    workloads = {}
    for name in [e for e in args.extra.split(",") if e and e != "none"]:
        wx = wlm.WORKLOADS[name]
        n, wt = cpu_workload_sample(wlm, wx, steps=2)
        workloads[name] = {"value": n / statistics.mean(wt), "unit": "tokens/s", "ms_per_step":
                           1e3 * statistics.mean(wt), "pass": "forward+backward, every projection",
                           "sample": f"leading {n} rows of the packed {wx.total_rows}-token batch, 2 steps "
                                     "(base weights: one random 256-row block repeated)"}
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": n_gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "tokens_per_gpu": wl.total_rows, "global_tokens": T,
                   "in_features": K, "out_features": N, "adapters": wl.n_adapters, "rank": wl.rank_choices[0],
                   "tile_rows": wl.tile_capacity,
                   "what": "numpy float32 restatement of lorafusion mock_ops.fused_lora_forward on bf16-rounded "
                           "inputs, host cores, one full forward of the global batch per step"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} full forwards of {T} tokens"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "fwd_bwd": fwd_bwd,
        "workloads": workloads,
        "repo_libraries_mapped": repo_libraries_mapped(),
        "lorafusion_b200_imported": any(m == "lorafusion_b200" or m.startswith("lorafusion_b200.")
                                        for m in sys.modules),
    }
    print(json.dumps(line), flush=True)
    return 0


# =============================================================================== GPU side
def global_packing(wl, total_rows):
    from lorafusion_b200.scheduler import Request, bucket_by_adapter, greedy_pack
    from lorafusion_b200.workloads import row_counts
    counts = row_counts(wl, total_rows)
    requests = [Request(i, i, c) for i, c in enumerate(counts)]
    groups = bucket_by_adapter(requests)
    return greedy_pack({g.adapter_id: g.total_rows for g in groups}, wl.tile_capacity)


def rank_projection(wl, projection, rows, routing, ranks, device, seed):
    """On-device bf16 tensors of one projection for a rank's rows (x, grad, W, adapters)."""
    import torch
    from lorafusion_b200.config import AdapterSpec
    _, K, N = wl.projections[projection]
    g = torch.Generator(device=device).manual_seed(seed)
    gw = torch.Generator(device=device).manual_seed(1000 + projection)
    T = len(rows)
    bf = torch.bfloat16
    x = torch.randn(T, K, device=device, generator=g, dtype=bf)
    grad = torch.randn(T, N, device=device, generator=g, dtype=bf)
    w = (torch.randn(N, K, device=device, generator=gw) / math.sqrt(K)).to(bf)
    lora_a = {i: (torch.randn(r, K, device=device, generator=gw) / math.sqrt(K)).to(bf) for i, r in enumerate(ranks)}
    lora_b = {i: (0.02 * torch.randn(N, r, device=device, generator=gw)).to(bf) for i, r in enumerate(ranks)}
    adapters = {i: AdapterSpec(i, r, float(2 * r), K, N) for i, r in enumerate(ranks)}
    return dict(x=x, grad=grad, w=w, lora_a=lora_a, lora_b=lora_b, adapters=adapters, routing=routing, T=T, K=K, N=N)


def run_ours(args):
    import torch
    import torch.distributed as dist

    from lorafusion_b200 import _native as nat
    from lorafusion_b200 import b200_ops
    from lorafusion_b200.sharding import PeerExchange, assign_bins, local_layout
    from lorafusion_b200.workloads import WORKLOADS, adapter_ranks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def rank_max(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if args.separate_launches:
        b200_ops.use_cooperative_launch(False)
    wl = WORKLOADS[args.workload]
    ranks = adapter_ranks(wl)
    packing = global_packing(wl, wl.total_rows * world)
    plan = assign_bins(packing.bins, world)
    rows, routing = local_layout(plan, packing.bins, rank, wl.tile_capacity)
    pr = rank_projection(wl, 0, rows, routing, ranks, device, seed=1000 + rank)
    T, K, N = pr["T"], pr["K"], pr["N"]
    global_T = sum(e - s for s, e in plan.bin_rows)
    routes = [(r.row_start, r.row_end, r.adapter_id) for r in routing.routes]
    counts = algorithmic_counts(routes, ranks, K, N, T)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
    prep = b200_ops.prepare_forward(pr["x"], pr["w"], pr["lora_a"], pr["lora_b"], pr["adapters"], pr["routing"])
    y = prep.new_output()
    SH, EX, BA = nat.LF_STAGE_SHRINK, nat.LF_STAGE_EXPAND, nat.LF_STAGE_BASE

    def timed(fn, steps, warmup, n_events):
        """Per-step event times (ms) of `fn(events)`; L2 flushed and the GPU kept busy before each step."""
        for _ in range(warmup):
            flush.zero_()
            fn(None)
        barrier()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(n_events)] for _ in range(steps)]
        for i in range(steps):
            flush.zero_()
            torch.cuda._sleep(100_000)  # keep the GPU busy while the host enqueues the step
            fn(ev[i])
        barrier()
        return [[ev[i][j].elapsed_time(ev[i][j + 1]) for j in range(n_events - 1)] for i in range(steps)]

    def bracket(fn):
        def step(ev):
            if ev:
                ev[0].record()
            fn()
            if ev:
                ev[1].record()
        return step

    default_stages = SH | EX | (nat.LF_STAGE_SEPARATE if args.separate_launches else 0)

    def fwd_staged(ev):
        if ev:
            ev[0].record()
        prep.launch(y, SH)
        if ev:
            ev[1].record()
        prep.launch(y, EX)
        if ev:
            ev[2].record()

    sampler = ClockSampler(local_rank)
    sampler.start()
    t = timed(bracket(lambda: prep.launch(y, default_stages)), args.steps, args.warmup, 2)
    clocks = sampler.stop()
    n_launch = prep.launch_count()  # reflects the path actually taken (co-scheduling switch included)
    step_local_ms = statistics.mean(s[0] for s in t)
    step_ms = rank_max(step_local_ms)
    value = global_T / (step_ms / 1e3)
    gpu_launches = n_launch * args.steps
    short = max(5, args.steps // 2)
    tsplit = timed(fwd_staged, short, 2, 3)  # the shrink and the fused GEMM as separate launches
    shrink_ms = statistics.mean(s[0] for s in tsplit)
    gemm_ms = statistics.mean(s[1] for s in tsplit)
    # yardsticks: our GEMM with LoRA disabled, and cuBLAS x @ W^T
    own_base_ms = statistics.mean(s[0] for s in timed(bracket(lambda: prep.launch(y, BA)), short, 2, 2))
    xw, wt = pr["x"], pr["w"].t()
    cublas_ms = statistics.mean(s[0] for s in timed(bracket(lambda: torch.matmul(xw, wt)), short, 2, 2))

    # e2e through the public host-batch call, host wall clock around call + synchronize
    x_host = pr["x"].cpu().pin_memory()
    y_host = torch.empty((T, N), dtype=torch.bfloat16).pin_memory()
    cur = torch.cuda.current_stream()

    def e2e_call():
        b200_ops.fused_lora_forward_host(x_host, pr["w"], pr["lora_a"], pr["lora_b"], pr["adapters"], pr["routing"],
                                         out=y_host)

    for _ in range(2):
        e2e_call()
    barrier()
    wall = []
    for _ in range(short):
        flush.zero_()
        cur.synchronize()
        t0 = time.perf_counter()
        e2e_call()
        cur.synchronize()
        wall.append(time.perf_counter() - t0)
    e2e_ms = rank_max(1e3 * statistics.mean(wall))

    # requests in, per-request results out (one device): C++ packing, lf_copy_rows gather,
    # fused forward, lf_copy_rows scatter
    coordinator = None
    if world == 1:
        from lorafusion_b200.coordinator import Coordinator
        from lorafusion_b200.scheduler import Request
        from lorafusion_b200.workloads import row_counts
        reqs = [Request(i, i, c) for i, c in enumerate(row_counts(wl, wl.total_rows))]
        gq = torch.Generator(device=device).manual_seed(7)
        req_x = {r.request_id: torch.randn(r.num_rows, K, device=device, generator=gq).to(torch.bfloat16)
                 for r in reqs}
        coord = Coordinator(pr["w"], pr["adapters"], pr["lora_a"], pr["lora_b"], tile_capacity=wl.tile_capacity)
        co_ms = statistics.mean(s[0] for s in timed(bracket(lambda: coord.run_batch(reqs, req_x)), short, 2, 2))
        coordinator = {"value": sum(r.num_rows for r in reqs) / (co_ms / 1e3), "unit": "tokens/s", "ms_per_step": co_ms,
                       "requests": len(reqs),
                       "path": "Coordinator.run_batch: greedy_pack (C++), lf_copy_rows gather, fused forward, "
                               "lf_copy_rows scatter; request tensors resident on the device"}

    peaks = load_peaks()
    backward = None
    fwd_bwd = None
    grad_dtype = torch.float32 if world > 1 else None
    rank_of = dict(enumerate(ranks))
    if not args.no_fwd_bwd:
        # the backward's stages as launches of their own: routed shrinks, grad_x GEMM, dA/dB grams
        bprep = b200_ops.prepare_backward(pr["grad"], pr["x"], pr["w"], pr["lora_a"], pr["lora_b"], pr["adapters"],
                                          pr["routing"])
        BS, BX, BG = nat.LF_BSTAGE_SHRINK, nat.LF_BSTAGE_GRAD_X, nat.LF_BSTAGE_GRAD_AB

        def bwd_staged(ev):
            for j, st in enumerate((BS, BX, BG)):
                if ev:
                    ev[j].record()
                bprep.launch(st)
            if ev:
                ev[3].record()

        tbs = timed(bwd_staged, short, 2, 4)
        b_shrink, b_gx, b_gram = (statistics.mean(s[j] for s in tbs) for j in range(3))
        gram_gbs = counts["gram_bytes"] / (b_gram / 1e3) / 1e9
        backward = {"stages_ms": {"routed_shrinks": b_shrink, "grad_x_gemm": b_gx, "grams_dA_dB": b_gram},
                    "gram_roofline": {"kernel": "tc_gram_kernel (dA and dB, one launch)", "bound": "hbm",
                                      "achieved": gram_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                                      "frac": gram_gbs / peaks["hbm_gbs"], "bytes_per_launch": counts["gram_bytes"],
                                      "ms_per_launch": b_gram}}

        # at N > 1 the spanning adapters' dA/dB are summed inside the dA/dB kernel over NVLink
        peer = PeerExchange(plan, rank_of, device) if world > 1 and plan.spanning else None

        def fb():
            b200_ops.fused_lora_forward(pr["x"], pr["w"], pr["lora_a"], pr["lora_b"], pr["adapters"], pr["routing"])
            b200_ops.fused_lora_backward(pr["grad"], pr["x"], pr["w"], pr["lora_a"], pr["lora_b"], pr["adapters"],
                                         pr["routing"], grad_dtype=grad_dtype, peer=peer)

        fb_ms = rank_max(statistics.mean(s[0] for s in timed(bracket(fb), short, 2, 2)))
        bwd_launches = b200_ops.last_launch_count()
        bwd_ms = rank_max(statistics.mean(s[0] for s in timed(bracket(
            lambda: b200_ops.fused_lora_backward(pr["grad"], pr["x"], pr["w"], pr["lora_a"], pr["lora_b"],
                                                 pr["adapters"], pr["routing"], grad_dtype=grad_dtype, peer=peer)),
            short, 2, 2)))
        if peer is not None:
            peer.close()
        fwd_bwd = {"value": global_T / (fb_ms / 1e3), "unit": "tokens/s", "ms_per_step": fb_ms,
                   "launches_per_step": n_launch + bwd_launches, "backward_ms": bwd_ms,
                   "tflops": counts["fwdbwd_flops"] * world / (fb_ms / 1e3) / 1e12,
                   "tflops_note": "whole job (all GPUs)",
                   "spanning_adapters": len(plan.spanning),
                   "cross_gpu_sum": "inside the dA/dB kernel (blocks pushed to every rank over NVLink peer "
                                    "mappings, summed in rank order)" if world > 1 else None}
    del prep, y, pr

    # multi-projection workloads, forward + backward, strong scaling over the N GPUs
    workloads = {}
    for name in [e for e in args.extra.split(",") if e and e != "none"]:
        workloads[name] = run_workload(name, WORKLOADS[name], world, rank, device, args, flush, barrier, rank_max,
                                       peaks)

    err = nat.device_error()
    if n_launch == 1:  # one kernel does the whole forward: shrink on spare CTA pairs, GEMM + expand
        dom_kernel = "tc_gemm_pair_kernel (co-scheduled routed shrink + base GEMM + LoRA expand)"
        dom_flops, dom_ms = counts["fwd_flops"], step_local_ms
    else:
        dom_kernel = "tc_gemm_pair_kernel (base GEMM + LoRA expand)"
        dom_flops, dom_ms = counts["gemm_flops"], gemm_ms
    gemm_tflops = dom_flops / (dom_ms / 1e3) / 1e12
    shrink_gbs = counts["shrink_bytes"] / (shrink_ms / 1e3) / 1e9
    pair_traffic = load_traffic("tc_gemm_pair_kernel", args.workload)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        limiter = use_all_host_cores()  # noqa: F841
        wlm = load_workloads_module()
        Tc, times, _ = cpu_headline_sample(wlm, wlm.WORKLOADS[args.workload], 1, budget_s=args.cpu_seconds)
        cpu = {"value": Tc / statistics.mean(times), "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
               "sample": f"{len(times)} full {Tc}-token forwards of the numpy float32 oracle "
                         f"({sum(times):.1f} s of CPU work)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": args.workload, "tokens_per_gpu": wl.total_rows, "global_tokens": global_T,
                       "in_features": K, "out_features": N, "adapters": wl.n_adapters, "rank": ranks[0],
                       "tile_rows": wl.tile_capacity, "routes_rank0": len(routes),
                       "parallelism": f"dp{world} over packed bins (no forward communication)",
                       "l2": "flushed (256 MiB write) before every timed step",
                       "pass": "forward (routed shrink + fused base GEMM/LoRA expand)"},
            "roofline": {"kernel": dom_kernel, "bound": "tensor",
                         "achieved": gemm_tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": gemm_tflops / peaks["bf16_tflops"], "traffic": pair_traffic,
                         "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of the fused GEMM "
                                           "launch of the two-launch forward (profiles/ncu_traffic.txt); ncu "
                                           "cannot capture the cooperative one-launch forward",
                         "peak_source": f"{peaks['source']} bf16 dense (burst)",
                         "flops_per_launch": dom_flops, "ms_per_launch": dom_ms, "launches_per_step": n_launch},
            "split_launches": {"shrink_ms": shrink_ms, "gemm_ms": gemm_ms, "total_ms": shrink_ms + gemm_ms},
            "shrink_roofline": {"kernel": "tc_shrink_kernel (standalone launch)", "bound": "hbm", "achieved": shrink_gbs,
                                "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": shrink_gbs / peaks["hbm_gbs"],
                                "bytes_per_launch": counts["shrink_bytes"], "ms_per_launch": shrink_ms},
            "vs_base_gemm": {"fused_fwd_ms": step_ms, "own_base_gemm_ms": own_base_ms, "cublas_base_gemm_ms": cublas_ms,
                             "fused_over_own_base": step_ms / own_base_ms, "fused_over_cublas": step_ms / cublas_ms,
                             "cublas_tflops": 2.0 * T * K * N / (cublas_ms / 1e3) / 1e12},
            "e2e": {"value": global_T / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": T * K * 2, "d2h_bytes_per_step": T * N * 2,
                    "timing": "host wall clock from before the call to after the stream synchronize, max over ranks",
                    "path": "b200_ops.fused_lora_forward_host -> lf_forward_host: pinned host x/y, 1024-row "
                            "chunks between a 256-row first and last chunk, enqueued by one native call, copies in "
                            "both directions overlapped with the fused forward; at N > 1 every rank's copies share "
                            "the host's PCIe and memory"},
            "backward": backward,
            "fwd_bwd": fwd_bwd,
            "workloads": workloads,
            "coordinator": coordinator,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": gpu_launches,
            "device_status": err,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_workload(name, wl, world, rank, device, args, flush, barrier, rank_max, peaks):
    """Forward + backward over every projection of `wl`, its tokens split over the ranks; at N > 1
    float32 adapter gradients and the all-reduce of spanning adapters per projection."""
    import torch

    from lorafusion_b200 import b200_ops
    from lorafusion_b200.sharding import PeerExchange, assign_bins, local_layout
    from lorafusion_b200.workloads import adapter_ranks

    ranks = adapter_ranks(wl)
    rank_of = dict(enumerate(ranks))
    packing = global_packing(wl, wl.total_rows)
    plan = assign_bins(packing.bins, world)
    rows, routing = local_layout(plan, packing.bins, rank, wl.tile_capacity)
    routes = [(r.row_start, r.row_end, r.adapter_id) for r in routing.routes]
    projs = [rank_projection(wl, p, rows, routing, ranks, device, seed=7 * p + 31 * rank)
             for p in range(len(wl.projections))]
    flops = sum(algorithmic_counts(routes, ranks, p["K"], p["N"], p["T"])["fwdbwd_flops"] for p in projs)
    grad_dtype = torch.float32 if world > 1 else None
    peer = PeerExchange(plan, rank_of, device) if world > 1 and plan.spanning else None

    def step(ev):
        if ev:
            ev[0].record()
        for p in projs:
            b200_ops.fused_lora_forward(p["x"], p["w"], p["lora_a"], p["lora_b"], p["adapters"], p["routing"])
        if ev:
            ev[1].record()
        for p in projs:  # spanning adapters' dA/dB summed across the GPUs inside each dA/dB kernel
            b200_ops.fused_lora_backward(p["grad"], p["x"], p["w"], p["lora_a"], p["lora_b"], p["adapters"],
                                         p["routing"], grad_dtype=grad_dtype, peer=peer)
        if ev:
            ev[2].record()

    steps = max(3, args.steps // 3)
    for _ in range(2):
        flush.zero_()
        step(None)
    barrier()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(steps)]
    for i in range(steps):
        flush.zero_()
        torch.cuda._sleep(100_000)
        step(ev[i])
    barrier()
    per = [[ev[i][j].elapsed_time(ev[i][j + 1]) for j in range(2)] for i in range(steps)]
    fwd_ms, bwd_ms = (statistics.mean(s[j] for s in per) for j in range(2))
    if peer is not None:
        peer.close()
    # per projection, stages as launches of their own (this rank): forward shrink / fused GEMM,
    # backward shrinks / grad_x GEMM / grams
    from lorafusion_b200 import _native as nat
    stages = {}
    for (pname, _, _), p in zip(wl.projections, projs):
        fp = b200_ops.prepare_forward(p["x"], p["w"], p["lora_a"], p["lora_b"], p["adapters"], p["routing"])
        bp = b200_ops.prepare_backward(p["grad"], p["x"], p["w"], p["lora_a"], p["lora_b"], p["adapters"],
                                       p["routing"], grad_dtype=grad_dtype)
        yp = fp.new_output()
        launches = [lambda: fp.launch(yp, nat.LF_STAGE_SHRINK), lambda: fp.launch(yp, nat.LF_STAGE_EXPAND),
                    lambda: bp.launch(nat.LF_BSTAGE_SHRINK), lambda: bp.launch(nat.LF_BSTAGE_GRAD_X),
                    lambda: bp.launch(nat.LF_BSTAGE_GRAD_AB)]
        for f in launches:
            f()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(len(launches) + 1)]
        flush.zero_()
        evs[0].record()
        for j, f in enumerate(launches):
            f()
            evs[j + 1].record()
        torch.cuda.synchronize()
        t_ = [evs[j].elapsed_time(evs[j + 1]) for j in range(len(launches))]
        stages[pname] = {"fwd_shrink": t_[0], "fwd_gemm": t_[1], "bwd_shrinks": t_[2], "bwd_grad_x": t_[3],
                         "bwd_grams": t_[4]}
        del fp, bp, yp
    local = fwd_ms + bwd_ms
    ms = rank_max(local)
    total_flops = flops
    if world > 1:
        t = torch.tensor([flops], dtype=torch.float64, device=device)
        torch.distributed.all_reduce(t)
        total_flops = float(t.item())
    tflops = total_flops / (ms / 1e3) / 1e12
    out = {"value": wl.total_rows / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
           "scaling": "strong", "global_tokens": wl.total_rows, "projections": [p[0] for p in wl.projections],
           "adapters": wl.n_adapters, "pass": "forward + backward over every projection per step",
           "rank0_ms": {"forward": fwd_ms, "backward": bwd_ms},
           "cross_gpu_sum": "inside each dA/dB kernel over NVLink peer mappings" if world > 1 else None,
           "rank0_stage_ms": stages,
           "spanning_adapters": len(plan.spanning),
           "roofline": {"bound": "tensor", "achieved": tflops, "peak": world * peaks["bf16_tflops_sustained"],
                        "unit": "TFLOP/s", "frac": tflops / (world * peaks["bf16_tflops_sustained"]),
                        "peak_source": f"{peaks['source']} bf16 dense (sustained: seconds-long step), "
                                       f"x {world} GPU(s)"},
           "l2": "flushed (256 MiB write) before every timed step; inputs larger than L2"}
    del projs
    torch.cuda.empty_cache()
    return out


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
