#!/usr/bin/env python
"""Benchmark of the fused multi-adapter LoRA forward on B200 (one process per GPU).

Workload (default): one bf16 projection 4096 -> 4096, 16 adapters of rank 16,
4096 tokens per GPU whose per-adapter row counts follow Zipf(1.1), packed into
128-row bins by the scheduler.  With N GPUs the global batch holds N x 4096
tokens; every rank computes the same packing and takes whole bins (weak
scaling: fixed work per GPU, no communication in the forward).

Printed by rank 0, one JSON line:
  value        whole-job tokens/s of the forward with inputs resident in HBM, CUDA
               events around each step (routed shrink + fused base GEMM/LoRA expand),
               L2 flushed (256 MiB write) before every step, max over ranks
  e2e          the same through the public plugin call (b200_ops.fused_lora_forward)
               with pinned host buffers: host->device copy of x, the op, device->host
               copy of y inside the timed region
  roofline     the fused GEMM kernel: algorithmic FLOPs / its event-timed duration
               against the measured bf16 peak; the shrink's HBM figure alongside
  cpu_baseline the CPU oracle (numpy float32 restatement of the reference op) on the
               host cores, rank 0 at N=1, a bounded sample of the same workload

``--impl reference`` times that CPU restatement of the reference's op instead.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "fused LoRA tokens/sec/GPU fwd & fwd+bwd; % bf16 roofline; 1/2/4/8 GPU"
WORKLOAD = "cfg2_h4096_a16_r16"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
L2_FLUSH_BYTES = 256 << 20


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=WORKLOAD)
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="budget of the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-fwd-bwd", action="store_true")
    ap.add_argument("--separate-launches", action="store_true",
                    help="shrink and fused GEMM as two ordinary launches (profilers refuse the cooperative one)")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]), "source": "measured"}
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


# --------------------------------------------------------------------------- workload
def global_layout(wl, n_gpus: int):
    from lorafusion_b200.scheduler import Request, bucket_by_adapter, greedy_pack
    from lorafusion_b200.workloads import row_counts
    counts = row_counts(wl, wl.total_rows * n_gpus)
    requests = [Request(i, i, c) for i, c in enumerate(counts)]
    groups = bucket_by_adapter(requests)
    packing = greedy_pack({g.adapter_id: g.total_rows for g in groups}, wl.tile_capacity)
    return packing


def local_problem(wl, n_gpus: int, rank: int, device):
    import torch
    from lorafusion_b200.config import AdapterSpec
    from lorafusion_b200.sharding import assign_bins, local_layout
    from lorafusion_b200.workloads import adapter_ranks
    packing = global_layout(wl, n_gpus)
    plan = assign_bins(packing.bins, n_gpus)
    rows, routing = local_layout(plan, packing.bins, rank, wl.tile_capacity)
    _, K, N = wl.projections[0]
    ranks = adapter_ranks(wl)
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    gw = torch.Generator(device=device).manual_seed(0)
    T = len(rows)
    x = torch.randn(T, K, device=device, generator=g).to(torch.bfloat16)
    grad = torch.randn(T, N, device=device, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device=device, generator=gw) / math.sqrt(K)).to(torch.bfloat16)
    lora_a = {i: (torch.randn(r, K, device=device, generator=gw) / math.sqrt(K)).to(torch.bfloat16)
              for i, r in enumerate(ranks)}
    lora_b = {i: (0.02 * torch.randn(N, r, device=device, generator=gw)).to(torch.bfloat16)
              for i, r in enumerate(ranks)}
    adapters = {i: AdapterSpec(i, r, float(2 * r), K, N) for i, r in enumerate(ranks)}
    return dict(x=x, grad=grad, w=w, lora_a=lora_a, lora_b=lora_b, adapters=adapters, routing=routing,
                plan=plan, T=T, K=K, N=N, global_T=sum(e - s for s, e in plan.bin_rows), ranks=ranks)


def algorithmic_counts(routing, ranks, K, N, T):
    R = sum((r.row_end - r.row_start) * ranks[r.adapter_id] for r in routing.routes)
    active = sorted({r.adapter_id for r in routing.routes})
    gemm_flops = 2.0 * T * K * N + 2.0 * R * N
    shrink_flops = 2.0 * R * K
    shrink_bytes = T * K * 2 + sum(ranks[a] * K * 2 for a in active) + R * 2
    return dict(R=R, gemm_flops=gemm_flops, shrink_flops=shrink_flops, shrink_bytes=shrink_bytes,
                fwd_flops=gemm_flops + shrink_flops, fwdbwd_flops=4.0 * T * K * N + 6.0 * R * (K + N))


# --------------------------------------------------------------------------- CPU oracle timing
def cpu_oracle_sample(wl, budget_s: float, max_steps: int | None = None):
    """Time the numpy restatement of the reference forward on full workload batches."""
    import numpy as np
    from oracle import mock_oracle
    from lorafusion_b200.workloads import adapter_ranks
    packing = global_layout(wl, 1)
    routes, cur = [], 0
    for entries in packing.bins:
        for a, n in entries:
            routes.append((cur, cur + n, a))
            cur += n
    _, K, N = wl.projections[0]
    rng = np.random.default_rng(0)
    x = mock_oracle.bf16_round(rng.standard_normal((cur, K), dtype=np.float32))
    w = mock_oracle.bf16_round(rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K))
    ranks = adapter_ranks(wl)
    a = {i: mock_oracle.bf16_round(rng.standard_normal((r, K), dtype=np.float32) / np.sqrt(K))
         for i, r in enumerate(ranks)}
    b = {i: mock_oracle.bf16_round(0.02 * rng.standard_normal((N, r), dtype=np.float32)) for i, r in enumerate(ranks)}
    sc = {i: 2.0 for i in range(len(ranks))}
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        mock_oracle.fused_lora_forward(x, w, a, b, sc, routes)
        times.append(time.perf_counter() - t0)
        if max_steps is not None and len(times) >= max_steps:
            break
        if max_steps is None and time.perf_counter() - t_start > budget_s:
            break
    return cur, times


def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads") for i in threadpool_info() if i.get("user_api") == "blas"]
        if n and n[0]:
            return int(n[0])
    except Exception:  # noqa: BLE001
        pass
    return os.cpu_count() or 1


# --------------------------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from lorafusion_b200.workloads import WORKLOADS
    wl = WORKLOADS[args.workload]
    T, warm = cpu_oracle_sample(wl, 0.0, max_steps=max(1, args.warmup))
    _, times = cpu_oracle_sample(wl, 0.0, max_steps=args.steps)
    ms = 1e3 * statistics.mean(times)
    value = T / (ms / 1e3)
    cores = cpu_threads()
    _, K, N = wl.projections[0]
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "tokens_per_step": T, "in_features": K, "out_features": N,
                   "adapters": wl.n_adapters, "rank": 16, "tile_rows": wl.tile_capacity,
                   "what": "numpy float32 restatement of lorafusion mock_ops.fused_lora_forward on bf16-rounded "
                           "inputs, host cores, one full 4096-token forward per step"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} full forwards of {T} tokens"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- our arm
def run_ours(args):
    import torch
    import torch.distributed as dist

    from lorafusion_b200 import _native as nat
    from lorafusion_b200 import b200_ops
    from lorafusion_b200.sharding import allreduce_spanning_grads
    from lorafusion_b200.workloads import WORKLOADS

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
    pr = local_problem(wl, world, rank, device)
    T, K, N = pr["T"], pr["K"], pr["N"]
    counts = algorithmic_counts(pr["routing"], pr["ranks"], K, N, T)
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

    default_stages = SH | EX | (nat.LF_STAGE_SEPARATE if args.separate_launches else 0)

    def fwd_default(ev):
        if ev:
            ev[0].record()
        prep.launch(y, default_stages)
        if ev:
            ev[1].record()

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
    t = timed(fwd_default, args.steps, args.warmup, 2)
    clocks = sampler.stop()
    n_launch = prep.launch_count()  # reflects the path actually taken (co-scheduling switch included)
    step_local_ms = statistics.mean(s[0] for s in t)
    step_ms = rank_max(step_local_ms)
    value = pr["global_T"] / (step_ms / 1e3)
    gpu_launches = n_launch * args.steps
    # breakdown with the shrink and the fused GEMM as separate launches
    tsplit = timed(fwd_staged, max(5, args.steps // 2), 2, 3)
    shrink_ms = statistics.mean(s[0] for s in tsplit)
    gemm_ms = statistics.mean(s[1] for s in tsplit)

    # yardsticks: our GEMM with LoRA disabled, and cuBLAS x @ W^T
    tb = timed(lambda ev: (ev and ev[0].record(), prep.launch(y, BA), ev and ev[1].record()),
               max(5, args.steps // 2), 2, 2)
    own_base_ms = statistics.mean(s[0] for s in tb)
    xw = pr["x"]
    wt = pr["w"].t()
    tc = timed(lambda ev: (ev and ev[0].record(), torch.matmul(xw, wt), ev and ev[1].record()),
               max(5, args.steps // 2), 2, 2)
    cublas_ms = statistics.mean(s[0] for s in tc)

    # e2e through the plugin call with pinned host buffers
    x_host = pr["x"].cpu().pin_memory()
    y_host = torch.empty((T, N), dtype=torch.bfloat16).pin_memory()

    def e2e(ev):
        if ev:
            ev[0].record()
        b200_ops.fused_lora_forward_host(x_host, pr["w"], pr["lora_a"], pr["lora_b"], pr["adapters"], pr["routing"],
                                         out=y_host)
        if ev:
            ev[1].record()

    te = timed(e2e, max(5, args.steps // 2), 2, 2)
    e2e_ms = rank_max(statistics.mean(s[0] for s in te))

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

        def cstep(ev):
            if ev:
                ev[0].record()
            coord.run_batch(reqs, req_x)
            if ev:
                ev[1].record()

        tco = timed(cstep, max(5, args.steps // 2), 2, 2)
        co_ms = statistics.mean(s[0] for s in tco)
        coordinator = {"value": sum(r.num_rows for r in reqs) / (co_ms / 1e3), "unit": "tokens/s", "ms_per_step": co_ms,
                       "requests": len(reqs),
                       "path": "Coordinator.run_batch: greedy_pack (C++), lf_copy_rows gather, fused forward, "
                               "lf_copy_rows scatter; request tensors resident on the device"}

    # forward + backward (with the all-reduce of spanning adapter gradients when N > 1)
    fwd_bwd = None
    if not args.no_fwd_bwd:
        def fb(ev):
            if ev:
                ev[0].record()
            b200_ops.fused_lora_forward(pr["x"], pr["w"], pr["lora_a"], pr["lora_b"], pr["adapters"], pr["routing"])
            gx, ga, gb = b200_ops.fused_lora_backward(pr["grad"], pr["x"], pr["w"], pr["lora_a"], pr["lora_b"],
                                                      pr["adapters"], pr["routing"])
            allreduce_spanning_grads(pr["plan"], ga, gb, dict(enumerate(pr["ranks"])), K, N, device)
            if ev:
                ev[1].record()

        tfb = timed(fb, max(5, args.steps // 2), 2, 2)
        fb_ms = rank_max(statistics.mean(s[0] for s in tfb))
        bwd_launches = b200_ops.last_launch_count()

        def bwd_only(ev):
            if ev:
                ev[0].record()
            b200_ops.fused_lora_backward(pr["grad"], pr["x"], pr["w"], pr["lora_a"], pr["lora_b"], pr["adapters"],
                                         pr["routing"])
            if ev:
                ev[1].record()

        tbo = timed(bwd_only, max(5, args.steps // 2), 2, 2)
        bwd_ms = rank_max(statistics.mean(s[0] for s in tbo))
        fwd_bwd = {"value": pr["global_T"] / (fb_ms / 1e3), "unit": "tokens/s", "ms_per_step": fb_ms,
                   "launches_per_step": n_launch + bwd_launches, "backward_ms": bwd_ms,
                   "tflops": counts["fwdbwd_flops"] * world / (fb_ms / 1e3) / 1e12,
                   "spanning_adapters": len(pr["plan"].spanning)}

    err = nat.device_error()
    peaks = load_peaks()
    if n_launch == 1:  # one kernel does the whole forward: shrink on spare CTA pairs, GEMM + expand
        dom_kernel = "tc_gemm_pair_kernel (co-scheduled routed shrink + base GEMM + LoRA expand)"
        dom_flops, dom_ms = counts["fwd_flops"], step_local_ms
    else:
        dom_kernel = "tc_gemm_pair_kernel (base GEMM + LoRA expand)"
        dom_flops, dom_ms = counts["gemm_flops"], gemm_ms
    gemm_tflops = dom_flops / (dom_ms / 1e3) / 1e12
    shrink_gbs = counts["shrink_bytes"] / (shrink_ms / 1e3) / 1e9
    # ncu cannot capture the co-scheduled (cooperative) launch; its DRAM traffic is unmeasured and
    # the two-launch path's capture of the fused GEMM is reported beside it
    pair_traffic = load_traffic("tc_gemm_pair_kernel", args.workload)
    traffic = pair_traffic if n_launch == 2 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        Tc, times = cpu_oracle_sample(wl, args.cpu_seconds)
        cpu = {"value": Tc / statistics.mean(times), "unit": "tokens/s", "cores": cpu_threads(), "kind": "port",
               "sample": f"{len(times)} full {Tc}-token forwards of the numpy float32 oracle "
                         f"({sum(times):.1f} s of CPU work)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": args.workload, "tokens_per_gpu": wl.total_rows, "global_tokens": pr["global_T"],
                       "in_features": K, "out_features": N, "adapters": wl.n_adapters, "rank": 16,
                       "tile_rows": wl.tile_capacity, "routes_rank0": len(pr["routing"].routes),
                       "parallelism": f"dp{world} over packed bins (no forward communication)",
                       "l2": "flushed (256 MiB write) before every timed step",
                       "pass": "forward (routed shrink + fused base GEMM/LoRA expand)"},
            "roofline": {"kernel": dom_kernel, "bound": "tensor",
                         "achieved": gemm_tflops, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": gemm_tflops / peaks["bf16_tflops"], "traffic": traffic,
                         "peak_source": f"{peaks['source']} bf16 dense (burst)",
                         "flops_per_launch": dom_flops, "ms_per_launch": dom_ms, "launches_per_step": n_launch,
                         "traffic_two_launch_gemm": pair_traffic},
            "split_launches": {"shrink_ms": shrink_ms, "gemm_ms": gemm_ms, "total_ms": shrink_ms + gemm_ms},
            "shrink_roofline": {"kernel": "tc_shrink_kernel (standalone launch)", "bound": "hbm", "achieved": shrink_gbs,
                                "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": shrink_gbs / peaks["hbm_gbs"],
                                "bytes_per_launch": counts["shrink_bytes"], "ms_per_launch": shrink_ms},
            "vs_base_gemm": {"fused_fwd_ms": step_ms, "own_base_gemm_ms": own_base_ms, "cublas_base_gemm_ms": cublas_ms,
                             "fused_over_own_base": step_ms / own_base_ms, "fused_over_cublas": step_ms / cublas_ms,
                             "cublas_tflops": 2.0 * T * K * N / (cublas_ms / 1e3) / 1e12},
            "e2e": {"value": pr["global_T"] / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": T * K * 2, "d2h_bytes_per_step": T * N * 2,
                    "path": "b200_ops.fused_lora_forward_host -> lf_forward_host: pinned host x/y, 1024-row "
                            "chunks enqueued by one native call, copies in both directions overlapped with the "
                            "fused forward"},
            "fwd_bwd": fwd_bwd,
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


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
