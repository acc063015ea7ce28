"""Seeded synthetic workloads for the fused multi-adapter LoRA op.

The five workloads below are the shapes the op is measured and checked on
(there is no dataset: every tensor is synthetic).  Each adapter is one
request whose ``request_id`` equals its ``adapter_id``; the routing comes from
the scheduler (``bucket_by_adapter -> greedy_pack -> build_microbatch``),
exactly as ``lorafusion/runtime/coordinator.py:48-56`` builds it.

Value distributions (all drawn in float32 from a seeded CPU generator, then
rounded to the problem dtype):

* ``x ~ N(0, 1)``, ``grad_out ~ N(0, 1)``
* ``W = randn(N, K) / sqrt(K)``
* ``A_i = randn(r_i, K) / sqrt(K)``, ``B_i = 0.02 * randn(N, r_i)``
* ``alpha_i = 2 r_i`` so every adapter's scaling is 2.0

Row counts: Zipf(s) over the adapters (``w_k = k^-s``,
``c_k = max(1, floor(w_k / sum(w) * T))``, the remainder added to ``c_1``), or
for the decode-like skew workload, 1-4 rows for every small adapter and the
rest in adapter 0.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

# Only numpy and the standard library at import time: the benchmark's CPU arm loads this file by
# itself, without the package or its native library.  torch and the scheduler are imported by the
# functions that build tensors or packings.


@dataclass(frozen=True)
class Workload:
    name: str
    description: str
    total_rows: int
    projections: tuple[tuple[str, int, int], ...]  # (name, in_features K, out_features N)
    n_adapters: int
    tile_capacity: int
    dtype: str  # "float32" or "bfloat16" (the torch dtype: torch_dtype())
    row_law: str  # "fixed", "zipf" or "skew"
    zipf_s: float = 1.1
    fixed_rows: tuple[int, ...] = ()
    ranks: tuple[int, ...] = field(default=())  # empty -> drawn by rank_choices
    rank_choices: tuple[int, ...] = (16,)
    backward: bool = True
    seed: int = 0


WORKLOADS: dict[str, Workload] = {
    "cfg1_fp32_small": Workload(
        "cfg1_fp32_small", "fp32 fwd+bwd, x[128,256], 4 adapters rank 8, rows [48,40,24,16], 16-row tiles",
        128, (("proj", 256, 256),), 4, 16, "float32", "fixed", fixed_rows=(48, 40, 24, 16),
        rank_choices=(8,)),
    "cfg2_h4096_a16_r16": Workload(
        "cfg2_h4096_a16_r16", "bf16 4096->4096, 16 adapters rank 16, 4096 tokens Zipf(1.1), 128-row tiles, fwd",
        4096, (("proj", 4096, 4096),), 16, 128, "bfloat16", "zipf", zipf_s=1.1,
        rank_choices=(16,), backward=False),
    "cfg3_llama8b_a64_mixed": Workload(
        "cfg3_llama8b_a64_mixed", "bf16 Llama-3-8B projections, 64 adapters ranks U{8,16,32,64}, 8192 tokens Zipf(1.1)",
        8192, (("q", 4096, 4096), ("k", 4096, 1024), ("v", 4096, 1024), ("o", 4096, 4096),
               ("gate", 4096, 14336), ("up", 4096, 14336), ("down", 14336, 4096)),
        64, 128, "bfloat16", "zipf", zipf_s=1.1, rank_choices=(8, 16, 32, 64)),
    "cfg4_decode_skew_a512": Workload(
        "cfg4_decode_skew_a512", "bf16 4096->4096, 512 adapters rank 16, 16384 tokens, one dominant adapter, 64-row tiles",
        16384, (("proj", 4096, 4096),), 512, 64, "bfloat16", "skew", rank_choices=(16,)),
    "cfg5_70b_a256_r64": Workload(
        "cfg5_70b_a256_r64", "bf16 70B projections, 256 adapters rank 64, 32768 tokens Zipf(1.0)",
        32768, (("q", 8192, 8192), ("o", 8192, 8192), ("gate", 8192, 28672), ("up", 8192, 28672),
                ("down", 28672, 8192)),
        256, 128, "bfloat16", "zipf", zipf_s=1.0, rank_choices=(64,)),
}


def zipf_row_counts(n_adapters: int, total: int, s: float) -> list[int]:
    w = [k ** (-s) for k in range(1, n_adapters + 1)]
    tot = sum(w)
    counts = [max(1, int(math.floor(wk / tot * total))) for wk in w]
    counts[0] += total - sum(counts)
    return counts


def skew_row_counts(n_adapters: int, total: int, seed: int) -> list[int]:
    rng = np.random.default_rng(seed)
    small = rng.integers(1, 5, size=n_adapters - 1).tolist()
    return [total - sum(small)] + small


def row_counts(wl: Workload, total_rows: int | None = None) -> list[int]:
    total = wl.total_rows if total_rows is None else total_rows
    if wl.row_law == "fixed":
        return list(wl.fixed_rows)
    if wl.row_law == "zipf":
        return zipf_row_counts(wl.n_adapters, total, wl.zipf_s)
    return skew_row_counts(wl.n_adapters, total, wl.seed)


def adapter_ranks(wl: Workload) -> list[int]:
    if wl.ranks:
        return list(wl.ranks)
    if len(wl.rank_choices) == 1:
        return [wl.rank_choices[0]] * wl.n_adapters
    rng = np.random.default_rng(wl.seed + 1)
    return [int(r) for r in rng.choice(np.array(wl.rank_choices), size=wl.n_adapters)]


def torch_dtype(wl: Workload):
    import torch
    return getattr(torch, wl.dtype)


def layout(wl: Workload, total_rows: int | None = None):
    """Requests and packing of a workload (no tensors): the scheduler's bins."""
    from lorafusion_b200.scheduler import Request, bucket_by_adapter, greedy_pack
    counts = row_counts(wl, total_rows)
    requests = [Request(request_id=i, adapter_id=i, num_rows=c) for i, c in enumerate(counts)]
    groups = bucket_by_adapter(requests)
    packing = greedy_pack({g.adapter_id: g.total_rows for g in groups}, wl.tile_capacity)
    return requests, packing


def _randn(gen, *shape: int):
    import torch
    return torch.randn(*shape, generator=gen, dtype=torch.float32)


@dataclass
class Problem:
    x: object                # torch.Tensor [T, K]
    base_weight: object      # [N, K]
    lora_a: dict             # adapter id -> [r, K]
    lora_b: dict             # adapter id -> [N, r]
    adapters: dict           # adapter id -> AdapterSpec
    routing: object
    row_order: list[int]
    grad_out: object | None  # [T, N]


def make_problem(
    wl: Workload,
    projection: int = 0,
    device="cpu",
    dtype=None,
    total_rows: int | None = None,
    with_grad: bool | None = None,
    seed: int | None = None,
) -> Problem:
    """Materialise one projection of a workload with seeded tensors."""
    import torch

    from lorafusion_b200.config import AdapterSpec
    from lorafusion_b200.scheduler import build_microbatch
    dtype = torch_dtype(wl) if dtype is None else dtype
    seed = wl.seed if seed is None else seed
    _, k_in, n_out = wl.projections[projection]
    ranks = adapter_ranks(wl)
    requests, packing = layout(wl, total_rows)
    gen = torch.Generator().manual_seed(seed * 7919 + projection)
    req_tensors = {r.request_id: _randn(gen, r.num_rows, k_in) for r in requests}
    fused_x, routing, row_order = build_microbatch(requests, req_tensors, packing)
    w = _randn(gen, n_out, k_in) / math.sqrt(k_in)
    lora_a, lora_b, adapters = {}, {}, {}
    for aid in range(wl.n_adapters):
        r = ranks[aid]
        lora_a[aid] = (_randn(gen, r, k_in) / math.sqrt(k_in)).to(device=device, dtype=dtype)
        lora_b[aid] = (0.02 * _randn(gen, n_out, r)).to(device=device, dtype=dtype)
        adapters[aid] = AdapterSpec(aid, r, float(2 * r), k_in, n_out)
    want_grad = wl.backward if with_grad is None else with_grad
    g = _randn(gen, fused_x.shape[0], n_out).to(device=device, dtype=dtype) if want_grad else None
    return Problem(
        x=fused_x.to(device=device, dtype=dtype),
        base_weight=w.to(device=device, dtype=dtype),
        lora_a=lora_a,
        lora_b=lora_b,
        adapters=adapters,
        routing=routing,
        row_order=row_order,
        grad_out=g,
    )
