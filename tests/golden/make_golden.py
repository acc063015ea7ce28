"""Generate golden fixtures by running lorafusion's own reference code.

Run where a checkout of the reference is available (read-only), giving its path:

    python tests/golden/make_golden.py --ref <path of the reference checkout>

It writes, next to this file:

* ``layout_golden.npz`` — for the five benchmark workloads and a set of edge
  cases: the reference scheduler's bins, routes and ``row_order``
  (``bucket_by_adapter -> greedy_pack -> build_microbatch``, as in
  ``lorafusion/runtime/coordinator.py:48-56``), and for every fused row the
  source ``(request_id, row)`` (recovered by pushing index-valued tensors
  through ``build_microbatch``), plus ``scatter_outputs`` round trips.
* ``ops_golden.npz`` — inputs and outputs of the reference
  ``lorafusion.ops.mock_ops`` forward and backward on small seeded problems:
  the fp32 workload ``cfg1`` and several edge cases (single route, split
  adapters, rank 1, one-row routes), and one bf16-rounded problem evaluated
  in fp32.

The fixtures are small and committed; the tests never read the reference.
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of a checkout of the reference (read only)")
    args = ap.parse_args()
    sys.path.insert(0, REPO)
    sys.path.insert(0, args.ref)

    from lorafusion.ops import mock_ops as ref_mock  # noqa: E402
    from lorafusion.ops.config import AdapterSpec as RAdapterSpec  # noqa: E402
    from lorafusion.ops.config import TileRoute as RTileRoute  # noqa: E402
    from lorafusion.ops.config import TileRoutingConfig as RRouting  # noqa: E402
    from lorafusion.scheduler.adapter_grouper import Request as RRequest  # noqa: E402
    from lorafusion.scheduler.adapter_grouper import bucket_by_adapter as r_bucket  # noqa: E402
    from lorafusion.scheduler.data_batcher import build_microbatch as r_build  # noqa: E402
    from lorafusion.scheduler.data_batcher import scatter_outputs as r_scatter  # noqa: E402
    from lorafusion.scheduler.milp_packer import greedy_pack as r_greedy  # noqa: E402

    from lorafusion_b200.workloads import WORKLOADS, row_counts  # noqa: E402

    # ------------------------------------------------------------------ layout
    cases: list[tuple[str, list[tuple[int, int, int]], int]] = []
    for name, wl in WORKLOADS.items():
        counts = row_counts(wl)
        cases.append((name, [(i, i, c) for i, c in enumerate(counts)], wl.tile_capacity))
    rng = np.random.default_rng(1234)
    # interleaved arrivals, several requests per adapter, adapters above capacity
    for cap in (1, 7, 16, 64, 128):
        reqs = []
        for rid in range(40):
            aid = int(rng.integers(0, 9))
            reqs.append((rid, aid, int(rng.integers(1, 3 * cap + 5))))
        cases.append((f"mixed_cap{cap}", reqs, cap))
    cases.append(("single_request", [(5, 3, 200)], 64))
    cases.append(("exact_capacity", [(0, 0, 64), (1, 1, 64), (2, 2, 128)], 64))
    cases.append(("demo_like", [(i, i // 6, int(rng.integers(5, 120))) for i in range(18)], 64))

    layout: dict[str, np.ndarray] = {}
    names = []
    for name, reqs, cap in cases:
        requests = [RRequest(rid, aid, n) for rid, aid, n in reqs]
        groups = r_bucket(requests)
        packing = r_greedy({g.adapter_id: g.total_rows for g in groups}, cap)
        # index-valued request tensors: column 0 = request id, column 1 = row
        tensors = {
            r.request_id: torch.stack(
                [torch.full((r.num_rows,), float(r.request_id), dtype=torch.float64),
                 torch.arange(r.num_rows, dtype=torch.float64)], dim=1)
            for r in requests
        }
        fused, routing, row_order = r_build(requests, tensors, packing)
        scattered = r_scatter(fused, row_order)
        bins_flat = np.array([(b, aid, n) for b, entries in enumerate(packing.bins) for aid, n in entries],
                             dtype=np.int64).reshape(-1, 3)
        routes = np.array([(rt.row_start, rt.row_end, rt.adapter_id) for rt in routing.routes],
                          dtype=np.int64).reshape(-1, 3)
        scat_keys = np.array(list(scattered.keys()), dtype=np.int64)
        scat_rows = np.concatenate([scattered[k][:, 1].numpy() for k in scattered]).astype(np.int64) \
            if scattered else np.zeros(0, np.int64)
        layout[f"{name}/requests"] = np.array(reqs, dtype=np.int64).reshape(-1, 3)
        layout[f"{name}/cap"] = np.array(cap, dtype=np.int64)
        layout[f"{name}/bins"] = bins_flat
        layout[f"{name}/routes"] = routes
        layout[f"{name}/num_tiles"] = np.array(routing.num_tiles(), dtype=np.int64)
        layout[f"{name}/row_order"] = np.array(row_order, dtype=np.int64)
        layout[f"{name}/source"] = fused.numpy().astype(np.int64)
        layout[f"{name}/scatter_keys"] = scat_keys
        layout[f"{name}/scatter_rows"] = scat_rows
        names.append(name)
    layout["names"] = np.array(names)
    np.savez_compressed(os.path.join(HERE, "layout_golden.npz"), **layout)

    # ------------------------------------------------------------------ ops
    ops: dict[str, np.ndarray] = {}
    op_names = []

    def add_case(name, x, w, a, b, ranks, alphas, routes, g, round_bf16=False):
        if round_bf16:
            to = lambda t: t.to(torch.bfloat16).to(torch.float32)  # noqa: E731
            x, w, g = to(x), to(w), to(g)
            a = {k: to(v) for k, v in a.items()}
            b = {k: to(v) for k, v in b.items()}
        adapters = {aid: RAdapterSpec(aid, ranks[aid], alphas[aid], w.shape[1], w.shape[0]) for aid in a}
        routing = RRouting(tile_size=16, routes=[RTileRoute(s, e, aid) for s, e, aid in routes])
        y = ref_mock.fused_lora_forward(x, w, a, b, adapters, routing)
        gx, ga, gb = ref_mock.fused_lora_backward(g, x, w, a, b, adapters, routing)
        p = f"{name}/"
        ops[p + "x"] = x.numpy()
        ops[p + "w"] = w.numpy()
        ops[p + "g"] = g.numpy()
        ops[p + "routes"] = np.array(routes, dtype=np.int64).reshape(-1, 3)
        ops[p + "adapter_ids"] = np.array(sorted(a), dtype=np.int64)
        ops[p + "ranks"] = np.array([ranks[k] for k in sorted(a)], dtype=np.int64)
        ops[p + "alphas"] = np.array([alphas[k] for k in sorted(a)], dtype=np.float64)
        for k in sorted(a):
            ops[p + f"a{k}"] = a[k].numpy()
            ops[p + f"b{k}"] = b[k].numpy()
        ops[p + "y"] = y.numpy()
        ops[p + "gx"] = gx.numpy()
        ops[p + "grad_keys"] = np.array(list(ga.keys()), dtype=np.int64)
        for k in ga:
            ops[p + f"ga{k}"] = ga[k].numpy()
            ops[p + f"gb{k}"] = gb[k].numpy()
        ops[p + "bf16"] = np.array(round_bf16)
        op_names.append(name)

    def rand_case(name, seed, T, K, N, routes, ranks, round_bf16=False):
        gen = torch.Generator().manual_seed(seed)
        x = torch.randn(T, K, generator=gen)
        w = torch.randn(N, K, generator=gen) / K ** 0.5
        a = {aid: torch.randn(r, K, generator=gen) / K ** 0.5 for aid, r in ranks.items()}
        b = {aid: 0.02 * torch.randn(N, r, generator=gen) for aid, r in ranks.items()}
        g = torch.randn(T, N, generator=gen)
        alphas = {aid: float(2 * r) for aid, r in ranks.items()}
        add_case(name, x, w, a, b, ranks, alphas, routes, g, round_bf16)

    # cfg1 exactly as the fp32 workload builds it
    from lorafusion_b200.workloads import make_problem  # noqa: E402
    wl = WORKLOADS["cfg1_fp32_small"]
    pr = make_problem(wl, with_grad=True)
    routes1 = [(r.row_start, r.row_end, r.adapter_id) for r in pr.routing.routes]
    add_case("cfg1", pr.x, pr.base_weight, pr.lora_a, pr.lora_b,
             {k: v.rank for k, v in pr.adapters.items()}, {k: v.alpha for k, v in pr.adapters.items()},
             routes1, pr.grad_out)
    rand_case("single_route", 11, 64, 96, 80, [(0, 64, 0)], {0: 8})
    rand_case("split_adapter", 12, 200, 128, 64,
              [(0, 70, 1), (70, 75, 0), (75, 140, 1), (140, 141, 2), (141, 200, 0)], {0: 4, 1: 16, 2: 8})
    rand_case("rank1_one_row_routes", 13, 24, 32, 48,
              [(i, i + 1, i % 5) for i in range(24)], {k: 1 + (k % 2) for k in range(5)})
    rand_case("unused_adapter", 14, 40, 64, 40, [(0, 25, 2), (25, 40, 0)], {0: 8, 1: 8, 2: 8})
    rand_case("bf16_mixed_ranks", 15, 256, 128, 160,
              [(0, 100, 0), (100, 128, 1), (128, 130, 2), (130, 200, 3), (200, 256, 0)],
              {0: 16, 1: 8, 2: 32, 3: 64}, round_bf16=True)
    ops["names"] = np.array(op_names)
    np.savez_compressed(os.path.join(HERE, "ops_golden.npz"), **ops)
    print("wrote", len(names), "layout cases and", len(op_names), "op cases")


if __name__ == "__main__":
    main()
