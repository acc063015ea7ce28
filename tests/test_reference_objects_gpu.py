"""The reference's own object shapes through the B200 op.

lorafusion's caller passes its own dataclasses (``lorafusion/ops/config.py:14-69``: AdapterSpec with
``adapter_id, rank, alpha, in_features, out_features`` and a ``scaling`` property; TileRoute with
``row_start, row_end, adapter_id``; TileRoutingConfig with ``tile_size, routes`` and
``validate(total_rows)``), and its Coordinator calls ``backend.fused_lora_forward(fused_x,
base_weight, lora_a, lora_b, adapters, routing)`` (``lorafusion/runtime/coordinator.py:58-65``).
The stand-ins below are frozen dataclasses with exactly those fields and members, written here
(the reference itself is not importable on the GPU host); the op reads only attributes, so they
must behave as this package's own classes do.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import pytest
import torch

from oracle import mock_oracle

pytestmark = pytest.mark.gpu

BF16_TOL = dict(rtol=2e-2, atol=2e-2)


@dataclass(frozen=True)
class RefAdapterSpec:
    adapter_id: int
    rank: int
    alpha: float
    in_features: int
    out_features: int

    @property
    def scaling(self) -> float:
        return self.alpha / self.rank


@dataclass(frozen=True)
class RefTileRoute:
    row_start: int
    row_end: int
    adapter_id: int

    @property
    def num_rows(self) -> int:
        return self.row_end - self.row_start


@dataclass(frozen=True)
class RefTileRoutingConfig:
    tile_size: int
    routes: list = field(default_factory=list)

    def validate(self, total_rows: int) -> None:
        expect = 0
        for r in self.routes:
            if r.row_start != expect:
                raise ValueError(f"Routing gap/overlap at row {r.row_start}, expected {expect}")
            expect = r.row_end
        if expect != total_rows:
            raise ValueError(f"Routing covers {expect} rows, expected {total_rows}")


def _problem(seed=19):
    rng = np.random.default_rng(seed)
    T, K, N = 700, 384, 512
    ranks = {3: 16, 7: 8, 11: 32}
    r16 = mock_oracle.bf16_round
    x = r16(rng.standard_normal((T, K), dtype=np.float32))
    g = r16(rng.standard_normal((T, N), dtype=np.float32))
    w = r16(rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K))
    a = {i: r16(rng.standard_normal((r, K), dtype=np.float32) / np.sqrt(K)) for i, r in ranks.items()}
    b = {i: r16(0.02 * rng.standard_normal((N, r), dtype=np.float32)) for i, r in ranks.items()}
    routes = [(0, 128, 3), (128, 200, 7), (200, 256, 3), (256, 384, 11), (384, 700, 7)]
    return T, K, N, ranks, x, g, w, a, b, routes


def test_reference_dataclasses_through_forward_and_backward():
    from lorafusion_b200 import b200_ops
    T, K, N, ranks, x, g, w, a, b, routes = _problem()
    dev = lambda v: torch.from_numpy(v).to("cuda", torch.bfloat16)  # noqa: E731
    specs = {i: RefAdapterSpec(i, r, 2.0 * r, K, N) for i, r in ranks.items()}
    routing = RefTileRoutingConfig(128, [RefTileRoute(s, e, i) for s, e, i in routes])
    da, db = {i: dev(v) for i, v in a.items()}, {i: dev(v) for i, v in b.items()}
    y = b200_ops.fused_lora_forward(dev(x), dev(w), da, db, specs, routing)
    gx, ga, gb = b200_ops.fused_lora_backward(dev(g), dev(x), dev(w), da, db, specs, routing)
    f = mock_oracle.as_f64
    sc = {i: 2.0 for i in ranks}
    ry = mock_oracle.fused_lora_forward(f(x), f(w), f(a), f(b), sc, routes)
    rgx, rga, rgb = mock_oracle.fused_lora_backward(f(g), f(x), f(w), f(a), f(b), sc, routes)
    for name, got, ref in [("y", y, ry), ("grad_x", gx, rgx)] + [(f"ga{k}", ga[k], rga[k]) for k in rga] + \
            [(f"gb{k}", gb[k], rgb[k]) for k in rgb]:
        ok, msg = mock_oracle.allclose_report(got.float().cpu().numpy(), ref, **BF16_TOL)
        assert ok, f"{name}: {msg}"
    assert list(ga) == [3, 7, 11]  # first appearance in the routes, like the reference's dicts
    # the reference's validate runs first and its ValueError propagates
    bad = RefTileRoutingConfig(128, [RefTileRoute(0, 100, 3), RefTileRoute(120, 700, 7)])
    with pytest.raises(ValueError, match="gap/overlap"):
        b200_ops.fused_lora_forward(dev(x), dev(w), da, db, specs, bad)
    # an adapter id the dicts do not hold: KeyError, as the reference's dict lookups raise
    missing = RefTileRoutingConfig(128, [RefTileRoute(0, 700, 5)])
    with pytest.raises(KeyError):
        b200_ops.fused_lora_forward(dev(x), dev(w), da, db, specs, missing)


def test_coordinator_shaped_loop_with_reference_specs():
    """The reference Coordinator's run_batch steps (bucket, pack, build the fused batch, call the
    backend, scatter) with the reference's AdapterSpec objects and b200_ops as the backend."""
    from lorafusion_b200 import b200_ops
    from lorafusion_b200.coordinator import Coordinator
    from lorafusion_b200.scheduler import Request
    T, K, N, ranks, x, g, w, a, b, routes = _problem(23)
    dev = lambda v: torch.from_numpy(np.ascontiguousarray(v)).to("cuda", torch.bfloat16)  # noqa: E731
    specs = {i: RefAdapterSpec(i, r, 2.0 * r, K, N) for i, r in ranks.items()}
    reqs = [Request(0, 3, 150), Request(1, 7, 90), Request(2, 11, 60), Request(3, 3, 33)]
    rng = np.random.default_rng(5)
    xs = {r.request_id: mock_oracle.bf16_round(rng.standard_normal((r.num_rows, K), dtype=np.float32)) for r in reqs}
    coord = Coordinator(dev(w), specs, {i: dev(v) for i, v in a.items()}, {i: dev(v) for i, v in b.items()},
                        tile_capacity=64, backend=b200_ops)
    out = coord.run_batch(reqs, {rid: dev(v) for rid, v in xs.items()})
    f = mock_oracle.as_f64
    for r in reqs:
        aid = r.adapter_id
        ref = mock_oracle.fused_lora_forward(f(xs[r.request_id]), f(w), {aid: f(a[aid])}, {aid: f(b[aid])},
                                             {aid: 2.0}, [(0, r.num_rows, aid)])
        ok, msg = mock_oracle.allclose_report(out[r.request_id].float().cpu().numpy(), ref, **BF16_TOL)
        assert ok, f"request {r.request_id}: {msg}"
