"""Fused-batch assembly on the GPU (lorafusion/scheduler/data_batcher.py:18-103) and the
request-in/result-out runtime (lorafusion/runtime/coordinator.py:42-67).

``build_microbatch`` and ``scatter_outputs`` move rows with one ``lf_copy_rows`` launch for CUDA
tensors; their results must equal the reference semantics (the CPU torch path, pinned to the
reference's golden layouts in test_scheduler.py) byte for byte.  The Coordinator must return,
per request, the oracle's forward of that request's rows.
"""

import ctypes
import zlib

import numpy as np
import pytest
import torch

from oracle import mock_oracle

pytestmark = pytest.mark.gpu

BF16_TOL = dict(rtol=2e-2, atol=2e-2)


@pytest.fixture(scope="module", autouse=True)
def _require_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")


def _requests(counts, adapters):
    from lorafusion_b200.scheduler import Request
    return [Request(i, a, c) for i, (c, a) in enumerate(zip(counts, adapters))]


def _pack(reqs, cap):
    from lorafusion_b200.scheduler import bucket_by_adapter, greedy_pack
    return greedy_pack({g.adapter_id: g.total_rows for g in bucket_by_adapter(reqs)}, cap)


def _tensors(reqs, K, dtype, seed, strided=False):
    g = torch.Generator().manual_seed(seed)
    out = {}
    for r in reqs:
        t = torch.randn(r.num_rows, K + (3 if strided else 0), generator=g).to(dtype)
        out[r.request_id] = t[:, :K] if strided else t
    return out


CASES = [
    # (name, counts, adapters, K, dtype, cap, strided)
    ("bf16_aligned", [300, 5, 1, 94, 200, 100], [0, 1, 2, 3, 0, 1], 256, torch.bfloat16, 128, False),
    ("f32_row148B", [40, 17, 3, 64], [2, 2, 0, 1], 37, torch.float32, 16, False),
    ("bf16_row10B", [9, 1, 30], [0, 1, 0], 5, torch.bfloat16, 8, False),
    ("f16_strided", [130, 70, 12], [1, 0, 1], 64, torch.float16, 64, True),
    ("one_row", [1], [0], 8, torch.bfloat16, 128, False),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_device_gather_and_scatter_are_byte_exact(case):
    from lorafusion_b200.scheduler import build_microbatch, scatter_outputs
    name, counts, adapters, K, dtype, cap, strided = case
    reqs = _requests(counts, adapters)
    packing = _pack(reqs, cap)
    host = _tensors(reqs, K, dtype, zlib.crc32(name.encode()), strided)
    dev = {k: v.cuda() for k, v in host.items()}
    if strided:  # keep the row stride of the CUDA tensors wider than the row
        dev = {k: torch.nn.functional.pad(v.cuda(), (0, 3))[:, :K] for k, v in host.items()}
        assert all(t.stride(0) == K + 3 for t in dev.values())
    fx_ref, rt_ref, order_ref = build_microbatch(reqs, host, packing)
    fx, rt, order = build_microbatch(reqs, dev, packing)
    assert fx.is_cuda and fx.dtype == fx_ref.dtype and fx.shape == fx_ref.shape
    assert order == order_ref and rt.routes == rt_ref.routes and rt.tile_size == rt_ref.tile_size
    assert torch.equal(fx.cpu().view(torch.uint8), fx_ref.contiguous().view(torch.uint8))
    out_ref = scatter_outputs(fx_ref, order_ref)
    out = scatter_outputs(fx, order)
    assert list(out.keys()) == list(out_ref.keys())
    for k in out_ref:
        assert out[k].is_cuda and out[k].is_contiguous() and out[k].shape == out_ref[k].shape
        assert torch.equal(out[k].cpu().view(torch.uint8), out_ref[k].contiguous().view(torch.uint8))
        assert torch.equal(out[k].cpu(), host[k])  # every row of every request comes back in order


def test_device_gather_at_config_layouts():
    """cfg2 and cfg4 layouts (39 and 747 routes, requests split across bins), K = 64."""
    from lorafusion_b200.scheduler import build_microbatch, scatter_outputs
    from lorafusion_b200.workloads import WORKLOADS, row_counts
    for wl_name in ("cfg2_h4096_a16_r16", "cfg4_decode_skew_a512"):
        wl = WORKLOADS[wl_name]
        counts = row_counts(wl, wl.total_rows)
        reqs = _requests(counts, list(range(len(counts))))
        packing = _pack(reqs, wl.tile_capacity)
        host = _tensors(reqs, 64, torch.bfloat16, 5)
        fx_ref, _, order_ref = build_microbatch(reqs, host, packing)
        fx, _, order = build_microbatch(reqs, {k: v.cuda() for k, v in host.items()}, packing)
        assert order == order_ref
        assert torch.equal(fx.cpu(), fx_ref)
        out = scatter_outputs(fx, order)
        assert list(out.keys()) == list(scatter_outputs(fx_ref, order_ref).keys())
        for k, v in out.items():
            assert torch.equal(v.cpu(), host[k])


def test_mixed_dtypes_promote_like_cat_and_scatter_rejects_short_output():
    from lorafusion_b200.scheduler import build_microbatch, scatter_outputs
    reqs = _requests([20, 7], [0, 1])
    packing = _pack(reqs, 16)
    host = {0: torch.randn(20, 12).half(), 1: torch.randn(7, 12)}
    fx_ref, _, order = build_microbatch(reqs, host, packing)
    fx, _, _ = build_microbatch(reqs, {k: v.cuda() for k, v in host.items()}, packing)
    assert fx.dtype == fx_ref.dtype == torch.float32
    assert torch.equal(fx.cpu(), fx_ref)
    with pytest.raises(IndexError):
        scatter_outputs(fx[:5], order)


def test_copy_rows_c_abi_runs():
    """lf_copy_rows directly: three runs with different strides, one launch."""
    from lorafusion_b200 import _native as nat
    src = torch.arange(40 * 24, dtype=torch.int32, device="cuda").view(40, 24)
    dst = torch.zeros(30, 16, dtype=torch.int32, device="cuda")
    runs = (nat.RowRun * 3)()
    spec = [(src[0], dst[0], 24 * 4, 16 * 4, 10), (src[30, 4:], dst[10], 24 * 4, 16 * 4, 10),
            (src[12, 8:], dst[20], 48 * 4, 16 * 4, 10)]
    row0 = 0
    for i, (s, d, ss, ds, n) in enumerate(spec):
        runs[i].src, runs[i].dst, runs[i].src_stride, runs[i].dst_stride = s.data_ptr(), d.data_ptr(), ss, ds
        runs[i].rows, runs[i].row0 = n, row0
        row0 += n
    table = torch.frombuffer(bytearray(bytes(runs)), dtype=torch.uint8).cuda()
    rc = nat.lib().lf_copy_rows(table.data_ptr(), 3, 16 * 4, row0, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    ref = torch.cat([src[0:10, 0:16], src[30:40, 4:20], src[12:32:2, 8:24]])
    assert torch.equal(dst, ref)
    assert nat.lib().lf_copy_rows(None, 1, 64, 10, None) == nat.LF_ERR_INVALID_ARG
    assert nat.lib().lf_copy_rows(None, 0, 64, 0, None) == 0


def test_coordinator_end_to_end_matches_oracle():
    """Requests in, per-request outputs out, through the B200 backend (the default)."""
    from lorafusion_b200.config import AdapterSpec
    from lorafusion_b200.coordinator import Coordinator
    K, N = 256, 384
    ranks = {0: 16, 1: 8, 2: 32}
    rng = np.random.default_rng(3)
    rnd = lambda *s: mock_oracle.bf16_round(rng.standard_normal(s).astype(np.float32))  # noqa: E731
    w = mock_oracle.bf16_round(rnd(N, K) / np.sqrt(K))
    a = {i: mock_oracle.bf16_round(rnd(r, K) / np.sqrt(K)) for i, r in ranks.items()}
    b = {i: mock_oracle.bf16_round(0.02 * rnd(N, r)) for i, r in ranks.items()}
    adapters = {i: AdapterSpec(i, r, 2.0 * r, K, N) for i, r in ranks.items()}
    reqs = _requests([150, 3, 90, 200, 41], [0, 1, 2, 0, 1])
    xs = {r.request_id: rnd(r.num_rows, K) for r in reqs}
    to = lambda v: torch.from_numpy(np.ascontiguousarray(v)).cuda().bfloat16()  # noqa: E731
    coord = Coordinator(to(w), adapters, {i: to(v) for i, v in a.items()}, {i: to(v) for i, v in b.items()},
                        tile_capacity=128)
    out = coord.run_batch(reqs, {rid: to(v) for rid, v in xs.items()})
    assert sorted(out) == [r.request_id for r in reqs]
    for r in reqs:
        x = xs[r.request_id]
        aid = r.adapter_id
        f = mock_oracle.as_f64
        ref = mock_oracle.fused_lora_forward(f(x), f(w), {aid: f(a[aid])}, {aid: f(b[aid])}, {aid: 2.0},
                                             [(0, r.num_rows, aid)])
        ok, msg = mock_oracle.allclose_report(out[r.request_id].float().cpu().numpy(), ref, **BF16_TOL)
        assert ok, f"request {r.request_id}: {msg}"
    from lorafusion_b200 import _native as nat
    assert nat.device_error() == 0
