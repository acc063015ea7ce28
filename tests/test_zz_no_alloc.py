"""The allocation-free forward entry point (lf_forward_noalloc).

It exists for callers that can only hand the operator their input and output buffers — e.g.
plugin interfaces that give an operator no device allocator, or processes whose device memory
is fully planned up front — so it cannot ask them for a workspace.  These tests call it through
the C ABI and compare it with the ordinary lf_forward (caller-provided workspace), within the
bf16 tolerance the other GPU tests use, on two consecutive calls: the shared scratch array keeps
the previous call's contents, which must not leak into the next result.

This file is collected last on purpose (a failure here leaves every other test already run).
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import mock_oracle

pytestmark = pytest.mark.gpu

BF16_TOL = dict(rtol=2e-2, atol=2e-2)


def _problem(seed, sizes, ranks, K, N):
    from lorafusion_b200 import b200_ops
    from lorafusion_b200.config import AdapterSpec, TileRoute, TileRoutingConfig
    g = torch.Generator(device="cuda").manual_seed(seed)
    T = sum(sizes)
    x = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(N, K, device="cuda", generator=g) / K ** 0.5).bfloat16()
    a = {i: (torch.randn(r, K, device="cuda", generator=g) / K ** 0.5).bfloat16() for i, r in ranks.items()}
    b = {i: (0.02 * torch.randn(N, r, device="cuda", generator=g)).bfloat16() for i, r in ranks.items()}
    ad = {i: AdapterSpec(i, r, 2.0 * r, K, N) for i, r in ranks.items()}
    routes, cur = [], 0
    for i, n in enumerate(sizes):
        routes.append(TileRoute(cur, cur + n, i % len(ranks)))
        cur += n
    return b200_ops.prepare_forward(x, w, a, b, ad, TileRoutingConfig(128, routes))


def _with_workspace(prep):
    from lorafusion_b200 import _native as nat
    y = prep.new_output()
    rc = nat.lib().lf_forward(ctypes.byref(prep.prob), ctypes.byref(prep.plan.info), prep.plan.table_dev.data_ptr(),
                              y.data_ptr(), prep.ws.data_ptr(), prep.ws.numel(),
                              torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    return y


def _no_alloc(prep):
    from lorafusion_b200 import _native as nat
    y = torch.full((prep.T, prep.N), float("nan"), dtype=prep.dtype, device="cuda")
    rc = nat.lib().lf_forward_noalloc(ctypes.byref(prep.prob), ctypes.byref(prep.plan.info),
                                      prep.plan.table_dev.data_ptr(), y.data_ptr(),
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == 0, nat.status_text(rc)
    return y


def _close(got, ref, what):
    ok, msg = mock_oracle.allclose_report(got.float().cpu().numpy(), ref.float().cpu().numpy(), **BF16_TOL)
    assert ok, f"{what}: {msg}"


def test_no_alloc_forward_matches_workspace_forward_twice():
    from lorafusion_b200 import _native as nat
    first = _problem(1, [700, 3, 180, 141], {0: 16, 1: 8, 2: 32}, 512, 768)
    second = _problem(2, [128, 90, 38, 300], {0: 64, 1: 16}, 384, 256)
    for prep in (first, second):  # two calls in a row, different layouts and ranks
        ref = _with_workspace(prep)
        got = _no_alloc(prep)
        torch.cuda.synchronize()
        _close(got, ref, f"T={prep.T}")
        assert torch.isfinite(got.float()).all()
    again = _no_alloc(first)  # the array now holds the second problem's scratch
    _close(again, _with_workspace(first), "repeat of the first problem")
    assert nat.device_error() == 0


def test_no_alloc_rejects_scratch_beyond_its_array():
    from lorafusion_b200 import _native as nat
    prep = _problem(3, [256], {0: 16}, 64, 64)
    info = nat.PlanInfo()
    ctypes.memmove(ctypes.byref(info), ctypes.byref(prep.plan.info), ctypes.sizeof(info))
    info.n_segtiles = 1 << 20  # would need 128 MiB of scratch at rank 16
    y = prep.new_output()
    rc = nat.lib().lf_forward_noalloc(ctypes.byref(prep.prob), ctypes.byref(info), prep.plan.table_dev.data_ptr(),
                                      y.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == nat.LF_ERR_CAPACITY
    assert nat.lib().lf_forward_workspace_bytes(ctypes.byref(info), nat.LF_BF16) > (16 << 20)
