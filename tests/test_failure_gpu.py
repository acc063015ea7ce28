"""Failure detection on the GPU, in the form that faults nothing: every wait inside the kernels is
bounded, and a wait that runs out reports a status the host reads (lf_device_error) while the
kernel unwinds (stops its CTA, lets its copies and MMAs land, frees tensor memory, returns).

The test shortens the limit to 50 ms and makes one co-scheduled forward's GEMM CTAs wait for a
ready value that no shrink item publishes (lf_inject_stale_ready).  The launch must end, the
status must be a timeout code, and the next normal forward must be correct.  Nothing here traps,
faults or hangs a GPU: the flag that is never set is only waited for up to the limit.
"""

import numpy as np
import pytest
import torch

from oracle import mock_oracle

pytestmark = pytest.mark.gpu

BF16_TOL = dict(rtol=2e-2, atol=2e-2)


def _problem():
    from lorafusion_b200.config import AdapterSpec, TileRoute, TileRoutingConfig
    rng = np.random.default_rng(9)
    T, K, N = 1024, 512, 768
    ranks = {0: 16, 1: 8, 2: 32}
    r16 = mock_oracle.bf16_round
    x = r16(rng.standard_normal((T, K), dtype=np.float32))
    w = r16(rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K))
    a = {i: r16(rng.standard_normal((r, K), dtype=np.float32) / np.sqrt(K)) for i, r in ranks.items()}
    b = {i: r16(0.02 * rng.standard_normal((N, r), dtype=np.float32)) for i, r in ranks.items()}
    routes = [(0, 300, 0), (300, 305, 1), (305, 700, 2), (700, 1024, 0)]
    t = lambda v: torch.from_numpy(v).to("cuda", torch.bfloat16)  # noqa: E731
    ad = {i: AdapterSpec(i, r, 2.0 * r, K, N) for i, r in ranks.items()}
    rt = TileRoutingConfig(128, [TileRoute(s, e, i) for s, e, i in routes])
    f = mock_oracle.as_f64
    ref = mock_oracle.fused_lora_forward(f(x), f(w), f(a), f(b), {i: 2.0 for i in ranks}, routes)
    return (t(x), t(w), {i: t(v) for i, v in a.items()}, {i: t(v) for i, v in b.items()}, ad, rt), ref


def test_bounded_wait_runs_out_and_reports_status():
    from lorafusion_b200 import _native as nat
    from lorafusion_b200 import b200_ops
    args, ref = _problem()
    b200_ops.use_cooperative_launch(True)
    assert nat.device_error() == 0
    y = b200_ops.fused_lora_forward(*args)  # warm: slabs, tables, kernels loaded
    if b200_ops.last_launch_count() != 1:
        pytest.skip("the shrink does not run inside the GEMM launch on this device")
    assert nat.device_error() == 0
    nat.set_wait_limit(50_000_000)  # 50 ms
    try:
        nat.check(nat.lib().lf_inject_stale_ready(1), "lf_inject_stale_ready")
        b200_ops.fused_lora_forward(*args)
        code = nat.device_error()  # synchronizes: the launch ended
        assert code in (nat.ERR_TIMEOUT_FULL, nat.ERR_TIMEOUT_EMPTY, nat.ERR_TIMEOUT_ACC, nat.ERR_TIMEOUT_DRAIN,
                        nat.ERR_TIMEOUT_FLAG), hex(code)
    finally:
        nat.check(nat.lib().lf_inject_stale_ready(0), "lf_inject_stale_ready")
        nat.set_wait_limit(0)
    # the context is usable and the next call is correct
    y = b200_ops.fused_lora_forward(*args)
    ok, msg = mock_oracle.allclose_report(y.float().cpu().numpy(), ref, **BF16_TOL)
    assert ok, msg
    assert nat.device_error() == 0


def test_wait_limit_arguments():
    from lorafusion_b200 import _native as nat
    L = nat.lib()
    assert L.lf_set_wait_limit(10) == nat.LF_ERR_INVALID_ARG          # below 1 ms
    assert L.lf_set_wait_limit(61_000_000_000) == nat.LF_ERR_INVALID_ARG
    assert L.lf_set_wait_limit(0) == nat.LF_OK
    assert L.lf_inject_stale_ready(-1) == nat.LF_ERR_INVALID_ARG


def test_injected_tool_turns_co_scheduling_off_by_default():
    """Under an injected CUDA tool (Nsight Compute sets NV_NSIGHT_INJECTION_* for its target), whose
    kernel replay breaks launches whose CTAs wait on each other, the library starts with
    co-scheduled launches off; without one, on."""
    import os
    import subprocess
    import sys
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = "from lorafusion_b200 import _native as nat; print(nat.co_scheduling()[0])"
    tool_vars = ("CUDA_INJECTION64_PATH", "NV_NSIGHT_INJECTION_TRANSPORT_TYPE", "NV_COMPUTE_PROFILER_PERFWORKS_DIR",
                 "NVIDIA_PROCESS_INJECTION_CRASH_REPORTING")
    clean = {k: v for k, v in os.environ.items() if k not in tool_vars}
    plain = subprocess.run([sys.executable, "-c", code], cwd=repo, env=clean, capture_output=True, text=True,
                           timeout=300)
    tooled = subprocess.run([sys.executable, "-c", code], cwd=repo, env=dict(clean, NV_NSIGHT_INJECTION_TRANSPORT_TYPE="uds"),
                            capture_output=True, text=True, timeout=300)
    assert plain.returncode == 0 and tooled.returncode == 0, plain.stderr + tooled.stderr
    assert plain.stdout.split()[-1] == "1" and tooled.stdout.split()[-1] == "0"
