"""GPU parity of the B200 op against the CPU oracle (pinned to the reference's golden outputs).

Tolerance rule, elementwise: ``|got - ref| <= atol + rtol * |ref|`` with
  bf16 / f16 inputs: rtol = atol = 2e-2,
  float32 inputs:    rtol = atol = 1e-5,
where ``ref`` is the oracle evaluated in float64 on the very values the GPU gets (bf16/f16
problems: the rounded values), i.e. the exact math of the reference's formula.  Full-size
problems, too large for the CPU oracle, compare with the same formula evaluated on the GPU in
float32 without TF32.  Routing tables are checked bit-exactly on the CPU (tests/test_native_abi.py).
"""

import zlib

import numpy as np
import pytest
import torch

from conftest import op_case
from oracle import mock_oracle

pytestmark = pytest.mark.gpu

BF16_TOL = dict(rtol=2e-2, atol=2e-2)
FP32_TOL = dict(rtol=1e-5, atol=1e-5)


@pytest.fixture(scope="module", autouse=True)
def _require_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from lorafusion_b200 import _native
    _native.lib()
    yield
    assert _native.device_error() == 0, "a kernel reported a bounded-wait timeout"


def _ops():
    from lorafusion_b200 import b200_ops
    return b200_ops


def _cfg():
    from lorafusion_b200.config import AdapterSpec, TileRoute, TileRoutingConfig
    return AdapterSpec, TileRoute, TileRoutingConfig


def _to_torch(case, dtype, dev="cuda"):
    AdapterSpec, TileRoute, TileRoutingConfig = _cfg()
    K = case["x"].shape[1]
    N = case["w"].shape[0]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device=dev, dtype=dtype)  # noqa: E731
    ad = {i: AdapterSpec(i, case["ranks"][i], case["alphas"][i], K, N) for i in case["a"]}
    routing = TileRoutingConfig(16, [TileRoute(s, e, a) for s, e, a in case["routes"]])
    return (t(case["x"]), t(case["w"]), {i: t(v) for i, v in case["a"].items()},
            {i: t(v) for i, v in case["b"].items()}, ad, routing, t(case["g"]))


def _check(got, ref, tol, what):
    ok, msg = mock_oracle.allclose_report(got.float().cpu().numpy(), ref, **tol)
    assert ok, f"{what}: {msg}"


def _oracle_outputs(case):
    """The oracle's forward and backward, in float64, on the case's inputs."""
    f = mock_oracle.as_f64
    sc = {i: case["alphas"][i] / case["ranks"][i] for i in case["ranks"]}
    x, w, g, a, b = f(case["x"]), f(case["w"]), f(case["g"]), f(case["a"]), f(case["b"])
    y = mock_oracle.fused_lora_forward(x, w, a, b, sc, case["routes"])
    gx, ga, gb = mock_oracle.fused_lora_backward(g, x, w, a, b, sc, case["routes"])
    return dict(case, y=y, gx=gx, ga=ga, gb=gb, grad_keys=list(ga.keys()))


def _run_and_compare(case, dtype, tol, backward=True):
    ops = _ops()
    x, w, a, b, ad, routing, g = _to_torch(case, dtype)
    y = ops.fused_lora_forward(x, w, a, b, ad, routing)
    assert y.dtype == dtype and y.shape == (x.shape[0], w.shape[0])
    _check(y, case["y"], tol, "forward")
    if not backward:
        return
    gx, ga, gb = ops.fused_lora_backward(g, x, w, a, b, ad, routing)
    _check(gx, case["gx"], tol, "grad_x")
    assert list(ga.keys()) == case["grad_keys"] and list(gb.keys()) == case["grad_keys"]
    for k in case["grad_keys"]:
        assert ga[k].shape == case["ga"][k].shape and ga[k].is_contiguous()
        assert gb[k].shape == case["gb"][k].shape and gb[k].is_contiguous()
        _check(ga[k], case["ga"][k], tol, f"grad_a[{k}]")
        _check(gb[k], case["gb"][k], tol, f"grad_b[{k}]")


@pytest.mark.parametrize("name", ["cfg1", "single_route", "split_adapter", "rank1_one_row_routes", "unused_adapter"])
def test_fp32_matches_reference_golden(ops_golden, name):
    """The golden cases' inputs (the reference's own fixtures); outputs against the float64 oracle
    (which tests/test_oracle_golden.py pins to the reference's outputs)."""
    case = op_case(ops_golden, name)
    assert list(_oracle_outputs(case)["ga"].keys()) == case["grad_keys"]
    _run_and_compare(_oracle_outputs(case), torch.float32, FP32_TOL)


def test_bf16_matches_reference_golden(ops_golden):
    case = op_case(ops_golden, "bf16_mixed_ranks")
    _run_and_compare(_oracle_outputs(case), torch.bfloat16, BF16_TOL)


def _random_case(seed, T, K, N, routes, ranks, dtype):
    rng = np.random.default_rng(seed)
    rnd = lambda *s: rng.standard_normal(s).astype(np.float32)  # noqa: E731
    rounder = mock_oracle.bf16_round if dtype == torch.bfloat16 else (
        (lambda v: v.astype(np.float16).astype(np.float32)) if dtype == torch.float16 else (lambda v: v))
    case = {"x": rounder(rnd(T, K)), "w": rounder(rnd(N, K) / np.sqrt(K)), "g": rounder(rnd(T, N))}
    case["a"] = {i: rounder(rnd(r, K) / np.sqrt(K)) for i, r in ranks.items()}
    case["b"] = {i: rounder(0.02 * rnd(N, r)) for i, r in ranks.items()}
    case["ranks"] = dict(ranks)
    case["alphas"] = {i: float(2 * r) for i, r in ranks.items()}
    case["routes"] = routes
    return _oracle_outputs(case)


def _routes_from_sizes(sizes, adapters):
    out, cur = [], 0
    for n, a in zip(sizes, adapters):
        out.append((cur, cur + n, a))
        cur += n
    return out


SHAPES = [
    # (T, K, N, route sizes, route adapters, ranks)
    ("aligned_r16", 512, 256, 512, [128, 128, 256], [0, 1, 2], {0: 16, 1: 16, 2: 16}),
    ("misaligned_r16", 700, 512, 768, [300, 5, 1, 94, 200, 100], [0, 1, 2, 3, 0, 1], {0: 16, 1: 16, 2: 16, 3: 16}),
    ("rank8_pad", 300, 256, 256, [100, 200], [0, 1], {0: 8, 1: 8}),
    ("rank32", 384, 256, 512, [150, 234], [1, 0], {0: 32, 1: 32}),
    ("rank64", 384, 512, 256, [64, 64, 256], [0, 1, 2], {0: 64, 1: 64, 2: 64}),
    ("mixed_ranks", 640, 384, 384, [200, 37, 3, 150, 250], [0, 1, 2, 3, 1], {0: 8, 1: 16, 2: 32, 3: 64}),
    ("ragged_k_n", 333, 200, 264, [111, 222], [0, 1], {0: 16, 1: 16}),
    ("many_small", 256, 256, 256, [4] * 64, list(range(64)), {i: 16 for i in range(64)}),
    ("tiny", 3, 64, 64, [1, 2], [0, 1], {0: 4, 1: 16}),
    ("n_small", 130, 64, 8, [65, 65], [0, 1], {0: 16, 1: 16}),
]


@pytest.mark.parametrize("shape", SHAPES, ids=[s[0] for s in SHAPES])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32], ids=["bf16", "f16", "f32"])
def test_random_shapes_match_oracle(shape, dtype):
    _, T, K, N, sizes, adapters, ranks = shape
    routes = _routes_from_sizes(sizes, adapters)
    case = _random_case(zlib.crc32(shape[0].encode()) % 1000, T, K, N, routes, ranks, dtype)
    _run_and_compare(case, dtype, FP32_TOL if dtype == torch.float32 else BF16_TOL)


def test_cfg2_layout_reduced_width_matches_oracle():
    """The benchmark's routing (cfg2: 4096 tokens, 16 adapters, Zipf 1.1, 128-row bins) at K = N = 512."""
    from lorafusion_b200.workloads import WORKLOADS, layout
    from lorafusion_b200.scheduler import build_microbatch
    wl = WORKLOADS["cfg2_h4096_a16_r16"]
    reqs, packing = layout(wl)
    tensors = {r.request_id: torch.zeros(r.num_rows, 1) for r in reqs}
    _, routing, _ = build_microbatch(reqs, tensors, packing)
    routes = [(r.row_start, r.row_end, r.adapter_id) for r in routing.routes]
    case = _random_case(7, 4096, 512, 512, routes, {i: 16 for i in range(16)}, torch.bfloat16)
    _run_and_compare(case, torch.bfloat16, BF16_TOL)


def _check_dev(got, ref, tol, what, worst=None):
    """The tolerance rule (|got - ref| <= atol + rtol |ref|) evaluated on the GPU, for tensors too
    large to copy to the host; records the worst |err| / tol in `worst` (a dict) when given."""
    got = got.float()
    err = (got - ref).abs()
    lim = tol["atol"] + tol["rtol"] * ref.abs()
    bad = (err > lim) | ~torch.isfinite(got)
    n_bad = int(bad.sum())
    ratio = float((err / lim).max()) if err.numel() else 0.0
    if worst is not None:
        worst[what] = ratio
    assert n_bad == 0, f"{what}: {n_bad}/{got.numel()} outside tol, worst |err|/tol {ratio:.3f}, " \
                       f"max abs err {err.max().item():.3e}"


def _full_size_cases():
    from lorafusion_b200.workloads import WORKLOADS
    out = []
    for name in ("cfg2_h4096_a16_r16", "cfg3_llama8b_a64_mixed", "cfg4_decode_skew_a512", "cfg5_70b_a256_r64"):
        for p, (pname, _, _) in enumerate(WORKLOADS[name].projections):
            out.append((name, p, f"{name.split('_')[0]}_{pname}"))
    return out


FULL_SIZE = _full_size_cases()


@pytest.mark.parametrize("wl_name,proj", [(w, p) for w, p, _ in FULL_SIZE], ids=[i for _, _, i in FULL_SIZE])
def test_full_size_against_torch_fp32(wl_name, proj):
    """Every projection of every workload at full size (cfg2; cfg3's seven Llama-3-8B projections
    with ranks 8-64; cfg4: 512 adapters, 747 routes; cfg5's five 70B projections, rank 64, 32768
    tokens): forward and backward against the reference's formula evaluated on the GPU in float32
    without TF32, under the plain bf16 rule; the worst |err| / tol of each tensor is printed."""
    from lorafusion_b200.workloads import WORKLOADS, make_problem
    ops = _ops()
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    pr = make_problem(WORKLOADS[wl_name], projection=proj, device="cuda", with_grad=True)
    y = ops.fused_lora_forward(pr.x, pr.base_weight, pr.lora_a, pr.lora_b, pr.adapters, pr.routing)
    gx, ga, gb = ops.fused_lora_backward(pr.grad_out, pr.x, pr.base_weight, pr.lora_a, pr.lora_b, pr.adapters,
                                         pr.routing)
    x, w, g = pr.x.float(), pr.base_weight.float(), pr.grad_out.float()
    ref_y = x @ w.t()
    ref_gx = g @ w
    ref_ga, ref_gb = {}, {}
    for r in pr.routing.routes:
        s = pr.adapters[r.adapter_id].scaling
        a, b = pr.lora_a[r.adapter_id].float(), pr.lora_b[r.adapter_id].float()
        xs, gs = x[r.row_start:r.row_end], g[r.row_start:r.row_end]
        xa = xs @ a.t()
        ref_y[r.row_start:r.row_end] += s * (xa @ b.t())
        gxa = s * (gs @ b)
        ref_gx[r.row_start:r.row_end] += gxa @ a
        ref_ga[r.adapter_id] = ref_ga.get(r.adapter_id, 0) + gxa.t() @ xs
        ref_gb[r.adapter_id] = ref_gb.get(r.adapter_id, 0) + s * (gs.t() @ xa)
    worst: dict[str, float] = {}
    _check_dev(y, ref_y, BF16_TOL, "forward", worst)
    del ref_y, y
    _check_dev(gx, ref_gx, BF16_TOL, "grad_x", worst)
    assert list(ga.keys()) == list(ref_ga.keys()) and list(gb.keys()) == list(ref_gb.keys())
    for k in ref_ga:
        _check_dev(ga[k], ref_ga[k], BF16_TOL, f"grad_a[{k}]", worst)
        _check_dev(gb[k], ref_gb[k], BF16_TOL, f"grad_b[{k}]", worst)
    wa = max(v for k, v in worst.items() if k.startswith("grad_a"))
    wb = max(v for k, v in worst.items() if k.startswith("grad_b"))
    print(f"\nworst |err|/tol {wl_name} projection {proj}: forward {worst['forward']:.3f} grad_x "
          f"{worst['grad_x']:.3f} grad_a {wa:.3f} grad_b {wb:.3f}")
    if wl_name.startswith("cfg2"):  # base part alone: zero B gives exactly the base GEMM; compare with cuBLAS
        zero_b = {k: torch.zeros_like(v) for k, v in pr.lora_b.items()}
        y0 = ops.fused_lora_forward(pr.x, pr.base_weight, pr.lora_a, zero_b, pr.adapters, pr.routing)
        _check_dev(y0, (pr.x @ pr.base_weight.t()).float(), BF16_TOL, "base GEMM vs cuBLAS")
    from lorafusion_b200 import _native as nat
    assert nat.device_error() == 0


def test_deterministic_and_repeatable():
    ops = _ops()
    routes = _routes_from_sizes([300, 5, 400, 319], [0, 1, 2, 0])
    case = _random_case(3, 1024, 512, 512, routes, {0: 16, 1: 32, 2: 64}, torch.bfloat16)
    x, w, a, b, ad, routing, g = _to_torch(case, torch.bfloat16)
    y1 = ops.fused_lora_forward(x, w, a, b, ad, routing)
    y2 = ops.fused_lora_forward(x, w, a, b, ad, routing)
    assert torch.equal(y1, y2)
    r1 = ops.fused_lora_backward(g, x, w, a, b, ad, routing)
    r2 = ops.fused_lora_backward(g, x, w, a, b, ad, routing)
    assert torch.equal(r1[0], r2[0])
    for k in r1[1]:
        assert torch.equal(r1[1][k], r2[1][k]) and torch.equal(r1[2][k], r2[2][k])


def test_edge_cases():
    ops = _ops()
    AdapterSpec, TileRoute, TileRoutingConfig = _cfg()
    dev = "cuda"
    # empty batch
    K, N = 64, 32
    w = torch.randn(N, K, device=dev)
    a = {0: torch.randn(4, K, device=dev)}
    b = {0: torch.randn(N, 4, device=dev)}
    ad = {0: AdapterSpec(0, 4, 8.0, K, N), 1: AdapterSpec(1, 4, 8.0, K, N)}
    y = ops.fused_lora_forward(torch.empty(0, K, device=dev), w, a, b, ad, TileRoutingConfig(16, []))
    assert y.shape == (0, N)
    # a zero-length route still yields (zero) gradients for its adapter, like the reference
    x = torch.randn(5, K, device=dev)
    g = torch.randn(5, N, device=dev)
    a[1] = torch.randn(4, K, device=dev)
    b[1] = torch.randn(N, 4, device=dev)
    rt = TileRoutingConfig(16, [TileRoute(0, 0, 1), TileRoute(0, 5, 0)])
    gx, ga, gb = ops.fused_lora_backward(g, x, w, a, b, ad, rt)
    assert list(ga) == [1, 0]
    assert torch.count_nonzero(ga[1]) == 0 and torch.count_nonzero(gb[1]) == 0
    # unknown adapter -> KeyError; bad routing -> ValueError
    with pytest.raises(KeyError):
        ops.fused_lora_forward(x, w, a, b, ad, TileRoutingConfig(16, [TileRoute(0, 5, 7)]))
    with pytest.raises(ValueError):
        ops.fused_lora_forward(x, w, a, b, ad, TileRoutingConfig(16, [TileRoute(0, 4, 0)]))
    # non-contiguous activations and an fp32 base weight with bf16 activations (LoRA factors with
    # the workloads' magnitudes: A ~ N(0, 1/sqrt(K)), B ~ 0.02 N(0, 1))
    xb = torch.randn(K, 40, device=dev, dtype=torch.bfloat16).t()
    ab = {0: (a[0] / K ** 0.5).bfloat16(), 1: (a[1] / K ** 0.5).bfloat16()}
    bb = {0: (0.02 * b[0]).bfloat16(), 1: (0.02 * b[1]).bfloat16()}
    rt2 = TileRoutingConfig(16, [TileRoute(0, 40, 0)])
    y = ops.fused_lora_forward(xb, w, ab, bb, ad, rt2)
    f = lambda t: t.double().cpu().numpy()  # noqa: E731
    ref = f(xb) @ f(w.bfloat16()).T + 2.0 * (f(xb) @ f(ab[0]).T) @ f(bb[0]).T
    _check(y, ref, BF16_TOL, "non-contiguous x")


def test_expand_rounds_lora_intermediate_like_reference():
    """The LoRA expand reads S = s x A_i^T rounded once to the input dtype (bf16 here), as the
    reference's own bf16 / fp16 paths round x A_i^T before multiplying by B_i (mock_ops in bf16,
    triton_ops.py:337).  With LoRA factors of magnitude 1 (A, B ~ N(0, 1): |S B| terms ~ 10) that
    rounding is visible in y; the result matches the float64 oracle with the same single rounding
    of S under the plain bf16 rule.  The gradients dA / dB read S as hi + lo (about 16 bits) and
    match the unrounded oracle."""
    ops = _ops()
    AdapterSpec, TileRoute, TileRoutingConfig = _cfg()
    K, N, T = 64, 32, 300
    g0 = torch.Generator().manual_seed(5)
    r16 = lambda t: t.bfloat16().double()  # noqa: E731
    x, w = r16(torch.randn(T, K, generator=g0)), r16(torch.randn(N, K, generator=g0) / K ** 0.5)
    g = r16(torch.randn(T, N, generator=g0))
    a = {0: r16(torch.randn(4, K, generator=g0)), 1: r16(torch.randn(8, K, generator=g0))}
    b = {0: r16(torch.randn(N, 4, generator=g0)), 1: r16(torch.randn(N, 8, generator=g0))}
    ad = {0: AdapterSpec(0, 4, 8.0, K, N), 1: AdapterSpec(1, 8, 16.0, K, N)}
    routes = [(0, 170, 0), (170, 300, 1)]
    rt = TileRoutingConfig(16, [TileRoute(s0, e0, i) for s0, e0, i in routes])
    dev = lambda t: t.to("cuda", torch.bfloat16)  # noqa: E731
    y = ops.fused_lora_forward(dev(x), dev(w), {i: dev(v) for i, v in a.items()}, {i: dev(v) for i, v in b.items()},
                               ad, rt)
    ref = x @ w.T
    for s0, e0, i in routes:
        s_int = r16(2.0 * (x[s0:e0] @ a[i].T))  # the expand's operand: s x A^T rounded once to bf16
        ref[s0:e0] += s_int @ b[i].T
    _check(y, ref.numpy(), BF16_TOL, "forward with bf16-rounded LoRA intermediate")
    _, ga, gb = ops.fused_lora_backward(dev(g), dev(x), dev(w), {i: dev(v) for i, v in a.items()},
                                        {i: dev(v) for i, v in b.items()}, ad, rt)
    sc = {0: 2.0, 1: 2.0}
    _, rga, rgb = mock_oracle.fused_lora_backward(g.numpy(), x.numpy(), w.numpy(), {i: v.numpy() for i, v in a.items()},
                                                  {i: v.numpy() for i, v in b.items()}, sc, routes)
    for k in rga:
        _check(ga[k], rga[k], BF16_TOL, f"grad_a[{k}]")
        _check(gb[k], rgb[k], BF16_TOL, f"grad_b[{k}]")


@pytest.mark.parametrize("single_cta", [False, True], ids=["cta_pair", "single_cta"])
def test_gemm_tilings_match_oracle(single_cta):
    """Both GEMM tilings (256x256 on CTA pairs, 128x256 on single CTAs), odd row-tile count."""
    from lorafusion_b200 import _native as nat
    ops = _ops()
    routes = _routes_from_sizes([130, 3, 250, 97, 160], [0, 1, 2, 0, 3])  # 640 rows = 5 row tiles
    case = _random_case(11, 640, 320, 520, routes, {0: 16, 1: 8, 2: 32, 3: 16}, torch.bfloat16)
    x, w, a, b, ad, routing, _ = _to_torch(case, torch.bfloat16)
    prep = ops.prepare_forward(x, w, a, b, ad, routing)
    y = prep.new_output()
    stages = nat.LF_STAGE_SHRINK | nat.LF_STAGE_EXPAND | (nat.LF_STAGE_SINGLE_CTA if single_cta else 0)
    prep.launch(y, stages)
    _check(y, case["y"], BF16_TOL, "forward")
    y0 = prep.new_output()
    prep.launch(y0, nat.LF_STAGE_BASE | (nat.LF_STAGE_SINGLE_CTA if single_cta else 0))
    _check(y0, case["x"] @ case["w"].T, BF16_TOL, "base GEMM only")


@pytest.mark.parametrize("mode", ["prologue", "dedicated", "separate"],
                         ids=["shrink_prologue", "shrink_pairs", "separate_shrinks"])
def test_co_scheduling_switch_matches_oracle(mode):
    """Forward and backward with the routed shrinks inside the GEMM launch (forward 1 launch,
    backward 2), either as every CTA's prologue or on dedicated CTA pairs, and as launches of
    their own (2 and 3, S_f taken from the forward); all match the oracle."""
    ops = _ops()
    routes = _routes_from_sizes([300, 5, 1, 94, 200, 100, 324], [0, 1, 2, 3, 0, 1, 2])  # 1024 rows
    case = _random_case(23, 1024, 512, 768, routes, {0: 16, 1: 8, 2: 32, 3: 64}, torch.bfloat16)
    co_scheduled = mode != "separate"
    ops.use_cooperative_launch(co_scheduled, shrink_prologue=mode == "prologue")
    try:
        x, w, a, b, ad, routing, g = _to_torch(case, torch.bfloat16)
        y = ops.fused_lora_forward(x, w, a, b, ad, routing)
        assert ops.last_launch_count() == (1 if co_scheduled else 2)
        gx, ga, gb = ops.fused_lora_backward(g, x, w, a, b, ad, routing)
        # the backward follows a forward on the same x: S_f comes from it (no x . A^T shrink)
        assert ops.last_launch_count() == (2 if co_scheduled else 3)
    finally:
        ops.use_cooperative_launch(True)
    _check(y, case["y"], BF16_TOL, "forward")
    _check(gx, case["gx"], BF16_TOL, "grad_x")
    for k in case["grad_keys"]:
        _check(ga[k], case["ga"][k], BF16_TOL, f"grad_a[{k}]")
        _check(gb[k], case["gb"][k], BF16_TOL, f"grad_b[{k}]")
    from lorafusion_b200 import _native as nat
    assert nat.device_error() == 0


def test_k_split_tail_matches_whole_tiles():
    """The GEMM's last round, when at most half full, runs its tiles as K-split parts on the idle
    CTA pairs (partial fp32 tiles summed in part order by the last part).  2560 x 4096 with the
    shrink in its own launch: 160 tiles on 74 pairs, 12 tail tiles in 4 K parts each.  The result
    equals whole tiles up to fp32 summation order, is repeatable bit for bit, and matches the
    oracle; without cooperative launches the tail is not split."""
    from lorafusion_b200 import _native as nat
    ops = _ops()
    routes = _routes_from_sizes([700, 3, 1100, 257, 500], [0, 1, 2, 0, 3])  # 2560 rows
    case = _random_case(41, 2560, 512, 4096, routes, {0: 16, 1: 8, 2: 32, 3: 16}, torch.bfloat16)
    x, w, a, b, ad, routing, g = _to_torch(case, torch.bfloat16)
    prep = ops.prepare_forward(x, w, a, b, ad, routing)

    def run(stages_list):
        y = prep.new_output()
        for st in stages_list:
            prep.launch(y, st)
        return y

    two = [nat.LF_STAGE_SHRINK, nat.LF_STAGE_EXPAND]
    base = [nat.LF_STAGE_BASE]
    y_split, y_split2, base_split = run(two), run(two), run(base)
    ops.use_cooperative_launch(False)
    try:
        y_whole, base_whole = run(two), run(base)
    finally:
        ops.use_cooperative_launch(True)
    assert torch.equal(y_split, y_split2)
    torch.testing.assert_close(y_split.float(), y_whole.float(), rtol=1e-2, atol=2e-2)
    torch.testing.assert_close(base_split.float(), base_whole.float(), rtol=1e-2, atol=2e-2)
    _check(y_split, case["y"], BF16_TOL, "forward, K-split tail")
    _check(base_split, case["x"] @ case["w"].T, BF16_TOL, "base GEMM, K-split tail")
    assert nat.device_error() == 0


def test_k_split_small_problem_uses_all_pairs():
    """Fewer tiles than CTA pairs (T=300, N=768: 6 tiles) and no co-scheduled shrink: each tile is
    cut into 4 K parts; forward and the base GEMM match the oracle."""
    from lorafusion_b200 import _native as nat
    ops = _ops()
    routes = _routes_from_sizes([100, 77, 123], [0, 1, 0])
    case = _random_case(43, 300, 1024, 768, routes, {0: 16, 1: 32}, torch.bfloat16)
    x, w, a, b, ad, routing, g = _to_torch(case, torch.bfloat16)
    prep = ops.prepare_forward(x, w, a, b, ad, routing)
    y = prep.new_output()
    prep.launch(y, nat.LF_STAGE_SHRINK)
    prep.launch(y, nat.LF_STAGE_EXPAND)
    _check(y, case["y"], BF16_TOL, "forward, K-split small problem")
    y0 = prep.new_output()
    prep.launch(y0, nat.LF_STAGE_BASE)
    _check(y0, case["x"] @ case["w"].T, BF16_TOL, "base GEMM, K-split small problem")
    assert nat.device_error() == 0


def test_host_forward_streams_chunks_bit_exact():
    """fused_lora_forward_host (pinned host batch, row chunks, copies overlapped) equals one
    fused_lora_forward over the whole batch bit for bit; routes cross chunk boundaries."""
    ops = _ops()
    routes = _routes_from_sizes([700, 3, 281, 1000, 57, 259], [0, 1, 2, 0, 3, 1])  # 2300 rows
    case = _random_case(31, 2300, 512, 384, routes, {0: 16, 1: 8, 2: 32, 3: 16}, torch.bfloat16)
    x, w, a, b, ad, routing, _ = _to_torch(case, torch.bfloat16)
    ref = ops.fused_lora_forward(x, w, a, b, ad, routing)
    x_host = x.cpu().pin_memory()
    for chunk in (256, 1024, 4096):
        y = ops.fused_lora_forward_host(x_host, w, a, b, ad, routing, chunk_rows=chunk)
        torch.cuda.current_stream().synchronize()
        assert not y.is_cuda and torch.equal(y, ref.cpu()), chunk
    out = torch.empty((2300, 384), dtype=torch.bfloat16).pin_memory()
    assert ops.fused_lora_forward_host(x_host, w, a, b, ad, routing, out=out) is out
    torch.cuda.current_stream().synchronize()
    assert torch.equal(out, ref.cpu())
    with pytest.raises(ValueError):
        ops.fused_lora_forward_host(x_host, w, a, b, ad, routing, chunk_rows=100)
    with pytest.raises(ValueError):
        ops.fused_lora_forward_host(x, w, a, b, ad, routing)
    _check(ref, case["y"], BF16_TOL, "forward")


@pytest.mark.parametrize("dtype,K", [(torch.float32, 96), (torch.float16, 50)], ids=["f32", "f16_ragged_k"])
def test_host_forward_other_dtypes_and_cuda_core_path(dtype, K):
    """The host-streamed forward in float32 and with a K the tensor-core path cannot address
    (CUDA-core kernels): chunk results equal the whole-batch forward and match the oracle."""
    ops = _ops()
    routes = _routes_from_sizes([300, 1, 400, 99], [1, 0, 1, 2])  # 800 rows
    case = _random_case(37, 800, K, 136, routes, {0: 4, 1: 16, 2: 8}, dtype)
    x, w, a, b, ad, routing, _ = _to_torch(case, dtype)
    ref = ops.fused_lora_forward(x, w, a, b, ad, routing)
    y = ops.fused_lora_forward_host(x.cpu().pin_memory(), w, a, b, ad, routing, chunk_rows=256)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(y, ref.cpu())
    _check(y, case["y"], FP32_TOL if dtype == torch.float32 else BF16_TOL, "host forward")


def test_backward_reuses_forward_s_only_for_unchanged_inputs():
    """The backward takes S_f = s x A^T from a forward on the very same x and A (fewer launches,
    same gradients as recomputing it) and recomputes it once x has changed in place."""
    ops = _ops()
    routes = _routes_from_sizes([300, 5, 1, 94, 200, 100, 324], [0, 1, 2, 3, 0, 1, 2])
    case = _random_case(41, 1024, 512, 768, routes, {0: 16, 1: 8, 2: 32, 3: 16}, torch.bfloat16)
    x, w, a, b, ad, routing, g = _to_torch(case, torch.bfloat16)
    ops.clear_weight_cache()
    ref = ops.fused_lora_backward(g, x, w, a, b, ad, routing)  # no forward yet: computes S_f itself
    n_plain = ops.last_launch_count()
    ops.fused_lora_forward(x, w, a, b, ad, routing)
    got = ops.fused_lora_backward(g, x, w, a, b, ad, routing)  # reuses the forward's S_f
    assert ops.last_launch_count() <= n_plain
    for r_t, g_t in zip((ref[0],), (got[0],)):
        _check(g_t, r_t.float().cpu().numpy(), BF16_TOL, "grad_x")
    for k in ref[1]:
        _check(got[1][k], ref[1][k].float().cpu().numpy(), BF16_TOL, f"grad_a[{k}]")
        _check(got[2][k], ref[2][k].float().cpu().numpy(), BF16_TOL, f"grad_b[{k}]")
        _check(got[2][k], case["gb"][k], BF16_TOL, f"grad_b[{k}] vs oracle")
    # x changes in place after the forward: its saved S_f must not be used
    ops.fused_lora_forward(x, w, a, b, ad, routing)
    x.mul_(-1.0)
    gx2, ga2, gb2 = ops.fused_lora_backward(g, x, w, a, b, ad, routing)
    neg = _oracle_outputs(dict(case, x=-case["x"]))
    for k in neg["gb"]:
        _check(gb2[k], neg["gb"][k], BF16_TOL, f"grad_b[{k}] after x changed")
        _check(ga2[k], neg["ga"][k], BF16_TOL, f"grad_a[{k}] after x changed")
    from lorafusion_b200 import _native as nat
    assert nat.device_error() == 0


@pytest.mark.parametrize("reuse_sf", [False, True], ids=["s_f_recomputed", "s_f_from_forward"])
def test_float32_adapter_gradients(reuse_sf):
    """grad_dtype=torch.float32: the adapter gradients come back in float32 (unrounded sums, what a
    multi-GPU caller all-reduces) and match the oracle; grad_x stays bf16 and equals the default
    call's bit for bit; bf16 rounding of the float32 blocks equals the default call's blocks."""
    ops = _ops()
    routes = _routes_from_sizes([300, 5, 1, 94, 200, 100, 324], [0, 1, 2, 3, 0, 1, 2])
    case = _random_case(47, 1024, 512, 768, routes, {0: 16, 1: 8, 2: 32, 3: 64}, torch.bfloat16)
    x, w, a, b, ad, routing, g = _to_torch(case, torch.bfloat16)
    ops.clear_weight_cache()
    if reuse_sf:
        ops.fused_lora_forward(x, w, a, b, ad, routing)
    gx32, ga32, gb32 = ops.fused_lora_backward(g, x, w, a, b, ad, routing, grad_dtype=torch.float32)
    if reuse_sf:
        ops.fused_lora_forward(x, w, a, b, ad, routing)
    gx, ga, gb = ops.fused_lora_backward(g, x, w, a, b, ad, routing)
    assert gx32.dtype == torch.bfloat16 and torch.equal(gx32, gx)
    for k in case["grad_keys"]:
        assert ga32[k].dtype == torch.float32 and gb32[k].dtype == torch.float32
        assert ga32[k].shape == ga[k].shape and gb32[k].shape == gb[k].shape
        _check(ga32[k], case["ga"][k], BF16_TOL, f"grad_a[{k}]")
        _check(gb32[k], case["gb"][k], BF16_TOL, f"grad_b[{k}]")
        assert torch.equal(ga32[k].bfloat16(), ga[k]) and torch.equal(gb32[k].bfloat16(), gb[k])
    with pytest.raises(ValueError):
        ops.fused_lora_backward(g, x, w, a, b, ad, routing, grad_dtype=torch.float16)


def test_cuda_core_path_warns_for_bf16():
    """A bf16 problem TMA cannot address (K not a multiple of 8) runs on CUDA cores with a
    CudaCorePathWarning, and still matches the oracle."""
    ops = _ops()
    routes = _routes_from_sizes([40, 27], [0, 1])
    case = _random_case(53, 67, 60, 72, routes, {0: 16, 1: 8}, torch.bfloat16)
    x, w, a, b, ad, routing, g = _to_torch(case, torch.bfloat16)
    ops._WARNED_SHAPES.clear()
    with pytest.warns(ops.CudaCorePathWarning):
        y = ops.fused_lora_forward(x, w, a, b, ad, routing)
    _check(y, case["y"], BF16_TOL, "forward")


@pytest.mark.parametrize("order", ["shrink_gx_gab", "shrink_gab_gx", "all_at_once"])
def test_backward_stages_match_oracle(order):
    """lf_backward_stages: routed shrinks, grad_x GEMM and dA/dB grams as launches of their own, in
    either order after the shrinks, match the oracle (float32 adapter gradients)."""
    from lorafusion_b200 import _native as nat
    ops = _ops()
    routes = _routes_from_sizes([300, 5, 1, 94, 200, 100, 324], [0, 1, 2, 3, 0, 1, 2])
    case = _random_case(59, 1024, 512, 768, routes, {0: 16, 1: 8, 2: 32, 3: 64}, torch.bfloat16)
    x, w, a, b, ad, routing, g = _to_torch(case, torch.bfloat16)
    prep = ops.prepare_backward(g, x, w, a, b, ad, routing, grad_dtype=torch.float32)
    SH, GX, GAB = nat.LF_BSTAGE_SHRINK, nat.LF_BSTAGE_GRAD_X, nat.LF_BSTAGE_GRAD_AB
    seq = {"shrink_gx_gab": [SH, GX, GAB], "shrink_gab_gx": [SH, GAB, GX], "all_at_once": [SH | GX | GAB]}[order]
    for st in seq:
        prep.launch(st)
    gx, ga, gb = prep.grads()
    _check(gx, case["gx"], BF16_TOL, "grad_x")
    assert list(ga) == case["grad_keys"]
    for k in case["grad_keys"]:
        assert ga[k].dtype == torch.float32
        _check(ga[k], case["ga"][k], BF16_TOL, f"grad_a[{k}]")
        _check(gb[k], case["gb"][k], BF16_TOL, f"grad_b[{k}]")
    assert nat.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32], ids=["bf16", "f16", "f32"])
def test_ranks_above_64_match_oracle(dtype):
    """Adapters of rank 65 and 130 (carried as virtual slots of at most 64 ranks over the same rows)
    beside a rank-16 one: forward and backward match the oracle; gradient shapes are the adapters'
    own [r, K] / [N, r], contiguous."""
    routes = _routes_from_sizes([200, 130, 3, 267], [0, 1, 2, 1])
    case = _random_case(61, 600, 256, 320, routes, {0: 65, 1: 130, 2: 16}, dtype)
    _run_and_compare(case, dtype, FP32_TOL if dtype == torch.float32 else BF16_TOL)
    from lorafusion_b200 import _native as nat
    assert nat.device_error() == 0
