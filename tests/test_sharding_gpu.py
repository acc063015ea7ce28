"""The CUDA path sharded across ranks, checked against the oracle on the whole batch.

Two processes on cuda:0 form a gloo group.  Every rank computes the same global packing, takes its
row ranges (sharding.assign_bins / local_layout), runs b200_ops forward and backward on its rows
(adapter gradients in float32) and sums the gradients of adapters that span both ranks with
sharding.allreduce_spanning_grads.  The parent puts the ranks' rows back in global order and
compares y, grad_x and every adapter's dA / dB with the float64 oracle of the whole batch under the
plain bf16 rule (mock_ops.py:88-93 sums an adapter's gradient over all its routes).

Both processes share one GPU, so co-scheduled (cooperative) launches are turned off in them: the
per-rank math under test is the same in both launch modes, which the single-process tests cover.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

K, N, CAP = 512, 384, 128
COUNTS = [1500, 420, 260, 130, 64, 33, 9, 3]
RANKS = [16, 8, 32, 16, 64, 8, 16, 4]


def _global_problem():
    from oracle import mock_oracle
    from lorafusion_b200.scheduler import Request, bucket_by_adapter, greedy_pack
    reqs = [Request(i, i, c) for i, c in enumerate(COUNTS)]
    groups = bucket_by_adapter(reqs)
    packing = greedy_pack({g.adapter_id: g.total_rows for g in groups}, CAP)
    T = sum(COUNTS)
    rng = np.random.default_rng(17)
    r16 = mock_oracle.bf16_round
    x = r16(rng.standard_normal((T, K), dtype=np.float32))
    g = r16(rng.standard_normal((T, N), dtype=np.float32))
    w = r16(rng.standard_normal((N, K), dtype=np.float32) / np.sqrt(K))
    a = {i: r16(rng.standard_normal((r, K), dtype=np.float32) / np.sqrt(K)) for i, r in enumerate(RANKS)}
    b = {i: r16(0.02 * rng.standard_normal((N, r), dtype=np.float32)) for i, r in enumerate(RANKS)}
    routes, cur = [], 0
    for entries in packing.bins:
        for aid, n in entries:
            routes.append((cur, cur + n, aid))
            cur += n
    return packing, x, g, w, a, b, routes


def _worker(rank, world, port, result_q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from lorafusion_b200 import _native as nat
        from lorafusion_b200 import b200_ops
        from lorafusion_b200.config import AdapterSpec
        from lorafusion_b200.sharding import allreduce_spanning_grads, assign_bins, local_layout
        torch.cuda.set_device(0)
        b200_ops.use_cooperative_launch(False)
        packing, x, g, w, a, b, _ = _global_problem()
        plan = assign_bins(packing.bins, world)
        rows, local = local_layout(plan, packing.bins, rank, CAP)
        dev = lambda v: torch.from_numpy(np.ascontiguousarray(v)).to("cuda", torch.bfloat16)  # noqa: E731
        xl, gl = dev(x[rows]), dev(g[rows])
        wd = dev(w)
        ad = {i: dev(v) for i, v in a.items()}
        bd = {i: dev(v) for i, v in b.items()}
        specs = {i: AdapterSpec(i, r, 2.0 * r, K, N) for i, r in enumerate(RANKS)}
        y = b200_ops.fused_lora_forward(xl, wd, ad, bd, specs, local)
        gx, ga, gb = b200_ops.fused_lora_backward(gl, xl, wd, ad, bd, specs, local, grad_dtype=torch.float32)
        allreduce_spanning_grads(plan, ga, gb, dict(enumerate(RANKS)), K, N, torch.device("cuda"))
        torch.cuda.synchronize()
        out = {"rows": rows, "y": y.float().cpu().numpy(), "gx": gx.float().cpu().numpy(),
               "ga": {k: v.float().cpu().numpy() for k, v in ga.items()},
               "gb": {k: v.float().cpu().numpy() for k, v in gb.items()},
               "spanning": list(plan.spanning), "status": nat.device_error()}
        result_q.put((rank, out))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        result_q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_cuda_path_matches_whole_batch_oracle():
    from oracle import mock_oracle
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, out = q.get(timeout=300)
            res[r] = out
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert isinstance(res[r], dict), res[r]
        assert res[r]["status"] == 0
    assert res[0]["spanning"] and res[0]["spanning"] == res[1]["spanning"]

    packing, x, g, w, a, b, routes = _global_problem()
    f = mock_oracle.as_f64
    sc = {i: 2.0 for i in range(len(RANKS))}
    ry = mock_oracle.fused_lora_forward(f(x), f(w), f(a), f(b), sc, routes)
    rgx, rga, rgb = mock_oracle.fused_lora_backward(f(g), f(x), f(w), f(a), f(b), sc, routes)
    tol = dict(rtol=2e-2, atol=2e-2)
    y = np.zeros_like(ry)
    gx = np.zeros_like(rgx)
    for r in range(world):
        y[res[r]["rows"]] = res[r]["y"]
        gx[res[r]["rows"]] = res[r]["gx"]
    assert sorted(res[0]["rows"] + res[1]["rows"]) == list(range(x.shape[0]))
    for name, got, ref in (("y", y, ry), ("grad_x", gx, rgx)):
        ok, msg = mock_oracle.allclose_report(got, ref, **tol)
        assert ok, f"{name}: {msg}"
    for aid in rga:
        holders = [r for r in range(world) if aid in res[r]["ga"]]
        assert holders, aid
        if aid in res[0]["spanning"]:
            assert holders == list(range(world))
        for r in holders:
            for name, got, ref in (("grad_a", res[r]["ga"][aid], rga[aid]), ("grad_b", res[r]["gb"][aid], rgb[aid])):
                ok, msg = mock_oracle.allclose_report(got, ref, **tol)
                assert ok, f"rank {r} {name}[{aid}]: {msg}"
