"""The dA/dB kernel's own exchange of spanning adapters' gradients across GPUs (lf_backward_peer).

One process per GPU (needs two GPUs; each rank on its own device, so the ranks' kernels that wait
for each other run on different GPUs).  Every rank takes its rows of the same global packing and
runs the backward with ``peer=PeerExchange(...)``: blocks of adapters that span both ranks are
pushed into both ranks' exchange buffers over peer mappings and summed in rank order inside the
kernel.  The parent checks every adapter's dA / dB (both ranks, identical bit for bit for spanning
adapters) and grad_x against the float64 oracle of the whole batch (mock_ops.py:88-93 sums an
adapter's gradient over all its routes), over three calls (both halves of the exchange buffers).
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
RANKS = [130, 8, 32, 16, 16, 8, 16, 4]  # adapter 0 (spans both ranks): rank 130, three virtual slots


def _global_problem():
    from oracle import mock_oracle
    from lorafusion_b200.scheduler import Request, bucket_by_adapter, greedy_pack
    reqs = [Request(i, i, c) for i, c in enumerate(COUNTS)]
    groups = bucket_by_adapter(reqs)
    packing = greedy_pack({g.adapter_id: g.total_rows for g in groups}, CAP)
    T = sum(COUNTS)
    rng = np.random.default_rng(19)
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
    peer = None
    try:
        from lorafusion_b200 import _native as nat
        from lorafusion_b200 import b200_ops
        from lorafusion_b200.config import AdapterSpec
        from lorafusion_b200.sharding import PeerExchange, assign_bins, local_layout
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        packing, x, g, w, a, b, _ = _global_problem()
        plan = assign_bins(packing.bins, world)
        rows, local = local_layout(plan, packing.bins, rank, CAP)
        t = lambda v: torch.from_numpy(np.ascontiguousarray(v)).to(dev, torch.bfloat16)  # noqa: E731
        xl, gl, wd = t(x[rows]), t(g[rows]), t(w)
        ad = {i: t(v) for i, v in a.items()}
        bd = {i: t(v) for i, v in b.items()}
        specs = {i: AdapterSpec(i, r, 2.0 * r, K, N) for i, r in enumerate(RANKS)}
        peer = PeerExchange(plan, dict(enumerate(RANKS)), dev)
        b200_ops.fused_lora_forward(xl, wd, ad, bd, specs, local)
        calls = []
        for _ in range(3):  # odd and even generations: both halves of the exchange buffers
            gx, ga, gb = b200_ops.fused_lora_backward(gl, xl, wd, ad, bd, specs, local, grad_dtype=torch.float32,
                                                      peer=peer)
            torch.cuda.synchronize()
            calls.append({"gx": gx.float().cpu().numpy(), "ga": {k: v.cpu().numpy() for k, v in ga.items()},
                          "gb": {k: v.cpu().numpy() for k, v in gb.items()}})
        result_q.put((rank, {"rows": rows, "calls": calls, "spanning": list(plan.spanning),
                             "status": nat.device_error()}))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        result_q.put((rank, repr(e)))
        raise
    finally:
        if peer is not None:
            peer.close()
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_in_kernel_exchange_matches_whole_batch_oracle(world):
    """With four ranks some spanning adapters are not held by every rank: those ranks receive the
    holders' sums without computing any block of them."""
    from oracle import mock_oracle
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"the in-kernel exchange needs one GPU per rank ({world} GPUs)")
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
    spanning = res[0]["spanning"]
    assert spanning and all(res[r]["spanning"] == spanning for r in range(world))
    packing, x, g, w, a, b, routes = _global_problem()
    f = mock_oracle.as_f64
    sc = {i: 2.0 for i in range(len(RANKS))}
    rgx, rga, rgb = mock_oracle.fused_lora_backward(f(g), f(x), f(w), f(a), f(b), sc, routes)
    tol = dict(rtol=2e-2, atol=2e-2)
    for c in range(3):
        gx = np.zeros_like(rgx)
        for r in range(world):
            gx[res[r]["rows"]] = res[r]["calls"][c]["gx"]
        ok, msg = mock_oracle.allclose_report(gx, rgx, **tol)
        assert ok, f"call {c} grad_x: {msg}"
        for aid in rga:
            holders = [r for r in range(world) if aid in res[r]["calls"][c]["ga"]]
            assert holders, aid
            if aid in spanning:
                assert holders == list(range(world))
                for key in ("ga", "gb"):  # the same sums on every rank, bit for bit
                    for r in range(1, world):
                        assert np.array_equal(res[0]["calls"][c][key][aid], res[r]["calls"][c][key][aid]), (c, key, aid)
            for r in holders:
                for name, got, ref in (("grad_a", res[r]["calls"][c]["ga"][aid], rga[aid]),
                                       ("grad_b", res[r]["calls"][c]["gb"][aid], rgb[aid])):
                    ok, msg = mock_oracle.allclose_report(got, ref, **tol)
                    assert ok, f"call {c} rank {r} {name}[{aid}]: {msg}"


def _withheld_worker(rank, world, port, result_q):
    """Call 1 on both ranks; call 2 on rank 0 only (rank 1 withholds its blocks, between steps, with
    nothing of its own in flight) under a 50 ms wait limit; call 3 on both ranks again."""
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    peer = None
    try:
        from lorafusion_b200 import _native as nat
        from lorafusion_b200 import b200_ops
        from lorafusion_b200.config import AdapterSpec
        from lorafusion_b200.sharding import PeerExchange, assign_bins, local_layout
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        packing, x, g, w, a, b, _ = _global_problem()
        plan = assign_bins(packing.bins, world)
        rows, local = local_layout(plan, packing.bins, rank, CAP)
        t = lambda v: torch.from_numpy(np.ascontiguousarray(v)).to(dev, torch.bfloat16)  # noqa: E731
        xl, gl, wd = t(x[rows]), t(g[rows]), t(w)
        ad = {i: t(v) for i, v in a.items()}
        bd = {i: t(v) for i, v in b.items()}
        specs = {i: AdapterSpec(i, r, 2.0 * r, K, N) for i, r in enumerate(RANKS)}
        peer = PeerExchange(plan, dict(enumerate(RANKS)), dev)
        b200_ops.fused_lora_forward(xl, wd, ad, bd, specs, local)

        def backward():
            _, ga, gb = b200_ops.fused_lora_backward(gl, xl, wd, ad, bd, specs, local, grad_dtype=torch.float32,
                                                     peer=peer)
            torch.cuda.synchronize()
            return {k: v.cpu().numpy() for k, v in ga.items()}, {k: v.cpu().numpy() for k, v in gb.items()}

        first = backward()
        status_first = nat.device_error()
        dist.barrier()
        code = 0
        if rank == 0:
            nat.set_wait_limit(50_000_000)
            try:
                backward()
                code = nat.device_error()  # reads and clears the code the timed-out polls recorded
            finally:
                nat.set_wait_limit(0)
        else:
            peer.next_gen()  # the generation rank 0 used alone: skipped, so the next call pairs again
        dist.barrier()
        again = backward()
        same = all(np.array_equal(first[0][k], again[0][k]) for k in first[0]) and \
            all(np.array_equal(first[1][k], again[1][k]) for k in first[1])
        result_q.put((rank, {"code": code, "status_first": status_first, "status": nat.device_error(),
                             "same": same}))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        result_q.put((rank, repr(e)))
        raise
    finally:
        if peer is not None:
            peer.close()
        dist.destroy_process_group()


def test_withheld_blocks_time_out_and_the_next_call_recovers():
    """A rank that does not take part in a call (its blocks never arrive) makes the other rank's
    polls of the exchange run out: the call returns, lf_device_error reports ERR_TIMEOUT_FLAG,
    and the next call on both ranks gives the first call's sums bit for bit."""
    from lorafusion_b200 import _native as nat
    world = 2
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip("the in-kernel exchange needs one GPU per rank (2 GPUs)")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_withheld_worker, args=(r, world, port, q)) for r in range(world)]
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
        assert res[r]["status_first"] == 0 and res[r]["status"] == 0, res[r]
        assert res[r]["same"], r
    assert res[0]["code"] == nat.ERR_TIMEOUT_FLAG, hex(res[0]["code"])
