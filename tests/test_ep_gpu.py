"""The reference's EP mode on GPUs: two ranks (processes, one GPU each) hold half of the experts
each, run tmoe_ep_layer (local experts + NCCL all-reduce), and must agree with the one-rank oracle
layer: ids bit-exact, outputs within the strict bound.  Needs two GPUs (skipped otherwise)."""
import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle as O
from tests.common import maxabs_over_rms, nrms, quantized_experts

pytestmark = pytest.mark.gpu

needs_two = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                               reason="needs two GPUs")


def _case(H, I, E, T, seed):
    rng = np.random.default_rng(seed)
    gate = quantized_experts(rng, O.TYPE_Q4_K, E, I, H, exact=False)
    up = quantized_experts(rng, O.TYPE_Q4_K, E, I, H, exact=False)
    down = quantized_experts(rng, O.TYPE_Q6_K, E, H, I, exact=False)
    rw = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float32)
    return gate, up, down, rw, x


def _rank(rank, world, uid, shape, q):
    import tetraeder_b200 as tb
    from tetraeder_b200 import moe
    H, I, E, k, T, seed = shape
    torch.cuda.set_device(rank)
    gate, up, down, rw, x = _case(H, I, E, T, seed)
    per = E // world
    sl = slice(rank * per, (rank + 1) * per)
    cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    layer = tb.MoeLayer(H, I, E, k, gate_type=O.TYPE_Q4_K, up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q6_K,
                        max_tokens=T, device=rank)
    comm = moe.EPComm(uid, world, rank, device=rank, timeout_s=120.0)
    try:
        table = torch.tensor(moe.ep_id_map(E, world, rank), dtype=torch.int32, device="cuda")
        ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
        out = moe.ep_moe_ffn(layer, comm, cu(x), moe.ExpertWeights(cu(gate[sl]), cu(up[sl]), cu(down[sl])), table,
                             router_w=cu(rw), ids_out=ids)
        for _ in range(2):  # the same call again: counters and buffers are reused between calls
            out = moe.ep_moe_ffn(layer, comm, cu(x), moe.ExpertWeights(cu(gate[sl]), cu(up[sl]), cu(down[sl])),
                                 table, router_w=cu(rw), ids_out=ids, out=out)
        torch.cuda.synchronize()
        layer.check()
        q.put((rank, out.cpu().numpy(), ids.cpu().numpy()))
    finally:
        comm.close()
        layer.close()


@needs_two
@pytest.mark.parametrize("shape", [(512, 256, 16, 4, 32, 5), (2048, 768, 128, 8, 64, 6)])
def test_ep_layer_two_ranks_equals_one(shape):
    from tetraeder_b200 import moe
    H, I, E, k, T, seed = shape
    world = 2
    uid = moe.EPComm.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, uid, shape, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    gate, up, down, rw, x = _case(H, I, E, T, seed)
    want, want_ids, _ = O.layer(x, k, gate, up, down, H, I, E, router_w=rw, gate_type=O.TYPE_Q4_K,
                                up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q6_K)
    for rank, out, ids in res:
        assert np.array_equal(ids, want_ids), f"rank {rank}: routing differs"
        n, m = nrms(out, want), maxabs_over_rms(out, want)
        assert n <= 1e-3 and m <= 1e-2, f"rank {rank}: nrms={n:.2e} maxabs/rms={m:.2e}"


def _rank_a2a(rank, world, uid, shape, q):
    import tetraeder_b200 as tb
    from tetraeder_b200 import moe
    H, I, E, k, T, seed = shape  # T: tokens per rank
    torch.cuda.set_device(rank)
    gate, up, down, rw, x = _case(H, I, E, world * T, seed)
    per = E // world
    sl = slice(rank * per, (rank + 1) * per)
    cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    layer = tb.MoeLayer(H, I, E, k, gate_type=O.TYPE_Q4_K, up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q6_K,
                        max_tokens=world * T, device=rank)
    comm = moe.EPComm(uid, world, rank, device=rank, timeout_s=120.0)
    try:
        wts = moe.ExpertWeights(cu(gate[sl]), cu(up[sl]), cu(down[sl]))
        xs = cu(x[rank * T:(rank + 1) * T])
        ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
        out = moe.ep_a2a_moe_ffn(layer, comm, xs, wts, router_w=cu(rw), ids_out=ids)
        for _ in range(2):  # again: the exchange buffers are reused between calls
            out = moe.ep_a2a_moe_ffn(layer, comm, xs, wts, router_w=cu(rw), ids_out=ids, out=out)
        torch.cuda.synchronize()
        layer.check()
        q.put((rank, out.cpu().numpy(), ids.cpu().numpy()))
    finally:
        comm.close()
        layer.close()


@needs_two
@pytest.mark.parametrize("shape", [(512, 256, 16, 4, 32, 7), (2048, 768, 128, 8, 64, 8), (512, 256, 16, 4, 512, 9)],
                         ids=["tiny", "30B decode", "tiny large-batch"])
def test_ep_a2a_two_ranks_equal_the_one_rank_layer(shape):
    """Mode B: each rank holds half of the tokens of a global batch and half of the experts; the
    tokens of each rank must come out as the one-rank oracle layer computes them."""
    from tetraeder_b200 import moe
    H, I, E, k, T, seed = shape
    world = 2
    uid = moe.EPComm.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_a2a, args=(r, world, uid, shape, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    gate, up, down, rw, x = _case(H, I, E, world * T, seed)
    want, want_ids, _ = O.layer(x, k, gate, up, down, H, I, E, router_w=rw, gate_type=O.TYPE_Q4_K,
                                up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q6_K)
    for rank, out, ids in res:
        rows = slice(rank * T, (rank + 1) * T)
        assert np.array_equal(ids, want_ids[rows]), f"rank {rank}: routing differs"
        n, m = nrms(out, want[rows]), maxabs_over_rms(out, want[rows])
        bound = (1e-3, 2.5e-2) if T * world * k >= 4096 else (1e-3, 1e-2)
        assert n <= bound[0] and m <= bound[1], f"rank {rank}: nrms={n:.2e} maxabs/rms={m:.2e}"


def _rank_a2a_silent_peer(rank, world, uid, done, q):
    """Both ranks make one all-to-all call; then rank 0 calls again and rank 1 does not.  Rank 1
    keeps its handle (rank 0 writes into its buffers) until rank 0 has finished."""
    import os
    import time
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import tetraeder_b200 as tb
    from tetraeder_b200 import moe
    H, I, E, k, T, seed = 512, 256, 16, 4, 32, 11
    torch.cuda.set_device(rank)
    gate, up, down, rw, x = _case(H, I, E, world * T, seed)
    per = E // world
    sl = slice(rank * per, (rank + 1) * per)
    cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    layer = tb.MoeLayer(H, I, E, k, gate_type=O.TYPE_Q4_K, up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q6_K,
                        max_tokens=world * T, device=rank)
    comm = moe.EPComm(uid, world, rank, device=rank, timeout_s=60.0)
    try:
        wts = moe.ExpertWeights(cu(gate[sl]), cu(up[sl]), cu(down[sl]))
        xs = cu(x[rank * T:(rank + 1) * T])
        out = moe.ep_a2a_moe_ffn(layer, comm, xs, wts, router_w=cu(rw))
        torch.cuda.synchronize()
        layer.check()
        if rank == 0:
            t0 = time.monotonic()
            err = None
            try:
                moe.ep_a2a_moe_ffn(layer, comm, xs, wts, router_w=cu(rw), out=out)  # rank 1 never answers
                layer.check()
            except tb.TmoeError as e:
                err = str(e)
            dt = time.monotonic() - t0
            if err and "TMOE_E_COMM" in err:  # the NCCL exchange (buffers not mapped): its own deadline
                err = None
            # the context is still usable: a plain one-rank layer call on the same handle
            solo = tb.MoeLayer(H, I, E, k, gate_type=O.TYPE_Q4_K, up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q6_K,
                               max_tokens=T, device=rank)
            full = moe.ExpertWeights(cu(gate), cu(up), cu(down))
            solo.moe_ffn(xs, full, router_w=cu(rw))
            solo.check()
            solo.close()
            q.put((rank, err, dt))
            done.set()
        else:
            done.wait(timeout=120)
            q.put((rank, None, 0.0))
    finally:
        comm.close()
        layer.close()


@needs_two
def test_ep_a2a_silent_peer_ends_in_a_bounded_wait():
    """The exchange over peer memory waits for each peer's messages with a bounded device wait: a
    peer that never answers makes the wait run out (about 1 s per direction), the error is latched
    and reported by check(), and the GPU context stays usable.  No kernel faults or hangs; the
    failure is a rank that does not make the call (NVLS is off)."""
    from tetraeder_b200 import moe
    world = 2
    uid = moe.EPComm.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    done = ctx.Event()
    procs = [ctx.Process(target=_rank_a2a_silent_peer, args=(r, world, uid, done, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict((r, (e, dt)) for r, e, dt in (q.get(timeout=300) for _ in range(world)))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    err, dt = res[0]
    if err is None:
        pytest.skip("the ranks exchanged through NCCL (the peers' buffers could not be mapped)")
    assert "TMOE_E_DEVICE" in err or "timeout" in err.lower(), err
    assert 1.5 < dt < 30.0, dt
