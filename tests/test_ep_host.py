"""Expert parallelism on the host (no GPU): the contiguous expert partition and the exchange of the
reference's EP mode (qwen3moe_shard.rs:1038-1056) run as two gloo ranks on CPU, the oracle standing
in for each rank's local layer.  The CUDA path does the same exchange with NCCL (test_ep_gpu.py)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O
from tetraeder_b200.moe import ep_id_map
from tests.common import nrms, quantized_experts

H, I, E, K_USED, T = 512, 256, 16, 4, 32


@pytest.mark.parametrize("n_expert,n_ranks", [(16, 1), (16, 2), (16, 4), (128, 8)])
def test_ep_id_map_partitions_contiguously(n_expert, n_ranks):
    per = n_expert // n_ranks
    seen = np.zeros(n_expert, dtype=int)
    for r in range(n_ranks):
        m = np.array(ep_id_map(n_expert, n_ranks, r))
        own = np.nonzero(m >= 0)[0]
        assert list(own) == list(range(r * per, (r + 1) * per))  # contiguous by id
        assert list(m[own]) == list(range(per))  # local slots in id order
        seen[own] += 1
    assert np.all(seen == 1)


def test_ep_id_map_rejects_uneven_split():
    with pytest.raises(ValueError):
        ep_id_map(10, 4, 0)


def _case(seed=11):
    rng = np.random.default_rng(seed)
    gate = quantized_experts(rng, O.TYPE_Q4_K, E, I, H, exact=True)
    up = quantized_experts(rng, O.TYPE_Q4_K, E, I, H, exact=True)
    down = quantized_experts(rng, O.TYPE_Q4_K, E, H, I, exact=True)
    rw = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float32)
    return gate, up, down, rw, x


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        gate, up, down, rw, x = _case()
        per = E // world
        sl = slice(rank * per, (rank + 1) * per)
        table = np.array(ep_id_map(E, world, rank), dtype=np.int32)
        part, ids, w = O.layer(x, K_USED, gate[sl], up[sl], down[sl], H, I, E, router_w=rw,
                               gate_type=O.TYPE_Q4_K, up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q4_K, id_map=table)
        t = torch.from_numpy(part.copy())
        dist.all_reduce(t, op=dist.ReduceOp.SUM)  # the reference's b.reduce
        q.put((rank, t.numpy(), ids))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_ep_allreduce_mode_equals_one_rank(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=180) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    gate, up, down, rw, x = _case()
    want, want_ids, _ = O.layer(x, K_USED, gate, up, down, H, I, E, router_w=rw, gate_type=O.TYPE_Q4_K,
                                up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q4_K)
    for rank, out, ids in res:
        assert np.array_equal(ids, want_ids), f"rank {rank}: routing differs"
        # the partial sums are added in another order than one rank's fold: float rounding only
        assert nrms(out, want) <= 1e-6, f"rank {rank}"
