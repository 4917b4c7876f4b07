"""Failure detection without a GPU fault.

The reference's executor turns a failed step into an error on every rank instead of a hang
(crates/executor/src/exec.rs:164-177).  Here the same rule holds on the device and on the
communicator:

  - a bounded device wait on a flag that nothing sets gives up after its limit, latches the
    handle's error flag and lets the stream go on: the next check() raises TMOE_E_DEVICE, and the
    same handle then computes a layer correctly (the context stayed usable);
  - the same wait ends normally when the host releases the flag (pinned, device-mapped memory);
  - a communicator whose second rank never joins ends tmoe_comm_init with TMOE_E_COMM within its
    deadline (the communicator is aborted), in a child process with NVLS off.

Nothing here faults, traps or hangs a GPU: the waits are bounded and nothing waits on another
kernel of the same device."""
import multiprocessing
import os
import threading
import time

import numpy as np
import pytest
import torch

import oracle as O
import tetraeder_b200 as tb
from tests.common import maxabs_over_rms, nrms

pytestmark = pytest.mark.gpu


def _tiny_layer_check(layer):
    H, I, E, k, T = 512, 256, 16, 4, 8
    rng = np.random.default_rng(4)
    gate = O.quantize(O.TYPE_Q4_K, (rng.standard_normal((E, I, H)) * 0.02).astype(np.float32))
    up = O.quantize(O.TYPE_Q4_K, (rng.standard_normal((E, I, H)) * 0.02).astype(np.float32))
    down = O.quantize(O.TYPE_Q4_K, (rng.standard_normal((E, H, I)) * 0.02).astype(np.float32))
    rw = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float32)
    cu = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    out = layer.moe_ffn(cu(x), tb.ExpertWeights(cu(gate), cu(up), cu(down)), router_w=cu(rw))
    layer.check()
    ids, w, _, _ = O.route(x, k, router_w=rw)
    want = O.experts(x, ids, w, gate, up, down, H, I, E)
    got = out.cpu().numpy()
    assert nrms(got, want) <= 1e-3 and maxabs_over_rms(got, want) <= 1e-2


def _layer():
    return tb.MoeLayer(512, 256, 16, 4, gate_type=O.TYPE_Q4_K, up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q4_K,
                       max_tokens=8)


def test_bounded_device_wait_runs_out_and_the_context_stays_usable():
    layer = _layer()
    try:
        flag = torch.zeros(1, dtype=torch.int32, device="cuda")  # nothing ever sets it to 1
        torch.cuda.synchronize()
        t0 = time.monotonic()
        layer.wait_flag(flag, 1, limit_ns=2_000_000)  # 2 ms
        with pytest.raises(tb.TmoeError, match="TMOE_E_DEVICE") as exc:
            layer.check()
        elapsed = time.monotonic() - t0
        assert "bounded wait" in str(exc.value)
        assert elapsed < 0.5, f"the 2 ms wait took {elapsed:.3f} s to give up"
        layer.check()  # the flag was read and cleared
        _tiny_layer_check(layer)  # the same handle and context compute correctly afterwards
    finally:
        layer.close()


def test_bounded_device_wait_ends_when_the_host_releases_the_flag():
    layer = _layer()
    try:
        flag = torch.zeros(1, dtype=torch.int32).pin_memory()
        layer.wait_flag(flag, 7, limit_ns=0)  # the default limit, one second
        layer.wait_flag(torch.full((1,), 3, dtype=torch.int32, device="cuda"), 3)  # already equal
        t0 = time.monotonic()
        releaser = threading.Timer(0.05, lambda: flag.fill_(7))
        releaser.start()
        layer.check()  # returns once the stream has passed the wait, with no error latched
        elapsed = time.monotonic() - t0
        releaser.join()
        assert 0.03 <= elapsed < 0.9, f"released after 50 ms, the stream waited {elapsed:.3f} s"
        with pytest.raises(tb.TmoeError, match="TMOE_E_INVALID"):
            layer.wait_flag(torch.zeros(2, dtype=torch.int32)[1:], 1)  # pageable host memory
    finally:
        layer.close()


def _lonely_rank(q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import tetraeder_b200 as tb_
    from tetraeder_b200 import moe
    torch.cuda.set_device(0)
    uid = moe.EPComm.unique_id()
    t0 = time.monotonic()
    try:
        moe.EPComm(uid, 2, 0, device=0, timeout_s=3.0)  # rank 1 never calls
        q.put(("joined", time.monotonic() - t0))
    except tb_.TmoeError as e:
        q.put((str(e), time.monotonic() - t0))


def test_comm_init_ends_with_an_error_when_a_rank_never_joins():
    ctx = multiprocessing.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely_rank, args=(q,))
    p.start()
    try:
        msg, elapsed = q.get(timeout=120)
    finally:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
            p.join()
    assert msg.startswith("TMOE_E_COMM"), msg
    assert elapsed < 30, f"init gave up after {elapsed:.1f} s against a 3 s deadline"
