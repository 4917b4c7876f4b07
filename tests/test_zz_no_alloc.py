"""tmoe_mul_mat_id_noalloc (the allocation-free variant of tmoe_mul_mat_id, scratch in a static
device array) against tmoe_mul_mat_id on the same inputs, through the C ABI.  Collected last (the
file name) so that it also runs after everything else has used the library on this device."""
import ctypes as C

import numpy as np
import pytest
import torch

import oracle as O
import tetraeder_b200 as tb
from tests.common import XorShift, make_ids

pytestmark = pytest.mark.gpu


def _call(layer, fn, qt, W, b, ids, out):
    n_w, N, rs = W.shape
    T, b1, K = b.shape
    n_used = ids.shape[1]
    return getattr(layer.lib, fn)(layer.h, None, qt, C.c_void_p(W.data_ptr()), rs, N * rs, K, N, n_w,
                                  C.c_void_p(b.data_ptr()), b1, C.c_void_p(ids.data_ptr()), n_used, T,
                                  C.c_void_p(out.data_ptr()))


@pytest.mark.parametrize("qt", [O.TYPE_Q4_K, O.TYPE_Q6_K])
@pytest.mark.parametrize("tokens,b1_used", [(1, False), (16, True), (64, False)])
def test_noalloc_matches_mul_mat_id_twice(qt, tokens, b1_used):
    K, N, E, used = 512, 64, 16, 4
    rng = XorShift(0x5EED ^ (qt * 100 + tokens))
    W = torch.from_numpy(O.quantize(qt, rng.f32(E * N * K).reshape(E, N, K))).cuda()
    b1 = used if b1_used else 1
    b = torch.from_numpy(rng.f32(tokens * b1 * K).reshape(tokens, b1, K)).cuda()
    layer = tb.MoeLayer(512, 256, E, used, max_tokens=tokens)
    for call in range(2):  # two calls in a row, different ids (30% of them -1)
        ids = torch.from_numpy(make_ids(rng, E, used, tokens, 30)).cuda()
        want = torch.full((tokens, used, N), float("nan"), device="cuda")
        got = torch.full((tokens, used, N), float("nan"), device="cuda")
        assert _call(layer, "tmoe_mul_mat_id", qt, W, b, ids, want) == 0
        rc = _call(layer, "tmoe_mul_mat_id_noalloc", qt, W, b, ids, got)
        assert rc == 0, layer.lib.tmoe_last_error(layer.h)
        layer.check()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        idn = ids.cpu().numpy()
        assert np.all(g[idn < 0] == 0.0), f"call {call}: rows of id -1 must be exactly zero"
        scale = max(float(np.abs(w).max()), 1e-6)
        assert float(np.abs(g - w).max()) / scale <= 1e-4, f"call {call}"
    layer.close()


def test_noalloc_rejects_calls_beyond_its_scratch():
    K, N, E, used, T = 8192, 16, 2, 8, 512  # 512 rows x 8 KiB of Q8_K rows > 2 MiB
    layer = tb.MoeLayer(512, 256, 16, used, max_tokens=8)
    W = torch.zeros((E, N, O.row_size(O.TYPE_Q4_K, K)), dtype=torch.uint8, device="cuda")
    b = torch.zeros((T, 1, K), device="cuda")
    ids = torch.zeros((T, used), dtype=torch.int32, device="cuda")
    out = torch.empty((T, used, N), device="cuda")
    rc = _call(layer, "tmoe_mul_mat_id_noalloc", O.TYPE_Q4_K, W, b, ids, out)
    assert tb._lib.ERRORS.get(rc) == "TMOE_E_INVALID"
    assert b"scratch" in layer.lib.tmoe_last_error(layer.h)
    layer.close()


def _scratch_bytes(rows, K, P, qt):
    """The scratch size the header states for one call (five parts rounded up to 256 bytes, plus
    25,344 bytes of per-slot tables and counters)."""
    al = lambda v: (v + 255) // 256 * 256
    nbw = 2 if qt == O.TYPE_Q4_K else 4
    nb = K // 256
    return al(rows * K) + al(rows * nb * 4) + 2 * al(rows * nb * nbw * 4) + al(P * 4 + 16) + 25344


def test_noalloc_accepts_the_largest_call_that_fits_and_rejects_the_next():
    K, N, E, used = 2048, 16, 16, 8
    T = 1
    while _scratch_bytes(T + 1, K, (T + 1) * used, O.TYPE_Q4_K) <= 2 << 20:
        T += 1
    rng = XorShift(0xB0B)
    W = torch.from_numpy(O.quantize(O.TYPE_Q4_K, rng.f32(E * N * K).reshape(E, N, K))).cuda()
    layer = tb.MoeLayer(K, 768, E, used, max_tokens=T + 1)
    b = torch.from_numpy(rng.f32((T + 1) * K).reshape(T + 1, 1, K)).cuda()
    ids = torch.from_numpy(make_ids(rng, E, used, T + 1, 10)).cuda()
    for call in range(2):
        want = torch.full((T, used, N), float("nan"), device="cuda")
        got = torch.full((T, used, N), float("nan"), device="cuda")
        assert _call(layer, "tmoe_mul_mat_id", O.TYPE_Q4_K, W, b[:T], ids[:T], want) == 0
        rc = _call(layer, "tmoe_mul_mat_id_noalloc", O.TYPE_Q4_K, W, b[:T], ids[:T], got)
        assert rc == 0, layer.lib.tmoe_last_error(layer.h)
        layer.check()
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert float(np.abs(g - w).max()) / max(float(np.abs(w).max()), 1e-6) <= 1e-4, f"call {call} at T={T}"
    out = torch.empty((T + 1, used, N), device="cuda")
    rc = _call(layer, "tmoe_mul_mat_id_noalloc", O.TYPE_Q4_K, W, b, ids, out)
    assert tb._lib.ERRORS.get(rc) == "TMOE_E_INVALID", f"T={T + 1} must not fit"
    assert f"needs {_scratch_bytes(T + 1, K, (T + 1) * used, O.TYPE_Q4_K)} bytes".encode() in \
        layer.lib.tmoe_last_error(layer.h)
    layer.close()
