"""The Q6_K 8-row fragment order (TMOE_TYPE_Q6_K_R8, tmoe_prepack) on the CPU: the numpy restatement
that the GPU tests hold the device's bytes to is a permutation of each 8-row group's bytes that
matches the byte map the kernels use, and the entry point's argument checks refuse bad calls before
any device work."""
import ctypes as C

import numpy as np
import pytest

from tests.common import q6r_pack, q6r_unpack
from tetraeder_b200 import _lib


def byte_map(g, off):
    """Unit offset of byte `off` of row g's ggml super-block, written out case by case."""
    if off < 128:  # ql: off = 64h + 16i + 4t4 + j
        h, i, t4, j = off // 64, (off // 16) % 4, (off // 4) % 4, off % 4
        return 768 * h + 16 * (4 * g + t4) + 4 * i + j
    if off < 192:  # qh: off - 128 = 32h + 16i + 4t4 + j
        o = off - 128
        h, i, t4, j = o // 32, (o // 16) % 2, (o // 4) % 4, o % 4
        return 768 * h + 512 + 8 * (4 * g + t4) + 4 * i + j
    if off < 208:
        return 1536 + 16 * g + off - 192
    return 1664 + 2 * g + off - 208


def test_byte_map_is_a_permutation_of_the_unit():
    assert sorted(byte_map(g, o) for g in range(8) for o in range(210)) == list(range(1680))


@pytest.mark.parametrize("nb", [1, 3, 6])
def test_numpy_packer_follows_the_byte_map(nb):
    rng = np.random.default_rng(nb)
    n, rows = 2, 16
    W = rng.integers(0, 256, (n, rows, nb * 210), dtype=np.uint8)
    P = q6r_pack(W)
    assert P.shape == W.shape and sorted(P.ravel().tolist()) == sorted(W.ravel().tolist())
    units = P.reshape(n, rows // 8, nb, 1680)
    for m in range(n):
        for r in range(rows):
            for b in range(nb):
                blk = W[m, r, 210 * b:210 * (b + 1)]
                u = units[m, r // 8, b]
                idx = [byte_map(r % 8, o) for o in range(210)]
                assert np.array_equal(u[idx], blk)


@pytest.mark.parametrize("n,rows,nb", [(1, 8, 1), (3, 64, 3), (2, 2048, 3), (2, 4096, 6)])
def test_pack_unpack_round_trip(n, rows, nb):
    """Repacking is a pure permutation within each 8-row group: unpacking gives the ggml bytes back, and a
    packed matrix differs from its source unless the group's bytes happen to be symmetric."""
    rng = np.random.default_rng(rows * 10 + nb)
    W = rng.integers(0, 256, (n, rows, nb * 210), dtype=np.uint8)
    P = q6r_pack(W)
    assert np.array_equal(q6r_unpack(P), W)
    assert not np.array_equal(P, W)
    # each 8-row group maps onto itself: the same multiset of bytes per (matrix, group)
    g = W.reshape(n, rows // 8, -1)
    assert np.array_equal(np.sort(P.reshape(n, rows // 8, -1), axis=-1), np.sort(g, axis=-1))


def test_prepack_argument_checks_without_a_gpu():
    lib = _lib.load()
    raw = np.zeros(8192, np.uint8)
    base = raw.ctypes.data + (-raw.ctypes.data) % 16  # 16-byte aligned host addresses: never dereferenced
    src, dst = C.c_void_p(base), C.c_void_p(base + 4096)

    def call(qtype, s, nb1, nb2, rows, K, mats, d):
        rc = lib.tmoe_prepack(qtype, s, nb1, nb2, rows, K, mats, d, None)
        return rc, (lib.tmoe_last_error(None) or b"").decode()

    rc, msg = call(_lib.TYPE_Q4_K, src, 144, 144 * 8, 8, 256, 1, dst)
    assert rc == _lib.TMOE_E_UNSUPPORTED and "only Q6_K" in msg
    for rows, K in ((8, 300), (12, 256), (8, 16640)):  # K not a multiple of 256 or too large; rows % 8
        rc, msg = call(_lib.TYPE_Q6_K, src, 210, 210 * rows, rows, K, 1, dst)
        assert rc == _lib.TMOE_E_INVALID and "multiple" in msg
    rc, msg = call(_lib.TYPE_Q6_K, src, 200, 210 * 8, 8, 256, 1, dst)
    assert rc == _lib.TMOE_E_INVALID and "overlap" in msg  # rows closer than a row
    rc, msg = call(_lib.TYPE_Q6_K, src, 210, 210 * 4, 8, 256, 2, dst)
    assert rc == _lib.TMOE_E_INVALID and "overlap" in msg  # matrices closer than rows * nb1
    rc, msg = call(_lib.TYPE_Q6_K, src, 210, 210 * 8, 8, 256, 1, C.c_void_p(base + 1024))
    assert rc == _lib.TMOE_E_INVALID and "src and dst overlap" in msg
    rc, msg = call(_lib.TYPE_Q6_K, src, 210, 210 * 8, 8, 256, 1, C.c_void_p(base + 4104))
    assert rc == _lib.TMOE_E_INVALID and "aligned" in msg
    rc, msg = call(_lib.TYPE_Q6_K, None, 210, 210 * 8, 8, 256, 1, dst)
    assert rc == _lib.TMOE_E_INVALID and "null" in msg
    assert call(_lib.TYPE_Q6_K, None, 210, 0, 0, 256, 0, None)[0] == _lib.TMOE_OK  # nothing to do
