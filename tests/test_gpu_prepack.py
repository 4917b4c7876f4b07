"""Q6_K expert tensors repacked by tmoe_prepack (TMOE_TYPE_Q6_K_R8) on the GPU: the device's bytes
equal the numpy restatement of the layout, and every product over the packed tensors is bit for bit
the product over the Q6_K tensors they came from (the decode GEMV in one- and two-group passes, the
gate/up GEMV, the large-batch path's f16 dequantisation, mul_mat_id), which the parity tests hold to
the oracle; one case is also held to the oracle directly."""
import zlib

import numpy as np
import pytest
import torch

import oracle as O
import tetraeder_b200 as tb
from tetraeder_b200 import moe
from tests.common import XorShift, make_ids, quantized_experts, q6r_pack
from tests.test_gpu_parity import _layer_case, assert_close, cuda, host

pytestmark = pytest.mark.gpu
R8 = moe.TYPE_Q6_K_R8


@pytest.mark.parametrize("n,rows,nb,row_pad,mat_pad", [(3, 64, 3, 0, 0), (2, 2048, 3, 0, 0), (4, 32, 6, 0, 0),
                                                       (3, 40, 2, 14, 0), (2, 16, 1, 0, 48)])
def test_prepack_bytes_equal_the_numpy_layout(n, rows, nb, row_pad, mat_pad):
    rng = np.random.default_rng(n * 100 + rows + nb)
    rb = nb * 210
    W = rng.integers(0, 256, (n, rows, rb), dtype=np.uint8)
    # the source with padded rows / matrices (nb1 > row size, nb2 > rows * nb1)
    nb1 = rb + row_pad
    nb2 = rows * nb1 + mat_pad
    src = np.zeros(n * nb2 + 16, np.uint8)
    for m in range(n):
        for r in range(rows):
            src[m * nb2 + r * nb1:m * nb2 + r * nb1 + rb] = W[m, r]
    s = cuda(src)
    out = torch.empty((n, rows, rb), dtype=torch.uint8, device="cuda")
    lib = tb._lib.load()
    tb._lib.check(lib.tmoe_prepack(moe.TYPE_Q6_K, moe._ptr(s), nb1, nb2, rows, nb * 256, n, moe._ptr(out),
                                   moe._stream(None)), None)
    torch.cuda.synchronize()
    assert np.array_equal(host(out), q6r_pack(W))
    if row_pad == 0 and mat_pad == 0:
        assert np.array_equal(host(moe.prepack(cuda(W))), q6r_pack(W))


def _run(H, I, E, k, T, gt, dt, gate, up, down, rw, x):
    layer = tb.MoeLayer(H, I, E, k, gate_type=gt, up_type=gt, down_type=dt, max_tokens=T)
    wts = tb.ExpertWeights(gate, up, down)
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    out = layer.moe_ffn(cuda(x), wts, router_w=cuda(rw), ids_out=ids, w_out=w)
    layer.check()
    res = host(out), host(ids), host(w)
    layer.close()
    return res


PACKED_CASES = [
    # (name, H, I, E, k, T, gate/up type, pack gate/up too): one-group passes (T = 1, 64), two-group
    # passes (T = 512), the large-batch path's dequantisation (T = 1024: 8192 pairs), Q6_K gate/up
    ("C2 T=1", 2048, 768, 128, 8, 1, O.TYPE_Q4_K, False),
    ("C2 T=64", 2048, 768, 128, 8, 64, O.TYPE_Q4_K, False),
    ("C2 T=512", 2048, 768, 128, 8, 512, O.TYPE_Q4_K, False),
    ("C2 T=1024 large batch", 2048, 768, 128, 8, 1024, O.TYPE_Q4_K, False),
    ("235B-shaped K=1536 T=64", 4096, 1536, 16, 8, 64, O.TYPE_Q4_K, False),
    ("tiny Q6_K gate/up T=4", 512, 256, 16, 4, 4, O.TYPE_Q6_K, True),
    ("tiny Q6_K gate/up T=256", 512, 256, 16, 4, 256, O.TYPE_Q6_K, True),
]


@pytest.mark.parametrize("case", PACKED_CASES, ids=[c[0] for c in PACKED_CASES])
def test_layer_over_packed_tensors_is_bitwise_the_q6k_layer(case):
    name, H, I, E, k, T, gt, pack_gu = case
    gate, up, down, rw, x = _layer_case(H, I, E, k, T, gt, O.TYPE_Q6_K, zlib.crc32(name.encode()) & 0xffff,
                                        exact=False)
    g, u, d = cuda(gate), cuda(up), cuda(down)
    want = _run(H, I, E, k, T, gt, O.TYPE_Q6_K, g, u, d, rw, x)
    gp, up_ = (moe.prepack(g), moe.prepack(u)) if pack_gu else (g, u)
    got = _run(H, I, E, k, T, R8 if pack_gu else gt, R8, gp, up_, moe.prepack(d), rw, x)
    for a, b in zip(got, want):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), name


def test_layer_over_packed_down_matches_the_oracle():
    H, I, E, k, T = 2048, 768, 128, 8, 16
    gate, up, down, rw, x = _layer_case(H, I, E, k, T, O.TYPE_Q4_K, O.TYPE_Q6_K, 1616, exact=False)
    out, ids, w = _run(H, I, E, k, T, O.TYPE_Q4_K, R8, cuda(gate), cuda(up), moe.prepack(cuda(down)), rw, x)
    want_ids, want_w, _, _ = O.route(x, k, router_w=rw)
    assert np.array_equal(ids, want_ids) and np.array_equal(w.view(np.uint32), want_w.view(np.uint32))
    want = O.experts(x, want_ids, want_w, gate, up, down, H, I, E, O.TYPE_Q4_K, O.TYPE_Q4_K, O.TYPE_Q6_K)
    assert_close(out, want, what="packed down")


@pytest.mark.parametrize("tokens", [1, 64, 512])
def test_mul_mat_id_over_packed_tensors_is_bitwise_q6k(tokens):
    K, N, E, used = 512, 64, 16, 4
    rng = XorShift(0x51ED27 ^ tokens)
    W = quantized_experts(np.random.default_rng(tokens), O.TYPE_Q6_K, E, N, K, exact=False)
    b = rng.f32(tokens * used * K).reshape(tokens, used, K)
    ids = make_ids(rng, E, used, tokens, 30)
    layer = tb.MoeLayer(512, 256, E, used, max_tokens=tokens)
    Wd, bd, idd = cuda(W), cuda(b), cuda(ids)
    want = host(layer.mul_mat_id(O.TYPE_Q6_K, Wd, bd, idd))
    got = host(layer.mul_mat_id(R8, moe.prepack(Wd), bd, idd))
    layer.check()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.all(got[ids < 0] == 0.0)
