"""CPU tests of the oracle (the checker of the CUDA path): pinned against gguf-py's decoders
(tests/golden/kquant_dequant.npz) and against the properties the reference's own tests assert."""
import os

import numpy as np
import pytest

import oracle as O
from tests.common import XorShift, group_pairs, make_ids, routing

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kquant_dequant.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


@pytest.mark.parametrize("name,qt,nb", [("q4_k", O.TYPE_Q4_K, 144), ("q6_k", O.TYPE_Q6_K, 210)])
def test_dequant_bit_exact_with_gguf_py(golden, name, qt, nb):
    blocks, want = golden[name + "_blocks"], golden[name + "_values"]
    got = O.dequantize(qt, blocks, blocks.shape[0] * 256).reshape(want.shape)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("name,qt,bound", [("q4_k", O.TYPE_Q4_K, 0.12), ("q6_k", O.TYPE_Q6_K, 0.03)])
def test_quantiser_round_trip(golden, name, qt, bound):
    """Our own Q4_K/Q6_K fit: the bytes are deterministic and reproduce the source closely."""
    src = golden[name + "_source"]
    q = O.quantize(qt, src)
    assert np.array_equal(q.reshape(-1), golden[name + "_blocks"][48:].reshape(-1))
    back = O.dequantize(qt, q, src.size).reshape(src.shape)
    rms = np.sqrt(np.mean(src[src != 0] ** 2))
    assert np.sqrt(np.mean((back - src) ** 2)) / rms < bound
    assert np.all(back[3] == 0.0)


def test_half_conversions():
    h = np.arange(0, 65536, 7, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([O.lib().tmo_f16_to_f32(int(v)) for v in h], dtype=np.float32)
    fin = np.isfinite(ref)
    assert np.array_equal(got[fin], ref[fin])
    rng = np.random.default_rng(3)
    vals = np.concatenate([rng.normal(0, 50, 3000), rng.normal(0, 1e-5, 3000), [65504, 65519.9, 6e-8, 3e-8]]).astype(np.float32)
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16).view(np.uint16)
    got = np.array([O.lib().tmo_f32_to_f16(float(v)) for v in vals], dtype=np.uint16)
    assert np.array_equal(got, want)


def test_q8k_quantiser_semantics():
    """ggml quantize_row_q8_K_ref: the first element of largest magnitude maps to -127, values in
    [-128, 127] (127 clamp), bsums are the 16-element sums, d = 1/iscale."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal(1024).astype(np.float32)
    x[300] = 7.0
    x[301] = -7.0  # tie in magnitude: the first one wins
    b = O.quantize_q8k(x)
    assert b[1]["qs"][300 - 256] == -127
    assert b[1]["qs"][301 - 256] == 127
    for blk in b:
        assert np.array_equal(blk["bsums"], blk["qs"].astype(np.int32).reshape(16, 16).sum(1))
    z = O.quantize_q8k(np.zeros(256, np.float32))
    assert z[0]["d"] == 0 and not z[0]["qs"].any()
    rt = O.dequantize_q8k(b)
    assert np.max(np.abs(rt - x)) <= np.max([np.abs(blk["d"]) for blk in b]) * 0.5 + 1e-7


@pytest.mark.parametrize("qt", [O.TYPE_Q4_K, O.TYPE_Q6_K])
@pytest.mark.parametrize("ncols", [256, 1536, 4096])
def test_vec_dot_within_iqk_bound(qt, ncols):
    """iqk_kernels.rs:8,128-147: against an f64 dot of dequantised weights and the Q8_K round trip
    of the activation, each output within 1e-5 * sum|w*x| + 1e-6."""
    rng = np.random.default_rng(ncols + qt)
    w = O.quantize(qt, rng.uniform(-1, 1, (24, ncols)).astype(np.float32))
    x = rng.uniform(-1, 1, ncols).astype(np.float32)
    xq = O.quantize_q8k(x)
    xd = O.dequantize_q8k(xq).astype(np.float64)
    fn = O.lib().tmo_vec_dot_q4k_q8k if qt == O.TYPE_Q4_K else O.lib().tmo_vec_dot_q6k_q8k
    for r in range(w.shape[0]):
        row = np.ascontiguousarray(w[r])
        got = fn(ncols, row.ctypes.data, xq.ctypes.data)
        wd = O.dequantize(qt, row, ncols).astype(np.float64)
        ref = float(np.dot(wd, xd))
        assert abs(got - ref) <= 1e-5 * float(np.sum(np.abs(wd * xd))) + 1e-6


@pytest.mark.parametrize("qt", [O.TYPE_Q4_K, O.TYPE_Q6_K])
def test_simd_dots_equal_the_scalar_restatement(qt):
    """The AVX2 dots that mul_mat_id runs (byte multiply-adds, as ggml's CPU path) against the
    scalar restatement, bit for bit: fitted rows, random valid blocks (every nibble, scale and high
    bit pattern), and activations at the Q8_K extremes."""
    from tests.common import random_kquant_bytes
    rng = np.random.default_rng(qt)
    ncols = 2048
    rows = [O.quantize(qt, rng.uniform(-1, 1, (16, ncols)).astype(np.float32)),
            random_kquant_bytes(rng, qt, 64, ncols, 1.0)]
    xs = [rng.uniform(-1, 1, ncols), rng.standard_normal(ncols) * 30,
          np.where(rng.random(ncols) < 0.5, -1.0, 1.0) * 127]
    scalar = O.lib().tmo_vec_dot_q4k_q8k if qt == O.TYPE_Q4_K else O.lib().tmo_vec_dot_q6k_q8k
    simd = O.lib().tmo_vec_dot_q4k_q8k_simd if qt == O.TYPE_Q4_K else O.lib().tmo_vec_dot_q6k_q8k_simd
    for x in xs:
        xq = O.quantize_q8k(np.asarray(x, np.float32))
        for block in rows:
            for r in range(block.shape[0]):
                row = np.ascontiguousarray(block[r])
                a = np.float32(scalar(ncols, row.ctypes.data, xq.ctypes.data))
                b = np.float32(simd(ncols, row.ctypes.data, xq.ctypes.data))
                assert a.view(np.uint32) == b.view(np.uint32), (r, float(a), float(b))


@pytest.mark.parametrize("qt", [O.TYPE_Q4_K, O.TYPE_Q6_K])
def test_multi_column_dots_equal_the_scalar_restatement(qt):
    """The dots mul_mat_id runs (one weight row against up to eight activation rows, scales applied to
    the 16-bit pair sums in vector registers) against the scalar restatement, column by column and bit for
    bit, with 1 to 8 columns, random valid blocks and activations at the Q8_K extremes."""
    import ctypes as C
    from tests.common import random_kquant_bytes
    rng = np.random.default_rng(100 + qt)
    ncols = 1536
    rows = np.concatenate([O.quantize(qt, rng.uniform(-1, 1, (8, ncols)).astype(np.float32)),
                           random_kquant_bytes(rng, qt, 24, ncols, 1.0)])
    cols = [O.quantize_q8k(np.asarray(x, np.float32)) for x in
            (rng.uniform(-1, 1, ncols), rng.standard_normal(ncols) * 30,
             np.where(rng.random(ncols) < 0.5, -1.0, 1.0) * 127, rng.standard_normal(ncols),
             rng.uniform(-1, 1, ncols) * 5, rng.standard_normal(ncols) * 0.01,
             np.where(rng.random(ncols) < 0.5, 127.0, -127.0), rng.standard_normal(ncols) * 100)]
    scalar = O.lib().tmo_vec_dot_q4k_q8k if qt == O.TYPE_Q4_K else O.lib().tmo_vec_dot_q6k_q8k
    for nc in range(1, 9):
        xs = (C.c_void_p * 8)(*[c.ctypes.data for c in cols])
        for r in range(rows.shape[0]):
            row = np.ascontiguousarray(rows[r])
            out = np.zeros(8, np.float32)
            O.lib().tmo_dot_cols(qt, ncols, row.ctypes.data, xs, nc, out.ctypes.data)
            for c in range(nc):
                want = np.float32(scalar(ncols, row.ctypes.data, cols[c].ctypes.data))
                assert out[c].view(np.uint32) == want.view(np.uint32), (nc, r, c)


@pytest.mark.parametrize("T,H,E,norm", [(5, 128, 16, False), (9, 768, 40, True), (16, 2048, 128, False),
                                       (3, 4096, 64, True), (4, 200, 8, False)])
def test_route_logits_equal_the_scalar_router_dot(T, H, E, norm):
    """tmo_route's logits (32 lanes in vector registers over lane-major copies when H % 128 == 0) are
    tmo_router_dot's bits for every (token, expert), with and without the norm, over values of mixed scale."""
    rng = np.random.default_rng(T * 1000 + H + E)
    x = (rng.standard_normal((T, H)) * rng.choice([1e-3, 1.0, 30.0], (T, H))).astype(np.float32)
    rw = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    nw = rng.uniform(0.5, 1.5, H).astype(np.float32)
    _, _, xn, lg = O.route(x, min(4, E), router_w=rw, norm=norm, norm_w=nw if norm else None)
    dot = O.lib().tmo_router_dot
    for t in range(T):
        row = np.ascontiguousarray(xn[t])
        for e in range(E):
            want = np.float32(dot(rw[e].ctypes.data, row.ctypes.data, H))
            assert lg[t, e].view(np.uint32) == want.view(np.uint32), (t, e)


TYPES = [O.TYPE_Q4_K, O.TYPE_Q6_K]


@pytest.mark.parametrize("qt", TYPES)
@pytest.mark.parametrize("tokens", [1, 8, 64])
@pytest.mark.parametrize("b1_used", [False, True])
def test_mul_mat_id_matches_per_expert_and_zero_rows(qt, tokens, b1_used):
    """mul_mat_id_skip.rs sweep (k=512, n=64, E=16, used=4, 30% -1 ids): equals a per-expert
    product within TOL_CPU = 1e-4 of the largest value; -1 rows are exactly zero."""
    K, N, E, used = 512, 64, 16, 4
    rng = XorShift(0x9E3779B97F4A7C15 + qt + tokens)
    W = O.quantize(qt, rng.f32(E * N * K).reshape(E, N, K))
    b1 = used if b1_used else 1
    b = rng.f32(tokens * b1 * K).reshape(tokens, b1, K)
    ids = make_ids(rng, E, used, tokens, 30)
    got = O.mul_mat_id(qt, W, K, N, E, b, ids)
    want = np.zeros_like(got)
    for t in range(tokens):
        for j in range(used):
            e = ids[t, j]
            if e < 0:
                continue
            col = b[t, 0 if b1 == 1 else j]
            xq = O.quantize_q8k(col)
            fn = O.lib().tmo_vec_dot_q4k_q8k if qt == O.TYPE_Q4_K else O.lib().tmo_vec_dot_q6k_q8k
            for r in range(N):
                row = np.ascontiguousarray(W[e, r])
                want[t, j, r] = fn(K, row.ctypes.data, xq.ctypes.data)
    neg = ids < 0
    assert np.all(got[neg] == 0.0)
    scale = max(np.abs(want).max(), 1e-6)
    assert np.abs(got - want).max() / scale <= 1e-4
    # and the f64 mode agrees within the K-quant envelope
    f64 = O.mul_mat_id(qt, W, K, N, E, b, ids, mode=O.MODE_F64)
    assert np.abs(f64 - got).max() / scale <= 1e-4


def test_sort_pairs_matches_group_pairs_order():
    """qwen3moe.rs:2951-2988: every pair lands once, in increasing pair order, each expert with
    all its rows."""
    chosen, n_used = routing()
    ids = chosen.reshape(-1, n_used)
    counts, offsets, perm = O.sort_pairs(ids, 32)
    assert perm.size == chosen.size
    for e in range(32):
        seg = perm[offsets[e]:offsets[e + 1]].tolist()
        assert seg == group_pairs(chosen, n_used, {e})
        assert counts[e] == int(np.sum(chosen == e))
    assert sorted(perm.tolist()) == list(range(chosen.size))


def test_sort_pairs_skips_negative_ids():
    ids = np.array([[3, -1, 0], [0, 3, -1]], dtype=np.int32)
    counts, offsets, perm = O.sort_pairs(ids, 4)
    assert counts.tolist() == [2, 0, 0, 2]
    assert perm.tolist() == [2, 3, 0, 4]


def test_router_top_k_ties_lower_index():
    logits = np.zeros((1, 16), dtype=np.float32)
    logits[0, [3, 7, 9]] = 1.0
    ids, w, probs = O.softmax_topk(logits, 4)
    assert ids[0].tolist() == [3, 7, 9, 0]
    assert np.all(np.diff(probs[0][ids[0]]) <= 0)
    np.testing.assert_allclose(w.sum(), 1.0, rtol=1e-6)


def test_router_clamp_and_renormalisation():
    """w = sel / clamp(sum sel, 6.1035156e-5) (qwen3moe.rs:2886-2888)."""
    rng = np.random.default_rng(9)
    logits = rng.standard_normal((64, 128)).astype(np.float32)
    ids, w, probs = O.softmax_topk(logits, 8)
    sel = np.take_along_axis(probs, ids, 1)
    np.testing.assert_allclose(w, sel / sel.sum(1, keepdims=True), rtol=2e-6)
    # descending, distinct ids
    assert np.all(np.diff(sel, axis=1) <= 0)
    assert all(len(set(r)) == 8 for r in ids.tolist())


def test_exp_canon_accuracy():
    xs = np.concatenate([-np.logspace(-8, np.log10(87), 2000), [0.0, -0.5, -87.0]]).astype(np.float32)
    got = np.array([O.exp_canon(float(v)) for v in xs])
    ref = np.exp(xs.astype(np.float64))
    assert np.max(np.abs(got - ref) / ref) < 4e-7
    assert O.exp_canon(-88.0) == 0.0


def test_router_logits_canonical_order_close_to_f64():
    rng = np.random.default_rng(11)
    x = rng.standard_normal((4, 2048)).astype(np.float32)
    w = (rng.standard_normal((128, 2048)) * 0.02).astype(np.float32)
    got = O.router_logits(x, w)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    assert np.max(np.abs(got - ref)) < 1e-5


def test_experts_reference_layer_small():
    """The C1 tiny layer (T=32, H=512, E=16, k=4, I=256, all Q4_K): q8k mode is within the
    north-star tolerance of the f64 mode, and -1 choices contribute nothing."""
    rng = np.random.default_rng(20261201)
    H, I, E, k, T = 512, 256, 16, 4, 32
    gate = O.quantize(O.TYPE_Q4_K, (rng.standard_normal((E, I, H)) * 0.02).astype(np.float32))
    up = O.quantize(O.TYPE_Q4_K, (rng.standard_normal((E, I, H)) * 0.02).astype(np.float32))
    down = O.quantize(O.TYPE_Q4_K, (rng.standard_normal((E, H, I)) * 0.02).astype(np.float32))
    router = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float32)
    out, ids, w = O.layer(x, k, gate, up, down, H, I, E, router_w=router)
    assert ids.shape == (T, k) and np.all((ids >= 0) & (ids < E))
    ref = O.experts(x, ids, w, gate, up, down, H, I, E, mode=O.MODE_F64)
    from tests.common import nrms, maxabs_over_rms
    assert nrms(out, ref) < 1e-2 and maxabs_over_rms(out, ref) < 5e-2
    ids2 = ids.copy()
    ids2[:, -1] = -1
    out2 = O.experts(x, ids2, w, gate, up, down, H, I, E)
    # the same as dropping the last choice's weight
    w3 = w.copy()
    w3[:, -1] = 0.0
    out3 = O.experts(x, ids, w3, gate, up, down, H, I, E)
    np.testing.assert_allclose(out2, out3, rtol=0, atol=1e-6)
