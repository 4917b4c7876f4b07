"""Parity of the CUDA path (through the C ABI) with the CPU oracle on the same seeded inputs.

Bit-exact: selected expert ids, router weights, logits, the per-expert permutation, the device
quantiser's bytes.  Outputs: the decode path emulates ggml's Q8_K activations exactly, so it is
held to a strict bound (normalised RMS <= 1e-3, max-abs <= 1e-2 x RMS) as well as the north-star
bound (normalised RMS <= 1e-2, max-abs <= 5e-2 x RMS)."""
import os
import zlib

import numpy as np
import pytest
import torch

import oracle as O
import tetraeder_b200 as tb
from tetraeder_b200 import moe
from tests.common import (NORTH_MAXABS, NORTH_NRMS, XorShift, make_ids, maxabs_over_rms, nrms,
                          quantized_experts, routing)

pytestmark = pytest.mark.gpu

STRICT_NRMS, STRICT_MAXABS = 1e-3, 1e-2
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kquant_dequant.npz")


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    return t.detach().cpu().numpy()


def assert_close(got, want, strict=True, what=""):
    n, m = nrms(got, want), maxabs_over_rms(got, want)
    assert n <= NORTH_NRMS and m <= NORTH_MAXABS, f"{what}: north-star bound nrms={n:.2e} maxabs/rms={m:.2e}"
    if strict:
        assert n <= STRICT_NRMS and m <= STRICT_MAXABS, f"{what}: strict bound nrms={n:.2e} maxabs/rms={m:.2e}"


# ------------------------------------------------------------------------------------ routing
@pytest.mark.parametrize("T,H,E,k", [(32, 512, 16, 4), (1, 2048, 128, 8), (64, 2048, 128, 8),
                                     (8192, 2048, 128, 8), (64, 4096, 128, 8), (1100, 768, 40, 6), (1100, 768, 128, 8),
                                     (1024, 4096, 128, 8)])
def test_route_bit_exact(T, H, E, k):
    rng = np.random.default_rng(T * 7 + H)
    x = rng.standard_normal((T, H)).astype(np.float32)
    rw = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    layer = tb.MoeLayer(H, 256, E, k, max_tokens=T)
    _, w, ids, lg = layer.router(cuda(x), router_w=cuda(rw), want_logits=True)
    want_ids, want_w, _, want_lg = O.route(x, k, router_w=rw)
    assert np.array_equal(host(lg).view(np.uint32), want_lg.view(np.uint32))
    assert np.array_equal(host(ids), want_ids)
    assert np.array_equal(host(w).view(np.uint32), want_w.view(np.uint32))


def test_route_with_rms_norm_bit_exact():
    rng = np.random.default_rng(1)
    T, H, E, k = 64, 2048, 128, 8
    x = (rng.standard_normal((T, H)) * 3).astype(np.float32)
    nw = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    rw = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    layer = tb.MoeLayer(H, 768, E, k, max_tokens=T, rms_eps=1e-6)
    xn, w, ids = layer.router(cuda(x), router_w=cuda(rw), ffn_norm=cuda(nw), use_norm=True)
    want_ids, want_w, want_xn, _ = O.route(x, k, router_w=rw, norm=True, norm_w=nw, eps=1e-6)
    assert np.array_equal(host(xn).view(np.uint32), want_xn.view(np.uint32))
    assert np.array_equal(host(ids), want_ids)
    assert np.array_equal(host(w).view(np.uint32), want_w.view(np.uint32))


def test_route_from_logits_ties_to_lower_index():
    T, E, k = 16, 128, 8
    rng = np.random.default_rng(2)
    logits = np.round(rng.standard_normal((T, E)) * 2).astype(np.float32)  # many exact ties
    logits[0] = 0.0
    layer = tb.MoeLayer(2048, 768, E, k, max_tokens=T)
    _, w, ids = layer.router(None, logits=cuda(logits))
    want_ids, want_w, _ = O.softmax_topk(logits, k)
    assert np.array_equal(host(ids), want_ids)
    assert host(ids)[0].tolist() == list(range(8))
    assert np.array_equal(host(w).view(np.uint32), want_w.view(np.uint32))


# ------------------------------------------------------------------------------------ dispatch
def test_dispatch_matches_group_pairs_routing():
    chosen, n_used = routing()
    ids = chosen.reshape(-1, n_used)
    layer = tb.MoeLayer(2048, 768, 32, n_used, max_tokens=ids.shape[0])
    counts, offsets, perm = layer.dispatch(cuda(ids), 32)
    c, o, p = O.sort_pairs(ids, 32)
    assert np.array_equal(host(counts), c) and np.array_equal(host(offsets), o)
    assert np.array_equal(host(perm)[: o[-1]], p)


@pytest.mark.parametrize("T,E,k,neg", [(1, 128, 8, 0), (5, 16, 4, 20), (8, 128, 8, 30), (16, 64, 4, 10),
                                       (64, 128, 8, 30), (8192, 128, 8, 10), (4096, 64, 6, 50)])
def test_dispatch_bit_exact(T, E, k, neg):
    """The dispatch against the oracle's stable sort: the ranking sort of up to 64 pairs (the first four
    cases, 64 pairs exactly in the fourth), the one-CTA and the many-CTA sorts."""
    rng = np.random.default_rng(T + E)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    ids[rng.random(ids.shape) < neg / 100] = -1
    layer = tb.MoeLayer(2048, 768, E, k, max_tokens=T)
    counts, offsets, perm = layer.dispatch(cuda(ids), E)
    c, o, p = O.sort_pairs(ids, E)
    assert np.array_equal(host(counts), c) and np.array_equal(host(offsets), o)
    assert np.array_equal(host(perm)[: o[-1]], p)


def test_dispatch_bit_exact_under_skew():
    """A few experts take most pairs (ids drawn with replacement, Zipf-like): the many-CTA sort must
    still give the one-CTA order."""
    T, E, k = 8192, 128, 8
    rng = np.random.default_rng(5)
    wts = 1.0 / np.arange(1, E + 1) ** 1.2
    ids = rng.choice(E, size=(T, k), p=wts / wts.sum()).astype(np.int32)
    ids[rng.random(ids.shape) < 0.05] = -1
    layer = tb.MoeLayer(2048, 768, E, k, max_tokens=T)
    counts, offsets, perm = layer.dispatch(cuda(ids), E)
    c, o, p = O.sort_pairs(ids, E)
    assert np.array_equal(host(counts), c) and np.array_equal(host(offsets), o)
    assert np.array_equal(host(perm)[: o[-1]], p)


# ------------------------------------------------------------------------------------ quantiser
@pytest.mark.parametrize("qt", [O.TYPE_Q4_K, O.TYPE_Q6_K])
def test_device_quantiser_bytes_equal_oracle(qt):
    rng = np.random.default_rng(qt)
    x = (rng.standard_normal((96, 2048)) * 0.02).astype(np.float32)
    x[3] = 0.0
    x[5] = np.abs(x[5])
    got = host(moe.quantize(qt, cuda(x)))
    assert np.array_equal(got, O.quantize(qt, x))


@pytest.mark.parametrize("name,qt", [("q4_k", O.TYPE_Q4_K), ("q6_k", O.TYPE_Q6_K)])
def test_device_dequantiser_equals_gguf_py(name, qt):
    g = np.load(GOLDEN)
    blocks, want = g[name + "_blocks"], g[name + "_values"]
    got = host(moe.dequantize(qt, cuda(blocks), blocks.shape[0] * 256)).reshape(want.shape)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ------------------------------------------------------------------------------------ mul_mat_id
@pytest.mark.parametrize("qt", [O.TYPE_Q4_K, O.TYPE_Q6_K])
@pytest.mark.parametrize("tokens", [1, 8, 64, 512])
@pytest.mark.parametrize("b1_used", [False, True])
def test_mul_mat_id_sweep(qt, tokens, b1_used):
    """The mul_mat_id_skip.rs sweep: k=512, n=64, E=16, used=4, 30% -1 ids, a warm run that
    leaves stale rows first; -1 rows exactly zero, the rest within 1e-4 of the largest value of
    the CPU (oracle) mul_mat_id."""
    K, N, E, used = 512, 64, 16, 4
    rng = XorShift(0x9E3779B97F4A7C15 ^ (qt * 1000 + tokens))
    W = O.quantize(qt, rng.f32(E * N * K).reshape(E, N, K))
    b1 = used if b1_used else 1
    b = rng.f32(tokens * b1 * K).reshape(tokens, b1, K)
    ids = make_ids(rng, E, used, tokens, 30)
    warm = make_ids(rng, E, used, tokens, 0)
    layer = tb.MoeLayer(512, 256, E, used, max_tokens=tokens)
    Wd, bd = cuda(W), cuda(b)
    out = layer.mul_mat_id(qt, Wd, bd, cuda(warm))
    layer.mul_mat_id(qt, Wd, bd, cuda(ids), out=out)
    layer.check()
    got = host(out)
    want = O.mul_mat_id(qt, W, K, N, E, b, ids)
    assert np.all(got[ids < 0] == 0.0)
    scale = max(float(np.abs(want).max()), 1e-6)
    assert float(np.abs(got - want).max()) / scale <= 1e-4


def test_mul_mat_id_30b_gate_up_shape():
    """The timing test's shape (mul_mat_id_skip.rs:302-330): q4_K, k=2048, n=768, E=128, top-8,
    512 tokens."""
    K, N, E, used, T = 2048, 768, 128, 8, 512
    rng = np.random.default_rng(7)
    W = quantized_experts(rng, O.TYPE_Q4_K, E, N, K, exact=False)
    b = rng.uniform(-1, 1, (T, 1, K)).astype(np.float32)
    ids = np.stack([rng.permutation(E)[:used] for _ in range(T)]).astype(np.int32)
    layer = tb.MoeLayer(K, N, E, used, max_tokens=T)
    got = host(layer.mul_mat_id(O.TYPE_Q4_K, cuda(W), cuda(b), cuda(ids)))
    want = O.mul_mat_id(O.TYPE_Q4_K, W, K, N, E, b, ids)
    scale = float(np.abs(want).max())
    assert float(np.abs(got - want).max()) / scale <= 1e-4


def test_mul_mat_id_allocates_nothing_within_the_create_bound():
    """The handle's mul_mat_id scratch is sized by tmoe_create (T*b1 and T*n_used up to
    max_tokens*n_expert_used, K up to max(n_embd, n_ff)): calls within it leave the device's free
    memory as it was, and a call beyond it is refused before any launch."""
    H, I, E, used, T = 2048, 768, 32, 8, 64
    rng = np.random.default_rng(11)
    W = cuda(quantized_experts(rng, O.TYPE_Q6_K, E, H, I, exact=False))
    b = cuda(rng.uniform(-1, 1, (T, used, I)).astype(np.float32))
    ids = cuda(np.stack([rng.permutation(E)[:used] for _ in range(T)]).astype(np.int32))
    layer = tb.MoeLayer(H, I, E, used, max_tokens=T)
    out = torch.empty((T, used, H), device="cuda")
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        layer.mul_mat_id(O.TYPE_Q6_K, W, b, ids, out=out)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0, "mul_mat_id allocated device memory"
    layer.check()
    want = O.mul_mat_id(O.TYPE_Q6_K, host(W), I, H, E, host(b), host(ids))
    assert float(np.abs(host(out) - want).max()) / float(np.abs(want).max()) <= 1e-4
    big = torch.zeros((16 * T, used, I), device="cuda")
    with pytest.raises(tb.TmoeError, match="TMOE_E_INVALID"):
        layer.mul_mat_id(O.TYPE_Q6_K, W, big, cuda(np.zeros((16 * T, used), np.int32)))
    layer.close()


# ------------------------------------------------------------------------------------ layer
def _layer_case(H, I, E, k, T, gate_t, down_t, seed, exact):
    rng = np.random.default_rng(seed)
    gate = quantized_experts(rng, gate_t, E, I, H, exact=exact)
    up = quantized_experts(rng, gate_t, E, I, H, exact=exact)
    down = quantized_experts(rng, down_t, E, H, I, exact=exact)
    rw = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float32)
    return gate, up, down, rw, x


LAYER_CASES = [
    # (name, H, I, E, k, T, gate/up type, down type, exact quantiser)
    ("C1 tiny", 512, 256, 16, 4, 32, O.TYPE_Q4_K, O.TYPE_Q4_K, True),
    ("C2 30B T=1", 2048, 768, 128, 8, 1, O.TYPE_Q4_K, O.TYPE_Q6_K, False),
    ("C2 30B T=4", 2048, 768, 128, 8, 4, O.TYPE_Q4_K, O.TYPE_Q6_K, False),
    ("C2 30B T=16", 2048, 768, 128, 8, 16, O.TYPE_Q4_K, O.TYPE_Q6_K, False),
    ("C2 30B T=64", 2048, 768, 128, 8, 64, O.TYPE_Q4_K, O.TYPE_Q6_K, False),
    ("235B shape T=64", 4096, 1536, 32, 8, 64, O.TYPE_Q4_K, O.TYPE_Q4_K, False),
    # more tokens per expert (12, 32 and 64 pairs an expert): the GEMVs' two-group passes, and more passes
    ("C2 30B T=192", 2048, 768, 128, 8, 192, O.TYPE_Q4_K, O.TYPE_Q6_K, False),
    ("C2 30B T=512", 2048, 768, 128, 8, 512, O.TYPE_Q4_K, O.TYPE_Q6_K, False),
    ("tiny Q6_K gate/up T=256", 512, 256, 16, 4, 256, O.TYPE_Q6_K, O.TYPE_Q6_K, True),
]


@pytest.mark.parametrize("case", LAYER_CASES, ids=[c[0] for c in LAYER_CASES])
def test_layer_parity(case):
    name, H, I, E, k, T, gt, dt, exact = case
    # a seed of the case's name that does not change between processes (str hashes do)
    gate, up, down, rw, x = _layer_case(H, I, E, k, T, gt, dt, zlib.crc32(name.encode()) & 0xffff, exact)
    layer = tb.MoeLayer(H, I, E, k, gate_type=gt, up_type=gt, down_type=dt, max_tokens=T)
    wts = tb.ExpertWeights(cuda(gate), cuda(up), cuda(down))
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    out = layer.moe_ffn(cuda(x), wts, router_w=cuda(rw), ids_out=ids, w_out=w)
    layer.check()
    want_ids, want_w, _, _ = O.route(x, k, router_w=rw)
    assert np.array_equal(host(ids), want_ids), name
    assert np.array_equal(host(w).view(np.uint32), want_w.view(np.uint32)), name
    want = O.experts(x, want_ids, want_w, gate, up, down, H, I, E, gt, gt, dt)
    assert_close(host(out), want, what=name)


def test_experts_with_negative_ids_and_stale_workspace():
    H, I, E, k, T = 2048, 768, 64, 8, 48
    gate, up, down, rw, x = _layer_case(H, I, E, k, T, O.TYPE_Q4_K, O.TYPE_Q6_K, 5, False)
    rng = np.random.default_rng(6)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.01, 0.3, (T, k)).astype(np.float32)
    ids_neg = ids.copy()
    ids_neg[rng.random(ids.shape) < 0.4] = -1
    ids_neg[0] = -1  # a token with no expert at all
    layer = tb.MoeLayer(H, I, E, k, max_tokens=T)
    wts = tb.ExpertWeights(cuda(gate), cuda(up), cuda(down))
    layer.weighted_experts(cuda(x), cuda(ids), cuda(w), wts)  # fills the workspace
    out = host(layer.weighted_experts(cuda(x), cuda(ids_neg), cuda(w), wts))
    layer.check()
    want = O.experts(x, ids_neg, w, gate, up, down, H, I, E, down_type=O.TYPE_Q6_K)
    assert np.all(out[0] == 0.0)
    assert_close(out, want, what="negative ids")


def test_expert_parallel_id_map_matches_local_share():
    """EP on one GPU: rank r of g holds experts [r*E/g, (r+1)*E/g); the map sends the rest to -1
    (qwen3moe_shard.rs:617-626); the partial sums over the ranks add up to the whole layer."""
    H, I, E, k, T, g = 2048, 768, 32, 8, 16, 4
    gate, up, down, rw, x = _layer_case(H, I, E, k, T, O.TYPE_Q4_K, O.TYPE_Q6_K, 8, False)
    layer = tb.MoeLayer(H, I, E, k, max_tokens=T)
    total = np.zeros((T, H), dtype=np.float64)
    span = E // g
    for r in range(g):
        table = np.array([e - r * span if r * span <= e < (r + 1) * span else -1 for e in range(E)], np.int32)
        sl = slice(r * span, (r + 1) * span)
        wts = tb.ExpertWeights(cuda(gate[sl]), cuda(up[sl]), cuda(down[sl]))
        part = host(layer.moe_ffn(cuda(x), wts, router_w=cuda(rw), id_map=cuda(table)))
        ids, w, _, _ = O.route(x, k, router_w=rw)
        want = O.experts(x, O.map_ids(ids, table), w, gate[sl], up[sl], down[sl], H, I, span,
                         down_type=O.TYPE_Q6_K)
        assert_close(part, want, what=f"rank {r}")
        total += part
    ids, w, _, _ = O.route(x, k, router_w=rw)
    whole = O.experts(x, ids, w, gate, up, down, H, I, E, down_type=O.TYPE_Q6_K)
    assert_close(total.astype(np.float32), whole, what="sum over ranks")


def test_bad_expert_id_is_reported():
    H, I, E, k, T = 512, 256, 8, 2, 4
    gate, up, down, rw, x = _layer_case(H, I, E, k, T, O.TYPE_Q4_K, O.TYPE_Q4_K, 9, True)
    layer = tb.MoeLayer(H, I, E, k, gate_type=O.TYPE_Q4_K, up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q4_K, max_tokens=T)
    wts = tb.ExpertWeights(cuda(gate), cuda(up), cuda(down))
    ids = np.array([[0, 9]] * T, dtype=np.int32)
    w = np.full((T, k), 0.5, np.float32)
    layer.weighted_experts(cuda(x), cuda(ids), cuda(w), wts)
    with pytest.raises(tb.TmoeError, match="TMOE_E_INVALID"):
        layer.check()
    layer.check()  # the flag was cleared


def test_misaligned_tensors_are_rejected():
    H, I, E, k = 512, 256, 4, 2
    layer = tb.MoeLayer(H, I, E, k, gate_type=O.TYPE_Q4_K, up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q4_K, max_tokens=4)
    buf = torch.zeros(E * I * 288 + 8, dtype=torch.uint8, device="cuda")
    bad = buf[8:].view(E, I, 288)
    good = torch.zeros(E, I, 288, dtype=torch.uint8, device="cuda")
    down = torch.zeros(E, H, 144, dtype=torch.uint8, device="cuda")
    x = torch.zeros(4, H, device="cuda")
    ids = torch.zeros(4, k, dtype=torch.int32, device="cuda")
    w = torch.ones(4, k, device="cuda")
    with pytest.raises(tb.TmoeError, match="aligned"):
        layer.weighted_experts(x, ids, w, tb.ExpertWeights(bad, good, down))


def test_layer_bf16_input_equals_f32_of_the_same_values():
    """tmoe_layer_bf16 (bf16 activations at the boundary): the rows are widened to f32 exactly, so
    the layer's ids, weights and output equal tmoe_layer's on the f32 values bit for bit, and both
    meet the oracle on them; with the router norm too."""
    H, I, E, k, T = 2048, 768, 128, 8, 16
    gate, up, down, rw, _ = _layer_case(H, I, E, k, T, O.TYPE_Q4_K, O.TYPE_Q6_K, 21, False)
    g = torch.Generator(device="cuda")
    g.manual_seed(22)
    xb = torch.randn((T, H), generator=g, device="cuda").to(torch.bfloat16)
    nw = cuda((1 + 0.1 * np.random.default_rng(23).standard_normal(H)).astype(np.float32))
    layer = tb.MoeLayer(H, I, E, k, max_tokens=T)
    wts = tb.ExpertWeights(cuda(gate), cuda(up), cuda(down))
    for use_norm in (False, True):
        ids_b, ids_f = (torch.empty((T, k), dtype=torch.int32, device="cuda") for _ in range(2))
        ob = layer.moe_ffn(xb, wts, router_w=cuda(rw), ffn_norm=nw, use_norm=use_norm, ids_out=ids_b)
        of = layer.moe_ffn(xb.float(), wts, router_w=cuda(rw), ffn_norm=nw, use_norm=use_norm, ids_out=ids_f)
        layer.check()
        assert torch.equal(ids_b, ids_f) and torch.equal(ob, of), f"use_norm={use_norm}"
    x = host(xb.float())
    want_ids, want_w, _, _ = O.route(x, k, router_w=rw)
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    out = layer.moe_ffn(xb, wts, router_w=cuda(rw), ids_out=ids)
    layer.check()
    assert np.array_equal(host(ids), want_ids)
    assert_close(host(out), O.experts(x, want_ids, want_w, gate, up, down, H, I, E, O.TYPE_Q4_K, O.TYPE_Q4_K,
                                      O.TYPE_Q6_K), what="bf16 input")
    layer.close()
