"""Parity at the configurations bench.py reports, against the CPU oracle on the same inputs.

The weights are drawn the way bench.py draws them: N(0, 0.02) on the device, quantised by the
device quantiser (whose bytes equal the oracle quantiser's, tests/test_gpu_parity.py), so each
case is the benchmarked layer itself, not a smaller stand-in:

  C2 prefill     --mode prefill: the Qwen3-30B-A3B layer (H 2048, I 768, 128 experts, top-8,
                 gate/up Q4_K, down Q6_K) at T = 8192, on the grouped tcgen05 GEMMs;
  C4 decode      --shape 235b: the Qwen3-235B-A22B layer (H 4096, I 1536, 128 experts, all Q4_K)
                 at T = 64 (decode GEMV) and T = 4096 (grouped GEMMs), all 128 experts resident
                 (1.36 GB);
  C5 streamed    --mode streamed: the 30B layer at T = 8192 with logits ~N(0,1) plus a Zipf(1.2)
                 bias over a seeded expert permutation, 64 of the 128 experts in device slots and
                 all of them in a pinned host store, the slots starting with the 64 most-favoured
                 experts of the bias.

Bars: expert ids bit-exact (ties to the lower index); outputs within the north-star bound
(normalised RMS <= 1e-2, max-abs <= 5e-2 x output RMS) and the stricter bound of each regime
(decode GEMV 1e-3 / 1e-2; grouped GEMMs 1e-3 / 2.5e-2, the fp16 down product being their only
departure from the reference's integer sums).  The streamed case also holds the device planner's
chunks, slot maps, loads, slot table and counters to oracle/slots.py for two steps, and its output
bit for bit to the resident layer's.  The oracle takes about 10-25 s per case on 16 host threads.
"""
import numpy as np
import pytest
import torch

import oracle as O
from oracle import slots as S
import tetraeder_b200 as tb
from tetraeder_b200 import moe
from tests.common import NORTH_MAXABS, NORTH_NRMS, maxabs_over_rms, nrms

pytestmark = pytest.mark.gpu

GEMV_NRMS, GEMV_MAXABS = 1e-3, 1e-2
GEMM_NRMS, GEMM_MAXABS = 1e-3, 2.5e-2


def bench_weights(H, I, E, gt, dt, seed):
    """Router f32 [E, H] and stacked expert tensors drawn as bench.make_layers draws them."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    rw = torch.randn((E, H), generator=g, device=dev) * 0.02
    gate = moe.quantize(gt, torch.randn((E, I, H), generator=g, device=dev) * 0.02)
    up = moe.quantize(gt, torch.randn((E, I, H), generator=g, device=dev) * 0.02)
    down = moe.quantize(dt, torch.randn((E, H, I), generator=g, device=dev) * 0.02)
    torch.cuda.synchronize()
    return rw, tb.ExpertWeights(gate, up, down)


def host(t):
    return t.cpu().numpy()


def check_bounds(got, want, strict, what):
    n, m = nrms(got, want), maxabs_over_rms(got, want)
    assert n <= NORTH_NRMS and m <= NORTH_MAXABS, f"{what}: north-star bound nrms={n:.2e} maxabs/rms={m:.2e}"
    assert n <= strict[0] and m <= strict[1], f"{what}: nrms={n:.2e} maxabs/rms={m:.2e} (bound {strict})"


LAYER_CASES = [
    # (name, H, I, E, k, T, gate/up type, down type, grouped GEMMs expected)
    ("C2 prefill T=8192", 2048, 768, 128, 8, 8192, O.TYPE_Q4_K, O.TYPE_Q6_K, True),
    ("C4 235B decode T=64", 4096, 1536, 128, 8, 64, O.TYPE_Q4_K, O.TYPE_Q4_K, False),
    ("C4 235B prefill T=4096", 4096, 1536, 128, 8, 4096, O.TYPE_Q4_K, O.TYPE_Q4_K, True),
]


@pytest.mark.parametrize("case", LAYER_CASES, ids=[c[0] for c in LAYER_CASES])
def test_bench_layer_config_matches_oracle(case):
    name, H, I, E, k, T, gt, dt, gemm = case
    rw, wts = bench_weights(H, I, E, gt, dt, 20261201 + T)
    g = torch.Generator(device="cuda")
    g.manual_seed(20261202 + T)
    x = torch.randn((T, H), generator=g, device="cuda")
    layer = tb.MoeLayer(H, I, E, k, gate_type=gt, up_type=gt, down_type=dt, max_tokens=T)
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    try:
        layer.profile(True)
        out = layer.moe_ffn(x, wts, router_w=rw, ids_out=ids, w_out=w)
        phases = layer.profile_collect()
        layer.profile(False)
        layer.check()
        # the regime bench.py reports ran: the grouped GEMMs take no separate Q8_K pass of the
        # SwiGLU rows; the decode GEMV does
        assert ("quant_act" not in phases) == gemm, f"{name}: phases {sorted(phases)}"
        xh, rwh = host(x), host(rw)
        want_ids, want_w, _, _ = O.route(xh, k, router_w=rwh)
        assert np.array_equal(host(ids), want_ids), f"{name}: expert ids"
        assert np.array_equal(host(w).view(np.uint32), want_w.view(np.uint32)), f"{name}: weights"
        want, want_act = O.experts(xh, want_ids, want_w, host(wts.gate), host(wts.up), host(wts.down), H, I, E,
                                   gt, gt, dt, want_act=True)
        check_bounds(host(out), want, (GEMM_NRMS, GEMM_MAXABS) if gemm else (GEMV_NRMS, GEMV_MAXABS), name)
        if name.startswith("C2 prefill"):
            rounded_gate_up_leave_the_bound(layer, xh, want_ids, want_w, wts, want, want_act, H, I, E, k)
    finally:
        layer.close()


def to_bf16(a):
    """f32 -> nearest bf16 (ties to even), returned as f32."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16 << 16
    return u.astype(np.uint32).view(np.float32)


def rounded_gate_up_leave_the_bound(layer, x, ids, w, wts, want, act_exact, H, I, E, k):
    """Why the large-batch gate/up stays on exact integer operands (Q8_K int8 x Q4_K sc*q, both
    exact in fp16) rather than the plain 16-bit tiles of a dequantise-then-GEMM design: the SwiGLU
    output goes through Q8_K before the down product (the reference's CPU arithmetic), and gate/up
    values computed from rounded weights move some activations across a Q8_K rounding boundary.
    On this benchmarked case bf16 weights (the dequantised tiles a bf16 GEMM would read) leave the
    north-star max-abs bound, and fp16 weights leave the 2.5e-2 bound the exact design meets, while
    the same down product and combine on the exact activations reproduce the oracle.

    The model is kind to the rounded designs: only the weights are rounded (the Q8_K activations
    stay exact) and the dot products are accumulated in float64.  The down product of every variant
    is tmoe_mul_mat_id (the exact Q8_K integer path) and the combine folds the choices in order."""
    T = x.shape[0]
    xq = O.dequantize_q8k(O.quantize_q8k(x)).reshape(T, H).astype(np.float64)
    gate, up, down = host(wts.gate), host(wts.up), wts.down

    def finish(act):
        dn = host(layer.mul_mat_id(O.TYPE_Q6_K, down, torch.from_numpy(np.ascontiguousarray(act, np.float32)).cuda(),
                                   torch.from_numpy(ids).cuda()))
        o = dn[:, 0] * w[:, :1]
        for j in range(1, k):
            o = o + dn[:, j] * w[:, j:j + 1]
        return o

    exact = finish(act_exact)
    assert nrms(exact, want) <= 1e-5, "the down product and combine of the model must reproduce the oracle"
    fp16 = lambda a: a.astype(np.float16).astype(np.float32)  # noqa: E731
    for rnd, what, bound in ((to_bf16, "bf16", NORTH_MAXABS), (fp16, "fp16", GEMM_MAXABS)):
        act = np.empty((T, k, I), np.float32)
        for e in range(E):
            tt, jj = np.nonzero(ids == e)
            if not len(tt):
                continue
            wg = rnd(O.dequantize(O.TYPE_Q4_K, gate[e], I * H)).reshape(I, H).astype(np.float64)
            wu = rnd(O.dequantize(O.TYPE_Q4_K, up[e], I * H)).reshape(I, H).astype(np.float64)
            g, u = (xq[tt] @ wg.T).astype(np.float32), (xq[tt] @ wu.T).astype(np.float32)
            act[tt, jj] = g / (np.float32(1) + np.exp(-g)) * u
        m = maxabs_over_rms(finish(act), want)
        assert m > bound, f"{what} gate/up weights: max-abs {m:.3e} x RMS is inside {bound}"


def zipf_logits(T, E, seed, gen, s=1.2):
    """bench.py's C5 routing: logits ~N(0,1) plus -s ln(rank + 1) over a seeded permutation."""
    perm = np.random.default_rng(seed).permutation(E)
    bias = np.empty(E, np.float32)
    bias[perm] = -s * np.log(np.arange(1, E + 1, dtype=np.float64))
    return torch.randn((T, E), generator=gen, device="cuda") + torch.from_numpy(bias).cuda(), perm


def test_c5_streamed_t8192_64_of_128_slots():
    H, I, E, k, T, NS = 2048, 768, 128, 8, 8192, 64
    gt, dt = O.TYPE_Q4_K, O.TYPE_Q6_K
    rw, wts = bench_weights(H, I, E, gt, dt, 20261201)
    del rw
    store = tb.ExpertWeights(*(t.cpu().pin_memory() for t in (wts.gate, wts.up, wts.down)))
    slots = tb.ExpertWeights(*(torch.zeros((NS,) + tuple(t.shape[1:]), dtype=torch.uint8, device="cuda")
                               for t in (wts.gate, wts.up, wts.down)))
    layer = tb.MoeLayer(H, I, E, k, gate_type=gt, up_type=gt, down_type=dt, max_tokens=T)
    cache = tb.SlotCache(layer, slots, store)
    ref = S.LayerSlots(E, NS)
    g = torch.Generator(device="cuda")
    g.manual_seed(20261206)
    try:
        _, perm = zipf_logits(1, E, 20261206, g)
        hot = [int(e) for e in perm[:NS]]
        cache.make_resident(hot)
        S.make_resident(ref, hot)
        total = np.zeros(E, np.int64)
        for step in range(2):
            x = torch.randn((T, H), generator=g, device="cuda")
            lg, _ = zipf_logits(T, E, 20261206, g)
            ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
            out = layer.moe_ffn_streamed(x, cache, logits=lg, ids_out=ids)
            resident = layer.moe_ffn(x, wts, logits=lg)
            layer.check()
            got_ids = host(ids)
            want_ids, want_w, _ = O.softmax_topk(host(lg), k)
            assert np.array_equal(got_ids, want_ids), f"step {step}: routing"
            steps_ref = S.step(ref, got_ids.reshape(-1))
            n, maps, loads = cache.last_plan()
            assert n == len(steps_ref), f"step {step}: chunks {n} != {len(steps_ref)}"
            assert n >= 2, "the skewed batch must need more than one chunk of 64 slots"
            for c in range(n):
                _, _, ld, m = steps_ref[c]
                assert maps[c] == m and loads[c] == ld, f"step {step} chunk {c}: plan"
            owner, stats, counts = cache.state()
            assert owner == ref.owner, f"step {step}: slot table"
            assert stats == (ref.hits, ref.misses, ref.bypass), f"step {step}: counters"
            total += np.bincount(got_ids.reshape(-1), minlength=E)
            assert counts == total.tolist()
            a, b = host(out), host(resident)
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), f"step {step}: streamed != resident"
            if step == 0:
                want = O.experts(host(x), want_ids, want_w, store.gate.numpy(), store.up.numpy(),
                                 store.down.numpy(), H, I, E, gt, gt, dt)
                check_bounds(a, want, (GEMM_NRMS, GEMM_MAXABS), "C5 streamed")
        for s_, e in enumerate(cache.state()[0]):
            if e >= 0:
                assert torch.equal(slots.gate[s_].cpu(), store.gate[e]) and torch.equal(slots.down[s_].cpu(),
                                                                                       store.down[e])
    finally:
        cache.close()
        layer.close()
