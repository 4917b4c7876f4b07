"""The streamed layer step over an expert-slot cache (a10): fewer device slots than experts, the
rest in a pinned host store.  Per step, the device planner must produce the reference planner's
chunks, slot maps and loads (oracle/slots.py, pinned against the reference's LayerSlots tests), the
slot table must evolve like the reference's LRU, and the layer output must be bit-identical to the
resident layer's (the same kernels compute every pair; only the grouping into chunks differs)."""
import numpy as np
import pytest
import torch

import oracle as O
from oracle import slots as S
import tetraeder_b200 as tb
from tests.common import maxabs_over_rms, nrms, quantized_experts

pytestmark = pytest.mark.gpu


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def pinned(a):
    return torch.from_numpy(np.ascontiguousarray(a)).pin_memory()


def zipf_logits(rng, T, E, s=1.2):
    """Router logits ~N(0,1) plus a Zipf(s) bias over a seeded expert permutation."""
    perm = rng.permutation(E)
    bias = np.empty(E, np.float32)
    bias[perm] = -s * np.log(np.arange(1, E + 1, dtype=np.float64))
    return (rng.standard_normal((T, E)) + bias).astype(np.float32)


def _weights(rng, H, I, E, gt, dt, exact):
    gate = quantized_experts(rng, gt, E, I, H, exact=exact)
    up = quantized_experts(rng, gt, E, I, H, exact=exact)
    down = quantized_experts(rng, dt, E, H, I, exact=exact)
    return gate, up, down


def _check_plan(cache, ref_layer, ids, steps_ref):
    n, maps, loads = cache.last_plan()
    assert n == len(steps_ref), f"chunks {n} != {len(steps_ref)}"
    for c in range(cache.max_chunks):
        if c < n:
            chunk, slots, ld, m = steps_ref[c]
            assert maps[c] == m, f"chunk {c} map"
            assert loads[c] == ld, f"chunk {c} loads"
        else:
            assert all(v == -1 for v in maps[c]) and loads[c] == []
    owner, stats, counts = cache.state()
    assert owner == ref_layer.owner
    assert stats == (ref_layer.hits, ref_layer.misses, ref_layer.bypass)
    return counts


CASES = [
    # name, H, I, E, k, slots, T, gate/up type, down type, exact, zipf
    ("tiny 6 slots T=32", 512, 256, 16, 4, 6, 32, O.TYPE_Q4_K, O.TYPE_Q4_K, True, False),
    ("tiny 5 slots prefill T=1536", 512, 256, 16, 4, 5, 1536, O.TYPE_Q4_K, O.TYPE_Q4_K, True, True),
    ("30B 64 slots T=64", 2048, 768, 128, 8, 64, 64, O.TYPE_Q4_K, O.TYPE_Q6_K, False, True),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_streamed_layer_matches_resident_and_planner(case):
    name, H, I, E, k, NS, T, gt, dt, exact, zipf = case
    rng = np.random.default_rng(7 + len(name))
    gate, up, down = _weights(rng, H, I, E, gt, dt, exact)
    layer = tb.MoeLayer(H, I, E, k, gate_type=gt, up_type=gt, down_type=dt, max_tokens=T)
    resident = tb.ExpertWeights(cuda(gate), cuda(up), cuda(down))
    store = tb.ExpertWeights(pinned(gate), pinned(up), pinned(down))
    slots = tb.ExpertWeights(*(torch.zeros((NS,) + a.shape[1:], dtype=torch.uint8, device="cuda")
                               for a in (gate, up, down)))
    cache = tb.SlotCache(layer, slots, store)
    ref = S.LayerSlots(E, NS)
    total = np.zeros(E, np.int64)
    try:
        for step in range(3):
            x = rng.standard_normal((T, H)).astype(np.float32)
            lg = zipf_logits(rng, T, E) if zipf else rng.standard_normal((T, E)).astype(np.float32)
            ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
            out = layer.moe_ffn_streamed(cuda(x), cache, logits=cuda(lg), ids_out=ids)
            want_out = layer.moe_ffn(cuda(x), resident, logits=cuda(lg))
            layer.check()
            got_ids = ids.cpu().numpy()
            want_ids, want_w, _ = O.softmax_topk(lg, k)
            assert np.array_equal(got_ids, want_ids), f"{name} step {step}: routing"
            steps_ref = S.step(ref, got_ids.reshape(-1))
            counts = _check_plan(cache, ref, got_ids, steps_ref)
            total += np.bincount(got_ids.reshape(-1), minlength=E)
            assert counts == total.tolist()
            a, b = out.cpu().numpy(), want_out.cpu().numpy()
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), \
                f"{name} step {step}: streamed != resident (max |d| {np.abs(a - b).max():.3e})"
            if step == 0:  # and the oracle, once
                want = O.experts(x, want_ids, want_w, gate, up, down, H, I, E, gt, gt, dt)
                n, m = nrms(a, want), maxabs_over_rms(a, want)
                assert n <= 1e-2 and m <= 5e-2, f"{name}: nrms={n:.2e} maxabs/rms={m:.2e}"
        # the slots hold the experts the table says they hold, byte for byte
        owner, _, _ = cache.state()
        for s_, e in enumerate(owner):
            if e >= 0:
                assert torch.equal(slots.gate[s_].cpu(), store.gate[e]) and torch.equal(slots.down[s_].cpu(),
                                                                                       store.down[e])
    finally:
        cache.close()
        layer.close()


def test_make_resident_and_hot_set_follow_the_reference():
    H, I, E, k, NS = 512, 256, 16, 4, 4
    rng = np.random.default_rng(3)
    gate, up, down = _weights(rng, H, I, E, O.TYPE_Q4_K, O.TYPE_Q4_K, True)
    layer = tb.MoeLayer(H, I, E, k, gate_type=O.TYPE_Q4_K, up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q4_K,
                        max_tokens=8)
    store = tb.ExpertWeights(pinned(gate), pinned(up), pinned(down))
    slots = tb.ExpertWeights(*(torch.zeros((NS,) + a.shape[1:], dtype=torch.uint8, device="cuda")
                               for a in (gate, up, down)))
    cache = tb.SlotCache(layer, slots, store)
    ref = S.LayerSlots(E, NS)
    try:
        cache.make_resident([7, 1, 2])
        S.make_resident(ref, [7, 1, 2])
        cache.make_resident([1, 3, 9])  # 1 hits; 3 takes the free slot; 9 evicts the LRU (7)
        S.make_resident(ref, [1, 3, 9])
        owner, stats, _ = cache.state()
        assert owner == ref.owner and stats == (ref.hits, ref.misses, ref.bypass)
        cache.set_hot_set([5, 9])
        missing = ref.set_hot_set([5, 9])
        S.make_resident(ref, missing)
        owner, stats, _ = cache.state()
        assert owner == ref.owner and stats == (ref.hits, ref.misses, ref.bypass)
        for s_, e in enumerate(owner):
            if e >= 0:
                assert torch.equal(slots.up[s_].cpu(), store.up[e])
    finally:
        cache.close()
        layer.close()


def test_all_pinned_slots_report_no_free_slot():
    H, I, E, k, NS, T = 512, 256, 16, 4, 2, 8
    rng = np.random.default_rng(4)
    gate, up, down = _weights(rng, H, I, E, O.TYPE_Q4_K, O.TYPE_Q4_K, True)
    layer = tb.MoeLayer(H, I, E, k, gate_type=O.TYPE_Q4_K, up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q4_K,
                        max_tokens=T)
    store = tb.ExpertWeights(pinned(gate), pinned(up), pinned(down))
    slots = tb.ExpertWeights(*(torch.zeros((NS,) + a.shape[1:], dtype=torch.uint8, device="cuda")
                               for a in (gate, up, down)))
    cache = tb.SlotCache(layer, slots, store)
    try:
        cache.set_hot_set([0, 1])
        lg = np.full((T, E), -4.0, np.float32)
        lg[:, 2:2 + k] = 4.0  # every token routes to experts 2..5, none of them resident
        layer.moe_ffn_streamed(cuda(rng.standard_normal((T, H)).astype(np.float32)), cache, logits=cuda(lg))
        with pytest.raises(tb.TmoeError, match="all pinned"):
            layer.check()
        _, stats, _ = cache.state()
        assert stats == (0, 2, 1)  # the two pins were loaded as misses; the first routed miss bypassed
    finally:
        cache.close()
        layer.close()


def test_streamed_steps_with_pinned_experts_follow_the_reference():
    """Pins cut the victims a chunk's misses can take; when the misses could outnumber them the
    planner must make the reference's serial lookups (which may then evict the chunk's own
    entries).  Every step is checked against the oracle."""
    H, I, E, k, NS, T = 512, 256, 16, 4, 5, 24
    rng = np.random.default_rng(11)
    gate, up, down = _weights(rng, H, I, E, O.TYPE_Q4_K, O.TYPE_Q4_K, True)
    layer = tb.MoeLayer(H, I, E, k, gate_type=O.TYPE_Q4_K, up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q4_K,
                        max_tokens=T)
    resident = tb.ExpertWeights(cuda(gate), cuda(up), cuda(down))
    store = tb.ExpertWeights(pinned(gate), pinned(up), pinned(down))
    slots = tb.ExpertWeights(*(torch.zeros((NS,) + a.shape[1:], dtype=torch.uint8, device="cuda")
                               for a in (gate, up, down)))
    cache = tb.SlotCache(layer, slots, store)
    ref = S.LayerSlots(E, NS)
    try:
        cache.set_hot_set([3, 9])
        S.make_resident(ref, ref.set_hot_set([3, 9]))
        for step in range(4):
            x = rng.standard_normal((T, H)).astype(np.float32)
            lg = zipf_logits(rng, T, E)
            ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
            out = layer.moe_ffn_streamed(cuda(x), cache, logits=cuda(lg), ids_out=ids)
            want_out = layer.moe_ffn(cuda(x), resident, logits=cuda(lg))
            got_ids = ids.cpu().numpy()
            try:
                steps_ref = S.step(ref, got_ids.reshape(-1))
            except RuntimeError:  # the oracle found every slot pinned: so must the device
                with pytest.raises(tb.TmoeError, match="all pinned"):
                    layer.check()
                break
            layer.check()
            _check_plan(cache, ref, got_ids, steps_ref)
            # the reference's make_resident makes plain lookups, so with pins a chunk's late miss can
            # evict the chunk's own earlier entry (two experts then share a slot); only without that
            # are the outputs those of the resident experts
            shared = any(len(set(sl)) < len(sl) for _, sl, _, _ in steps_ref)
            if not shared:
                assert np.array_equal(out.cpu().numpy().view(np.uint32), want_out.cpu().numpy().view(np.uint32))
    finally:
        cache.close()
        layer.close()


def test_replayed_routing_trace_routes_as_recorded(tmp_path):
    """Recorded routing (a tetraeder-routing v1 trace) replayed through the streamed layer: the
    logits of each recorded step make the layer's own top-k pick exactly the recorded ids, the
    planner follows the reference's LRU over them, and the output matches the oracle."""
    from tetraeder_b200.trace import LayerStep, TraceHeader, TraceReader, TraceWriter
    H, I, E, k, NS, T = 512, 256, 16, 4, 6, 32
    rng = np.random.default_rng(11)
    gate, up, down = _weights(rng, H, I, E, O.TYPE_Q4_K, O.TYPE_Q4_K, True)
    path = tmp_path / "routing.bin"
    with TraceWriter(path, TraceHeader(2, E, k, vram_slots=NS, ram_slots=E)) as w:
        for step in range(4):
            for il in range(2):
                lg = zipf_logits(rng, T, E)
                w.layer_step(step, il, O.softmax_topk(lg, k)[0])
            if step == 1:
                w.hot_refresh(step)
    with TraceReader(path) as r:
        recorded = [s for s in r if isinstance(s, LayerStep) and s.layer == 1]
    assert len(recorded) == 4
    layer = tb.MoeLayer(H, I, E, k, gate_type=O.TYPE_Q4_K, up_type=O.TYPE_Q4_K, down_type=O.TYPE_Q4_K, max_tokens=T)
    store = tb.ExpertWeights(pinned(gate), pinned(up), pinned(down))
    slots = tb.ExpertWeights(*(torch.zeros((NS,) + a.shape[1:], dtype=torch.uint8, device="cuda")
                               for a in (gate, up, down)))
    cache = tb.SlotCache(layer, slots, store)
    ref = S.LayerSlots(E, NS)
    try:
        for s in recorded:
            x = rng.standard_normal((T, H)).astype(np.float32)
            lg = s.logits(E)
            ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
            out = layer.moe_ffn_streamed(cuda(x), cache, logits=cuda(lg), ids_out=ids)
            layer.check()
            assert np.array_equal(ids.cpu().numpy(), s.ids), f"step {s.step}: routing differs from the trace"
            _check_plan(cache, ref, s.ids, S.step(ref, s.ids.reshape(-1)))
            want_ids, want_w, _ = O.softmax_topk(lg, k)
            want = O.experts(x, want_ids, want_w, gate, up, down, H, I, E, O.TYPE_Q4_K, O.TYPE_Q4_K, O.TYPE_Q4_K)
            assert nrms(out.cpu().numpy(), want) < 1e-3
    finally:
        cache.close()
        layer.close()
