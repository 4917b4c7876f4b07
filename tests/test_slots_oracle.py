"""The slot-cache restatement (oracle/slots.py) pinned against the known answers of the reference's
own unit tests of `LayerSlots` (crates/memory/src/slots.rs:618-761) and the planner's order
(crates/model/src/experts.rs:624-662)."""
from oracle import slots as S
from oracle.slots import BYPASS, HIT, MISS, Lookup


def test_lru_evicts_the_oldest_unpinned():  # slots.rs:618-643
    layer = S.LayerSlots(8, 3)
    layer.set_hot_set([7])
    assert layer.lookup(7) == Lookup(MISS, 0, -1)
    assert layer.lookup(1).slot == 1
    assert layer.lookup(2).slot == 2
    assert layer.lookup(1) == Lookup(HIT, 1)
    assert layer.lookup(3) == Lookup(MISS, 2, 2)  # 2 is the oldest unpinned; 7 is older but pinned
    assert layer.lookup(7) == Lookup(HIT, 0)
    assert (layer.hits, layer.misses) == (2, 4)


def test_full_of_pinned_bypasses():  # slots.rs:645-653
    layer = S.LayerSlots(8, 2)
    layer.set_hot_set([0, 1])
    layer.lookup(0)
    layer.lookup(1)
    assert layer.lookup(5).kind == BYPASS
    assert layer.bypass == 1


def test_shrink_moves_pinned_and_evicts_the_rest():  # slots.rs:655-673
    layer = S.LayerSlots(8, 4)
    for e in [0, 1, 2, 3]:
        layer.lookup(e)
    layer.set_hot_set([3])
    evicted, moved = layer.set_active(2)
    assert layer.active == 2
    assert len(moved) == 1 and moved[0][0] == 3 and moved[0][2] < 2
    assert 0 <= layer.slot_of(3) < 2
    assert len(layer.table) == 2
    evicted, moved = layer.set_active(4)
    assert not evicted and not moved and layer.active == 4


def test_active_never_drops_below_the_hot_set():  # slots.rs:675-681
    layer = S.LayerSlots(8, 4)
    layer.set_hot_set([0, 1, 2])
    layer.set_active(0)
    assert layer.active == 3


def test_clear_forgets_residents_and_keeps_stats_and_pins():  # slots.rs:683-703
    layer = S.LayerSlots(8, 2)
    layer.set_hot_set([5])
    layer.lookup(5)
    layer.lookup(1)
    layer.clear()
    assert len(layer.table) == 0 and layer.slot_of(5) == -1 and layer.owner[0] == -1
    assert layer.pinned[5] and layer.misses == 2
    assert layer.lookup(1) == Lookup(MISS, 0, -1)


def test_lookup_except_spares_the_protected():  # slots.rs:739-753
    layer = S.LayerSlots(8, 2)
    layer.lookup(1)
    layer.lookup(2)
    assert layer.lookup_except(3, [1]) == Lookup(MISS, 1, 2)
    assert layer.lookup_except(4, [1, 3]).kind == BYPASS


def test_hot_set_from_counts():  # slots.rs:755-761
    assert S.hot_from_counts([5, 0, 9, 5, 1], 3) == [2, 0, 3]
    assert S.hot_from_counts([0, 0], 4) == []


def test_plan_orders_hits_first_then_first_appearance_and_chunks():
    layer = S.LayerSlots(16, 3)
    for e in (9, 4):
        layer.lookup(e)
    chosen = [7, 4, 2, 9, 7, 5, 4, 11]  # distinct in first appearance: 7 4 2 9 5 11
    assert S.distinct(chosen) == [7, 4, 2, 9, 5, 11]
    assert S.plan(layer, chosen) == [[4, 9, 7], [2, 5, 11]]


def test_step_maps_each_chunk_and_loads_its_misses():
    layer = S.LayerSlots(16, 3)
    for e in (9, 4):
        layer.lookup(e)
    chunks = S.step(layer, [7, 4, 2, 9, 7, 5, 4, 11])
    (c0, s0, l0, m0), (c1, s1, l1, m1) = chunks
    assert c0 == [4, 9, 7] and s0 == [1, 0, 2] and l0 == [(7, 2)]
    assert m0[4] == 1 and m0[9] == 0 and m0[7] == 2 and m0.count(-1) == 13
    # the second chunk evicts in LRU order: 4 (stamp 3), 9 (4), then 7 (5)
    assert c1 == [2, 5, 11] and s1 == [1, 0, 2] and l1 == [(2, 1), (5, 0), (11, 2)]
    assert layer.misses == 6 and layer.hits == 2
