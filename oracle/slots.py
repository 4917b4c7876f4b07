"""CPU restatement of the reference's expert-slot cache and streamed-step planner (TEST
INFRASTRUCTURE: the checker of the device-side slot planner; never part of the product).

Follows, in the reference tree:
- `LayerSlots` (crates/memory/src/slots.rs:67-262): `lookup` / `lookup_except` (:131-177: hit ->
  refresh the stamp; miss -> the first free slot below `active`, else the unpinned slot with the
  smallest stamp that is not protected; none -> bypass), `clear` (:181-185), `set_hot_set`
  (:189-207), `set_active` (:211-255);
- `hot_from_counts` (the top experts by routing count, ties to the lower id, zero counts dropped;
  pinned by slots.rs:755-761);
- `Streamer::distinct` / `plan` (crates/model/src/experts.rs:624-662): the distinct experts of a
  layer step in order of first appearance, resident ones first, in chunks of `active`;
- `make_resident` (experts.rs:1507-1543): a plain `lookup` per expert of a chunk, a load for each
  miss, an error on a bypass;
- `map_ids` (crates/model/src/qwen3moe.rs:2108-2120) for the one-chunk case.

Pure Python: the tables are at most a few hundred entries.
"""
from __future__ import annotations

from dataclasses import dataclass, field

HIT, MISS, BYPASS = "hit", "miss", "bypass"


@dataclass
class Lookup:
    kind: str
    slot: int = -1
    evicted: int = -1  # -1: none

    def __eq__(self, other):  # compare like the reference's enum
        return (self.kind, self.slot, self.evicted) == (other.kind, other.slot, other.evicted)


@dataclass
class LayerSlots:
    experts: int
    max: int
    active: int = -1
    table: dict = field(default_factory=dict)
    owner: list = field(default_factory=list)
    stamp: list = field(default_factory=list)
    clock: int = 0
    pinned: list = field(default_factory=list)
    pinned_count: int = 0
    hits: int = 0
    misses: int = 0
    bypass: int = 0

    def __post_init__(self):
        self.active = self.max
        self.owner = [-1] * self.max
        self.stamp = [0] * self.max
        self.pinned = [False] * self.experts

    def slot_of(self, e: int) -> int:
        return self.table.get(e, -1)

    def lookup(self, e: int) -> Lookup:
        return self.lookup_except(e, ())

    def lookup_except(self, e: int, protect) -> Lookup:
        if e >= self.experts or e < 0:
            self.bypass += 1
            return Lookup(BYPASS)
        self.clock += 1
        if e in self.table:
            s = self.table[e]
            self.stamp[s] = self.clock
            self.hits += 1
            return Lookup(HIT, s)
        slot = -1
        for s in range(self.active):  # the first free slot
            if self.owner[s] < 0:
                slot = s
                break
        if slot < 0:  # else the least recently used unpinned, unprotected slot (first on ties)
            best = None
            for s in range(self.active):
                o = self.owner[s]
                if o >= 0 and not self.pinned[o] and o not in protect:
                    if best is None or self.stamp[s] < self.stamp[best]:
                        best = s
            if best is None:
                self.bypass += 1
                return Lookup(BYPASS)
            slot = best
        evicted = self.owner[slot]
        if evicted >= 0:
            del self.table[evicted]
        self.owner[slot] = e
        self.table[e] = slot
        self.stamp[slot] = self.clock
        self.misses += 1
        return Lookup(MISS, slot, evicted)

    def clear(self):
        self.table.clear()
        self.owner = [-1] * self.max
        self.stamp = [0] * self.max

    def set_hot_set(self, hot) -> list:
        self.pinned = [False] * self.experts
        self.pinned_count = 0
        for e in hot:
            if self.pinned_count < self.active and 0 <= e < self.experts and not self.pinned[e]:
                self.pinned[e] = True
                self.pinned_count += 1
        return [e for e in range(self.experts) if self.pinned[e] and e not in self.table]

    def set_active(self, n: int):
        n = min(max(n, self.pinned_count), self.max)
        evicted, moved = [], []
        for slot in range(self.active - 1, n - 1, -1):
            e = self.owner[slot]
            if e < 0:
                continue
            self.owner[slot] = -1
            del self.table[e]
            if not self.pinned[e]:
                evicted.append((e, slot))
                continue
            to = next((s for s in range(n) if self.owner[s] < 0), None)
            if to is None:
                cands = [s for s in range(n) if self.owner[s] >= 0 and not self.pinned[self.owner[s]]]
                to = min(cands, key=lambda s: self.stamp[s])
            old = self.owner[to]
            if old >= 0:
                del self.table[old]
                evicted.append((old, to))
            self.owner[to] = e
            self.table[e] = to
            self.stamp[to] = self.stamp[slot]
            moved.append((e, slot, to))
        self.active = n
        return evicted, moved


def hot_from_counts(counts, n: int) -> list:
    """The top `n` experts by count, ties to the lower id, zero counts left out."""
    order = sorted((e for e in range(len(counts)) if counts[e] > 0), key=lambda e: (-counts[e], e))
    return order[:n]


def distinct(chosen) -> list:
    """Distinct experts in order of first appearance (experts.rs:624-639)."""
    seen, out = set(), []
    for e in chosen:
        e = int(e)
        if e not in seen:
            seen.add(e)
            out.append(e)
    return out


def plan(layer: LayerSlots, chosen) -> list:
    """Chunks of a layer step: resident experts first, then the misses, each part in order of first
    appearance, cut into chunks of `active` (experts.rs:644-662)."""
    d = distinct(chosen)
    hits = [e for e in d if layer.slot_of(e) >= 0]
    misses = [e for e in d if layer.slot_of(e) < 0]
    order = hits + misses
    n = max(layer.active, 1)
    return [order[i:i + n] for i in range(0, len(order), n)]


def make_resident(layer: LayerSlots, chunk) -> tuple[list, list]:
    """Slots of the chunk's experts and the (expert, slot) loads of its misses (experts.rs:1507-1527).
    A bypass raises, as the reference's `no free expert slot (all pinned)` error does."""
    slots, loads = [], []
    for e in chunk:
        r = layer.lookup(e)
        if r.kind == BYPASS:
            raise RuntimeError("no free expert slot (all pinned)")
        slots.append(r.slot)
        if r.kind == MISS:
            loads.append((e, r.slot))
    return slots, loads


def step(layer: LayerSlots, chosen) -> list:
    """One streamed layer step: per chunk, (chunk, slots, loads, map) where map[e] is the slot of
    expert e for the experts of the chunk and -1 for every other expert."""
    out = []
    for chunk in plan(layer, chosen):
        slots, loads = make_resident(layer, chunk)
        m = [-1] * layer.experts
        for e, s in zip(chunk, slots):
            m[e] = s
        out.append((chunk, slots, loads, m))
    return out
