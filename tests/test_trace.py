"""The routing-trace reader and writer (csrc/trace.cu, tetraeder_b200/trace.py) against the
reference's own tests of the format (crates/memory/src/replay/trace.rs:332-437): round trips with
1- and 2-byte ids, a file cut at every byte, bad ids and lengths, corrupt token counts, foreign
headers; plus the header's JSON as serde_json writes it, and replay logits that reproduce the
recorded choice through the router's top-k.  CPU only."""
import json
import struct

import numpy as np
import pytest

import oracle as O
from tetraeder_b200.trace import HotRefresh, LayerStep, TraceError, TraceHeader, TraceReader, TraceWriter


def header(n_expert):
    h = TraceHeader(3, n_expert, 2)
    h.model = "test"
    h.vram_slots = 4
    h.ram_slots = 8
    h.expert_bytes = [100, 200, 300]
    return h


def write_sample(path, n_expert):
    big = n_expert - 1
    with TraceWriter(path, header(n_expert)) as w:
        w.layer_step(0, 0, [0, big, 1, 2], predicted=[3, 4, 5, 6])
        w.layer_step(0, 1, [7, 8, 9, big], predicted2=[1, 1, 2, 2])
        w.hot_refresh(0)
        w.layer_step(1, 2, [5, big], predicted=[1, 2], predicted2=[big, 0])
    return path.read_bytes()


@pytest.mark.parametrize("n_expert", [128, 1000])
def test_roundtrip(tmp_path, n_expert):
    """roundtrip_u8_ids / roundtrip_u16_ids (trace.rs:367-404)."""
    p = tmp_path / "t.bin"
    write_sample(p, n_expert)
    big = n_expert - 1
    with TraceReader(p) as r:
        assert r.header == header(n_expert)
        assert r.header.id_bytes == (1 if n_expert <= 256 else 2)
        recs = list(r)
    assert len(recs) == 4
    s0 = recs[0]
    assert isinstance(s0, LayerStep) and (s0.step, s0.layer, s0.n_tokens) == (0, 0, 2)
    assert s0.ids.tolist() == [[0, big], [1, 2]] and s0.predicted.tolist() == [[3, 4], [5, 6]]
    assert s0.predicted2 is None
    assert recs[1].predicted is None and recs[1].predicted2.reshape(-1).tolist() == [1, 1, 2, 2]
    assert recs[2] == HotRefresh(0)
    assert recs[3].step == 1 and recs[3].layer == 2 and recs[3].predicted2.reshape(-1).tolist() == [big, 0]


def test_header_json_is_serde_json_compact(tmp_path):
    """The header line as serde_json serialises TraceHeader: declaration order, no spaces, no
    `profile` when absent; with a profile, it is appended."""
    p = tmp_path / "t.bin"
    data = write_sample(p, 128)
    line = data[:data.index(b"\n")].decode()
    assert line == ('{"format":"tetraeder-routing","version":1,"model":"test","n_layer":3,"n_expert":128,'
                    '"n_used":2,"id_bytes":1,"vram_slots":4,"ram_slots":8,"prefetch_depth":0,'
                    '"hot_source":"first_prefill","ubatch":0,"prompt_hash":"","expert_bytes":[100,200,300]}')
    h = header(4)
    h.profile = [[1, 2, 3, 4], [5, 6, 7, 8], [0, 0, 0, 9]]
    h.model = 'quote " and \\ and \n and ∆'
    with TraceWriter(tmp_path / "p.bin", h) as w:
        w.layer_step(7, 1, [3, 0])
    with TraceReader(tmp_path / "p.bin") as r:
        assert r.header == h
        assert json.loads(r.header_json) == json.loads(h.to_json())
        assert r.header_json.endswith('"profile":[[1,2,3,4],[5,6,7,8],[0,0,0,9]]}')
        assert [s.ids.tolist() for s in r] == [[[3, 0]]]


def test_truncated_file_is_an_error_not_a_crash(tmp_path):
    """truncated_file_is_an_error_not_a_panic (trace.rs:416-441)."""
    p = tmp_path / "t.bin"
    data = write_sample(p, 128)
    full = 4
    header_len = data.index(b"\n") + 1
    errors = 0
    cut_path = tmp_path / "cut.bin"
    for cut in range(len(data)):
        cut_path.write_bytes(data[:cut])
        try:
            r = TraceReader(cut_path)
        except TraceError:
            assert cut < header_len
            continue
        got, failed = [], False
        try:
            for rec in r:
                got.append(rec)
        except TraceError:
            failed = True
        r.close()
        if failed:
            errors += 1
        else:
            assert len(got) < full  # a cut on a record boundary: fewer records, never more
    assert errors > 0


def test_rejects_bad_ids_and_lengths(tmp_path):
    """rejects_bad_ids_and_lengths (trace.rs:443-449): nothing of a rejected record is written."""
    p = tmp_path / "t.bin"
    with TraceWriter(p, header(16)) as w:
        with pytest.raises(TraceError, match="out of range"):
            w.layer_step(0, 0, [0, 16])
        with pytest.raises(TraceError, match="out of range"):
            w.layer_step(0, 0, [-1, 2])
        with pytest.raises(TraceError):
            w.layer_step(0, 0, [0, 1, 2])
        with pytest.raises(TraceError, match="ids for"):
            w.layer_step(0, 0, [0, 1], predicted=[1, 2, 3, 4])
        w.layer_step(0, 0, [0, 15])
    with TraceReader(p) as r:
        assert [s.ids.tolist() for s in r] == [[[0, 15]]]


@pytest.mark.parametrize("n_tokens", [2**32 - 1, 2**20 + 1, 2**20])
def test_corrupt_token_count_is_an_error(tmp_path, n_tokens):
    """corrupt_token_count_is_an_error_not_a_huge_allocation (trace.rs:451-467)."""
    p = tmp_path / "t.bin"
    with TraceWriter(p, header(128)):
        pass
    rec = bytes([0]) + struct.pack("<IHI", 0, 0, n_tokens) + bytes([3])
    p.write_bytes(p.read_bytes() + rec)
    with TraceReader(p) as r:
        with pytest.raises(TraceError):
            next(r)


def test_rejects_foreign_headers(tmp_path):
    """rejects_foreign_headers (trace.rs:469-473), and the header check (trace.rs:75-89)."""
    cases = [b"{}\n", b"not json\n", b'{"format":"other"}\n']
    good = json.loads(header(128).to_json())
    for k, v in [("format", "other"), ("version", 2), ("id_bytes", 2), ("n_used", 0), ("expert_bytes", [1]),
                 ("n_layer", -1), ("n_layer", 1.5), ("ubatch", 2**32)]:
        cases.append((json.dumps({**good, k: v}) + "\n").encode())
    missing = dict(good)
    del missing["hot_source"]
    cases.append((json.dumps(missing) + "\n").encode())
    cases.append(b'{"format":"tetraeder-routing","format":"tetraeder-routing"}\n')
    for i, blob in enumerate(cases):
        p = tmp_path / f"h{i}.bin"
        p.write_bytes(blob)
        with pytest.raises(TraceError):
            TraceReader(p)
    # unknown fields are ignored, as serde does
    p = tmp_path / "extra.bin"
    p.write_bytes((json.dumps({**good, "future_field": {"x": [1, None]}}) + "\n").encode())
    with TraceReader(p) as r:
        assert r.header == header(128) and list(r) == []


def test_replay_logits_reproduce_the_recorded_choice():
    """A recorded step replayed through the router: softmax top-k of LayerStep.logits (the oracle's
    routing, lower index first on ties) gives back the recorded ids in order."""
    rng = np.random.default_rng(5)
    E, k, T = 128, 8, 64
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    s = LayerStep(0, 0, T, ids)
    got, _, _, _ = O.route(np.zeros((T, 16), np.float32), k, logits=s.logits(E))
    assert np.array_equal(got, ids)
