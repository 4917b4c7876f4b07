"""The GGUF reader (csrc/gguf.cu, tetraeder_b200/gguf.py) against gguf-py's GGUFReader on files that
gguf-py writes: metadata of every kind, the tensor index (types, shapes, absolute offsets, sizes),
the bytes, split models, and the reference's error cases (crates/model/src/gguf.rs:236-400); the
qwen3moe hyperparameters against the expectations of the reference's own fixture test
(crates/model/tests/desc.rs:16-27) on a file of the same shape.  CPU only."""
import os
import struct

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")

from tests.gguf_fixture import write_moe_gguf  # noqa: E402
from tetraeder_b200 import _lib  # noqa: E402
from tetraeder_b200.gguf import ArrayValue, GgufError, GgufFile, type_size  # noqa: E402


def _gguf_py_value(field):
    """A gguf-py field as the reader exposes it (arrays: their length only)."""
    if field.types[0] == gguf.GGUFValueType.ARRAY:
        return ArrayValue(len(field.data))
    return field.contents()


def test_type_table_matches_gguf_py():
    from gguf.constants import GGML_QUANT_SIZES
    for t, (blck, nbytes) in GGML_QUANT_SIZES.items():
        assert type_size(int(t)) == (blck, nbytes), t
    for removed in (4, 5, 31, 32, 33, 36, 37, 38, 1000):
        with pytest.raises(GgufError):
            type_size(removed)


@pytest.fixture(scope="module")
def moe_file(tmp_path_factory):
    p = tmp_path_factory.mktemp("gguf") / "m.gguf"
    written = write_moe_gguf(p, n_layer=2, n_expert=4)
    return p, written


def test_metadata_matches_gguf_py(moe_file):
    path, _ = moe_file
    r = gguf.GGUFReader(str(path))
    with GgufFile(path) as g:
        keys = [k for k in r.fields if not k.startswith("GGUF.")]
        assert g.keys() == keys
        for k in keys:
            assert g.get(k) == _gguf_py_value(r.fields[k]), k
        assert g.get("test.f32") == float(np.float32(0.1))
        assert g.get("test.i64") == -(1 << 60) and g.get("test.u64") == 1 << 60
        assert g.get("no.such.key") is None
        with pytest.raises(GgufError, match="missing key `no.such.key`"):
            g.u64("no.such.key")
        with pytest.raises(GgufError, match="wrong type"):
            g.u64("test.str")
        with pytest.raises(GgufError, match="wrong type"):
            g.u64("test.i8")  # negative signed: not a u64 (gguf.rs:421-427)
        assert g.u64("test.u16") == 60000
        with pytest.raises(GgufError, match="wrong type"):
            g.f32("test.u32")


def test_tensor_index_and_bytes_match_gguf_py(moe_file):
    path, written = moe_file
    r = gguf.GGUFReader(str(path))
    with GgufFile(path) as g:
        assert [t.name for t in g.tensors] == [t.name for t in r.tensors]
        for t, rt in zip(g.tensors, r.tensors):
            assert t.type == int(rt.tensor_type), t.name
            ne = tuple(int(x) for x in rt.shape) + (1,) * (4 - len(rt.shape))
            assert t.ne == ne, t.name
            assert t.offset == rt.data_offset, t.name
            assert t.nbytes == rt.n_bytes, t.name
            got = g.read(t.name)
            assert np.array_equal(got, np.asarray(rt.data).view(np.uint8).reshape(-1)), t.name
            assert np.array_equal(got, written[t.name][1].view(np.uint8).reshape(-1)), t.name
        # a byte range inside a tensor, and ranges outside it
        t = g.tensor("blk.1.ffn_down_exps.weight")
        assert np.array_equal(g.read(t.name, 1000, 77), g.read(t.name)[1000:1077])
        with pytest.raises(GgufError, match="outside tensor"):
            g.read(t.name, t.nbytes - 10, 11)
        with pytest.raises(GgufError, match="missing tensor `nope`"):
            g.tensor("nope")


def test_expert_slabs_tile_the_stacked_tensors(moe_file):
    """The reference's expert_slabs_tile_the_stacked_tensors (crates/model/tests/desc.rs:75-98)."""
    path, written = moe_file
    with GgufFile(path) as g:
        E = g.hparams.n_expert
        for il in range(g.hparams.n_layer):
            for name in ("ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"):
                t = g.layer_tensor(il, name)
                slabs = [t.slab(i) for i in range(E)]
                assert t.slab(E) is None and t.slab(-1) is None
                assert slabs[0].offset == t.offset and sum(s.len for s in slabs) == t.nbytes
                for a, b in zip(slabs, slabs[1:]):
                    assert b.offset == a.offset + a.len
            down = g.layer_tensor(il, "ffn_down_exps")
            for e in range(E):
                _, _, ds = g.expert_slabs(il, e)
                got = g.read(down.name, ds.offset - down.offset, ds.len)
                assert np.array_equal(got, written[down.name][1][e].reshape(-1))
        host = g.load_experts(1, device=None, first=1, count=2)
        assert np.array_equal(host.gate.numpy(), written["blk.1.ffn_gate_exps.weight"][1][1:3])
        assert np.array_equal(host.down.numpy(), written["blk.1.ffn_down_exps.weight"][1][1:3])
        with pytest.raises(GgufError, match="out of range"):
            g.load_experts(0, device=None, first=3, count=2)


def test_hparams_of_the_reference_fixture_shape(tmp_path):
    """A file of the reference fixture's shape (xtask/tiny_moe.py: 2 layers, 64 wide, 4 heads, 2 KV
    heads of 16, 8 experts, top-2, 32-wide experts, 260 tokens, F16 matrices) gives the hparams
    the reference asserts (crates/model/tests/desc.rs:16-27)."""
    p = tmp_path / "tiny.gguf"
    write_moe_gguf(p, n_layer=2, n_embd=64, n_head=4, n_head_kv=2, head_dim=16, n_expert=8, n_used=2, n_ff=32,
                   n_vocab=260, gate_type=1, down_type=1, extra_kv=False)
    with GgufFile(p) as g:
        h = g.hparams
        assert (h.n_layer, h.n_embd, h.n_head, h.n_head_kv, h.head_dim) == (2, 64, 4, 2, 16)
        assert (h.n_expert, h.n_expert_used, h.n_ff_exp) == (8, 2, 32)
        assert h.n_vocab == 260
        assert not h.tied_output
        assert g.expert_types(0) == (1, 1, 1)
        # desc.rs:94-97: one expert's three F16 slabs, and the out-of-range ones
        assert sum(s.len for s in g.expert_slabs(1, 3)) == 3 * 32 * 64 * 2
        with pytest.raises(GgufError):
            g.expert_slabs(0, 8)
        with pytest.raises(GgufError):
            g.expert_slabs(2, 0)
        with pytest.raises(GgufError, match="Q4_K"):
            g.load_moe_layer(0, device="cpu")
    p2 = tmp_path / "tied.gguf"
    write_moe_gguf(p2, n_layer=1, tied=True, extra_kv=False)
    with GgufFile(p2) as g:
        assert g.hparams.tied_output


def test_split_model(tmp_path):
    """A split model (gguf-py's split writer, llama.cpp's naming) opens from its first shard and
    merges the tensor index; the other shards are rejected as entry points (gguf.rs:241-279)."""
    written = write_moe_gguf(tmp_path / "s.gguf", n_layer=2, split_max_tensors=6)
    shards = sorted(os.listdir(tmp_path))
    assert len(shards) >= 3 and shards[0].endswith(f"-00001-of-{len(shards):05d}.gguf"), shards
    first = tmp_path / shards[0]
    with GgufFile(first) as g:
        assert g.n_shards == len(shards)
        assert sorted(t.name for t in g.tensors) == sorted(written)
        assert {t.shard for t in g.tensors} == set(range(len(shards)))
        for t in g.tensors:
            assert np.array_equal(g.read(t.name), written[t.name][1].view(np.uint8).reshape(-1)), t.name
        assert g.hparams.n_layer == 2
    with pytest.raises(GgufError, match="not the first shard"):
        GgufFile(tmp_path / shards[1])
    renamed = tmp_path / "renamed.gguf"
    os.rename(first, renamed)
    with pytest.raises(GgufError, match="should be named"):
        GgufFile(renamed)
    os.rename(renamed, first)
    os.remove(tmp_path / shards[-1])
    with pytest.raises(GgufError, match="cannot read GGUF"):
        GgufFile(first)


def test_corrupt_files(tmp_path, moe_file):
    path, _ = moe_file
    data = open(path, "rb").read()

    def case(blob, match):
        p = tmp_path / "bad.gguf"
        p.write_bytes(blob)
        with pytest.raises(GgufError, match=match):
            GgufFile(p)

    case(b"GGML" + data[4:], "bad magic")
    case(data[:4] + struct.pack("<I", 2) + data[8:], "unsupported GGUF version 2")
    case(data[:8] + struct.pack("<Q", 1 << 40) + data[16:], "implausible counts")
    case(data[:200], "truncated")
    case(data[:-1000], "runs past the end")
    case(b"", "bad magic")
    with pytest.raises(GgufError, match="cannot read GGUF"):
        GgufFile(tmp_path / "absent.gguf")
    lib = _lib.load()
    assert lib.tmoe_gguf_n_tensors(None) == -1
    assert lib.tmoe_gguf_open(None, None) == -1


def _reference_fixture():
    """The reference's own fixture model (tests/fixtures/tiny-qwen3moe-f16.gguf of the tetraeder tree,
    written by its xtask/tiny_moe.py), found through TETRAEDER_REFERENCE = the root of that tree."""
    root = os.environ.get("TETRAEDER_REFERENCE")
    p = os.path.join(root, "tests", "fixtures", "tiny-qwen3moe-f16.gguf") if root else None
    if not p or not os.path.exists(p):
        pytest.skip("TETRAEDER_REFERENCE does not point at a tetraeder tree with its fixture model")
    return p


def test_reference_fixture_matches_golden():
    """This reader on the reference's fixture model agrees with gguf-py's reading of it, as recorded
    in tests/golden/tiny_qwen3moe_f16.json by tests/golden/make_gguf_golden.py: every metadata value,
    the tensor index (type, shape, absolute offset, size) and the sha256 of every tensor's bytes; and
    the hparams are those the reference's desc test asserts (crates/model/tests/desc.rs:16-27)."""
    import hashlib
    import json
    path = _reference_fixture()
    here = os.path.dirname(os.path.abspath(__file__))
    with open(os.path.join(here, "golden", "tiny_qwen3moe_f16.json")) as f:
        gold = json.load(f)
    assert os.path.getsize(path) == gold["bytes"]
    with GgufFile(path) as g:
        assert sorted(g.keys()) == sorted(gold["kv"])
        for k, v in gold["kv"].items():
            got = g.get(k)
            assert got == (ArrayValue(v["array_len"]) if isinstance(v, dict) else v), k
        assert [t.name for t in g.tensors] == [t["name"] for t in gold["tensors"]]
        for t, gt in zip(g.tensors, gold["tensors"]):
            assert t.type == gt["type"], t.name
            assert t.ne == tuple(gt["shape"]) + (1,) * (4 - len(gt["shape"])), t.name
            assert (t.offset, t.nbytes) == (gt["offset"], gt["nbytes"]), t.name
            assert hashlib.sha256(g.read(t.name).tobytes()).hexdigest() == gt["sha256"], t.name
        h = g.hparams
        assert (h.n_layer, h.n_embd, h.n_head, h.n_head_kv, h.head_dim) == (2, 64, 4, 2, 16)
        assert (h.n_expert, h.n_expert_used, h.n_ff_exp, h.n_vocab) == (8, 2, 32, 260)
        assert sum(s.len for s in g.expert_slabs(1, 3)) == 3 * 32 * 64 * 2
