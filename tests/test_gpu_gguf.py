"""GGUF loading onto the device (tmoe_gguf_load through GgufFile.load_experts / load_moe_layer): the
bytes that land in HBM equal the file's (tensors larger than one 64 MB bounce buffer included), and
a MoE layer run on the loaded tensors -- resident, and streamed from a pinned store loaded from the
file -- matches the CPU oracle on the weights gguf-py wrote."""
import numpy as np
import pytest
import torch

gguf = pytest.importorskip("gguf")

import oracle as O  # noqa: E402
import tetraeder_b200 as tb  # noqa: E402
from tests.common import nrms  # noqa: E402
from tests.gguf_fixture import write_moe_gguf  # noqa: E402
from tetraeder_b200.gguf import GgufFile  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    p = tmp_path_factory.mktemp("gg") / "tiny.gguf"
    written = write_moe_gguf(p, n_layer=1, n_embd=512, n_ff=256, n_expert=16, n_used=4, gate_type=12, down_type=12,
                             extra_kv=False)
    return p, written


def _oracle_layer(written, x, k):
    g = written["blk.0.ffn_gate_exps.weight"][1]
    u = written["blk.0.ffn_up_exps.weight"][1]
    d = written["blk.0.ffn_down_exps.weight"][1]
    rw = written["blk.0.ffn_gate_inp.weight"][1]
    E, I, H = g.shape[0], g.shape[1], x.shape[1]
    ids, w, _, _ = O.route(x, k, router_w=rw)
    return ids, O.experts(x, ids, w, g, u, d, H, I, E, O.TYPE_Q4_K, O.TYPE_Q4_K, O.TYPE_Q4_K)


def test_loaded_layer_matches_the_oracle(tiny):
    path, written = tiny
    with GgufFile(path) as f:
        hp = f.hparams
        rw, norm, ex = f.load_moe_layer(0, "cuda")
        for name, t in (("ffn_gate_exps", ex.gate), ("ffn_up_exps", ex.up), ("ffn_down_exps", ex.down)):
            assert np.array_equal(t.cpu().numpy(), written[f"blk.0.{name}.weight"][1]), name
        assert torch.equal(rw.cpu(), torch.from_numpy(written["blk.0.ffn_gate_inp.weight"][1]))
        assert torch.equal(norm.cpu(), torch.from_numpy(written["blk.0.ffn_norm.weight"][1]))
    T = 24
    x = np.random.default_rng(3).standard_normal((T, hp.n_embd)).astype(np.float32)
    layer = tb.MoeLayer(hp.n_embd, hp.n_ff_exp, hp.n_expert, hp.n_expert_used, gate_type=12, up_type=12,
                        down_type=12, max_tokens=T)
    ids = torch.empty((T, hp.n_expert_used), dtype=torch.int32, device="cuda")
    out = layer.moe_ffn(torch.from_numpy(x).cuda(), ex, router_w=rw, ids_out=ids)
    layer.check()
    want_ids, want = _oracle_layer(written, x, hp.n_expert_used)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert nrms(out.cpu().numpy(), want) < 1e-3
    layer.close()


def test_streamed_layer_from_a_store_loaded_from_the_file(tiny):
    path, written = tiny
    with GgufFile(path) as f:
        hp = f.hparams
        rw, _, _ = f.load_moe_layer(0, "cuda")
        store = f.load_experts(0, device=None, pinned=True)
    assert np.array_equal(store.down.numpy(), written["blk.0.ffn_down_exps.weight"][1])
    NS = 6
    slots = tb.ExpertWeights(*(torch.zeros((NS,) + tuple(t.shape[1:]), dtype=torch.uint8, device="cuda")
                               for t in (store.gate, store.up, store.down)))
    T = 16
    x = np.random.default_rng(4).standard_normal((T, hp.n_embd)).astype(np.float32)
    layer = tb.MoeLayer(hp.n_embd, hp.n_ff_exp, hp.n_expert, hp.n_expert_used, gate_type=12, up_type=12,
                        down_type=12, max_tokens=T)
    cache = tb.SlotCache(layer, slots, store)
    out = layer.moe_ffn_streamed(torch.from_numpy(x).cuda(), cache, router_w=rw)
    layer.check()
    _, want = _oracle_layer(written, x, hp.n_expert_used)
    assert nrms(out.cpu().numpy(), want) < 1e-3
    cache.close()
    layer.close()


def test_large_tensors_land_byte_exact(tmp_path):
    """96 C2-shaped experts: gate/up 85 MB and down 124 MB per tensor, more than one bounce buffer."""
    p = tmp_path / "big.gguf"
    written = write_moe_gguf(p, n_layer=1, n_embd=2048, n_ff=768, n_expert=96, n_used=8, gate_type=12,
                             down_type=14, quantise=False, extra_kv=False, n_vocab=64)
    with GgufFile(p) as f:
        ex = f.load_experts(0, device="cuda")
        part = f.load_experts(0, device="cuda", first=37, count=11)
    for name, t, tp in (("ffn_gate_exps", ex.gate, part.gate), ("ffn_up_exps", ex.up, part.up),
                        ("ffn_down_exps", ex.down, part.down)):
        want = torch.from_numpy(written[f"blk.0.{name}.weight"][1])
        assert torch.equal(t.cpu(), want), name
        assert torch.equal(tp.cpu(), want[37:48]), name
