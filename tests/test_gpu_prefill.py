"""The large-batch regime (T * k >= 6144 pairs): gate/up on the integer MMA path (exact Q8_K block
sums, as on the reference CPU path) and the down product as a grouped tcgen05 GEMM with fp16
operands (the SwiGLU activations through the same Q8_K round trip as on the reference path, then
fp16; the down weights dequantised to fp16), checked against the CPU oracle on the same inputs.

The fp16 down product is the only departure from the reference's integer sums; a numpy model of
exactly these roundings puts the 30B-shaped case at 3.4e-4 normalised RMS and 9.5e-3 x RMS max-abs,
so the bound here is 1e-3 / 2.5e-2 (1e-2 / 5e-2, is checked too).  fp16 in
gate/up instead moves enough activations across a Q8_K rounding boundary to reach 5.6e-2 max-abs,
which is why gate/up stay integer."""
import numpy as np
import pytest
import torch

import oracle as O
import tetraeder_b200 as tb
from tests.common import maxabs_over_rms, nrms, quantized_experts

pytestmark = pytest.mark.gpu

NORTH_NRMS, NORTH_MAXABS = 1e-2, 5e-2
PREFILL_NRMS, PREFILL_MAXABS = 1e-3, 2.5e-2


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _case(H, I, E, T, gt, dt, seed, exact):
    rng = np.random.default_rng(seed)
    gate = quantized_experts(rng, gt, E, I, H, exact=exact)
    up = quantized_experts(rng, gt, E, I, H, exact=exact)
    down = quantized_experts(rng, dt, E, H, I, exact=exact)
    rw = (rng.standard_normal((E, H)) * 0.02).astype(np.float32)
    x = rng.standard_normal((T, H)).astype(np.float32)
    return gate, up, down, rw, x


PREFILL_CASES = [
    # (name, H, I, E, k, T, gate/up type, down type, exact quantiser)
    ("tiny T=1536", 512, 256, 16, 4, 1536, O.TYPE_Q4_K, O.TYPE_Q4_K, True),
    ("C2 30B T=768", 2048, 768, 128, 8, 768, O.TYPE_Q4_K, O.TYPE_Q6_K, False),
    ("C4 235B shape T=768", 4096, 1536, 16, 8, 768, O.TYPE_Q4_K, O.TYPE_Q4_K, False),
]


@pytest.mark.parametrize("case", PREFILL_CASES, ids=[c[0] for c in PREFILL_CASES])
def test_prefill_layer_parity(case):
    name, H, I, E, k, T, gt, dt, exact = case
    gate, up, down, rw, x = _case(H, I, E, T, gt, dt, 100 + len(name), exact)
    layer = tb.MoeLayer(H, I, E, k, gate_type=gt, up_type=gt, down_type=dt, max_tokens=T)
    wts = tb.ExpertWeights(cuda(gate), cuda(up), cuda(down))
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    layer.profile(True)
    out = layer.moe_ffn(cuda(x), wts, router_w=cuda(rw), ids_out=ids, w_out=w)
    phases = layer.profile_collect()
    layer.profile(False)
    # the grouped GEMMs ran, not the decode GEMV (whose activations take a separate Q8_K pass)
    assert "gate_up" in phases and "quant_act" not in phases, f"{name}: phases {sorted(phases)}"
    out2 = layer.moe_ffn(cuda(x), wts, router_w=cuda(rw))  # again: tiles and buffers are reused
    layer.check()
    want_ids, want_w, _, _ = O.route(x, k, router_w=rw)
    assert np.array_equal(ids.cpu().numpy(), want_ids), name
    want = O.experts(x, want_ids, want_w, gate, up, down, H, I, E, gt, gt, dt)
    for got in (out.cpu().numpy(), out2.cpu().numpy()):
        n, m = nrms(got, want), maxabs_over_rms(got, want)
        assert n <= NORTH_NRMS and m <= NORTH_MAXABS, f"{name}: north-star bound nrms={n:.2e} maxabs/rms={m:.2e}"
        assert n <= PREFILL_NRMS and m <= PREFILL_MAXABS, f"{name}: nrms={n:.2e} maxabs/rms={m:.2e}"
    layer.close()
