"""The decode step of the whole Qwen3-MoE model (tetraeder_b200.model) against the CPU oracle of the
same step (oracle/model.py), on a tiny qwen3moe GGUF written by gguf-py with Q4_K/Q6_K matrices:
several sequences decoded over several positions (the F16 KV cache grows step by step), eager and
replayed from a CUDA graph; plus the attention op alone against a float64 softmax over a random
cache, at both head sizes and with a long context (many splits)."""
import numpy as np
import pytest
import torch

gguf = pytest.importorskip("gguf")

import oracle as O  # noqa: E402
from oracle.model import Matrix, ModelOracle  # noqa: E402
import tetraeder_b200 as tb  # noqa: E402
from tests.common import nrms  # noqa: E402
from tests.gguf_fixture import write_moe_gguf  # noqa: E402
from tetraeder_b200.gguf import GgufFile  # noqa: E402
from tetraeder_b200.model import Qwen3MoeModel  # noqa: E402

pytestmark = pytest.mark.gpu


def _oracle_weights(written, hp):
    w = {}
    for name, (t, arr) in written.items():
        if t == O.TYPE_F32 and (arr.ndim == 1 or name.endswith("ffn_gate_inp.weight")):
            w[name] = arr
        elif name.endswith("_exps.weight"):
            w[name] = Matrix(t, arr, arr.shape[0] * arr.shape[1], 0)
        else:
            rows = arr.shape[0]
            cols = arr.shape[1] if t in (O.TYPE_F16, O.TYPE_F32) else hp.n_embd if not name.endswith(
                "attn_output.weight") else hp.n_head * hp.head_dim
            w[name] = Matrix(t, arr, rows, cols)
    return w


@pytest.fixture(scope="module")
def tiny_model(tmp_path_factory):
    p = tmp_path_factory.mktemp("model") / "tiny-qwen3moe.gguf"
    written = write_moe_gguf(p, n_layer=2, n_embd=512, n_head=4, n_head_kv=2, head_dim=128, n_expert=8, n_used=2,
                             n_ff=256, n_vocab=512, gate_type=12, down_type=14, attn_types=(12, 12, 14, 12),
                             embd_type=12, out_type=14, extra_kv=False)
    return p, written


def test_decode_steps_match_the_oracle(tiny_model):
    path, written = tiny_model
    B, steps, n_ctx = 3, 6, 64
    with GgufFile(path) as f:
        hp = f.hparams
        model = Qwen3MoeModel.from_gguf(f, max_batch=B, n_ctx=n_ctx)
    ref = ModelOracle(hp, _oracle_weights(written, hp), B, n_ctx)
    rng = np.random.default_rng(5)
    start = np.array([0, 3, 17], dtype=np.int32)  # sequences at different lengths
    try:
        for s in range(steps):
            toks = rng.integers(0, hp.n_vocab, B).astype(np.int32)
            pos = (start + s).astype(np.int32)
            got = model.decode(torch.from_numpy(toks).cuda(), torch.from_numpy(pos).cuda()).cpu().numpy()
            model.check()
            want = ref.decode(toks, pos)  # positions never written read as zeros on both sides
            n = nrms(got, want)
            # Attention's probabilities enter the tensor cores as f16 (as in ggml's flash attention); the
            # next projection re-quantises its input to Q8_K, which turns those last-bit differences into
            # a few flipped 8-bit roundings per step: about 1.5e-2 of the logits over two layers here.
            # The ops themselves are held tighter below.
            assert n < 5e-2, f"step {s}: logits nrms {n:.2e}"
        nt = model.next_tokens.cpu().numpy()
        assert np.array_equal(nt, np.argmax(got, axis=1)), "argmax"
    finally:
        model.close()


def test_graph_replay_matches_eager(tiny_model):
    path, _ = tiny_model
    B, n_ctx = 2, 32
    with GgufFile(path) as f:
        a = Qwen3MoeModel.from_gguf(f, max_batch=B, n_ctx=n_ctx)
        b = Qwen3MoeModel.from_gguf(f, max_batch=B, n_ctx=n_ctx)
    toks = torch.tensor([5, 9], dtype=torch.int32, device="cuda")
    pos = torch.tensor([0, 0], dtype=torch.int32, device="cuda")
    try:
        b.decode(toks, pos)  # sizes the projections' workspace, fills position 0
        a.decode(toks, pos)
        torch.cuda.synchronize()
        g = b.graph(toks, pos)
        for step in range(1, 4):
            toks.copy_(torch.tensor([step * 7 % 512, step * 11 % 512], dtype=torch.int32))
            pos.fill_(step)
            want = a.decode(toks, pos).clone()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(b.logits[:B], want), f"step {step}"
        b.check()
        del g
    finally:
        a.close()
        b.close()


@pytest.mark.parametrize("hd,nh,nkv,ctx", [(128, 32, 4, 4096), (64, 4, 2, 100), (128, 8, 8, 1)])
def test_attention_op_against_float64(hd, nh, nkv, ctx):
    B = 3
    layer = tb.MoeLayer(512, 256, 8, 2, gate_type=12, up_type=12, down_type=12, max_tokens=4)
    lib, h = layer.lib, layer.h
    rng = np.random.default_rng(hd + nh)
    kc = (rng.standard_normal((B, ctx, nkv, hd)) * 0.5).astype(np.float16)
    vc = rng.standard_normal((B, ctx, nkv, hd)).astype(np.float16)
    q = rng.standard_normal((B, nh, hd)).astype(np.float32)
    k = rng.standard_normal((B, nkv, hd)).astype(np.float32)
    v = rng.standard_normal((B, nkv, hd)).astype(np.float32)
    pos = np.array([ctx - 1, ctx // 2, 0], dtype=np.int32)
    d_kc, d_vc = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    out = torch.empty((B, nh, hd), device="cuda")
    nbytes = lib.tmoe_attn_decode_scratch_bytes(h, B, nh, nkv, hd, ctx)
    scratch = torch.empty(nbytes // 4 + 1, device="cuda")
    import ctypes as C
    dq, dk, dv, dp = (torch.from_numpy(a).cuda() for a in (q, k, v, pos))
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    scale = 1.0 / np.sqrt(hd)
    assert lib.tmoe_attn_decode(h, None, P(dq), P(dk), P(dv), P(d_kc), P(d_vc), P(dp), B, nh, nkv, hd, ctx, scale,
                                P(scratch), P(out)) == 0
    layer.check()
    got = out.cpu().numpy()
    G = nh // nkv
    q16 = q.astype(np.float16)  # the Q operand as flash attention takes it over an F16 cache
    for b in range(B):
        kc[b, pos[b]] = k[b].astype(np.float16)
        vc[b, pos[b]] = v[b].astype(np.float16)
        K, V = kc[b, :pos[b] + 1].astype(np.float64), vc[b, :pos[b] + 1].astype(np.float64)
        for hh in range(nh):
            s = K[:, hh // G] @ q16[b, hh].astype(np.float64) * np.float64(np.float32(scale))
            e = np.exp(s - s.max())
            want = e @ V[:, hh // G] / e.sum()
            # Q, K, P and V enter the tensor cores as f16 (f32 accumulation), as in ggml's own flash attention
            assert np.abs(got[b, hh] - want).max() < 5e-3 * max(1.0, np.abs(want).max()), (b, hh)
    # the new rows landed in the caches
    assert np.array_equal(d_kc.cpu().numpy()[np.arange(B), pos], k.astype(np.float16))
    layer.close()


@pytest.mark.parametrize("qtype,K,N,T", [(12, 2048, 4096, 64), (14, 2048, 512, 3), (12, 512, 151936 // 64 * 16, 5),
                                         (12, 4096, 2048, 64), (12, 2048, 512, 50), (12, 1024, 256, 1),
                                         (14, 2048, 512, 64)])
def test_mul_mat_against_the_oracle(qtype, K, N, T):
    """tmoe_mul_mat (one matrix, every row of x) against the oracle's mul_mat_id with one expert, and
    reuse_x: a second matrix of the same family over the same x, and the guard on a mismatch.  The
    Q4_K shapes with few row tiles take the K-split product (2 or 4 slices, ragged token groups)."""
    import ctypes as C
    rng = np.random.default_rng(K + N + T)
    W = np.ascontiguousarray(O.quantize(qtype, (rng.standard_normal((N, K)) * 0.05).astype(np.float32)))
    W2 = np.ascontiguousarray(O.quantize(qtype, (rng.standard_normal((16, K)) * 0.05).astype(np.float32)))
    x = rng.standard_normal((T, K)).astype(np.float32)
    layer = tb.MoeLayer(512, 256, 8, 2, gate_type=12, up_type=12, down_type=12, max_tokens=4)
    lib, h = layer.lib, layer.h
    dW, dW2, dx = (torch.from_numpy(a).cuda() for a in (W, W2, x))
    out, out2 = torch.empty((T, N), device="cuda"), torch.empty((T, 16), device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    nb1 = W.shape[1] if W.ndim == 2 else W.shape[-1]
    assert lib.tmoe_mul_mat(h, None, qtype, P(dW), nb1, K, N, P(dx), T, 0, P(out)) == 0
    assert lib.tmoe_mul_mat(h, None, qtype, P(dW2), nb1, K, 16, P(dx), T, 1, P(out2)) == 0
    other = 14 if qtype == 12 else 12
    assert lib.tmoe_mul_mat(h, None, other, P(dW2), nb1, K, 16, P(dx), T, 1, P(out2)) != 0  # another family
    layer.check()
    for w_, o_, n_ in ((W, out, N), (W2, out2, 16)):
        want = O.mul_mat_id(qtype, w_.reshape(1, n_, -1), K, n_, 1, x[:, None, :], np.zeros((T, 1), np.int32))[:, 0]
        got = o_.cpu().numpy()
        assert np.abs(got - want).max() <= 1e-4 * max(1.0, np.abs(want).max())
    layer.close()


@pytest.mark.parametrize("d,n_rot", [(128, 128), (64, 32)])
def test_qk_norm_rope_against_the_oracle(d, n_rot):
    """The fused per-head norms + NeoX RoPE of Q and K against the oracle's rms_norm and rope_neox."""
    import ctypes as C
    from oracle.model import rms_norm, rope_neox
    T, nh, nkv, base, eps = 5, 8, 2, 1e6, 1e-6
    rng = np.random.default_rng(d + n_rot)
    q = rng.standard_normal((T, nh, d)).astype(np.float32)
    k = rng.standard_normal((T, nkv, d)).astype(np.float32)
    qw = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    kw = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    pos = np.array([0, 1, 7, 300, 4095], dtype=np.int32)
    layer = tb.MoeLayer(512, 256, 8, 2, gate_type=12, up_type=12, down_type=12, max_tokens=4)
    dq, dk, dqw, dkw, dp = (torch.from_numpy(a).cuda() for a in (q, k, qw, kw, pos))
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    assert layer.lib.tmoe_qk_norm_rope(layer.h, None, P(dq), P(dk), P(dqw), P(dkw), P(dp), T, nh, nkv, d, n_rot,
                                       base, eps) == 0
    layer.check()
    for got, x, w in ((dq, q, qw), (dk, k, kw)):
        want = rope_neox(rms_norm(x, w, eps), pos, n_rot, base)
        assert np.abs(got.cpu().numpy() - want).max() < 1e-4 * max(1.0, np.abs(want).max())
    layer.close()


@pytest.mark.parametrize("rows,H", [(3, 2048), (64, 2048), (2048, 4096), (4097, 2048), (64, 100)])
def test_rms_norm_bit_exact(rows, H):
    """tmoe_rms_norm against the oracle's rms_norm, bit for bit: a CTA per row (few long rows) and
    a warp per row (many rows, or short ones), with and without the weight."""
    import ctypes as C
    from oracle.model import rms_norm
    rng = np.random.default_rng(rows * 7 + H)
    x = (rng.standard_normal((rows, H)) * rng.uniform(0.01, 30.0, (rows, 1))).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)
    layer = tb.MoeLayer(512, 256, 8, 2, gate_type=12, up_type=12, down_type=12, max_tokens=4)
    dx, dw = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    out = torch.empty_like(dx)
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    for wt, wn in ((P(dw), w), (None, None)):
        assert layer.lib.tmoe_rms_norm(layer.h, None, P(dx), wt, 1e-6, rows, H, P(out)) == 0
        layer.check()
        assert np.array_equal(out.cpu().numpy(), rms_norm(x, wn, 1e-6))
    layer.close()


@pytest.mark.parametrize("rows,n", [(64, 151936), (5, 151935), (2, 7)])
def test_argmax_first_index(rows, n):
    """tmoe_argmax against numpy's argmax (the first index of the maximum): planted ties on the same
    row, a row of -inf, both the four-wide (n % 4 == 0) and the scalar path."""
    import ctypes as C
    rng = np.random.default_rng(rows + n)
    x = rng.standard_normal((rows, n)).astype(np.float32)
    x[0, n // 3] = x[0, n - 1] = x[0, 1] = 50.0  # three ties: index 1 wins
    x[-1, :] = -np.inf
    if rows > 2:
        x[1, n - 1] = 99.0  # the maximum at the row's last element
    layer = tb.MoeLayer(512, 256, 8, 2, gate_type=12, up_type=12, down_type=12, max_tokens=4)
    dx = torch.from_numpy(x).cuda()
    out = torch.empty(rows, dtype=torch.int32, device="cuda")
    assert layer.lib.tmoe_argmax(layer.h, None, C.c_void_p(dx.data_ptr()), rows, n, C.c_void_p(out.data_ptr())) == 0
    layer.check()
    assert np.array_equal(out.cpu().numpy(), np.argmax(x, axis=1).astype(np.int32))
    layer.close()


def test_mul_mat_beyond_l2_matches_row_slices():
    """A matrix larger than L2 (here 67.7 MB of Q4_K) takes the batch as one entry, its token passes
    over each row tile back to back; its rows must equal, bit for bit, those of the same matrix
    multiplied in two halves below the threshold (16-token groups: the same token columns per
    pass, the same per-row sums).  The halves' path is held to the oracle by the tests above."""
    import ctypes as C
    K, N, T = 256, 470016, 64
    layer = tb.MoeLayer(512, 256, 8, 2, gate_type=12, up_type=12, down_type=12, max_tokens=4)
    lib, h = layer.lib, layer.h
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    w32 = torch.randn((N, K), device="cuda", generator=g) * 0.05
    W = torch.empty((N, 144), dtype=torch.uint8, device="cuda")
    assert lib.tmoe_quantize(12, C.c_void_p(w32.data_ptr()), N, K, C.c_void_p(W.data_ptr()),
                             C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    del w32
    x = torch.randn((T, K), device="cuda", generator=g)
    full = torch.empty((T, N), device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    assert lib.tmoe_mul_mat(h, None, 12, P(W), 144, K, N, P(x), T, 0, P(full)) == 0
    halves = []
    for r0, r1 in ((0, N // 2), (N // 2, N)):
        o = torch.empty((T, r1 - r0), device="cuda")
        assert lib.tmoe_mul_mat(h, None, 12, P(W[r0:r1]), 144, K, r1 - r0, P(x), T, 0, P(o)) == 0
        halves.append(o)
    layer.check()
    assert torch.equal(full, torch.cat(halves, dim=1))
    layer.close()


@pytest.mark.parametrize("hd,nh,nkv,S,pos0", [(128, 32, 4, 200, 37), (128, 4, 2, 64, 0), (64, 4, 2, 1, 5),
                                             (128, 8, 8, 130, 900)])
def test_prefill_attention_op_against_float64(hd, nh, nkv, S, pos0):
    """tmoe_attn_prefill: S new rows of one sequence (its third of three) after pos0 cached ones;
    each query i attends to positions 0 .. pos0 + i.  Against float64 attention over the
    f16-rounded operands; partial 64-query blocks, GQA up to 8 heads per KV head, a single query."""
    import ctypes as C
    n_seq, seq, ctx = 3, 2, pos0 + S + 10
    layer = tb.MoeLayer(512, 256, 8, 2, gate_type=12, up_type=12, down_type=12, max_tokens=4)
    lib, h = layer.lib, layer.h
    rng = np.random.default_rng(hd + nh + S)
    kc = (rng.standard_normal((n_seq, ctx, nkv, hd)) * 0.5).astype(np.float16)
    vc = rng.standard_normal((n_seq, ctx, nkv, hd)).astype(np.float16)
    q = rng.standard_normal((S, nh, hd)).astype(np.float32)
    k = (rng.standard_normal((S, nkv, hd)) * 0.5).astype(np.float32)
    v = rng.standard_normal((S, nkv, hd)).astype(np.float32)
    d_kc, d_vc = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    out = torch.full((S, nh, hd), float("nan"), device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    scale = 1.0 / np.sqrt(hd)
    assert lib.tmoe_attn_prefill(h, None, P(dq), P(dk), P(dv), P(d_kc), P(d_vc), seq, n_seq, pos0, S, nh, nkv, hd,
                                 ctx, scale, P(out)) == 0
    layer.check()
    got = out.cpu().numpy()
    kc[seq, pos0:pos0 + S] = k.astype(np.float16)
    vc[seq, pos0:pos0 + S] = v.astype(np.float16)
    G = nh // nkv
    q16 = q.astype(np.float16).astype(np.float64)
    for i in range(S):
        n = pos0 + i + 1
        K, V = kc[seq, :n].astype(np.float64), vc[seq, :n].astype(np.float64)
        for hh in range(nh):
            s = K[:, hh // G] @ q16[i, hh] * np.float64(np.float32(scale))
            e = np.exp(s - s.max())
            want = e @ V[:, hh // G] / e.sum()
            assert np.abs(got[i, hh] - want).max() < 5e-3 * max(1.0, np.abs(want).max()), (i, hh)
    # the new rows landed in this sequence's cache, and only there
    assert np.array_equal(d_kc.cpu().numpy(), kc) and np.array_equal(d_vc.cpu().numpy(), vc)
    with pytest.raises(tb.TmoeError, match="TMOE_E_INVALID"):
        _lib_check(lib, h, lib.tmoe_attn_prefill(h, None, P(dq), P(dk), P(dv), P(d_kc), P(d_vc), seq, n_seq,
                                                 ctx - S + 1, S, nh, nkv, hd, ctx, scale, P(out)))
    layer.close()


def _lib_check(lib, h, rc):
    from tetraeder_b200 import _lib
    _lib.check(rc, h)


def test_prefill_then_decode_matches_the_oracle(tiny_model):
    """A prompt of 45 tokens in one prefill step (three 16-token projection groups, a partial
    64-query attention block), then three decode steps of the same sequence; the oracle runs the
    same prompt row by row with the causal mask."""
    path, written = tiny_model
    S, n_ctx = 45, 64
    with GgufFile(path) as f:
        hp = f.hparams
        model = Qwen3MoeModel.from_gguf(f, max_batch=1, n_ctx=n_ctx)
    ref = ModelOracle(hp, _oracle_weights(written, hp), 1, n_ctx)
    rng = np.random.default_rng(9)
    prompt = rng.integers(0, hp.n_vocab, S).astype(np.int32)
    try:
        got = model.prefill(torch.from_numpy(prompt).cuda(), seq=0).cpu().numpy()
        model.check()
        want = ref.prefill(prompt, 0)
        assert nrms(got, want) < 5e-2, f"prefill logits nrms {nrms(got, want):.2e}"
        assert int(model.next_tokens[0]) == int(np.argmax(got[0]))
        for s in range(3):
            tok = rng.integers(0, hp.n_vocab, 1).astype(np.int32)
            pos = np.array([S + s], dtype=np.int32)
            got = model.decode(torch.from_numpy(tok).cuda(), torch.from_numpy(pos).cuda()).cpu().numpy()
            model.check()
            want = ref.decode(tok, pos)
            assert nrms(got, want) < 5e-2, f"decode step {s} after the prefill: nrms {nrms(got, want):.2e}"
    finally:
        model.close()


def test_chunked_prefill_equals_one_prefill(tiny_model):
    """The same prompt as one prefill step and as two chunks (the second at pos0 = 30 reads the
    first chunk's keys from the cache): the last logits agree to the f16 rounding of the cached
    keys, and both caches hold the same rows."""
    path, _ = tiny_model
    S, cut, n_ctx = 50, 30, 64
    with GgufFile(path) as f:
        one = Qwen3MoeModel.from_gguf(f, max_batch=2, n_ctx=n_ctx)
    prompt = torch.from_numpy(np.random.default_rng(3).integers(0, 512, S).astype(np.int32)).cuda()
    try:
        a = one.prefill(prompt, seq=1).clone()
        one.prefill(prompt[:cut], seq=0)
        b = one.prefill(prompt[cut:], seq=0, pos0=cut).clone()
        one.check()
        assert nrms(b.cpu().numpy(), a.cpu().numpy()) < 1e-2
        for il in range(len(one.kc)):
            assert torch.equal(one.kc[il][0, :S], one.kc[il][1, :S]) or \
                float((one.kc[il][0, :S].float() - one.kc[il][1, :S].float()).abs().max()) < 5e-2
    finally:
        one.close()


@pytest.mark.parametrize("qtype,K,N,T", [(12, 2048, 4096, 512), (14, 2048, 512, 2048), (12, 4096, 2048, 700)])
def test_mul_mat_prompt_batches_on_the_gemm(qtype, K, N, T):
    """From 512 tokens tmoe_mul_mat runs as one tcgen05 GEMM over the fp16-dequantised matrix (x
    through the Q8_K round trip, then fp16): held to the oracle's Q8_K mul_mat at the large-batch
    bound of the MoE layer's down GEMM (normalised RMS 1e-3, max-abs 2.5e-2 x RMS); reuse_x takes
    the same rows for a second matrix."""
    import ctypes as C
    from tests.common import maxabs_over_rms
    rng = np.random.default_rng(K + N + T)
    W = np.ascontiguousarray(O.quantize(qtype, (rng.standard_normal((N, K)) * 0.05).astype(np.float32)))
    W2 = np.ascontiguousarray(O.quantize(qtype, (rng.standard_normal((256, K)) * 0.05).astype(np.float32)))
    x = rng.standard_normal((T, K)).astype(np.float32)
    layer = tb.MoeLayer(512, 256, 8, 2, gate_type=12, up_type=12, down_type=12, max_tokens=4)
    lib, h = layer.lib, layer.h
    dW, dW2, dx = (torch.from_numpy(a).cuda() for a in (W, W2, x))
    out, out2 = torch.empty((T, N), device="cuda"), torch.empty((T, 256), device="cuda")
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731
    nb1 = W.shape[1]
    assert lib.tmoe_mul_mat(h, None, qtype, P(dW), nb1, K, N, P(dx), T, 0, P(out)) == 0
    assert lib.tmoe_mul_mat(h, None, qtype, P(dW2), nb1, K, 256, P(dx), T, 1, P(out2)) == 0
    layer.check()
    for w_, o_, n_ in ((W, out, N), (W2, out2, 256)):
        want = O.mul_mat_id(qtype, w_.reshape(1, n_, -1), K, n_, 1, x[:, None, :], np.zeros((T, 1), np.int32))[:, 0]
        got = o_.cpu().numpy()
        assert nrms(got, want) <= 1e-3 and maxabs_over_rms(got, want) <= 2.5e-2, \
            f"nrms {nrms(got, want):.2e} maxabs/rms {maxabs_over_rms(got, want):.2e}"
    layer.close()
