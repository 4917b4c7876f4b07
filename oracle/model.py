"""CPU oracle of the Qwen3-MoE decode and prefill steps around the MoE layer (config 3).  TEST INFRASTRUCTURE
ONLY: imported by tests/ as the checker of tetraeder_b200.model, never by the product.

Restates, per decode step of B sequences (one new token each):
  build_step (crates/model/src/qwen3moe.rs:2777-2806): x = get_rows(token_embd, tokens); per layer
    the attention block, then router + weighted_experts + sum_experts on ffn_inp, plus ffn_inp;
  attention() (crates/model/src/attn.rs:298-405): rms_norm(x) * attn_norm; q, k, v = Wq, Wk, Wv
    (ggml mul_mat: the Q8_K dot of the activations, as on the reference CPU path, here through the
    layer oracle's mul_mat_id with one expert); rms_norm per head times q_norm / k_norm; NeoX RoPE
    (attn.rs:225-236); K and V stored as F16 (set_rows into the F16 cache); softmax(q k^T / sqrt(d)) v
    over the sequence's positions 0..pos (the causal mask of attn.rs:425), with q converted to F16 as
    flash_attn_ext does for an F16 cache; Wo; plus x;
  head (qwen3moe.rs:2809-2826): rms_norm * output_norm, then `output` (or the tied token_embd).
Parity with ggml itself is not pinned (ggml is absent from the reference tree); the arithmetic
follows the published ops, in float32 with float64 where noted.
"""
from __future__ import annotations

import numpy as np

from . import TYPE_F16, TYPE_F32, dequantize, experts, mul_mat_id, route


def rms_norm(x, w, eps):
    """ggml rms_norm: the mean of squares summed in float64, the scale in float32, times w."""
    x = np.asarray(x, np.float32)
    mean = np.float32((x * x).astype(np.float64).sum(axis=-1) / x.shape[-1])
    scale = (np.float32(1.0) / np.sqrt(mean + np.float32(eps), dtype=np.float32)).astype(np.float32)
    out = (x * scale[..., None]).astype(np.float32)
    return out if w is None else (out * np.asarray(w, np.float32)).astype(np.float32)


def rope_neox(x, pos, n_rot, base):
    """x [T, n_head, d] float32; NeoX pairs (i, i + n_rot/2), theta = pos * base^(-2i/n_rot)."""
    x = np.array(x, np.float32)
    half = n_rot // 2
    i = np.arange(half, dtype=np.float64)
    theta = np.asarray(pos, np.float64)[:, None] * np.power(np.float64(base), -2.0 * i / n_rot)[None, :]
    c, s = np.cos(theta)[:, None, :], np.sin(theta)[:, None, :]
    x0, x1 = x[..., :half].astype(np.float64), x[..., half:n_rot].astype(np.float64)
    x[..., :half] = (x0 * c - x1 * s).astype(np.float32)
    x[..., half:n_rot] = (x0 * s + x1 * c).astype(np.float32)
    return x


class Matrix:
    """A ggml matrix [rows][cols]: quantised bytes (Q4_K/Q6_K) or F16/F32 values."""

    def __init__(self, qtype, data, rows, cols):
        self.type, self.data, self.rows, self.cols = qtype, np.ascontiguousarray(data), rows, cols

    def matmul(self, x):
        """W . x for x [T, cols] -> [T, rows]."""
        x = np.asarray(x, np.float32)
        if self.type in (TYPE_F32, TYPE_F16):
            w = self.data.view(np.float16 if self.type == TYPE_F16 else np.float32).reshape(self.rows, self.cols)
            return (x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)
        T = x.shape[0]
        out = mul_mat_id(self.type, self.data.reshape(1, self.rows, -1), self.cols, self.rows, 1, x[:, None, :],
                         np.zeros((T, 1), np.int32))
        return out[:, 0, :]

    def rows_f32(self, idx):
        if self.type in (TYPE_F32, TYPE_F16):
            w = self.data.view(np.float16 if self.type == TYPE_F16 else np.float32).reshape(self.rows, self.cols)
            return w[idx].astype(np.float32)
        rb = self.data.size // self.rows
        d = self.data.reshape(self.rows, rb)
        return np.stack([dequantize(self.type, d[i], self.cols) for i in idx]).astype(np.float32)


class ModelOracle:
    """The decode step of B sequences over per-layer F16 KV caches [B][n_ctx][n_kv][d]."""

    def __init__(self, hp, weights, max_batch, n_ctx):
        """weights: {name: Matrix or float32 array} with the GGUF tensor names; hp: an object with
        the Hparams fields (n_layer, n_embd, n_head, n_head_kv, head_dim, n_rot, n_expert,
        n_expert_used, n_ff_exp, n_vocab, rms_eps, rope_freq_base, tied_output)."""
        self.hp, self.w = hp, weights
        kv = hp.n_head_kv * hp.head_dim
        self.kc = [np.zeros((max_batch, n_ctx, kv), np.float16) for _ in range(hp.n_layer)]
        self.vc = [np.zeros((max_batch, n_ctx, kv), np.float16) for _ in range(hp.n_layer)]

    def attention(self, il, x, pos, seq=None):
        """Row b of x is the token of sequence seq[b] (default: b) at position pos[b]; its K/V row is
        stored, then it attends to that sequence's positions 0..pos[b] -- one token per sequence in
        a decode step, or the S tokens of one sequence in a prefill (rows in position order, so each
        row's keys are stored before it reads them: the causal mask)."""
        hp, w = self.hp, self.w
        seq = np.arange(x.shape[0]) if seq is None else np.asarray(seq)
        B, d, nh, nkv = x.shape[0], hp.head_dim, hp.n_head, hp.n_head_kv
        p = f"blk.{il}."
        cur = rms_norm(x, w[p + "attn_norm.weight"], hp.rms_eps)
        q = w[p + "attn_q.weight"].matmul(cur).reshape(B, nh, d)
        k = w[p + "attn_k.weight"].matmul(cur).reshape(B, nkv, d)
        v = w[p + "attn_v.weight"].matmul(cur)
        q = rope_neox(rms_norm(q, w[p + "attn_q_norm.weight"], hp.rms_eps), pos, hp.n_rot, hp.rope_freq_base)
        k = rope_neox(rms_norm(k, w[p + "attn_k_norm.weight"], hp.rms_eps), pos, hp.n_rot, hp.rope_freq_base)
        out = np.zeros((B, nh, d), np.float32)
        G = nh // nkv
        # flash_attn_ext over an F16 cache converts Q to F16 and scales the Q.K dot (ggml's CPU and CUDA paths)
        q16 = q.astype(np.float16).astype(np.float64)
        for b in range(B):
            sb = seq[b]
            self.kc[il][sb, pos[b]] = k[b].reshape(-1).astype(np.float16)
            self.vc[il][sb, pos[b]] = v[b].astype(np.float16)
            K = self.kc[il][sb, :pos[b] + 1].astype(np.float64).reshape(-1, nkv, d)
            V = self.vc[il][sb, :pos[b] + 1].astype(np.float64).reshape(-1, nkv, d)
            for h in range(nh):
                s = (K[:, h // G, :] @ q16[b, h]) * np.float64(np.float32(1.0 / np.sqrt(d)))
                e = np.exp(s - s.max())
                out[b, h] = (e @ V[:, h // G, :] / e.sum()).astype(np.float32)
        o = w[p + "attn_output.weight"].matmul(out.reshape(B, nh * d))
        return (x + o).astype(np.float32)

    def decode(self, tokens, pos):
        return self._step(tokens, pos, None)

    def prefill(self, tokens, seq, pos0=0):
        """The S tokens of sequence `seq` at positions pos0 .. pos0+S-1 in one step (build_step over a
        prompt); returns the logits of the last token [1, n_vocab]."""
        S = len(tokens)
        return self._step(tokens, pos0 + np.arange(S, dtype=np.int32), np.full(S, seq), last_only=True)

    def _step(self, tokens, pos, seq, last_only=False):
        hp, w = self.hp, self.w
        x = w["token_embd.weight"].rows_f32(np.asarray(tokens))
        for il in range(hp.n_layer):
            p = f"blk.{il}."
            ffn_inp = self.attention(il, x, np.asarray(pos), seq)
            ids, wt, xn, _ = route(ffn_inp, hp.n_expert_used, router_w=w[p + "ffn_gate_inp.weight"], norm=True,
                                   norm_w=w[p + "ffn_norm.weight"], eps=hp.rms_eps)
            g, u, dn = (w[p + n + ".weight"] for n in ("ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"))
            moe = experts(xn, ids, wt, g.data, u.data, dn.data, hp.n_embd, hp.n_ff_exp, hp.n_expert, g.type, u.type,
                          dn.type)
            x = (ffn_inp + moe).astype(np.float32)
        h = rms_norm(x[-1:] if last_only else x, w["output_norm.weight"], hp.rms_eps)
        head = w["token_embd.weight"] if hp.tied_output else w["output.weight"]
        return head.matmul(h)
