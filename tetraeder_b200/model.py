"""The decode step of the whole Qwen3-MoE model around the MoE layer (config 3): the reference's
build_step (crates/model/src/qwen3moe.rs:2777-2826) with attention() (crates/model/src/attn.rs:
246-405), one new token for each of B sequences, over F16 KV caches.  Every op is a libtmoe call:
tmoe_get_rows, tmoe_rms_norm, tmoe_mul_mat (the projections, on the decode GEMV),
tmoe_qk_norm_rope, tmoe_attn_decode, tmoe_add, the MoE layer (tmoe_layer with the FFN norm) and
tmoe_argmax; a step is stream-ordered and allocation-free, so it can be captured in a CUDA graph
(Qwen3MoeModel.graph).  Qwen3MoeModel.prefill runs the prompt of one sequence as one multi-token
step (tmoe_attn_prefill for the causal attention).

Weights come from a GGUF file (from_gguf: the reference's load_weights, qwen3moe.rs:2498-2584) or
are synthetic (synthetic: seeded N(0, std) weights quantised on the device)."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from .moe import ExpertWeights, MoeLayer, _ptr, _stream, row_size

TYPE_F32, TYPE_F16, TYPE_Q4_K, TYPE_Q6_K = 0, 1, 12, 14


@dataclass
class Matrix:
    """A ggml matrix of `rows` rows of `cols` values: uint8 bytes on the device ([rows, row bytes])."""
    type: int
    data: torch.Tensor
    rows: int
    cols: int

    @property
    def nb1(self) -> int:
        return self.data.shape[1]


def _row_bytes(t: int, cols: int) -> int:
    return cols * 4 if t == TYPE_F32 else cols * 2 if t == TYPE_F16 else row_size(t, cols)


class Qwen3MoeModel:
    def __init__(self, hp, weights: dict, max_batch: int, n_ctx: int, device: int = 0):
        """hp: tetraeder_b200.gguf.Hparams; weights: GGUF tensor name -> Matrix (matrices, the
        embedding) or float32 CUDA tensor (norms, router)."""
        self.hp, self.w, self.max_batch, self.n_ctx = hp, weights, max_batch, n_ctx
        self.device = torch.device("cuda", device)
        d, nh, nkv = hp.head_dim, hp.n_head, hp.n_head_kv
        gt, ut, dt = (self.w[f"blk.0.{n}.weight"].type for n in ("ffn_gate_exps", "ffn_up_exps", "ffn_down_exps"))
        self.moe = MoeLayer(hp.n_embd, hp.n_ff_exp, hp.n_expert, hp.n_expert_used, gate_type=gt, up_type=ut,
                            down_type=dt, max_tokens=max_batch, device=device, rms_eps=hp.rms_eps)
        self.lib, self.h = self.moe.lib, self.moe.h
        # The K and V projections run beside Q, each on a stream of its own with a handle of its own
        # (a handle's projection workspace serves one stream at a time): at decode batch sizes each
        # projection is a few hundred GEMV items, too few to fill the SMs alone.
        self._lanes = [MoeLayer(512, 256, 8, 2, gate_type=TYPE_Q4_K, up_type=TYPE_Q4_K, down_type=TYPE_Q4_K,
                                max_tokens=4, device=device) for _ in range(2)]
        self._side = [torch.cuda.Stream(device=self.device) for _ in range(2)]
        self._fork = torch.cuda.Event()
        self._join = [torch.cuda.Event() for _ in range(2)]
        self.experts = [ExpertWeights(*(self.w[f"blk.{il}.{n}.weight"].data.view(hp.n_expert, -1,
                                                                                  self.w[f"blk.{il}.{n}.weight"].nb1)
                                        for n in ("ffn_gate_exps", "ffn_up_exps", "ffn_down_exps")))
                        for il in range(hp.n_layer)]
        f = dict(dtype=torch.float32, device=self.device)
        B = max_batch
        self.kc = [torch.zeros((B, n_ctx, nkv, d), dtype=torch.float16, device=self.device) for _ in range(hp.n_layer)]
        self.vc = [torch.zeros((B, n_ctx, nkv, d), dtype=torch.float16, device=self.device) for _ in range(hp.n_layer)]
        self.x = torch.empty((B, hp.n_embd), **f)
        self.cur = torch.empty((B, hp.n_embd), **f)
        self.q = torch.empty((B, nh * d), **f)
        self.k = torch.empty((B, nkv * d), **f)
        self.v = torch.empty((B, nkv * d), **f)
        self.att = torch.empty((B, nh * d), **f)
        self.o = torch.empty((B, hp.n_embd), **f)
        self.ffn_inp = torch.empty((B, hp.n_embd), **f)
        self.moe_out = torch.empty((B, hp.n_embd), **f)
        self.logits = torch.empty((B, hp.n_vocab), **f)
        self.next_tokens = torch.empty((B,), dtype=torch.int32, device=self.device)
        nbytes = self.lib.tmoe_attn_decode_scratch_bytes(self.h, B, nh, nkv, d, n_ctx)
        _lib.check(nbytes if nbytes < 0 else 0, self.h)
        self.scratch = torch.empty((max(nbytes, 4) + 3) // 4, **f)

    # -- weights -------------------------------------------------------------------------
    @classmethod
    def from_gguf(cls, g, max_batch: int, n_ctx: int, device: int = 0) -> "Qwen3MoeModel":
        """Every tensor the step reads, from an open GgufFile (or a path)."""
        from .gguf import GgufFile
        own = not isinstance(g, GgufFile)
        g = GgufFile(g) if own else g
        try:
            hp = g.hparams
            dev = torch.device("cuda", device)
            w = {}
            for t in g.tensors:
                buf = torch.empty(t.nbytes, dtype=torch.uint8, device=dev)
                g.load(t.name, buf)
                if t.type == TYPE_F32 and (t.ne[1] == 1 or t.name.endswith("ffn_gate_inp.weight")):
                    w[t.name] = buf.view(torch.float32)
                else:
                    rows = t.ne[1] * t.ne[2] * t.ne[3]
                    w[t.name] = Matrix(t.type, buf.view(rows, -1), rows, t.ne[0])
            return cls(hp, w, max_batch, n_ctx, device)
        finally:
            if own:
                g.close()

    @classmethod
    def synthetic(cls, hp, max_batch: int, n_ctx: int, device: int = 0, seed: int = 1, attn_types=(12, 12, 14, 12),
                  expert_types=(12, 12, 14), embd_type=12, out_type=14, std=0.02) -> "Qwen3MoeModel":
        """Seeded N(0, std) weights quantised on the device (Q4_K_M-like types by default:
        attn_q/k/o Q4_K, attn_v Q6_K, experts Q4_K/Q4_K/Q6_K, token_embd Q4_K, output Q6_K)."""
        dev = torch.device("cuda", device)
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        lib = _lib.load()

        def mat(t, rows, cols, n=1, std_=std):
            data = torch.empty((n * rows, _row_bytes(t, cols)), dtype=torch.uint8, device=dev)
            for i in range(0, n * rows, max(1, (64 << 20) // (cols * 4))):  # chunks of about 64 MB of f32
                r = min(n * rows, i + max(1, (64 << 20) // (cols * 4))) - i
                x = torch.randn((r, cols), generator=gen, device=dev) * std_
                if t == TYPE_F32:
                    data[i:i + r].copy_(x.view(torch.uint8).view(r, -1))
                elif t == TYPE_F16:
                    data[i:i + r].copy_(x.half().view(torch.uint8).view(r, -1))
                else:
                    _lib.check(lib.tmoe_quantize(t, C.c_void_p(x.data_ptr()), r, cols,
                                                 C.c_void_p(data[i].data_ptr()), _stream(None)))
            return Matrix(t, data, n * rows, cols)

        def norm(n):
            return 1.0 + 0.1 * torch.randn((n,), generator=gen, device=dev)

        H, d, nh, nkv = hp.n_embd, hp.head_dim, hp.n_head, hp.n_head_kv
        w = {"token_embd.weight": mat(embd_type, hp.n_vocab, H, std_=0.5), "output_norm.weight": norm(H)}
        if not hp.tied_output:
            w["output.weight"] = mat(out_type, hp.n_vocab, H)
        for il in range(hp.n_layer):
            p = f"blk.{il}."
            w[p + "attn_norm.weight"] = norm(H)
            w[p + "attn_q.weight"] = mat(attn_types[0], nh * d, H)
            w[p + "attn_k.weight"] = mat(attn_types[1], nkv * d, H)
            w[p + "attn_v.weight"] = mat(attn_types[2], nkv * d, H)
            w[p + "attn_output.weight"] = mat(attn_types[3], H, nh * d)
            w[p + "attn_q_norm.weight"] = norm(d)
            w[p + "attn_k_norm.weight"] = norm(d)
            w[p + "ffn_norm.weight"] = norm(H)
            w[p + "ffn_gate_inp.weight"] = torch.randn((hp.n_expert, H), generator=gen, device=dev) * 0.5
            w[p + "ffn_gate_exps.weight"] = mat(expert_types[0], hp.n_ff_exp, H, hp.n_expert)
            w[p + "ffn_up_exps.weight"] = mat(expert_types[1], hp.n_ff_exp, H, hp.n_expert)
            w[p + "ffn_down_exps.weight"] = mat(expert_types[2], H, hp.n_ff_exp, hp.n_expert)
        torch.cuda.synchronize(dev)
        return cls(hp, w, max_batch, n_ctx, device)

    # -- the step ------------------------------------------------------------------------
    def _mm(self, m: Matrix, x: torch.Tensor, out: torch.Tensor, B: int, st, reuse: bool = False, h=None):
        h = self.h if h is None else h
        _lib.check(self.lib.tmoe_mul_mat(h, st, m.type, C.c_void_p(m.data.data_ptr()), m.nb1, m.cols, m.rows,
                                         _ptr(x), B, int(reuse), _ptr(out)), h)

    def _step(self, tokens: torch.Tensor, pos: torch.Tensor, B: int, stream):
        hp, w, L, h = self.hp, self.w, self.lib, self.h
        st = _stream(stream)
        main = torch.cuda.current_stream(self.device) if stream is None else stream
        d, nh, nkv, H = hp.head_dim, hp.n_head, hp.n_head_kv, hp.n_embd
        chk = lambda rc: _lib.check(rc, h)  # noqa: E731
        emb = w["token_embd.weight"]
        chk(L.tmoe_get_rows(h, st, emb.type, C.c_void_p(emb.data.data_ptr()), emb.nb1, H, emb.rows, _ptr(tokens), B,
                            _ptr(self.x)))
        for il in range(hp.n_layer):
            p = f"blk.{il}."
            chk(L.tmoe_rms_norm(h, st, _ptr(self.x), _ptr(w[p + "attn_norm.weight"]), hp.rms_eps, B, H, _ptr(self.cur)))
            wq, wk, wv = w[p + "attn_q.weight"], w[p + "attn_k.weight"], w[p + "attn_v.weight"]
            self._fork.record(main)
            for side, lane, wm, out, join in zip(self._side, self._lanes, (wk, wv), (self.k, self.v), self._join):
                side.wait_event(self._fork)
                self._mm(wm, self.cur, out, B, _stream(side), h=lane.h)
                join.record(side)
            self._mm(wq, self.cur, self.q, B, st)
            for join in self._join:
                main.wait_event(join)
            if d % 32 == 0 and d <= 128:  # the two norms and the two RoPEs in one launch
                chk(L.tmoe_qk_norm_rope(h, st, _ptr(self.q), _ptr(self.k), _ptr(w[p + "attn_q_norm.weight"]),
                                        _ptr(w[p + "attn_k_norm.weight"]), _ptr(pos), B, nh, nkv, d, hp.n_rot,
                                        hp.rope_freq_base, hp.rms_eps))
            else:
                chk(L.tmoe_rms_norm(h, st, _ptr(self.q), _ptr(w[p + "attn_q_norm.weight"]), hp.rms_eps, B * nh, d,
                                    _ptr(self.q)))
                chk(L.tmoe_rms_norm(h, st, _ptr(self.k), _ptr(w[p + "attn_k_norm.weight"]), hp.rms_eps, B * nkv, d,
                                    _ptr(self.k)))
                chk(L.tmoe_rope_neox(h, st, _ptr(self.q), _ptr(pos), B, nh, d, hp.n_rot, hp.rope_freq_base))
                chk(L.tmoe_rope_neox(h, st, _ptr(self.k), _ptr(pos), B, nkv, d, hp.n_rot, hp.rope_freq_base))
            chk(L.tmoe_attn_decode(h, st, _ptr(self.q), _ptr(self.k), _ptr(self.v), _ptr(self.kc[il]),
                                   _ptr(self.vc[il]), _ptr(pos), B, nh, nkv, d, self.n_ctx, 1.0 / d ** 0.5,
                                   _ptr(self.scratch), _ptr(self.att)))
            self._mm(w[p + "attn_output.weight"], self.att, self.o, B, st)
            chk(L.tmoe_add(h, st, _ptr(self.x), _ptr(self.o), _ptr(self.ffn_inp), B * H))
            self.moe.moe_ffn(self.ffn_inp[:B], self.experts[il], router_w=w[p + "ffn_gate_inp.weight"],
                             ffn_norm=w[p + "ffn_norm.weight"], use_norm=True, out=self.moe_out[:B], stream=stream)
            chk(L.tmoe_add(h, st, _ptr(self.ffn_inp), _ptr(self.moe_out), _ptr(self.x), B * H))
        chk(L.tmoe_rms_norm(h, st, _ptr(self.x), _ptr(w["output_norm.weight"]), hp.rms_eps, B, H, _ptr(self.cur)))
        head = w["token_embd.weight"] if hp.tied_output else w["output.weight"]
        self._mm(head, self.cur, self.logits, B, st)
        chk(L.tmoe_argmax(h, st, _ptr(self.logits), B, hp.n_vocab, _ptr(self.next_tokens)))

    def decode(self, tokens: torch.Tensor, pos: torch.Tensor, stream=None) -> torch.Tensor:
        """One decode step: tokens, pos int32 CUDA [B] (B <= max_batch; token b goes to position
        pos[b] of sequence b's cache and attends to its positions 0..pos[b]).  Returns the logits
        [B, n_vocab] (views of the model's buffers; the greedy next tokens are in next_tokens)."""
        B = tokens.shape[0]
        if B > self.max_batch or pos.shape[0] != B:
            raise ValueError(f"{B} tokens for a model of at most {self.max_batch} sequences")
        self._step(tokens, pos, B, stream)
        return self.logits[:B]

    # -- prefill ---------------------------------------------------------------------------
    def _prefill_buffers(self, S: int):
        """Buffers and the MoE handle of a prefill of up to S tokens (made on first use)."""
        if getattr(self, "_pf_cap", 0) >= S:
            return
        hp, f = self.hp, dict(dtype=torch.float32, device=self.device)
        d, nh, nkv, H = hp.head_dim, hp.n_head, hp.n_head_kv, hp.n_embd
        if getattr(self, "_pf_moe", None) is not None:
            self._pf_moe.close()
        self._pf_moe = MoeLayer(H, hp.n_ff_exp, hp.n_expert, hp.n_expert_used, gate_type=self.moe.cfg.gate_type,
                                up_type=self.moe.cfg.up_type, down_type=self.moe.cfg.down_type, max_tokens=S,
                                device=self.device.index, rms_eps=hp.rms_eps)
        self._pf = {n: torch.empty((S, c), **f) for n, c in
                    (("x", H), ("cur", H), ("q", nh * d), ("k", nkv * d), ("v", nkv * d), ("att", nh * d),
                     ("o", H), ("ffn_inp", H), ("moe_out", H))}
        self._pf_pos = torch.empty((S,), dtype=torch.int32, device=self.device)
        self._pf_cap = S

    def prefill(self, tokens: torch.Tensor, seq: int = 0, pos0: int = 0, stream=None) -> torch.Tensor:
        """The prompt step of one sequence (build_step over S tokens, attention_seqs with the causal
        mask, attn.rs:269-302): tokens int32 CUDA [S] go to positions pos0 .. pos0+S-1 of sequence
        `seq`'s caches, every layer runs on all S rows at once (the projections on the GEMV with token
        groups, the MoE layer on its large-batch path from S * k >= 6144 pairs, the causal attention
        on the tensor cores), and the head runs on the last row.  Returns its logits [1, n_vocab]; the
        greedy next token is next_tokens[0].  Decoding of the sequence then continues at pos0 + S."""
        hp, w, L, h = self.hp, self.w, self.lib, self.h
        S = tokens.shape[0]
        if not 0 <= seq < self.max_batch or pos0 < 0 or pos0 + S > self.n_ctx:
            raise ValueError(f"prefill of {S} tokens at {pos0} of sequence {seq}: the caches hold "
                             f"{self.max_batch} sequences of {self.n_ctx} positions")
        self._prefill_buffers(S)
        b = {n: t[:S] for n, t in self._pf.items()}
        st = _stream(stream)
        main = torch.cuda.current_stream(self.device) if stream is None else stream
        d, nh, nkv, H = hp.head_dim, hp.n_head, hp.n_head_kv, hp.n_embd
        chk = lambda rc: _lib.check(rc, h)  # noqa: E731
        pos = self._pf_pos[:S]
        with torch.cuda.stream(main):
            torch.arange(pos0, pos0 + S, dtype=torch.int32, device=self.device, out=pos)
        emb = w["token_embd.weight"]
        chk(L.tmoe_get_rows(h, st, emb.type, C.c_void_p(emb.data.data_ptr()), emb.nb1, H, emb.rows, _ptr(tokens), S,
                            _ptr(b["x"])))
        for il in range(hp.n_layer):
            p = f"blk.{il}."
            chk(L.tmoe_rms_norm(h, st, _ptr(b["x"]), _ptr(w[p + "attn_norm.weight"]), hp.rms_eps, S, H,
                                _ptr(b["cur"])))
            self._fork.record(main)
            for side, lane, wm, out, join in zip(self._side, self._lanes, (w[p + "attn_k.weight"], w[p + "attn_v.weight"]),
                                                 (b["k"], b["v"]), self._join):
                side.wait_event(self._fork)
                self._mm(wm, b["cur"], out, S, _stream(side), h=lane.h)
                join.record(side)
            self._mm(w[p + "attn_q.weight"], b["cur"], b["q"], S, st)
            for join in self._join:
                main.wait_event(join)
            chk(L.tmoe_qk_norm_rope(h, st, _ptr(b["q"]), _ptr(b["k"]), _ptr(w[p + "attn_q_norm.weight"]),
                                    _ptr(w[p + "attn_k_norm.weight"]), _ptr(pos), S, nh, nkv, d, hp.n_rot,
                                    hp.rope_freq_base, hp.rms_eps))
            chk(L.tmoe_attn_prefill(h, st, _ptr(b["q"]), _ptr(b["k"]), _ptr(b["v"]), _ptr(self.kc[il]),
                                    _ptr(self.vc[il]), seq, self.max_batch, pos0, S, nh, nkv, d, self.n_ctx,
                                    1.0 / d ** 0.5, _ptr(b["att"])))
            self._mm(w[p + "attn_output.weight"], b["att"], b["o"], S, st)
            chk(L.tmoe_add(h, st, _ptr(b["x"]), _ptr(b["o"]), _ptr(b["ffn_inp"]), S * H))
            self._pf_moe.moe_ffn(b["ffn_inp"], self.experts[il], router_w=w[p + "ffn_gate_inp.weight"],
                                 ffn_norm=w[p + "ffn_norm.weight"], use_norm=True, out=b["moe_out"], stream=stream)
            chk(L.tmoe_add(h, st, _ptr(b["ffn_inp"]), _ptr(b["moe_out"]), _ptr(b["x"]), S * H))
        last = b["x"][S - 1:]
        chk(L.tmoe_rms_norm(h, st, _ptr(last), _ptr(w["output_norm.weight"]), hp.rms_eps, 1, H, _ptr(self.cur)))
        head = w["token_embd.weight"] if hp.tied_output else w["output.weight"]
        self._mm(head, self.cur, self.logits, 1, st)
        chk(L.tmoe_argmax(h, st, _ptr(self.logits), 1, hp.n_vocab, _ptr(self.next_tokens)))
        return self.logits[:1]

    def graph(self, tokens: torch.Tensor, pos: torch.Tensor):
        """A CUDA graph of decode(tokens, pos) for these (fixed) token and position buffers:
        update them in place, then replay.  Run decode once before capturing (the projections'
        workspace is sized on first use)."""
        s = torch.cuda.Stream(device=self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.decode(tokens, pos, stream=s)
        return g

    def check(self):
        self.moe.check()
        if getattr(self, "_pf_moe", None) is not None:
            self._pf_moe.check()
        for lane in self._lanes:
            lane.check()

    def close(self):
        if getattr(self, "_pf_moe", None) is not None:
            self._pf_moe.close()
        for lane in self._lanes:
            lane.close()
        self.moe.close()
