"""Host-side mirror of Tetraeder's MoE-layer operator interface over the C ABI.

The names, argument meanings and error behaviour follow the reference's builder functions and
ggml ops (paths relative to the tetraeder project root):

  MoeLayer.router            crates/model/src/qwen3moe.rs:2871-2890   router()
  MoeLayer.weighted_experts  crates/model/src/qwen3moe.rs:2899-2914   weighted_experts() (+ the
                             sum_experts() fold of :2917-2923, done on device in choice order)
  MoeLayer.moe_ffn           crates/model/src/qwen3moe.rs:2892-2896   moe_ffn()
  MoeLayer.mul_mat_id        crates/ggml-sys/src/ggml/context.rs:322-336 Context::mul_mat_id
  MoeLayer.map_ids           crates/model/src/qwen3moe_shard.rs:1043-1050 get_rows(map, ids)

Tensors are torch CUDA tensors (plumbing only); the computation is the CUDA code of libtmoe.so.
Where ggml aborts on a bad shape, these raise TmoeError (or ValueError before the call).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import TYPE_Q4_K, TYPE_Q6_K, TYPE_Q6_K_R8, TmoeError

QK_K = 256
BLOCK_BYTES = {TYPE_Q4_K: 144, TYPE_Q6_K: 210, TYPE_Q6_K_R8: 210}


def row_size(qtype: int, ncols: int) -> int:
    if ncols % QK_K:
        raise ValueError(f"{ncols} columns is not a multiple of {QK_K}")
    return ncols // QK_K * BLOCK_BYTES[qtype]


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream):
    s = torch.cuda.current_stream() if stream is None else stream
    return C.c_void_p(s.cuda_stream)


@dataclass
class ExpertWeights:
    """Stacked (or slot) expert tensors in ggml layout: uint8 [n_slots, rows, row_size]."""
    gate: torch.Tensor
    up: torch.Tensor
    down: torch.Tensor

    def c_struct(self, host: bool = False) -> _lib.ExpertTensors:
        for t in (self.gate, self.up, self.down):
            if t.dtype != torch.uint8 or t.dim() != 3 or not t.is_contiguous():
                raise ValueError("expert tensors must be contiguous uint8 tensors [slots, rows, bytes]")
            if (not host and not t.is_cuda) or (host and (t.is_cuda or not t.is_pinned())):
                raise ValueError("expert tensors must be CUDA tensors" if not host else
                                 "a host expert store must be pinned CPU tensors")
        g, u, d = self.gate, self.up, self.down
        return _lib.ExpertTensors(g.data_ptr(), u.data_ptr(), d.data_ptr(),
                                  g.shape[2], g.shape[1] * g.shape[2],
                                  u.shape[2], u.shape[1] * u.shape[2],
                                  d.shape[2], d.shape[1] * d.shape[2], g.shape[0])


def quantize(qtype: int, x: torch.Tensor, stream=None) -> torch.Tensor:
    """quant::quantize on the device: f32 [..., ncols] -> uint8 [..., row_size(ncols)]."""
    lib = _lib.load()
    x = x.contiguous()
    ncols = x.shape[-1]
    nrows = x.numel() // ncols
    out = torch.empty(x.shape[:-1] + (row_size(qtype, ncols),), dtype=torch.uint8, device=x.device)
    _lib.check(lib.tmoe_quantize(qtype, _ptr(x), nrows, ncols, _ptr(out), _stream(stream)), None)
    return out


def dequantize(qtype: int, data: torch.Tensor, n: int, stream=None) -> torch.Tensor:
    """quant::to_f32 on the device -> f32 [n]."""
    lib = _lib.load()
    out = torch.empty(n, dtype=torch.float32, device=data.device)
    _lib.check(lib.tmoe_dequantize(qtype, _ptr(data.contiguous()), n, _ptr(out), _stream(stream)), None)
    return out


def prepack(W: torch.Tensor, stream=None) -> torch.Tensor:
    """tmoe_prepack, the optional explicit repack: Q6_K expert matrices uint8 [n_mats, rows, row_size]
    (rows % 8 == 0) -> a new tensor of the same shape and bytes in 8-row fragment order, to be used
    as TYPE_Q6_K_R8 wherever the Q6_K tensor was (products bit for bit the same)."""
    lib = _lib.load()
    if W.dtype != torch.uint8 or W.dim() != 3 or not W.is_cuda:
        raise ValueError("prepack takes a CUDA uint8 tensor [n_mats, rows, row_size]")
    n_mats, rows, rs = W.shape
    if rs % BLOCK_BYTES[TYPE_Q6_K]:
        raise ValueError("row size is not a whole number of Q6_K super-blocks")
    K = rs // BLOCK_BYTES[TYPE_Q6_K] * QK_K
    out = torch.empty((n_mats, rows, rs), dtype=torch.uint8, device=W.device)
    _lib.check(lib.tmoe_prepack(TYPE_Q6_K, _ptr(W), W.stride(1), W.stride(0), rows, K, n_mats, _ptr(out),
                                _stream(stream)), None)
    return out


class MoeLayer:
    """One handle of the C ABI: H, I, E, k, types and the workspace for `max_tokens`."""

    def __init__(self, n_embd: int, n_ff: int, n_expert: int, n_expert_used: int,
                 gate_type: int = TYPE_Q4_K, up_type: int = TYPE_Q4_K, down_type: int = TYPE_Q6_K,
                 max_tokens: int = 64, device: int | None = None, rms_eps: float = 1e-6):
        if not torch.cuda.is_available():
            raise RuntimeError("tetraeder_b200 needs a CUDA device (there is no CPU path)")
        self.lib = _lib.load()
        dev = torch.cuda.current_device() if device is None else device
        self.cfg = _lib.Config(n_embd, n_ff, n_expert, n_expert_used, gate_type, up_type, down_type,
                               max_tokens, dev, rms_eps)
        h = C.c_void_p()
        _lib.check(self.lib.tmoe_create(C.byref(self.cfg), C.byref(h)), None)
        self.h = h
        self.device = torch.device("cuda", dev)

    def close(self):
        if getattr(self, "h", None):
            self.lib.tmoe_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- per-kernel timing --------------------------------------------------------------------
    def profile(self, enable: bool = True):
        """Brackets every kernel of this handle with CUDA events (resets the totals)."""
        _lib.check(self.lib.tmoe_profile_enable(self.h, int(enable)), self.h)

    def profile_collect(self) -> dict:
        """{phase: (total_ms, launches)} accumulated since profile(True)."""
        n = len(_lib.PHASES)
        ms = (C.c_double * n)()
        cnt = (C.c_int64 * n)()
        _lib.check(self.lib.tmoe_profile_collect(self.h, ms, cnt), self.h)
        return {name: (ms[i], cnt[i]) for i, name in enumerate(_lib.PHASES) if cnt[i]}

    # -- ops ---------------------------------------------------------------------------------
    def check(self, stream=None):
        """Synchronises and raises if a kernel latched a device error."""
        _lib.check(self.lib.tmoe_check(self.h, _stream(stream)), self.h)

    def wait_flag(self, flag: torch.Tensor, value: int, limit_ns: int = 0, stream=None):
        """Holds the stream until flag[0] == value (an int32 word in device memory or in pinned host
        memory that the host writes); after limit_ns (<= 0: one second) the wait gives up and the
        next check() raises TMOE_E_DEVICE."""
        if flag.dtype != torch.int32:
            raise ValueError("the flag is an int32 word")
        _lib.check(self.lib.tmoe_wait_flag(self.h, _stream(stream), _ptr(flag), int(value), int(limit_ns)), self.h)

    def router(self, ffn_inp: torch.Tensor, router_w: torch.Tensor | None = None,
               logits: torch.Tensor | None = None, ffn_norm: torch.Tensor | None = None,
               use_norm: bool = False, stream=None, want_logits: bool = False):
        """-> (xn, weights [T, k], ids [T, k]) like router(); xn is None without the norm."""
        T = ffn_inp.shape[0] if ffn_inp is not None else logits.shape[0]
        k = self.cfg.n_expert_used
        ids = torch.empty((T, k), dtype=torch.int32, device=self.device)
        w = torch.empty((T, k), dtype=torch.float32, device=self.device)
        xn = torch.empty_like(ffn_inp) if use_norm else None
        lg = torch.empty((T, self.cfg.n_expert), dtype=torch.float32, device=self.device) if want_logits else None
        _lib.check(self.lib.tmoe_route(self.h, _stream(stream), _ptr(ffn_inp), T, int(use_norm),
                                       _ptr(ffn_norm), _ptr(router_w), _ptr(logits), _ptr(ids), _ptr(w),
                                       _ptr(xn), _ptr(lg)), self.h)
        return (xn, w, ids, lg) if want_logits else (xn, w, ids)

    def weighted_experts(self, xn: torch.Tensor, ids: torch.Tensor, w: torch.Tensor,
                         experts: ExpertWeights, out: torch.Tensor | None = None, stream=None):
        """down(silu(gate xn) * up xn) * w, summed over the choices in order -> [T, H]."""
        T = xn.shape[0]
        out = torch.empty((T, self.cfg.n_embd), dtype=torch.float32, device=self.device) if out is None else out
        st = experts.c_struct()
        _lib.check(self.lib.tmoe_experts(self.h, _stream(stream), _ptr(xn), T, _ptr(ids), _ptr(w),
                                         C.byref(st), _ptr(out)), self.h)
        return out

    def moe_ffn(self, x: torch.Tensor, experts: ExpertWeights, router_w: torch.Tensor | None = None,
                logits: torch.Tensor | None = None, id_map: torch.Tensor | None = None,
                ffn_norm: torch.Tensor | None = None, use_norm: bool = False, out=None, ids_out=None,
                w_out=None, stream=None):
        """router + (EP id map) + weighted_experts in one C call -> [T, H] f32.  x is f32 or bf16
        (tmoe_layer_bf16: widened exactly, then the same layer)."""
        T = x.shape[0]
        out = torch.empty((T, self.cfg.n_embd), dtype=torch.float32, device=self.device) if out is None else out
        st = experts.c_struct()
        fn = self.lib.tmoe_layer_bf16 if x.dtype == torch.bfloat16 else self.lib.tmoe_layer
        _lib.check(fn(self.h, _stream(stream), _ptr(x), T, int(use_norm), _ptr(ffn_norm),
                      _ptr(router_w), _ptr(logits), _ptr(id_map), C.byref(st), _ptr(out),
                      _ptr(ids_out), _ptr(w_out)), self.h)
        return out

    def moe_ffn_streamed(self, x: torch.Tensor, cache: "SlotCache", router_w: torch.Tensor | None = None,
                         logits: torch.Tensor | None = None, ffn_norm: torch.Tensor | None = None,
                         use_norm: bool = False, out=None, ids_out=None, w_out=None, stream=None):
        """The streamed step of `--expert-slots N < E` (qwen3moe.rs:2021-2050): route, plan the
        chunks on the device, page misses in from the cache's host store, compute from the slots."""
        T = x.shape[0]
        out = torch.empty((T, self.cfg.n_embd), dtype=torch.float32, device=self.device) if out is None else out
        _lib.check(self.lib.tmoe_streamed_layer(self.h, _stream(stream), cache.s, _ptr(x), T, int(use_norm),
                                                _ptr(ffn_norm), _ptr(router_w), _ptr(logits), _ptr(out),
                                                _ptr(ids_out), _ptr(w_out)), self.h)
        return out

    def mul_mat_id(self, qtype: int, W: torch.Tensor, b: torch.Tensor, ids: torch.Tensor,
                   out: torch.Tensor | None = None, stream=None):
        """ggml mul_mat_id: W uint8 [n_w, N, row_size(K)], b f32 [T, b1, K], ids [T, n_used]
        -> f32 [T, n_used, N]; rows of id -1 are exactly zero."""
        n_w, N, rs = W.shape
        T, b1, K = b.shape
        n_used = ids.shape[1]
        if rs != row_size(qtype, K):
            raise ValueError("W row size does not match K")
        out = torch.empty((T, n_used, N), dtype=torch.float32, device=self.device) if out is None else out
        _lib.check(self.lib.tmoe_mul_mat_id(self.h, _stream(stream), qtype, _ptr(W), rs, N * rs, K, N, n_w,
                                            _ptr(b), b1, _ptr(ids), n_used, T, _ptr(out)), self.h)
        return out

    def dispatch(self, ids: torch.Tensor, n_slots: int, stream=None):
        """Per-expert pairs of ids [T, k] -> (counts [n_slots], offsets [n_slots+1], perm [T*k]);
        perm[offsets[n_slots]:] is unused."""
        T = ids.shape[0]
        counts = torch.empty(n_slots, dtype=torch.int32, device=self.device)
        offsets = torch.empty(n_slots + 1, dtype=torch.int32, device=self.device)
        perm = torch.full((ids.numel(),), -1, dtype=torch.int32, device=self.device)
        _lib.check(self.lib.tmoe_dispatch(self.h, _stream(stream), _ptr(ids), T, n_slots, _ptr(counts),
                                          _ptr(offsets), _ptr(perm)), self.h)
        return counts, offsets, perm

    def map_ids(self, ids: torch.Tensor, table: torch.Tensor, stream=None):
        out = torch.empty_like(ids)
        _lib.check(self.lib.tmoe_map_ids(self.h, _stream(stream), _ptr(ids), ids.numel(), _ptr(table),
                                         table.numel(), _ptr(out)), self.h)
        return out


class SlotCache:
    """The expert-slot cache of one MoE layer (LayerSlots, crates/memory/src/slots.rs) with its
    table on the device: `slots` are the device slot tensors, `store` the layer's experts in
    pinned host memory."""

    def __init__(self, layer: "MoeLayer", slots: ExpertWeights, store: ExpertWeights):
        self.layer, self.slots, self.store = layer, slots, store  # the cache keeps their pointers
        self._st = slots.c_struct()
        self._store = store.c_struct(host=True)
        h = C.c_void_p()
        _lib.check(layer.lib.tmoe_slots_create(layer.h, C.byref(self._st), C.byref(self._store), C.byref(h)),
                   layer.h)
        self.s = h
        self.n_slots = slots.gate.shape[0]
        self.n_expert = layer.cfg.n_expert
        self.max_chunks = layer.lib.tmoe_slots_max_chunks(self.s)

    def close(self):
        if self.s:
            self.layer.lib.tmoe_slots_destroy(self.s)
            self.s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def make_resident(self, experts, stream=None):
        arr = (C.c_int32 * max(len(experts), 1))(*experts)
        _lib.check(self.layer.lib.tmoe_slots_make_resident(self.s, _stream(stream), arr, len(experts)),
                   self.layer.h)

    def set_hot_set(self, hot, stream=None):
        arr = (C.c_int32 * max(len(hot), 1))(*hot)
        _lib.check(self.layer.lib.tmoe_slots_set_hot_set(self.s, _stream(stream), arr, len(hot)), self.layer.h)

    def state(self, stream=None):
        """(owner per slot, (hits, misses, bypasses), routed pairs per expert)."""
        owner = (C.c_int32 * self.n_slots)()
        stats = (C.c_int64 * 3)()
        counts = (C.c_int64 * self.n_expert)()
        _lib.check(self.layer.lib.tmoe_slots_state(self.s, _stream(stream), owner, stats, counts), self.layer.h)
        return list(owner), tuple(stats), list(counts)

    def last_plan(self, stream=None):
        """(n_chunks, map [max_chunks][E], loads per chunk as (expert, slot) lists)."""
        mc, E, S = self.max_chunks, self.n_expert, self.n_slots
        n = C.c_int32()
        m = (C.c_int32 * (mc * E))()
        ld = (C.c_int32 * (mc * S * 2))()
        nl = (C.c_int32 * mc)()
        _lib.check(self.layer.lib.tmoe_slots_last_plan(self.s, _stream(stream), C.byref(n), m, ld, nl),
                   self.layer.h)
        maps = [list(m[c * E:(c + 1) * E]) for c in range(mc)]
        loads = [[(ld[(c * S + i) * 2], ld[(c * S + i) * 2 + 1]) for i in range(nl[c])] for c in range(mc)]
        return n.value, maps, loads


def ep_id_map(n_expert: int, n_ranks: int, rank: int) -> list[int]:
    """The global -> local slot table of `rank` when the experts are split contiguously by id over
    `n_ranks` ranks (qwen3moe_shard.rs:11-14, 617-626): rank r holds [r*E/g, (r+1)*E/g) as slots
    0..E/g-1; the other experts map to -1."""
    if n_ranks < 1 or not 0 <= rank < n_ranks or n_expert % n_ranks:
        raise ValueError("n_expert must split evenly over the ranks")
    per = n_expert // n_ranks
    return [e - rank * per if rank * per <= e < (rank + 1) * per else -1 for e in range(n_expert)]


class EPComm:
    """A rank's communicator of an expert-parallel group (NCCL, one rank per GPU).  Rank 0 makes
    the id with unique_id(); every rank passes the same bytes."""

    def __init__(self, uid: bytes, n_ranks: int, rank: int, device: int | None = None, timeout_s: float = 60.0):
        self.lib = _lib.load()
        if len(uid) != _lib.COMM_ID_BYTES:
            raise ValueError("communicator id must be 128 bytes")
        dev = torch.cuda.current_device() if device is None else device
        c = C.c_void_p()
        buf = C.create_string_buffer(uid, _lib.COMM_ID_BYTES)
        _lib.check_comm(self.lib.tmoe_comm_init(buf, n_ranks, rank, dev, timeout_s, C.byref(c)))
        self.c, self.n_ranks, self.rank, self.device = c, n_ranks, rank, dev

    @staticmethod
    def unique_id() -> bytes:
        buf = C.create_string_buffer(_lib.COMM_ID_BYTES)
        _lib.check_comm(_lib.load().tmoe_comm_unique_id(buf))
        return buf.raw

    def abort(self):
        if getattr(self, "c", None):
            self.lib.tmoe_comm_abort(self.c)

    def close(self):
        if getattr(self, "c", None):
            self.lib.tmoe_comm_destroy(self.c)
            self.c = None


def ep_moe_ffn(layer: "MoeLayer", comm: EPComm, x: torch.Tensor, experts: ExpertWeights, id_map: torch.Tensor,
               router_w: torch.Tensor | None = None, logits: torch.Tensor | None = None,
               ffn_norm: torch.Tensor | None = None, use_norm: bool = False, out: torch.Tensor | None = None,
               ids_out: torch.Tensor | None = None, w_out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """The reference's EP MoE layer on this rank: moe_ffn over this rank's experts (id_map: the
    device int32 [E] table of ep_id_map) summed over the ranks of `comm`; every rank gets `out`."""
    T = x.shape[0]
    out = torch.empty((T, layer.cfg.n_embd), dtype=torch.float32, device=layer.device) if out is None else out
    st = experts.c_struct()
    _lib.check(layer.lib.tmoe_ep_layer(layer.h, _stream(stream), comm.c, _ptr(x), T, int(use_norm), _ptr(ffn_norm),
                                       _ptr(router_w), _ptr(logits), _ptr(id_map), C.byref(st), _ptr(out),
                                       _ptr(ids_out), _ptr(w_out)), layer.h)
    return out


def ep_a2a_moe_ffn(layer: "MoeLayer", comm: EPComm, x: torch.Tensor, experts: ExpertWeights,
                   router_w: torch.Tensor | None = None, logits: torch.Tensor | None = None,
                   ffn_norm: torch.Tensor | None = None, use_norm: bool = False, out: torch.Tensor | None = None,
                   ids_out: torch.Tensor | None = None, w_out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Expert parallelism with token dispatch/combine over an all-to-all: `x` are this rank's own
    tokens, `experts` its contiguous share (E / ranks experts); `out` gets this rank's tokens.
    The layer's max_tokens must be ranks x the tokens per rank (it computes the rows the other
    ranks send)."""
    T = x.shape[0]
    out = torch.empty((T, layer.cfg.n_embd), dtype=torch.float32, device=layer.device) if out is None else out
    st = experts.c_struct()
    _lib.check(layer.lib.tmoe_ep_a2a_layer(layer.h, _stream(stream), comm.c, _ptr(x), T, int(use_norm),
                                           _ptr(ffn_norm), _ptr(router_w), _ptr(logits), C.byref(st), _ptr(out),
                                           _ptr(ids_out), _ptr(w_out)), layer.h)
    return out


__all__ = ["MoeLayer", "ExpertWeights", "TmoeError", "TYPE_Q4_K", "TYPE_Q6_K", "TYPE_Q6_K_R8", "row_size", "quantize",
           "dequantize", "prepack",
           "EPComm", "ep_moe_ffn", "ep_a2a_moe_ffn", "ep_id_map", "SlotCache"]
