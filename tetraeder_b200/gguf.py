"""GGUF model files over the C ABI (libtmoe.so's reader): the header reader of the reference's
crates/model/src/gguf.rs, the qwen3moe hyperparameters of crates/model/src/hparams.rs and the
tensor reads of load_weights (crates/model/src/qwen3moe.rs:2498-2584), narrowed to what the MoE
layer consumes: the router, the FFN norm and the stacked expert tensors.

  GgufFile                  <- Gguf (gguf.rs:89-99), opened by Gguf::open (:236-296), split models
                               from their first shard
  GgufFile.get/str/u64/f32  <- Gguf::get/str/u64/u64_or/f32/f32_or (:409-450), same type rules
  GgufFile.tensor           <- Gguf::tensor (:452-457); TensorInfo.slab <- TensorInfo::slab (:76-86)
  Hparams.from_gguf         <- Hparams::from_gguf (hparams.rs:65-109)
  GgufFile.expert_slabs     <- the gate/up/down slabs of one expert (hparams.rs ExpertSlabs)
  GgufFile.load_experts     <- load_weights' reads of the `_exps` tensors, into device memory (or a
                               pinned host store for the slot cache)

Errors raise GgufError with the reference's message forms ("missing key `…`", "missing tensor
`…`", "key `…` has the wrong type", "not a GGUF file (bad magic)", …)."""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

ARCH = "qwen3moe"
EXPERT_TENSORS = ("ffn_gate_exps", "ffn_up_exps", "ffn_down_exps")
TYPE_F32, TYPE_F16 = 0, 1
KIND_U64, KIND_I64, KIND_F64, KIND_BOOL, KIND_STR, KIND_ARRAY = range(6)


class GgufError(Exception):
    def __init__(self, msg: str, code: int = _lib.TMOE_E_INVALID):
        super().__init__(msg)
        self.code = code


def _check(rc: int):
    if rc != 0:
        raise GgufError(_lib.load().tmoe_gguf_last_error().decode(errors="replace"), rc)


def type_size(ggml_type: int) -> tuple[int, int]:
    """(block elements, bytes per block) of a ggml type id."""
    b, n = C.c_int32(), C.c_int32()
    _check(_lib.load().tmoe_gguf_type_size(ggml_type, C.byref(b), C.byref(n)))
    return b.value, n.value


def layer_name(il: int, what: str) -> str:
    return f"blk.{il}.{what}.weight"


@dataclass(frozen=True)
class Slab:
    shard: int
    offset: int
    len: int


@dataclass(frozen=True)
class TensorInfo:
    index: int
    name: str
    type: int
    ne: tuple
    shard: int
    offset: int
    nbytes: int

    def slab(self, i: int) -> Slab | None:
        """Slab i along ne[2] (an expert of a stacked expert tensor), or None past the end."""
        n = self.ne[2]
        if not 0 <= i < n:
            return None
        ln = self.nbytes // n
        return Slab(self.shard, self.offset + i * ln, ln)


@dataclass(frozen=True)
class ArrayValue:
    """A metadata array: only its length is kept (the reference skips the items)."""
    len: int


@dataclass
class Hparams:
    name: str
    n_layer: int
    n_ctx_train: int
    n_embd: int
    n_head: int
    n_head_kv: int
    head_dim: int
    n_rot: int
    n_expert: int
    n_expert_used: int
    n_ff_exp: int
    n_vocab: int
    rms_eps: float
    rope_freq_base: float
    tied_output: bool

    @staticmethod
    def from_gguf(g: "GgufFile") -> "Hparams":
        arch = g.str("general.architecture")
        if arch != ARCH:
            raise GgufError(f"corrupt GGUF: architecture `{arch}`, expected `{ARCH}`")

        def k(s):
            return f"{ARCH}.{s}"

        n_head = g.u64(k("attention.head_count"))
        n_embd = g.u64(k("embedding_length"))
        head_dim = g.u64_or(k("attention.key_length"), n_embd // max(n_head, 1))
        if g.u64_or(k("attention.value_length"), head_dim) != head_dim:
            raise GgufError("corrupt GGUF: key and value lengths differ")
        scaling = g.get(k("rope.scaling.type"))
        if scaling is not None and scaling != "none":
            raise GgufError("corrupt GGUF: rope scaling is not supported")
        tok = g.tensor("token_embd.weight")
        try:
            name = g.str("general.name")
        except GgufError:
            name = ARCH
        return Hparams(
            name=name,
            n_layer=g.u64(k("block_count")),
            n_ctx_train=g.u64(k("context_length")),
            n_embd=n_embd,
            n_head=n_head,
            n_head_kv=g.u64(k("attention.head_count_kv")),
            head_dim=head_dim,
            n_rot=g.u64_or(k("rope.dimension_count"), head_dim),
            n_expert=g.u64(k("expert_count")),
            n_expert_used=g.u64(k("expert_used_count")),
            n_ff_exp=g.u64(k("expert_feed_forward_length")),
            n_vocab=tok.ne[1],
            rms_eps=g.f32(k("attention.layer_norm_rms_epsilon")),
            rope_freq_base=g.f32_or(k("rope.freq_base"), 10000.0),
            tied_output=not g.has_tensor("output.weight"),
        )


class GgufFile:
    """An open GGUF model (all shards of a split model).  Use as a context manager or close()."""

    def __init__(self, path: str):
        self.lib = _lib.load()
        h = C.c_void_p()
        _check(self.lib.tmoe_gguf_open(str(path).encode(), C.byref(h)))
        self.h = h
        self.path = str(path)
        self.n_shards = int(self.lib.tmoe_gguf_n_shards(self.h))
        self.tensors = [self._info(i) for i in range(int(self.lib.tmoe_gguf_n_tensors(self.h)))]
        self._by_name = {t.name: t for t in self.tensors}
        self._hparams = None

    def close(self):
        if getattr(self, "h", None):
            self.lib.tmoe_gguf_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- metadata ------------------------------------------------------------------------
    def keys(self) -> list[str]:
        out = []
        for i in range(int(self.lib.tmoe_gguf_n_kv(self.h))):
            k = C.c_char_p()
            _check(self.lib.tmoe_gguf_kv_key(self.h, i, C.byref(k)))
            out.append(k.value.decode())
        return out

    def get(self, key: str):
        """The value of `key` (int, float, bool, str or ArrayValue), or None if absent."""
        kind, u, i, f, n = C.c_int32(), C.c_uint64(), C.c_int64(), C.c_double(), C.c_uint64()
        s = C.c_char_p()
        rc = self.lib.tmoe_gguf_kv(self.h, key.encode(), C.byref(kind), C.byref(u), C.byref(i), C.byref(f),
                                   C.byref(s), C.byref(n))
        if rc == _lib.TMOE_E_NOTFOUND:
            return None
        _check(rc)
        return {KIND_U64: lambda: u.value, KIND_I64: lambda: i.value, KIND_F64: lambda: f.value,
                KIND_BOOL: lambda: bool(u.value), KIND_STR: lambda: s.value.decode(),
                KIND_ARRAY: lambda: ArrayValue(n.value)}[kind.value]()

    def _kind(self, key):
        kind = C.c_int32()
        rc = self.lib.tmoe_gguf_kv(self.h, key.encode(), C.byref(kind), None, None, None, None, None)
        if rc == _lib.TMOE_E_NOTFOUND:
            raise GgufError(f"missing key `{key}`", rc)
        _check(rc)
        return kind.value

    def str(self, key: str) -> str:
        if self._kind(key) != KIND_STR:
            raise GgufError(f"key `{key}` has the wrong type")
        return self.get(key)

    def u64(self, key: str) -> int:
        kind = self._kind(key)
        v = self.get(key)
        if kind == KIND_U64 or (kind == KIND_I64 and v >= 0):
            return int(v)
        raise GgufError(f"key `{key}` has the wrong type")

    def u64_or(self, key: str, default: int) -> int:
        return self.u64(key) if self.get(key) is not None else default

    def f32(self, key: str) -> float:
        if self._kind(key) != KIND_F64:
            raise GgufError(f"key `{key}` has the wrong type")
        return float(np.float32(self.get(key)))

    def f32_or(self, key: str, default: float) -> float:
        return self.f32(key) if self.get(key) is not None else default

    @property
    def hparams(self) -> Hparams:
        if self._hparams is None:
            self._hparams = Hparams.from_gguf(self)
        return self._hparams

    # -- tensors -------------------------------------------------------------------------
    def _info(self, i: int) -> TensorInfo:
        name, ty, shard = C.c_char_p(), C.c_int32(), C.c_int32()
        ne = (C.c_int64 * 4)()
        off, nb = C.c_uint64(), C.c_uint64()
        _check(self.lib.tmoe_gguf_tensor_info(self.h, i, C.byref(name), C.byref(ty), ne, C.byref(shard),
                                              C.byref(off), C.byref(nb)))
        return TensorInfo(i, name.value.decode(), ty.value, tuple(ne), shard.value, off.value, nb.value)

    def has_tensor(self, name: str) -> bool:
        return name in self._by_name

    def tensor(self, name: str) -> TensorInfo:
        t = self._by_name.get(name)
        if t is None:
            raise GgufError(f"missing tensor `{name}`", _lib.TMOE_E_NOTFOUND)
        return t

    def layer_tensor(self, il: int, what: str) -> TensorInfo:
        return self.tensor(layer_name(il, what))

    def read(self, name: str, offset: int = 0, nbytes: int | None = None) -> np.ndarray:
        """Bytes [offset, offset + nbytes) of a tensor, into host memory."""
        t = self.tensor(name)
        n = t.nbytes - offset if nbytes is None else nbytes
        out = np.empty(n, dtype=np.uint8)
        _check(self.lib.tmoe_gguf_read(self.h, t.index, offset, n, out.ctypes.data_as(C.c_void_p)))
        return out

    def read_into(self, name: str, dst: torch.Tensor, offset: int = 0):
        """Bytes [offset, offset + dst.numel()) of a tensor into a CPU uint8 tensor (pinned or not)."""
        t = self.tensor(name)
        if dst.is_cuda or dst.dtype != torch.uint8 or not dst.is_contiguous():
            raise ValueError("dst must be a contiguous CPU uint8 tensor")
        _check(self.lib.tmoe_gguf_read(self.h, t.index, offset, dst.numel(), C.c_void_p(dst.data_ptr())))

    def load(self, name: str, out: torch.Tensor, offset: int = 0, stream=None):
        """Bytes [offset, offset + out.numel()) of a tensor into a CUDA uint8 tensor (returns once
        the copies have landed)."""
        t = self.tensor(name)
        if not out.is_cuda or out.dtype != torch.uint8 or not out.is_contiguous():
            raise ValueError("out must be a contiguous CUDA uint8 tensor")
        s = torch.cuda.current_stream(out.device) if stream is None else stream
        _check(self.lib.tmoe_gguf_load(self.h, t.index, offset, out.numel(), C.c_void_p(out.data_ptr()),
                                       out.device.index, C.c_void_p(s.cuda_stream)))

    # -- the MoE layer's tensors ------------------------------------------------------------
    def expert_slabs(self, il: int, e: int) -> tuple[Slab, Slab, Slab]:
        """Where expert e of layer il lives: its gate, up and down slabs."""
        parts = []
        for name in EXPERT_TENSORS:
            s = self.layer_tensor(il, name).slab(e)
            if s is None:
                raise GgufError(f"expert {e} out of range for layer {il}")
            parts.append(s)
        return tuple(parts)

    def load_experts(self, il: int, device=None, first: int = 0, count: int | None = None, pinned: bool = False):
        """Experts [first, first + count) of layer il as ExpertWeights (uint8 [count, rows, row
        bytes], ggml layout): on `device`, or with device=None in host memory (pinned=True: a store
        for SlotCache).  A contiguous run of experts is one contiguous read per matrix."""
        from .moe import ExpertWeights
        ts = [self.layer_tensor(il, n) for n in EXPERT_TENSORS]
        E = ts[0].ne[2]
        count = E - first if count is None else count
        if first < 0 or count < 1 or first + count > E or any(t.ne[2] != E for t in ts):
            raise GgufError(f"experts [{first}, {first + count}) out of range for layer {il} ({E} experts)")
        mats = []
        for t in ts:
            rows = t.ne[1]
            row_bytes = t.nbytes // (t.ne[1] * t.ne[2] * t.ne[3])
            slab = t.nbytes // E
            shape = (count, rows, row_bytes)
            if device is None:
                dst = torch.empty(shape, dtype=torch.uint8, pin_memory=pinned)
                self.read_into(t.name, dst.view(-1), first * slab)
            else:
                dst = torch.empty(shape, dtype=torch.uint8, device=device)
                self.load(t.name, dst.view(-1), first * slab)
            mats.append(dst)
        return ExpertWeights(*mats)

    def load_moe_layer(self, il: int, device):
        """(router weights f32 [E, H], ffn_norm f32 [H], ExpertWeights) of layer il on `device`, as
        the MoE layer consumes them; the expert types must be Q4_K or Q6_K."""
        hp = self.hparams
        gi, fn = self.layer_tensor(il, "ffn_gate_inp"), self.layer_tensor(il, "ffn_norm")
        if gi.type != TYPE_F32 or gi.ne[:2] != (hp.n_embd, hp.n_expert) or fn.type != TYPE_F32:
            raise GgufError(f"layer {il}: router and FFN norm must be F32 [{hp.n_embd}, {hp.n_expert}] / [{hp.n_embd}]")
        for n in EXPERT_TENSORS:
            t = self.layer_tensor(il, n)
            if t.type not in (_lib.TYPE_Q4_K, _lib.TYPE_Q6_K):
                raise GgufError(f"`{t.name}` has ggml type {t.type}; the MoE layer takes Q4_K (12) or Q6_K (14)",
                                _lib.TMOE_E_UNSUPPORTED)
        rw = torch.empty(gi.nbytes, dtype=torch.uint8, device=device)
        self.load(gi.name, rw)
        nw = torch.empty(fn.nbytes, dtype=torch.uint8, device=device)
        self.load(fn.name, nw)
        experts = self.load_experts(il, device=device)
        return rw.view(torch.float32).view(hp.n_expert, hp.n_embd), nw.view(torch.float32), experts

    def expert_types(self, il: int) -> tuple[int, int, int]:
        return tuple(self.layer_tensor(il, n).type for n in EXPERT_TENSORS)
