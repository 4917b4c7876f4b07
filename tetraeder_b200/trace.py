"""Routing traces (the `tetraeder-routing` v1 format of crates/memory/src/replay/trace.rs) over the C
ABI, for replaying recorded routing into the MoE layer and for recording a run's routing.

  TraceHeader            <- TraceHeader (trace.rs:27-90): the same fields; new(n_layer, n_expert,
                            n_used) derives the id width
  TraceReader            <- TraceReader (trace.rs:225-330): iterates LayerStep / HotRefresh records;
                            a truncated or corrupt record raises TraceError
  TraceWriter            <- TraceWriter (trace.rs:120-200)
  LayerStep.logits(E)    router logits whose top-k (lower index first on ties) is exactly the
                         step's recorded choice, in order, so a recorded step can be replayed through
                         the layer's own routing (tmoe_layer / tmoe_streamed_layer with `logits`)
"""
from __future__ import annotations

import ctypes as C
import json
from dataclasses import dataclass, field

import numpy as np

from . import _lib

FORMAT, VERSION = "tetraeder-routing", 1


class TraceError(Exception):
    def __init__(self, msg: str, code: int = _lib.TMOE_E_INVALID):
        super().__init__(msg)
        self.code = code


def _check(rc: int):
    if rc < 0:
        raise TraceError(_lib.load().tmoe_trace_last_error().decode(errors="replace"), rc)
    return rc


class _Info(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("version", "n_layer", "n_expert", "n_used", "id_bytes", "vram_slots",
                                         "ram_slots", "prefetch_depth", "ubatch")] + [("has_profile", C.c_int32)]


@dataclass
class TraceHeader:
    n_layer: int
    n_expert: int
    n_used: int
    format: str = FORMAT
    version: int = VERSION
    model: str = ""
    id_bytes: int = 0
    vram_slots: int = 0
    ram_slots: int = 0
    prefetch_depth: int = 0
    hot_source: str = "first_prefill"
    ubatch: int = 0
    prompt_hash: str = ""
    expert_bytes: list = field(default_factory=list)
    profile: list | None = None

    def __post_init__(self):
        if not self.id_bytes:
            self.id_bytes = 1 if self.n_expert <= 256 else 2
        if not self.expert_bytes:
            self.expert_bytes = [0] * self.n_layer

    def to_json(self) -> str:
        d = {k: getattr(self, k) for k in ("format", "version", "model", "n_layer", "n_expert", "n_used", "id_bytes",
                                           "vram_slots", "ram_slots", "prefetch_depth", "hot_source", "ubatch",
                                           "prompt_hash", "expert_bytes")}
        if self.profile is not None:
            d["profile"] = self.profile
        return json.dumps(d, separators=(",", ":"), ensure_ascii=False)


@dataclass
class LayerStep:
    step: int
    layer: int
    n_tokens: int
    ids: np.ndarray                       # int32 [n_tokens, n_used]
    predicted: np.ndarray | None = None
    predicted2: np.ndarray | None = None

    def logits(self, n_expert: int) -> np.ndarray:
        """f32 [n_tokens, n_expert] logits whose softmax top-k selects exactly `ids`, in order: choice
        j of a token gets 16 - j, every other expert 0 (distinct values, no ties to break)."""
        T, k = self.ids.shape
        lg = np.zeros((T, n_expert), dtype=np.float32)
        lg[np.arange(T)[:, None], self.ids] = (16.0 - np.arange(k, dtype=np.float32))[None, :]
        return lg


@dataclass
class HotRefresh:
    step: int


class TraceReader:
    def __init__(self, path):
        self.lib = _lib.load()
        h = C.c_void_p()
        _check(self.lib.tmoe_trace_open(str(path).encode(), C.byref(h)))
        self.h = h
        info = _Info()
        _check(self.lib.tmoe_trace_header(self.h, C.byref(info)))
        s = lambda f: self.lib.tmoe_trace_header_str(self.h, f.encode()).decode()  # noqa: E731
        eb = (C.c_uint64 * info.n_layer)()
        _check(self.lib.tmoe_trace_expert_bytes(self.h, eb))
        profile = None
        if info.has_profile:
            r, c = C.c_int64(), C.c_int64()
            _check(self.lib.tmoe_trace_profile(self.h, C.byref(r), C.byref(c), None))
            buf = np.zeros(r.value * max(c.value, 0), dtype=np.uint64)
            _check(self.lib.tmoe_trace_profile(self.h, None, None, buf.ctypes.data_as(C.c_void_p)))
            profile = buf.reshape(r.value, c.value).tolist()
        self.header = TraceHeader(n_layer=info.n_layer, n_expert=info.n_expert, n_used=info.n_used,
                                  format=s("format"), version=info.version, model=s("model"), id_bytes=info.id_bytes,
                                  vram_slots=info.vram_slots, ram_slots=info.ram_slots,
                                  prefetch_depth=info.prefetch_depth, hot_source=s("hot_source"), ubatch=info.ubatch,
                                  prompt_hash=s("prompt_hash"), expert_bytes=list(eb), profile=profile)
        self.header_json = self.lib.tmoe_trace_header_json(self.h).decode()

    def __iter__(self):
        return self

    def __next__(self):
        kind, step, layer, n, flags = C.c_int32(), C.c_uint32(), C.c_int32(), C.c_uint32(), C.c_int32()
        rc = _check(self.lib.tmoe_trace_next(self.h, C.byref(kind), C.byref(step), C.byref(layer), C.byref(n),
                                             C.byref(flags)))
        if rc == 0:
            raise StopIteration
        if kind.value == 1:
            return HotRefresh(step.value)
        k = self.header.n_used

        def ids(which):
            a = np.empty((n.value, k), dtype=np.int32)
            _check(self.lib.tmoe_trace_ids(self.h, which, a.ctypes.data_as(C.c_void_p)))
            return a

        return LayerStep(step.value, layer.value, n.value, ids(0), ids(1) if flags.value & 1 else None,
                         ids(2) if flags.value & 2 else None)

    def close(self):
        if getattr(self, "h", None):
            self.lib.tmoe_trace_close(self.h)
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


class TraceWriter:
    def __init__(self, path, header: TraceHeader):
        self.lib = _lib.load()
        self.header = header
        h = C.c_void_p()
        _check(self.lib.tmoe_trace_create(str(path).encode(), header.to_json().encode(), C.byref(h)))
        self.h = h

    def layer_step(self, step: int, layer: int, ids, predicted=None, predicted2=None):
        """ids (and predictions): [n_tokens, n_used] (or flat, token-major) integer arrays."""
        arrs = [None if a is None else np.ascontiguousarray(np.asarray(a), dtype=np.int32).reshape(-1)
                for a in (ids, predicted, predicted2)]
        n = arrs[0].size
        for a in arrs:
            if a is not None and a.size != n:
                raise TraceError(f"{a.size} ids for {n} expected")
        if n % self.header.n_used:
            raise TraceError(f"{n} ids is not a whole number of tokens of {self.header.n_used}")
        ptr = [None if a is None else a.ctypes.data_as(C.c_void_p) for a in arrs]
        _check(self.lib.tmoe_trace_write_step(self.h, step, layer, n // self.header.n_used, *ptr))

    def hot_refresh(self, step: int):
        _check(self.lib.tmoe_trace_write_refresh(self.h, step))

    def finish(self):
        if getattr(self, "h", None):
            h, self.h = self.h, None
            _check(self.lib.tmoe_trace_finish(h))

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.finish()
