"""CPU oracle of Tetraeder's Qwen3-MoE layer hot path (ctypes over libtmoe_oracle.so).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py, always as the checker or the
timed CPU stand-in for ggml's CPU mul_mat_id path (which is not present in the
reference tree: llama.cpp b12426 is an empty submodule).  The product
(tetraeder_b200) never imports this module.

Reference lines each function follows are listed in oracle/tmoe_oracle.h.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtmoe_oracle.so")

TYPE_F32, TYPE_F16, TYPE_Q4_K, TYPE_Q6_K, TYPE_Q8_K = 0, 1, 12, 14, 15
QK_K = 256
MODE_Q8K, MODE_F64 = 0, 1
BLOCK_BYTES = {TYPE_Q4_K: 144, TYPE_Q6_K: 210, TYPE_Q8_K: 292}

Q8K_DTYPE = np.dtype([("d", "<f4"), ("qs", "i1", (256,)), ("bsums", "<i2", (16,))])
assert Q8K_DTYPE.itemsize == 292

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc, OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
I64 = C.c_int64


def _declare(L):
    L.tmo_f16_to_f32.argtypes, L.tmo_f16_to_f32.restype = [C.c_uint16], C.c_float
    L.tmo_f32_to_f16.argtypes, L.tmo_f32_to_f16.restype = [C.c_float], C.c_uint16
    L.tmo_row_size.argtypes, L.tmo_row_size.restype = [C.c_int, I64], C.c_size_t
    L.tmo_quantize_q4k.argtypes = [P, P, I64, I64]
    L.tmo_quantize_q6k.argtypes = [P, P, I64, I64]
    L.tmo_dequantize.argtypes = [C.c_int, P, P, I64]
    L.tmo_quantize_q8k.argtypes = [P, P, I64]
    L.tmo_dequantize_q8k.argtypes = [P, P, I64]
    L.tmo_vec_dot_q4k_q8k.argtypes, L.tmo_vec_dot_q4k_q8k.restype = [I64, P, P], C.c_float
    L.tmo_vec_dot_q6k_q8k.argtypes, L.tmo_vec_dot_q6k_q8k.restype = [I64, P, P], C.c_float
    L.tmo_vec_dot_q4k_q8k_simd.argtypes, L.tmo_vec_dot_q4k_q8k_simd.restype = [I64, P, P], C.c_float
    L.tmo_vec_dot_q6k_q8k_simd.argtypes, L.tmo_vec_dot_q6k_q8k_simd.restype = [I64, P, P], C.c_float
    L.tmo_dot_cols.argtypes = [C.c_int, I64, P, P, C.c_int, P]
    L.tmo_exp_canon.argtypes, L.tmo_exp_canon.restype = [C.c_float], C.c_float
    L.tmo_router_dot.argtypes, L.tmo_router_dot.restype = [P, P, I64], C.c_float
    L.tmo_rms_norm.argtypes = [P, P, C.c_float, P, I64]
    L.tmo_softmax_topk.argtypes = [P, C.c_int, C.c_int, P, P, P]
    L.tmo_router_logits.argtypes = [P, P, I64, I64, I64, P]
    L.tmo_route.argtypes = [P, I64, I64, I64, C.c_int, C.c_int, P, C.c_float, P, P, P, P, P, P]
    L.tmo_map_ids.argtypes = [P, I64, P, I64, P]
    L.tmo_sort_pairs.argtypes, L.tmo_sort_pairs.restype = [P, I64, C.c_int, I64, P, P, P], I64
    L.tmo_mul_mat_id.argtypes = [C.c_int, P, C.c_size_t, C.c_size_t, I64, I64, I64, P, I64, I64, P,
                                 C.c_int, P, C.c_int, C.c_int]
    L.tmo_mul_mat_id.restype = C.c_int
    L.tmo_experts.argtypes = [P, I64, I64, I64, I64, C.c_int, P, P,
                              C.c_int, P, C.c_size_t, C.c_size_t,
                              C.c_int, P, C.c_size_t, C.c_size_t,
                              C.c_int, P, C.c_size_t, C.c_size_t, P, P, C.c_int, C.c_int]
    L.tmo_experts.restype = C.c_int


def _p(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


def row_size(qtype: int, ncols: int) -> int:
    return int(lib().tmo_row_size(qtype, ncols))


def quantize(qtype: int, x: np.ndarray) -> np.ndarray:
    """Our own Q4_K / Q6_K fit of x [..., ncols] -> uint8 [..., row_size]."""
    x = _c(x, np.float32)
    ncols = x.shape[-1]
    nrows = x.size // ncols
    out = np.zeros(x.shape[:-1] + (row_size(qtype, ncols),), dtype=np.uint8)
    fn = {TYPE_Q4_K: lib().tmo_quantize_q4k, TYPE_Q6_K: lib().tmo_quantize_q6k}[qtype]
    fn(_p(x), _p(out), nrows, ncols)
    return out


def dequantize(qtype: int, data: np.ndarray, n: int) -> np.ndarray:
    data = np.ascontiguousarray(data)
    out = np.empty(n, dtype=np.float32)
    lib().tmo_dequantize(qtype, _p(data), _p(out), n)
    return out


def quantize_q8k(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32).reshape(-1)
    out = np.zeros(x.size // QK_K, dtype=Q8K_DTYPE)
    lib().tmo_quantize_q8k(_p(x), _p(out), x.size)
    return out


def dequantize_q8k(blocks: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks)
    out = np.empty(blocks.size * QK_K, dtype=np.float32)
    lib().tmo_dequantize_q8k(_p(blocks), _p(out), out.size)
    return out


def exp_canon(x: float) -> float:
    return float(lib().tmo_exp_canon(float(x)))


def router_logits(xn: np.ndarray, router_w: np.ndarray) -> np.ndarray:
    xn = _c(xn, np.float32)
    router_w = _c(router_w, np.float32)
    T, H = xn.shape
    E = router_w.shape[0]
    out = np.empty((T, E), dtype=np.float32)
    lib().tmo_router_logits(_p(xn), _p(router_w), T, H, E, _p(out))
    return out


def route(x, k, router_w=None, logits=None, norm=False, norm_w=None, eps=1e-6):
    """Router of qwen3moe.rs:2871-2890 -> (ids int32 [T,k], w f32 [T,k], xn, logits)."""
    x = _c(x, np.float32)
    T, H = x.shape
    if router_w is not None:
        router_w = _c(router_w, np.float32)
        E = router_w.shape[0]
    else:
        logits = _c(logits, np.float32)
        E = logits.shape[1]
    if norm_w is not None:
        norm_w = _c(norm_w, np.float32)
    ids = np.empty((T, k), dtype=np.int32)
    w = np.empty((T, k), dtype=np.float32)
    xn = np.empty((T, H), dtype=np.float32)
    lg = np.empty((T, E), dtype=np.float32)
    lib().tmo_route(_p(x), T, H, E, k, int(bool(norm)), _p(norm_w), eps, _p(router_w), _p(logits),
                    _p(xn), _p(lg), _p(ids), _p(w))
    return ids, w, xn, lg


def softmax_topk(logits: np.ndarray, k: int):
    logits = _c(logits, np.float32)
    E = logits.shape[-1]
    rows = logits.reshape(-1, E)
    probs = np.empty_like(rows)
    ids = np.empty((rows.shape[0], k), dtype=np.int32)
    w = np.empty((rows.shape[0], k), dtype=np.float32)
    for r in range(rows.shape[0]):
        lib().tmo_softmax_topk(_p(rows[r]), E, k, _p(probs[r]), _p(ids[r]), _p(w[r]))
    return ids, w, probs


def map_ids(ids: np.ndarray, table: np.ndarray) -> np.ndarray:
    ids = _c(ids, np.int32)
    table = _c(table, np.int32)
    out = np.empty_like(ids)
    lib().tmo_map_ids(_p(ids), ids.size, _p(table), table.size, _p(out))
    return out


def sort_pairs(ids: np.ndarray, n_expert: int):
    """Per-expert pairs in token-major, choice-minor order -> (counts, offsets, perm)."""
    ids = _c(ids, np.int32)
    T, k = ids.shape
    counts = np.empty(n_expert, dtype=np.int32)
    offsets = np.empty(n_expert + 1, dtype=np.int32)
    perm = np.empty(T * k, dtype=np.int32)
    n = lib().tmo_sort_pairs(_p(ids), T, k, n_expert, _p(counts), _p(offsets), _p(perm))
    return counts, offsets, perm[:n].copy()


def mul_mat_id(qtype, W, K, N, E, b, ids, mode=MODE_Q8K, nb1=None, nb2=None, nthreads=0):
    """ggml mul_mat_id: W [E, N, row_size] bytes, b f32 [T, b1, K], ids [T, n_used] -> [T, n_used, N]."""
    W = np.ascontiguousarray(W)
    b = _c(b, np.float32)
    ids = _c(ids, np.int32)
    T, n_used = ids.shape
    b1 = b.shape[1]
    rs = row_size(qtype, K)
    nb1 = rs if nb1 is None else nb1
    nb2 = rs * N if nb2 is None else nb2
    out = np.empty((T, n_used, N), dtype=np.float32)
    rc = lib().tmo_mul_mat_id(qtype, _p(W), nb1, nb2, K, N, E, _p(b), b1, T, _p(ids), n_used,
                              _p(out), mode, nthreads)
    if rc:
        raise ValueError("tmo_mul_mat_id: invalid arguments")
    return out


def experts(x, ids, w, gate, up, down, H, I, E, gate_type=TYPE_Q4_K, up_type=TYPE_Q4_K,
            down_type=TYPE_Q4_K, mode=MODE_Q8K, nthreads=0, want_act=False):
    """weighted_experts + sum_experts (qwen3moe.rs:2899-2923) -> out f32 [T, H]."""
    x = _c(x, np.float32)
    ids = _c(ids, np.int32)
    w = _c(w, np.float32)
    gate, up, down = (np.ascontiguousarray(a) for a in (gate, up, down))
    T, k = ids.shape
    gr, ur, dr = row_size(gate_type, H), row_size(up_type, H), row_size(down_type, I)
    out = np.empty((T, H), dtype=np.float32)
    act = np.empty((T, k, I), dtype=np.float32) if want_act else None
    rc = lib().tmo_experts(_p(x), T, H, I, E, k, _p(ids), _p(w),
                           gate_type, _p(gate), gr, gr * I,
                           up_type, _p(up), ur, ur * I,
                           down_type, _p(down), dr, dr * H, _p(out), _p(act), mode, nthreads)
    if rc:
        raise ValueError("tmo_experts: invalid arguments")
    return (out, act) if want_act else out


def layer(x, k, gate, up, down, H, I, E, router_w=None, logits=None, gate_type=TYPE_Q4_K,
          up_type=TYPE_Q4_K, down_type=TYPE_Q4_K, mode=MODE_Q8K, nthreads=0, id_map=None):
    """router + (optional EP id map) + weighted_experts + sum_experts -> (out, ids, w)."""
    ids, w, xn, _ = route(x, k, router_w=router_w, logits=logits)
    used = ids if id_map is None else map_ids(ids, id_map)
    out = experts(xn, used, w, gate, up, down, H, I, E if id_map is None else int(id_map.max()) + 1,
                  gate_type, up_type, down_type, mode, nthreads)
    return out, ids, w
