"""ctypes binding of libtmoe.so (include/tmoe.h).  No fallback: if the library is missing or
cannot load, every call raises."""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtmoe.so")
HEADER = os.path.join(HERE, "..", "include", "tmoe.h")

TMOE_OK = 0
ERRORS = {-1: "TMOE_E_INVALID", -2: "TMOE_E_CUDA", -3: "TMOE_E_NOMEM", -4: "TMOE_E_UNSUPPORTED",
          -5: "TMOE_E_DEVICE", -6: "TMOE_E_COMM", -7: "TMOE_E_NOTFOUND"}
TMOE_E_INVALID, TMOE_E_UNSUPPORTED, TMOE_E_NOTFOUND = -1, -4, -7
TYPE_Q4_K, TYPE_Q6_K = 12, 14
TYPE_Q6_K_R8 = 270  # Q6_K in 8-row fragment order (tmoe_prepack)


class TmoeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class Config(C.Structure):
    _fields_ = [("n_embd", C.c_int32), ("n_ff", C.c_int32), ("n_expert", C.c_int32),
                ("n_expert_used", C.c_int32), ("gate_type", C.c_int32), ("up_type", C.c_int32),
                ("down_type", C.c_int32), ("max_tokens", C.c_int32), ("device", C.c_int32),
                ("rms_eps", C.c_float)]


class ExpertTensors(C.Structure):
    _fields_ = [("gate", C.c_void_p), ("up", C.c_void_p), ("down", C.c_void_p),
                ("gate_nb1", C.c_size_t), ("gate_nb2", C.c_size_t),
                ("up_nb1", C.c_size_t), ("up_nb2", C.c_size_t),
                ("down_nb1", C.c_size_t), ("down_nb2", C.c_size_t),
                ("n_slots", C.c_int32)]


P = C.c_void_p
I32, I64 = C.c_int32, C.c_int64
SIGNATURES = {
    "tmoe_version": ([], C.c_int),
    "tmoe_create": ([C.POINTER(Config), C.POINTER(C.c_void_p)], C.c_int),
    "tmoe_destroy": ([P], None),
    "tmoe_last_error": ([P], C.c_char_p),
    "tmoe_check": ([P, P], C.c_int),
    "tmoe_wait_flag": ([P, P, P, I32, I64], C.c_int),
    "tmoe_mul_mat_id": ([P, P, I32, P, C.c_size_t, C.c_size_t, I64, I64, I64, P, I64, P, I64, I64, P],
                        C.c_int),
    "tmoe_mul_mat_id_noalloc": ([P, P, I32, P, C.c_size_t, C.c_size_t, I64, I64, I64, P, I64, P, I64, I64, P],
                                C.c_int),
    "tmoe_route": ([P, P, P, I64, I32, P, P, P, P, P, P, P], C.c_int),
    "tmoe_experts": ([P, P, P, I64, P, P, C.POINTER(ExpertTensors), P], C.c_int),
    "tmoe_layer": ([P, P, P, I64, I32, P, P, P, P, C.POINTER(ExpertTensors), P, P, P], C.c_int),
    "tmoe_layer_bf16": ([P, P, P, I64, I32, P, P, P, P, C.POINTER(ExpertTensors), P, P, P], C.c_int),
    "tmoe_map_ids": ([P, P, P, I64, P, I64, P], C.c_int),
    "tmoe_dispatch": ([P, P, P, I64, I32, P, P, P], C.c_int),
    "tmoe_quantize": ([I32, P, I64, I64, P, P], C.c_int),
    "tmoe_dequantize": ([I32, P, I64, P, P], C.c_int),
    "tmoe_prepack": ([I32, P, C.c_size_t, C.c_size_t, I64, I64, I64, P, P], C.c_int),
    "tmoe_profile_enable": ([P, I32], C.c_int),
    "tmoe_profile_collect": ([P, P, P], C.c_int),
    "tmoe_comm_unique_id": ([P], C.c_int),
    "tmoe_comm_init": ([P, I32, I32, I32, C.c_double, C.POINTER(C.c_void_p)], C.c_int),
    "tmoe_comm_abort": ([P], C.c_int),
    "tmoe_comm_destroy": ([P], None),
    "tmoe_comm_last_error": ([], C.c_char_p),
    "tmoe_ep_layer": ([P, P, P, P, I64, I32, P, P, P, P, C.POINTER(ExpertTensors), P, P, P], C.c_int),
    "tmoe_ep_a2a_layer": ([P, P, P, P, I64, I32, P, P, P, C.POINTER(ExpertTensors), P, P, P], C.c_int),
    "tmoe_slots_create": ([P, C.POINTER(ExpertTensors), C.POINTER(ExpertTensors), C.POINTER(C.c_void_p)], C.c_int),
    "tmoe_slots_destroy": ([P], None),
    "tmoe_slots_max_chunks": ([P], C.c_int),
    "tmoe_slots_make_resident": ([P, P, P, I32], C.c_int),
    "tmoe_slots_set_hot_set": ([P, P, P, I32], C.c_int),
    "tmoe_slots_state": ([P, P, P, P, P], C.c_int),
    "tmoe_slots_last_plan": ([P, P, P, P, P, P], C.c_int),
    "tmoe_streamed_layer": ([P, P, P, P, I64, I32, P, P, P, P, P, P], C.c_int),
    "tmoe_gguf_open": ([C.c_char_p, C.POINTER(C.c_void_p)], C.c_int),
    "tmoe_gguf_close": ([P], None),
    "tmoe_gguf_last_error": ([], C.c_char_p),
    "tmoe_gguf_n_shards": ([P], I32),
    "tmoe_gguf_n_kv": ([P], I64),
    "tmoe_gguf_kv_key": ([P, I64, C.POINTER(C.c_char_p)], C.c_int),
    "tmoe_gguf_kv": ([P, C.c_char_p, P, P, P, P, C.POINTER(C.c_char_p), P], C.c_int),
    "tmoe_gguf_n_tensors": ([P], I64),
    "tmoe_gguf_find_tensor": ([P, C.c_char_p], I64),
    "tmoe_gguf_tensor_info": ([P, I64, C.POINTER(C.c_char_p), P, P, P, P, P], C.c_int),
    "tmoe_gguf_type_size": ([I32, P, P], C.c_int),
    "tmoe_gguf_read": ([P, I64, C.c_uint64, C.c_uint64, P], C.c_int),
    "tmoe_gguf_load": ([P, I64, C.c_uint64, C.c_uint64, P, I32, P], C.c_int),
    "tmoe_mul_mat": ([P, P, I32, P, C.c_size_t, I64, I64, P, I64, I32, P], C.c_int),
    "tmoe_get_rows": ([P, P, I32, P, C.c_size_t, I64, I64, P, I64, P], C.c_int),
    "tmoe_rms_norm": ([P, P, P, P, C.c_float, I64, I64, P], C.c_int),
    "tmoe_rope_neox": ([P, P, P, P, I64, I32, I32, I32, C.c_float], C.c_int),
    "tmoe_qk_norm_rope": ([P, P, P, P, P, P, P, I64, I32, I32, I32, I32, C.c_float, C.c_float], C.c_int),
    "tmoe_attn_decode_scratch_bytes": ([P, I32, I32, I32, I32, I32], I64),
    "tmoe_attn_decode": ([P, P, P, P, P, P, P, P, I32, I32, I32, I32, I32, C.c_float, P, P], C.c_int),
    "tmoe_attn_prefill": ([P, P, P, P, P, P, P, I32, I32, I32, I32, I32, I32, I32, I32, C.c_float, P], C.c_int),
    "tmoe_add": ([P, P, P, P, P, I64], C.c_int),
    "tmoe_argmax": ([P, P, P, I64, I64, P], C.c_int),
    "tmoe_trace_open": ([C.c_char_p, C.POINTER(C.c_void_p)], C.c_int),
    "tmoe_trace_close": ([P], None),
    "tmoe_trace_last_error": ([], C.c_char_p),
    "tmoe_trace_header": ([P, P], C.c_int),
    "tmoe_trace_header_json": ([P], C.c_char_p),
    "tmoe_trace_header_str": ([P, C.c_char_p], C.c_char_p),
    "tmoe_trace_expert_bytes": ([P, P], C.c_int),
    "tmoe_trace_profile": ([P, P, P, P], C.c_int),
    "tmoe_trace_next": ([P, P, P, P, P, P], C.c_int),
    "tmoe_trace_ids": ([P, I32, P], C.c_int),
    "tmoe_trace_create": ([C.c_char_p, C.c_char_p, C.POINTER(C.c_void_p)], C.c_int),
    "tmoe_trace_write_step": ([P, C.c_uint32, I32, C.c_uint32, P, P, P], C.c_int),
    "tmoe_trace_write_refresh": ([P, C.c_uint32], C.c_int),
    "tmoe_trace_finish": ([P], C.c_int),
}
COMM_ID_BYTES = 128
PHASES = ["rms_norm", "router_logits", "topk", "map_ids", "dispatch", "quant_x", "gate_up", "quant_act",
          "down", "combine", "slot_plan", "slot_page"]

_lib = None


def header_symbols() -> list[str]:
    """Every function the C ABI header declares."""
    with open(HEADER) as f:
        text = f.read()
    return re.findall(r"TMOE_API\s+[\w\s\*]+?\b(tmoe_\w+)\s*\(", text)


def load():
    """Loads libtmoe.so (building it first if it is absent and nvcc is here)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        from . import build as _build
        _build.build()
    lib = C.CDLL(LIB_PATH)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


def check(rc: int, handle=None):
    if rc != TMOE_OK:
        msg = load().tmoe_last_error(handle)
        raise TmoeError(rc, msg.decode() if msg else "")


def check_comm(rc: int):
    """For the communicator calls, whose errors are kept per thread."""
    if rc != TMOE_OK:
        msg = load().tmoe_comm_last_error()
        raise TmoeError(rc, msg.decode() if msg else "")
