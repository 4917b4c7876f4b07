//! Raw declarations of every entry point of `include/tmoe.h` (the C ABI of libtmoe.so), in the
//! header's order, with the structs and constants they use.  tests/test_tmoe_sys.py of the
//! repository holds the names, parameter names and types to the header's.
#![allow(non_camel_case_types, non_snake_case)]

use std::ffi::{c_char, c_int, c_void};

pub const TMOE_OK: c_int = 0;
pub const TMOE_E_INVALID: c_int = -1;
pub const TMOE_E_CUDA: c_int = -2;
pub const TMOE_E_NOMEM: c_int = -3;
pub const TMOE_E_UNSUPPORTED: c_int = -4;
pub const TMOE_E_DEVICE: c_int = -5;
pub const TMOE_E_COMM: c_int = -6;
pub const TMOE_E_NOTFOUND: c_int = -7;
pub const TMOE_TYPE_Q4_K: c_int = 12;
pub const TMOE_TYPE_Q6_K: c_int = 14;
pub const TMOE_TYPE_Q6_K_R8: c_int = 270;
pub const TMOE_COMM_ID_BYTES: c_int = 128;
pub const TMOE_GGUF_U64: c_int = 0;
pub const TMOE_GGUF_I64: c_int = 1;
pub const TMOE_GGUF_F64: c_int = 2;
pub const TMOE_GGUF_BOOL: c_int = 3;
pub const TMOE_GGUF_STR: c_int = 4;
pub const TMOE_GGUF_ARRAY: c_int = 5;
pub const TMOE_TRACE_STEP: c_int = 0;
pub const TMOE_TRACE_REFRESH: c_int = 1;
pub const TMOE_PHASE_RMS_NORM: c_int = 0;
pub const TMOE_PHASE_ROUTER_LOGITS: c_int = 1;
pub const TMOE_PHASE_TOPK: c_int = 2;
pub const TMOE_PHASE_MAP_IDS: c_int = 3;
pub const TMOE_PHASE_DISPATCH: c_int = 4;
pub const TMOE_PHASE_QUANT_X: c_int = 5;
pub const TMOE_PHASE_GATE_UP: c_int = 6;
pub const TMOE_PHASE_QUANT_ACT: c_int = 7;
pub const TMOE_PHASE_DOWN: c_int = 8;
pub const TMOE_PHASE_COMBINE: c_int = 9;
pub const TMOE_PHASE_SLOT_PLAN: c_int = 10;
pub const TMOE_PHASE_SLOT_PAGE: c_int = 11;
pub const TMOE_N_PHASES: c_int = 12;

/// The layer's shape, types and workspace size (`tmoe_config`).
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct tmoe_config {
    pub n_embd: i32,
    pub n_ff: i32,
    pub n_expert: i32,
    pub n_expert_used: i32,
    pub gate_type: i32,
    pub up_type: i32,
    pub down_type: i32,
    pub max_tokens: i32,
    pub device: i32,
    pub rms_eps: f32,
}

/// Stacked or slot expert tensors: device pointers into caller-owned ggml buffers.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct tmoe_expert_tensors {
    pub gate: *const c_void,
    pub up: *const c_void,
    pub down: *const c_void,
    pub gate_nb1: usize,
    pub gate_nb2: usize,
    pub up_nb1: usize,
    pub up_nb2: usize,
    pub down_nb1: usize,
    pub down_nb2: usize,
    pub n_slots: i32,
}

/// The numeric fields of a routing trace header.
#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct tmoe_trace_info {
    pub version: u32,
    pub n_layer: u32,
    pub n_expert: u32,
    pub n_used: u32,
    pub id_bytes: u32,
    pub vram_slots: u32,
    pub ram_slots: u32,
    pub prefetch_depth: u32,
    pub ubatch: u32,
    pub has_profile: i32,
}

macro_rules! opaque {
    ($($name:ident),*) => {$(
        #[repr(C)]
        pub struct $name {
            _private: [u8; 0],
        }
    )*};
}
opaque!(tmoe_handle, tmoe_comm, tmoe_slots, tmoe_gguf, tmoe_trace, tmoe_trace_writer);

#[link(name = "tmoe")]
extern "C" {
    pub fn tmoe_version() -> c_int;
    pub fn tmoe_create(cfg: *const tmoe_config, out: *mut *mut tmoe_handle) -> c_int;
    pub fn tmoe_destroy(h: *mut tmoe_handle);
    pub fn tmoe_last_error(h: *const tmoe_handle) -> *const c_char;
    pub fn tmoe_check(h: *mut tmoe_handle, stream: *mut c_void) -> c_int;
    pub fn tmoe_wait_flag(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        flag: *const i32,
        value: i32,
        limit_ns: i64,
    ) -> c_int;
    pub fn tmoe_mul_mat_id(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        ty: i32,
        W: *const c_void,
        nb1: usize,
        nb2: usize,
        K: i64,
        N: i64,
        n_w: i64,
        b: *const f32,
        b1: i64,
        ids: *const i32,
        n_used: i64,
        T: i64,
        out: *mut f32,
    ) -> c_int;
    pub fn tmoe_mul_mat_id_noalloc(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        ty: i32,
        W: *const c_void,
        nb1: usize,
        nb2: usize,
        K: i64,
        N: i64,
        n_w: i64,
        b: *const f32,
        b1: i64,
        ids: *const i32,
        n_used: i64,
        T: i64,
        out: *mut f32,
    ) -> c_int;
    pub fn tmoe_route(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        x: *const f32,
        T: i64,
        use_norm: i32,
        norm_w: *const f32,
        router_w: *const f32,
        logits: *const f32,
        ids_out: *mut i32,
        w_out: *mut f32,
        xn_out: *mut f32,
        logits_out: *mut f32,
    ) -> c_int;
    pub fn tmoe_experts(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        xn: *const f32,
        T: i64,
        ids: *const i32,
        w: *const f32,
        wts: *const tmoe_expert_tensors,
        out: *mut f32,
    ) -> c_int;
    pub fn tmoe_layer(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        x: *const f32,
        T: i64,
        use_norm: i32,
        norm_w: *const f32,
        router_w: *const f32,
        logits: *const f32,
        id_map: *const i32,
        wts: *const tmoe_expert_tensors,
        out: *mut f32,
        ids_out: *mut i32,
        w_out: *mut f32,
    ) -> c_int;
    pub fn tmoe_layer_bf16(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        x: *const uint16_t,
        T: i64,
        use_norm: i32,
        norm_w: *const f32,
        router_w: *const f32,
        logits: *const f32,
        id_map: *const i32,
        wts: *const tmoe_expert_tensors,
        out: *mut f32,
        ids_out: *mut i32,
        w_out: *mut f32,
    ) -> c_int;
    pub fn tmoe_comm_unique_id(id_out: *mut c_void) -> c_int;
    pub fn tmoe_comm_init(
        id: *const c_void,
        nranks: i32,
        rank: i32,
        device: i32,
        timeout_s: f64,
        out: *mut *mut tmoe_comm,
    ) -> c_int;
    pub fn tmoe_comm_abort(c: *mut tmoe_comm) -> c_int;
    pub fn tmoe_comm_destroy(c: *mut tmoe_comm);
    pub fn tmoe_comm_last_error() -> *const c_char;
    pub fn tmoe_ep_layer(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        comm: *mut tmoe_comm,
        x: *const f32,
        T: i64,
        use_norm: i32,
        norm_w: *const f32,
        router_w: *const f32,
        logits: *const f32,
        id_map: *const i32,
        wts: *const tmoe_expert_tensors,
        out: *mut f32,
        ids_out: *mut i32,
        w_out: *mut f32,
    ) -> c_int;
    pub fn tmoe_slots_create(
        h: *mut tmoe_handle,
        slots: *const tmoe_expert_tensors,
        store: *const tmoe_expert_tensors,
        out: *mut *mut tmoe_slots,
    ) -> c_int;
    pub fn tmoe_slots_destroy(s: *mut tmoe_slots);
    pub fn tmoe_slots_max_chunks(s: *const tmoe_slots) -> c_int;
    pub fn tmoe_slots_make_resident(
        s: *mut tmoe_slots,
        stream: *mut c_void,
        experts: *const i32,
        n: i32,
    ) -> c_int;
    pub fn tmoe_slots_set_hot_set(s: *mut tmoe_slots, stream: *mut c_void, hot: *const i32, n: i32) -> c_int;
    pub fn tmoe_slots_state(
        s: *mut tmoe_slots,
        stream: *mut c_void,
        owner: *mut i32,
        stats: *mut i64,
        counts: *mut i64,
    ) -> c_int;
    pub fn tmoe_slots_last_plan(
        s: *mut tmoe_slots,
        stream: *mut c_void,
        n_chunks: *mut i32,
        map: *mut i32,
        loads: *mut i32,
        n_loads: *mut i32,
    ) -> c_int;
    pub fn tmoe_streamed_layer(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        s: *mut tmoe_slots,
        x: *const f32,
        T: i64,
        use_norm: i32,
        norm_w: *const f32,
        router_w: *const f32,
        logits: *const f32,
        out: *mut f32,
        ids_out: *mut i32,
        w_out: *mut f32,
    ) -> c_int;
    pub fn tmoe_ep_a2a_layer(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        comm: *mut tmoe_comm,
        x: *const f32,
        T: i64,
        use_norm: i32,
        norm_w: *const f32,
        router_w: *const f32,
        logits: *const f32,
        wts: *const tmoe_expert_tensors,
        out: *mut f32,
        ids_out: *mut i32,
        w_out: *mut f32,
    ) -> c_int;
    pub fn tmoe_map_ids(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        ids: *const i32,
        n: i64,
        table: *const i32,
        n_table: i64,
        out: *mut i32,
    ) -> c_int;
    pub fn tmoe_dispatch(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        ids: *const i32,
        T: i64,
        n_slots: i32,
        counts: *mut i32,
        offsets: *mut i32,
        perm: *mut i32,
    ) -> c_int;
    pub fn tmoe_quantize(
        ty: i32,
        x: *const f32,
        nrows: i64,
        ncols: i64,
        out: *mut c_void,
        stream: *mut c_void,
    ) -> c_int;
    pub fn tmoe_dequantize(ty: i32, r#in: *const c_void, n: i64, out: *mut f32, stream: *mut c_void) -> c_int;
    pub fn tmoe_prepack(
        ty: i32,
        src: *const c_void,
        nb1: usize,
        nb2: usize,
        n_rows: i64,
        K: i64,
        n_mats: i64,
        dst: *mut c_void,
        stream: *mut c_void,
    ) -> c_int;
    pub fn tmoe_mul_mat(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        ty: i32,
        W: *const c_void,
        nb1: usize,
        K: i64,
        N: i64,
        x: *const f32,
        T: i64,
        reuse_x: i32,
        out: *mut f32,
    ) -> c_int;
    pub fn tmoe_get_rows(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        ty: i32,
        W: *const c_void,
        nb1: usize,
        K: i64,
        n_rows_w: i64,
        rows: *const i32,
        n: i64,
        out: *mut f32,
    ) -> c_int;
    pub fn tmoe_rms_norm(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        x: *const f32,
        w: *const f32,
        eps: f32,
        rows: i64,
        n: i64,
        out: *mut f32,
    ) -> c_int;
    pub fn tmoe_rope_neox(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        x: *mut f32,
        pos: *const i32,
        n_tok: i64,
        n_head: i32,
        head_dim: i32,
        n_rot: i32,
        freq_base: f32,
    ) -> c_int;
    pub fn tmoe_qk_norm_rope(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        q: *mut f32,
        k: *mut f32,
        q_norm: *const f32,
        k_norm: *const f32,
        pos: *const i32,
        T: i64,
        n_head: i32,
        n_kv: i32,
        head_dim: i32,
        n_rot: i32,
        freq_base: f32,
        eps: f32,
    ) -> c_int;
    pub fn tmoe_attn_decode_scratch_bytes(
        h: *mut tmoe_handle,
        B: i32,
        n_head: i32,
        n_kv: i32,
        head_dim: i32,
        n_ctx: i32,
    ) -> i64;
    pub fn tmoe_attn_decode(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        q: *const f32,
        k: *const f32,
        v: *const f32,
        k_cache: *mut c_void,
        v_cache: *mut c_void,
        pos: *const i32,
        B: i32,
        n_head: i32,
        n_kv: i32,
        head_dim: i32,
        n_ctx: i32,
        scale: f32,
        scratch: *mut c_void,
        out: *mut f32,
    ) -> c_int;
    pub fn tmoe_attn_prefill(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        q: *const f32,
        k: *const f32,
        v: *const f32,
        k_cache: *mut c_void,
        v_cache: *mut c_void,
        seq: i32,
        n_seq: i32,
        pos0: i32,
        S: i32,
        n_head: i32,
        n_kv: i32,
        head_dim: i32,
        n_ctx: i32,
        scale: f32,
        out: *mut f32,
    ) -> c_int;
    pub fn tmoe_add(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        a: *const f32,
        b: *const f32,
        out: *mut f32,
        n: i64,
    ) -> c_int;
    pub fn tmoe_argmax(
        h: *mut tmoe_handle,
        stream: *mut c_void,
        x: *const f32,
        rows: i64,
        n: i64,
        out: *mut i32,
    ) -> c_int;
    pub fn tmoe_gguf_open(path: *const c_char, out: *mut *mut tmoe_gguf) -> c_int;
    pub fn tmoe_gguf_close(g: *mut tmoe_gguf);
    pub fn tmoe_gguf_last_error() -> *const c_char;
    pub fn tmoe_gguf_n_shards(g: *const tmoe_gguf) -> i32;
    pub fn tmoe_gguf_n_kv(g: *const tmoe_gguf) -> i64;
    pub fn tmoe_gguf_kv_key(g: *const tmoe_gguf, i: i64, key: *mut *const c_char) -> c_int;
    pub fn tmoe_gguf_kv(
        g: *const tmoe_gguf,
        key: *const c_char,
        kind: *mut i32,
        u: *mut u64,
        i: *mut i64,
        f: *mut f64,
        s: *mut *const c_char,
        n: *mut u64,
    ) -> c_int;
    pub fn tmoe_gguf_n_tensors(g: *const tmoe_gguf) -> i64;
    pub fn tmoe_gguf_find_tensor(g: *const tmoe_gguf, name: *const c_char) -> i64;
    pub fn tmoe_gguf_tensor_info(
        g: *const tmoe_gguf,
        i: i64,
        name: *mut *const c_char,
        ty: *mut i32,
        ne: *mut i64,
        shard: *mut i32,
        offset: *mut u64,
        nbytes: *mut u64,
    ) -> c_int;
    pub fn tmoe_gguf_type_size(ty: i32, block_elems: *mut i32, block_bytes: *mut i32) -> c_int;
    pub fn tmoe_gguf_read(
        g: *const tmoe_gguf,
        tensor: i64,
        offset: u64,
        nbytes: u64,
        dst: *mut c_void,
    ) -> c_int;
    pub fn tmoe_gguf_load(
        g: *const tmoe_gguf,
        tensor: i64,
        offset: u64,
        nbytes: u64,
        dst: *mut c_void,
        device: i32,
        stream: *mut c_void,
    ) -> c_int;
    pub fn tmoe_trace_open(path: *const c_char, out: *mut *mut tmoe_trace) -> c_int;
    pub fn tmoe_trace_close(t: *mut tmoe_trace);
    pub fn tmoe_trace_last_error() -> *const c_char;
    pub fn tmoe_trace_header(t: *const tmoe_trace, info: *mut tmoe_trace_info) -> c_int;
    pub fn tmoe_trace_header_json(t: *const tmoe_trace) -> *const c_char;
    pub fn tmoe_trace_header_str(t: *const tmoe_trace, field: *const c_char) -> *const c_char;
    pub fn tmoe_trace_expert_bytes(t: *const tmoe_trace, out: *mut u64) -> c_int;
    pub fn tmoe_trace_profile(t: *const tmoe_trace, rows: *mut i64, cols: *mut i64, out: *mut u64) -> c_int;
    pub fn tmoe_trace_next(
        t: *mut tmoe_trace,
        kind: *mut i32,
        step: *mut u32,
        layer: *mut i32,
        n_tokens: *mut u32,
        flags: *mut i32,
    ) -> c_int;
    pub fn tmoe_trace_ids(t: *const tmoe_trace, which: i32, out: *mut i32) -> c_int;
    pub fn tmoe_trace_create(
        path: *const c_char,
        header_json: *const c_char,
        out: *mut *mut tmoe_trace_writer,
    ) -> c_int;
    pub fn tmoe_trace_write_step(
        w: *mut tmoe_trace_writer,
        step: u32,
        layer: i32,
        n_tokens: u32,
        ids: *const i32,
        predicted: *const i32,
        predicted2: *const i32,
    ) -> c_int;
    pub fn tmoe_trace_write_refresh(w: *mut tmoe_trace_writer, step: u32) -> c_int;
    pub fn tmoe_trace_finish(w: *mut tmoe_trace_writer) -> c_int;
    pub fn tmoe_profile_enable(h: *mut tmoe_handle, enable: i32) -> c_int;
    pub fn tmoe_profile_collect(h: *mut tmoe_handle, ms_out: *mut f64, count_out: *mut i64) -> c_int;
}
