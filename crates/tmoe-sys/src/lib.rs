//! Bindings to libtmoe, the B200-native MoE layer of Tetraeder's own Qwen3-MoE builder.
//!
//! `raw` declares the C ABI of `include/tmoe.h`; the types below wrap it the way `ggml-sys` wraps
//! ggml: `Result` instead of status codes, device pointers borrowed from ggml tensors (the library
//! never owns or copies weights), and `unsafe` kept to this crate.  A `Moe` belongs to one host
//! thread, like the builder that owns it (it is not `Send`).
//!
//! Where each call lands in the builder (paths from the tetraeder root):
//!   `Moe::layer`          moe_ffn()                  crates/model/src/qwen3moe.rs:2892-2896
//!   `Moe::route`          router()                   crates/model/src/qwen3moe.rs:2871-2890
//!   `Moe::experts`        weighted_experts() + sum_experts()  qwen3moe.rs:2899-2923
//!   `Moe::mul_mat_id`     Context::mul_mat_id        crates/ggml-sys/src/ggml/context.rs:322-336
//!   `Moe::ep_layer`       Sharded::build's MoE part and its all-reduce  qwen3moe_shard.rs:1038-1056
//!   `Slots`, `Moe::streamed_layer`  LayerSlots and the streamed step  crates/memory/src/slots.rs:67-262,
//!                         qwen3moe.rs:1829,2021-2050
//!   `GgufFile`            Gguf::open / tensor reads of load_weights  crates/model/src/gguf.rs:236-457

pub mod raw;

use std::ffi::{c_void, CStr, CString};
use std::marker::PhantomData;
use std::ptr;

pub use raw::{tmoe_config, tmoe_expert_tensors, TMOE_TYPE_Q4_K, TMOE_TYPE_Q6_K, TMOE_TYPE_Q6_K_R8};

/// A failed call: the negative `TMOE_E_*` code and the library's message.
#[derive(Debug, thiserror::Error)]
#[error("tmoe error {code}: {msg}")]
pub struct TmoeError {
    pub code: i32,
    pub msg: String,
}

/// A CUDA stream (`cudaStream_t`); null is the legacy default stream.
pub type Stream = *mut c_void;

fn message(p: *const std::ffi::c_char) -> String {
    if p.is_null() {
        return String::new();
    }
    unsafe { CStr::from_ptr(p) }.to_string_lossy().into_owned()
}

fn check(h: *const raw::tmoe_handle, rc: i32) -> Result<(), TmoeError> {
    if rc == raw::TMOE_OK {
        return Ok(());
    }
    Err(TmoeError { code: rc, msg: message(unsafe { raw::tmoe_last_error(h) }) })
}

/// The optional, explicit repack of Q6_K expert matrices into `TMOE_TYPE_Q6_K_R8` (the upload
/// path calls it once per tensor when it opts in; nothing repacks implicitly, as in ADR 0039).
/// `n_mats` matrices of `n_rows` x `k`, rows `nb1` and matrices `nb2` bytes apart, into `dst`.
///
/// # Safety
/// `src` and `dst` are device pointers of the sizes the header states, not overlapping, valid until
/// the stream has passed the call.
#[allow(clippy::too_many_arguments)]
pub unsafe fn prepack_q6k(src: *const u8, nb1: usize, nb2: usize, n_rows: i64, k: i64, n_mats: i64, dst: *mut u8,
                          stream: Stream) -> Result<(), TmoeError> {
    check(ptr::null(), raw::tmoe_prepack(raw::TMOE_TYPE_Q6_K, src.cast(), nb1, nb2, n_rows, k, n_mats, dst.cast(),
                                         stream))
}

/// One handle: the layer's shape and types and a workspace for `max_tokens`, on one device.
pub struct Moe {
    h: *mut raw::tmoe_handle,
    _not_send: PhantomData<*mut ()>,
}

impl Moe {
    pub fn new(cfg: &tmoe_config) -> Result<Self, TmoeError> {
        let mut h = ptr::null_mut();
        check(ptr::null(), unsafe { raw::tmoe_create(cfg, &mut h) })?;
        Ok(Moe { h, _not_send: PhantomData })
    }

    /// moe_ffn: route + experts + the weighted sum on `stream`.  `x`, `norm_w`, `router_w` and `out`
    /// are device pointers of ggml tensors; `wts` points at the stacked `ffn_{gate,up,down}_exps`
    /// slabs or slot tensors; `id_map` (nullable) maps global expert ids to slots or -1.
    ///
    /// # Safety
    /// Every pointer is a device pointer of the shape the header states, valid until the stream
    /// has passed the call.
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn layer(
        &mut self,
        stream: Stream,
        x: *const f32,
        t: i64,
        norm_w: *const f32,
        router_w: *const f32,
        id_map: *const i32,
        wts: &tmoe_expert_tensors,
        out: *mut f32,
        ids_out: *mut i32,
        w_out: *mut f32,
    ) -> Result<(), TmoeError> {
        let use_norm = i32::from(!norm_w.is_null());
        check(
            self.h,
            raw::tmoe_layer(self.h, stream, x, t, use_norm, norm_w, router_w, ptr::null(), id_map, wts, out, ids_out, w_out),
        )
    }

    /// router(): ids and weights of the top-k experts of each token (ties to the lower index).
    ///
    /// # Safety
    /// As for [`Moe::layer`].
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn route(
        &mut self,
        stream: Stream,
        x: *const f32,
        t: i64,
        norm_w: *const f32,
        router_w: *const f32,
        ids_out: *mut i32,
        w_out: *mut f32,
        xn_out: *mut f32,
    ) -> Result<(), TmoeError> {
        let use_norm = i32::from(!norm_w.is_null());
        check(
            self.h,
            raw::tmoe_route(self.h, stream, x, t, use_norm, norm_w, router_w, ptr::null(), ids_out, w_out, xn_out, ptr::null_mut()),
        )
    }

    /// weighted_experts() + sum_experts() over given ids (< 0: no contribution) and weights.
    ///
    /// # Safety
    /// As for [`Moe::layer`].
    pub unsafe fn experts(
        &mut self,
        stream: Stream,
        xn: *const f32,
        t: i64,
        ids: *const i32,
        w: *const f32,
        wts: &tmoe_expert_tensors,
        out: *mut f32,
    ) -> Result<(), TmoeError> {
        check(self.h, raw::tmoe_experts(self.h, stream, xn, t, ids, w, wts, out))
    }

    /// Context::mul_mat_id for a Q4_K/Q6_K expert tensor `[k, n, n_w]`.
    ///
    /// # Safety
    /// As for [`Moe::layer`].
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn mul_mat_id(
        &mut self,
        stream: Stream,
        ty: i32,
        w: *const u8,
        nb1: usize,
        nb2: usize,
        k: i64,
        n: i64,
        n_w: i64,
        b: *const f32,
        b1: i64,
        ids: *const i32,
        n_used: i64,
        t: i64,
        out: *mut f32,
    ) -> Result<(), TmoeError> {
        check(
            self.h,
            raw::tmoe_mul_mat_id(self.h, stream, ty, w.cast(), nb1, nb2, k, n, n_w, b, b1, ids, n_used, t, out),
        )
    }

    /// The reference's EP layer on this rank: `layer` over the experts this rank holds, summed over
    /// the ranks of `comm`.  Every rank makes the same calls in the same order.
    ///
    /// # Safety
    /// As for [`Moe::layer`].
    #[allow(clippy::too_many_arguments)]
    pub unsafe fn ep_layer(
        &mut self,
        stream: Stream,
        comm: &mut Comm,
        x: *const f32,
        t: i64,
        norm_w: *const f32,
        router_w: *const f32,
        id_map: *const i32,
        wts: &tmoe_expert_tensors,
        out: *mut f32,
    ) -> Result<(), TmoeError> {
        let use_norm = i32::from(!norm_w.is_null());
        check(
            self.h,
            raw::tmoe_ep_layer(
                self.h,
                stream,
                comm.c,
                x,
                t,
                use_norm,
                norm_w,
                router_w,
                ptr::null(),
                id_map,
                wts,
                out,
                ptr::null_mut(),
                ptr::null_mut(),
            ),
        )
    }

    /// The streamed step without the ids readback: plan, paging and chunks on the device.
    ///
    /// # Safety
    /// As for [`Moe::layer`].
    pub unsafe fn streamed_layer(
        &mut self,
        stream: Stream,
        slots: &mut Slots,
        x: *const f32,
        t: i64,
        router_w: *const f32,
        out: *mut f32,
    ) -> Result<(), TmoeError> {
        check(
            self.h,
            raw::tmoe_streamed_layer(
                self.h,
                stream,
                slots.s,
                x,
                t,
                0,
                ptr::null(),
                router_w,
                ptr::null(),
                out,
                ptr::null_mut(),
                ptr::null_mut(),
            ),
        )
    }

    /// Synchronises `stream`, then reads and clears the device error flag (a bounded wait that
    /// gave up, an expert id out of range, a miss with every slot pinned).
    pub fn check_device(&mut self, stream: Stream) -> Result<(), TmoeError> {
        check(self.h, unsafe { raw::tmoe_check(self.h, stream) })
    }
}

impl Drop for Moe {
    fn drop(&mut self) {
        unsafe { raw::tmoe_destroy(self.h) }
    }
}

/// The expert-slot cache of one layer (LayerSlots with its table on the device) over the layer's
/// slot tensors and its pinned host store.
pub struct Slots {
    s: *mut raw::tmoe_slots,
}

impl Slots {
    /// # Safety
    /// `slots` are device tensors and `store` pinned host tensors that outlive the cache.
    pub unsafe fn new(m: &Moe, slots: &tmoe_expert_tensors, store: &tmoe_expert_tensors) -> Result<Self, TmoeError> {
        let mut s = ptr::null_mut();
        check(m.h, raw::tmoe_slots_create(m.h, slots, store, &mut s))?;
        Ok(Slots { s })
    }
}

impl Drop for Slots {
    fn drop(&mut self) {
        unsafe { raw::tmoe_slots_destroy(self.s) }
    }
}

/// A rank's communicator of an expert-parallel group (NCCL, one rank per GPU).
pub struct Comm {
    c: *mut raw::tmoe_comm,
}

fn comm_check(rc: i32) -> Result<(), TmoeError> {
    if rc == raw::TMOE_OK {
        return Ok(());
    }
    Err(TmoeError { code: rc, msg: message(unsafe { raw::tmoe_comm_last_error() }) })
}

impl Comm {
    /// Rank 0 makes the id and hands its bytes to every rank.
    pub fn unique_id() -> Result<[u8; raw::TMOE_COMM_ID_BYTES as usize], TmoeError> {
        let mut id = [0u8; raw::TMOE_COMM_ID_BYTES as usize];
        comm_check(unsafe { raw::tmoe_comm_unique_id(id.as_mut_ptr().cast()) })?;
        Ok(id)
    }

    /// Joins the group; gives up with TMOE_E_COMM when the ranks have not all joined within
    /// `timeout_s` seconds.
    pub fn init(id: &[u8; raw::TMOE_COMM_ID_BYTES as usize], nranks: i32, rank: i32, device: i32,
                timeout_s: f64) -> Result<Self, TmoeError> {
        let mut c = ptr::null_mut();
        comm_check(unsafe { raw::tmoe_comm_init(id.as_ptr().cast(), nranks, rank, device, timeout_s, &mut c) })?;
        Ok(Comm { c })
    }

    /// Ends the communicator at once (a watchdog's call when a peer died).
    pub fn abort(&mut self) -> Result<(), TmoeError> {
        comm_check(unsafe { raw::tmoe_comm_abort(self.c) })
    }
}

impl Drop for Comm {
    fn drop(&mut self) {
        unsafe { raw::tmoe_comm_destroy(self.c) }
    }
}

/// An open GGUF model (every shard of a split model); replaces `Gguf::open` for the MoE tensors.
pub struct GgufFile {
    g: *mut raw::tmoe_gguf,
}

fn gguf_check(rc: i32) -> Result<(), TmoeError> {
    if rc == raw::TMOE_OK {
        return Ok(());
    }
    Err(TmoeError { code: rc, msg: message(unsafe { raw::tmoe_gguf_last_error() }) })
}

impl GgufFile {
    pub fn open(path: &std::path::Path) -> Result<Self, TmoeError> {
        let c = CString::new(path.as_os_str().as_encoded_bytes()).map_err(|_| TmoeError {
            code: raw::TMOE_E_INVALID,
            msg: "path contains a NUL byte".into(),
        })?;
        let mut g = ptr::null_mut();
        gguf_check(unsafe { raw::tmoe_gguf_open(c.as_ptr(), &mut g) })?;
        Ok(GgufFile { g })
    }

    /// (index, bytes) of a tensor by name (`Gguf::tensor`).
    pub fn tensor(&self, name: &str) -> Result<(i64, u64), TmoeError> {
        let c = CString::new(name).map_err(|_| TmoeError { code: raw::TMOE_E_INVALID, msg: "NUL in name".into() })?;
        let i = unsafe { raw::tmoe_gguf_find_tensor(self.g, c.as_ptr()) };
        if i < 0 {
            return Err(TmoeError { code: raw::TMOE_E_NOTFOUND, msg: format!("missing tensor `{name}`") });
        }
        let mut nbytes = 0u64;
        gguf_check(unsafe {
            raw::tmoe_gguf_tensor_info(
                self.g,
                i,
                ptr::null_mut(),
                ptr::null_mut(),
                ptr::null_mut(),
                ptr::null_mut(),
                ptr::null_mut(),
                &mut nbytes,
            )
        })?;
        Ok((i, nbytes))
    }

    /// Bytes `[off, off + len)` of tensor `i` into device memory (`dst`: a ggml tensor's data).
    ///
    /// # Safety
    /// `dst` is a device allocation of at least `len` bytes on `device`.
    pub unsafe fn load(&self, i: i64, off: u64, len: u64, dst: *mut c_void, device: i32, stream: Stream)
                       -> Result<(), TmoeError> {
        gguf_check(raw::tmoe_gguf_load(self.g, i, off, len, dst, device, stream))
    }
}

impl Drop for GgufFile {
    fn drop(&mut self) {
        unsafe { raw::tmoe_gguf_close(self.g) }
    }
}
