//! Raw bindings of `include/w4a8.h`, the C ABI of libwebyiq_w4a8.so.
//!
//! One `extern "C"` declaration per entry point of the header, same names, same
//! argument order and C types (`int32_t` -> i32, `size_t` -> usize, `void*` streams
//! and opaque handles -> *mut c_void).  The test `tests/test_rust_ffi.py` parses this
//! file and the header and checks that the two agree.
//!
//! Every call returns a `w4a8_status` (0 = OK); on error the message of the calling
//! thread is `w4a8_last_error()`.  `check` turns that pair into the reference
//! engine's `Result<(), String>` (crates/engine/src/graph.rs:368-380 style).

#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_int, c_void, CStr};

/// `w4a8_weight` (include/w4a8.h): a view of one converted tensor already in device
/// memory, `{w}.q` = u32[n, k/8] packed nibbles, `{w}.s` = per-group scales.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct w4a8_weight {
    pub q: *const c_void,
    pub s: *const c_void,
    pub n: i32,
    pub k: i32,
    pub group: i32,
    pub has_min: i32,
}

/// Opaque peer-memory exchange object of the column-split lm_head.
#[repr(C)]
pub struct w4a8_xchg {
    _private: [u8; 0],
}

pub type w4a8_status = c_int;

pub const W4A8_OK: w4a8_status = 0;
pub const W4A8_EINVAL: w4a8_status = 1;
pub const W4A8_ECUDA: w4a8_status = 2;
pub const W4A8_ENCCL: w4a8_status = 3;
pub const W4A8_ETIMEOUT: w4a8_status = 4;
pub const W4A8_ENOTSUP: w4a8_status = 5;

pub const W4A8_ACT_GROUP32: i32 = 0;
pub const W4A8_ACT_TOKEN: i32 = 1;

pub const W4A8_STORE: i32 = 0;
pub const W4A8_ADD: i32 = 1;
pub const W4A8_SWIGLU: i32 = 2;

pub const W4A8_GEMV_MAX_M: i32 = 16;
pub const W4A8_XCHG_HANDLE_BYTES: usize = 64;
pub const W4A8_XCHG_MAX_RANKS: i32 = 8;
pub const W4A8_XCHG_MAX_TOKENS: i32 = 16;

extern "C" {
    pub fn w4a8_weight_view(q: *const c_void, s: *const c_void, n: i32, k: i32, group: i32, has_min: i32,
                            out: *mut w4a8_weight) -> w4a8_status;
    pub fn w4a8_quant(x: *const f32, norm_w: *const f32, eps: f32, m: i32, k: i32, act: i32, xq: *mut i8,
                      xs: *mut f32, stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_gemv(w: *const w4a8_weight, xq: *const i8, xs: *const f32, act: i32, m: i32, mode: i32,
                     y: *mut f32, stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_gemv_x(w: *const w4a8_weight, x: *const f32, m: i32, mode: i32, y: *mut f32,
                       stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_gemv_xn(w: *const w4a8_weight, x: *const f32, norm_w: *const f32, eps: f32, m: i32, mode: i32,
                        y: *mut f32, stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_gemm(w: *const w4a8_weight, xq: *const i8, xs: *const f32, act: i32, m: i32, mode: i32,
                     y: *mut f32, stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_matmul(w: *const w4a8_weight, xq: *const i8, xs: *const f32, act: i32, m: i32, mode: i32,
                       y: *mut f32, stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_argmax(logits: *const f32, m: i32, v: i32, ids: *const u32, tok_out: *mut u32,
                       stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_lmhead_argmax(w: *const w4a8_weight, row_offset: i32, xq: *const i8, xs: *const f32, act: i32,
                              m: i32, logits: *mut f32, best_key: *mut u64, tok_out: *mut u32, ids: *const u32,
                              workspace: *mut c_void, workspace_bytes: usize, stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_lmhead_workspace_bytes(n: i32, m: i32) -> usize;
    pub fn w4a8_lmhead_argmax_noalloc(w: *const w4a8_weight, row_offset: i32, xq: *const i8, xs: *const f32,
                                      act: i32, m: i32, logits: *mut f32, best_key: *mut u64, tok_out: *mut u32,
                                      ids: *const u32, stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_lmhead_argmax_allreduce(w: *const w4a8_weight, row_offset: i32, xq: *const i8, xs: *const f32,
                                        act: i32, m: i32, logits: *mut f32, best_key: *mut u64,
                                        tok_out: *mut u32, ids: *const u32, workspace: *mut c_void,
                                        workspace_bytes: usize, nccl_comm: *mut c_void,
                                        stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_nccl_get_unique_id(id_out: *mut c_void) -> w4a8_status;
    pub fn w4a8_nccl_comm_init(nranks: i32, id: *const c_void, rank: i32, comm_out: *mut *mut c_void) -> w4a8_status;
    pub fn w4a8_nccl_comm_destroy(comm: *mut c_void) -> w4a8_status;
    pub fn w4a8_xchg_create(world: i32, rank: i32, handle_out: *mut c_void, out: *mut *mut w4a8_xchg) -> w4a8_status;
    pub fn w4a8_xchg_open(x: *mut w4a8_xchg, handles: *const c_void) -> w4a8_status;
    pub fn w4a8_xchg_destroy(x: *mut w4a8_xchg) -> w4a8_status;
    pub fn w4a8_lmhead_argmax_xchg(w: *const w4a8_weight, row_offset: i32, xq: *const i8, xs: *const f32,
                                   act: i32, m: i32, logits: *mut f32, best_key: *mut u64, tok_out: *mut u32,
                                   ids: *const u32, workspace: *mut c_void, workspace_bytes: usize,
                                   x: *mut w4a8_xchg, stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_gather_rows(src: *const w4a8_weight, ids: *const u32, rows: i32, dst_q: *mut c_void,
                            dst_s: *mut c_void, stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_spec_accept(tok: *mut u32, y: *const u32, e: *const u32, params: *const u32, ctl: *mut u32,
                            out: *mut u32, stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_attn_decode(qkv: *const f32, kc: *const c_void, vc: *const c_void, h: i32, kvh: i32, d: i32,
                            maxctx: i32, params: *const u32, m: i32, chunks: i32, part: *mut f32,
                            stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_attn_combine(part: *const f32, h: i32, kvh: i32, d: i32, maxctx: i32, params: *const u32, m: i32,
                             gsrc: *const f32, xq: *mut i8, xs: *mut f32, o_out: *mut f32,
                             stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_deltanet(proj: *const f32, conv_w: *const f32, conv_state: *mut f32, state: *mut f32, out: *mut f32,
                         neg_a: *const f32, dt_bias: *const f32, gate_norm: *const f32, params: *const u32, nh: i32,
                         m: i32, eps: f32, spec: i32, stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_group_dots(w: *const w4a8_weight, xq: *const i8, m: i32, dots: *mut i32,
                           stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_gemm_group_dots(w: *const w4a8_weight, xq: *const i8, m: i32, dots: *mut i32,
                                stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_set_pdl(enable: c_int);
    pub fn w4a8_set_gemv_kernel(tensor_core: c_int);
    pub fn w4a8_set_gemm_kernel(tensor_core: c_int);
    pub fn w4a8_device_error(code: *mut u32, stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_selftest_wait_timeout(stream: *mut c_void) -> w4a8_status;
    pub fn w4a8_last_error() -> *const c_char;
    pub fn w4a8_version() -> *const c_char;
}

/// The index carried by a packed argmax key (`w4a8_key_index`, a static inline in
/// the header): the low word holds the complement of the index, 0 for the empty key.
pub fn w4a8_key_index(key: u64) -> u32 {
    if key == 0 { 0 } else { !(key as u32) }
}

/// `Result<(), String>` of a call: the thread's `w4a8_last_error()` on failure.
pub fn check(st: w4a8_status) -> Result<(), String> {
    if st == W4A8_OK {
        Ok(())
    } else {
        let msg = unsafe { CStr::from_ptr(w4a8_last_error()) }.to_string_lossy().into_owned();
        Err(format!("w4a8 status {st}: {msg}"))
    }
}
