//! CUDA backend of `webyiq-engine` for B200 (sm_100a): the W4A8 matmul path of the
//! decode / verify / prefill graphs runs through libwebyiq_w4a8.so instead of the
//! WGSL pipelines (`gemv_q4q8.wgsl`, `gemm_q4q8.wgsl`, `quant.wgsl`, `argmax.wgsl`).
//!
//! It sits beside the wgpu backend and mirrors its pieces:
//!   - `CudaEngine::new` / `upload_shard` own one device buffer per manifest tensor,
//!     like `Engine::new` and `Engine::upload_shard` (crates/engine/src/lib.rs:41-48,
//!     177-187), with the same byte ranges of the same shard files;
//!   - `CudaBuilder::{gemv, gemm, matmul, quant, argmax, lm_head}` record one op each,
//!     like `Builder::{gemv, gemm, matmul, quant}` and the argmax of `head_ops`
//!     (crates/engine/src/graph.rs:190-222, 476-486), with the same shape checks and
//!     the same "missing tensor" errors;
//!   - `CudaPlan` issues the recorded ops of one step in order on one stream, and
//!     may capture them once into a CUDA graph that is replayed per token.
//! There is no CPU fallback: if the library or the GPU is missing, `CudaEngine::new`
//! fails.
//!
//! Not built in this repository (the image that holds it has no cargo); `build.rs`
//! beside `src/` compiles the library with nvcc for sm_100a and links it.

pub mod ffi;

use std::collections::HashMap;
use std::ffi::c_void;

use crate::manifest::Manifest;
use ffi::{check, w4a8_weight};

/// The engine's group size (crates/engine/src/manifest.rs:82: quant.group == 32).
pub const GROUP: u32 = 32;

// ---- the few CUDA runtime calls the backend makes (libcudart) ----
#[allow(non_camel_case_types)]
type cudaError_t = i32;
#[link(name = "cudart")]
extern "C" {
    fn cudaSetDevice(dev: i32) -> cudaError_t;
    fn cudaMalloc(p: *mut *mut c_void, bytes: usize) -> cudaError_t;
    fn cudaFree(p: *mut c_void) -> cudaError_t;
    fn cudaMemcpy(dst: *mut c_void, src: *const c_void, bytes: usize, kind: i32) -> cudaError_t;
    fn cudaMemset(p: *mut c_void, v: i32, bytes: usize) -> cudaError_t;
    fn cudaStreamCreateWithFlags(s: *mut *mut c_void, flags: u32) -> cudaError_t;
    fn cudaStreamDestroy(s: *mut c_void) -> cudaError_t;
    fn cudaStreamSynchronize(s: *mut c_void) -> cudaError_t;
    fn cudaStreamBeginCapture(s: *mut c_void, mode: i32) -> cudaError_t;
    fn cudaStreamEndCapture(s: *mut c_void, g: *mut *mut c_void) -> cudaError_t;
    fn cudaGraphInstantiate(e: *mut *mut c_void, g: *mut c_void, flags: u64) -> cudaError_t;
    fn cudaGraphLaunch(e: *mut c_void, s: *mut c_void) -> cudaError_t;
    fn cudaGraphExecDestroy(e: *mut c_void) -> cudaError_t;
    fn cudaGraphDestroy(g: *mut c_void) -> cudaError_t;
    fn cudaGetErrorString(e: cudaError_t) -> *const std::ffi::c_char;
}
const H2D: i32 = 1;
const D2H: i32 = 2;
const NON_BLOCKING: u32 = 1;
const CAPTURE_THREAD_LOCAL: i32 = 1;

fn cuda(e: cudaError_t, what: &str) -> Result<(), String> {
    if e == 0 {
        Ok(())
    } else {
        let s = unsafe { std::ffi::CStr::from_ptr(cudaGetErrorString(e)) }.to_string_lossy().into_owned();
        Err(format!("{what}: {s}"))
    }
}

/// One device allocation (a manifest tensor or an activation buffer).
pub struct DevBuf {
    pub ptr: *mut c_void,
    pub bytes: usize,
}

impl DevBuf {
    pub fn new(bytes: usize) -> Result<Self, String> {
        let mut p = std::ptr::null_mut();
        cuda(unsafe { cudaMalloc(&mut p, bytes.max(1)) }, "cudaMalloc")?;
        cuda(unsafe { cudaMemset(p, 0, bytes.max(1)) }, "cudaMemset")?;
        Ok(DevBuf { ptr: p, bytes })
    }
    pub fn write(&self, data: &[u8]) -> Result<(), String> {
        if data.len() > self.bytes {
            return Err(format!("write of {} bytes into a {}-byte buffer", data.len(), self.bytes));
        }
        cuda(unsafe { cudaMemcpy(self.ptr, data.as_ptr() as *const c_void, data.len(), H2D) }, "upload")
    }
    pub fn read(&self, out: &mut [u8]) -> Result<(), String> {
        cuda(unsafe { cudaMemcpy(out.as_mut_ptr() as *mut c_void, self.ptr, out.len().min(self.bytes), D2H) }, "download")
    }
}

impl Drop for DevBuf {
    fn drop(&mut self) {
        unsafe { cudaFree(self.ptr) };
    }
}

/// The CUDA counterpart of `Engine`'s weight table: one device buffer per tensor.
pub struct CudaEngine {
    manifest: Manifest,
    weights: HashMap<String, DevBuf>,
    pub stream: *mut c_void,
}

impl CudaEngine {
    /// Allocates every tensor of the manifest on `device` (nothing uploaded yet).
    pub fn new(manifest: Manifest, device: i32) -> Result<Self, String> {
        cuda(unsafe { cudaSetDevice(device) }, "cudaSetDevice")?;
        let mut weights = HashMap::new();
        for (name, t) in &manifest.tensors {
            weights.insert(name.clone(), DevBuf::new(t.bytes as usize)?);
        }
        let mut stream = std::ptr::null_mut();
        cuda(unsafe { cudaStreamCreateWithFlags(&mut stream, NON_BLOCKING) }, "stream")?;
        Ok(CudaEngine { manifest, weights, stream })
    }

    pub fn manifest(&self) -> &Manifest {
        &self.manifest
    }

    /// Upload every tensor stored in shard `idx`; `data` is the whole shard file
    /// (the byte ranges of `Engine::upload_shard`, lib.rs:177-187).
    pub fn upload_shard(&self, idx: usize, data: &[u8]) -> Result<(), String> {
        for (name, t) in &self.manifest.tensors {
            if t.shard == idx {
                let (s, e) = (t.offset as usize, (t.offset + t.bytes) as usize);
                if e > data.len() {
                    return Err(format!("shard {idx} too short for {name}"));
                }
                self.weights[name].write(&data[s..e])?;
            }
        }
        Ok(())
    }

    fn w(&self, name: &str) -> Result<&DevBuf, String> {
        self.weights.get(name).ok_or_else(|| format!("missing tensor {name}"))
    }

    /// The `w4a8_weight` view of q4 tensor pair `{w}.q` / `{w}.s` with n rows of k.
    pub fn weight(&self, w: &str, k: u32, n: u32) -> Result<w4a8_weight, String> {
        let (wq, ws) = (self.w(&format!("{w}.q"))?, self.w(&format!("{w}.s"))?);
        if wq.bytes != (n as usize) * (k as usize) / 2 {
            return Err(format!("{w}.q: {} bytes, expected {}x{} nibbles", wq.bytes, n, k));
        }
        // u32 (scale | min << 16) per group in the engine's format, f16 scale for symmetric shards
        let groups = (n as usize) * (k as usize / GROUP as usize);
        let has_min = if ws.bytes == groups * 4 { 1 } else if ws.bytes == groups * 2 { 0 } else {
            return Err(format!("{w}.s: {} bytes for {} groups", ws.bytes, groups));
        };
        let mut out = std::mem::MaybeUninit::<w4a8_weight>::uninit();
        check(unsafe { ffi::w4a8_weight_view(wq.ptr, ws.ptr, n as i32, k as i32, GROUP as i32, has_min, out.as_mut_ptr()) })?;
        Ok(unsafe { out.assume_init() })
    }
}

impl Drop for CudaEngine {
    fn drop(&mut self) {
        unsafe { cudaStreamDestroy(self.stream) };
    }
}

/// Decode (1 token), speculative verify (2) or prefill (a chunk): the `Path` of graph.rs.
#[derive(Clone, Copy, PartialEq, Eq, Debug)]
pub enum Path {
    Decode,
    Spec,
    Prefill,
}

/// Activations of one path: f32 x, int8 xq and the per-32 scales xs (graph.rs `Acts`).
pub struct Acts {
    pub rows: u32,
    pub xq: DevBuf,
    pub xs: DevBuf,
}

impl Acts {
    pub fn new(rows: u32, k_max: u32) -> Result<Self, String> {
        let (r, k) = (rows as usize, k_max as usize);
        Ok(Acts { rows, xq: DevBuf::new(r * k)?, xs: DevBuf::new(r * (k / 32) * 8)? })
    }
}

/// One recorded op: its name and the launch it makes on a stream.
pub struct CudaOp {
    pub name: &'static str,
    run: Box<dyn Fn(*mut c_void) -> Result<(), String>>,
}

/// Records ops over a `CudaEngine`, like the wgpu `Builder`.
pub struct CudaBuilder<'a> {
    e: &'a CudaEngine,
    pub ops: Vec<CudaOp>,
}

impl<'a> CudaBuilder<'a> {
    pub fn new(e: &'a CudaEngine) -> Self {
        CudaBuilder { e, ops: Vec::new() }
    }

    fn push(&mut self, name: &'static str, run: impl Fn(*mut c_void) -> i32 + 'static) {
        self.ops.push(CudaOp { name, run: Box::new(move |s| check(run(s))) });
    }

    /// y (+)= W x for `t` tokens (Builder::gemv, graph.rs:190-198; N % 8 == 0 as graph.rs:374).
    #[allow(clippy::too_many_arguments)]
    pub fn gemv(&mut self, name: &'static str, w: &str, k: u32, n: u32, mode: u32, t: u32, a: &Acts, y: &DevBuf) -> Result<(), String> {
        if n % 8 != 0 {
            return Err(format!("{name}: N = {n} is not a multiple of 8"));
        }
        let wt = self.e.weight(w, k, if mode == 2 { 2 * n } else { n })?;
        let (xq, xs, yp) = (a.xq.ptr as usize, a.xs.ptr as usize, y.ptr as usize);
        self.push(name, move |s| unsafe {
            ffi::w4a8_gemv(&wt, xq as *const i8, xs as *const f32, ffi::W4A8_ACT_GROUP32, t as i32, mode as i32, yp as *mut f32, s)
        });
        Ok(())
    }

    /// Prefill GEMM over the path's rows (Builder::gemm, graph.rs:200-205; N % 32, K % 128 as :375-376).
    #[allow(clippy::too_many_arguments)]
    pub fn gemm(&mut self, name: &'static str, w: &str, k: u32, n: u32, mode: u32, a: &Acts, y: &DevBuf) -> Result<(), String> {
        if n % 32 != 0 || k % 128 != 0 {
            return Err(format!("{name}: GEMM needs N % 32 == 0 and K % 128 == 0 (N = {n}, K = {k})"));
        }
        let wt = self.e.weight(w, k, if mode == 2 { 2 * n } else { n })?;
        let (m, xq, xs, yp) = (a.rows, a.xq.ptr as usize, a.xs.ptr as usize, y.ptr as usize);
        self.push(name, move |s| unsafe {
            ffi::w4a8_gemm(&wt, xq as *const i8, xs as *const f32, ffi::W4A8_ACT_GROUP32, m as i32, mode as i32, yp as *mut f32, s)
        });
        Ok(())
    }

    /// Builder::matmul (graph.rs:207-214): the GEMM for prefill, the GEMV otherwise.
    #[allow(clippy::too_many_arguments)]
    pub fn matmul(&mut self, path: Path, name: &'static str, w: &str, k: u32, n: u32, mode: u32, a: &Acts, y: &DevBuf) -> Result<(), String> {
        match path {
            Path::Prefill => self.gemm(name, w, k, n, mode, a, y),
            Path::Spec => self.gemv(name, w, k, n, mode, 2, a, y),
            Path::Decode => self.gemv(name, w, k, n, mode, 1, a, y),
        }
    }

    /// Builder::quant (graph.rs:216-222): rows of x (k wide), optionally RMSNorm'ed by `norm`.
    pub fn quant(&mut self, name: &'static str, k: u32, eps: f64, x: &DevBuf, norm: Option<&str>, a: &Acts) -> Result<(), String> {
        let nw = match norm {
            Some(n) => self.e.w(n)?.ptr as usize,
            None => 0,
        };
        let (xp, xq, xs, m) = (x.ptr as usize, a.xq.ptr as usize, a.xs.ptr as usize, a.rows);
        self.push(name, move |s| unsafe {
            ffi::w4a8_quant(xp as *const f32, nw as *const f32, eps as f32, m as i32, k as i32, ffi::W4A8_ACT_GROUP32,
                            xq as *mut i8, xs as *mut f32, s)
        });
        Ok(())
    }

    /// The argmax op of head_ops (graph.rs:484; argmax.wgsl, MAPPED when `ids` is given).
    pub fn argmax(&mut self, name: &'static str, logits: &DevBuf, m: u32, v: u32, ids: Option<&DevBuf>, tok: &DevBuf) {
        let (lp, ip, tp) = (logits.ptr as usize, ids.map_or(0, |b| b.ptr as usize), tok.ptr as usize);
        self.push(name, move |s| unsafe { ffi::w4a8_argmax(lp as *const f32, m as i32, v as i32, ip as *const u32, tp as *mut u32, s) });
    }

    /// head_ops (graph.rs:476-486) with the GEMV and the argmax fused: the token of
    /// the greedy step lands in `tok` (u32[t]); `ws` is a zeroed workspace of
    /// `w4a8_lmhead_workspace_bytes(vocab, t)` bytes, reused by every step.
    #[allow(clippy::too_many_arguments)]
    pub fn lm_head(&mut self, name: &'static str, w: &str, k: u32, vocab: u32, t: u32, a: &Acts, tok: &DevBuf, ws: &DevBuf) -> Result<(), String> {
        let need = unsafe { ffi::w4a8_lmhead_workspace_bytes(vocab as i32, t as i32) };
        if ws.bytes < need {
            return Err(format!("{name}: workspace of {} bytes, {need} needed", ws.bytes));
        }
        let wt = self.e.weight(w, k, vocab)?;
        let (xq, xs, tp, wp, wb) = (a.xq.ptr as usize, a.xs.ptr as usize, tok.ptr as usize, ws.ptr as usize, ws.bytes);
        self.push(name, move |s| unsafe {
            ffi::w4a8_lmhead_argmax(&wt, 0, xq as *const i8, xs as *const f32, ffi::W4A8_ACT_GROUP32, t as i32,
                                    std::ptr::null_mut(), std::ptr::null_mut(), tp as *mut u32, std::ptr::null(),
                                    wp as *mut c_void, wb, s)
        });
        Ok(())
    }
}

/// The ops of one step, issued in order on the engine's stream (the wgpu backend
/// submits its passes in queue order), optionally captured once into a CUDA graph.
pub struct CudaPlan {
    ops: Vec<CudaOp>,
    graph: *mut c_void,
    exec: *mut c_void,
}

impl CudaPlan {
    pub fn new(ops: Vec<CudaOp>) -> Self {
        CudaPlan { ops, graph: std::ptr::null_mut(), exec: std::ptr::null_mut() }
    }

    pub fn len(&self) -> usize {
        self.ops.len()
    }

    pub fn is_empty(&self) -> bool {
        self.ops.is_empty()
    }

    /// Issue every op on `stream` (no host synchronization).
    pub fn run(&self, stream: *mut c_void) -> Result<(), String> {
        if !self.exec.is_null() {
            return cuda(unsafe { cudaGraphLaunch(self.exec, stream) }, "cudaGraphLaunch");
        }
        for op in &self.ops {
            (op.run)(stream).map_err(|e| format!("{}: {e}", op.name))?;
        }
        Ok(())
    }

    /// Capture the ops once into a CUDA graph; `run` then replays it.  Run the plan
    /// once eagerly before capturing (the library sets per-device kernel attributes
    /// on first use).
    pub fn capture(&mut self, stream: *mut c_void) -> Result<(), String> {
        cuda(unsafe { cudaStreamBeginCapture(stream, CAPTURE_THREAD_LOCAL) }, "begin capture")?;
        let issued = self.ops.iter().try_for_each(|op| (op.run)(stream));
        let mut g = std::ptr::null_mut();
        let ended = cuda(unsafe { cudaStreamEndCapture(stream, &mut g) }, "end capture");
        issued?;
        ended?;
        let mut e = std::ptr::null_mut();
        cuda(unsafe { cudaGraphInstantiate(&mut e, g, 0) }, "instantiate")?;
        self.graph = g;
        self.exec = e;
        Ok(())
    }

    pub fn sync(stream: *mut c_void) -> Result<(), String> {
        cuda(unsafe { cudaStreamSynchronize(stream) }, "cudaStreamSynchronize")
    }
}

impl Drop for CudaPlan {
    fn drop(&mut self) {
        unsafe {
            if !self.exec.is_null() {
                cudaGraphExecDestroy(self.exec);
            }
            if !self.graph.is_null() {
                cudaGraphDestroy(self.graph);
            }
        }
    }
}

/// Surfaces a bounded device-side wait that gave up (`w4a8_device_error`).
pub fn device_error(stream: *mut c_void) -> Result<(), String> {
    let mut code = 0u32;
    check(unsafe { ffi::w4a8_device_error(&mut code, stream) }).map_err(|e| format!("{e} (device code {code})"))
}
