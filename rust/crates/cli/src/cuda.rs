//! `--backend cuda` for webyiq-cli: the `--ref` and `--bench` modes of
//! crates/cli/src/main.rs (:274-350) run on the CUDA backend of webyiq-engine
//! (crates/engine/src/cuda).  main.rs dispatches here when `--backend cuda` is
//! given, after parsing the same arguments:
//!
//!     "cuda" => return cuda::run(&args.model, args.reference.as_deref(), args.bench),
//!
//!   --ref <prefix>   op-level check of the W4A8 path on this GPU, the file protocol
//!                    of webyiq_cli (the C++ host of this repository):
//!                    <prefix>.json {"op": "matmul" | "lm_head", "weight": name,
//!                    "m": M, "mode": 0 | 1 | 2, "eps": e}, <prefix>.x.f32 (f32 [M, K]),
//!                    <prefix>.y.f32 (expected f32 [M, N]) or <prefix>.tok.u32;
//!                    quant + matmul (or the fused lm_head argmax) through CudaBuilder,
//!                    |y - ref| <= 1e-3 |ref| + 1e-3 rms(ref), tokens exact.
//!   --bench <iters>  every q4 weight of the manifest: the GEMV at M = 1 captured as
//!                    one decode-step graph and replayed <iters> times, GB/s from the
//!                    packed bytes.
//!
//! Not built in this repository (no cargo in its image).

use std::ffi::c_void;
use std::time::Instant;

use webyiq_engine::cuda::{ffi, Acts, CudaBuilder, CudaEngine, CudaPlan, DevBuf};
use webyiq_engine::Manifest;

fn read_f32(path: &str) -> Result<Vec<f32>, String> {
    let b = std::fs::read(path).map_err(|e| format!("{path}: {e}"))?;
    Ok(b.chunks_exact(4).map(|c| f32::from_le_bytes([c[0], c[1], c[2], c[3]])).collect())
}

fn as_bytes(v: &[f32]) -> &[u8] {
    unsafe { std::slice::from_raw_parts(v.as_ptr() as *const u8, v.len() * 4) }
}

fn load(model: &str) -> Result<CudaEngine, String> {
    let json = std::fs::read_to_string(format!("{model}/manifest.json")).map_err(|e| e.to_string())?;
    let m = Manifest::parse(&json)?;
    let shards = m.shards.clone();
    let e = CudaEngine::new(m, 0)?;
    for (i, s) in shards.iter().enumerate() {
        let data = std::fs::read(format!("{model}/{s}")).map_err(|e| format!("{s}: {e}"))?;
        e.upload_shard(i, &data)?;
    }
    Ok(e)
}

/// Shape (n, k) of q4 tensor `{w}.q` from the manifest.
fn shape(e: &CudaEngine, w: &str) -> Result<(u32, u32), String> {
    let t = e.manifest().tensors.get(&format!("{w}.q")).ok_or_else(|| format!("missing tensor {w}.q"))?;
    Ok((t.shape[0] as u32, t.shape[1] as u32))
}

fn reference(e: &CudaEngine, prefix: &str) -> Result<bool, String> {
    let spec: serde_json::Value =
        serde_json::from_str(&std::fs::read_to_string(format!("{prefix}.json")).map_err(|e| e.to_string())?)
            .map_err(|e| e.to_string())?;
    let op = spec["op"].as_str().unwrap_or("matmul");
    let w = spec["weight"].as_str().ok_or("spec: weight")?;
    let m = spec["m"].as_u64().unwrap_or(1) as u32;
    let mode = spec["mode"].as_u64().unwrap_or(0) as u32;
    let eps = spec["eps"].as_f64().unwrap_or(1e-6);
    let (n, k) = shape(e, w)?;
    let n_out = if mode == 2 { n / 2 } else { n };
    let x = read_f32(&format!("{prefix}.x.f32"))?;
    let dx = DevBuf::new(x.len() * 4)?;
    dx.write(as_bytes(&x))?;
    let acts = Acts::new(m, k)?;
    let mut b = CudaBuilder::new(e);
    b.quant("quant", k, eps, &dx, None, &acts)?;
    if op == "lm_head" {
        let tok = DevBuf::new(4 * m as usize)?;
        let ws = DevBuf::new(unsafe { ffi::w4a8_lmhead_workspace_bytes(n as i32, m as i32) })?;
        b.lm_head("lm_head", w, k, n, m, &acts, &tok, &ws)?;
        let plan = CudaPlan::new(b.ops);
        plan.run(e.stream)?;
        CudaPlan::sync(e.stream)?;
        let mut got = vec![0u8; 4 * m as usize];
        tok.read(&mut got)?;
        let want = std::fs::read(format!("{prefix}.tok.u32")).map_err(|e| e.to_string())?;
        return Ok(got == want[..got.len()]);
    }
    let y = DevBuf::new(4 * (m * n_out) as usize)?;
    if mode == 1 {
        y.write(as_bytes(&read_f32(&format!("{prefix}.y0.f32"))?))?;
    }
    if m > 16 { b.gemm("gemm", w, k, n_out, mode, &acts, &y)? } else { b.gemv("gemv", w, k, n_out, mode, m, &acts, &y)? }
    let plan = CudaPlan::new(b.ops);
    plan.run(e.stream)?;
    CudaPlan::sync(e.stream)?;
    let mut got = vec![0f32; (m * n_out) as usize];
    y.read(unsafe { std::slice::from_raw_parts_mut(got.as_mut_ptr() as *mut u8, got.len() * 4) })?;
    let want = read_f32(&format!("{prefix}.y.f32"))?;
    let rms = (want.iter().map(|v| (*v as f64).powi(2)).sum::<f64>() / want.len() as f64).sqrt();
    let bad = got.iter().zip(&want).filter(|(g, r)| ((**g - **r) as f64).abs() > 1e-3 * (**r as f64).abs() + 1e-3 * rms).count();
    println!("{op} {w}: m={m} n={n_out} k={k} mismatches {bad} of {}", got.len());
    Ok(bad == 0)
}

fn bench(e: &CudaEngine, iters: u32) -> Result<(), String> {
    let mut names: Vec<String> =
        e.manifest().tensors.iter().filter(|(n, t)| n.ends_with(".q") && t.dtype == "q4").map(|(n, _)| n[..n.len() - 2].to_string()).collect();
    names.sort();
    let kmax = names.iter().map(|w| shape(e, w).map(|s| s.1)).collect::<Result<Vec<_>, _>>()?.into_iter().max().unwrap_or(0);
    let nmax = names.iter().map(|w| shape(e, w).map(|s| s.0)).collect::<Result<Vec<_>, _>>()?.into_iter().max().unwrap_or(0);
    let acts = Acts::new(1024, kmax)?;
    let y = DevBuf::new(4 * 1024 * nmax as usize)?;
    let mut b = CudaBuilder::new(e);
    let mut bytes = 0usize;
    for w in &names {
        let (n, k) = shape(e, w)?;
        b.gemv("gemv", w, k, n, 0, 1, &acts, &y)?;
        bytes += (n as usize) * (k as usize) / 2 + (n as usize) * (k as usize / 32) * 4;
    }
    let mut plan = CudaPlan::new(b.ops);
    plan.run(e.stream)?; // first calls set per-device kernel attributes
    CudaPlan::sync(e.stream)?;
    plan.capture(e.stream)?;
    let t0 = Instant::now();
    for _ in 0..iters {
        plan.run(e.stream)?;
    }
    CudaPlan::sync(e.stream)?;
    let s = t0.elapsed().as_secs_f64() / iters as f64;
    println!("decode step: {} GEMVs, {:.1} us, {:.1} GB/s", plan.len(), s * 1e6, bytes as f64 / s / 1e9);
    webyiq_engine::cuda::device_error(e.stream as *mut c_void)?;
    Ok(())
}

/// Entry of `--backend cuda`; the exit code follows main.rs (0 ok, 1 mismatch).
pub fn run(model: &str, reference_prefix: Option<&str>, bench_iters: u32) -> Result<i32, String> {
    let e = load(model)?;
    if let Some(p) = reference_prefix {
        return Ok(if reference(&e, p)? { 0 } else { 1 });
    }
    if bench_iters > 0 {
        bench(&e, bench_iters)?;
    }
    Ok(0)
}
