//! Builds libwebyiq_w4a8.so for the CUDA backend (src/cuda): every .cu file of
//! webyiq_b200/csrc compiled by nvcc for sm_100a with the CUDA runtime linked
//! statically, then linked into this crate.  WEBYIQ_B200_DIR names the checkout of
//! the library (the directory holding include/ and webyiq_b200/csrc/).
//! Only the `cuda` feature builds it; the wgpu backend needs nothing from here.

use std::{env, path::PathBuf, process::Command};

fn main() {
    if env::var_os("CARGO_FEATURE_CUDA").is_none() {
        return;
    }
    let root = PathBuf::from(env::var("WEBYIQ_B200_DIR").expect("WEBYIQ_B200_DIR: path of the webyiq-b200 checkout"));
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());
    let csrc = root.join("webyiq_b200").join("csrc");
    let mut srcs: Vec<PathBuf> = std::fs::read_dir(&csrc)
        .expect("webyiq_b200/csrc")
        .map(|e| e.unwrap().path())
        .filter(|p| p.extension().map_or(false, |x| x == "cu"))
        .collect();
    srcs.sort();
    let nvcc = env::var("NVCC").unwrap_or_else(|_| "nvcc".into());
    let status = Command::new(nvcc)
        .args(["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
               "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
               "-shared", "-cudart", "static"])
        .arg(format!("-I{}", root.join("include").display()))
        .args(&srcs)
        .arg("-o")
        .arg(out.join("libwebyiq_w4a8.so"))
        .args(["-ldl", "-lpthread", "-lrt"])
        .status()
        .expect("running nvcc");
    assert!(status.success(), "nvcc failed");
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=dylib=webyiq_w4a8");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", out.display());
    // cudart for the backend's own buffer and graph calls
    let cuda_home = env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".into());
    println!("cargo:rustc-link-search=native={cuda_home}/lib64");
    println!("cargo:rerun-if-changed={}", csrc.display());
    println!("cargo:rerun-if-changed={}", root.join("include").join("w4a8.h").display());
    println!("cargo:rerun-if-env-changed=WEBYIQ_B200_DIR");
}
