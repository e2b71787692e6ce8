//! Builds libkivi_gpu.so from the CUDA sources of this repository with nvcc
//! for sm_100a (the recipe of kivi-cache-rs_b200/build.py) and links it.
//!
//! Environment: NVCC (default `nvcc`), CUDA_HOME (default /usr/local/cuda)
//! for the runtime library; KIVI_GPU_LIB_DIR skips the build and links a
//! prebuilt libkivi_gpu.so from that directory instead.
use std::env;
use std::fs;
use std::path::{Path, PathBuf};
use std::process::Command;

const NVCC_FLAGS: &[&str] = &[
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O2,-Wall",
    "-Xptxas",
    "-O3",
    "--expt-relaxed-constexpr",
];

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    // kivi-cache-rs_b200/rust/kivi-cache-sys -> kivi-cache-rs_b200/csrc, include/
    let pkg = manifest.join("../..");
    let csrc = pkg.join("csrc");
    let include = pkg.join("../include");
    println!("cargo:rerun-if-env-changed=KIVI_GPU_LIB_DIR");
    println!("cargo:rerun-if-env-changed=NVCC");
    if let Ok(dir) = env::var("KIVI_GPU_LIB_DIR") {
        println!("cargo:rustc-link-search=native={dir}");
        println!("cargo:rustc-link-lib=dylib=kivi_gpu");
        return;
    }
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());
    let nvcc = env::var("NVCC").unwrap_or_else(|_| "nvcc".to_string());
    let mut objs = Vec::new();
    let mut sources: Vec<PathBuf> = fs::read_dir(&csrc)
        .expect("csrc directory")
        .filter_map(|e| e.ok().map(|e| e.path()))
        .filter(|p| p.extension().map_or(false, |x| x == "cu"))
        .collect();
    sources.sort();
    for entry in fs::read_dir(&csrc).expect("csrc directory").flatten() {
        println!("cargo:rerun-if-changed={}", entry.path().display());
    }
    println!("cargo:rerun-if-changed={}", include.join("kivi_gpu.h").display());
    for src in &sources {
        let obj = out.join(format!("{}.o", src.file_name().unwrap().to_string_lossy()));
        run(Command::new(&nvcc)
            .args(NVCC_FLAGS)
            .arg("-I")
            .arg(&include)
            .arg("-c")
            .arg(src)
            .arg("-o")
            .arg(&obj));
        objs.push(obj);
    }
    let lib = out.join("libkivi_gpu.so");
    run(Command::new(&nvcc)
        .args(["-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC"])
        .arg("-o")
        .arg(&lib)
        .args(&objs));
    let cuda = env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".to_string());
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-search=native={}", Path::new(&cuda).join("lib64").display());
    println!("cargo:rustc-link-lib=dylib=kivi_gpu");
    println!("cargo:rustc-link-lib=dylib=cudart");
    // let dependants find the library at run time without an install step
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", out.display());
}

fn run(cmd: &mut Command) {
    let status = cmd.status().unwrap_or_else(|e| panic!("failed to run {cmd:?}: {e}"));
    assert!(status.success(), "{cmd:?} failed with {status}");
}
