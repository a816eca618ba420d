//! Builds libmyos_cuda from the package's CUDA/C++ sources with nvcc for
//! sm_100a (B200) and links it, with the CUDA runtime, into the crate.
//!
//! Environment:
//!   NVCC            nvcc to use (default: $CUDA_HOME/bin/nvcc, then `nvcc`)
//!   CUDA_HOME       CUDA toolkit root (default /usr/local/cuda)
//!   CUTLASS_INCLUDE CUTLASS/CuTe include directory (SM100 collectives) for
//!                   the tensor-core prefill GEMM; required
use std::env;
use std::path::{Path, PathBuf};
use std::process::Command;

const SOURCES: &[&str] = &[
    "kernels.cu",
    "engine.cu",
    "ops.cu",
    "noalloc.cu",
    "prefill.cu",
    "gemm_sm100.cu",
    "safetensors.cpp",
    "tp.cpp",
];

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    let pkg = manifest.join("../..");
    let csrc = pkg.join("csrc");
    let include = pkg.join("../include");
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());
    let cuda = env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".to_string());
    let nvcc = env::var("NVCC").unwrap_or_else(|_| {
        let p = Path::new(&cuda).join("bin/nvcc");
        if p.exists() { p.display().to_string() } else { "nvcc".to_string() }
    });
    let cutlass = env::var("CUTLASS_INCLUDE").expect("CUTLASS_INCLUDE must name the CUTLASS include dir");

    let mut objects = Vec::new();
    for src in SOURCES {
        let path = csrc.join(src);
        println!("cargo:rerun-if-changed={}", path.display());
        let obj = out.join(format!("{}.o", src));
        let mut cmd = Command::new(&nvcc);
        cmd.args(["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17"])
            .args(["-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"])
            .arg(format!("-I{}", include.display()))
            .arg(format!("-I{}", cutlass));
        if src.ends_with(".cpp") {
            cmd.args(["-x", "cu"]);
        }
        if src.starts_with("gemm_") {
            // the GEMM waits on its predecessor when launched with PDL
            cmd.arg("-DCUTLASS_ENABLE_GDC_FOR_SM100=1");
        }
        cmd.arg("-c").arg(&path).arg("-o").arg(&obj);
        let status = cmd.status().expect("failed to run nvcc");
        assert!(status.success(), "nvcc failed on {}", src);
        objects.push(obj);
    }
    // device link (relocatable device code is not used, but the step keeps
    // the archive self-contained), then the static archive
    let lib = out.join("libmyos_cuda.a");
    let status = Command::new("ar").arg("crs").arg(&lib).args(&objects).status().expect("ar");
    assert!(status.success(), "ar failed");
    println!("cargo:rerun-if-changed={}", include.join("myos_cuda.h").display());
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=static=myos_cuda");
    println!("cargo:rustc-link-search=native={}/lib64", cuda);
    println!("cargo:rustc-link-lib=static=cudart_static");
    for l in ["dl", "rt", "pthread", "stdc++"] {
        println!("cargo:rustc-link-lib={}", l);
    }
}
