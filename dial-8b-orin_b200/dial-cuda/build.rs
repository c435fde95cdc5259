//! Compiles the hand-written CUDA sources of ../csrc with nvcc for sm_100a
//! into a static library and links it, with the CUDA runtime, into the crate.
//!
//! nvcc: $NVCC, else $CUDA_HOME/bin/nvcc, else /usr/local/cuda/bin/nvcc.
//! No Triton, no NVRTC and no other architecture: the kernels use tcgen05,
//! TMEM and TMA and exist for sm_100a only.

use std::env;
use std::path::{Path, PathBuf};
use std::process::Command;

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    let csrc = manifest.join("..").join("csrc");
    let include = manifest.join("..").join("..").join("include");
    println!("cargo:rerun-if-changed={}", csrc.display());
    println!("cargo:rerun-if-changed={}", include.display());
    println!("cargo:rerun-if-env-changed=NVCC");
    println!("cargo:rerun-if-env-changed=CUDA_HOME");
    if env::var_os("CARGO_FEATURE_NO_CUDA_BUILD").is_some() {
        return;
    }
    let cuda_home = env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".to_string());
    let nvcc = env::var("NVCC").unwrap_or_else(|_| format!("{}/bin/nvcc", cuda_home));
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());

    let mut sources: Vec<PathBuf> = std::fs::read_dir(&csrc)
        .expect("csrc directory")
        .filter_map(|e| e.ok().map(|e| e.path()))
        .filter(|p| p.extension().map(|x| x == "cu").unwrap_or(false))
        .collect();
    sources.sort();
    assert!(!sources.is_empty(), "no .cu sources in {}", csrc.display());

    let mut objects = Vec::new();
    for src in &sources {
        let obj = out.join(Path::new(src.file_stem().unwrap()).with_extension("o"));
        let status = Command::new(&nvcc)
            .args(["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17"])
            .args(["--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-fvisibility=hidden"])
            .arg(format!("-I{}", include.display()))
            .arg(format!("-I{}", csrc.display()))
            .arg("-c")
            .arg(src)
            .arg("-o")
            .arg(&obj)
            .status()
            .unwrap_or_else(|e| panic!("running {}: {}", nvcc, e));
        assert!(status.success(), "nvcc failed on {}", src.display());
        objects.push(obj);
    }
    let lib = out.join("libdial_cuda.a");
    let _ = std::fs::remove_file(&lib);
    let status = Command::new("ar").arg("crs").arg(&lib).args(&objects).status().expect("running ar");
    assert!(status.success(), "ar failed");

    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=static=dial_cuda");
    println!("cargo:rustc-link-search=native={}/lib64", cuda_home);
    println!("cargo:rustc-link-lib=dylib=cudart");
    println!("cargo:rustc-link-lib=dylib=stdc++");
    println!("cargo:rustc-link-lib=dylib=dl");
}
