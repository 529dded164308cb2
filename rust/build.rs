// build.rs for the Clove crate: compiles the CUDA decode library for sm_100a
// with nvcc and links it, so `CudaBackend` needs no prebuilt artefact.
//
// Not compiled in this repository (no Rust toolchain here); the same nvcc
// command lines are what clove_b200/build.py runs.  Set CLOVE_B200_DIR to
// this repository's root (the .cu sources are under clove_b200/csrc, the
// public headers under include/).
use std::env;
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let root = PathBuf::from(env::var("CLOVE_B200_DIR").expect("CLOVE_B200_DIR: path of the clove_b200 sources"));
    let csrc = root.join("clove_b200").join("csrc");
    let include = root.join("include");
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());
    let nvcc = env::var("NVCC").unwrap_or_else(|_| "/usr/local/cuda/bin/nvcc".to_string());
    let mut objects = Vec::new();
    for entry in std::fs::read_dir(&csrc).expect("read csrc") {
        let path = entry.unwrap().path();
        if path.extension().map(|e| e == "cu").unwrap_or(false) {
            let obj = out.join(path.file_stem().unwrap()).with_extension("o");
            let status = Command::new(&nvcc)
                .args(["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-lineinfo"])
                .args(["-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr", "-I"])
                .arg(&include)
                .arg("-c")
                .arg(&path)
                .arg("-o")
                .arg(&obj)
                .status()
                .expect("run nvcc");
            assert!(status.success(), "nvcc failed for {}", path.display());
            println!("cargo:rerun-if-changed={}", path.display());
            objects.push(obj);
        }
    }
    // one shared library, as the Python side loads it
    let lib = out.join("libclove_cuda.so");
    let status = Command::new(&nvcc)
        .args(["-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o"])
        .arg(&lib)
        .args(&objects)
        .arg("-lcudart")
        .status()
        .expect("link libclove_cuda.so");
    assert!(status.success(), "linking libclove_cuda.so failed");
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=dylib=clove_cuda");
    println!("cargo:rustc-link-search=native=/usr/local/cuda/lib64");
    println!("cargo:rustc-link-lib=dylib=cudart");
    println!("cargo:rerun-if-changed={}", include.join("clove_cuda.h").display());
}
