// Builds the CUDA static library for sm_100a (nvcc through the library's
// Makefile) and links it with the static CUDA runtime.  Environment:
//   KRIKIL_B200_DIR  checkout of this repository (default: the parent of this crate)
//   CUDA_HOME        CUDA toolkit (default /usr/local/cuda)
use std::env;
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let root = env::var("KRIKIL_B200_DIR")
        .map(PathBuf::from)
        .unwrap_or_else(|_| PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join(".."));
    let lib_dir = root.join("krikil_rs_b200");
    let cuda = PathBuf::from(env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".into()));

    let status = Command::new("make")
        .arg("-C")
        .arg(&lib_dir)
        .arg("-j8")
        .arg("lib/libkrikil_cuda.a")
        .env("NVCC", cuda.join("bin/nvcc"))
        .status()
        .expect("running make for the CUDA library");
    assert!(status.success(), "building krikil_rs_b200/lib/libkrikil_cuda.a failed");

    println!("cargo:rustc-link-search=native={}", lib_dir.join("lib").display());
    println!("cargo:rustc-link-lib=static=krikil_cuda");
    println!("cargo:rustc-link-search=native={}", cuda.join("lib64").display());
    println!("cargo:rustc-link-lib=static=cudart_static");
    for l in ["stdc++", "dl", "rt", "pthread"] {
        println!("cargo:rustc-link-lib={}", l);
    }
    println!("cargo:rerun-if-env-changed=KRIKIL_B200_DIR");
    println!("cargo:rerun-if-changed={}", root.join("include/krikil_cuda.h").display());
    println!("cargo:rerun-if-changed={}", lib_dir.join("csrc").display());
}
