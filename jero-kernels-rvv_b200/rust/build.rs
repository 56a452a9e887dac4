//! Generates the raw FFI declarations of include/jkb200.h with bindgen and links libjkb200.so
//! (built by `make -C jero-kernels-rvv_b200`, nvcc for sm_100a) and the CUDA runtime, whose
//! memory calls the safe wrappers use to stage host slices.
//!
//! Not compiled in this repository (no Rust toolchain in the build image).
use std::env;
use std::path::PathBuf;

fn main() {
    let pkg = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("..");
    let header = pkg.join("..").join("include").join("jkb200.h");
    let cuda = env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".into());
    println!("cargo:rerun-if-changed={}", header.display());
    println!("cargo:rustc-link-search=native={}", pkg.display());
    println!("cargo:rustc-link-lib=dylib=jkb200");
    println!("cargo:rustc-link-search=native={cuda}/lib64");
    println!("cargo:rustc-link-lib=dylib=cudart");
    let bindings = bindgen::Builder::default()
        .header(header.to_string_lossy())
        .allowlist_function("jkb_.*")
        .allowlist_type("jkb_.*")
        .allowlist_var("JKB_.*")
        .derive_default(true)
        .generate()
        .expect("bindgen of include/jkb200.h");
    let out = PathBuf::from(env::var("OUT_DIR").unwrap()).join("jkb200.rs");
    bindings.write_to_file(out).expect("write bindings");
}
