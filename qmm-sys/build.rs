//! Links libqmm.so, the CUDA library behind include/qmm.h.
//!
//! The library is built by `python -m qwen_imager_b200.build` (nvcc, sm_100a)
//! into `qwen_imager_b200/_build/libqmm.so` beside this crate.  Set
//! `QMM_LIB_DIR` to link a copy installed elsewhere.
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = match env::var("QMM_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap())
            .join("..")
            .join("qwen_imager_b200")
            .join("_build"),
    };
    println!("cargo:rerun-if-env-changed=QMM_LIB_DIR");
    println!("cargo:rerun-if-changed=../include/qmm.h");
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=qmm");
}
