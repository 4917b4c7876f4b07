//! Links the prebuilt libtmoe.so (nvcc, sm_100a, the CUDA runtime linked statically; NCCL is a
//! dynamic dependency of the library).  TMOE_LIB_DIR names its directory; without it the
//! in-tree build next to this crate's sources is used (tetraeder_b200/libtmoe.so, made by
//! `python -m tetraeder_b200.build`).

use std::path::PathBuf;

fn main() {
    let dir = match std::env::var("TMOE_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").unwrap()).join("../../tetraeder_b200"),
    };
    if !dir.join("libtmoe.so").exists() {
        panic!("libtmoe.so not found in {} (set TMOE_LIB_DIR)", dir.display());
    }
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=tmoe");
    // the library is found at run time where it was linked from
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
    println!("cargo:rerun-if-env-changed=TMOE_LIB_DIR");
    println!("cargo:rerun-if-changed={}", dir.join("libtmoe.so").display());
}
