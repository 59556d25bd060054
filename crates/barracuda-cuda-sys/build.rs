//! Links libbarracuda_fhe.so.
//!
//! The library is built outside cargo (`python -m barracuda_b200.build`, which
//! runs nvcc for sm_100a) and lands in `barracuda_b200/lib/`.  Point
//! `BARRACUDA_FHE_LIB_DIR` at that directory; without it the build looks in
//! the repository's default output directory relative to this crate.

use std::path::PathBuf;

fn main() {
    println!("cargo:rerun-if-env-changed=BARRACUDA_FHE_LIB_DIR");
    let dir = match std::env::var("BARRACUDA_FHE_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => {
            let manifest = PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").expect("CARGO_MANIFEST_DIR"));
            manifest.join("..").join("..").join("barracuda_b200").join("lib")
        }
    };
    if !dir.join("libbarracuda_fhe.so").exists() {
        println!(
            "cargo:warning=libbarracuda_fhe.so not found in {} (build it with `python -m barracuda_b200.build` \
             or set BARRACUDA_FHE_LIB_DIR)",
            dir.display()
        );
    }
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=barracuda_fhe");
    // the loader finds the library next to the binary's rpath entry
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}
