//! Links librxla_b200.so.  The library is built by `python -m rxla_b200.build`
//! next to the Python package (`rxla_b200/librxla_b200.so`); point
//! RXLA_B200_LIB_DIR at another directory to link a copy elsewhere.
use std::path::PathBuf;

fn main() {
    println!("cargo:rerun-if-env-changed=RXLA_B200_LIB_DIR");
    let dir = std::env::var_os("RXLA_B200_LIB_DIR").map(PathBuf::from).unwrap_or_else(|| {
        PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").unwrap()).join("../../rxla_b200")
    });
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=rxla_b200");
    // the handlers must stay loaded for the process lifetime
    // (crates/rxla-pjrt/src/runtime.rs:276-279): embed the directory as rpath
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}
