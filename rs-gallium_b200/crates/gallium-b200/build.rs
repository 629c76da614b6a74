//! Builds libgallium_b200.so with the repository's Makefile (nvcc, sm_100a)
//! and links it.  GALLIUM_B200_DIR overrides where the library's sources
//! (the directory holding the Makefile) live.
use std::env;
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let dir = env::var("GALLIUM_B200_DIR").map(PathBuf::from).unwrap_or_else(|_| {
        PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("../..")
    });
    let status = Command::new("make")
        .arg("-C")
        .arg(&dir)
        .arg(format!("-j{}", env::var("NUM_JOBS").unwrap_or_else(|_| "8".into())))
        .status()
        .expect("running make (needs nvcc for sm_100a)");
    assert!(status.success(), "make -C {} failed", dir.display());
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=gallium_b200");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
    println!("cargo:rerun-if-changed={}", dir.join("csrc").display());
    println!("cargo:rerun-if-changed={}", dir.join("../include/gallium_b200.h").display());
    println!("cargo:rerun-if-env-changed=GALLIUM_B200_DIR");
}
