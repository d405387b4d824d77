//! Builds libslmkv.so (nvcc, sm_100a) with the library's own Makefile and
//! links it. The library lands in small-lm-rs_b200/slmkv/ next to the
//! Python mirror; its directory goes on the rpath so a binary finds it.
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let manifest = PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").expect("cargo sets it"));
    let pkg = manifest.join("../..").canonicalize().expect("small-lm-rs_b200 directory");
    let csrc = pkg.join("csrc");
    let libdir = pkg.join("slmkv");
    let status = Command::new("make")
        .arg("-C")
        .arg(&csrc)
        .status()
        .expect("running make for libslmkv");
    assert!(status.success(), "building libslmkv.so failed");
    println!("cargo:rustc-link-search=native={}", libdir.display());
    println!("cargo:rustc-link-lib=dylib=slmkv");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", libdir.display());
    println!("cargo:rerun-if-changed={}", csrc.display());
    println!("cargo:rerun-if-changed={}", pkg.join("../include/slmkv.h").display());
}
