// Builds libforgesort.so for sm_100a with the repository's own build step
// (nvcc; gpu-forge_b200/build.py) and links it.  Replaces forge-sort's
// build.rs, which compiled shaders/sort.metal with `xcrun metal`.
//
// NOT COMPILED: no cargo on the image this was written on.
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let manifest = PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").expect("CARGO_MANIFEST_DIR"));
    // gpu-forge_b200/rust/forge-sort -> repository root
    let root = std::env::var("FORGESORT_B200_ROOT")
        .map(PathBuf::from)
        .unwrap_or_else(|_| manifest.join("../../.."));
    let pkg = root.join("gpu-forge_b200");
    let python = std::env::var("PYTHON").unwrap_or_else(|_| "python3".to_string());
    let status = Command::new(python)
        .arg(pkg.join("build.py"))
        .status()
        .expect("running gpu-forge_b200/build.py (needs nvcc)");
    assert!(status.success(), "building libforgesort.so failed");
    let libdir = pkg.join("forge_sort");
    println!("cargo:rustc-link-search=native={}", libdir.display());
    println!("cargo:rustc-link-lib=dylib=forgesort");
    // let binaries find the library without LD_LIBRARY_PATH
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", libdir.display());
    println!("cargo:rerun-if-changed={}", pkg.join("csrc").display());
    println!("cargo:rerun-if-changed={}", root.join("include").display());
    println!("cargo:rerun-if-env-changed=FORGESORT_B200_ROOT");
}
