//! Build hook: the role `nexus-core/build.rs:14-81` plays for the Metal shader
//! (there it runs `xcrun metal` / `metallib` and exports WEAVER_METALLIB,
//! `build.rs:62-81`).  Here it compiles every `aether_nexus_b200/csrc/*.cu`
//! for sm_100a with nvcc (through the repository's own build script, which
//! rebuilds only stale objects) and links the resulting shared library.
//!
//! WEAVER_B200_ROOT points at this repository; by default it is two levels
//! above this crate.

use std::env;
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").expect("CARGO_MANIFEST_DIR"));
    let root = env::var("WEAVER_B200_ROOT")
        .map(PathBuf::from)
        .unwrap_or_else(|_| manifest.join("..").join(".."));
    let pkg = root.join("aether_nexus_b200");
    let python = env::var("PYTHON").unwrap_or_else(|_| "python3".to_string());
    let status = Command::new(&python)
        .arg(pkg.join("build.py"))
        .status()
        .unwrap_or_else(|e| panic!("running {python} {}: {e}", pkg.join("build.py").display()));
    assert!(status.success(), "nvcc build of libweaver_cuda.so failed");
    println!("cargo:rustc-link-search=native={}", pkg.display());
    println!("cargo:rustc-link-lib=dylib=weaver_cuda");
    println!("cargo:rerun-if-changed={}", pkg.join("csrc").display());
    println!("cargo:rerun-if-changed={}", root.join("include").join("weaver_cuda.h").display());
    println!("cargo:rerun-if-env-changed=WEAVER_B200_ROOT");
}
