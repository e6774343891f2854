// Links libagpu.so: from $AGPU_LIB_DIR, else from the Python package
// directory next to this crate (any-gpu_b200/any_gpu, where build.py puts it),
// and records that directory as the run-time search path.
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = env::var("AGPU_LIB_DIR").map(PathBuf::from).unwrap_or_else(|_| {
        PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("..").join("any_gpu")
    });
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=agpu");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
    println!("cargo:rerun-if-env-changed=AGPU_LIB_DIR");
}
