//! Links libqwqmm.so.  The library is built in-tree next to its Python
//! package (`make -C qw_b200/csrc`); QW_B200_LIB_DIR overrides the directory.
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = env::var("QW_B200_LIB_DIR").map(PathBuf::from).unwrap_or_else(|_| {
        PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("../../qw_b200")
    });
    println!("cargo:rerun-if-env-changed=QW_B200_LIB_DIR");
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=qwqmm");
    // the runtime finds the library where it was linked from
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}
