// Link libphyzb200.so. It is built by phyz_b200/build.py into the
// repository's phyz_b200/ folder; PHYZB200_LIB_DIR points at the folder that
// holds it (default: that folder, relative to this crate in the repository).
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = match env::var("PHYZB200_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("../../phyz_b200"),
    };
    println!("cargo:rerun-if-env-changed=PHYZB200_LIB_DIR");
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=phyzb200");
    // the library locates itself at run time only through the loader
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}
