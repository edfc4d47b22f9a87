//! Points the linker at libteenyformers_b200.so.  The library is built by
//! `python -m teenyformers_b200.build` into teenyformers_b200/lib/ of this
//! repository; TEENYFORMERS_B200_LIB_DIR overrides the directory.

use std::{env, path::PathBuf};

fn main() {
    let dir = env::var("TEENYFORMERS_B200_LIB_DIR").map(PathBuf::from).unwrap_or_else(|_| {
        PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap())
            .join("../../teenyformers_b200/lib")
    });
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=teenyformers_b200");
    println!("cargo:rerun-if-env-changed=TEENYFORMERS_B200_LIB_DIR");
}
