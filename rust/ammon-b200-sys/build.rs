//! Links libammon_b200.so, built in-tree by `python -m ammon_b200.build` into
//! <repo>/ammon_b200/. AMMON_B200_LIB_DIR overrides the directory.
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = match env::var("AMMON_B200_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => {
            let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
            manifest.join("..").join("..").join("ammon_b200")
        }
    };
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=ammon_b200");
    println!("cargo:rerun-if-env-changed=AMMON_B200_LIB_DIR");
    println!("cargo:rerun-if-changed=../../include/ammon_b200.h");
}
