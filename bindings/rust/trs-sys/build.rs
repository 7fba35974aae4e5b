//! Links libtrs_b200.so.  TRS_B200_LIB_DIR names the directory holding it;
//! by default the package directory of this repository, where
//! `python -m tensorrs_b200.build` puts it.
use std::env;
use std::path::PathBuf;

fn main() {
    let dir = match env::var("TRS_B200_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("../../../tensorrs_b200"),
    };
    println!("cargo:rerun-if-env-changed=TRS_B200_LIB_DIR");
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=trs_b200");
    // the library is loaded from the same directory at run time
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}
