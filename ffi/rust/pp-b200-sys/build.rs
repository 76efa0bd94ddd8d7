//! Links libpp_b200.so.  PP_B200_LIB_DIR names the directory that holds it;
//! by default the library built in place by pop2-bezier_b200/build_native.py
//! in this repository (three levels above this crate).
use std::env;
use std::path::PathBuf;

fn main() {
    println!("cargo:rerun-if-env-changed=PP_B200_LIB_DIR");
    let dir = match env::var("PP_B200_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => {
            let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").expect("cargo sets CARGO_MANIFEST_DIR"));
            manifest.join("..").join("..").join("..").join("pop2-bezier_b200")
        }
    };
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=pp_b200");
    // the library resolves the CUDA runtime of the process (shared libcudart)
    println!("cargo:rustc-link-lib=dylib=cudart");
}
