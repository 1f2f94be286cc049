// Links librg_npu.so.  RG_NPU_LIB_DIR names the directory holding it (the
// repository's rustgears_b200/ after `python -m rustgears_b200.build`); the
// default is that directory relative to this crate.
use std::env;
use std::path::PathBuf;

fn main() {
    println!("cargo:rerun-if-env-changed=RG_NPU_LIB_DIR");
    let dir = match env::var("RG_NPU_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap()).join("../../rustgears_b200"),
    };
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=rg_npu");
    // the library resolves NCCL and the CUDA driver at load time through its own rpath
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}
