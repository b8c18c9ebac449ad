//! Links libvfr_retrieval.so (built by vocal-fast-rs_b200/build.py) and the
//! CUDA runtime.  VFR_RETRIEVAL_LIB_DIR names the directory holding the
//! library; CUDA_HOME (default /usr/local/cuda) the CUDA toolkit.

fn main() {
    println!("cargo:rerun-if-env-changed=VFR_RETRIEVAL_LIB_DIR");
    println!("cargo:rerun-if-env-changed=CUDA_HOME");
    let lib_dir = std::env::var("VFR_RETRIEVAL_LIB_DIR").unwrap_or_else(|_| {
        let manifest = std::env::var("CARGO_MANIFEST_DIR").expect("cargo sets CARGO_MANIFEST_DIR");
        format!("{manifest}/../../vocal-fast-rs_b200")
    });
    let cuda = std::env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".into());
    println!("cargo:rustc-link-search=native={lib_dir}");
    println!("cargo:rustc-link-search=native={cuda}/lib64");
    println!("cargo:rustc-link-lib=dylib=vfr_retrieval");
    println!("cargo:rustc-link-lib=dylib=cudart");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{lib_dir}");
}
