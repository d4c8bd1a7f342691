//! Links libmarian_cuda.so (built by marian_cuda/build.py: every csrc/*.cu
//! for sm_100a, CUDA runtime linked statically, so only the driver is needed
//! at run time).
fn main() {
    println!("cargo:rerun-if-env-changed=MARIAN_CUDA_LIB_DIR");
    let dir = std::env::var("MARIAN_CUDA_LIB_DIR")
        .expect("set MARIAN_CUDA_LIB_DIR to the directory holding libmarian_cuda.so");
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=marian_cuda");
    // let the server binary find the library next to its own rpath
    println!("cargo:rustc-link-arg=-Wl,-rpath,{dir}");
}
