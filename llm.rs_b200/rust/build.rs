// build.rs for the reference crate: link the B200 library.  UNVERIFIED (no
// Rust toolchain in this image).  LLMRS_CUDA_LIB_DIR points at the folder that
// holds libllmrs_cuda.so (built by `python llm.rs_b200/build.py`).
fn main() {
    if let Ok(dir) = std::env::var("LLMRS_CUDA_LIB_DIR") {
        println!("cargo:rustc-link-search=native={}", dir);
        println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir);
    }
    println!("cargo:rustc-link-lib=dylib=llmrs_cuda");
    println!("cargo:rerun-if-env-changed=LLMRS_CUDA_LIB_DIR");
}
