// Builds libgguf_cuda.so (nvcc, sm_100a) from ../../csrc and links it.
fn main() {
    let manifest = std::env::var("CARGO_MANIFEST_DIR").expect("CARGO_MANIFEST_DIR");
    let root = std::path::Path::new(&manifest).join("../..");
    let csrc = root.join("csrc");
    let lib = root.join("lib");
    let st = std::process::Command::new("make")
        .arg("-C")
        .arg(&csrc)
        .status()
        .expect("make not found");
    assert!(st.success(), "nvcc build of libgguf_cuda failed");
    println!("cargo:rustc-link-search=native={}", lib.display());
    println!("cargo:rustc-link-lib=dylib=gguf_cuda");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", lib.display());
    println!("cargo:rerun-if-changed={}", csrc.display());
}
