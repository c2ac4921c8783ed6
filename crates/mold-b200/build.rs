// Links libmold_b200.so, built from the CUDA sources of this repository by
// `python -m mold_b200.build` (nvcc, -gencode arch=compute_100a,code=sm_100a).
// MOLD_B200_LIB_DIR names the directory that holds it.
fn main() {
    let dir = std::env::var("MOLD_B200_LIB_DIR").unwrap_or_else(|_| "../../mold_b200".to_string());
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=mold_b200");
    println!("cargo:rerun-if-env-changed=MOLD_B200_LIB_DIR");
}
