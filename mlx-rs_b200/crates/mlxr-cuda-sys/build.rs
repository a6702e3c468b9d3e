// Links the prebuilt libmlxr_moe.so (python mlx-rs_b200/build.py builds it
// with nvcc for sm_100a and a static cudart): MLXR_CUDA_LIB_DIR names the
// directory that holds it.
fn main() {
    let dir = std::env::var("MLXR_CUDA_LIB_DIR").expect("path to libmlxr_moe.so");
    println!("cargo:rustc-link-search=native={dir}");
    println!("cargo:rustc-link-lib=dylib=mlxr_moe");
    println!("cargo:rerun-if-env-changed=MLXR_CUDA_LIB_DIR");
}
