// Links libhct_b200.so.  HCT_B200_LIB_DIR names the directory that holds it
// (built by `python -m haagenti_b200.build`, which leaves it in haagenti_b200/).
fn main() {
    println!("cargo:rerun-if-env-changed=HCT_B200_LIB_DIR");
    if let Ok(dir) = std::env::var("HCT_B200_LIB_DIR") {
        println!("cargo:rustc-link-search=native={dir}");
    } else {
        let here = std::path::PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").unwrap());
        let dir = here.join("../../haagenti_b200");
        println!("cargo:rustc-link-search=native={}", dir.display());
    }
    println!("cargo:rustc-link-lib=dylib=hct_b200");
}
