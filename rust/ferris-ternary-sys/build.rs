// Links libferris_ternary.so.  FERRIS_TERNARY_LIB_DIR names the directory that
// holds it (the package directory of the Python build, ferrisres_b200/, by
// default relative to this crate).
fn main() {
    let dir = std::env::var("FERRIS_TERNARY_LIB_DIR")
        .unwrap_or_else(|_| concat!(env!("CARGO_MANIFEST_DIR"), "/../../ferrisres_b200").to_string());
    println!("cargo:rustc-link-search=native={}", dir);
    println!("cargo:rustc-link-lib=dylib=ferris_ternary");
    println!("cargo:rerun-if-env-changed=FERRIS_TERNARY_LIB_DIR");
}
