// build.rs -- links libtambear_gb.so (include/tambear_gb.h, sm_100a).
// Not compiled here: no Rust toolchain in this build environment.
//
// The library is built by nvcc, not by cargo: either point TAMBEAR_GB_DIR at a folder that already
// holds libtambear_gb.so (e.g. winrapids_b200/ after `python winrapids_b200/build.py`), or set
// TAMBEAR_GB_SRC to the repository root and this script runs that build (every CUDA source with
// -gencode arch=compute_100a,code=sm_100a) and links the result.
use std::env;
use std::path::PathBuf;
use std::process::Command;

fn main() {
    println!("cargo:rerun-if-env-changed=TAMBEAR_GB_DIR");
    println!("cargo:rerun-if-env-changed=TAMBEAR_GB_SRC");
    let dir: PathBuf = if let Ok(dir) = env::var("TAMBEAR_GB_DIR") {
        PathBuf::from(dir)
    } else {
        let src = PathBuf::from(env::var("TAMBEAR_GB_SRC").expect(
            "set TAMBEAR_GB_DIR (folder of libtambear_gb.so) or TAMBEAR_GB_SRC (repository root)",
        ));
        let status = Command::new("python3")
            .arg(src.join("winrapids_b200").join("build.py"))
            .status()
            .expect("running winrapids_b200/build.py (needs nvcc 12.8+ for sm_100a)");
        assert!(status.success(), "building libtambear_gb.so failed");
        println!("cargo:rerun-if-changed={}", src.join("winrapids_b200").join("csrc").display());
        println!("cargo:rerun-if-changed={}", src.join("include").join("tambear_gb.h").display());
        src.join("winrapids_b200")
    };
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=tambear_gb");
    println!("cargo:rustc-link-lib=dylib=cudart");
    // the loader finds the library next to the binary or through this rpath
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}
