// UNVERIFIED (see Cargo.toml). Builds libslc.so (nvcc, sm_100a only) in the
// starlight_b200 checkout named by STARLIGHT_B200_ROOT and links it.
use std::env;
use std::path::PathBuf;
use std::process::Command;

fn main() {
    let root = PathBuf::from(
        env::var("STARLIGHT_B200_ROOT").expect("STARLIGHT_B200_ROOT: path of the starlight_b200 checkout"),
    );
    let status = Command::new(env::var("PYTHON").unwrap_or_else(|_| "python3".into()))
        .args(["-m", "starlight_b200.build"])
        .current_dir(&root)
        .status()
        .expect("running python -m starlight_b200.build");
    assert!(status.success(), "libslc build failed");
    let lib = root.join("starlight_b200");
    println!("cargo:rustc-link-search=native={}", lib.display());
    println!("cargo:rustc-link-lib=dylib=slc");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", lib.display());
    println!("cargo:rerun-if-env-changed=STARLIGHT_B200_ROOT");
    println!("cargo:rerun-if-changed={}", root.join("include/starlight_cuda.h").display());
}
