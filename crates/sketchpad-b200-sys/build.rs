//! Builds libsketchpad_b200.so from sketchpad_b200/csrc/*.cu with nvcc (sm_100a only) and links
//! it.  Set SKETCHPAD_B200_LIB_DIR to link a library built elsewhere instead
//! (`python -m sketchpad_b200.build` writes it to sketchpad_b200/).
use std::env;
use std::path::{Path, PathBuf};
use std::process::Command;

fn main() {
    println!("cargo:rerun-if-env-changed=SKETCHPAD_B200_LIB_DIR");
    println!("cargo:rerun-if-env-changed=NVCC");
    if let Ok(dir) = env::var("SKETCHPAD_B200_LIB_DIR") {
        println!("cargo:rustc-link-search=native={dir}");
        println!("cargo:rustc-link-lib=dylib=sketchpad_b200");
        return;
    }
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    let root = manifest.join("../..").canonicalize().expect("repository root");
    let csrc = root.join("sketchpad_b200/csrc");
    let include = root.join("include");
    let out = PathBuf::from(env::var("OUT_DIR").unwrap());
    let nvcc = env::var("NVCC").unwrap_or_else(|_| "/usr/local/cuda/bin/nvcc".to_string());
    let arch = ["-gencode", "arch=compute_100a,code=sm_100a"];
    let mut objs = Vec::new();
    let mut sources: Vec<PathBuf> = std::fs::read_dir(&csrc)
        .expect("sketchpad_b200/csrc")
        .filter_map(|e| e.ok().map(|e| e.path()))
        .filter(|p| p.extension().map_or(false, |x| x == "cu"))
        .collect();
    sources.sort();
    for src in &sources {
        println!("cargo:rerun-if-changed={}", src.display());
        let obj = out.join(Path::new(src.file_stem().unwrap()).with_extension("o"));
        let ok = Command::new(&nvcc)
            .args(arch)
            .args(["-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC",
                   "--expt-relaxed-constexpr"])
            .arg(format!("-I{}", include.display()))
            .arg("-c").arg(src).arg("-o").arg(&obj)
            .status()
            .expect("nvcc");
        assert!(ok.success(), "nvcc failed for {}", src.display());
        objs.push(obj);
    }
    for h in std::fs::read_dir(&csrc).unwrap().filter_map(|e| e.ok().map(|e| e.path())) {
        if h.extension().map_or(false, |x| x == "cuh") {
            println!("cargo:rerun-if-changed={}", h.display());
        }
    }
    println!("cargo:rerun-if-changed={}", include.join("sketchpad_b200.h").display());
    let lib = out.join("libsketchpad_b200.so");
    let ok = Command::new(&nvcc)
        .args(arch)
        .args(["-shared", "-rdc=true", "-Xcompiler", "-fPIC", "-o"])
        .arg(&lib)
        .args(&objs)
        .status()
        .expect("nvcc link");
    assert!(ok.success(), "nvcc device link failed");
    println!("cargo:rustc-link-search=native={}", out.display());
    println!("cargo:rustc-link-lib=dylib=sketchpad_b200");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", out.display());
}
