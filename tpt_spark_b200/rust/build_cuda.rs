// build_cuda.rs -- the nvcc step of tpt-spark's src-tauri/build.rs under the engine-cuda
// feature (the reference's build.rs:1-3 only calls tauri_build::build()).
//
// Not compiled here: there is no cargo or rustc on the machines this repository is built and
// tested on.  It runs the same compiler and flags as tpt_spark_b200/_build.py, which builds
// and tests libtptc here.
//
// Use from build.rs:
//
//     mod build_cuda;
//     fn main() {
//         #[cfg(feature = "engine-cuda")]
//         build_cuda::compile_libtptc("../tpt_spark_b200/csrc", "../include");
//         tauri_build::build()
//     }

use std::path::Path;
use std::process::Command;

/// The flags tpt_spark_b200/_build.py passes (sm_100a only; the runtime linked statically).
const NVCC_FLAGS: &[&str] = &[
    "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr", "-DTPTC_BUILD",
];

fn nvcc() -> String {
    std::env::var("NVCC").unwrap_or_else(|_| "nvcc".to_string())
}

/// Compiles every .cu / .cpp of `csrc` for sm_100a into OUT_DIR/libtptc.so and tells cargo
/// to link it.  NCCL is opened at run time (dlopen), so no NCCL link flag is needed.
pub fn compile_libtptc(csrc: &str, include: &str) {
    let out = std::env::var("OUT_DIR").expect("OUT_DIR");
    let mut sources: Vec<_> = std::fs::read_dir(csrc)
        .expect("csrc")
        .filter_map(|e| e.ok().map(|e| e.path()))
        .filter(|p| matches!(p.extension().and_then(|x| x.to_str()), Some("cu") | Some("cpp")))
        .collect();
    sources.sort();
    let mut objects = Vec::new();
    for src in &sources {
        let obj = Path::new(&out).join(format!("{}.o", src.file_name().unwrap().to_string_lossy()));
        let mut cmd = Command::new(nvcc());
        cmd.args(NVCC_FLAGS).arg(format!("-I{include}")).arg(format!("-I{csrc}"));
        if src.extension().and_then(|x| x.to_str()) == Some("cpp") {
            cmd.args(["-x", "cu"]); // the host files share the .cuh helpers
        }
        let ok = cmd.arg("-c").arg(src).arg("-o").arg(&obj).status().expect("nvcc").success();
        assert!(ok, "nvcc failed on {}", src.display());
        objects.push(obj);
        println!("cargo:rerun-if-changed={}", src.display());
    }
    let so = Path::new(&out).join("libtptc.so");
    let ok = Command::new(nvcc())
        .args(["-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static", "-o"])
        .arg(&so)
        .args(&objects)
        .args(["-ldl", "-lpthread", "-lrt"])
        .status()
        .expect("nvcc link")
        .success();
    assert!(ok, "linking libtptc.so failed");
    println!("cargo:rerun-if-changed={include}/tptc.h");
    println!("cargo:rustc-link-search=native={out}");
    println!("cargo:rustc-link-lib=dylib=tptc");
}
