"""Builds the native libraries of quanta.cpp_b200 in-tree (sm_100a only).

    python quanta.cpp_b200/build.py          # or __graft_entry__.build()
    python quanta.cpp_b200/build.py --stamps # the phase-timed library (lib_stamps/, -DQNT_PHASE_STAMPS) for timeline.py

Outputs (git-ignored, shipped with the repository snapshot):
    quanta.cpp_b200/lib/libquanta_b200.so   CUDA kernels + engine + the C ABI of include/quanta_b200.h
    quanta.cpp_b200/lib/libqnt_synth.so     seeded random-init .qnt writer
    quanta.cpp_b200/lib/quanta_b200         command-line driver (selftest / gen / bench / checkbatch / checkhead / run)
Objects go to quanta.cpp_b200/_build/.  Rebuilds only what changed (source or header mtimes).
"""
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3", f"-I{CSRC}", f"-I{ROOT / 'include'}",
                  "--expt-relaxed-constexpr"]

# CUDA translation units (host files that include device headers are compiled as CUDA too)
CU_SOURCES = ["ops.cu", "layer_kernels.cu", "attention.cu", "head_kernels.cu", "sampler_wide.cu", "nll.cu", "gemm_tc.cu", "engine.cpp", "capi.cpp", "sampler.cpp", "sampler_noalloc.cpp"]
HOST_SOURCES = ["qnt_file.cpp", "exp_table.cpp", "tokenizer.cpp", "device_layout.cpp"]


def _newer(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _headers():
    return [p for p in CSRC.rglob("*") if p.suffix in (".h", ".cuh")] + [ROOT / "include" / "quanta_b200.h"]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed: " + " ".join(map(str, cmd)) + "\n" + r.stdout + r.stderr)
    return r


def build(verbose: bool = False, jobs: int = 0, stamps: bool = False) -> None:
    build_dir, lib_dir = (PKG / "_build_stamps", PKG / "lib_stamps") if stamps else (BUILD, LIB)
    build_dir.mkdir(exist_ok=True)
    lib_dir.mkdir(exist_ok=True)
    nvflags = NVFLAGS + (["-DQNT_PHASE_STAMPS"] if stamps else [])
    hdrs = _headers()
    todo = []
    objs = []
    for src in CU_SOURCES:
        s = CSRC / src
        if not s.exists():
            continue
        o = build_dir / (src + ".o")
        objs.append(o)
        if _newer(o, [s] + hdrs):
            cmd = [NVCC] + nvflags + (["-x", "cu"] if s.suffix == ".cpp" else []) + ["-c", str(s), "-o", str(o)]
            todo.append(cmd)
    for src in HOST_SOURCES:
        s = CSRC / src
        o = build_dir / (src + ".o")
        objs.append(o)
        if _newer(o, [s] + hdrs):
            todo.append(["g++", "-O3", "-std=c++17", "-fPIC", f"-I{CSRC}", "-c", str(s), "-o", str(o)])
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        for r in ex.map(_run, todo):
            if verbose and (r.stdout or r.stderr):
                print(r.stdout + r.stderr)
    so = lib_dir / "libquanta_b200.so"
    if _newer(so, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", str(so)] + [str(o) for o in objs] + ["-lpthread"])
    if stamps:
        return
    synth = LIB / "libqnt_synth.so"
    ssrc = CSRC / "synth" / "qnt_synth.cpp"
    if _newer(synth, [ssrc, CSRC / "synth" / "qnt_synth.h"]):
        _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-march=x86-64-v3", "-o", str(synth), str(ssrc), "-pthread"])
    cli_src = CSRC / "cli" / "main.cpp"
    cli = LIB / "quanta_b200"
    if cli_src.exists() and _newer(cli, [cli_src, so] + hdrs):
        _run(["g++", "-O2", "-std=c++17", f"-I{ROOT / 'include'}", "-o", str(cli), str(cli_src), f"-L{LIB}", "-lquanta_b200",
              f"-Wl,-rpath,$ORIGIN", "-pthread"])


if __name__ == "__main__":
    st = "--stamps" in sys.argv
    build(verbose="-v" in sys.argv, stamps=st)
    print("built", PKG / "lib_stamps" if st else LIB)
