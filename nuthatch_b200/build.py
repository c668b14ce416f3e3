"""In-tree build of the native libraries.

    python -m nuthatch_b200.build                # product + synthetic-model writer
    python -m nuthatch_b200.build --all          # also the checker (oracle/, oracle/_ref)
    python -m nuthatch_b200.build --phase-trace  # also the phase-timestamp diagnostic library

Outputs (git-ignored, shipped with the tree):
    nuthatch_b200/lib/libnuthatch_b200.so              kernels (sm_100a) + host C++ + C ABI
    nuthatch_b200/lib/libnh_synth.so                   seeded synthetic GGUF writer
    nuthatch_b200/lib/libnuthatch_b200_phase_trace.so  the same with per-CTA phase timestamps
                                                       (python -m nuthatch_b200.phase_trace)
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
OBJ = LIB / "obj"
INCLUDE = ROOT / "include"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
                     f"-I{INCLUDE}", f"-I{CSRC}"]
CXX_FLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wextra", f"-I{INCLUDE}", f"-I{CSRC}",
             f"-I{CUDA_HOME / 'include'}"]


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")


def _digest(paths: list[Path], extra: str) -> str:
    h = hashlib.sha256(extra.encode())
    for p in sorted(paths):
        h.update(str(p).encode())
        h.update(p.read_bytes())
    return h.hexdigest()


def _headers() -> list[Path]:
    return sorted(list(INCLUDE.rglob("*.h")) + list(CSRC.rglob("*.h")) + list(CSRC.rglob("*.cuh")) +
                  list(CSRC.rglob("*.inc")))


def build_product(verbose: bool = False, phase_trace: bool = False) -> Path:
    """Compiles kernels/*.cu (nvcc, sm_100a) and host/*.cc, links the shared library
    (with phase_trace: the diagnostic variant, NH_PHASE_TRACE defined)."""
    name = "libnuthatch_b200_phase_trace" if phase_trace else "libnuthatch_b200"
    obj = OBJ / "phase_trace" if phase_trace else OBJ
    LIB.mkdir(parents=True, exist_ok=True)
    obj.mkdir(parents=True, exist_ok=True)
    out = LIB / f"{name}.so"
    nvcc_flags = NVCC_FLAGS + (["-DNH_PHASE_TRACE"] if phase_trace else [])
    cu = sorted((CSRC / "kernels").glob("*.cu"))
    cc = sorted((CSRC / "host").glob("*.cc"))
    stamp = LIB / f"{name}.stamp"
    digest = _digest(cu + cc + _headers(), " ".join(nvcc_flags + CXX_FLAGS))
    if out.exists() and stamp.exists() and stamp.read_text() == digest:
        return out
    jobs = []
    for src in cu:
        jobs.append([NVCC, *nvcc_flags, "-c", str(src), "-o", str(obj / (src.stem + ".cu.o"))])
    for src in cc:
        jobs.append(["g++", *CXX_FLAGS, "-c", str(src), "-o", str(obj / (src.stem + ".cc.o"))])
    with cf.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 4))) as ex:
        list(ex.map(_run, jobs))
    objs = [str(obj / (s.stem + ".cu.o")) for s in cu] + [str(obj / (s.stem + ".cc.o")) for s in cc]
    _run([NVCC, *ARCH, "-shared", "-o", str(out), *objs, "-lcudart_static", "-lrt", "-ldl", "-lpthread"])
    stamp.write_text(digest)
    if verbose:
        print(f"built {out}")
    return out


def build_synth(verbose: bool = False) -> Path:
    LIB.mkdir(parents=True, exist_ok=True)
    src = CSRC / "synth" / "synth_gguf.cc"
    out = LIB / "libnh_synth.so"
    stamp = LIB / "libnh_synth.stamp"
    digest = _digest([src], "synth")
    if out.exists() and stamp.exists() and stamp.read_text() == digest:
        return out
    _run(["g++", "-O3", "-std=c++17", "-fPIC", "-shared", "-pthread", "-Wall", "-Wextra", str(src), "-o", str(out)])
    stamp.write_text(digest)
    if verbose:
        print(f"built {out}")
    return out


def build_checker(verbose: bool = False) -> None:
    """The oracle (always) and oracle/_ref (only where the reference tree exists)."""
    # The same g++ as the product (libstdc++ linked as a shared library): a
    # checker with its own static copy misbehaves once the process has also
    # loaded the shared libstdc++ (numpy and torch do).
    _run(["make", "-s", "-C", str(ROOT / "oracle"), "ORACLE_CXX=g++"])
    # oracle/_ref is built only where the reference checkout is named by the
    # NUTHATCH_REFERENCE environment variable; the tests that use it skip
    # when it has not been built.
    ref_env = os.environ.get("NUTHATCH_REFERENCE", "")
    ref = Path(ref_env) if ref_env else None
    if ref is not None and (ref / "src" / "cache" / "cache_policy.cc").exists():
        _run(["make", "-s", "-C", str(ROOT / "oracle"), "ref", f"REF={ref}", "ORACLE_CXX=g++"])
    if verbose:
        print("built oracle")


def build_all(verbose: bool = False) -> None:
    build_synth(verbose)
    build_product(verbose)
    build_checker(verbose)


if __name__ == "__main__":
    if "--all" in sys.argv:
        build_all(verbose=True)
    else:
        build_synth(verbose=True)
        build_product(verbose=True)
    if "--phase-trace" in sys.argv:
        build_product(verbose=True, phase_trace=True)
