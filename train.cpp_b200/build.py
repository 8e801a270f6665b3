"""Build step for the native libraries of train.cpp_b200 (run by __graft_entry__.build()).

  lib/libtrc_cuda.so          the sm_100a kernels + C ABI (include/trc_cuda.h); needs only nvcc
  lib/libtrc_cuda_backend.so  the C++ Device/BufferType/Buffer drop-in for train.cpp; compiled
                              against train.cpp's public headers, so it is only built where the
                              train.cpp source tree is available (TRC_REFERENCE_DIR)

Everything is built in-tree so the shared objects travel with the repository snapshot.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CU_SOURCES = ["capi.cu", "runtime.cu", "dequant.cu", "elementwise.cu", "mul_mat_simt.cu", "gemm_tf32x3.cu",
              "static_staging.cu", "train_ops.cu", "probe_tc.cu"]


def _run(cmd: list[str], log: Path | None = None) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if log is not None:
        log.write_text(res.stdout + res.stderr)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_cuda(force: bool = False) -> Path:
    """Compile libtrc_cuda.so for sm_100a (relocatable device code, static cudart)."""
    LIB.mkdir(exist_ok=True)
    out = LIB / "libtrc_cuda.so"
    deps = [CSRC / s for s in CU_SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps += [ROOT / "include" / "trc_cuda.h", ROOT / "include" / "trc_cuda_runtime.h"]
    if not force and not _stale(out, deps):
        return out
    cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-rdc=true", "-shared",
           "-Xcompiler", "-fPIC", "-Xptxas", "-v", f"-I{ROOT / 'include'}",
           "-o", str(out), *[str(CSRC / s) for s in CU_SOURCES]]
    _run(cmd, LIB / "libtrc_cuda.build.log")
    return out


def reference_dir() -> Path | None:
    """The train.cpp source tree: $TRC_REFERENCE_DIR, else a checkout named `reference` beside this
    repository. None (with a note on stderr) when neither holds train.cpp's headers; the parts that
    compile against them (the C++ backend, the reference's CPU library, the drop-in test program)
    are then skipped and their prebuilt files, if any, are used."""
    env = os.environ.get("TRC_REFERENCE_DIR")
    d = Path(env) if env else ROOT.parent / "reference"
    if (d / "include" / "traincpp" / "trc_backend.h").exists():
        return d
    sys.stderr.write(f"build: no train.cpp source tree at {d} (set TRC_REFERENCE_DIR); "
                     "skipping the parts built against it\n")
    return None


def build_backend(force: bool = False) -> Path | None:
    """Compile the C++ drop-in backend against train.cpp's headers (skipped without them)."""
    ref = reference_dir()
    out = LIB / "libtrc_cuda_backend.so"
    if ref is None:
        return out if out.exists() else None
    cuda_lib = build_cuda()
    src = PKG / "backend" / "trc_cuda_backend.cpp"
    deps = [src, PKG / "backend" / "trc_cuda_backend.h", ROOT / "include" / "trc_cuda.h",
            ROOT / "include" / "trc_cuda_runtime.h", cuda_lib]
    if not force and not _stale(out, deps):
        return out
    cuda_inc = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"
    cmd = ["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-Wall", "-Wextra", "-Wno-unused-parameter",
           f"-I{ref / 'include'}", f"-I{ROOT / 'include'}", f"-I{cuda_inc}",
           "-o", str(out), str(src), f"-L{LIB}", "-ltrc_cuda", "-Wl,-rpath,$ORIGIN"]
    _run(cmd)
    return out


if __name__ == "__main__":
    print(build_cuda(force="--force" in sys.argv))
    print(build_backend(force="--force" in sys.argv))
