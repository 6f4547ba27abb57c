"""Build the focal_b200 native libraries in-tree.

    python -m focal_b200.build          # both libraries
    python -m focal_b200.build --lib    # only the C-ABI library
    python -m focal_b200.build --timeline  # also the per-unit timeline variant

Outputs (next to this file, so they travel with the source tree):

* ``libfocal_b200.so`` — the CUDA kernels behind the C ABI of
  ``include/focal_b200.h``; nvcc, ``-gencode arch=compute_100a,code=sm_100a``,
  static CUDA runtime, no PyTorch dependency.
* ``_C.<abi>.so`` — the thin PyTorch extension (``csrc/torch_ext.cpp``) that
  validates tensors with the reference's messages and calls the C ABI.

Object files go to ``<repo>/_build`` (not committed).  Each step is skipped
when its output is newer than all of its inputs.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
ROOT = PKG.parent
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB = PKG / "libfocal_b200.so"
TIMELINE_LIB = PKG / "libfocal_b200_timeline.so"
CU_SOURCES = ["capi.cu", "w4a16_gemv.cu", "w4a16_tiles.cu", "gqa_decode.cu"]
HEADERS = ["common.cuh", "host_common.h", "w4a16_tiles.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "-Xptxas", "-warn-spills",
]


def _nvcc() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def _newer(out: Path, inputs) -> bool:
    if not out.exists():
        return False
    t = out.stat().st_mtime
    return all(Path(i).stat().st_mtime <= t for i in inputs)


def _run(cmd, log: Path | None = None):
    res = subprocess.run(cmd, capture_output=True, text=True)
    if log is not None:
        log.write_text(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"command failed ({res.returncode}): {' '.join(map(str, cmd))}\n"
                           f"{res.stdout}\n{res.stderr}")
    return res


def build_library(verbose: bool = False, timeline: bool = False) -> Path:
    """The C-ABI library; with `timeline`, its diagnostic variant
    libfocal_b200_timeline.so (-DFOCAL_TIMELINE: the GEMV kernel stamps SM
    cycles per CTA, sub-pipeline, unit and phase into shared memory and copies
    them to a buffer set with focal_tl_set), used only by bench.py --timeline."""
    bdir = BUILD / "timeline" if timeline else BUILD
    out = TIMELINE_LIB if timeline else LIB
    bdir.mkdir(parents=True, exist_ok=True)
    nvcc = _nvcc()
    deps = [CSRC / h for h in HEADERS] + [INCLUDE / "focal_b200.h"]
    extra = ["-DFOCAL_TIMELINE"] if timeline else []
    objs = []
    jobs = []
    for src in CU_SOURCES:
        obj = bdir / (Path(src).stem + ".o")
        objs.append(obj)
        if not _newer(obj, [CSRC / src] + deps):
            cmd = [nvcc, *NVCC_FLAGS, *extra, "-Xptxas", "-v", "-c", str(CSRC / src), "-o", str(obj)]
            jobs.append((cmd, bdir / (Path(src).stem + ".log")))
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for f in [ex.submit(_run, c, l) for c, l in jobs]:
            f.result()
    if not _newer(out, objs):
        _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static",
              "-Xlinker", f"-soname,{out.name}", "-o", str(out), *map(str, objs)])
    if verbose:
        for src in CU_SOURCES:
            log = bdir / (Path(src).stem + ".log")
            if log.exists():
                print(log.read_text())
    return out


def torch_ext_path() -> Path:
    return PKG / ("_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_torch_ext(verbose: bool = False) -> Path:
    """Compile csrc/torch_ext.cpp against the installed PyTorch (no CUDA code)."""
    import torch
    from torch.utils import cpp_extension as ce

    out = torch_ext_path()
    src = CSRC / "torch_ext.cpp"
    if _newer(out, [src, INCLUDE / "focal_b200.h", LIB]):
        return out
    BUILD.mkdir(exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    py_inc = sysconfig.get_paths()["include"]
    incs = ce.include_paths(device_type="cuda")
    libdirs = ce.library_paths(device_type="cuda")
    cxx = os.environ.get("CXX", "g++")
    cmd = [cxx, "-O3", "-std=c++17", "-fPIC", "-shared", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_API_INCLUDE_EXTENSION_H", "-DTORCH_EXTENSION_NAME=_C",
           f"-I{py_inc}", f"-I{INCLUDE}", *[f"-I{i}" for i in incs],
           str(src), "-o", str(out),
           *[f"-L{d}" for d in libdirs],
           f"-L{PKG}", "-lfocal_b200", "-Wl,-rpath,$ORIGIN",
           "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python"]
    _run(cmd, BUILD / "torch_ext.log")
    if verbose:
        print("built", out)
    return out


def build_all(verbose: bool = False):
    build_library(verbose)
    build_torch_ext(verbose)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--lib", action="store_true", help="only the C-ABI library")
    ap.add_argument("--timeline", action="store_true",
                    help="also the per-unit timeline variant of the C-ABI library (bench.py --timeline)")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    build_library(a.verbose)
    if a.timeline:
        build_library(a.verbose, timeline=True)
    if not a.lib:
        build_torch_ext(a.verbose)
    print("ok")


if __name__ == "__main__":
    sys.exit(main())
