"""Builds libesm_b200.so in-tree (esm-cpp_b200/esm_b200/libesm_b200.so).

Device translation units (csrc/*.cu) are compiled by nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a); the C++ host (csrc/host/*.cpp) by
g++ with the reference's release flags (-O3 -fno-math-errno), so host-side
float code such as the RoPE tables rounds exactly like the reference's.
The CUDA runtime is linked statically: the library needs only the driver.

    python esm-cpp_b200/build.py [--force] [--jobs N]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
OUT_SO = PKG_ROOT / "esm_b200" / "libesm_b200.so"
OBJ = PKG_ROOT / "_build"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = GENCODE + [
    "-O3", "-std=c++17", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC",
    "-Xptxas", "-warn-spills", f"-I{CSRC}", f"-I{REPO / 'include'}",
]
CXX = shutil.which("g++") or "g++"
CXX_FLAGS = [
    "-O3", "-fno-math-errno", "-std=c++20", "-fPIC", "-Wall", "-Wno-unused-function",
    f"-I{CSRC}", f"-I{CSRC / 'host'}", f"-I{REPO / 'include'}", f"-I{CUDA_HOME / 'include'}",
]


def _sources():
    cu = sorted(CSRC.glob("*.cu"))
    cpp = sorted((CSRC / "host").glob("*.cpp"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted((CSRC / "host").glob("*.h")) + [REPO / "include" / "esm_b200.h"]
    return cu, cpp, headers


def _compile(src: Path, force: bool, newest_header: float) -> Path:
    obj = OBJ / (src.stem + (".cu.o" if src.suffix == ".cu" else ".o"))
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header):
        return obj
    if src.suffix == ".cu":
        cmd = [NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    else:
        cmd = [CXX, *CXX_FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = True) -> Path:
    """Compiles and links the library; returns the path of the .so."""
    OBJ.mkdir(exist_ok=True)
    cu, cpp, headers = _sources()
    newest_header = max(h.stat().st_mtime for h in headers)
    srcs = cu + cpp
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, newest_header), srcs))
    newest_obj = max(o.stat().st_mtime for o in objs)
    if force or not OUT_SO.exists() or OUT_SO.stat().st_mtime < newest_obj:
        cmd = [CXX, "-shared", "-o", str(OUT_SO), *map(str, objs),
               f"-L{CUDA_HOME / 'lib64'}", "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"built {OUT_SO.relative_to(REPO)}")
    return OUT_SO


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    a = ap.parse_args(argv)
    build(force=a.force, jobs=a.jobs)
    return 0


if __name__ == "__main__":
    sys.exit(main())
