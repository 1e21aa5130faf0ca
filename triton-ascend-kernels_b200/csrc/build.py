"""Build libtak_b200.so (all CUDA kernels + the C ABI) for sm_100a, in-tree.

    python triton-ascend-kernels_b200/csrc/build.py [-j N] [--clean]

Objects go to csrc/_build/, the library to triton-ascend-kernels_b200/lib/.
Incremental: a .cu is recompiled when it or any header in csrc/ or include/
is newer than its object.
"""

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
BUILD = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIB_DIR, "libtak_b200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-rdc=true", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                "-I" + os.path.join(REPO, "include"), "-Xptxas", "-warn-spills"]


def _newest_header():
    hs = glob.glob(os.path.join(HERE, "*.cuh")) + glob.glob(os.path.join(HERE, "*.h")) + \
        glob.glob(os.path.join(REPO, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src, verbose):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), _newest_header()):
        return obj, None
    cmd = [NVCC] + FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f"$ {' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
    if verbose:
        sys.stderr.write(r.stderr)
    return obj, None


def build(jobs=None, verbose=False, clean=False):
    if clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(HERE, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    errs = [e for _, e in results if e]
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    objs = [o for o, _ in results]
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-rdc=true", "-Xcompiler", "-fPIC", "-o", LIB] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n$ {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", action="store_true", help="print ptxas register / spill report")
    ap.add_argument("--clean", action="store_true")
    args = ap.parse_args()
    print(build(args.j, args.v, args.clean))
