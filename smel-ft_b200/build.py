"""Build libsmelb.so (all CUDA sources of smelb) for sm_100a, in-tree, with nvcc.

Usage: python smel-ft_b200/build.py [--force] [--jobs N]
The library lands next to the Python package (smel-ft_b200/smelb/libsmelb.so) so it travels with the source tree.
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "smelb", "libsmelb.so")
SOURCES = ["host.cu", "kernels.cu", "gemm.cu", "ops.cu", "ep.cu", "gemv.cu", "dense.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fPIC,-O2", "-I" + os.path.join(HERE, "..", "include")]


def _deps_mtime():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [os.path.join(HERE, "..", "include", "smelb.h")]
    return max(os.path.getmtime(f) for f in files if os.path.isfile(f))


def build(force=False, jobs=4, verbose=False, extra=(), out=OUT, build_dir=BUILD):
    """Compile every source to an object and link the shared library. Returns the library path."""
    os.makedirs(build_dir, exist_ok=True)
    if not force and os.path.exists(out) and os.path.getmtime(out) >= _deps_mtime():
        return out

    def compile_one(src):
        obj = os.path.join(build_dir, src.replace(".cu", ".o"))
        cmd = [NVCC, *FLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = out + ".tmp"
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=4)
    ap.add_argument("--ptxas-v", action="store_true", help="print register / spill / smem usage")
    a = ap.parse_args()
    extra = ("-Xptxas", "-v") if a.ptxas_v else ()
    print(build(force=a.force or a.ptxas_v, jobs=a.jobs, verbose=a.ptxas_v, extra=extra))
    sys.exit(0)
