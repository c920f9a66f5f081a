"""Build libeuclid_b200.so (the C-ABI engine) in-tree for sm_100a.

    python euclid-cuda_b200/build.py [--force] [-j N]

Each .cu under csrc/ is compiled separately (in parallel) with
`-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`, then linked into a
shared library next to this file.  The CUDA runtime is linked statically so the
library does not depend on which libcudart the host process (torch) loaded.
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libeuclid_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xcompiler", "-fvisibility=hidden"]
SOURCES = ["api.cu", "k_prep.cu", "k_tc.cu", "k_tc_fast.cu", "k_simt.cu", "k_recompute.cu", "k_centers.cu", "k_seed.cu",
           "k_cert.cu", "noalloc.cu"]


def _deps():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(HERE, "..", "include", "euclid_b200.h"))
    return max(os.path.getmtime(h) for h in hs)


def _compile(src, force, extra):
    s = os.path.join(CSRC, src)
    o = os.path.join(OBJ, src.replace(".cu", ".o"))
    if not force and os.path.exists(o) and os.path.getmtime(o) > max(os.path.getmtime(s), _deps()):
        return o, None
    cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", s, "-o", o]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return o, f"{' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
    return o, None


def build(force=False, jobs=None, verbose=False, extra=()):
    os.makedirs(OBJ, exist_ok=True)
    jobs = jobs or min(len(SOURCES), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(jobs) as ex:
        res = list(ex.map(lambda s: _compile(s, force, list(extra)), SOURCES))
    errs = [e for _, e in res if e]
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    objs = [o for o, _ in res]
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs, "-lrt", "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"[build] {LIB}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--ptxas-v", action="store_true", help="print register / smem usage")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    try:
        build(a.force or a.ptxas_v, a.j, True, extra)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
