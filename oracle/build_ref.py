"""Build recipe for the reference's own CUDA extensions (test infrastructure only).

This is part of the oracle: it compiles the UNMODIFIED sources of
inEXASCALE/euclid-cuda, where they lie in the read-only reference checkout,
into ``oracle/_ref/`` (git-ignored, but copied along with the rest of the tree).
The resulting modules are used by ``tests/golden/make_golden.py`` to
produce golden vectors on a B200 and by the GPU parity tests to compare against
the reference kernels directly.  Nothing in the product imports them.

Module name            sources (reference file names)
---------------------  ------------------------------------------------------
ref_euclidean_cuda     euclidean_cuda.cpp, euclidean_kernels.cu
ref_euclidean_mix      euclidean_cuda_mix.cpp, euclidean_kernels_mix.cu,
                       euclidean_kernels.cu (mix calls compute_norms_rowmajor_float
                       and form_mixed_and_list_rowmajor, euclidean_kernels_mix.cu:944,953)
ref_euclidean_tiled    euclidean_cuda_tiled.cpp, euclidean_kernels_tiled.cu,
                       euclidean_kernels_tiled_tc.cu
ref_euclidean_uniform  euclidean_cuda_uniform.cpp, euclidean_kernels_uniform.cu
ref_euclidean_advanced euclidean_cuda_advanced.cpp, euclidean_kernels_advanced.cu
ref_center_kernels     center_kernels.cu (its PYBIND11_MODULE is in the .cu, center_kernels.cu:252)

Usage:  python oracle/build_ref.py [--src DIR] [--only NAME ...]

The sources are read from --src, else $EUCLID_REFERENCE_SRC, else the reference checkout
beside this repository (../reference); without them the recipe skips itself.
"""
import argparse
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")

EXTENSIONS = {
    "ref_euclidean_cuda": ["euclidean_cuda.cpp", "euclidean_kernels.cu"],
    "ref_euclidean_mix": ["euclidean_cuda_mix.cpp", "euclidean_kernels_mix.cu", "euclidean_kernels.cu"],
    "ref_euclidean_tiled": ["euclidean_cuda_tiled.cpp", "euclidean_kernels_tiled.cu",
                            "euclidean_kernels_tiled_tc.cu"],
    "ref_euclidean_uniform": ["euclidean_cuda_uniform.cpp", "euclidean_kernels_uniform.cu"],
    "ref_euclidean_advanced": ["euclidean_cuda_advanced.cpp", "euclidean_kernels_advanced.cu"],
    "ref_center_kernels": ["center_kernels.cu"],
}


def built(name):
    return os.path.exists(os.path.join(OUT, name + ".so"))


def build_one(name, src_dir, verbose=False):
    from torch.utils import cpp_extension
    bdir = os.path.join(OUT, "build_" + name)
    os.makedirs(bdir, exist_ok=True)
    sources = [os.path.join(src_dir, s) for s in EXTENSIONS[name]]
    t0 = time.time()
    cpp_extension.load(
        name=name,
        sources=sources,
        build_directory=bdir,
        extra_include_paths=[src_dir],
        extra_cflags=["-O3"],
        extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"],
        extra_ldflags=["-lcublas"],
        verbose=verbose,
        is_python_module=True,
    )
    so = os.path.join(bdir, name + ".so")
    os.replace(so, os.path.join(OUT, name + ".so"))
    print(f"[build_ref] {name}: {time.time() - t0:.0f}s", flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=os.environ.get("EUCLID_REFERENCE_SRC",
                                                   os.path.join(os.path.dirname(HERE), "..", "reference")))
    ap.add_argument("--only", nargs="*")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    if not os.path.isdir(a.src):
        print(f"[build_ref] reference sources not found at {a.src}; skipping")
        return 0
    os.makedirs(OUT, exist_ok=True)
    # torch's extension builder refuses to run without an arch list when no GPU is visible
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    names = a.only or list(EXTENSIONS)
    for n in names:
        if built(n) and not a.force:
            print(f"[build_ref] {n}: up to date")
            continue
        build_one(n, a.src, a.verbose)
    return 0


if __name__ == "__main__":
    sys.exit(main())
