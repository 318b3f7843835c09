"""Builds the reference's own CUTLASS-free CUDA kernels of this path for
sm_100a into oracle/_ref/ (test infrastructure: only the GPU parity tests and
bench.py's reference comparisons load them; the product never does).

The reference compiles these translation units as torch extensions through
its own build system (coexecution/kernels/build.py, ampere_ada/*.py).  This
recipe compiles the same source files where they lie, with the flags that
build system gives each of them and the B200 architecture:

  * coexecution/kernels/ampere_ada/csrc/integer_dispatch.cu (+
    common/source_identity.cpp): `pir2_integer_dispatch::prepare`, the
    native per-row activation pack the reference dispatches to on a CUDA
    device (build.py:23-29: `--fmad=false --ftz=false`, no CUTLASS);
  * coexecution/kernels/ampere_ada/csrc/int4_gemv.cu:
    `pir2_int4_gemv::gemv`, the exact single-row INT4 GEMV (no CUTLASS).

The CUTLASS-based reference kernels (integer_gemm.cu, the FP4/FP8 CUTLASS
linears) need the CUTLASS submodule, which is absent: not built.

usage: python -m oracle.ref_build [reference_root]
Writes oracle/_ref/<name>/<name>.so; skips a library that is newer than its
sources.  Requires the reference checkout (it is not read at run time).
"""

import hashlib
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
ARCH = "-gencode=arch=compute_100a,code=sm_100a"

# name -> (sources relative to coexecution/kernels, nvcc flags, defines)
TARGETS = {
    "ref_integer_dispatch": (
        ("ampere_ada/csrc/integer_dispatch.cu", "common/source_identity.cpp"),
        ("--fmad=false", "--ftz=false"),
        {"PIR2_KERNEL_NAMESPACE": "pir2_integer_dispatch"},
    ),
    "ref_int4_gemv": (
        ("ampere_ada/csrc/int4_gemv.cu",),
        ("--ftz=false",),
        {},
    ),
}


def library_path(name):
    return os.path.join(OUT, name, name + ".so")


def _identity(paths):
    h = hashlib.sha256()
    for p in paths:
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def build(reference_root, verbose=False):
    """Compiles every target whose library is missing or older than its
    sources.  Returns {name: path}."""
    from torch.utils.cpp_extension import load

    kernels = os.path.join(reference_root, "coexecution", "kernels")
    built = {}
    for name, (sources, flags, defines) in TARGETS.items():
        paths = [os.path.join(kernels, s) for s in sources]
        out = library_path(name)
        if os.path.exists(out) and all(os.path.getmtime(out) >= os.path.getmtime(p) for p in paths):
            built[name] = out
            continue
        ident = _identity(paths)
        defs = dict(defines)
        defs.update({
            "PIR2_BUILD_SOURCE_ID": f'\\"{ident}\\"',
            "PIR2_GEMV_SOURCE_ID": f'\\"{ident}\\"',
        })
        dflags = [f"-D{k}={v}" for k, v in defs.items()]
        build_dir = os.path.join(OUT, name)
        os.makedirs(build_dir, exist_ok=True)
        load(
            name=name,
            sources=paths,
            extra_cflags=["-O3", "-std=c++17", *dflags],
            extra_cuda_cflags=["-O3", "-std=c++17", *flags, ARCH, *dflags],
            build_directory=build_dir,
            is_python_module=False,
            verbose=verbose,
        )
        built[name] = out
    return built


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PIR2_REFERENCE", "")
    if not root or not os.path.isdir(root):
        raise SystemExit("usage: python -m oracle.ref_build <reference checkout>")
    for name, path in build(root, verbose=True).items():
        print(name, path)
