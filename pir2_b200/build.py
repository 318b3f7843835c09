"""Builds libpir2b.so in-tree with nvcc for sm_100a.

`python -m pir2_b200.build` compiles pir2_b200/csrc/pir2b.cu (one translation
unit that includes every kernel and the C ABI) into pir2_b200/libpir2b.so.
The build is skipped when the library is newer than every source file.
"""

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ROOT = os.path.dirname(HERE)
OUTPUT = os.path.join(HERE, "libpir2b.so")

NVCC_FLAGS = [
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-shared",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-O2",
]


def sources():
    files = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))]
    files.append(os.path.join(ROOT, "include", "pir2b.h"))
    return [f for f in files if f.endswith((".cu", ".cuh", ".h"))]


def nvcc():
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(found):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build")
    return found


def up_to_date():
    if not os.path.exists(OUTPUT):
        return False
    built = os.path.getmtime(OUTPUT)
    return all(os.path.getmtime(f) <= built for f in sources())


def build(force=False, verbose=False):
    if not force and up_to_date():
        return OUTPUT
    command = [nvcc(), *NVCC_FLAGS, "-o", OUTPUT + ".tmp", os.path.join(CSRC, "pir2b.cu")]
    if verbose:
        command.insert(1, "-Xptxas=-v")
        print(" ".join(command))
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{result.stdout}\n{result.stderr}")
    if verbose:
        print(result.stderr)
    os.replace(OUTPUT + ".tmp", OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
