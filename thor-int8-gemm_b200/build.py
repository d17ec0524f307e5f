"""Build the C-ABI shared library libthor_int8_gemm_b200.so in place (sm_100a), and the
small CPython module _t8g_capsule that serves the `_C.cutlass_int8_dequant` proxy straight
from DLPack capsules (linked against the library, found next to it at run time).

    python thor-int8-gemm_b200/build.py [--force]

nvcc cross-compiles for sm_100a on a machine without a GPU; the resulting .so files sit next
to this file and are what the Python layer loads.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_NAME = "libthor_int8_gemm_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
SOURCES = [os.path.join(CSRC, "t8g.cu")]
# generated at build time: the SwiGLU kernels' sigmoid table (csrc/sigmoid_table.c)
GEN_DIR = os.path.join(HERE, "_build")
SIGMOID_GEN_SOURCE = os.path.join(CSRC, "sigmoid_table.c")
SIGMOID_TABLE = os.path.join(GEN_DIR, "sigmoid_table.inc")
DEPENDS = SOURCES + [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith(".cuh")] + [
    os.path.join(ROOT, "include", "thor_int8_gemm_b200.h"), SIGMOID_GEN_SOURCE]

EXT_SOURCE = os.path.join(CSRC, "capsule.c")
EXT_PATH = os.path.join(HERE, "_t8g_capsule" + sysconfig.get_config_var("EXT_SUFFIX"))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xptxas", "-v",
]


def nvcc_path() -> str:
    cand = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in cand:
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found (set NVCC or put CUDA's bin on PATH)")


def c_compiler() -> str:
    return os.environ.get("CC") or shutil.which("gcc") or "cc"


def generate_sigmoid_table(path: str = SIGMOID_TABLE) -> str:
    """Compile and run csrc/sigmoid_table.c, writing the table's initialiser list to `path`."""
    os.makedirs(os.path.dirname(path), exist_ok=True)
    exe = os.path.join(os.path.dirname(path), "sigmoid_table_gen")
    cmd = [c_compiler(), "-O2", "-std=c11", "-o", exe, SIGMOID_GEN_SOURCE, "-lm"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"compiling {os.path.basename(SIGMOID_GEN_SOURCE)} failed ({proc.returncode})")
    tmp = path + ".tmp"
    proc = subprocess.run([exe, tmp], capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"sigmoid table generator failed ({proc.returncode})")
    os.replace(tmp, path)
    return path


def up_to_date() -> bool:
    if not os.path.exists(LIB_PATH):
        return False
    t = os.path.getmtime(LIB_PATH)
    return all(os.path.getmtime(p) <= t for p in DEPENDS if os.path.exists(p))


def build_ext(force: bool = False) -> str:
    """Compile the capsule module (C, against Python's headers and the library)."""
    deps = [EXT_SOURCE, LIB_PATH, os.path.join(ROOT, "include", "thor_int8_gemm_b200.h")]
    if not force and os.path.exists(EXT_PATH) and all(os.path.getmtime(p) <= os.path.getmtime(EXT_PATH) for p in deps):
        return EXT_PATH
    cc = c_compiler()
    tmp = EXT_PATH + ".tmp"
    cmd = [cc, "-O2", "-shared", "-fPIC", "-std=c11", "-I" + sysconfig.get_paths()["include"], "-o", tmp, EXT_SOURCE,
           "-L" + HERE, "-lthor_int8_gemm_b200", "-Wl,-rpath,$ORIGIN"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"building {os.path.basename(EXT_PATH)} failed ({proc.returncode})")
    os.replace(tmp, EXT_PATH)
    return EXT_PATH


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library (and the capsule module) if any source is newer; return the
    library's path."""
    if not force and up_to_date():
        build_ext()
        return LIB_PATH
    generate_sigmoid_table()
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I" + GEN_DIR, "-o", tmp, *SOURCES]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    log_path = os.path.join(HERE, "build.log")
    with open(log_path, "w") as f:
        f.write(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"nvcc failed ({proc.returncode}); see {log_path}")
    os.replace(tmp, LIB_PATH)
    if verbose:
        sys.stdout.write(proc.stderr)
    build_ext(force=True)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
