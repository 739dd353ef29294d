"""Build recipe for the sm_100a shared library (``libcpgemm.so``), built in-tree.

The library is one translation unit (``csrc/capi.cu``) holding the C ABI of ``include/cpgemm.h``,
the tcgen05 GEMM kernels and the scheduler/FastDivmod device helpers.  It links the CUDA runtime
statically and reaches ``cuTensorMapEncodeTiled`` through the runtime's driver entry-point
query, so it needs no link against ``libcuda``.
"""
import os
import shutil
import subprocess

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
LIB_NAME = "libcpgemm.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

SOURCES = [os.path.join(CSRC, "capi.cu")]
# Every source and header of csrc/ and the public header: a change to any of them rebuilds.
DEPENDS = SOURCES + sorted(
    os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))
) + [os.path.join(INCLUDE, "cpgemm.h")]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put the CUDA toolkit on PATH")


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(s) > t for s in DEPENDS if os.path.exists(s))


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile ``libcpgemm.so`` next to this file (skipped when it is newer than its sources)."""
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", *SOURCES, "-o", tmp]
    if verbose:
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force=True, verbose=True))
