"""Build libtreesa_b200.so in-tree for sm_100a.

    python -m treesa_gpu_b200.build [--force]

Steps: (1) compile and run csrc/gen_expf_fixups.cpp, which tabulates the negative floats where the host
libm's expf differs from the device's correctly rounded expf (csrc/gen/expf_fixups.h); (2) nvcc the
kernels, the host scheduler and the NCCL layer into one shared library next to this file.
"""
import hashlib
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
GEN = os.path.join(CSRC, "gen")
LIB = os.path.join(HERE, "libtreesa_b200.so")
ROOT = os.path.dirname(HERE)
SOURCES = ["tsa_kernels.cu", "tsa_host.cpp", "tsa_comm.cpp", "tsa_resample_noalloc.cu", "tsa_spectral.cu"]
HEADERS = ["tsa_core.h", "tsa_exp_table.h", "tsa_kernels.cuh", "tsa_comm.h"]
ARCH = "-gencode=arch=compute_100a,code=sm_100a"


def _cxx():
    return "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else (shutil.which("g++") or "g++")


def _nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _run(cmd, log=None):
    p = subprocess.run(cmd, capture_output=True, text=True)
    if log:
        with open(log, "w") as f:
            f.write(" ".join(cmd) + "\n" + p.stdout + p.stderr)
    if p.returncode != 0:
        raise RuntimeError(f"command failed ({p.returncode}): {' '.join(cmd)}\n{p.stdout[-4000:]}{p.stderr[-4000:]}")
    return p


def _digest(paths):
    h = hashlib.sha256()
    for p in paths:
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


def gen_fixups(force=False):
    os.makedirs(GEN, exist_ok=True)
    out = os.path.join(GEN, "expf_fixups.h")
    exe = os.path.join(GEN, "gen_expf_fixups")
    src = [os.path.join(CSRC, f) for f in ("gen_expf_fixups.cpp", "tsa_core.h", "tsa_exp_table.h")]
    stamp = os.path.join(GEN, "fixups.stamp")
    dig = _digest(src)
    if not force and os.path.exists(out) and os.path.exists(stamp) and open(stamp).read() == dig:
        return out
    _run([_cxx(), "-O2", "-std=c++17", "-fopenmp", "-ffp-contract=off", "-o", exe,
          os.path.join(CSRC, "gen_expf_fixups.cpp"), "-lm"])
    _run([exe, out])
    with open(stamp, "w") as f:
        f.write(dig)
    return out


def build(force=False, verbose=False):
    """Build the library (no-op when sources are unchanged).  Returns the library path."""
    fix = gen_fixups(force)
    srcs = [os.path.join(CSRC, f) for f in SOURCES]
    deps = srcs + [os.path.join(CSRC, f) for f in HEADERS] + [os.path.join(ROOT, "include", "treesa_b200.h"), fix,
                                                              os.path.abspath(__file__)]
    stamp = os.path.join(GEN, "lib.stamp")
    dig = _digest(deps)
    if not force and os.path.exists(LIB) and os.path.exists(stamp) and open(stamp).read() == dig:
        return LIB
    tmp = LIB + ".tmp"
    cmd = [_nvcc(), ARCH, "-O3", "-lineinfo", "-std=c++17", "-ccbin", _cxx(), "-Xcompiler", "-fPIC,-fopenmp,-O3",
           "-Xcompiler", "-ffp-contract=off", "-Xptxas", "-v", "-shared", "-o", tmp] + srcs + ["-lgomp", "-ldl"]
    _run(cmd, log=os.path.join(GEN, "ptxas.log"))
    os.replace(tmp, LIB)
    with open(stamp, "w") as f:
        f.write(dig)
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
