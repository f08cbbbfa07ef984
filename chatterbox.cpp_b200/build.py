"""Build recipe for libt3b200.so (sm_100a) and its generated exp table.

python chatterbox.cpp_b200/build.py            # builds in place
The generated fix-up table and objects go to chatterbox.cpp_b200/_build/.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libt3b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd):
    print("+", " ".join(cmd), flush=True)
    subprocess.check_call(cmd)


def _newer(target, deps):
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def build(force=False, verbose_ptxas=False):
    os.makedirs(BUILD, exist_ok=True)
    gen = os.path.join(BUILD, "gen_expf_fixup")
    inc = os.path.join(BUILD, "expf_fixup.inc")
    gsrc = [os.path.join(CSRC, "gen_expf_fixup.cpp"), os.path.join(CSRC, "t3_expf.h")]
    if force or not _newer(gen, gsrc):
        _run(["g++", "-O2", "-std=c++17", "-ffp-contract=off", "-I", CSRC, gsrc[0], "-o", gen, "-lpthread"])
    if force or not _newer(inc, [gen]):
        _run([gen, inc])
    srcs = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))]
    srcs.append(os.path.join(HERE, "..", "include", "t3b200.h"))
    if force or not _newer(LIB, srcs + [inc]):
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
               "-I", BUILD, "-I", CSRC, os.path.join(CSRC, "t3b_abi.cu"), "-o", LIB]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        _run(cmd)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv)
