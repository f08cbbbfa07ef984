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
    build_dropin(force)
    return LIB


DROPIN_LIB = os.path.join(HERE, "libt3b200_dropin.so")
DROPIN_TEST = os.path.join(BUILD, "t3_dropin_main")


def build_dropin(force=False):
    """The C++ mirror of chatterbox.cpp's T3 API (csrc/t3_dropin.cpp) as
    libt3b200_dropin.so, and the run_t3-style test program linked to it."""
    inc = os.path.join(HERE, "..", "include")
    src = os.path.join(CSRC, "t3_dropin.cpp")
    deps = [src, os.path.join(inc, "t3b200_dropin.hpp"), os.path.join(inc, "t3b200.h"), LIB]
    gxx = "/usr/bin/g++" if os.path.exists("/usr/bin/g++") else "g++"
    if force or not _newer(DROPIN_LIB, deps):
        _run([gxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-I", inc, src, "-o", DROPIN_LIB,
              "-L", HERE, "-lt3b200", "-Wl,-rpath,$ORIGIN"])
    main = os.path.join(HERE, "..", "tests", "cpp", "t3_dropin_main.cpp")
    if force or not _newer(DROPIN_TEST, [main, DROPIN_LIB]):
        _run([gxx, "-O2", "-std=c++17", "-I", inc, main, "-o", DROPIN_TEST, "-L", HERE, "-lt3b200_dropin",
              "-lt3b200", "-Wl,-rpath," + HERE])
    return DROPIN_LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv)
