"""Builds libcljxla_b200.so in-tree (clj-xla_b200/lib/) for sm_100a.

Host C++ is compiled with g++, CUDA sources with nvcc
(-gencode arch=compute_100a,code=sm_100a), and the library links the CUDA
runtime statically so the JVM (or ctypes) host only needs the driver.
Incremental: objects are rebuilt when their source or any header is newer.
"""
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
SRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "lib", "obj")
LIB = os.path.join(PKG, "lib", "libcljxla_b200.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
INC = ["-I" + os.path.join(ROOT, "include"), "-I" + SRC, "-I" + os.path.join(CUDA, "include")]


def _newest_header():
    hs = glob.glob(os.path.join(SRC, "*.h")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    return max((os.path.getmtime(h) for h in hs), default=0)


def _compile(src, hdr_time, verbose):
    base = os.path.basename(src)
    obj = os.path.join(OBJ, base + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_time):
        return obj, None
    if src.endswith(".cu"):
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
               "--expt-relaxed-constexpr", *INC, "-c", src, "-o", obj]
        if os.environ.get("CLJXLA_PTXAS_V"):
            cmd.insert(1, "-Xptxas=-v")
    else:
        cmd = ["g++", "-O2", "-g", "-std=c++17", "-fPIC", "-fvisibility=hidden", "-Wall",
               "-Wno-unused-function", *INC, "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f"{' '.join(cmd)}\n{r.stdout}{r.stderr}"
    if os.environ.get("CLJXLA_PTXAS_V") and r.stderr:
        print(r.stderr, file=sys.stderr)
    return obj, None


def build(verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(SRC, "*.cc")) + glob.glob(os.path.join(SRC, "*.cu")))
    ht = _newest_header()
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        results = list(ex.map(lambda s: _compile(s, ht, verbose), srcs))
    errs = [e for _, e in results if e]
    if errs:
        raise RuntimeError("build failed:\n" + "\n".join(errs))
    objs = [o for o, _ in results]
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs,
               "-Xlinker", "--exclude-libs,ALL", "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
