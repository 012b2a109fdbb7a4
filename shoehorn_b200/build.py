"""Build libshoehorn_cuda.so in-tree for sm_100a with nvcc.

The encoders reproduce the reference's f32 arithmetic bit for bit, so the
floating-point flags are part of the contract: no FMA contraction
(-fmad=false), IEEE division and square root, no flush-to-zero.
"""
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libshoehorn_cuda.so")
BUILD_DIR = os.path.join(HERE, "_build")
SOURCES = ["api.cu", "kquant.cu", "decode.cu", "iq.cu", "iq_host.cpp", "noalloc.cu"]
HEADERS = ["common.cuh", "kernels.cuh", "decode.cuh", "fuse.cuh", "iq_host.h", "iq_tables.h"]
HOST = os.path.join(HERE, "host")
HOST_SOURCES = ["gguf.cpp", "imatrix.cpp", "solver.cpp", "pipeline.cpp", "synthetic.cpp", "host_api.cpp"]
HOST_HEADERS = ["gguf.hpp", "imatrix.hpp", "solver.hpp", "pipeline.hpp", "shard.hpp"]
HOST_LIB = os.path.join(HERE, "libshoehorn_host.so")
CLI = os.path.join(HERE, "shoehorn-gpu")
CUDA_INC = "/usr/local/cuda/include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FP = ["-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false"]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def _flags():
    return ["-O3", "-std=c++17", "-lineinfo", *ARCH, *FP, "-Xcompiler", "-fPIC,-O2",
            "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose=False, extra=()):
    os.makedirs(BUILD_DIR, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "shoehorn_cuda.h")]
    objs, jobs = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD_DIR, src + ".o")
        objs.append(o)
        if _stale(o, [s, *hdrs, __file__]):
            jobs.append([nvcc(), *_flags(), *extra, "-c", s, "-o", o])
    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, flush=True)
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        list(ex.map(run, jobs))
    if jobs or _stale(OUT, objs):
        run([nvcc(), *ARCH, "-shared", "-o", OUT, *objs])
    # host pipeline (C++): libshoehorn_host.so and the shoehorn-gpu CLI
    hh = [os.path.join(HOST, h) for h in HOST_HEADERS] + [os.path.join(ROOT, "include", "shoehorn_cuda.h")]
    hobjs, hjobs = [], []
    gxx = ["g++", "-std=c++17", "-O2", "-fPIC", "-Wall", "-Wextra", "-I", os.path.join(ROOT, "include"), "-I", HOST,
           "-I", CUDA_INC]
    for src in HOST_SOURCES + ["cli.cpp"]:
        sp = os.path.join(HOST, src)
        o = os.path.join(BUILD_DIR, "host_" + src + ".o")
        hobjs.append(o)
        if _stale(o, [sp, *hh, __file__]):
            hjobs.append([*gxx, "-c", sp, "-o", o])
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, max(1, len(hjobs)))) as ex:
        list(ex.map(run, hjobs))
    lib_objs = hobjs[:-1]
    link_common = ["-L" + HERE, "-lshoehorn_cuda", "-Xlinker", "-rpath=$ORIGIN", "-lpthread"]
    if hjobs or _stale(HOST_LIB, lib_objs + [OUT]):
        run([nvcc(), *ARCH, "-shared", "-o", HOST_LIB, *lib_objs, *link_common])
    if hjobs or _stale(CLI, hobjs + [OUT]):
        run([nvcc(), *ARCH, "-o", CLI, *hobjs, *link_common])
    return OUT


if __name__ == "__main__":
    verbose = "-v" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas" in sys.argv else []
    print(build(verbose=verbose, extra=extra))
