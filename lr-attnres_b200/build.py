"""Build libattnres_b200.so (sm_100a) in-tree with nvcc.

Usage: python lr-attnres_b200/build.py [--verbose]
The shared library lands next to the Python package
(lr-attnres_b200/attnres_b200/libattnres_b200.so) so that it travels with the
source tree; nothing is installed into site-packages.
"""
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
OUT = os.path.join(HERE, "attnres_b200", "libattnres_b200.so")
SOURCES = ["abi.cu", "lrid.cu", "lrid_warp.cu", "lrid_stream_fwd.cu", "lrid_stream_bwd_f32.cu",
           "lrid_stream_bwd_f16.cu", "lrid_stream_bwd_bf16.cu", "base.cu", "keyproj.cu", "kvfused.cu", "keyproj_bwd.cu", "kvbwd.cu", "phase1.cu", "phase2.cu", "headnorm.cu", "summary.cu", "noalloc.cu", "launch_cache.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr"]


def nvcc():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose=False, force=False):
    deps = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    deps.append(os.path.join(INCLUDE, "attnres_b200.h"))
    if not force and not _stale(OUT, deps):
        return OUT
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs, cmds = [], []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        cmd = [nvcc(), *ARCH, *FLAGS, "-I", INCLUDE, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        cmds.append(cmd)
        objs.append(obj)
    # translation units compile independently: run them in parallel, the
    # slowest (the kernel-template instantiations) first
    jobs = max(1, min(len(cmds), os.cpu_count() or 1))
    with concurrent.futures.ThreadPoolExecutor(jobs) as ex:
        for r in list(ex.map(lambda c: subprocess.run(c, capture_output=not verbose, text=True), cmds)):
            if r.returncode != 0:
                sys.stderr.write((r.stdout or "") + (r.stderr or ""))
                raise subprocess.CalledProcessError(r.returncode, r.args)
    tmp = OUT + ".tmp"
    cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
