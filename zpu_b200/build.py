"""Builds libzpucuda.so in-tree with nvcc for sm_100a.

    python -m zpu_b200.build          # incremental
    python -m zpu_b200.build --force  # everything

Steps: generate the fused-region catalogue (csrc/gen_regions.py ->
csrc/regions_gen.cuh), compile every csrc/*.cu to an object in parallel,
link them into zpu_b200/libzpucuda.so (CUDA runtime linked statically).
"""
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libzpucuda.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", CSRC, "-I", INCLUDE,
         "--expt-relaxed-constexpr", "-Xcudafe", "--diag_suppress=177"]


def _headers():
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, obj, verbose):
    cmd = [NVCC] + ARCH + FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s%s" % (src, r.stdout, r.stderr))
    return r.stderr if verbose else ""


def build(force=False, verbose=False, jobs=None):
    os.makedirs(OBJ, exist_ok=True)
    gen = os.path.join(CSRC, "regions_gen.cuh")
    gen_py = os.path.join(CSRC, "gen_regions.py")
    if force or _stale(gen, [gen_py]):
        subprocess.run([sys.executable, gen_py, gen], check=True)
    hdrs = _headers()
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    todo = []
    objs = []
    for s in srcs:
        o = os.path.join(OBJ, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            todo.append((s, o))
    reports = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            for rep in ex.map(lambda so: _compile(so[0], so[1], verbose), todo):
                reports.append(rep)
    if force or todo or _stale(LIB, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s%s" % (r.stdout, r.stderr))
    return "\n".join(x for x in reports if x)


if __name__ == "__main__":
    out = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    if out:
        print(out)
    print("built", LIB)
