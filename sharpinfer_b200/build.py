"""Build libsharpinfer_b200.so (sm_100a) in-tree with nvcc.

Each csrc/*.cu file is compiled to an object under _build/ (rebuilt when the
file or any csrc header changed) and the objects are linked into
sharpinfer_b200/libsharpinfer_b200.so.  Cross-compiles without a GPU.
"""
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libsharpinfer_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-I" + os.path.join(ROOT, "include"), "--expt-relaxed-constexpr",
]
LIBS = ["-lcudart", "-lpthread"]


def _headers_mtime():
    m = 0.0
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh", ".hpp")):
                m = max(m, os.path.getmtime(os.path.join(d, f)))
    return m


def _compile(src, verbose_ptxas=False):
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    cmd = [NVCC] + FLAGS + (["-Xptxas", "-v"] if verbose_ptxas else []) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (src, r.stdout, r.stderr))
    return obj, r.stderr


def build(force=False, verbose_ptxas=False, jobs=None):
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))
    hdr = _headers_mtime()
    todo = []
    for s in srcs:
        o = os.path.join(OBJ, os.path.basename(s) + ".o")
        if force or verbose_ptxas or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), hdr):
            todo.append(s)
    logs = {}
    if todo:
        with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as ex:
            for s, (o, err) in zip(todo, ex.map(lambda s: _compile(s, verbose_ptxas), todo)):
                logs[s] = err
    objs = [os.path.join(OBJ, os.path.basename(s) + ".o") for s in srcs]
    if todo or not os.path.exists(LIB):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + LIBS
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s\n%s" % (r.stdout, r.stderr))
    return LIB, logs


if __name__ == "__main__":
    lib, logs = build(force="--force" in sys.argv, verbose_ptxas="--ptxas" in sys.argv)
    for s, e in logs.items():
        if e.strip():
            print("==", os.path.basename(s))
            print(e)
    print(lib)
