"""Build libtabinfer_b200.so (sm_100a) in-tree with nvcc.

Each .cu is compiled separately (parallel) with
  -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo -Xcompiler -fPIC
and linked into one shared library next to the Python package, so the GPU box
loads exactly the file built here.  IEEE division/sqrt stay on (no fast math):
several kernels are bit-exact with the reference's arithmetic.
"""
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
OUT = os.path.join(PKG, "libtabinfer_b200.so")
OBJ = os.path.join(REPO, "_build", "obj")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def sources():
    return sorted(f for f in os.listdir(HERE) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(HERE, f) for f in os.listdir(HERE) if f.endswith((".cuh", ".h"))]
    inc = os.path.join(REPO, "include")
    hs += [os.path.join(inc, f) for f in os.listdir(inc) if f.endswith(".h")]
    return hs


def _compile(src, verbose):
    obj = os.path.join(OBJ, src[:-3] + ".o")
    srcp = os.path.join(HERE, src)
    newest = max([os.path.getmtime(srcp), os.path.getmtime(__file__)] + [os.path.getmtime(h) for h in _headers()])
    if os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj, ""
    cmd = [NVCC] + ARCH + FLAGS + ["-I" + os.path.join(REPO, "include"), "-c", srcp, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    p = subprocess.run(cmd, capture_output=True, text=True)
    if p.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (src, " ".join(cmd), p.stderr))
    return obj, p.stderr


def build(verbose=False, jobs=8):
    os.makedirs(OBJ, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(jobs) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    objs = [r[0] for r in results]
    if verbose:
        for s, (_, log) in zip(srcs, results):
            if log:
                print("==", s, "\n" + log)
    if not os.path.exists(OUT) or max(os.path.getmtime(o) for o in objs) > os.path.getmtime(OUT):
        cmd = [NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", OUT + ".tmp"] + objs + ["-ldl"]
        subprocess.check_call(cmd)
        os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
