"""Build recipe for the CPU oracle and the transcribed CPU baseline.

Test infrastructure only: produces oracle/liboracle.so (the parity checker,
tb_oracle.c) and oracle/libcpuref.so (the timed CPU transcription of the
reference's CPU path, tb_cpu_ref.c).  Neither is part of the product.

The reference itself (Rust n2-kernels, JavaScript/WGSL engine) cannot be built
here: there is no cargo and no node in this image, so there is no oracle/_ref.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))

TARGETS = [
    # (output, sources, extra flags)
    ("liboracle.so", ["tb_oracle.c"], ["-O2"]),
    ("libcpuref.so", ["tb_cpu_ref.c"], ["-O3", "-mavx2", "-pthread"]),
]


def _stale(out, srcs):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs + [os.path.abspath(__file__)])


def build(force=False, verbose=False):
    for out, srcs, flags in TARGETS:
        out_p = os.path.join(HERE, out)
        src_p = [os.path.join(HERE, s) for s in srcs]
        if not force and not _stale(out_p, src_p):
            continue
        cmd = (["gcc", "-shared", "-fPIC", "-std=c11", "-ffp-contract=off",
                "-fno-fast-math", "-Wall", "-D_GNU_SOURCE"] + flags + src_p
               + ["-o", out_p + ".tmp", "-lm"])
        if verbose:
            print(" ".join(cmd))
        subprocess.check_call(cmd)
        os.replace(out_p + ".tmp", out_p)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
