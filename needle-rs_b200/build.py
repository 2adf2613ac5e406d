"""Builds libneedle_c.so (the C-ABI library: host engine + sm_100a kernels).

Usage: python needle-rs_b200/build.py [--debug]
Output: needle-rs_b200/libneedle_c.so (in-tree; it is what the tests,
smoke() and bench.py load).  Objects go to needle-rs_b200/_build/.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libneedle_c.so")
BUILD = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CU = ["int4_matmul.cu", "attention.cu", "head.cu", "tc_gemm.cu", "tc_attn.cu", "ffn_noalloc.cu", "measure.cu"]
CPP = ["safetensors.cpp", "frontend.cpp", "engine.cpp", "capi.cpp"]


def sources():
    return [os.path.join(SRC, f) for f in CU + CPP] + [
        os.path.join(SRC, f) for f in os.listdir(SRC) if f.endswith((".h", ".cuh"))
    ] + [os.path.join(HERE, "..", "include", f) for f in ("needle.h", "needle_b200.h")]


def up_to_date():
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(s) <= t for s in sources() if os.path.exists(s))


def build(force=False, debug=False):
    if not force and up_to_date():
        return OUT
    from concurrent.futures import ThreadPoolExecutor

    os.makedirs(BUILD, exist_ok=True)
    opt = ["-O0", "-g", "-G"] if debug else ["-O3"]
    common = ["-std=c++17", "-Xcompiler", "-fPIC", "-lineinfo", "-I" + SRC] + opt
    cmds, objs = [], []
    for f in CU + CPP:
        o = os.path.join(BUILD, f + ".o")
        cmd = [NVCC] + ARCH + common + ["-c", os.path.join(SRC, f), "-o", o]
        if f.endswith(".cpp"):
            cmd[1:1] = ["-x", "cu"]
        cmds.append(cmd)
        objs.append(o)
    # one nvcc per translation unit, in parallel
    with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as ex:
        for r in list(ex.map(lambda c: subprocess.run(c), cmds)):
            if r.returncode != 0:
                raise subprocess.CalledProcessError(r.returncode, r.args)
    subprocess.run([NVCC] + ARCH + ["-shared", "--cudart=static", "-o", OUT] + objs, check=True)
    return OUT


if __name__ == "__main__":
    build(force=True, debug="--debug" in sys.argv)
    print(OUT)
