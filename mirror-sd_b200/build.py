"""Build the sm_100a CUDA library ``lib/libdflash_b200.so`` in-tree with nvcc.

    python mirror-sd_b200/build.py [--force] [--verbose]

Only nvcc and g++ are needed (no GPU); the result is what the Python host
(`_native.py`) loads with ctypes and what the C ABI in include/dflash_b200.h
describes.
"""
import argparse
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libdflash_b200.so")
SOURCES = ["quant.cu", "w8_tc.cu", "attention.cu", "attention_tc.cu", "tc_gemm.cu", "lm_head.cu", "misc.cu", "anchor.cu",
           "f32_path.cu", "dflash_api.cu"]
HEADERS = ["common.cuh", "kernels.cuh"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def _nvcc():
    for cand in [os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"]:
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def _digest():
    h = hashlib.sha256()
    for f in SOURCES + HEADERS:
        with open(os.path.join(CSRC, f), "rb") as fh:
            h.update(fh.read())
    with open(os.path.join(ROOT, "include", "dflash_b200.h"), "rb") as fh:
        h.update(fh.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def build(force=False, verbose=False, jobs=None):
    os.makedirs(LIB_DIR, exist_ok=True)
    stamp = LIB + ".sha256"
    dig = _digest()
    if not force and os.path.exists(LIB) and os.path.exists(stamp):
        with open(stamp) as fh:
            if fh.read().strip() == dig:
                return LIB
    objs = []
    procs = []
    for src in SOURCES:
        obj = os.path.join(LIB_DIR, src.replace(".cu", ".o"))
        cmd = [_nvcc(), *NVCC_FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        txt = out.decode(errors="replace")
        if p.returncode != 0:
            failed.append((src, txt))
        elif verbose and txt.strip():
            print(txt)
    if failed:
        msg = "\n".join(f"--- {s}\n{t}" for s, t in failed)
        raise RuntimeError(f"nvcc failed:\n{msg}")
    tmp = LIB + ".tmp"
    link = [_nvcc(), "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", tmp]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    for o in objs:
        os.remove(o)
    with open(stamp, "w") as fh:
        fh.write(dig)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    sys.exit(0)
