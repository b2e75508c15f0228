"""Build recipe of the CUDA library: nvcc for sm_100a, in-tree output
nightrun_b200/libnrcuda.so. Usable as `python -m nightrun_b200.build`.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libnrcuda.so")
SOURCES = ["gemv.cu", "mma.cu", "ops.cu", "attn.cu", "synth.cu", "engine.cu", "api.cu", "noalloc.cu", "sample.cu", "tp.cu", "mma_kq.cu", "gguf.cu"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def nvcc_flags():
    return ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
            "-Xcompiler", "-fPIC,-ffp-contract=off,-fno-fast-math", "-I", os.path.join(ROOT, "include"),
            "-I", CSRC, "--expt-relaxed-constexpr"]


def build(verbose=False, jobs=None):
    """Compile every .cu to an object in parallel, then link the shared library."""
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    procs = []
    objs = []
    for src in SOURCES:
        obj = os.path.join(objdir, src.replace(".cu", ".o"))
        objs.append(obj)
        srcp = os.path.join(CSRC, src)
        deps = [srcp] + [os.path.join(CSRC, h) for h in os.listdir(CSRC) if h.endswith((".cuh", ".h"))]
        deps.append(os.path.join(ROOT, "include", "nrcuda.h"))
        if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
            continue
        cmd = [NVCC] + nvcc_flags() + ["-c", srcp, "-o", obj]
        if verbose:
            cmd.append("-Xptxas=-v")
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        text = out.decode(errors="replace")
        if p.returncode != 0:
            failed.append((src, text))
        elif verbose and text.strip():
            print(f"== {src}\n{text}")
    if failed:
        for src, text in failed:
            sys.stderr.write(f"== nvcc failed on {src}\n{text}\n")
        raise RuntimeError("nvcc failed: " + ", ".join(s for s, _ in failed))
    link = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", OUT] + objs + ["-lcudart", "-ldl"]
    subprocess.check_call(link)
    return OUT


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(OUT)
