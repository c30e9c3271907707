"""Build libsa3k.so (the sm_100a kernels + the C ABI) in-tree with nvcc.

    python sa3.cpp_b200/build.py [-v]

Objects go to sa3.cpp_b200/_build/, the shared library to sa3.cpp_b200/lib/libsa3k.so.
The CUDA runtime is linked statically and the driver is reached through
cudaGetDriverEntryPoint, so the library also loads on a machine without a GPU driver (every
call then returns an error: there is no CPU fallback).
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "lib")
NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", os.path.join(os.path.dirname(HERE), "include")]
SOURCES = ["quant.cu", "gemm_tc.cu", "gemm_r16.cu", "lora.cu", "adamw.cu", "attention.cu", "attention_tc.cu", "dit_ops.cu", "linear.cu", "dit.cu", "api.cu", "dp.cu", "gguf_io.cu", "checkpoint.cu", "lora_chain.cu", "materialize.cu", "sa3_train.cpp"]


def _compile(src, verbose):
    obj = os.path.join(OBJ, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    deps = [path] + [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    deps += [os.path.join(os.path.dirname(HERE), "include", h) for h in ("sa3k.h", "sa3_train.h")]
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(d) for d in deps):
        return obj, ""
    cmd = [NVCC, *ARCH, *FLAGS, "-c", path, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose=False):
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIB, exist_ok=True)
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    if verbose:
        for _, log in results:
            if log:
                print(log)
    out = os.path.join(LIB, "libsa3k.so")
    objs = [o for o, _ in results]
    if not os.path.exists(out) or os.path.getmtime(out) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", out, *objs, "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return out


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
