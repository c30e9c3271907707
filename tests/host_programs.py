"""Builds the C and C++ programs under tests/c against include/ and the in-tree libsa3k.so."""
import os
import subprocess

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(REPO, "sa3.cpp_b200", "lib")


def build(src, out_dir):
    """Compiles tests/c/<src> (gcc for .c, g++ for .cpp, warnings as errors) into out_dir."""
    import build as sa3k_build   # sa3.cpp_b200/build.py (incremental)
    sa3k_build.build()
    path = os.path.join(REPO, "tests", "c", src)
    exe = os.path.join(out_dir, os.path.splitext(src)[0])
    if src.endswith(".c"):
        cmd = ["gcc", "-std=c11"]
    else:
        cmd = ["g++", "-std=c++17"]
    cmd += ["-O2", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(REPO, "include"), path, "-o", exe,
            "-L", LIBDIR, "-lsa3k", f"-Wl,-rpath,{LIBDIR}", "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile of {src} failed:\n{r.stdout}\n{r.stderr}")
    return exe
