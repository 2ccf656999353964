"""Build the in-tree CUDA library libexactb200.so for sm_100a (nvcc, no torch dependency).

Every .cu file compiles to its own object in parallel (whole-program device code per file, no
relocatable device code: the translation units share only inline header code), then one nvcc
call links the shared library."""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(ROOT, "_build")
LIB = os.path.join(HERE, "libexactb200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include"), "-I", SRC]
LIBS = ["-ldl"]                       # NCCL (tensor parallelism) is opened at run time


def sources():
    return sorted(os.path.join(SRC, f) for f in os.listdir(SRC) if f.endswith(".cu"))


def headers():
    hs = [os.path.join(SRC, f) for f in os.listdir(SRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(ROOT, "include", "exactb200.h")]


def needs_build():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in sources() + headers())


def _obj(src):
    return os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")


def build(force=False, verbose=False, extra=()):
    if not force and not needs_build():
        return LIB
    os.makedirs(OBJ, exist_ok=True)
    newest_header = max(os.path.getmtime(p) for p in headers())
    flags = ARCH + FLAGS + list(extra)

    def compile_one(src):
        o = _obj(src)
        if (not force and os.path.exists(o) and os.path.getmtime(o) > os.path.getmtime(src)
                and os.path.getmtime(o) > newest_header and not extra):
            return None
        cmd = [NVCC] + flags + ["-c", "-o", o + ".tmp", src]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            return f"{src}:\n{r.stdout}{r.stderr}"
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)
        os.replace(o + ".tmp", o)
        return None

    with ThreadPoolExecutor(max_workers=max(1, min(len(sources()), os.cpu_count() or 4))) as ex:
        errs = [e for e in ex.map(compile_one, sources()) if e]
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    cmd = [NVCC] + ARCH + ["-shared", "-o", LIB + ".tmp"] + [_obj(s) for s in sources()] + LIBS
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, extra=[a for a in sys.argv[1:] if a != "--force"])
