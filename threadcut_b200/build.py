"""Build libthreadcut_b200.so in-tree for sm_100a: `python -m threadcut_b200.build`.

One nvcc invocation over the single translation unit csrc/threadcut_b200.cu; the CUDA runtime is
linked statically so the library loads next to torch's own runtime without version coupling.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc", "threadcut_b200.cu")
OUT = os.path.join(HERE, "libthreadcut_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC", "-cudart", "static",
         "-I", os.path.join(ROOT, "include")]


def nvcc():
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found; the CUDA 12.8+ toolkit is required to build threadcut_b200")
    return exe


def sources():
    csrc = os.path.join(HERE, "csrc")
    return [os.path.join(csrc, f) for f in sorted(os.listdir(csrc)) if f.endswith((".cu", ".cuh"))]


def up_to_date():
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    deps = sources() + [os.path.join(ROOT, "include", "threadcut_b200.h"), __file__]
    return all(os.path.getmtime(p) <= t for p in deps)


def build(force=False, verbose=False):
    """Compile the library if any source is newer than it. Returns the .so path."""
    if not force and up_to_date():
        return OUT
    tmp = OUT + ".tmp"
    cmd = [nvcc()] + ARCH + FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-o", tmp, SRC]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        sys.stdout.write(res.stdout + res.stderr)
    os.replace(tmp, OUT)
    return OUT


HOST_SRC = os.path.join(HERE, "csrc", "host_binding.cpp")
HOST_DIR = os.path.join(HERE, "_host")
HOST_NAME = "threadcut_b200_host"
HOST_OUT = os.path.join(HOST_DIR, HOST_NAME + ".so")


def build_host(force=False):
    """Compile the host-only Python binding (csrc/host_binding.cpp, torch C++ API, no device code)
    into threadcut_b200/_host/ with torch's extension builder. Returns the .so path."""
    if not force and os.path.exists(HOST_OUT) and os.path.getmtime(HOST_OUT) >= os.path.getmtime(HOST_SRC):
        return HOST_OUT
    from torch.utils import cpp_extension
    os.makedirs(HOST_DIR, exist_ok=True)
    cpp_extension.load(name=HOST_NAME, sources=[HOST_SRC], build_directory=HOST_DIR, extra_cflags=["-O2"],
                       with_cuda=True, verbose=False)
    return HOST_OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
    print(build_host(force="--force" in sys.argv))
