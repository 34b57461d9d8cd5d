"""Build the CUDA library in-tree (nvcc, sm_100a only).

    python -m latticequant_b200._build [-v]

produces ``latticequant_b200/liblq_b200.so`` next to this file.  Each
``csrc/*.cu`` compiles to its own object under ``_build/`` (in parallel,
and only when it or a shared header changed), then nvcc links the objects.
The library links the CUDA runtime statically and has no torch dependency:
the Python side talks to it through ctypes with raw device pointers.
"""
import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liblq_b200.so")
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
HEADER = os.path.join(HERE, "..", "include", "latticequant_b200.h")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC"]
MAP = os.path.join(CSRC, "liblq_b200.map")
LFLAGS = ["-shared", "-cudart", "static", "-Xlinker", "--version-script=" + MAP]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + [HEADER]


def _obj(src: str) -> str:
    return os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(p) > t for p in deps if os.path.exists(p))


def needs_build() -> bool:
    return _stale(LIB, sources() + _headers() + [MAP])


def _compile(nvcc: str, src: str, verbose: bool):
    cmd = [nvcc] + ARCH + CFLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-c", "-o", _obj(src) + ".tmp", src]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode == 0:
        os.replace(_obj(src) + ".tmp", _obj(src))
    return src, r


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    nvcc = os.environ.get("NVCC", "nvcc")
    os.makedirs(OBJ, exist_ok=True)
    hdrs = _headers()
    todo = [s for s in sources() if force or _stale(_obj(s), [s] + hdrs)]
    with ThreadPoolExecutor(max_workers=max(1, min(len(todo), os.cpu_count() or 1))) as ex:
        results = list(ex.map(lambda s: _compile(nvcc, s, verbose), todo))
    failed = [(s, r) for s, r in results if r.returncode != 0]
    for s, r in results:
        if verbose or r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
    if failed:
        raise RuntimeError("nvcc failed on " + ", ".join(os.path.basename(s) for s, _ in failed))
    cmd = [nvcc] + ARCH + LFLAGS + ["-o", LIB + ".tmp"] + [_obj(s) for s in sources()]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed linking liblq_b200.so")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv or "-v" in sys.argv))
