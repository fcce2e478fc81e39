"""Build the in-tree shared libraries for sm_100a.

  libmpb200.so       -- the device layer: CUDA kernels + the C ABI of
                        include/miniprefix_b200.h
  libmpb200_host.so  -- the C++ host layer (page pool, prefix cache, KV manager,
                        scheduler, engine, runner) + the C ABI of
                        include/miniprefix_b200_host.h; links libmpb200.so

nvcc cross-compiles without a GPU. Outputs stay next to this file so they travel
with the repository snapshot; nothing is installed.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
DEVICE_LIB = os.path.join(HERE, "libmpb200.so")
HOST_LIB = os.path.join(HERE, "libmpb200_host.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{CSRC}"]
# Extra nvcc flags for tuning builds, e.g. MPB_NVCC_FLAGS="-DMPB_GATE_UP_BN=128" (the
# compile-time switches are documented where they are defined); empty by default.
COMMON += os.environ.get("MPB_NVCC_FLAGS", "").split()

DEVICE_SOURCES = ["attention.cu", "attention_shared.cu", "attention_prefill.cu", "tc_gemm.cu", "fused_ops.cu", "context.cu", "operator.cu", "operator_noalloc.cu"]
HOST_SOURCES = []  # filled in by host/ when present


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)


def _headers() -> list[str]:
    out = []
    for d in (CSRC, os.path.join(CSRC, "host"), INCLUDE):
        if os.path.isdir(d):
            out += [os.path.join(d, f) for f in os.listdir(d) if f.endswith((".h", ".cuh", ".hpp"))]
    return out


def build_device(force: bool = False) -> str:
    """Compile each stale .cu (newer than its object, or any header newer) in
    parallel, then link the shared library if any object changed."""
    from concurrent.futures import ThreadPoolExecutor

    sources = [os.path.join(CSRC, s) for s in DEVICE_SOURCES]
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    headers = _headers()
    objects = [os.path.join(objdir, os.path.basename(s) + ".o") for s in sources]
    todo = [(s, o) for s, o in zip(sources, objects) if force or _stale(o, [s] + headers)]
    if todo:
        with ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as pool:
            list(pool.map(lambda so: _run([NVCC, *ARCH, *COMMON, "-c", so[0], "-o", so[1]]), todo))
    if todo or _stale(DEVICE_LIB, objects):
        _run([NVCC, *ARCH, "-shared", "-o", DEVICE_LIB, *objects])
    return DEVICE_LIB


def host_sources() -> list[str]:
    d = os.path.join(CSRC, "host")
    if not os.path.isdir(d):
        return []
    return sorted(os.path.join(d, f) for f in os.listdir(d) if f.endswith(".cpp"))


def build_host(force: bool = False) -> str | None:
    sources = host_sources()
    if not sources:
        return None
    if not force and not _stale(HOST_LIB, sources + [DEVICE_LIB] + _headers()):
        return HOST_LIB
    _run(["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-Wextra", f"-I{INCLUDE}",
          f"-I{os.path.join(CSRC, 'host')}", *sources, "-o", HOST_LIB, f"-L{HERE}", "-lmpb200",
          "-Wl,-rpath,$ORIGIN", "-Wl,--no-undefined"])
    return HOST_LIB


WORKER_DIR = os.path.join(CSRC, "worker")
EXECUTABLES = {"mpb200_worker": "worker_main.cpp", "mpb200_stress": "stress_main.cpp"}


def build_executables(force: bool = False) -> list[str]:
    """The protocol worker and the lifecycle stress harness, linked against the
    host library (in-tree, next to it)."""
    out = []
    for exe, src in EXECUTABLES.items():
        path, source = os.path.join(HERE, exe), os.path.join(WORKER_DIR, src)
        if not os.path.exists(source):
            continue
        headers = [os.path.join(CSRC, "host", f) for f in os.listdir(os.path.join(CSRC, "host")) if f.endswith(".h")]
        if force or _stale(path, [source, HOST_LIB] + headers):
            _run(["g++", "-O2", "-std=c++17", "-Wall", "-Wextra", f"-I{INCLUDE}", f"-I{os.path.join(CSRC, 'host')}",
                  source, "-o", path, f"-L{HERE}", "-lmpb200_host", "-lmpb200", "-Wl,-rpath,$ORIGIN"])
        out.append(path)
    return out


def build(force: bool = False) -> None:
    build_device(force)
    build_host(force)
    build_executables(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
