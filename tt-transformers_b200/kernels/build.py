"""Compiles the CUDA sources under csrc/ into one shared library, in the source tree.

nvcc builds each .cu file for sm_100a; the objects are linked into
kernels/_build/libttb200-<hash>.so, where <hash> covers the sources and the flags, so a
changed source is compiled again and an unchanged one never is. The first call in a
fresh checkout compiles everything (about a minute) and prints a line per file.
"""

from __future__ import annotations

import concurrent.futures
import fcntl
import hashlib
import os
import shutil
import subprocess
import sys
import tempfile

CSRC = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "csrc")
BUILD_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build")
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
]


class BuildError(RuntimeError):
    pass


def _say(message: str) -> None:
    print(f"[tt_transformers_b200] {message}", file=sys.stderr, flush=True)


def find_nvcc() -> str:
    candidates = [os.environ.get("TTB200_NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for c in candidates:
        if c and os.path.isfile(c) and os.access(c, os.X_OK):
            return c
    raise BuildError("nvcc was not found (looked at $TTB200_NVCC, PATH and /usr/local/cuda/bin/nvcc); "
                     "the CUDA kernels cannot be compiled and there is no other implementation")


def source_files():
    names = sorted(n for n in os.listdir(CSRC) if n.endswith(".cu"))
    headers = sorted(n for n in os.listdir(CSRC) if n.endswith((".cuh", ".h")))
    return names, headers


def source_hash() -> str:
    h = hashlib.sha256()
    names, headers = source_files()
    for n in names + headers:
        h.update(n.encode())
        with open(os.path.join(CSRC, n), "rb") as f:
            h.update(f.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()[:16]


def library_path() -> str:
    return os.path.join(BUILD_DIR, f"libttb200-{source_hash()}.so")


def _compile_one(nvcc: str, name: str, out_dir: str) -> str:
    obj = os.path.join(out_dir, name[:-3] + ".o")
    cmd = [nvcc, *NVCC_FLAGS, "-I", CSRC, "-c", os.path.join(CSRC, name), "-o", obj]
    _say(f"compiling {name} for sm_100a ...")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise BuildError(f"nvcc failed on {name}:\n{proc.stdout}\n{proc.stderr}")
    return obj


def build(force: bool = False) -> str:
    """Build the library if this source state has not been built yet; return its path."""
    target = library_path()
    if os.path.isfile(target) and not force:
        return target
    os.makedirs(BUILD_DIR, exist_ok=True)
    lock_path = os.path.join(BUILD_DIR, ".lock")
    with open(lock_path, "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)       # one builder at a time; the others wait and find the result
        try:
            if os.path.isfile(target) and not force:
                return target
            nvcc = find_nvcc()
            names, _ = source_files()
            _say(f"building the CUDA kernels ({len(names)} files); this happens once per source state")
            work = tempfile.mkdtemp(prefix="obj-", dir=BUILD_DIR)
            try:
                with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as pool:
                    objects = list(pool.map(lambda n: _compile_one(nvcc, n, work), names))
                tmp_so = os.path.join(work, "lib.so")
                link = [nvcc, "-shared", "-o", tmp_so, *objects, "-lcudart"]
                _say("linking ...")
                proc = subprocess.run(link, capture_output=True, text=True)
                if proc.returncode != 0:
                    raise BuildError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
                os.replace(tmp_so, target)
            finally:
                shutil.rmtree(work, ignore_errors=True)
            for old in os.listdir(BUILD_DIR):     # older builds of other source states
                if old.startswith("libttb200-") and os.path.join(BUILD_DIR, old) != target:
                    try:
                        os.remove(os.path.join(BUILD_DIR, old))
                    except OSError:
                        pass
            _say(f"built {os.path.relpath(target)}")
            return target
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)
