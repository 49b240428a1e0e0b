"""Builds liblrmcuda.so in-tree for sm_100a with nvcc (no JIT cache, so the library travels with the checkout).

    python -m rosylnalive_b200.build [-v]

Every source is compiled with ``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``; ptxas register/spill
reports go to rosylnalive_b200/_build/ptxas.log. Objects are rebuilt only when a source or header is newer.
"""

from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "liblrmcuda.so")

SOURCES = [
    "device.cu",
    "catalog_kernels.cu",
    "rope_host.cpp",
    "ops.cu",
    "gemm_tcgen05.cu",
    "gemm_decode.cu",
    "qwen_kernels.cu",
    "flash_tc.cu",
    "qwen_engine.cu",
    "decode_attn_static.cu",
    "safetensors.cpp",
    "tokenizer.cpp",
]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fno-fast-math",
                     "--expt-relaxed-constexpr", "-Xptxas", "-v", "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build liblrmcuda.so")


def _headers():
    hs = [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]
    hs += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return hs


def _kernel_set_hash() -> bytes:
    """SHA-256 over the kernel sources and the compile flags: the CUDA counterpart of the reference's ShaderSetHash
    (a different source or flag set is a different kernel set)."""
    h = hashlib.sha256()
    for f in sorted(SOURCES) + sorted(os.path.basename(x) for x in _headers() if x.startswith(CSRC)):
        with open(os.path.join(CSRC, f), "rb") as fh:
            h.update(f.encode() + b"\0" + fh.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.digest()


def _write_hash_source() -> str:
    path = os.path.join(BUILD, "kernel_set_hash.cpp")
    digest = _kernel_set_hash()
    text = ("#include <stdint.h>\nextern const uint8_t lrm_kernel_set_hash[32];\n"
            "const uint8_t lrm_kernel_set_hash[32] = {" + ", ".join(str(b) for b in digest) + "};\n")
    old = open(path).read() if os.path.exists(path) else None
    if old != text:
        with open(path, "w") as f:
            f.write(text)
    return path


def _compile(src: str, obj: str, verbose: bool) -> str:
    cmd = [nvcc(), "-c", src, "-o", obj] + NVCC_FLAGS
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"compiled {os.path.basename(src)}", flush=True)
    return r.stderr


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    newest_header = max((os.path.getmtime(h) for h in _headers()), default=0)
    jobs = []
    srcs = [os.path.join(CSRC, s) for s in SOURCES] + [_write_hash_source()]
    objs = []
    for src in srcs:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        stale = force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), newest_header)
        if stale:
            jobs.append((src, obj))
    logs = {}
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            futs = {ex.submit(_compile, s, o, verbose): s for s, o in jobs}
            for f in cf.as_completed(futs):
                logs[os.path.basename(futs[f])] = f.result()
        with open(os.path.join(BUILD, "ptxas.log"), "a") as f:
            for k, v in sorted(logs.items()):
                f.write(f"==== {k}\n{v}\n")
    if jobs or not os.path.exists(LIB):
        cmd = [nvcc(), "-shared", "-o", LIB] + objs + ARCH
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        if verbose:
            print(f"linked {LIB}", flush=True)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
