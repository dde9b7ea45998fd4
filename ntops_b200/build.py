"""Builds libntops_b200.so, the sm_100a kernel library behind ``ntops_b200.torch``.

Every ``csrc/*.cu`` file is compiled by nvcc for ``sm_100a`` into ``_build/`` (in parallel,
recompiled only when a source or header is newer than its object) and linked into
``ntops_b200/libntops_b200.so``.  The library links the CUDA runtime statically and reaches the
driver API through ``cudaGetDriverEntryPoint``, so it needs nothing but the NVIDIA driver at
run time and has no torch dependency.

Usage: ``python ntops_b200/build.py [--debug] [--jobs N]`` (run as a script: importing the
package itself needs the built library).
"""

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
BUILD_DIR = os.path.join(PKG_DIR, "_build")
LIB_NAME = "libntops_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc():
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(cuda_home, "bin", "nvcc")
    if os.path.exists(cand):
        return cand
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def _flags(debug):
    flags = ARCH_FLAGS + [
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        "--expt-relaxed-constexpr",
        "-I" + INCLUDE,
        "-I" + CSRC,
    ]
    if debug:
        flags.append("-DNTB_DEBUG=1")
    return flags


def _sources():
    return sorted(
        os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu")
    )


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _needs_build(src, obj, header_mtime):
    if not os.path.exists(obj):
        return True
    m = os.path.getmtime(obj)
    return os.path.getmtime(src) > m or header_mtime > m


def build(debug=False, jobs=None, verbose=False):
    """Compiles and links the library; returns its path."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    nvcc = _nvcc()
    flags = _flags(debug)
    header_mtime = max((os.path.getmtime(h) for h in _headers()), default=0.0)
    srcs = _sources()
    objs = []
    todo = []
    for src in srcs:
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if _needs_build(src, obj, header_mtime):
            todo.append((src, obj))

    def compile_one(pair):
        src, obj = pair
        cmd = [nvcc] + flags + ["-c", src, "-o", obj + ".tmp"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
        os.replace(obj + ".tmp", obj)
        if verbose:
            print(f"compiled {os.path.basename(src)}", flush=True)
        return res.stderr

    jobs = jobs or max(1, os.cpu_count() or 1)
    if todo:
        with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as ex:
            for _ in ex.map(compile_one, todo):
                pass
    lib_stale = (not os.path.exists(LIB_PATH)) or any(
        os.path.getmtime(o) > os.path.getmtime(LIB_PATH) for o in objs
    )
    if lib_stale or todo:
        cmd = [nvcc] + ARCH_FLAGS + ["-shared", "-o", LIB_PATH + ".tmp"] + objs
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args(argv)
    path = build(debug=args.debug, jobs=args.jobs, verbose=True)
    print(path)


if __name__ == "__main__":
    sys.exit(main())
