"""Build the in-tree C-ABI library ``libvggt_sparse.so`` for sm_100a.

Each ``csrc/*.cu`` is compiled to an object under ``_build/`` (in parallel)
and linked with ``nvcc -shared``.  The library lands next to this file so it
travels with the source tree.  Run ``python -m vggt_sparse.build`` (with the
package's parent directory on ``sys.path``) or call ``build()``.
"""
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)                 # sparse-attention-vggt_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD_DIR = os.path.join(ROOT, "_build")
LIB_PATH = os.path.join(PKG_DIR, "libvggt_sparse.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I" + INCLUDE, "-I" + CSRC] + ARCH_FLAGS


def _nvcc():
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; set NVCC or add CUDA to PATH")
    return cand


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(nvcc, src, obj, extra):
    cmd = [nvcc, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (src, res.stdout, res.stderr))
    return res.stderr


def build(force=False, verbose=False, ptxas_info=False):
    """Compile every CUDA source for sm_100a and link the shared library."""
    nvcc = _nvcc()
    os.makedirs(BUILD_DIR, exist_ok=True)
    headers = _headers()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    jobs = []
    objs = []
    for src in sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or ptxas_info or _stale(obj, [src, *headers]):
            jobs.append((src, obj))
    logs = []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, extra) for s, o in jobs]
            for f in futs:
                logs.append(f.result())
    if force or jobs or _stale(LIB_PATH, objs):
        cmd = [nvcc, "-shared", *ARCH_FLAGS, "-o", LIB_PATH, *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError("link failed:\n%s\n%s" % (res.stdout, res.stderr))
    if verbose:
        for log in logs:
            sys.stderr.write(log)
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True, ptxas_info="--ptxas" in sys.argv)
    print(path)
