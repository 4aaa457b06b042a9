"""Build ``libbgattn.so`` in-tree with nvcc for sm_100a (no JIT, no torch extension cache).

    python -m bitgpu_b200.build          # or bitgpu_b200.build.build()

Each ``csrc/*.cu`` compiles to an object in parallel, then one shared library links them with
the static CUDA runtime.  No fast-math: parity paths rely on IEEE division / sqrt.
"""
import concurrent.futures as cf
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libbgattn.so")
BUILD = os.path.join(HERE, "_build")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _compile(src, obj, extra):
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr}")
    return r.stderr


def build(verbose=False, extra=()):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    objs = [os.path.join(BUILD, f[:-3] + ".o") for f in srcs]
    extra = list(extra) + (["-Xptxas", "-v"] if verbose else [])
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        logs = list(ex.map(lambda so: _compile(os.path.join(CSRC, so[0]), so[1], extra), zip(srcs, objs)))
    tmp = OUT + ".tmp"
    r = subprocess.run([nvcc(), *ARCH, "-shared", "-o", tmp, *objs], capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, OUT)
    if verbose:
        for s, lg in zip(srcs, logs):
            print(f"== {s}\n{lg}")
    return OUT


if __name__ == "__main__":
    import sys
    print(build(verbose="-v" in sys.argv))
