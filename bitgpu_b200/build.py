"""Build ``libbgattn.so`` in-tree with nvcc for sm_100a (no JIT, no torch extension cache).

    python -m bitgpu_b200.build          # or bitgpu_b200.build.build()
    python -m bitgpu_b200.build --trace /tmp/libbgattn_trace.so   # timing-trace build (BG_TRACE)

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


def build(verbose=False, extra=(), out=None):
    """Compile every csrc/*.cu and link ``out`` (default: the in-tree libbgattn.so).  A build with
    ``extra=("-DBG_TRACE",)`` and its own ``out`` adds the %globaltimer trace of the decode and
    split-KV exchange kernels (bg_trace_read / bg_ptrace_read); load it with BGATTN_LIB=<out>."""
    out = out or OUT
    bdir = BUILD if out == OUT else os.path.join(os.path.dirname(os.path.abspath(out)), "_build_" + os.path.basename(out))
    os.makedirs(bdir, exist_ok=True)
    srcs = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    objs = [os.path.join(bdir, f[:-3] + ".o") for f in srcs]
    extra = list(extra) + (["-Xptxas", "-v"] if verbose else [])
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        logs = list(ex.map(lambda so: _compile(os.path.join(CSRC, so[0]), so[1], extra), zip(srcs, objs)))
    tmp = out + ".tmp"
    r = subprocess.run([nvcc(), *ARCH, "-shared", "-o", tmp, *objs], capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, out)
    if verbose:
        for s, lg in zip(srcs, logs):
            print(f"== {s}\n{lg}")
    return out


if __name__ == "__main__":
    import sys
    if "--trace" in sys.argv:  # python -m bitgpu_b200.build --trace OUT.so
        print(build(verbose="-v" in sys.argv, extra=("-DBG_TRACE",), out=sys.argv[sys.argv.index("--trace") + 1]))
    else:
        print(build(verbose="-v" in sys.argv))
