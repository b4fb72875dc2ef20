"""Build libsheep_b200.so in-tree: every CUDA source for sm_100a, the C sources
with the host compiler, one shared library under sheep_b200/lib/.

    python -m sheep_b200.build [-v] [--force]
"""
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "lib", "libsheep_b200.so")
LIB_CHECKED = os.path.join(HERE, "lib", "libsheep_b200_checked.so")
LIB_TRACE = os.path.join(HERE, "lib", "libsheep_b200_trace.so")
CLI_SRC = os.path.join(HERE, "cli", "sml_gpu_fwd.c")
CLI = os.path.join(HERE, "lib", "sml-gpu-fwd")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fopenmp",
                     "-Xcompiler", "-fPIC", "-Xptxas", "-warn-spills"]
CC_FLAGS = ["-O2", "-fPIC", "-fopenmp", "-std=gnu11", "-Wall", "-Wno-unused-function"]
INCS = ["-I" + os.path.join(ROOT, "include"), "-I" + CSRC]


def _nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _cc():
    # the image's default CC may lack OpenMP; the system gcc has it
    for c in ("/usr/bin/gcc", shutil.which("gcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("gcc not found")


def _sources():
    cu = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    c = sorted(f for f in os.listdir(CSRC) if f.endswith(".c"))
    return cu, c


def _deps():
    return [os.path.join(CSRC, f) for f in os.listdir(CSRC)] + [
        os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build(verbose=False, force=False, checked=False, trace=False):
    """Compile every source (sm_100a for CUDA) and link the in-tree library.
    checked=True builds libsheep_b200_checked.so with in-kernel bounds checks
    that record a failing site instead of making the access (-DSB_CHECKED)."""
    obj = OBJ + ("_checked" if checked else "_trace" if trace else "")
    lib = LIB_CHECKED if checked else LIB_TRACE if trace else LIB
    os.makedirs(obj, exist_ok=True)
    os.makedirs(os.path.dirname(lib), exist_ok=True)
    cu, c = _sources()
    deps = _deps()
    if not force and not _stale(lib, deps):
        if lib == LIB:
            build_cli(verbose)
        return lib
    extra = (["-DSB_CHECKED"] if checked else []) + (["-DSB_TRACE"] if trace else [])
    nvcc, cc = _nvcc(), _cc()
    jobs = []
    for f in cu:
        o = os.path.join(obj, f[:-3] + ".o")
        jobs.append([nvcc] + NVCC_FLAGS + extra + INCS + ["-c", os.path.join(CSRC, f), "-o", o])
    for f in c:
        o = os.path.join(obj, f[:-2] + ".o")
        jobs.append([cc] + CC_FLAGS + INCS + ["-c", os.path.join(CSRC, f), "-o", o])
    logs = []
    with cf.ThreadPoolExecutor(max_workers=max(2, os.cpu_count() or 2)) as ex:
        for out in ex.map(lambda j: _run(j, verbose), jobs):
            logs.append(out)
    objs = [os.path.join(obj, f[:-3] + ".o") for f in cu] + [os.path.join(obj, f[:-2] + ".o") for f in c]
    _run([nvcc] + ARCH + ["-shared", "-o", lib] + objs + ["-lgomp", "-lcuda"], verbose)
    if verbose:
        for l in logs:
            if l.strip():
                print(l)
    if lib == LIB:
        build_cli(verbose, force=True)
    return lib


def build_cli(verbose=False, force=False):
    """The sml-gpu-fwd command line (sheep_b200/cli), linked against the
    in-tree library (found next to it at run time)."""
    deps = [CLI_SRC, LIB] + [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]
    if not force and not _stale(CLI, deps):
        return CLI
    _run([_cc(), "-O2", "-std=gnu11", "-Wall", "-I" + os.path.join(ROOT, "include"), CLI_SRC, "-o", CLI,
          "-L" + os.path.dirname(LIB), "-lsheep_b200", "-Wl,-rpath,$ORIGIN", "-lm"], verbose)
    return CLI


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="--force" in sys.argv, checked="--checked" in sys.argv,
                trace="--trace" in sys.argv))
