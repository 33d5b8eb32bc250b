"""Build libnufft_b200.so (sm_100a) in-tree with nvcc.

    python mlx_nufft_b200/build.py   [--force] [--ptxas-v]
                                     [--out PATH -DNAME=VALUE ...]

(run it as a script: importing the package needs the built library).

Each CUDA / C++ source under csrc/ is compiled to an object in
mlx_nufft_b200/_build/ (in parallel, skipped when up to date) and linked
into mlx_nufft_b200/libnufft_b200.so against cuFFT.  The architecture is
fixed to sm_100a (B200); no other target is built.  `--out` with `-D`
macros writes a tuning variant (objects in a folder beside it) that the
package loads when NUFFT_B200_LIB names it.
"""

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
LIB = os.path.join(HERE, "libnufft_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ["sizing.cpp", "points.cu", "spread.cu", "interp.cu", "interp_tma.cu",
           "deconv.cu", "fft1.cu", "plan.cu", "noalloc.cu"]


def _cuda_home():
    home = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH")
    if home and os.path.isdir(home):
        return home
    nvcc = shutil.which("nvcc")
    if nvcc:
        return os.path.dirname(os.path.dirname(os.path.realpath(nvcc)))
    return "/usr/local/cuda"


def _nvcc():
    return os.path.join(_cuda_home(), "bin", "nvcc")


def _deps(src):
    """Source plus every header it may include (coarse: all csrc headers)."""
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC)
            if f.endswith((".h", ".cuh"))]
    return [os.path.join(CSRC, src)] + hdrs + [os.path.join(INCLUDE, "nufft_b200.h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose=False, ptxas_v=False, build_dir=BUILD, defines=()):
    obj = os.path.join(build_dir, src.rsplit(".", 1)[0] + ".o")
    if not _stale(obj, _deps(src)):
        return obj
    cmd = [_nvcc(), "-c", os.path.join(CSRC, src), "-o", obj, "-O3",
           "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
           "-I", INCLUDE, "-I", CSRC] + ARCH + list(defines)
    if src.endswith(".cpp"):
        cmd += ["-x", "cu"]
    if ptxas_v:
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if ptxas_v:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose=False, force=False, ptxas_v=False, out=None, defines=()):
    """Compile and link libnufft_b200.so (or the variant `out` built with
    the -D flags in `defines`); returns its path."""
    lib = out or LIB
    build_dir = BUILD if out is None else os.path.splitext(out)[0] + "_obj"
    os.makedirs(build_dir, exist_ok=True)
    if force:
        for f in os.listdir(build_dir):
            if f.endswith(".o"):
                os.remove(os.path.join(build_dir, f))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, ptxas_v, build_dir,
                                              defines), SOURCES))
    if force or _stale(lib, objs):
        libdir = os.path.join(_cuda_home(), "lib64")
        cmd = [_nvcc(), "-shared", "-o", lib] + objs + ARCH + [
            "-L", libdir, "-lcufft", "-Xlinker", f"-rpath={libdir}"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return lib


if __name__ == "__main__":
    argv = sys.argv[1:]
    out = os.path.abspath(argv[argv.index("--out") + 1]) if "--out" in argv else None
    defs = [a for a in argv if a.startswith("-D")]
    print(build(verbose=True, force="--force" in argv,
                ptxas_v="--ptxas-v" in argv, out=out, defines=defs))
