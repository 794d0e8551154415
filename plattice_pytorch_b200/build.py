"""Build libplattice_b200.so (sm_100a) in-tree with nvcc.

The 16 feature dimensions are separate translation units (plattice_pd.cu with
-DPL_PD=n) compiled in parallel, plus the C-ABI unit; objects go to
plattice_pytorch_b200/_build/, the library next to this file.  Rebuilds only
what is older than its sources.

    python -m plattice_pytorch_b200.build [--jobs N] [--verbose-ptxas]
"""
import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libplattice_b200.so")
ROOT = os.path.dirname(HERE)
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr"] + ARCH


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libplattice_b200.so")


def _deps():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + glob.glob(os.path.join(CSRC, "*.h")) + [os.path.join(ROOT, "include", "plattice.h"),
                                                           os.path.abspath(__file__)])


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    return r.returncode, " ".join(cmd), r.stdout


def build(jobs=None, verbose_ptxas=False, force=False):
    """Compile and link; returns the library path."""
    os.makedirs(BUILD, exist_ok=True)
    deps = _deps()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    units = []
    for pd in range(1, 17):
        obj = os.path.join(BUILD, f"plattice_pd{pd}.o")
        units.append((obj, [nvcc()] + NVCC_FLAGS + extra + [f"-DPL_PD={pd}", "-c",
                                                           os.path.join(CSRC, "plattice_pd.cu"), "-o", obj]))
    for name in ("plattice_capi", "plattice_runtime", "plattice_noalloc"):
        obj = os.path.join(BUILD, f"{name}.o")
        units.append((obj, [nvcc()] + NVCC_FLAGS + extra + ["-c", os.path.join(CSRC, f"{name}.cu"), "-o", obj]))
    todo = [(o, c) for o, c in units if force or _stale(o, deps)]
    if todo:
        jobs = jobs or max(1, min(len(todo), os.cpu_count() or 4))
        with cf.ThreadPoolExecutor(jobs) as ex:
            for rc, cmd, out in ex.map(lambda oc: _run(oc[1]), todo):
                if rc != 0 or verbose_ptxas:
                    sys.stderr.write(out)
                if rc != 0:
                    raise RuntimeError(f"nvcc failed ({rc}): {cmd}")
    objs = [o for o, _ in units]
    if force or todo or _stale(LIB, objs):
        rc, cmd, out = _run([nvcc()] + ARCH + ["-shared", "-o", LIB] + objs)
        if rc != 0:
            sys.stderr.write(out)
            raise RuntimeError(f"link failed: {cmd}")
    return LIB


TORCH_EXT = os.path.join(HERE, "_plattice_torch.so")


def build_torch_extension(force=False):
    """Compile csrc/plattice_torch.cpp (PermutoLatticeFunction in C++) as the
    torch extension module _plattice_torch, next to this file; returns its path."""
    src = os.path.join(CSRC, "plattice_torch.cpp")
    deps = [src, os.path.join(ROOT, "include", "plattice.h"), os.path.abspath(__file__)]
    if not force and not _stale(TORCH_EXT, deps):
        return TORCH_EXT
    from torch.utils.cpp_extension import load
    bdir = os.path.join(BUILD, "torch_ext")
    os.makedirs(bdir, exist_ok=True)
    load(name="_plattice_torch", sources=[src], build_directory=bdir, extra_cflags=["-O3"],
         extra_include_paths=[os.path.join(ROOT, "include")], with_cuda=True, verbose=False)
    built = os.path.join(bdir, "_plattice_torch.so")
    shutil.copyfile(built, TORCH_EXT + ".tmp")
    os.replace(TORCH_EXT + ".tmp", TORCH_EXT)
    return TORCH_EXT


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.jobs, a.verbose_ptxas, a.force))
    print(build_torch_extension(a.force))


if __name__ == "__main__":
    main()
