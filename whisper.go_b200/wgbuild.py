"""Build recipe of the B200 decoder library and its helpers.

  libwgdec.so  CUDA kernels + C ABI (csrc/*.cu), sm_100a only
  libwggen.so  synthetic-model generator + reference quantiser (gen/wg_gen.c)
  oracle/liboracle.so  CPU oracle (test infrastructure; built by its Makefile)

All outputs are written in-tree so they travel with the repository snapshot.
"""
import os
import pathlib
import subprocess

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.environ.get("NVCC", os.path.join(CUDA_HOME, "bin", "nvcc"))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

LIB = PKG / "libwgdec.so"
GEN = PKG / "libwggen.so"
ORACLE = ROOT / "oracle" / "liboracle.so"


def _stale(out, srcs):
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(s.stat().st_mtime > t for s in srcs)


def _run(cmd, cwd=None):
    r = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed: %s\n%s\n%s" % (" ".join(map(str, cmd)), r.stdout, r.stderr))
    return r.stdout + r.stderr


def build_lib(force=False, verbose_ptxas=False):
    """Compiles every csrc/*.cu for sm_100a (one nvcc process per file, in
    parallel; objects under _build/) and links libwgdec.so."""
    srcs = sorted((PKG / "csrc").glob("*.cu"))
    deps = srcs + sorted((PKG / "csrc").glob("*.cuh")) + [ROOT / "include" / "wg_decoder.h"]
    if not force and not _stale(LIB, deps):
        return ""
    from concurrent.futures import ThreadPoolExecutor
    obj_dir = ROOT / "_build"
    obj_dir.mkdir(exist_ok=True)
    flags = [*ARCH, "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC"]
    if verbose_ptxas:
        flags = ["-Xptxas", "-v", *flags]
    objs = [obj_dir / (s.stem + ".o") for s in srcs]
    with ThreadPoolExecutor(max_workers=max(1, min(len(srcs), os.cpu_count() or 1))) as ex:
        logs = list(ex.map(lambda so: _run([NVCC, *flags, "-c", "-o", str(so[1]), str(so[0])]), zip(srcs, objs)))
    tmp = LIB.with_suffix(".so.tmp")
    logs.append(_run([NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]))
    os.replace(tmp, LIB)  # the library is never seen half-written
    return "".join(logs)


def build_gen(force=False):
    src = PKG / "gen" / "wg_gen.c"
    if not force and not _stale(GEN, [src, ROOT / "include" / "wg_decoder.h"]):
        return ""
    return _run(["gcc", "-O2", "-fopenmp", "-fPIC", "-shared", "-Wall", "-o", str(GEN), str(src), "-lm"])


def build_oracle(force=False):
    if force and ORACLE.exists():
        ORACLE.unlink()
    return _run(["make", "-s", "-C", str(ROOT / "oracle")])


def build_all(force=False):
    build_gen(force)
    build_oracle(force)
    build_lib(force)


if __name__ == "__main__":
    import sys
    build_all(force="--force" in sys.argv)
    print("built", LIB, GEN, ORACLE)
