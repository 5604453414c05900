"""Builds the native libraries of the B200 operator plugin in-tree.

Outputs (under ``dl-inference_b200/lib/``):

* ``libdli_sm100.so``      — the C-ABI kernel library (``include/dli_sm100.h``),
                             CUDA sources in ``csrc/`` compiled for sm_100a.
* ``libdli_core.so``       — the host runtime (``core/``): tensors, graph JSON,
                             operator registry, engine, KV cache, weights loader.
* ``libdli_sm100_ops.so``  — the operator plugin exporting
                             ``dli_register_operators`` (``plugin/``).
* ``libdli_triton_aot_ops.so`` — a copy of the plugin under the reference
                             plugin's file name, so scripts that load the
                             reference plugin by name pick this one up.
* ``python/dli/_dli_native*.so`` — the pybind11 binding behind ``import dli``.

Usage: ``python dl-inference_b200/build.py [--only kernels|core|plugin|binding] [-j N]``.
Compilation is incremental (an object is rebuilt when any source or header of
its group is newer).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
BUILD = PKG / "_build"
LIB = PKG / "lib"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
CUDA_HOME = Path(NVCC).resolve().parent.parent


def _torch_paths() -> tuple[Path, list[Path], Path]:
    import torch  # noqa: F401  (only for its install location)

    tdir = Path(torch.__file__).resolve().parent
    incs = [tdir / "include", tdir / "include" / "torch" / "csrc" / "api" / "include"]
    return tdir, incs, tdir / "lib"


def _newest(paths: list[Path]) -> float:
    return max((p.stat().st_mtime for p in paths if p.exists()), default=0.0)


def _run(cmd: list[str]) -> None:
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd)}\n{proc.stdout}")


def _compile_all(jobs: list[tuple[list[str], Path, list[Path]]], workers: int) -> list[Path]:
    """Each job: (command without -o, object path, dependency files)."""
    todo = []
    objs = []
    for cmd, obj, deps in jobs:
        objs.append(obj)
        if not obj.exists() or obj.stat().st_mtime < _newest(deps):
            todo.append(cmd + ["-o", str(obj)])
    if todo:
        with cf.ThreadPoolExecutor(max_workers=workers) as pool:
            list(pool.map(_run, todo))
    return objs


def build_kernels(workers: int) -> Path:
    src = PKG / "csrc"
    out = BUILD / "kernels"
    out.mkdir(parents=True, exist_ok=True)
    headers = list(src.glob("*.cuh")) + [ROOT / "include" / "dli_sm100.h"]
    jobs = []
    for cu in sorted(src.glob("*.cu")):
        cmd = [NVCC, *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
               "-I", str(ROOT / "include"), "-c", str(cu)]
        jobs.append((cmd, out / (cu.stem + ".o"), [cu, *headers]))
    objs = _compile_all(jobs, workers)
    LIB.mkdir(exist_ok=True)
    so = LIB / "libdli_sm100.so"
    if not so.exists() or so.stat().st_mtime < _newest(objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(so), *map(str, objs), "-lcudart"])
    return so


def _cxx_flags(tinc: list[Path]) -> list[str]:
    flags = ["-O2", "-std=c++17", "-fPIC", "-D_GLIBCXX_USE_CXX11_ABI=1",
             "-I", str(PKG / "core" / "include"), "-I", str(ROOT / "include"),
             "-I", str(CUDA_HOME / "include")]
    for p in tinc:
        flags += ["-isystem", str(p)]
    return flags


def _torch_abi_flag() -> str:
    import torch

    return f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"


def build_core(workers: int) -> Path:
    _, tinc, tlib = _torch_paths()
    src = PKG / "core" / "src"
    out = BUILD / "core"
    out.mkdir(parents=True, exist_ok=True)
    headers = list((PKG / "core" / "include" / "dli").glob("*.h")) + list(src.glob("*.h")) + [
        ROOT / "include" / "dli_sm100.h"]
    flags = [f for f in _cxx_flags(tinc) if not f.startswith("-D_GLIBCXX")] + [_torch_abi_flag()]
    jobs = []
    for cc in sorted(src.glob("*.cc")):
        jobs.append((["g++", *flags, "-c", str(cc)], out / (cc.stem + ".o"), [cc, *headers]))
    objs = _compile_all(jobs, workers)
    so = LIB / "libdli_core.so"
    deps = objs + [LIB / "libdli_sm100.so"]
    if not so.exists() or so.stat().st_mtime < _newest(deps):
        _run(["g++", "-shared", "-o", str(so), *map(str, objs), f"-L{LIB}", "-ldli_sm100",
              f"-L{tlib}", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda",
              f"-L{CUDA_HOME / 'lib64'}", "-lcudart", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{tlib}",
              f"-Wl,-rpath,{CUDA_HOME / 'lib64'}", "-ldl"])
    return so


def _nccl_paths() -> tuple[Path, Path] | None:
    try:
        import nvidia.nccl as nccl_pkg  # type: ignore
    except Exception:
        return None
    base = Path(list(nccl_pkg.__path__)[0])
    inc, lib = base / "include", base / "lib"
    return (inc, lib) if (inc / "nccl.h").exists() else None


def build_plugin(workers: int) -> Path:
    _, tinc, tlib = _torch_paths()
    src = PKG / "plugin"
    out = BUILD / "plugin"
    out.mkdir(parents=True, exist_ok=True)
    headers = list((PKG / "core" / "include" / "dli").glob("*.h")) + list(src.glob("*.h")) + [
        ROOT / "include" / "dli_sm100.h"]
    flags = [f for f in _cxx_flags(tinc) if not f.startswith("-D_GLIBCXX")] + [_torch_abi_flag()]
    nccl = _nccl_paths()
    if nccl:
        flags += ["-DDLI_WITH_NCCL=1", "-isystem", str(nccl[0])]
    jobs = []
    for cc in sorted(src.glob("*.cc")):
        jobs.append((["g++", *flags, "-c", str(cc)], out / (cc.stem + ".o"), [cc, *headers]))
    objs = _compile_all(jobs, workers)
    so = LIB / "libdli_sm100_ops.so"
    deps = objs + [LIB / "libdli_core.so", LIB / "libdli_sm100.so"]
    if not so.exists() or so.stat().st_mtime < _newest(deps):
        link = ["g++", "-shared", "-o", str(so), *map(str, objs), f"-L{LIB}", "-ldli_core",
                "-ldli_sm100", f"-L{tlib}", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda",
                f"-L{CUDA_HOME / 'lib64'}", "-lcudart", "-Wl,-rpath,$ORIGIN",
                f"-Wl,-rpath,{tlib}", f"-Wl,-rpath,{CUDA_HOME / 'lib64'}"]
        if nccl:
            nccl_so = sorted(nccl[1].glob("libnccl.so*"))
            if nccl_so:
                link += [str(nccl_so[0]), f"-Wl,-rpath,{nccl[1]}"]
        _run(link)
    alias = LIB / "libdli_triton_aot_ops.so"
    if not alias.exists() or alias.stat().st_mtime < so.stat().st_mtime:
        shutil.copy2(so, alias)
    return so


def build_binding(workers: int) -> Path:
    import pybind11

    _, tinc, tlib = _torch_paths()
    src = PKG / "core" / "binding" / "python_bindings.cc"
    out = BUILD / "binding"
    out.mkdir(parents=True, exist_ok=True)
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    dest = PKG / "python" / "dli" / f"_dli_native{suffix}"
    headers = list((PKG / "core" / "include" / "dli").glob("*.h"))
    py_inc = sysconfig.get_paths()["include"]
    flags = [f for f in _cxx_flags(tinc) if not f.startswith("-D_GLIBCXX")] + [
        _torch_abi_flag(), "-isystem", py_inc, "-isystem", pybind11.get_include(),
        "-DTORCH_EXTENSION_NAME=_dli_native", "-fvisibility=hidden"]
    obj = out / "python_bindings.o"
    _compile_all([(["g++", *flags, "-c", str(src)], obj, [src, *headers])], workers)
    deps = [obj, LIB / "libdli_core.so"]
    if not dest.exists() or dest.stat().st_mtime < _newest(deps):
        _run(["g++", "-shared", "-o", str(dest), str(obj), f"-L{LIB}", "-ldli_core", f"-L{tlib}",
              "-lc10", "-ltorch_cpu", "-ltorch", "-ltorch_python", f"-Wl,-rpath,{LIB}",
              f"-Wl,-rpath,{tlib}"])
    return dest


STEPS = {"kernels": build_kernels, "core": build_core, "plugin": build_plugin,
         "binding": build_binding}


def build(only: str | None = None, workers: int | None = None) -> None:
    workers = workers or max(2, min(16, os.cpu_count() or 2))
    order = [only] if only else ["kernels", "core", "plugin", "binding"]
    for step in order:
        if step in ("core", "plugin", "binding") and not any((PKG / "core" / "src").glob("*.cc")):
            continue
        STEPS[step](workers)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", choices=sorted(STEPS))
    ap.add_argument("-j", type=int, default=None)
    args = ap.parse_args()
    build(args.only, args.j)
    return 0


if __name__ == "__main__":
    sys.exit(main())
