"""Build recipe for libglq.so (sm_100a only).

Compiles every ``csrc/*.cu`` translation unit with nvcc for
``-gencode arch=compute_100a,code=sm_100a`` and links them into
``gemm_lab_qualification_b200/libglq.so`` in-tree, next to this file, so the
shared library travels with the source tree.  The CUDA runtime is linked
statically; the driver is reached at run time through
``cudaGetDriverEntryPointByVersion``, so the library loads (but reports
``GLQ_ERR_DEVICE``) on a machine without a GPU.

Also builds the native CLI ``gemm_bench`` (csrc/gemm_bench.cu) when present.

Usage: ``python -m gemm_lab_qualification_b200.build [--force]``.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = PACKAGE_DIR.parent / "include"
BUILD_DIR = PACKAGE_DIR.parent / "_build"
LIBRARY = PACKAGE_DIR / "libglq.so"
BENCH_BINARY = PACKAGE_DIR / "gemm_bench"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}"]
LIBRARY_SOURCES = ["glq_api.cu", "glq_tc.cu", "glq_gemv.cu", "glq_generic.cu"]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path("/usr/local/cuda/bin/nvcc")
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")


def _stale(target: Path, inputs: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in inputs)


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _compile(source: Path, obj: Path, extra: list[str]) -> None:
    cmd = [nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, *extra, "-c", str(source), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {source.name}:\n{proc.stderr}\n{proc.stdout}")


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link libglq.so; returns its path."""
    BUILD_DIR.mkdir(exist_ok=True)
    sources = [CSRC / s for s in LIBRARY_SOURCES]
    headers = _headers()
    objects = []
    jobs = []
    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as pool:
        for src in sources:
            obj = BUILD_DIR / (src.stem + ".o")
            objects.append(obj)
            if force or _stale(obj, [src, *headers]):
                jobs.append(pool.submit(_compile, src, obj, ["-Xptxas", "-v"] if verbose else []))
        for job in jobs:
            job.result()
    if force or _stale(LIBRARY, objects):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objects)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link of libglq.so failed:\n{proc.stderr}")
        os.replace(tmp, LIBRARY)
    return LIBRARY


def build_bench(force: bool = False) -> Path | None:
    """Build the gemm_bench CLI against libglq.so (cuBLASLt comparator)."""
    src = CSRC / "gemm_bench.cu"
    if not src.exists():
        return None
    lib = build_library(force=force)
    if force or _stale(BENCH_BINARY, [src, lib, *_headers()]):
        cmd = [nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, str(src), "-o", str(BENCH_BINARY),
               f"-L{PACKAGE_DIR}", "-lglq", "-lcublasLt", "-lcublas",
               "-Xlinker", "-rpath", "-Xlinker", "$ORIGIN"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"gemm_bench build failed:\n{proc.stderr}")
    return BENCH_BINARY


def torch_binding_path() -> Path:
    import sysconfig
    return PACKAGE_DIR / ("_glq_torch" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_torch_binding(force: bool = False) -> Path:
    """Build _glq_torch (csrc/glq_torch.cpp): the operator API's checks and
    launch in one native call, linked against libglq.so and torch."""
    import sysconfig

    import torch
    import torch.utils.cpp_extension as cpp_ext

    src = CSRC / "glq_torch.cpp"
    out = torch_binding_path()
    lib = build_library(force=force)
    if not (force or _stale(out, [src, lib, *_headers()])):
        return out
    try:
        includes = cpp_ext.include_paths(device_type="cuda")
    except TypeError:
        includes = cpp_ext.include_paths(cuda=True)
    includes = [*includes, sysconfig.get_paths()["include"], str(INCLUDE)]
    torch_lib = cpp_ext.library_paths()[0]
    tmp = out.with_suffix(".tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           "-DTORCH_EXTENSION_NAME=_glq_torch", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *cpp_ext._get_pybind11_abi_build_flags(), *[f"-I{p}" for p in includes], str(src), "-o", str(tmp),
           f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python",
           f"-L{PACKAGE_DIR}", "-lglq", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"_glq_torch build failed:\n{proc.stderr}")
    os.replace(tmp, out)
    return out


def main(argv: list[str]) -> int:
    force = "--force" in argv
    verbose = "-v" in argv or "--verbose" in argv
    print(build_library(force=force, verbose=verbose))
    print(build_torch_binding(force=force))
    bench = build_bench(force=force)
    if bench is not None:
        print(bench)
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv[1:]))
