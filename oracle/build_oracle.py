"""Build recipe for the oracle's compiled parts.  TEST INFRASTRUCTURE ONLY.

* ``oracle/_build/libcrt_oracle.so`` -- the C restatement ``crt_oracle.c``.
* ``oracle/_ref/crt_cpu_ref*.so`` -- the reference's own CPU CRT,
  ``src/fp_emulation/csrc/crt_reconstruct.cpp`` of thezettascale/fp-emulation,
  compiled from its source file (a pybind11/torch extension, built with g++
  against the installed torch, the way the reference's ``_cpu_crt.py:11-25``
  JIT-builds it).
* ``oracle/_ref/crt_cuda_ref*.so`` -- the reference's own CUDA path,
  ``src/fp_emulation/csrc/crt_kernel.cu`` (cuBLASLt batched INT8 GEMM,
  ``mod_reduce`` and ``crt_kernel``), compiled with nvcc for sm_100a the way
  ``_cuda_crt.py:11-21`` JIT-builds it, so the benchmark can time the
  reference's GPU path on the same B200 (``oracle/reference_cuda.py``).

The reference sources are read from the reference package installed in
``baseline/_ref`` (its package data carries ``csrc/``), or from the directory
named by ``FPEMU_REFERENCE_SRC`` (a reference ``src/fp_emulation``).  They are
only built where those sources are present; the compiled modules travel with
the repository so tests and the benchmark can use them where they are absent.

``-march=native`` from the reference's flags is replaced by a portable x86-64
level because the module is compiled in one container and run on another
host.  The CRT is ISO C++ without contraction either way, so the bits do not
depend on it.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent


def reference_src() -> Path:
    """The reference's ``fp_emulation`` package directory (holding csrc/)."""
    env = os.environ.get("FPEMU_REFERENCE_SRC")
    return Path(env) if env else REPO / "baseline" / "_ref" / "fp_emulation"


def gcc_libdir() -> str:
    """gcc's own library directory (libgomp.so lives there, off the default link path)."""
    out = subprocess.run(["gcc", "-print-file-name=libgomp.so"], capture_output=True, text=True).stdout.strip()
    return os.path.dirname(out) if out and os.path.isabs(out) else ""


def _env():
    env = dict(os.environ)
    lib = gcc_libdir()
    if lib:
        env["LIBRARY_PATH"] = lib + (":" + env["LIBRARY_PATH"] if env.get("LIBRARY_PATH") else "")
    return env


def build_oracle_lib(force: bool = False) -> Path:
    out = HERE / "_build" / "libcrt_oracle.so"
    src = HERE / "crt_oracle.c"
    if out.exists() and not force and out.stat().st_mtime >= src.stat().st_mtime:
        return out
    out.parent.mkdir(exist_ok=True)
    cmd = ["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared",
           str(src), "-o", str(out), "-lm", "-lgomp"]
    subprocess.run(cmd, check=True, env=_env())
    return out


def ref_module_path() -> Path | None:
    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    p = HERE / "_ref" / f"crt_cpu_ref{suffix}"
    return p if p.exists() else None


def build_ref_crt(force: bool = False) -> Path | None:
    """Compile the reference's crt_reconstruct.cpp into oracle/_ref (if its source exists)."""
    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    out = HERE / "_ref" / f"crt_cpu_ref{suffix}"
    REF_CRT = reference_src() / "csrc" / "crt_reconstruct.cpp"
    if not REF_CRT.exists():
        return out if out.exists() else None
    if out.exists() and not force:
        return out
    out.parent.mkdir(exist_ok=True)
    import torch
    from torch.utils import cpp_extension as ce

    inc = [f"-I{p}" for p in ce.include_paths()] + [f"-I{sysconfig.get_paths()['include']}"]
    libdir = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = (["g++", "-O3", "-march=x86-64-v2", "-fopenmp", "-fPIC", "-shared", "-std=c++17",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=crt_cpu_ref",
            "-DTORCH_API_INCLUDE_EXTENSION_H"] + inc +
           [str(REF_CRT), "-o", str(out), f"-L{libdir}", "-lc10", "-ltorch", "-ltorch_cpu",
            "-ltorch_python", "-lgomp", f"-Wl,-rpath,{libdir}"])
    subprocess.run(cmd, check=True, env=_env())
    return out


def ref_cuda_module_path() -> Path | None:
    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    p = HERE / "_ref" / f"crt_cuda_ref{suffix}"
    return p if p.exists() else None


def build_ref_cuda(force: bool = False) -> Path | None:
    """Compile the reference's crt_kernel.cu into oracle/_ref (if its source exists):
    nvcc for sm_100a with torch's extension flags, linked to cuBLASLt."""
    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    out = HERE / "_ref" / f"crt_cuda_ref{suffix}"
    src = reference_src() / "csrc" / "crt_kernel.cu"
    if not src.exists():
        return out if out.exists() else None
    if out.exists() and not force and out.stat().st_mtime >= src.stat().st_mtime:
        return out
    out.parent.mkdir(exist_ok=True)
    import torch
    from torch.utils import cpp_extension as ce

    torch_inc = os.path.join(os.path.dirname(torch.__file__), "include")
    inc = [torch_inc, os.path.join(torch_inc, "torch", "csrc", "api", "include"), sysconfig.get_paths()["include"]]
    libdir = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    nvcc = os.path.join(ce.CUDA_HOME or "/usr/local/cuda", "bin", "nvcc")
    cmd = ([nvcc, "-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
            "-Xcompiler", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=crt_cuda_ref",
            "-DTORCH_API_INCLUDE_EXTENSION_H"] + list(ce.COMMON_NVCC_FLAGS) + [f"-I{p}" for p in inc] +
           [str(src), "-o", str(out), f"-L{libdir}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
            "-ltorch_cuda", "-ltorch_python", "-lcublasLt", f"-Xlinker=-rpath={libdir}"])
    subprocess.run(cmd, check=True, env=_env())
    return out


def load_ref_crt():
    """Import the compiled reference CRT module, or return None if it was never built."""
    p = ref_module_path()
    if p is None:
        return None
    import importlib.util

    import torch  # noqa: F401  (the module links against libtorch)

    spec = importlib.util.spec_from_file_location("crt_cpu_ref", str(p))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build_oracle_lib(force="--force" in sys.argv))
    print(build_ref_crt(force="--force" in sys.argv))
    print(build_ref_cuda(force="--force" in sys.argv))
