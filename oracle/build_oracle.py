"""Build recipe for the oracle's compiled parts.  TEST INFRASTRUCTURE ONLY.

* ``oracle/_build/libcrt_oracle.so`` -- the C restatement ``crt_oracle.c``.
* ``oracle/_ref/crt_cpu_ref*.so`` -- the reference's own CPU CRT,
  ``src/fp_emulation/csrc/crt_reconstruct.cpp`` of thezettascale/fp-emulation,
  compiled from the file where it lies in the read-only reference tree (a
  pybind11/torch extension, built here with g++ against the installed torch,
  the way the reference's ``_cpu_crt.py:11-25`` JIT-builds it).  Only built
  when that tree is present; the compiled module travels with the repository
  so tests and the benchmark can use it where the reference tree is absent.

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
REF_CRT = Path("/root/reference/src/fp_emulation/csrc/crt_reconstruct.cpp")
GCC_LIBDIR = "/usr/lib/gcc/x86_64-linux-gnu/13"  # holds libgomp.so; not on the default link path


def _env():
    env = dict(os.environ)
    env["LIBRARY_PATH"] = GCC_LIBDIR + (":" + env["LIBRARY_PATH"] if env.get("LIBRARY_PATH") else "")
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
    """Compile the reference's crt_reconstruct.cpp into oracle/_ref (if the tree exists)."""
    suffix = sysconfig.get_config_var("EXT_SUFFIX")
    out = HERE / "_ref" / f"crt_cpu_ref{suffix}"
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
