"""Build the parity checkers (test infrastructure, never the product).

* ``oracle/liboracle.so`` -- the plain-C restatement in flashlog_oracle.c.
* ``oracle/_ref/flashlog_ref_cpu*.so`` and ``oracle/_ref/flashlog_ref_csr*.so`` --
  the reference's own CPU extension (flashlog_kernel/source/flashlog.cpp) and
  CSR builder (flashlog_kernel/source/csr.cpp), compiled directly from their
  source files with g++ against torch's headers.  The reference's JIT loader is
  not used.  These are only built when the reference sources are present (the
  build container); the GPU box uses the prebuilt files, which travel with the
  repository snapshot.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))


def reference_root():
    """The reference checkout: $FLASHLOG_REFERENCE, else BASELINE.json's reference_path (None if neither)."""
    root = os.environ.get("FLASHLOG_REFERENCE")
    if not root:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                root = json.load(f).get("reference_path")
        except (OSError, ValueError):
            root = None
    return root or None


_ROOT = reference_root()
REF_SOURCE = os.environ.get("FLASHLOG_REFERENCE_SOURCE",
                            os.path.join(_ROOT, "flashlog_kernel", "source") if _ROOT else os.path.join(HERE, "_absent"))
REF_OUT = os.path.join(HERE, "_ref")
ORACLE_SO = os.path.join(HERE, "liboracle.so")


def _run(cmd):
    subprocess.run(cmd, check=True)


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_oracle(force=False):
    src = os.path.join(HERE, "flashlog_oracle.c")
    if force or _stale(ORACLE_SO, [src]):
        _run(["gcc", "-O2", "-std=c11", "-Wall", "-fPIC", "-shared", "-o", ORACLE_SO, src, "-lm"])
    return ORACLE_SO


def _torch_flags():
    import torch
    from torch.utils import cpp_extension as ce
    inc = []
    for p in ce.include_paths():
        inc += ["-I", p]
    inc += ["-I", sysconfig.get_paths()["include"]]
    libdir = ce.library_paths()[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cflags = ["-O3", "-std=c++17", "-fPIC", "-shared", "-fopenmp", "-DAT_PARALLEL_OPENMP",
              "-DTORCH_API_INCLUDE_EXTENSION_H", f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    ldflags = ["-L", libdir, "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python",
               f"-Wl,-rpath,{libdir}", "-fopenmp"]
    return inc, cflags, ldflags


def ref_module_path(name):
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(REF_OUT, name + suffix)


def build_reference(force=False):
    """Compile the reference CPU extension from its sources, if present."""
    cpu_src = os.path.join(REF_SOURCE, "flashlog.cpp")
    csr_src = os.path.join(REF_SOURCE, "csr.cpp")
    if not (os.path.exists(cpu_src) and os.path.exists(csr_src)):
        return None
    os.makedirs(REF_OUT, exist_ok=True)
    inc, cflags, ldflags = _torch_flags()
    outs = {}
    for name, src, extra in (("flashlog_ref_cpu", cpu_src, ["-I", REF_SOURCE]),
                             ("flashlog_ref_csr", csr_src, [])):
        out = ref_module_path(name)
        if force or _stale(out, [src]):
            _run(["g++", *cflags, f"-DTORCH_EXTENSION_NAME={name}", *extra, *inc, src, "-o", out, *ldflags])
        outs[name] = out
    return outs


def build_reference_cuda(force=False):
    """Compile the reference's full extension, CUDA kernels included, from its sources, if present.

    flashlog.cu goes through nvcc for sm_100a, flashlog.cpp through g++ with
    WITH_CUDA defined (which binds the *_cuda functions), and both link
    against libtorch's CUDA libraries into oracle/_ref/flashlog_ref_cuda*.so.
    This is the reference's own GPU code, used on the GPU box only to record
    fixtures of its CUDA-only paths (tests/golden/make_golden_cuda.py); the
    product never loads it.
    """
    cu_src = os.path.join(REF_SOURCE, "flashlog.cu")
    cpp_src = os.path.join(REF_SOURCE, "flashlog.cpp")
    if not (os.path.exists(cu_src) and os.path.exists(cpp_src)):
        return None
    name = "flashlog_ref_cuda"
    out = ref_module_path(name)
    if not (force or _stale(out, [cu_src, cpp_src, os.path.join(REF_SOURCE, "flashlog.h")])):
        return out
    os.makedirs(REF_OUT, exist_ok=True)
    import torch
    from torch.utils import cpp_extension as ce
    inc = []
    for p in ce.include_paths("cuda"):
        inc += ["-I", p]
    inc += ["-I", sysconfig.get_paths()["include"], "-I", REF_SOURCE]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = ["-DWITH_CUDA", "-DTORCH_API_INCLUDE_EXTENSION_H", f"-DTORCH_EXTENSION_NAME={name}",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    cu_obj = os.path.join(REF_OUT, "flashlog_cu.o")
    cpp_obj = os.path.join(REF_OUT, "flashlog_cpp.o")
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    _run([nvcc, "-c", cu_src, "-o", cu_obj, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
          "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", *defs, *inc])
    _run(["g++", "-c", cpp_src, "-o", cpp_obj, "-O3", "-std=c++17", "-fPIC", "-fopenmp", "-DAT_PARALLEL_OPENMP",
          *defs, *inc])
    libdirs = ce.library_paths("cuda")
    ld = []
    for d in libdirs:
        ld += ["-L", d, f"-Wl,-rpath,{d}"]
    _run(["g++", "-shared", "-o", out, cpp_obj, cu_obj, *ld, "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
          "-ltorch_cuda", "-ltorch_python", "-lcudart", "-fopenmp"])
    for o in (cu_obj, cpp_obj):
        os.remove(o)
    return out


def main():
    build_oracle(force="--force" in sys.argv)
    print("oracle:", ORACLE_SO)
    outs = build_reference(force="--force" in sys.argv)
    print("reference:", outs if outs else "sources not present; prebuilt files used if any")
    cu = build_reference_cuda(force="--force" in sys.argv)
    print("reference cuda:", cu if cu else "sources not present; prebuilt file used if any")


if __name__ == "__main__":
    main()
