"""Builds the native parts of torch_kunlun_b200 in-tree.

* ``libtk_kernels.so`` -- the sm_100a CUDA kernels behind the C ABI declared
  in ``include/tk_kernels.h`` (nvcc, ``-gencode arch=compute_100a,code=sm_100a``).
* ``_C*.so`` -- the C++ PrivateUse1 backend (torch extension) that registers
  the ``kunlun`` device and calls the C ABI.

Both land next to this file so they travel with the source tree; nothing is
installed into site-packages.  Run it as a script,
``python torch_kunlun_b200/_build.py [--force]``, so that the package (and a
possibly stale extension) is not imported while the extension is rebuilt.
"""

from __future__ import annotations

import glob
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

KERNEL_SOURCES = ["capi.cu", "quant.cu", "qgemm.cu", "eltwise.cu", "rowops.cu", "conv.cu", "noalloc.cu", "attention.cu", "conv_tc.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
KERNEL_LIB = os.path.join(PKG, "libtk_kernels.so")


def _nccl_dir() -> str:
    import importlib.util
    spec = importlib.util.find_spec("nvidia.nccl")
    if spec and spec.submodule_search_locations:
        return list(spec.submodule_search_locations)[0]
    return "/usr"


NCCL_DIR = _nccl_dir()


def _newer(target: str, sources) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(s) <= t for s in sources)


def _run(cmd, cwd=None):
    print("+", " ".join(cmd), flush=True)
    subprocess.check_call(cmd, cwd=cwd)


def build_kernels(force: bool = False, verbose_ptxas: bool = False) -> str:
    srcs = [os.path.join(CSRC, s) for s in KERNEL_SOURCES]
    deps = srcs + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        [os.path.join(ROOT, "include", "tk_kernels.h")]
    if not force and _newer(KERNEL_LIB, deps):
        return KERNEL_LIB
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        [os.path.join(ROOT, "include", "tk_kernels.h")]
    objs, cmds = [], []
    for s in srcs:
        o = os.path.join(objdir, os.path.basename(s) + ".o")
        objs.append(o)
        if not force and _newer(o, [s] + headers):
            continue  # object is newer than its source and every shared header
        cmd = [NVCC, *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
               "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
               "-I", os.path.join(ROOT, "include"), "-c", s, "-o", o]
        if verbose_ptxas:
            cmd.insert(1, "-Xptxas=-v")
        cmds.append(cmd)
    # the translation units are independent: compile them concurrently
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as ex:
        list(ex.map(_run, cmds))
    _run([NVCC, *ARCH_FLAGS, "-shared", "-cudart", "shared", "-o", KERNEL_LIB, *objs,
          "-Xlinker", "-soname=libtk_kernels.so", "-Xlinker", f"-rpath,{CUDA_HOME}/lib64"])
    return KERNEL_LIB


def build_extension(force: bool = False) -> str:
    """Compile the PrivateUse1 backend (_C) against torch and libtk_kernels."""
    from torch.utils import cpp_extension

    build_kernels(force=force)
    srcs = sorted(glob.glob(os.path.join(CSRC, "host", "*.cpp")))
    if not srcs:
        return ""
    ext_suffix = sysconfig.get_config_var("EXT_SUFFIX")
    target = os.path.join(PKG, "_C" + ext_suffix)
    deps = srcs + glob.glob(os.path.join(CSRC, "host", "*.h")) + [KERNEL_LIB]
    if not force and _newer(target, deps):
        return target
    build_dir = os.path.join(PKG, "_build", "ext")
    os.makedirs(build_dir, exist_ok=True)
    # the freshly built module links libtk_kernels.so; make it resolvable for
    # the import that load() performs (the installed copy finds it via $ORIGIN)
    import ctypes
    ctypes.CDLL(KERNEL_LIB, mode=ctypes.RTLD_GLOBAL)
    cpp_extension.load(
        name="_C",
        sources=srcs,
        extra_cflags=["-O2", "-std=c++17", f"-I{os.path.join(ROOT, 'include')}",
                      f"-I{NCCL_DIR}/include", f"-I{CUDA_HOME}/include"],
        extra_ldflags=[f"-L{PKG}", "-ltk_kernels", f"-L{CUDA_HOME}/lib64", "-lcudart",
                       f"-L{NCCL_DIR}/lib", "-l:libnccl.so.2",
                       "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{NCCL_DIR}/lib",
                       f"-Wl,-rpath,{CUDA_HOME}/lib64"],
        build_directory=build_dir,
        with_cuda=False,
        is_python_module=True,
        verbose=False,
    )
    built = glob.glob(os.path.join(build_dir, "_C*.so"))
    if not built:
        raise RuntimeError("extension build produced no _C shared object")
    import shutil
    shutil.copy2(built[0], target)
    return target


def build_all(force: bool = False) -> None:
    build_kernels(force=force)
    build_extension(force=force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
