"""Build ``libxops_b200.so`` (all sm_100a kernels + the C ABI) in-tree.

``python -m torch_npu_ops_b200.build [--force] [-j N]``

Each ``csrc/*.cu`` is compiled by nvcc for ``sm_100a`` into ``_build/`` and
the objects are linked into ``torch_npu_ops_b200/libxops_b200.so``.  A file is
rebuilt when it, or any header under ``csrc/`` or ``include/``, is newer than
its object.  No torch headers are involved: the library is plain CUDA C++
with an ``extern "C"`` surface.
"""

import argparse
import concurrent.futures as cf
import glob
import os
import re
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libxops_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "-Xptxas", "-warn-spills"]


def _nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found (set NVCC or install the CUDA toolkit)")


_INC = re.compile(r'^\s*#\s*include\s*"([^"]+)"', re.M)


def _deps(path, seen=None):
    """The file and every local header it includes, transitively."""
    seen = set() if seen is None else seen
    if path in seen:
        return seen
    seen.add(path)
    with open(path) as f:
        text = f.read()
    for name in _INC.findall(text):
        for d in (os.path.dirname(path), CSRC, INCLUDE, os.path.join(CSRC, "runtime"),
                  os.path.join(CSRC, "torch_api")):
            cand = os.path.join(d, name)
            if os.path.exists(cand):
                _deps(cand, seen)
                break
    return seen


def _stale(src, obj):
    if not os.path.exists(obj):
        return True
    m = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > m for d in _deps(src))


def _compile(nvcc, src, obj, verbose):
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return src, r.returncode, r.stdout + r.stderr


def build(force=False, jobs=None, verbose=False):
    """Compile what is stale and (re)link the shared library; returns its path."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    todo = []
    objs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or _stale(s, o):
            todo.append((s, o))
    failed = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            for src, rc, out in ex.map(lambda so: _compile(nvcc, so[0], so[1], verbose), todo):
                if out.strip() and (rc != 0 or verbose):
                    sys.stderr.write(f"--- {os.path.basename(src)}\n{out}\n")
                if rc != 0:
                    failed.append(src)
    if failed:
        raise RuntimeError("nvcc failed for: " + ", ".join(os.path.basename(f) for f in failed))
    if todo or not os.path.exists(LIB):
        cmd = [nvcc, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


TORCH_API_SRCS = ["torch_api/ops_impl.cpp", "torch_api/op_register.cpp",
                  "runtime/kernel_registry.cpp", "runtime/packed_launch.cpp"]


def _ext_path():
    import sysconfig
    return os.path.join(PKG, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_torch_api(force=False, jobs=None):
    """Compile the C++ torch API (xllm::kernel::npu / npu_ops + the pybind
    module ``torch_npu_ops_b200._C``) against libtorch, linked to
    libxops_b200.so with an $ORIGIN rpath."""
    import sysconfig
    import torch
    from torch.utils import cpp_extension as ce
    out = _ext_path()
    srcs = [os.path.join(CSRC, s) for s in TORCH_API_SRCS]
    objs = [os.path.join(BUILD, "api_" + os.path.basename(s)[:-4] + ".o") for s in srcs]
    cxx = os.environ.get("CXX", "g++")
    inc = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], INCLUDE, CSRC,
                                                  os.path.join(CSRC, "torch_api"),
                                                  os.path.join(CSRC, "runtime")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    flags = ["-O2", "-std=c++17", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
             "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H", "-w"]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or _stale(s, o)]
    os.makedirs(BUILD, exist_ok=True)

    def cc(so):
        cmd = [cxx, *flags, *[f"-I{d}" for d in inc], "-c", so[0], "-o", so[1]]
        r = subprocess.run(cmd, capture_output=True, text=True)
        return so[0], r.returncode, r.stdout + r.stderr

    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or len(todo)) as ex:
            for src, rc, txt in ex.map(cc, todo):
                if rc != 0:
                    raise RuntimeError(f"g++ failed for {src}:\n{txt[-4000:]}")
    if todo or not os.path.exists(out) or os.path.getmtime(LIB) > os.path.getmtime(out):
        libdirs = ce.library_paths(device_type="cuda")
        cmd = [cxx, "-shared", "-o", out, *objs, *[f"-L{d}" for d in libdirs], "-L" + PKG,
               "-lxops_b200", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
               "-ltorch_python", "-Wl,-rpath,$ORIGIN",
               *[f"-Wl,-rpath,{d}" for d in libdirs]]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link of the torch API failed:\n" + r.stdout + r.stderr)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true", help="pass -Xptxas -v")
    ap.add_argument("--no-torch-api", action="store_true", help="skip the C++ torch API module")
    a = ap.parse_args()
    print(build(a.force, a.j, a.verbose))
    if not a.no_torch_api:
        print(build_torch_api(a.force, a.j))


if __name__ == "__main__":
    main()
