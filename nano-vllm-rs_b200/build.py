"""Build recipe for the in-tree libraries of this package.

  libnvb.so       CUDA kernels + C ABI (include/nvb_attention.h), sm_100a only.
  libnvb_host.so  host runtime pieces and the scheduler (include/nvb_host.h,
                  include/nvb_engine.h), plain C++.
  libnvb_model.so the Qwen3 runner around the attention path
                  (include/nvb_engine.h), CUDA + cuBLAS.

Run ``python nano-vllm-rs_b200/build.py`` or ``__graft_entry__.build()``.
Outputs go to nano-vllm-rs_b200/_lib/ (git-ignored, travels with the tree).
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "_lib"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd):
    print("+", " ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def _stale(target: Path, sources) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(s).stat().st_mtime > t for s in sources)


def build_cuda(force=False):
    LIB.mkdir(exist_ok=True)
    out = LIB / "libnvb.so"
    sources = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + [ROOT / "include" / "nvb_attention.h"]
    if force or _stale(out, sources):
        nvcc = os.environ.get("NVCC", "nvcc")
        _run([nvcc, "-std=c++17", "-O3", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
              f"-I{ROOT / 'include'}", f"-I{CSRC}", CSRC / "nvb_unity.cu", "-o", out])
    return out


def build_host(force=False):
    LIB.mkdir(exist_ok=True)
    out = LIB / "libnvb_host.so"
    src_dir = CSRC / "host"
    sources = list(src_dir.glob("*.cpp")) + list(src_dir.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    cpps = sorted(src_dir.glob("*.cpp"))
    if not cpps:
        return None
    if force or _stale(out, sources):
        cxx = os.environ.get("CXX", "g++")
        _run([cxx, "-std=c++17", "-O2", "-fPIC", "-shared", f"-I{ROOT / 'include'}", *cpps, "-o", out])
    return out


def build_model(force=False):
    """libnvb_model.so: the Qwen3 runner around the attention path (cuBLAS
    GEMMs, the layer kernels, the sampler), linked against libnvb.so and
    libnvb_host.so in the same directory."""
    LIB.mkdir(exist_ok=True)
    out = LIB / "libnvb_model.so"
    src_dir = CSRC / "model"
    cus = sorted(src_dir.glob("*.cu"))
    sources = cus + list(src_dir.glob("*.cuh")) + list((ROOT / "include").glob("*.h")) + [LIB / "libnvb.so",
                                                                                          LIB / "libnvb_host.so"]
    if force or _stale(out, sources):
        nvcc = os.environ.get("NVCC", "nvcc")
        _run([nvcc, "-std=c++17", "-O3", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
              f"-I{ROOT / 'include'}", f"-I{src_dir}", *cus, "-o", out, f"-L{LIB}", "-lnvb", "-lnvb_host",
              "-lcublas", "-Xlinker", "-rpath=$ORIGIN"])
    return out


def build_all(force=False):
    return build_cuda(force), build_host(force), build_model(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
