"""Build the in-tree libraries of the B200 NVFP4 Gated DeltaNet path.

    python blackwell-kernel-sm_120_b200/build.py            # product libraries
    python blackwell-kernel-sm_120_b200/build.py --oracle   # + the CPU oracle (test infrastructure)

Outputs (git-ignored, carried to GPU hosts with the tree):
  lib/libgdn_b200.so      C ABI (include/gdn_b200.h), every kernel for sm_100a
  lib/libgdn_sm120_op.so  torch custom ops in the reference's `gdn_sm120`
                          namespace (src/ops/gdn_op.cu:103-110 of the reference),
                          linked against libgdn_b200.so
  lib/libgdn_sm120_plugin.so  the TensorRT-LLM plugin face (include/gdn_trt_plugin.h)
                          over the C ABI, linked against libgdn_b200.so

nvcc cross-compiles for sm_100a without a GPU.  Objects are rebuilt only when a
source or header is newer than the object.
"""
from __future__ import annotations

import argparse
import os
import pathlib
import shutil
import subprocess
import sys
import sysconfig

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
OBJ = PKG / "_build"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}",
]

CUDA_SOURCES = [
    CSRC / "runtime" / "status.cu",
    CSRC / "runtime" / "pool.cu",
    CSRC / "runtime" / "peer_allreduce.cu",
    CSRC / "kernel" / "nvfp4_kernels.cu",
    CSRC / "kernel" / "gdn_decode.cu",
    CSRC / "kernel" / "gdn_prefill.cu",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _headers() -> list[pathlib.Path]:
    return list(CSRC.rglob("*.cuh")) + list(CSRC.rglob("*.h")) + list(INCLUDE.glob("*.h"))


def _stale(target: pathlib.Path, deps: list[pathlib.Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def build_capi(verbose: bool = False, ptxas_verbose: bool = False) -> pathlib.Path:
    nvcc = _nvcc()
    OBJ.mkdir(exist_ok=True)
    LIB.mkdir(exist_ok=True)
    headers = _headers()
    objs = []
    for src in CUDA_SOURCES:
        if not src.exists():
            continue
        obj = OBJ / (src.stem + ".o")
        if _stale(obj, [src, *headers]) or ptxas_verbose:
            extra = ["-Xptxas", "-v"] if ptxas_verbose else []
            _run([nvcc, *NVCC_FLAGS, *extra, "-c", src, "-o", obj], verbose)
        objs.append(obj)
    so = LIB / "libgdn_b200.so"
    if _stale(so, objs):
        # Static CUDA runtime: the library loads without LD_LIBRARY_PATH and
        # interoperates with any runtime through driver-level streams/pointers.
        _run([nvcc, *ARCH, "-shared", "-o", so, *objs, "-Xcompiler", "-fPIC"], verbose)
    return so


def build_torch_op(verbose: bool = False) -> pathlib.Path | None:
    """libgdn_sm120_op.so: torch.ops.gdn_sm120.* over the C ABI."""
    try:
        import torch  # noqa: F401
        from torch.utils import cpp_extension
    except Exception as exc:  # pragma: no cover - torch is part of the image
        print(f"torch unavailable, skipping torch op: {exc}", file=sys.stderr)
        return None
    src = CSRC / "ops" / "gdn_torch_op.cpp"
    so = LIB / "libgdn_sm120_op.so"
    capi = LIB / "libgdn_b200.so"
    if not _stale(so, [src, capi, *_headers()]):
        return so
    inc = cpp_extension.include_paths(device_type="cuda")
    libdirs = cpp_extension.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           f"-I{INCLUDE}", *[f"-I{p}" for p in inc], f"-I{sysconfig.get_paths()['include']}",
           "-I/usr/local/cuda/include", src, "-o", so,
           *[f"-L{p}" for p in libdirs], f"-L{LIB}", "-lgdn_b200", "-lc10", "-lc10_cuda", "-ltorch_cpu",
           "-ltorch_cuda", "-ltorch", "-Wl,-rpath,$ORIGIN", *[f"-Wl,-rpath,{p}" for p in libdirs]]
    _run(cmd, verbose)
    return so


def build_plugin(verbose: bool = False) -> pathlib.Path:
    """libgdn_sm120_plugin.so: the plugin class of include/gdn_trt_plugin.h and
    its C entry points; needs no TensorRT."""
    src = CSRC / "plugin" / "gdn_trt_plugin.cpp"
    so = LIB / "libgdn_sm120_plugin.so"
    capi = LIB / "libgdn_b200.so"
    if not _stale(so, [src, capi, *_headers()]):
        return so
    cuda_lib = pathlib.Path("/usr/local/cuda/lib64")
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden", "-Wall", f"-I{INCLUDE}",
           "-I/usr/local/cuda/include", src, "-o", so, f"-L{LIB}", "-lgdn_b200", f"-L{cuda_lib}", "-lcudart",
           "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{cuda_lib}"]
    _run(cmd, verbose)
    return so


def reference_dir() -> pathlib.Path:
    """The reference checkout: $GDN_REFERENCE_DIR, else a checkout named
    `reference` beside this repository."""
    env = os.environ.get("GDN_REFERENCE_DIR")
    return pathlib.Path(env) if env else ROOT.parent / "reference"


def build_oracle(verbose: bool = False) -> None:
    """The CPU oracle (test infrastructure); the reference leg only where the
    reference checkout exists."""
    oracle = ROOT / "oracle"
    _run(["make", "-C", oracle, "-s"], verbose)
    ref = reference_dir()
    if (ref / "src" / "kernel" / "gdn_state_update_ref.cu").exists():
        _run(["make", "-C", oracle, "-s", "ref", f"REF={ref}"], verbose)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--oracle", action="store_true")
    ap.add_argument("--no-torch", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print ptxas register/smem usage")
    args = ap.parse_args()
    build_capi(args.verbose, args.ptxas)
    build_plugin(args.verbose)
    if not args.no_torch:
        build_torch_op(args.verbose)
    if args.oracle:
        build_oracle(args.verbose)


if __name__ == "__main__":
    main()
