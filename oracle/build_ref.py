"""Compile the reference's decode kernels (qwen3-8b-fp8_rtx-5090/kernels/decode.cu) into oracle/_ref/.

Test infrastructure only: the result is the GPU checker for bit-exactness tests (tests/test_ref_gpu.py). The
source is read where it lies in the reference checkout; nothing is copied into this repository. This is a
direct nvcc command of our own (not the reference's JIT loader): sm_100a, -O3, the same flags the reference
passes to its JIT build (-O3 -lineinfo), torch's extension headers for its pybind11 module.
    python oracle/build_ref.py [--ref <reference checkout>/qwen3-8b-fp8_rtx-5090]
(default: refpath.engine_dir(), i.e. $QK_REFERENCE_DIR or a `reference` folder beside the repository)
"""
import argparse
import os
import subprocess
import sys
import sysconfig

import torch
from torch.utils import cpp_extension

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import refpath  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=refpath.engine_dir())
    args = ap.parse_args()
    src = os.path.join(args.ref, "kernels", "decode.cu")
    out_dir = os.path.join(HERE, "_ref")
    os.makedirs(out_dir, exist_ok=True)
    out = os.path.join(out_dir, "ref_decode.so")
    if os.path.exists(out) and os.path.getmtime(out) > os.path.getmtime(src):
        print(f"{out} is up to date")
        return
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    inc = cpp_extension.include_paths() + [sysconfig.get_paths()["include"]]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = [os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc"), "-gencode", "arch=compute_100a,code=sm_100a",
           "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-shared", "-Xcompiler", "-fPIC,-O3",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=ref_decode", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__", "-D__CUDA_NO_BFLOAT16_CONVERSIONS__",
           "-D__CUDA_NO_HALF2_OPERATORS__"]
    cmd += [f"-I{p}" for p in inc]
    cmd += [src, "-o", out, f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
            "-ltorch_python", f"-Xlinker", f"-rpath={torch_lib}"]
    print(" ".join(cmd))
    subprocess.run(cmd, check=True)


if __name__ == "__main__":
    sys.exit(main())
