"""Builds the reference's cuBLASLt FFN extension (WAMInfer/_cublaslt_inference.cpp)
unchanged from its own source file, into baseline/_ref/ (git-ignored; it travels
to the GPU box with the working tree).  bench.py times it as the reference's
prepared-FFN GPU path on the same B200.

    python baseline/build_reference_cublaslt.py <directory holding the WAMInfer package>

The build mirrors the reference's own JIT recipe (WAMInfer/ffn.py:21-35: -O3,
the nvidia.cublas wheel's headers and libcublasLt), with an explicit sm_100a
arch list instead of the build machine's (absent) GPU.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"


def build(checkout: str) -> Path:
    import nvidia.cublas
    from torch.utils.cpp_extension import load

    source = Path(checkout) / "WAMInfer" / "_cublaslt_inference.cpp"
    if not source.exists():
        raise FileNotFoundError(source)
    OUT.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    root = Path(nvidia.cublas.__path__[0])
    load(
        name="wam_infer_ffn_v1",
        sources=[str(source)],
        extra_include_paths=[str(root / "include")],
        extra_ldflags=[str(root / "lib/libcublasLt.so.12")],
        extra_cflags=["-O3"],
        with_cuda=True,
        build_directory=str(OUT),
        verbose=False,
    )
    return OUT / "wam_infer_ffn_v1.so"


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: build_reference_cublaslt.py <directory holding the WAMInfer package>")
    print(build(sys.argv[1]))
