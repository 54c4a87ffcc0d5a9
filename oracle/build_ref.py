"""TEST INFRASTRUCTURE ONLY: compile the reference's own block-diagonal CUDA kernel.

The reference ships one native file, ``flash_eq/cuda/csrc/block_diagonal.cu``
(hmblair/flash-eq), bound with pybind11 as ``_block_diagonal_cuda`` exposing
``forward`` and ``backward`` (block_diagonal.cu:1758-1761).  This script compiles
that file where it lies, for sm_100a, into ``oracle/_ref/`` so GPU parity tests
can run the reference kernel next to ours on the same inputs.  The reference's
own build system is not used; the source is not copied.

The output is git-ignored but travels to the GPU box with the working tree.
"""
from __future__ import annotations

import argparse
import os
import sys


def main() -> int:
    ap = argparse.ArgumentParser()
    here = os.path.dirname(os.path.abspath(__file__))
    default_ref = os.environ.get("FEQ_REFERENCE_ROOT") or os.path.join(os.path.dirname(os.path.dirname(here)),
                                                                        "reference")
    ap.add_argument("--ref", default=default_ref,
                    help="reference source tree ($FEQ_REFERENCE_ROOT, else 'reference' beside this repository)")
    ap.add_argument("--out", default=os.path.join(os.path.dirname(__file__), "_ref"))
    args = ap.parse_args()

    src = os.path.join(args.ref, "flash_eq", "cuda", "csrc", "block_diagonal.cu")
    if not os.path.isfile(src):
        print(f"reference kernel source not found: {src}")
        return 0
    os.makedirs(args.out, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils.cpp_extension import load

    load(
        name="_block_diagonal_cuda",
        sources=[src],
        build_directory=os.path.abspath(args.out),
        extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"],
        extra_cflags=["-O3"],
        verbose=False,
        is_python_module=True,
    )
    print("built reference kernel into", args.out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
