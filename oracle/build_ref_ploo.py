"""Build the reference's own torch extension (``PLOO``) for sm_100a.

TEST INFRASTRUCTURE ONLY: the result is the reference arm of the benchmark and
a parity target of the GPU tests, never part of the product.

The sources are used unmodified from the reference tree (permuto.cpp,
permutohedral.cu).  The nvcc flags are the reference's own (setup.py:13-18),
with its sm_86 gencode replaced by sm_100a, because an sm_86-only cubin carries
no PTX and cannot run on a B200.  The module is named ``PLOO_ref`` so that it
cannot be mistaken for the product.

usage: python build_ref_ploo.py <reference dir> <output dir>
"""
import os
import sys


def main():
    ref, out = sys.argv[1], sys.argv[2]
    os.makedirs(out, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    from torch.utils.cpp_extension import load

    load(
        name="PLOO_ref",
        sources=[os.path.join(ref, "permuto.cpp"), os.path.join(ref, "permutohedral.cu")],
        extra_cuda_cflags=["-O3", "--use_fast_math", "-std=c++17",
                           "-gencode=arch=compute_100a,code=sm_100a"],
        extra_cflags=["-O3", "-std=c++17"],
        build_directory=out,
        verbose=False,
    )


if __name__ == "__main__":
    main()
