"""FP8/FP4 conversions and FP8 scaled GEMM for PyTorch on NVIDIA B200 (sm_100a).

Importing the package registers the `fp8_mps::*` custom ops and, on a CUDA
build with a GPU, the CUDA-key overrides of aten::_to_copy, aten::copy_ and
aten::_scaled_mm (same plugin surface as the MPS package it replaces; the
`torch.backends` entry point imports it at `import torch`).
"""
import fp4_fp8_for_torch_mps.ops  # noqa: F401
