"""cuvit -- B200 (sm_100a) implementation of Cu-Vit's hot path.

The compute lives in libcuvit_b200.so (CUDA kernels for tcgen05/TMA behind a C ABI,
include/cuvit_b200.h); this package mirrors the reference's operator and model API over it.
"""

from . import cvw, errors, kernels
from ._lib import LIBRARY_PATH, library
from .errors import (CudaError, CuvitError, DeviceTimeout, InvalidArgument, LengthError,
                     Unsupported, WeightError)
from .kernels import (GemmBatch, GemmEpilogue, GemmProblem, gemm_problem, launch_add,
                      launch_add_broadcast, launch_attention, launch_broadcast,
                      launch_extract_patches, launch_gelu, launch_gemm, launch_gemm_ex,
                      launch_layer_norm, launch_softmax)
from .vit import (PRECISION_BF16, PRECISION_FP32, PRECISION_TF32, VisionTransformer, VitConfig,
                  random_weights, tensor_specs)

__all__ = [
    "LIBRARY_PATH", "library", "cvw", "errors", "kernels",
    "CudaError", "CuvitError", "DeviceTimeout", "InvalidArgument", "LengthError", "Unsupported",
    "WeightError", "GemmBatch", "GemmEpilogue", "GemmProblem", "gemm_problem", "launch_add",
    "launch_add_broadcast", "launch_attention", "launch_broadcast", "launch_extract_patches",
    "launch_gelu", "launch_gemm", "launch_gemm_ex", "launch_layer_norm", "launch_softmax",
    "PRECISION_BF16", "PRECISION_FP32", "PRECISION_TF32", "VisionTransformer", "VitConfig",
    "random_weights", "tensor_specs",
]
