"""ctypes binding of include/cuvit_b200.h.

The shared library is built in-tree (cu-vit_b200/build.py) and loaded from cuvit/_lib/.
There is no fallback: if the library is missing, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import pathlib
import threading

# CUVIT_LIBRARY_VARIANT=timeline loads the diagnostic build whose kernels stamp a device
# timeline (cu-vit_b200/build.py --timeline); anything else loads the product library.
LIBRARY_PATH = pathlib.Path(__file__).resolve().parent / "_lib" / (
    "libcuvit_b200_timeline.so" if os.environ.get("CUVIT_LIBRARY_VARIANT") == "timeline"
    else "libcuvit_b200.so")

OK = 0
INVALID_ARGUMENT = 1
LENGTH_ERROR = 2
CUDA_ERROR = 3
DEVICE_TIMEOUT = 4
UNSUPPORTED = 5
RUNTIME_ERROR = 6
OUT_OF_MEMORY = 7

LAYOUT_NO_TRANSPOSE = 0
LAYOUT_TRANSPOSED = 1
DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_TF32 = 2
MATH_FP32 = 0
MATH_TF32 = 1
MATH_BF16 = 2


class GemmBatchC(ctypes.Structure):
    _fields_ = [
        ("count", ctypes.c_int),
        ("stride_a", ctypes.c_int64),
        ("stride_b", ctypes.c_int64),
        ("stride_c", ctypes.c_int64),
        ("inner", ctypes.c_int),
        ("outer_stride_a", ctypes.c_int64),
        ("outer_stride_b", ctypes.c_int64),
        ("outer_stride_c", ctypes.c_int64),
    ]


class GemmEpilogueC(ctypes.Structure):
    _fields_ = [("accumulate", ctypes.c_int), ("gelu", ctypes.c_int)]


class GemmProblemC(ctypes.Structure):
    _fields_ = [
        ("m", ctypes.c_int),
        ("n", ctypes.c_int),
        ("k", ctypes.c_int),
        ("layout", ctypes.c_int),
        ("alpha", ctypes.c_float),
        ("lda", ctypes.c_int),
        ("ldb", ctypes.c_int),
        ("ldc", ctypes.c_int),
        ("batch", GemmBatchC),
        ("epilogue", GemmEpilogueC),
    ]


class VitConfigC(ctypes.Structure):
    _fields_ = [
        ("image_size", ctypes.c_int),
        ("patch_size", ctypes.c_int),
        ("channels", ctypes.c_int),
        ("embed_dim", ctypes.c_int),
        ("depth", ctypes.c_int),
        ("heads", ctypes.c_int),
        ("mlp_hidden", ctypes.c_int),
        ("classes", ctypes.c_int),
        ("layer_norm_epsilon", ctypes.c_float),
    ]


class LaunchRecordC(ctypes.Structure):
    _fields_ = [
        ("kind", ctypes.c_int),
        ("layer", ctypes.c_int),
        ("flops", ctypes.c_double),
        ("bytes", ctypes.c_double),
        ("milliseconds", ctypes.c_float),
    ]


class PreprocessingC(ctypes.Structure):
    _fields_ = [("size", ctypes.c_int), ("crop_fraction", ctypes.c_float),
                ("mean", ctypes.c_float * 3), ("stddev", ctypes.c_float * 3)]


class TimelineRecordC(ctypes.Structure):
    _fields_ = [(name, ctypes.c_ulonglong) for name in (
        "grid", "first_ns", "last_ns", "warps", "cta0_entry_ns", "cta0_exit_ns",
        "cta0_entry_clock", "cta0_exit_clock")]


LAUNCH_KINDS = ["patches", "tokens", "gemm_patch", "layer_norm", "gemm_qkv", "attention",
                "gemm_proj", "gemm_fc1", "gemm_fc2", "gemm_head"]

_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); the full list of symbols include/cuvit_b200.h declares.
SIGNATURES = {
    "cuvit_status_string": (ctypes.c_char_p, [_i]),
    "cuvit_last_error_message": (ctypes.c_char_p, []),
    "cuvit_version": (_i, []),
    "cuvit_gemm_problem_init": (None, [ctypes.POINTER(GemmProblemC), _i, _i, _i, _i]),
    "cuvit_gemm": (_i, [_vp, _vp, _vp, _vp, ctypes.POINTER(GemmProblemC), _vp]),
    "cuvit_set_math_mode": (_i, [_i]),
    "cuvit_get_math_mode": (_i, []),
    "cuvit_gemm_ex": (_i, [_vp, _vp, _vp, _vp, _i, _i, ctypes.POINTER(GemmProblemC), _vp]),
    "cuvit_layer_norm": (_i, [_vp, _vp, _vp, _vp, _i, _i, _f, _vp]),
    "cuvit_layer_norm_ex": (_i, [_vp, _i64, _vp, _vp, _vp, _i, _i64, _i, _i, _f, _vp]),
    "cuvit_gelu": (_i, [_vp, _vp, _i64, _vp]),
    "cuvit_softmax": (_i, [_vp, _vp, _i, _i, _vp]),
    "cuvit_softmax_ex": (_i, [_vp, _vp, _i, _i, _i64, _vp]),
    "cuvit_extract_patches": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _vp]),
    "cuvit_extract_patches_ex": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _vp]),
    "cuvit_add": (_i, [_vp, _vp, _i64, _vp]),
    "cuvit_add_broadcast": (_i, [_vp, _vp, _i64, _i, _vp]),
    "cuvit_broadcast": (_i, [_vp, _vp, _i64, _i64, _i, _vp]),
    "cuvit_init_tokens": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "cuvit_convert_f32_to_bf16": (_i, [_vp, _vp, _i64, _vp]),
    "cuvit_round_to_tf32": (_i, [_vp, _vp, _i64, _vp]),
    "cuvit_logits_top_k": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "cuvit_attention": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _f, _vp]),
    "cuvit_device_status": (_i, [ctypes.POINTER(ctypes.c_uint)]),
    "cuvit_launch_count": (ctypes.c_longlong, []),
    "cuvit_selftest_bounded_wait": (_i, [ctypes.c_ulonglong]),
    "cuvit_vit_config_default": (None, [ctypes.POINTER(VitConfigC)]),
    "cuvit_vit_config_validate": (_i, [ctypes.POINTER(VitConfigC)]),
    "cuvit_vit_tensor_count": (_i, [ctypes.POINTER(VitConfigC)]),
    "cuvit_vit_tensor_info": (
        _i,
        [ctypes.POINTER(VitConfigC), _i, ctypes.c_char_p, _sz, ctypes.POINTER(_i64),
         ctypes.POINTER(_i)],
    ),
    "cuvit_vit_create_from_host": (
        _i, [ctypes.POINTER(VitConfigC), ctypes.POINTER(_vp), _i, _i, _i, _i, ctypes.POINTER(_vp)]
    ),
    "cuvit_vit_create_from_file": (
        _i, [ctypes.POINTER(VitConfigC), ctypes.c_char_p, _i, _i, _i, ctypes.POINTER(_vp)]
    ),
    "cuvit_vit_destroy": (_i, [_vp]),
    "cuvit_vit_forward": (_i, [_vp, _vp, _vp, _i, _vp]),
    "cuvit_vit_forward_host": (_i, [_vp, _vp, _vp, _i, _vp]),
    "cuvit_vit_forward_host_async": (_i, [_vp, _vp, _vp, _i, _vp]),
    "cuvit_vit_set_host_chunk": (_i, [_vp, _i]),
    "cuvit_vit_forward_graph": (_i, [_vp, _vp, _vp, _i, _vp]),
    "cuvit_vit_forward_profiled": (
        _i, [_vp, _vp, _vp, _i, _vp, ctypes.POINTER(LaunchRecordC), _i, ctypes.POINTER(_i)]
    ),
    "cuvit_vit_max_batch": (_i, [_vp]),
    "cuvit_vit_weight_bytes": (_sz, [_vp]),
    "cuvit_vit_activation_bytes": (_sz, [_vp]),
    "cuvit_vit_image_elements": (_sz, [_vp]),
    "cuvit_vit_host_image_bytes": (_sz, [_vp]),
    "cuvit_vit_launches_per_forward": (_i, [_vp, _i]),
    "cuvit_preprocessing_default": (None, [ctypes.POINTER(PreprocessingC)]),
    "cuvit_preprocess": (_i, [_vp, _i, _i, _i, ctypes.c_int64, ctypes.POINTER(PreprocessingC),
                              _vp, _vp]),
    "cuvit_shard": (_i, [_i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "cuvit_comm_unique_id": (_i, [_vp, _sz]),
    "cuvit_comm_create": (_i, [_vp, _i, _i, _i, ctypes.POINTER(_vp)]),
    "cuvit_comm_destroy": (_i, [_vp]),
    "cuvit_gather_logits": (_i, [_vp, _vp, _vp, _i, _i, _i, _vp]),
    "cuvit_replicas_create": (
        _i, [ctypes.POINTER(VitConfigC), ctypes.POINTER(_vp), _i, _i, _i, ctypes.POINTER(_i), _i,
             ctypes.POINTER(_vp)]
    ),
    "cuvit_replicas_destroy": (_i, [_vp]),
    "cuvit_replicas_device_count": (_i, [_vp]),
    "cuvit_replicas_forward_host": (_i, [_vp, _vp, _vp, _i]),
    "cuvit_replicas_forward": (_i, [_vp, _vp, _i, _vp, _i, _i]),
    "cuvit_timeline_available": (_i, []),
    "cuvit_timeline_reset": (_i, []),
    "cuvit_timeline_read": (_i, [ctypes.POINTER(TimelineRecordC), _i, ctypes.POINTER(_i)]),
}

_lock = threading.Lock()
_library: ctypes.CDLL | None = None


def library() -> ctypes.CDLL:
    """Loads libcuvit_b200.so once and attaches every signature. Raises when missing."""
    global _library
    with _lock:
        if _library is None:
            if not LIBRARY_PATH.exists():
                raise RuntimeError(
                    f"{LIBRARY_PATH} is not built; run __graft_entry__.build() or "
                    "python cu-vit_b200/build.py (no CPU fallback exists)"
                )
            lib = ctypes.CDLL(str(LIBRARY_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                function = getattr(lib, name)
                function.restype = restype
                function.argtypes = argtypes
            _library = lib
        return _library


def last_error() -> str:
    message = library().cuvit_last_error_message()
    return message.decode() if message else ""
