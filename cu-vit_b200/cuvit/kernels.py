"""The reference's operator API (include/cuvit/kernels.hpp) over the C ABI.

Names, argument order and meaning follow the reference's free functions: launch_gemm,
launch_layer_norm, launch_gelu, launch_softmax, launch_extract_patches, launch_add,
launch_add_broadcast, launch_broadcast; plus launch_attention, the fused replacement of
the Q.K^T -> softmax -> .V sequence. Pointers are device addresses: an int, or any object
with data_ptr() (a torch tensor). Streams are a cudaStream_t as an int, None (the legacy
default stream) or an object with a cuda_stream attribute (torch.cuda.Stream).
"""

from __future__ import annotations

import ctypes
import dataclasses

from . import _lib
from .errors import check

LAYOUT_NO_TRANSPOSE = _lib.LAYOUT_NO_TRANSPOSE
LAYOUT_TRANSPOSED = _lib.LAYOUT_TRANSPOSED
DTYPE_F32 = _lib.DTYPE_F32
DTYPE_BF16 = _lib.DTYPE_BF16
DTYPE_TF32 = _lib.DTYPE_TF32
MATH_FP32 = _lib.MATH_FP32
MATH_TF32 = _lib.MATH_TF32
MATH_BF16 = _lib.MATH_BF16


def _ptr(value) -> ctypes.c_void_p:
    if value is None:
        return ctypes.c_void_p(0)
    if hasattr(value, "data_ptr"):
        return ctypes.c_void_p(value.data_ptr())
    return ctypes.c_void_p(int(value))


def _stream(stream) -> ctypes.c_void_p:
    if stream is None:
        return ctypes.c_void_p(0)
    if hasattr(stream, "cuda_stream"):
        return ctypes.c_void_p(stream.cuda_stream)
    return ctypes.c_void_p(int(stream))


@dataclasses.dataclass
class GemmBatch:
    """reference: GemmBatch, include/cuvit/kernels.hpp:46-59."""

    count: int = 1
    stride_a: int = 0
    stride_b: int = 0
    stride_c: int = 0
    inner: int = 0
    outer_stride_a: int = 0
    outer_stride_b: int = 0
    outer_stride_c: int = 0


@dataclasses.dataclass
class GemmEpilogue:
    """reference: GemmEpilogue, include/cuvit/kernels.hpp:30-36."""

    accumulate: bool = False
    gelu: bool = False


@dataclasses.dataclass
class GemmProblem:
    """reference: GemmProblem, include/cuvit/kernels.hpp:74-85."""

    m: int = 0
    n: int = 0
    k: int = 0
    layout: int = LAYOUT_NO_TRANSPOSE
    alpha: float = 1.0
    lda: int = 0
    ldb: int = 0
    ldc: int = 0
    batch: GemmBatch = dataclasses.field(default_factory=GemmBatch)
    epilogue: GemmEpilogue = dataclasses.field(default_factory=GemmEpilogue)

    def to_c(self) -> _lib.GemmProblemC:
        b = self.batch
        return _lib.GemmProblemC(
            self.m, self.n, self.k, self.layout, self.alpha, self.lda, self.ldb, self.ldc,
            _lib.GemmBatchC(b.count, b.stride_a, b.stride_b, b.stride_c, b.inner,
                            b.outer_stride_a, b.outer_stride_b, b.outer_stride_c),
            _lib.GemmEpilogueC(int(self.epilogue.accumulate), int(self.epilogue.gelu)),
        )


def gemm_problem(m: int, n: int, k: int, layout: int) -> GemmProblem:
    """reference: gemm_problem(), include/cuvit/kernels.hpp:89-96."""
    return GemmProblem(m=m, n=n, k=k, layout=layout)


def launch_gemm(a, b, bias, c, problem: GemmProblem, stream=None) -> None:
    """reference: launch_gemm (kernels.hpp:98-99). FP32 operands, process math mode."""
    p = problem.to_c()
    check(_lib.library().cuvit_gemm(_ptr(a), _ptr(b), _ptr(bias), _ptr(c), ctypes.byref(p),
                                    _stream(stream)))


def launch_gemm_ex(a, b, bias, c, problem: GemmProblem, c_dtype: int = DTYPE_F32,
                   math: int = MATH_BF16, stream=None) -> None:
    """Typed GEMM: bf16 operands for MATH_BF16, float otherwise; C in c_dtype."""
    p = problem.to_c()
    check(_lib.library().cuvit_gemm_ex(_ptr(a), _ptr(b), _ptr(bias), _ptr(c), c_dtype, math,
                                       ctypes.byref(p), _stream(stream)))


def set_math_mode(math: int) -> None:
    check(_lib.library().cuvit_set_math_mode(math))


def get_math_mode() -> int:
    return _lib.library().cuvit_get_math_mode()


def launch_layer_norm(input, gamma, beta, output, rows: int, columns: int,
                      epsilon: float = 1.0e-6, stream=None) -> None:
    """reference: launch_layer_norm (kernels.hpp:107-109)."""
    check(_lib.library().cuvit_layer_norm(_ptr(input), _ptr(gamma), _ptr(beta), _ptr(output),
                                          rows, columns, epsilon, _stream(stream)))


def launch_layer_norm_ex(input, input_row_stride: int, gamma, beta, output, out_dtype: int,
                         output_row_stride: int, rows: int, columns: int,
                         epsilon: float = 1.0e-6, stream=None) -> None:
    check(_lib.library().cuvit_layer_norm_ex(_ptr(input), input_row_stride, _ptr(gamma),
                                             _ptr(beta), _ptr(output), out_dtype,
                                             output_row_stride, rows, columns, epsilon,
                                             _stream(stream)))


def launch_gelu(input, output, count: int, stream=None) -> None:
    """reference: launch_gelu (kernels.hpp:117-118)."""
    check(_lib.library().cuvit_gelu(_ptr(input), _ptr(output), count, _stream(stream)))


def launch_softmax(input, output, rows: int, columns: int, stream=None) -> None:
    """reference: launch_softmax (kernels.hpp:122-123)."""
    check(_lib.library().cuvit_softmax(_ptr(input), _ptr(output), rows, columns,
                                       _stream(stream)))


def launch_softmax_ex(input, output, rows: int, columns: int, row_stride: int,
                      stream=None) -> None:
    check(_lib.library().cuvit_softmax_ex(_ptr(input), _ptr(output), rows, columns, row_stride,
                                          _stream(stream)))


def launch_extract_patches(images, patches, batch: int, channels: int, height: int, width: int,
                           patch: int, stream=None) -> None:
    """reference: launch_extract_patches (kernels.hpp:137-138)."""
    check(_lib.library().cuvit_extract_patches(_ptr(images), _ptr(patches), batch, channels,
                                               height, width, patch, _stream(stream)))


def launch_extract_patches_ex(images, patches, out_dtype: int, batch: int, channels: int,
                              height: int, width: int, patch: int, stream=None) -> None:
    check(_lib.library().cuvit_extract_patches_ex(_ptr(images), _ptr(patches), out_dtype, batch,
                                                  channels, height, width, patch,
                                                  _stream(stream)))


def launch_add(accumulator, addend, count: int, stream=None) -> None:
    """reference: launch_add (kernels.hpp:141-142)."""
    check(_lib.library().cuvit_add(_ptr(accumulator), _ptr(addend), count, _stream(stream)))


def launch_add_broadcast(accumulator, addend, count: int, batch: int, stream=None) -> None:
    """reference: launch_add_broadcast (kernels.hpp:147-148)."""
    check(_lib.library().cuvit_add_broadcast(_ptr(accumulator), _ptr(addend), count, batch,
                                             _stream(stream)))


def launch_broadcast(destination, source, count: int, destination_stride: int, batch: int,
                     stream=None) -> None:
    """reference: launch_broadcast (kernels.hpp:153-154)."""
    check(_lib.library().cuvit_broadcast(_ptr(destination), _ptr(source), count,
                                         destination_stride, batch, _stream(stream)))


def launch_init_tokens(tokens, class_token, position, batch: int, tokens_per_image: int,
                       embed: int, stream=None) -> None:
    check(_lib.library().cuvit_init_tokens(_ptr(tokens), _ptr(class_token), _ptr(position),
                                           batch, tokens_per_image, embed, _stream(stream)))


def launch_convert_f32_to_bf16(input, output, count: int, stream=None) -> None:
    check(_lib.library().cuvit_convert_f32_to_bf16(_ptr(input), _ptr(output), count,
                                                   _stream(stream)))


def launch_round_to_tf32(input, output, count: int, stream=None) -> None:
    check(_lib.library().cuvit_round_to_tf32(_ptr(input), _ptr(output), count,
                                             _stream(stream)))


def launch_logits_top_k(logits, indices, values, probabilities, batch: int, classes: int,
                        k: int, stream=None) -> None:
    """reference: report_top (src/main.cpp:90-114) on the device: per row the k largest
    logits (descending; equal logits by ascending class index) with their softmax
    probabilities, into int32 / float32 / float32 arrays [batch, k]."""
    check(_lib.library().cuvit_logits_top_k(_ptr(logits), batch, classes, k, _ptr(indices),
                                            _ptr(values), _ptr(probabilities),
                                            _stream(stream)))


def launch_attention(qkv, context, dtype: int, batch: int, tokens: int, heads: int,
                     head_dim: int, scale: float, stream=None) -> None:
    """Fused Q.K^T -> softmax -> .V (replaces src/model/vit.cu:198-242)."""
    check(_lib.library().cuvit_attention(_ptr(qkv), _ptr(context), dtype, batch, tokens, heads,
                                         head_dim, scale, _stream(stream)))


def launch_preprocess(pixels, tensor, batch: int, width: int, height: int, size: int = 224,
                      crop_fraction: float = 0.9, mean=(0.5, 0.5, 0.5), stddev=(0.5, 0.5, 0.5),
                      image_stride: int = 0, stream=None) -> None:
    """Device preprocessing (replaces cuvit::preprocess, src/runtime/image.cpp:90-135):
    `batch` interleaved uint8 RGB images -> planar float [batch, 3, size, size]."""
    settings = _lib.PreprocessingC(size, crop_fraction, (ctypes.c_float * 3)(*mean),
                                   (ctypes.c_float * 3)(*stddev))
    check(_lib.library().cuvit_preprocess(_ptr(pixels), batch, width, height, image_stride,
                                          ctypes.byref(settings), _ptr(tensor),
                                          _stream(stream)))


def device_status() -> int:
    """Synchronises the current device, returns and clears its status bits (raises on a
    device-side timeout)."""
    flags = ctypes.c_uint(0)
    check(_lib.library().cuvit_device_status(ctypes.byref(flags)))
    return flags.value


def launch_count() -> int:
    return int(_lib.library().cuvit_launch_count())
