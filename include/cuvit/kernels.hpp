// cuvit/kernels.hpp -- Cu-Vit's C++ operator API (reference: include/cuvit/kernels.hpp) on
// top of the B200 library's C ABI (cuvit_b200.h).
//
// Same namespace, types, function names, signatures and default arguments as the
// reference, and the same exceptions: std::invalid_argument for bad arguments,
// std::length_error past the CUDA grid limit, cuvit::CudaError for a failed launch. Code
// written against the reference recompiles unchanged and links against libcuvit_b200.so.
//
// launch_gemm runs in the library's process-wide math mode, CUVIT_MATH_FP32 by default:
// FP32-faithful products on the tensor cores (3xTF32), within the reference's FP32
// tolerances. set_gemm_math(CUVIT_MATH_TF32) trades that for one TF32 pass.
#pragma once

#include "cuvit/cuda_check.hpp"
#include "cuvit_b200.h"

#include <cuda_runtime_api.h>

#include <cstdint>
#include <stdexcept>
#include <string>

namespace cuvit {

/// How the right-hand operand of a GEMM is stored (reference kernels.hpp:16-21).
enum class GemmLayout {
    /// B is [K, N]: C[m][n] = sum_k A[m][k] * B[k][n].
    kNoTranspose,
    /// B is [N, K]: C[m][n] = sum_k A[m][k] * B[n][k].
    kTransposed,
};

/// What a GEMM does to each result before storing it (reference kernels.hpp:30-36).
struct GemmEpilogue {
    bool accumulate = false;
    bool gelu = false;
};

/// Which batch element a GEMM instance works on (reference kernels.hpp:46-59).
struct GemmBatch {
    int count = 1;
    std::int64_t stride_a = 0;
    std::int64_t stride_b = 0;
    std::int64_t stride_c = 0;
    int inner = 0;
    std::int64_t outer_stride_a = 0;
    std::int64_t outer_stride_b = 0;
    std::int64_t outer_stride_c = 0;
};

/// A batched GEMM with optional bias, scale and epilogue (reference kernels.hpp:74-85).
struct GemmProblem {
    int m = 0;
    int n = 0;
    int k = 0;
    GemmLayout layout = GemmLayout::kNoTranspose;
    float alpha = 1.0F;
    int lda = 0;
    int ldb = 0;
    int ldc = 0;
    GemmBatch batch;
    GemmEpilogue epilogue;
};

[[nodiscard]] inline GemmProblem gemm_problem(int m, int n, int k, GemmLayout layout) {
    GemmProblem problem;
    problem.m = m;
    problem.n = n;
    problem.k = k;
    problem.layout = layout;
    return problem;
}

namespace detail {

/// Maps a C-ABI status to the exception the reference's launcher would have thrown.
inline void raise_on(int status) {
    if (status == CUVIT_OK) {
        return;
    }
    const std::string message = cuvit_last_error_message();
    switch (status) {
    case CUVIT_INVALID_ARGUMENT:
        throw std::invalid_argument(message);
    case CUVIT_LENGTH_ERROR:
        throw std::length_error(message);
    case CUVIT_CUDA_ERROR:
    case CUVIT_OUT_OF_MEMORY:
        throw CudaError(cudaGetLastError(), message);
    default:
        throw std::runtime_error(std::string(cuvit_status_string(status)) + ": " + message);
    }
}

inline cuvit_gemm_problem to_c(const GemmProblem& p) {
    cuvit_gemm_problem c{};
    c.m = p.m;
    c.n = p.n;
    c.k = p.k;
    c.layout = p.layout == GemmLayout::kTransposed ? CUVIT_LAYOUT_TRANSPOSED
                                                   : CUVIT_LAYOUT_NO_TRANSPOSE;
    c.alpha = p.alpha;
    c.lda = p.lda;
    c.ldb = p.ldb;
    c.ldc = p.ldc;
    c.batch.count = p.batch.count;
    c.batch.stride_a = p.batch.stride_a;
    c.batch.stride_b = p.batch.stride_b;
    c.batch.stride_c = p.batch.stride_c;
    c.batch.inner = p.batch.inner;
    c.batch.outer_stride_a = p.batch.outer_stride_a;
    c.batch.outer_stride_b = p.batch.outer_stride_b;
    c.batch.outer_stride_c = p.batch.outer_stride_c;
    c.epilogue.accumulate = p.epilogue.accumulate ? 1 : 0;
    c.epilogue.gelu = p.epilogue.gelu ? 1 : 0;
    return c;
}

inline cuvit_stream_t stream_of(cudaStream_t stream) {
    return reinterpret_cast<cuvit_stream_t>(stream);
}

} // namespace detail

/// Selects launch_gemm's arithmetic: CUVIT_MATH_FP32 (default) or CUVIT_MATH_TF32.
inline void set_gemm_math(int math) { detail::raise_on(cuvit_set_math_mode(math)); }

inline void launch_gemm(const float* a, const float* b, const float* bias, float* c,
                        const GemmProblem& problem, cudaStream_t stream = nullptr) {
    const cuvit_gemm_problem p = detail::to_c(problem);
    detail::raise_on(cuvit_gemm(a, b, bias, c, &p, detail::stream_of(stream)));
}

inline void launch_layer_norm(const float* input, const float* gamma, const float* beta,
                              float* output, int rows, int columns, float epsilon = 1.0e-6F,
                              cudaStream_t stream = nullptr) {
    detail::raise_on(cuvit_layer_norm(input, gamma, beta, output, rows, columns, epsilon,
                                      detail::stream_of(stream)));
}

inline void launch_gelu(const float* input, float* output, std::int64_t count,
                        cudaStream_t stream = nullptr) {
    detail::raise_on(cuvit_gelu(input, output, count, detail::stream_of(stream)));
}

inline void launch_softmax(const float* input, float* output, int rows, int columns,
                           cudaStream_t stream = nullptr) {
    detail::raise_on(cuvit_softmax(input, output, rows, columns, detail::stream_of(stream)));
}

inline void launch_extract_patches(const float* images, float* patches, int batch, int channels,
                                   int height, int width, int patch,
                                   cudaStream_t stream = nullptr) {
    detail::raise_on(cuvit_extract_patches(images, patches, batch, channels, height, width, patch,
                                           detail::stream_of(stream)));
}

inline void launch_add(float* accumulator, const float* addend, std::int64_t count,
                       cudaStream_t stream = nullptr) {
    detail::raise_on(cuvit_add(accumulator, addend, count, detail::stream_of(stream)));
}

inline void launch_add_broadcast(float* accumulator, const float* addend, std::int64_t count,
                                 int batch, cudaStream_t stream = nullptr) {
    detail::raise_on(
        cuvit_add_broadcast(accumulator, addend, count, batch, detail::stream_of(stream)));
}

inline void launch_broadcast(float* destination, const float* source, std::int64_t count,
                             std::int64_t destination_stride, int batch,
                             cudaStream_t stream = nullptr) {
    detail::raise_on(cuvit_broadcast(destination, source, count, destination_stride, batch,
                                     detail::stream_of(stream)));
}

/// Fused Q.K^T -> softmax -> .V over a packed [batch * tokens, 3 * heads * 64] projection
/// (replaces the three launches of the reference's src/model/vit.cu:205-242).
inline void launch_attention(const void* qkv, void* context, int dtype, int batch, int tokens,
                             int heads, int head_dim, float scale, cudaStream_t stream = nullptr) {
    detail::raise_on(cuvit_attention(qkv, context, dtype, batch, tokens, heads, head_dim, scale,
                                     detail::stream_of(stream)));
}

// Device counterpart of cuvit::preprocess (include/cuvit/image.hpp of the reference, a host
// function there): `batch` interleaved 8-bit RGB images of width x height on the device,
// image_stride bytes apart (0 = packed), to the planar [batch, 3, size, size] model input,
// bit-identical to the reference's host result. Throws std::invalid_argument where the
// reference does (empty image, size <= 0, crop fraction outside (0, 1], zero deviation).
inline void launch_preprocess(const std::uint8_t* pixels, int batch, int width, int height,
                              const cuvit_preprocessing& settings, float* tensor,
                              std::int64_t image_stride = 0, cudaStream_t stream = nullptr) {
    detail::raise_on(cuvit_preprocess(pixels, batch, width, height, image_stride, &settings,
                                      tensor, detail::stream_of(stream)));
}

} // namespace cuvit
