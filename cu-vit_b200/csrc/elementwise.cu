// Memory-bound operators: layer norm, softmax, GELU, residual add, broadcasts, patch
// gather, token initialisation and FP32 -> BF16 conversion. Each has a vectorised fast
// path (128-bit loads, one warp per row for the row reductions, values held in registers so
// a row is read from HBM once) and a general path for shapes or alignments it cannot take.
// Validation follows the reference launchers in src/kernels/normalization.cu:224-350.
#include "elementwise.hpp"

#include "cuvit_b200.h"
#include "ptx.cuh"
#include "runtime.hpp"

#include <cuda_bf16.h>

#include <cstdint>
#include <type_traits>

namespace cuvit::ops {
namespace {

constexpr int kThreads = 256;
constexpr int kWarp = 32;
constexpr int kRowsPerBlock = kThreads / kWarp;
constexpr int kMaxVec = 8; // float4 per lane held in registers: rows of up to 1024 floats
constexpr int kMaxSoftmaxPerLane = 32;

bool aligned(const void* pointer, int bytes) {
    return reinterpret_cast<uintptr_t>(pointer) % bytes == 0;
}

__device__ __forceinline__ float warp_sum(float value) {
#pragma unroll
    for (int offset = 16; offset > 0; offset /= 2) {
        value += __shfl_xor_sync(0xFFFFFFFFu, value, offset);
    }
    return value;
}

__device__ __forceinline__ float warp_max(float value) {
#pragma unroll
    for (int offset = 16; offset > 0; offset /= 2) {
        value = fmaxf(value, __shfl_xor_sync(0xFFFFFFFFu, value, offset));
    }
    return value;
}

__device__ __forceinline__ void store4(float* out, float4 value) {
    *reinterpret_cast<float4*>(out) = value;
}

__device__ __forceinline__ void store4(__nv_bfloat16* out, float4 value) {
    uint2 packed;
    packed.x = dev::pack_bf16x2(value.x, value.y);
    packed.y = dev::pack_bf16x2(value.z, value.w);
    *reinterpret_cast<uint2*>(out) = packed;
}

__device__ __forceinline__ void store1(float* out, float value) { *out = value; }
__device__ __forceinline__ void store1(__nv_bfloat16* out, float value) {
    *out = __float2bfloat16_rn(value);
}

// Float storage holding values rounded to the nearest TF32 value (CUVIT_DTYPE_TF32).
struct Tf32 {
    float value;
};

__device__ __forceinline__ void store4(Tf32* out, float4 value) {
    *reinterpret_cast<float4*>(out) =
        make_float4(dev::round_to_tf32(value.x), dev::round_to_tf32(value.y),
                    dev::round_to_tf32(value.z), dev::round_to_tf32(value.w));
}

__device__ __forceinline__ void store1(Tf32* out, float value) {
    out->value = dev::round_to_tf32(value);
}

bool valid_storage(int dtype) {
    return dtype == CUVIT_DTYPE_F32 || dtype == CUVIT_DTYPE_BF16 || dtype == CUVIT_DTYPE_TF32;
}

// ---- layer norm ---------------------------------------------------------------------------

// One warp per row, the row held in registers. The mean is the sum of deviations from the
// row's first element plus that element, which keeps a large common offset from swamping
// the spread (the reference's origin shift, src/kernels/normalization.cu:59-70); the
// variance is the biased mean of squared deviations from that mean.
// Sum over the kLanes lanes of an aligned group of a warp (every lane of the warp takes part).
template <int kLanes>
__device__ __forceinline__ float group_sum(float value) {
#pragma unroll
    for (int offset = kLanes / 2; offset > 0; offset /= 2) {
        value += __shfl_xor_sync(0xFFFFFFFFu, value, offset);
    }
    return value;
}

// kLanes lanes per row (32 / kLanes rows per warp), so short rows still give each lane several
// vectors in flight: 32 for rows of more than 512 floats, 16 above 256, else 8. With 32 the
// reduction order is the whole-warp one.
template <typename Out, int kLanes>
__global__ void __launch_bounds__(kThreads)
    layer_norm_warp_kernel(const float* __restrict__ input, long long in_stride,
                           const float* __restrict__ gamma, const float* __restrict__ beta,
                           Out* __restrict__ output, long long out_stride, int rows, int columns,
                           float epsilon, int reverse) {
    dev::timeline_enter();
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    constexpr int kRowsPerWarp = kWarp / kLanes;
    const int slot = (blockIdx.x * kRowsPerBlock + threadIdx.x / kWarp) * kRowsPerWarp +
                     (threadIdx.x % kWarp) / kLanes;
    const int lane = threadIdx.x % kLanes;
    // A group past the last row stays for the shuffles of the others in its warp.
    const bool valid = slot < rows;
    const int row = valid ? (reverse ? rows - 1 - slot : slot) : 0;
    const float4* const in4 = reinterpret_cast<const float4*>(input + row * in_stride);
    const int vectors = columns / 4;
    float4 x[kMaxVec];
    const float origin = valid ? __ldg(input + row * in_stride) : 0.0F;
    float sum = 0.0F;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
        const int v = lane + i * kLanes;
        if (valid && v < vectors) {
            x[i] = __ldg(in4 + v);
            sum += (x[i].x - origin) + (x[i].y - origin) + (x[i].z - origin) + (x[i].w - origin);
        }
    }
    const float mean = origin + group_sum<kLanes>(sum) / static_cast<float>(columns);
    float squares = 0.0F;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
        const int v = lane + i * kLanes;
        if (valid && v < vectors) {
            const float a = x[i].x - mean, b = x[i].y - mean, c = x[i].z - mean,
                        d = x[i].w - mean;
            squares += a * a + b * b + c * c + d * d;
        }
    }
    const float inverse =
        rsqrtf(group_sum<kLanes>(squares) / static_cast<float>(columns) + epsilon);
    const float4* const g4 = reinterpret_cast<const float4*>(gamma);
    const float4* const b4 = reinterpret_cast<const float4*>(beta);
    Out* const out = output + row * out_stride;
#pragma unroll
    for (int i = 0; i < kMaxVec; ++i) {
        const int v = lane + i * kLanes;
        if (valid && v < vectors) {
            const float4 g = __ldg(g4 + v);
            const float4 b = __ldg(b4 + v);
            float4 y;
            y.x = (x[i].x - mean) * inverse * g.x + b.x;
            y.y = (x[i].y - mean) * inverse * g.y + b.y;
            y.z = (x[i].z - mean) * inverse * g.z + b.z;
            y.w = (x[i].w - mean) * inverse * g.w + b.w;
            store4(out + 4 * v, y);
        }
    }
    dev::timeline_exit();
}

__device__ float block_sum(float value, float* scratch) {
    value = warp_sum(value);
    const int lane = threadIdx.x % kWarp;
    const int warp = threadIdx.x / kWarp;
    __syncthreads();
    if (lane == 0) {
        scratch[warp] = value;
    }
    __syncthreads();
    float total = 0.0F;
    for (int i = 0; i < static_cast<int>(blockDim.x) / kWarp; ++i) {
        total += scratch[i];
    }
    return total;
}

// General shapes: one block per row, three passes over global memory.
template <typename Out>
__global__ void __launch_bounds__(kThreads)
    layer_norm_block_kernel(const float* __restrict__ input, long long in_stride,
                            const float* __restrict__ gamma, const float* __restrict__ beta,
                            Out* __restrict__ output, long long out_stride, int columns,
                            float epsilon, int reverse) {
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    __shared__ float scratch[kThreads / kWarp];
    const long long row = reverse ? gridDim.x - 1 - blockIdx.x : blockIdx.x;
    const float* const x = input + row * in_stride;
    const float origin = x[0];
    float sum = 0.0F;
    for (int c = threadIdx.x; c < columns; c += blockDim.x) {
        sum += x[c] - origin;
    }
    const float mean = origin + block_sum(sum, scratch) / static_cast<float>(columns);
    float squares = 0.0F;
    for (int c = threadIdx.x; c < columns; c += blockDim.x) {
        const float d = x[c] - mean;
        squares += d * d;
    }
    const float inverse =
        rsqrtf(block_sum(squares, scratch) / static_cast<float>(columns) + epsilon);
    Out* const out = output + row * out_stride;
    for (int c = threadIdx.x; c < columns; c += blockDim.x) {
        store1(out + c, (x[c] - mean) * inverse * gamma[c] + beta[c]);
    }
}

// ---- softmax ------------------------------------------------------------------------------

// One warp per row, up to 1024 columns held in registers; safe in place.
__global__ void __launch_bounds__(kThreads)
    softmax_warp_kernel(const float* input, float* output, int rows, int columns,
                        long long stride) {
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const int row = blockIdx.x * kRowsPerBlock + threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    if (row >= rows) {
        return;
    }
    const float* const x = input + row * stride;
    float values[kMaxSoftmaxPerLane];
    float maximum = -INFINITY;
#pragma unroll
    for (int i = 0; i < kMaxSoftmaxPerLane; ++i) {
        const int c = lane + i * kWarp;
        values[i] = c < columns ? x[c] : -INFINITY;
        maximum = fmaxf(maximum, values[i]);
    }
    maximum = warp_max(maximum);
    float sum = 0.0F;
#pragma unroll
    for (int i = 0; i < kMaxSoftmaxPerLane; ++i) {
        const int c = lane + i * kWarp;
        values[i] = c < columns ? expf(values[i] - maximum) : 0.0F;
        sum += values[i];
    }
    const float inverse = 1.0F / warp_sum(sum);
    float* const y = output + row * stride;
#pragma unroll
    for (int i = 0; i < kMaxSoftmaxPerLane; ++i) {
        const int c = lane + i * kWarp;
        if (c < columns) {
            y[c] = values[i] * inverse;
        }
    }
}

__global__ void __launch_bounds__(kThreads)
    softmax_block_kernel(const float* input, float* output, int columns, long long stride) {
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    __shared__ float scratch[kThreads / kWarp];
    __shared__ float shared_max;
    const long long row = blockIdx.x;
    const float* const x = input + row * stride;
    float* const y = output + row * stride;
    float maximum = -INFINITY;
    for (int c = threadIdx.x; c < columns; c += blockDim.x) {
        maximum = fmaxf(maximum, x[c]);
    }
    maximum = warp_max(maximum);
    if (threadIdx.x % kWarp == 0) {
        scratch[threadIdx.x / kWarp] = maximum;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float total = scratch[0];
        for (int i = 1; i < static_cast<int>(blockDim.x) / kWarp; ++i) {
            total = fmaxf(total, scratch[i]);
        }
        shared_max = total;
    }
    __syncthreads();
    const float row_max = shared_max;
    float sum = 0.0F;
    for (int c = threadIdx.x; c < columns; c += blockDim.x) {
        sum += expf(x[c] - row_max);
    }
    const float inverse = 1.0F / block_sum(sum, scratch);
    for (int c = threadIdx.x; c < columns; c += blockDim.x) {
        y[c] = expf(x[c] - row_max) * inverse;
    }
}

// ---- elementwise --------------------------------------------------------------------------

__global__ void gelu_kernel(const float* __restrict__ input, float* __restrict__ output,
                            long long count, int vectorised) {
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (vectorised) {
        const long long vectors = count / 4;
        for (; i < vectors; i += stride) {
            const float4 x = reinterpret_cast<const float4*>(input)[i];
            reinterpret_cast<float4*>(output)[i] = make_float4(
                dev::gelu_erf(x.x), dev::gelu_erf(x.y), dev::gelu_erf(x.z), dev::gelu_erf(x.w));
        }
        for (long long j = vectors * 4 + static_cast<long long>(blockIdx.x) * blockDim.x +
                           threadIdx.x;
             j < count; j += stride) {
            output[j] = dev::gelu_erf(input[j]);
        }
    } else {
        for (; i < count; i += stride) {
            output[i] = dev::gelu_erf(input[i]);
        }
    }
}

__global__ void add_kernel(float* __restrict__ accumulator, const float* __restrict__ addend,
                           long long count, int vectorised) {
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (vectorised) {
        const long long vectors = count / 4;
        for (; i < vectors; i += stride) {
            float4 a = reinterpret_cast<float4*>(accumulator)[i];
            const float4 b = reinterpret_cast<const float4*>(addend)[i];
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
            reinterpret_cast<float4*>(accumulator)[i] = a;
        }
        for (long long j = vectors * 4 + static_cast<long long>(blockIdx.x) * blockDim.x +
                           threadIdx.x;
             j < count; j += stride) {
            accumulator[j] += addend[j];
        }
    } else {
        for (; i < count; i += stride) {
            accumulator[i] += addend[i];
        }
    }
}

__global__ void add_broadcast_kernel(float* __restrict__ accumulator,
                                     const float* __restrict__ addend, long long count,
                                     long long total) {
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += stride) {
        accumulator[i] += addend[i % count];
    }
}

__global__ void broadcast_kernel(float* __restrict__ destination,
                                 const float* __restrict__ source, long long count,
                                 long long destination_stride, long long total) {
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += stride) {
        const long long slot = i / count;
        const long long offset = i - slot * count;
        destination[slot * destination_stride + offset] = source[offset];
    }
}

// tokens[b][t][e] = pos[t][e] + (t == 0 ? cls[e] : 0). Image blockIdx.y; its elements in
// grid-stride order, so the position index is the element index itself (a 64-bit modulo per
// element held the old flat form to 0.76 of the write bandwidth).
__global__ void init_tokens_kernel(float* __restrict__ tokens, const float* __restrict__ cls,
                                   const float* __restrict__ pos, long long per_image,
                                   int embed, int vectorised) {
    dev::timeline_enter();
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long first = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    float* const image = tokens + static_cast<long long>(blockIdx.y) * per_image;
    if (vectorised) {
        const float4* const pos4 = reinterpret_cast<const float4*>(pos);
        const float4* const cls4 = reinterpret_cast<const float4*>(cls);
        float4* const image4 = reinterpret_cast<float4*>(image);
        for (long long i = first; i < per_image / 4; i += stride) {
            float4 value = __ldg(pos4 + i);
            if (i * 4 < embed) {
                const float4 c = __ldg(cls4 + i);
                value.x = c.x + value.x;
                value.y = c.y + value.y;
                value.z = c.z + value.z;
                value.w = c.w + value.w;
            }
            image4[i] = value;
        }
    } else {
        for (long long i = first; i < per_image; i += stride) {
            image[i] = i < embed ? cls[i] + pos[i] : pos[i];
        }
    }
    dev::timeline_exit();
}

__global__ void convert_bf16_kernel(const float* __restrict__ input,
                                    __nv_bfloat16* __restrict__ output, long long count) {
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += stride) {
        output[i] = __float2bfloat16_rn(input[i]);
    }
}

__global__ void round_tf32_kernel(const float* input, float* output, long long count) {
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += stride) {
        output[i] = dev::round_to_tf32(input[i]);
    }
}

// patches[b*P + p][c*pp + r*patch + q] = images[b][c][pr*patch + r][pc*patch + q]
// (src/kernels/normalization.cu:159-192). Vectorised: 4 consecutive q per thread.
template <typename Out, int Vec>
__global__ void extract_patches_kernel(const float* __restrict__ images, Out* __restrict__ patches,
                                       int channels, int height, int width, int patch,
                                       int across, int per_image, long long total) {
    dev::timeline_enter();
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const int area = patch * patch;
    const int row_length = channels * area;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
         i < total / Vec; i += stride) {
        const long long index = i * Vec;
        const int element = static_cast<int>(index % row_length);
        const long long global_patch = index / row_length;
        const long long image = global_patch / per_image;
        const int patch_index = static_cast<int>(global_patch % per_image);
        const int channel = element / area;
        const int within = element % area;
        const int local_row = within / patch;
        const int local_col = within % patch;
        const int source_row = (patch_index / across) * patch + local_row;
        const int source_col = (patch_index % across) * patch + local_col;
        const long long source =
            (image * channels + channel) * static_cast<long long>(height) * width +
            static_cast<long long>(source_row) * width + source_col;
        if constexpr (Vec == 4) {
            store4(patches + index, __ldg(reinterpret_cast<const float4*>(images + source)));
        } else {
            store1(patches + index, __ldg(images + source));
        }
    }
    dev::timeline_exit();
}

// The same gather, one block per (image, row of patches): the block reads that strip of the
// image (channels x patch rows x width) with coalesced 16-byte loads along image rows and
// writes each 4-value group to its patch, so consecutive threads write consecutive 4-value
// groups of a patch row. Needs patch and width multiples of 4. In = __nv_bfloat16 (images the
// host already rounded, with Out = __nv_bfloat16) moves 4 values as 8 bytes unchanged.
template <typename In, typename Out>
__global__ void __launch_bounds__(kThreads)
    extract_patch_rows_kernel(const In* __restrict__ images, Out* __restrict__ patches,
                              int channels, int height, int width, int patch, int across,
                              int patch_rows, int reverse) {
    dev::timeline_enter();
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const int slot = static_cast<int>(blockIdx.x);
    const int strip = reverse ? static_cast<int>(gridDim.x) - 1 - slot : slot;
    const int image = strip / patch_rows;
    const int pr = strip - image * patch_rows;
    const int area = patch * patch;
    const long long row_length = static_cast<long long>(channels) * area;
    const In* const base = images + static_cast<long long>(image) * channels * height * width +
                           static_cast<long long>(pr) * patch * width;
    Out* const out = patches + (static_cast<long long>(image) * patch_rows * across +
                                static_cast<long long>(pr) * across) * row_length;
    // Thread (x, y): the 4-pixel group x of every image row y, y + blockDim.y, ... of the strip
    // (channels * patch rows). The group's patch and place in it are fixed per thread, and the
    // row index advances without division: per-element divisions by the runtime extents held
    // the one-dimensional form to its issue rate (0.64 of the copy bandwidth).
    const int quad = static_cast<int>(threadIdx.x);
    const int column = quad * 4;
    const int pc = column / patch;
    const int q = column - pc * patch;
    const In* const source_column = base + column;
    Out* const target_column = out + pc * row_length + q;
    const int rows = channels * patch;
    const int step = static_cast<int>(blockDim.y); // <= patch (host guarantee)
    using Vector = std::conditional_t<std::is_same_v<In, float>, float4, uint2>;
    constexpr int kUnroll = 4; // loads in flight per thread before their stores
    int channel = 0;
    int r = static_cast<int>(threadIdx.y);
    for (int row = static_cast<int>(threadIdx.y); row < rows; row += step * kUnroll) {
        Vector value[kUnroll];
        Out* target[kUnroll];
        int c = channel;
        int rr = r;
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            target[u] = nullptr;
            if (row + u * step < rows) {
                value[u] = __ldg(reinterpret_cast<const Vector*>(
                    source_column + static_cast<long long>(c) * height * width +
                    static_cast<long long>(rr) * width));
                target[u] = target_column + c * area + rr * patch;
            }
            rr += step;
            if (rr >= patch) {
                rr -= patch;
                ++c;
            }
        }
        channel = c;
        r = rr;
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            if (target[u] != nullptr) {
                if constexpr (std::is_same_v<In, float>) {
                    store4(target[u], value[u]);
                } else {
                    static_assert(std::is_same_v<Out, __nv_bfloat16>,
                                  "bfloat16 images give bfloat16");
                    *reinterpret_cast<uint2*>(target[u]) = value[u];
                }
            }
        }
    }
    dev::timeline_exit();
}

// Top-k report (report_top, src/main.cpp:90-114), one warp per row: the row maximum and sum
// of exponentials, then k rounds of a warp-wide argmax over the entries that come after the
// previous pick in (logit descending, index ascending) order.
__global__ void __launch_bounds__(kThreads)
    top_k_kernel(const float* __restrict__ logits, int batch, int classes, int k,
                 int* __restrict__ indices, float* __restrict__ values,
                 float* __restrict__ probabilities) {
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const int row = blockIdx.x * kRowsPerBlock + threadIdx.x / kWarp;
    const int lane = threadIdx.x % kWarp;
    if (row >= batch) {
        return;
    }
    const float* const x = logits + static_cast<long long>(row) * classes;
    // NaN logits take no part: fmaxf drops them from the maximum, the sum skips them, and the
    // picks below never select one (every comparison with NaN is false). The sum and the
    // probabilities are double, as in report_top.
    float maximum = -INFINITY;
    for (int c = lane; c < classes; c += kWarp) {
        maximum = fmaxf(maximum, __ldg(x + c));
    }
    maximum = warp_max(maximum);
    double total = 0.0;
    for (int c = lane; c < classes; c += kWarp) {
        const float v = __ldg(x + c);
        if (v == v) {
            total += exp(static_cast<double>(v) - static_cast<double>(maximum));
        }
    }
#pragma unroll
    for (int offset = 16; offset > 0; offset /= 2) {
        total += __shfl_xor_sync(0xFFFFFFFFu, total, offset);
    }
    float last_value = INFINITY;
    int last_index = -1;
    const long long out = static_cast<long long>(row) * k;
    for (int r = 0; r < k; ++r) {
        float best_value = -INFINITY;
        int best_index = -1;
        for (int c = lane; c < classes; c += kWarp) {
            const float v = __ldg(x + c);
            const bool after = v < last_value || (v == last_value && c > last_index);
            if (after && (best_index < 0 || v > best_value)) {
                best_value = v;
                best_index = c;
            }
        }
#pragma unroll
        for (int offset = 16; offset > 0; offset /= 2) {
            const float other_value = __shfl_xor_sync(0xFFFFFFFFu, best_value, offset);
            const int other_index = __shfl_xor_sync(0xFFFFFFFFu, best_index, offset);
            const bool better =
                other_index >= 0 &&
                (best_index < 0 || other_value > best_value ||
                 (other_value == best_value && other_index < best_index));
            if (better) {
                best_value = other_value;
                best_index = other_index;
            }
        }
        if (lane == 0) {
            indices[out + r] = best_index;
            values[out + r] = best_index < 0 ? NAN : best_value;
            probabilities[out + r] =
                best_index < 0
                    ? 0.0F
                    : static_cast<float>(exp(static_cast<double>(best_value) -
                                             static_cast<double>(maximum)) /
                                         total);
        }
        if (best_index >= 0) {
            last_value = best_value;
            last_index = best_index;
        }
    }
}

// Grid for a grid-stride loop over count items, or -1 when the reference would have
// exceeded the CUDA grid limit (src/kernels/normalization.cu:214-220).
long long elementwise_grid(long long count) {
    const long long blocks = (count + kThreads - 1) / kThreads;
    if (blocks > 0x7FFFFFFFLL) {
        return -1;
    }
    return blocks < 148 * 16 ? blocks : 148 * 16;
}

int layer_norm_impl(const float* input, long long in_stride, const float* gamma,
                    const float* beta, void* output, int out_dtype, long long out_stride,
                    int rows, int columns, float epsilon, cudaStream_t stream) {
    if (rows == 0 || columns == 0) {
        return CUVIT_OK;
    }
    if (rows < 0 || columns < 0) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "Layer norm dimensions cannot be negative");
    }
    if (input == nullptr || gamma == nullptr || beta == nullptr || output == nullptr) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "Layer norm operands cannot be null");
    }
    if (!valid_storage(out_dtype)) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "unknown layer norm output type");
    }
    if (in_stride == 0) {
        in_stride = columns;
    }
    if (out_stride == 0) {
        out_stride = columns;
    }
    if (in_stride < columns || out_stride < columns) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "layer norm row stride is below the row");
    }
    const int out_bytes = out_dtype == CUVIT_DTYPE_BF16 ? 2 : 4;
    const int reverse = host::reverse_sweep() ? 1 : 0;
    const bool fast = columns % 4 == 0 && columns <= 4 * kWarp * kMaxVec && aligned(input, 16) &&
                      aligned(gamma, 16) && aligned(beta, 16) && in_stride % 4 == 0 &&
                      aligned(output, 4 * out_bytes) && out_stride % 4 == 0;
    const auto run = [&](auto* out) {
        using Out = std::remove_pointer_t<decltype(out)>;
        if (fast) {
            const int vectors = columns / 4;
            const int lanes = vectors > 16 * kMaxVec ? 32 : (vectors > 8 * kMaxVec ? 16 : 8);
            const int rows_per_block = kRowsPerBlock * (kWarp / lanes);
            const unsigned blocks =
                static_cast<unsigned>((rows + rows_per_block - 1) / rows_per_block);
            auto* kernel = lanes == 32   ? &layer_norm_warp_kernel<Out, 32>
                           : lanes == 16 ? &layer_norm_warp_kernel<Out, 16>
                                         : &layer_norm_warp_kernel<Out, 8>;
            host::pdl_launch(kernel, blocks, kThreads, 0, stream, input, in_stride, gamma, beta,
                             out, out_stride, rows, columns, epsilon, reverse);
        } else {
            host::pdl_launch(layer_norm_block_kernel<Out>, rows, kThreads, 0, stream, input,
                             in_stride, gamma, beta, out, out_stride, columns, epsilon,
                             reverse);
        }
    };
    if (out_dtype == CUVIT_DTYPE_BF16) {
        run(static_cast<__nv_bfloat16*>(output));
    } else if (out_dtype == CUVIT_DTYPE_TF32) {
        run(static_cast<Tf32*>(output));
    } else {
        run(static_cast<float*>(output));
    }
    return host::after_launch("layer_norm");
}

int softmax_impl(const float* input, float* output, int rows, int columns, long long stride,
                 cudaStream_t stream) {
    if (rows == 0 || columns == 0) {
        return CUVIT_OK;
    }
    if (rows < 0 || columns < 0) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "Softmax dimensions cannot be negative");
    }
    if (input == nullptr || output == nullptr) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "Softmax operands cannot be null");
    }
    if (stride == 0) {
        stride = columns;
    }
    if (stride < columns) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "softmax row stride is below the row");
    }
    if (columns <= kWarp * kMaxSoftmaxPerLane) {
        const unsigned blocks = static_cast<unsigned>((rows + kRowsPerBlock - 1) / kRowsPerBlock);
        host::pdl_launch(softmax_warp_kernel, blocks, kThreads, 0, stream, input, output, rows,
                         columns, stride);
    } else {
        host::pdl_launch(softmax_block_kernel, rows, kThreads, 0, stream, input, output,
                         columns, stride);
    }
    return host::after_launch("softmax");
}

// Block of the strip kernel: one thread per 4-pixel group of an image row (x) and as many rows
// at once as fit about 256 threads (y), at most one patch of rows.
constexpr int kMaxStripQuads = 1024;
dim3 strip_block(int width, int patch) {
    const int quads = width / 4;
    int y = kThreads / quads;
    y = y < 1 ? 1 : (y > patch ? patch : y);
    return dim3(static_cast<unsigned>(quads), static_cast<unsigned>(y));
}

int extract_patches_impl(const float* images, void* patches, int out_dtype, int batch,
                         int channels, int height, int width, int patch, cudaStream_t stream) {
    if (batch == 0) {
        return CUVIT_OK;
    }
    if (batch < 0 || channels <= 0 || height <= 0 || width <= 0 || patch <= 0) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "Patch extraction dimensions must be positive");
    }
    if (height % patch != 0 || width % patch != 0) {
        return host::fail(CUVIT_INVALID_ARGUMENT,
                          "Patch extraction needs the image to divide into whole patches");
    }
    if (images == nullptr || patches == nullptr) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "Patch extraction operands cannot be null");
    }
    if (!valid_storage(out_dtype)) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "unknown patch output type");
    }
    const int across = width / patch;
    const int per_image = (height / patch) * across;
    const long long total =
        static_cast<long long>(batch) * per_image * channels * patch * patch;
    const long long grid = elementwise_grid(total);
    if (grid < 0) {
        return host::fail(CUVIT_LENGTH_ERROR, "Elementwise launch exceeds the CUDA grid limit");
    }
    const bool bf16 = out_dtype == CUVIT_DTYPE_BF16;
    const bool vec = patch % 4 == 0 && width % 4 == 0 && aligned(images, 16) &&
                     aligned(patches, bf16 ? 8 : 16);
    const unsigned blocks = static_cast<unsigned>(grid);
    const long long strips = static_cast<long long>(batch) * (height / patch);
    const bool by_rows = vec && strips <= 0x7FFFFFFFLL && width / 4 <= kMaxStripQuads;
    const auto run = [&](auto* out) {
        using Out = std::remove_pointer_t<decltype(out)>;
        if (by_rows) {
            host::pdl_launch(extract_patch_rows_kernel<float, Out>, static_cast<unsigned>(strips),
                             strip_block(width, patch), 0, stream, images, out, channels, height,
                             width, patch, across, height / patch,
                             host::reverse_sweep() ? 1 : 0);
        } else if (vec) {
            host::pdl_launch(extract_patches_kernel<Out, 4>, blocks, kThreads, 0, stream,
                             images, out, channels, height, width, patch, across, per_image,
                             total);
        } else {
            host::pdl_launch(extract_patches_kernel<Out, 1>, blocks, kThreads, 0, stream,
                             images, out, channels, height, width, patch, across, per_image,
                             total);
        }
    };
    if (bf16) {
        run(static_cast<__nv_bfloat16*>(patches));
    } else if (out_dtype == CUVIT_DTYPE_TF32) {
        run(static_cast<Tf32*>(patches));
    } else {
        run(static_cast<float*>(patches));
    }
    return host::after_launch("extract_patches");
}

} // namespace

bool bf16_patch_gather_supported(int height, int width, int patch) {
    return patch > 0 && patch % 4 == 0 && width % 4 == 0 && height % patch == 0 &&
           width % patch == 0 && width / 4 <= kMaxStripQuads;
}

int extract_patches_bf16(const __nv_bfloat16* images, __nv_bfloat16* patches, int batch,
                         int channels, int height, int width, int patch, cudaStream_t stream) {
    if (batch == 0) {
        return CUVIT_OK;
    }
    if (batch < 0 || channels <= 0 || !bf16_patch_gather_supported(height, width, patch) ||
        !aligned(images, 8) || !aligned(patches, 8)) {
        return host::fail(CUVIT_INVALID_ARGUMENT,
                          "bfloat16 patch gather needs whole patches, patch and width multiples "
                          "of 4 and 8-byte aligned buffers");
    }
    const long long strips = static_cast<long long>(batch) * (height / patch);
    if (strips > 0x7FFFFFFFLL) {
        return host::fail(CUVIT_LENGTH_ERROR, "Elementwise launch exceeds the CUDA grid limit");
    }
    host::pdl_launch(extract_patch_rows_kernel<__nv_bfloat16, __nv_bfloat16>,
                     static_cast<unsigned>(strips), strip_block(width, patch), 0, stream, images,
                     patches,
                     channels, height, width, patch, width / patch, height / patch,
                     host::reverse_sweep() ? 1 : 0);
    return host::after_launch("extract_patches");
}

} // namespace cuvit::ops

using cuvit::host::fail;
using namespace cuvit::ops;

extern "C" {

int cuvit_layer_norm(const float* input, const float* gamma, const float* beta, float* output,
                     int rows, int columns, float epsilon, cuvit_stream_t stream) {
    return layer_norm_impl(input, columns, gamma, beta, output, CUVIT_DTYPE_F32, columns, rows,
                           columns, epsilon, reinterpret_cast<cudaStream_t>(stream));
}

int cuvit_layer_norm_ex(const float* input, int64_t input_row_stride, const float* gamma,
                        const float* beta, void* output, int out_dtype,
                        int64_t output_row_stride, int rows, int columns, float epsilon,
                        cuvit_stream_t stream) {
    return layer_norm_impl(input, input_row_stride, gamma, beta, output, out_dtype,
                           output_row_stride, rows, columns, epsilon,
                           reinterpret_cast<cudaStream_t>(stream));
}

int cuvit_softmax(const float* input, float* output, int rows, int columns,
                  cuvit_stream_t stream) {
    return softmax_impl(input, output, rows, columns, columns,
                        reinterpret_cast<cudaStream_t>(stream));
}

int cuvit_softmax_ex(const float* input, float* output, int rows, int columns,
                     int64_t row_stride, cuvit_stream_t stream) {
    return softmax_impl(input, output, rows, columns, row_stride,
                        reinterpret_cast<cudaStream_t>(stream));
}

int cuvit_gelu(const float* input, float* output, int64_t count, cuvit_stream_t stream) {
    if (count == 0) {
        return CUVIT_OK;
    }
    if (count < 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "GELU element count cannot be negative");
    }
    if (input == nullptr || output == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "GELU operands cannot be null");
    }
    const long long grid = elementwise_grid(count);
    if (grid < 0) {
        return fail(CUVIT_LENGTH_ERROR, "Elementwise launch exceeds the CUDA grid limit");
    }
    const int vec = aligned(input, 16) && aligned(output, 16) ? 1 : 0;
    cuvit::host::pdl_launch(gelu_kernel, static_cast<unsigned>(grid), kThreads, 0,
                            reinterpret_cast<cudaStream_t>(stream), input, output, count, vec);
    return cuvit::host::after_launch("gelu");
}

int cuvit_add(float* accumulator, const float* addend, int64_t count, cuvit_stream_t stream) {
    if (count == 0) {
        return CUVIT_OK;
    }
    if (count < 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "Residual add element count cannot be negative");
    }
    if (accumulator == nullptr || addend == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "Residual add operands cannot be null");
    }
    const long long grid = elementwise_grid(count);
    if (grid < 0) {
        return fail(CUVIT_LENGTH_ERROR, "Elementwise launch exceeds the CUDA grid limit");
    }
    const int vec = aligned(accumulator, 16) && aligned(addend, 16) ? 1 : 0;
    cuvit::host::pdl_launch(add_kernel, static_cast<unsigned>(grid), kThreads, 0,
                            reinterpret_cast<cudaStream_t>(stream), accumulator, addend, count,
                            vec);
    return cuvit::host::after_launch("add");
}

int cuvit_add_broadcast(float* accumulator, const float* addend, int64_t count, int batch,
                        cuvit_stream_t stream) {
    if (count == 0 || batch == 0) {
        return CUVIT_OK;
    }
    if (count < 0 || batch < 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "Broadcast add extents cannot be negative");
    }
    if (accumulator == nullptr || addend == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "Broadcast add operands cannot be null");
    }
    const long long total = count * batch;
    const long long grid = elementwise_grid(total);
    if (grid < 0) {
        return fail(CUVIT_LENGTH_ERROR, "Elementwise launch exceeds the CUDA grid limit");
    }
    cuvit::host::pdl_launch(add_broadcast_kernel, static_cast<unsigned>(grid), kThreads, 0,
                            reinterpret_cast<cudaStream_t>(stream), accumulator, addend, count,
                            total);
    return cuvit::host::after_launch("add_broadcast");
}

int cuvit_broadcast(float* destination, const float* source, int64_t count,
                    int64_t destination_stride, int batch, cuvit_stream_t stream) {
    if (count == 0 || batch == 0) {
        return CUVIT_OK;
    }
    if (count < 0 || batch < 0 || destination_stride < count) {
        return fail(CUVIT_INVALID_ARGUMENT, "Broadcast extents are inconsistent");
    }
    if (destination == nullptr || source == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "Broadcast operands cannot be null");
    }
    const long long total = count * batch;
    const long long grid = elementwise_grid(total);
    if (grid < 0) {
        return fail(CUVIT_LENGTH_ERROR, "Elementwise launch exceeds the CUDA grid limit");
    }
    cuvit::host::pdl_launch(broadcast_kernel, static_cast<unsigned>(grid), kThreads, 0,
                            reinterpret_cast<cudaStream_t>(stream), destination, source, count,
                            destination_stride, total);
    return cuvit::host::after_launch("broadcast");
}

int cuvit_extract_patches(const float* images, float* patches, int batch, int channels,
                          int height, int width, int patch, cuvit_stream_t stream) {
    return extract_patches_impl(images, patches, CUVIT_DTYPE_F32, batch, channels, height,
                                width, patch, reinterpret_cast<cudaStream_t>(stream));
}

int cuvit_extract_patches_ex(const float* images, void* patches, int out_dtype, int batch,
                             int channels, int height, int width, int patch,
                             cuvit_stream_t stream) {
    return extract_patches_impl(images, patches, out_dtype, batch, channels, height, width,
                                patch, reinterpret_cast<cudaStream_t>(stream));
}

int cuvit_init_tokens(float* tokens, const float* class_token, const float* position,
                      int batch, int tokens_per_image, int embed, cuvit_stream_t stream) {
    if (batch == 0) {
        return CUVIT_OK;
    }
    if (batch < 0 || tokens_per_image <= 0 || embed <= 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "token initialisation extents must be positive");
    }
    if (tokens == nullptr || class_token == nullptr || position == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "token initialisation operands cannot be null");
    }
    const long long per_image = static_cast<long long>(tokens_per_image) * embed;
    if (elementwise_grid(per_image * batch) < 0 || batch > 65535) {
        return fail(CUVIT_LENGTH_ERROR, "Elementwise launch exceeds the CUDA grid limit");
    }
    const int vec = embed % 4 == 0 && aligned(tokens, 16) && aligned(class_token, 16) &&
                            aligned(position, 16)
                        ? 1
                        : 0;
    // About 16 blocks per SM in all, spread over the images (each image's row blockIdx.y).
    const long long items = vec ? per_image / 4 : per_image;
    long long across = (items + kThreads - 1) / kThreads;
    const long long share = (148LL * 16 + batch - 1) / batch;
    across = across < share ? across : share;
    const dim3 grid(static_cast<unsigned>(across < 1 ? 1 : across), static_cast<unsigned>(batch));
    cuvit::host::pdl_launch(init_tokens_kernel, grid, kThreads, 0,
                            reinterpret_cast<cudaStream_t>(stream), tokens, class_token, position,
                            per_image, embed, vec);
    return cuvit::host::after_launch("init_tokens");
}

int cuvit_convert_f32_to_bf16(const float* input, void* output, int64_t count,
                              cuvit_stream_t stream) {
    if (count == 0) {
        return CUVIT_OK;
    }
    if (count < 0 || input == nullptr || output == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "conversion arguments are invalid");
    }
    const long long grid = elementwise_grid(count);
    if (grid < 0) {
        return fail(CUVIT_LENGTH_ERROR, "Elementwise launch exceeds the CUDA grid limit");
    }
    cuvit::host::pdl_launch(convert_bf16_kernel, static_cast<unsigned>(grid), kThreads, 0,
                            reinterpret_cast<cudaStream_t>(stream), input,
                            static_cast<__nv_bfloat16*>(output), count);
    return cuvit::host::after_launch("convert_f32_to_bf16");
}

int cuvit_round_to_tf32(const float* input, float* output, int64_t count,
                        cuvit_stream_t stream) {
    if (count == 0) {
        return CUVIT_OK;
    }
    if (count < 0 || input == nullptr || output == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "rounding arguments are invalid");
    }
    const long long grid = elementwise_grid(count);
    if (grid < 0) {
        return fail(CUVIT_LENGTH_ERROR, "Elementwise launch exceeds the CUDA grid limit");
    }
    cuvit::host::pdl_launch(round_tf32_kernel, static_cast<unsigned>(grid), kThreads, 0,
                            reinterpret_cast<cudaStream_t>(stream), input, output, count);
    return cuvit::host::after_launch("round_to_tf32");
}

int cuvit_logits_top_k(const float* logits, int batch, int classes, int k, int* indices,
                       float* values, float* probabilities, cuvit_stream_t stream) {
    if (batch == 0) {
        return CUVIT_OK;
    }
    if (batch < 0 || classes <= 0 || k < 1 || k > classes) {
        return fail(CUVIT_INVALID_ARGUMENT,
                    "top-k needs a non-negative batch, positive classes and 1 <= k <= classes");
    }
    if (logits == nullptr || indices == nullptr || values == nullptr ||
        probabilities == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "top-k operands cannot be null");
    }
    const long long blocks = (static_cast<long long>(batch) + kRowsPerBlock - 1) / kRowsPerBlock;
    if (blocks > 0x7FFFFFFFLL) {
        return fail(CUVIT_LENGTH_ERROR, "Elementwise launch exceeds the CUDA grid limit");
    }
    cuvit::host::pdl_launch(top_k_kernel, static_cast<unsigned>(blocks), kThreads, 0,
                            reinterpret_cast<cudaStream_t>(stream), logits, batch, classes, k,
                            indices, values, probabilities);
    return cuvit::host::after_launch("top_k");
}

} // extern "C"
