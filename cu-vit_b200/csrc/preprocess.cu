// Image preprocessing on the device: the B200 counterpart of cuvit::preprocess
// (src/runtime/image.cpp:90-135), which the reference runs on the host for every image before
// copying it to the GPU. One thread per output pixel maps its (row, column) back to a source
// coordinate (resize of the shorter side to round(size / crop_fraction) and the centre crop
// folded into one affine map), samples the interleaved 8-bit RGB source bilinearly with
// edge clamping (image.cpp:39-56), scales to [0, 1] and normalises each channel, writing the
// planar [3, size, size] float tensor the model's patch gather reads.
//
// Every float operation is the reference's, in its order, with round-to-nearest intrinsics so
// no multiply-add is contracted: results are bit-identical to the reference's host code.
#include "cuvit_b200.h"
#include "ptx.cuh"
#include "runtime.hpp"

#include <cmath>
#include <cstdint>
#include <string>

namespace cuvit::pre {
namespace {

constexpr int kStripColumns = 32; // output columns per block (threadIdx.x)
constexpr int kRowsPerBlock = 8;  // rows a block covers per step (threadIdx.y)
constexpr int kThreads = kStripColumns * kRowsPerBlock;

struct Params {
    int width;
    int height;
    int size;
    long long image_stride; // bytes between consecutive source images
    float origin_x;
    float origin_y;
    float step;
    float mean[3];
    float stddev[3];
    // 1 / stddev when every stddev is a power of two (then x / stddev == x * (1 / stddev)
    // exactly: both are the one rounding of the same real number), else zeros.
    float inverse_stddev[3];
    int multiply;
};

// Exact conversions that keep the per-pixel work off the special-function (XU) pipe, which
// the conversions alone would saturate (about 26 XU operations per output pixel). An integer
// 0 <= v < 2^23 OR-ed into the mantissa of 2^23 is the float 2^23 + v, so subtracting 2^23
// leaves float(v); adding 1.5 * 2^23 to a float of magnitude below 2^22 rounds it to the
// nearest integer, held in the low mantissa bits.
__device__ __forceinline__ float small_int_to_float(uint32_t v) {
    return __fsub_rn(__uint_as_float(0x4B000000u | v), 8388608.0F);
}

// float(int(floor(x))) for |x| < 2^22 (so +0.0 where floor(x) is a zero).
__device__ __forceinline__ float floor_small(float x) {
    const float nearest = __fsub_rn(__fadd_rn(x, 12582912.0F), 12582912.0F);
    return nearest > x ? __fsub_rn(nearest, 1.0F) : nearest;
}

// The int value of an integral float f, |f| < 2^22.
__device__ __forceinline__ int integral_to_int(float f) {
    return __float_as_int(__fadd_rn(f, 12582912.0F)) - 0x4B400000;
}

// Image blockIdx.z. A block is 32 output columns (threadIdx.x) by 8 rows (threadIdx.y) of a
// column strip; a thread keeps its column, so the horizontal half of the source map (x, its
// taps and weights) is computed once, and walks the rows blockIdx.y * 8 + threadIdx.y,
// stepping gridDim.y * 8.
__global__ void __launch_bounds__(kThreads)
    preprocess_kernel(const uint8_t* __restrict__ pixels, float* __restrict__ tensor,
                      const Params p) {
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const int column = static_cast<int>(blockIdx.x) * kStripColumns + static_cast<int>(threadIdx.x);
    if (column >= p.size) {
        return;
    }
    const int image_index = static_cast<int>(blockIdx.z);
    const uint8_t* const image = pixels + static_cast<long long>(image_index) * p.image_stride;
    const int plane = p.size * p.size; // at most 46340^2 < 2^31 (checked on the host)
    float* const out = tensor + static_cast<long long>(image_index) * 3 * plane;
    const long long row_bytes = static_cast<long long>(p.width) * 3;
    // x = origin_x + (column + 0.5) * step - 0.5, left to right (image.cpp:127-128); the
    // taps (image.cpp:39-56): left = int(floor(x)), dx = x - float(left), clamped neighbours.
    const float x = __fsub_rn(
        __fadd_rn(p.origin_x,
                  __fmul_rn(__fadd_rn(small_int_to_float(static_cast<uint32_t>(column)), 0.5F),
                            p.step)),
        0.5F);
    const float left_f = floor_small(x);
    const int left = integral_to_int(left_f);
    const float dx = __fsub_rn(x, left_f);
    const float wx = __fsub_rn(1.0F, dx);
    const int c0 = 3 * min(max(left, 0), p.width - 1);
    const int c1 = 3 * min(max(left + 1, 0), p.width - 1);
    for (int row = static_cast<int>(blockIdx.y) * kRowsPerBlock + static_cast<int>(threadIdx.y);
         row < p.size; row += static_cast<int>(gridDim.y) * kRowsPerBlock) {
        const float y = __fsub_rn(
            __fadd_rn(p.origin_y,
                      __fmul_rn(__fadd_rn(small_int_to_float(static_cast<uint32_t>(row)), 0.5F),
                                p.step)),
            0.5F);
        const float top_f = floor_small(y);
        const int top = integral_to_int(top_f);
        const float dy = __fsub_rn(y, top_f);
        const float wy = __fsub_rn(1.0F, dy);
        const uint8_t* const r0 = image + min(max(top, 0), p.height - 1) * row_bytes;
        const uint8_t* const r1 = image + min(max(top + 1, 0), p.height - 1) * row_bytes;
        const int i = row * p.size + column;
#pragma unroll
        for (int channel = 0; channel < 3; ++channel) {
            const float tl = small_int_to_float(__ldg(r0 + c0 + channel));
            const float tr = small_int_to_float(__ldg(r0 + c1 + channel));
            const float bl = small_int_to_float(__ldg(r1 + c0 + channel));
            const float br = small_int_to_float(__ldg(r1 + c1 + channel));
            const float top_edge = __fadd_rn(__fmul_rn(tl, wx), __fmul_rn(tr, dx));
            const float bottom_edge = __fadd_rn(__fmul_rn(bl, wx), __fmul_rn(br, dx));
            const float sample = __fadd_rn(__fmul_rn(top_edge, wy), __fmul_rn(bottom_edge, dy));
            const float centred = __fsub_rn(__fdiv_rn(sample, 255.0F), p.mean[channel]);
            out[channel * plane + i] = p.multiply != 0
                                           ? __fmul_rn(centred, p.inverse_stddev[channel])
                                           : __fdiv_rn(centred, p.stddev[channel]);
        }
    }
}

} // namespace
} // namespace cuvit::pre

extern "C" {

void cuvit_preprocessing_default(cuvit_preprocessing* settings) {
    if (settings == nullptr) {
        return;
    }
    settings->size = 224;
    settings->crop_fraction = 0.9F;
    for (int c = 0; c < 3; ++c) {
        settings->mean[c] = 0.5F;
        settings->stddev[c] = 0.5F;
    }
}

int cuvit_preprocess(const uint8_t* pixels, int batch, int width, int height,
                     int64_t image_stride, const cuvit_preprocessing* settings, float* tensor,
                     cuvit_stream_t stream) {
    using cuvit::host::fail;
    if (settings == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "preprocessing settings cannot be null");
    }
    if (batch < 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "The batch cannot be negative");
    }
    if (batch == 0) {
        return CUVIT_OK;
    }
    // The reference's checks and messages (src/runtime/image.cpp:91-99, 116-119), all of them
    // before any work.
    if (width <= 0 || height <= 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "Cannot preprocess an empty image");
    }
    if (settings->size <= 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "The preprocessing size must be positive");
    }
    if (!(settings->crop_fraction > 0.0F) || settings->crop_fraction > 1.0F) {
        return fail(CUVIT_INVALID_ARGUMENT, "The crop fraction must lie in (0, 1]");
    }
    for (int c = 0; c < 3; ++c) {
        if (settings->stddev[c] == 0.0F) {
            return fail(CUVIT_INVALID_ARGUMENT,
                        "A preprocessing standard deviation cannot be zero");
        }
    }
    if (pixels == nullptr || tensor == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "preprocessing buffers cannot be null");
    }
    const long long packed = static_cast<long long>(width) * height * 3;
    const long long stride = image_stride == 0 ? packed : image_stride;
    if (stride < packed) {
        return fail(CUVIT_INVALID_ARGUMENT,
                    "The image stride is smaller than one interleaved RGB image");
    }
    if (batch > 65535) {
        return fail(CUVIT_LENGTH_ERROR, "preprocessing launch exceeds the CUDA grid limit");
    }
    // The device kernel's exact integer/float conversions hold coordinates below 2^22 and its
    // output plane in 32-bit indices.
    if (width >= (1 << 22) || height >= (1 << 22) || settings->size > 46340) {
        return fail(CUVIT_LENGTH_ERROR,
                    "device preprocessing takes images below 4194304 pixels a side and sizes "
                    "up to 46340");
    }

    // The source window of the output (image.cpp:103-111), on the host in float as there.
    cuvit::pre::Params p{};
    p.width = width;
    p.height = height;
    p.size = settings->size;
    p.image_stride = stride;
    const float resized =
        std::round(static_cast<float>(settings->size) / settings->crop_fraction);
    const int shorter = width < height ? width : height;
    const float scale = static_cast<float>(shorter) / resized;
    const float crop = static_cast<float>(settings->size) * scale;
    p.origin_x = (static_cast<float>(width) - crop) * 0.5F;
    p.origin_y = (static_cast<float>(height) - crop) * 0.5F;
    p.step = crop / static_cast<float>(settings->size);
    p.multiply = 1;
    for (int c = 0; c < 3; ++c) {
        p.mean[c] = settings->mean[c];
        p.stddev[c] = settings->stddev[c];
        // A power of two whose reciprocal is a normal float: dividing by it and multiplying by
        // the reciprocal give the same rounding of the same real number.
        int exponent = 0;
        const float mantissa = std::frexp(settings->stddev[c], &exponent);
        const bool power_of_two = std::fabs(mantissa) == 0.5F && exponent >= -124 &&
                                  exponent <= 126;
        p.inverse_stddev[c] = power_of_two ? 1.0F / settings->stddev[c] : 0.0F;
        p.multiply = p.multiply != 0 && power_of_two ? 1 : 0;
    }

    const cuvit::host::DeviceContext* device = nullptr;
    CUVIT_TRY(cuvit::host::current_context(&device));
    // Column strips x row groups x images; enough row groups for about four waves of
    // resident blocks, each thread then walking size / (8 * groups) rows.
    const int strips = (settings->size + cuvit::pre::kStripColumns - 1) / cuvit::pre::kStripColumns;
    const long long wanted_blocks = 4LL * device->sm_count * (2048 / cuvit::pre::kThreads);
    const long long per_group = static_cast<long long>(strips) * batch;
    long long groups = (wanted_blocks + per_group - 1) / per_group;
    const long long max_groups =
        (settings->size + cuvit::pre::kRowsPerBlock - 1) / cuvit::pre::kRowsPerBlock;
    groups = groups < 1 ? 1 : (groups > max_groups ? max_groups : groups);
    const dim3 grid(static_cast<unsigned>(strips), static_cast<unsigned>(groups),
                    static_cast<unsigned>(batch));
    const dim3 block(cuvit::pre::kStripColumns, cuvit::pre::kRowsPerBlock);
    cuvit::host::pdl_launch(cuvit::pre::preprocess_kernel, grid, block, 0,
                            reinterpret_cast<cudaStream_t>(stream), pixels, tensor, p);
    return cuvit::host::after_launch("preprocess_kernel");
}

} // extern "C"
