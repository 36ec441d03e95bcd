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

constexpr int kThreads = 256;

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
};

__device__ __forceinline__ float tap(const uint8_t* image, const Params& p, int column, int row,
                                     int channel) {
    column = min(max(column, 0), p.width - 1);
    row = min(max(row, 0), p.height - 1);
    return static_cast<float>(
        __ldg(image + (static_cast<long long>(row) * p.width + column) * 3 + channel));
}

// The planar output of image blockIdx.y, pixels in grid-stride order.
__global__ void __launch_bounds__(kThreads)
    preprocess_kernel(const uint8_t* __restrict__ pixels, float* __restrict__ tensor,
                      const Params p) {
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    const int image_index = static_cast<int>(blockIdx.y);
    const uint8_t* const image = pixels + static_cast<long long>(image_index) * p.image_stride;
    const long long plane = static_cast<long long>(p.size) * p.size;
    float* const out = tensor + static_cast<long long>(image_index) * 3 * plane;
    for (long long i = static_cast<long long>(blockIdx.x) * kThreads + threadIdx.x; i < plane;
         i += static_cast<long long>(gridDim.x) * kThreads) {
        const int row = static_cast<int>(i / p.size);
        const int column = static_cast<int>(i - static_cast<long long>(row) * p.size);
        // x = origin_x + (column + 0.5) * step - 0.5, left to right (image.cpp:127-128)
        const float x = __fsub_rn(
            __fadd_rn(p.origin_x, __fmul_rn(__fadd_rn(static_cast<float>(column), 0.5F), p.step)),
            0.5F);
        const float y = __fsub_rn(
            __fadd_rn(p.origin_y, __fmul_rn(__fadd_rn(static_cast<float>(row), 0.5F), p.step)),
            0.5F);
        const float fx = floorf(x);
        const float fy = floorf(y);
        const int left = static_cast<int>(fx);
        const int top = static_cast<int>(fy);
        const float dx = __fsub_rn(x, static_cast<float>(left));
        const float dy = __fsub_rn(y, static_cast<float>(top));
        const float wx = __fsub_rn(1.0F, dx);
        const float wy = __fsub_rn(1.0F, dy);
#pragma unroll
        for (int channel = 0; channel < 3; ++channel) {
            const float top_edge = __fadd_rn(__fmul_rn(tap(image, p, left, top, channel), wx),
                                             __fmul_rn(tap(image, p, left + 1, top, channel), dx));
            const float bottom_edge =
                __fadd_rn(__fmul_rn(tap(image, p, left, top + 1, channel), wx),
                          __fmul_rn(tap(image, p, left + 1, top + 1, channel), dx));
            const float sample = __fadd_rn(__fmul_rn(top_edge, wy), __fmul_rn(bottom_edge, dy));
            const float value = __fdiv_rn(sample, 255.0F);
            out[channel * plane + i] =
                __fdiv_rn(__fsub_rn(value, p.mean[channel]), p.stddev[channel]);
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
    for (int c = 0; c < 3; ++c) {
        p.mean[c] = settings->mean[c];
        p.stddev[c] = settings->stddev[c];
    }

    const cuvit::host::DeviceContext* device = nullptr;
    CUVIT_TRY(cuvit::host::current_context(&device));
    const long long plane = static_cast<long long>(settings->size) * settings->size;
    long long blocks = (plane + cuvit::pre::kThreads - 1) / cuvit::pre::kThreads;
    const long long cap = 4LL * device->sm_count * 8 / batch + 1;
    blocks = blocks < cap ? blocks : cap;
    const dim3 grid(static_cast<unsigned>(blocks), static_cast<unsigned>(batch));
    cuvit::host::pdl_launch(cuvit::pre::preprocess_kernel, grid, cuvit::pre::kThreads, 0,
                            reinterpret_cast<cudaStream_t>(stream), pixels, tensor, p);
    return cuvit::host::after_launch("preprocess_kernel");
}

} // extern "C"
