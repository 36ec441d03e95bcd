// Host-side plumbing shared by every operator: status codes with a per-thread detail
// message, the per-device context (SM count, device status word, the driver's tensor-map
// encoder), and helpers to encode TMA descriptors.
#pragma once

#include "cuvit_b200.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <string>
#include <utility>

namespace cuvit::host {

// Records a detail message for the calling thread and returns the status unchanged.
int fail(int status, const std::string& message);
// Turns a CUDA error into CUVIT_CUDA_ERROR with the call text; CUVIT_OK on success.
int check_cuda(cudaError_t error, const char* what);
void clear_error();

#define CUVIT_TRY_CUDA(expression)                                                                 \
    do {                                                                                           \
        const int cuvit_try_status_ = ::cuvit::host::check_cuda((expression), #expression);       \
        if (cuvit_try_status_ != CUVIT_OK) {                                                       \
            return cuvit_try_status_;                                                              \
        }                                                                                          \
    } while (0)

#define CUVIT_TRY(expression)                                                                      \
    do {                                                                                           \
        const int cuvit_try_status_ = (expression);                                                \
        if (cuvit_try_status_ != CUVIT_OK) {                                                       \
            return cuvit_try_status_;                                                              \
        }                                                                                          \
    } while (0)

// After a launch: map cudaGetLastError() to a status and count the launch.
int after_launch(const char* kernel);

// Whether kernels are launched with programmatic stream serialization (dependent launch), so
// that a kernel's prologue overlaps the tail of the one before it: inside a DependentLaunch
// scope that enables it on this thread, or always / never when the environment sets
// CUVIT_PDL=1 / 0. The model runner enables it for small passes only: ViT-Ti/16 TF32 at
// batch 32 ran 5% faster with it, while the power-capped ViT-B/16 BF16 pass at batch 256 ran
// about 3% slower (the overlap raises power draw, and the clock drops).
bool pdl_enabled();

class DependentLaunch {
  public:
    explicit DependentLaunch(bool enable);
    ~DependentLaunch();
    DependentLaunch(const DependentLaunch&) = delete;
    DependentLaunch& operator=(const DependentLaunch&) = delete;

  private:
    bool previous_;
};

// Launches a kernel of this library with the programmatic-stream-serialization attribute
// when enabled (every kernel here waits on griddepcontrol before touching global memory).
// A launch error surfaces through cudaGetLastError() in the caller's after_launch().
template <typename... KernelArgs, typename... Args>
void pdl_launch(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem,
                cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t config{};
    config.gridDim = grid;
    config.blockDim = block;
    config.dynamicSmemBytes = smem;
    config.stream = stream;
    cudaLaunchAttribute attribute{};
    attribute.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute.val.programmaticStreamSerializationAllowed = 1;
    if (pdl_enabled()) {
        config.attrs = &attribute;
        config.numAttrs = 1;
    }
    cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

// Order in which launches made on this thread walk their output tiles, rows or (image, head)
// pairs: first to last (the default), or last to first while a ReverseSweep is alive. Results
// do not depend on it. The model runner alternates it from one launch to the next, so each
// kernel starts on the rows the previous one wrote last, which are still in L2.
bool reverse_sweep();

class ReverseSweep {
  public:
    explicit ReverseSweep(bool reverse);
    ~ReverseSweep();
    ReverseSweep(const ReverseSweep&) = delete;
    ReverseSweep& operator=(const ReverseSweep&) = delete;

  private:
    bool previous_;
};

struct DeviceContext {
    int device = -1;
    int sm_count = 0;
    int major = 0;
    int minor = 0;
    size_t max_smem_optin = 0;
    unsigned* status = nullptr; // device address of the status word
};

// Context of the current device, initialised on first use (thread-safe).
int current_context(const DeviceContext** context);

// Reads the current device's status word without clearing it (after the caller has
// synchronized the work it wants covered). CUVIT_DEVICE_TIMEOUT when a bounded wait gave up.
int peek_device_status();

// True for sm_100 parts, where the tcgen05 kernels can run.
bool is_blackwell(const DeviceContext& context);

// Runs setup(device) once per (key, current device) and returns its result, then and on every
// later call for that pair. Kernel attributes (the dynamic shared-memory limit) and occupancy
// are per device: a process driving several GPUs must set them on each, not once per process.
cudaError_t once_per_device(const void* key, const std::function<cudaError_t(int device)>& setup);

// Raises kernel's dynamic shared-memory limit to `bytes` on the current device (once per
// device).
cudaError_t allow_dynamic_smem(const void* kernel, int bytes);

using TensorMapEncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                       const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                       const cuuint32_t*, CUtensorMapInterleave,
                                       CUtensorMapSwizzle, CUtensorMapL2promotion,
                                       CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver, fetched through the runtime's entry-point query.
int tensor_map_encoder(TensorMapEncodeFn* function);

// A strided tensor of up to 4 dimensions, innermost first. strides_bytes[i] is the distance
// between consecutive indices of dimension i+1.
struct TmaTensor {
    const void* base = nullptr;
    CUtensorMapDataType type = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    int element_bytes = 4;
    int rank = 2;
    uint64_t dims[4] = {1, 1, 1, 1};
    uint64_t strides_bytes[3] = {0, 0, 0};
    uint32_t box[4] = {1, 1, 1, 1};
    // 16-byte chunks swizzled over 128-byte rows, or 32-byte chunks (the only smem layout
    // the tensor core accepts for MN-major 32-bit operands).
    CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B;
};

// Whether TMA can describe the tensor: 16-byte aligned base, strides multiples of 16 bytes
// and below 2^40, extents below 2^32, box inner extent of at most 128 bytes.
bool tma_describable(const TmaTensor& tensor);

// Encodes a 128-byte-swizzled tiled descriptor (zero fill out of bounds).
int encode_tma(const TmaTensor& tensor, CUtensorMap* map);

} // namespace cuvit::host
