#include "runtime.hpp"

#include "ptx.cuh"

#include <algorithm>
#include <atomic>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

namespace cuvit::host {
namespace {

thread_local std::string t_last_error;
std::atomic<long long> g_launches{0};

// The device status word. One per device that loads this library; kernels receive its
// device address (from cudaGetSymbolAddress) and set bits when a bounded wait expires.
__device__ unsigned g_device_status;

constexpr int kMaxDevices = 64;
DeviceContext g_contexts[kMaxDevices];
std::once_flag g_context_once[kMaxDevices];
int g_context_status[kMaxDevices];

// One thread waits on an mbarrier that nothing ever arrives on; the bounded wait gives up
// after limit_ns, sets the status bit and the kernel returns normally.
__global__ void bounded_wait_selftest_kernel(unsigned* status, unsigned long long limit_ns) {
    __shared__ __align__(8) unsigned long long barrier;
    const uint32_t bar = cuvit::dev::smem_u32(&barrier);
    cuvit::dev::mbar_init(bar, 1);
    cuvit::dev::fence_barrier_init();
    cuvit::dev::mbar_wait(bar, 0, status, limit_ns);
}

int init_context(int device, DeviceContext* context) {
    cudaDeviceProp properties{};
    CUVIT_TRY_CUDA(cudaGetDeviceProperties(&properties, device));
    context->device = device;
    context->sm_count = properties.multiProcessorCount;
    context->major = properties.major;
    context->minor = properties.minor;
    context->max_smem_optin = properties.sharedMemPerBlockOptin;
    void* address = nullptr;
    CUVIT_TRY_CUDA(cudaGetSymbolAddress(&address, g_device_status));
    context->status = static_cast<unsigned*>(address);
    CUVIT_TRY_CUDA(cudaMemset(context->status, 0, sizeof(unsigned)));
    CUVIT_TRY_CUDA(cudaDeviceSynchronize());
    return CUVIT_OK;
}

} // namespace

int fail(int status, const std::string& message) {
    t_last_error = message;
    return status;
}

void clear_error() { t_last_error.clear(); }

int check_cuda(cudaError_t error, const char* what) {
    if (error == cudaSuccess) {
        return CUVIT_OK;
    }
    return fail(error == cudaErrorMemoryAllocation ? CUVIT_OUT_OF_MEMORY : CUVIT_CUDA_ERROR,
                std::string("CUDA call failed: ") + what + " (" + cudaGetErrorName(error) + ": " +
                    cudaGetErrorString(error) + ")");
}

int after_launch(const char* kernel) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    const cudaError_t error = cudaGetLastError();
    if (error != cudaSuccess) {
        return fail(CUVIT_CUDA_ERROR, std::string("launch of ") + kernel + " failed (" +
                                          cudaGetErrorName(error) + ": " +
                                          cudaGetErrorString(error) + ")");
    }
    return CUVIT_OK;
}

int current_context(const DeviceContext** context) {
    int device = 0;
    CUVIT_TRY_CUDA(cudaGetDevice(&device));
    if (device < 0 || device >= kMaxDevices) {
        return fail(CUVIT_UNSUPPORTED, "device ordinal out of range");
    }
    std::call_once(g_context_once[device], [device]() {
        g_context_status[device] = init_context(device, &g_contexts[device]);
    });
    if (g_context_status[device] != CUVIT_OK) {
        return fail(g_context_status[device], "device context initialisation failed");
    }
    *context = &g_contexts[device];
    return CUVIT_OK;
}

bool is_blackwell(const DeviceContext& context) { return context.major == 10; }

namespace {
std::mutex g_once_mutex;
std::map<std::pair<const void*, int>, cudaError_t> g_once_results;
} // namespace

cudaError_t once_per_device(const void* key, const std::function<cudaError_t(int device)>& setup) {
    int device = 0;
    const cudaError_t error = cudaGetDevice(&device);
    if (error != cudaSuccess) {
        return error;
    }
    const std::lock_guard<std::mutex> lock(g_once_mutex);
    const auto found = g_once_results.find({key, device});
    if (found != g_once_results.end()) {
        return found->second;
    }
    const cudaError_t result = setup(device);
    g_once_results.emplace(std::make_pair(key, device), result);
    return result;
}

cudaError_t allow_dynamic_smem(const void* kernel, int bytes) {
    return once_per_device(kernel, [kernel, bytes](int) {
        return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    });
}

int peek_device_status() {
    const DeviceContext* context = nullptr;
    CUVIT_TRY(current_context(&context));
    unsigned value = 0;
    CUVIT_TRY_CUDA(cudaMemcpy(&value, context->status, sizeof(value), cudaMemcpyDeviceToHost));
    if (value & cuvit::dev::kStatusTimeout) {
        return fail(CUVIT_DEVICE_TIMEOUT,
                    "a kernel gave up on a bounded device-side wait; outputs are undefined "
                    "(cuvit_device_status() clears the flag)");
    }
    return CUVIT_OK;
}

namespace {
thread_local bool t_reverse_sweep = false;
} // namespace

bool reverse_sweep() { return t_reverse_sweep; }

ReverseSweep::ReverseSweep(bool reverse) : previous_(t_reverse_sweep) {
    t_reverse_sweep = reverse;
}

ReverseSweep::~ReverseSweep() { t_reverse_sweep = previous_; }

thread_local bool t_dependent_launch = false;

bool pdl_enabled() {
    // CUVIT_PDL=1 or 0 decides for every launch; unset, the innermost DependentLaunch does.
    static const int forced = []() {
        const char* value = std::getenv("CUVIT_PDL");
        if (value == nullptr) {
            return -1;
        }
        return std::strcmp(value, "1") == 0 ? 1 : (std::strcmp(value, "0") == 0 ? 0 : -1);
    }();
    return forced >= 0 ? forced == 1 : t_dependent_launch;
}

DependentLaunch::DependentLaunch(bool enable) : previous_(t_dependent_launch) {
    t_dependent_launch = enable;
}

DependentLaunch::~DependentLaunch() { t_dependent_launch = previous_; }

int tensor_map_encoder(TensorMapEncodeFn* function) {
    static TensorMapEncodeFn cached = nullptr;
    static std::once_flag once;
    static int status = CUVIT_OK;
    std::call_once(once, []() {
        void* entry = nullptr;
        cudaDriverEntryPointQueryResult query{};
        const cudaError_t error =
            cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &entry, cudaEnableDefault, &query);
        if (error != cudaSuccess || query != cudaDriverEntryPointSuccess || entry == nullptr) {
            status = CUVIT_UNSUPPORTED;
            return;
        }
        cached = reinterpret_cast<TensorMapEncodeFn>(entry);
    });
    if (status != CUVIT_OK) {
        return fail(status, "cuTensorMapEncodeTiled is not available from the driver");
    }
    *function = cached;
    return CUVIT_OK;
}

bool tma_describable(const TmaTensor& tensor) {
    const auto base = reinterpret_cast<uintptr_t>(tensor.base);
    if (base % 16 != 0 || tensor.rank < 1 || tensor.rank > 4) {
        return false;
    }
    for (int dim = 0; dim < tensor.rank; ++dim) {
        if (tensor.dims[dim] == 0 || tensor.dims[dim] >= (1ull << 32)) {
            return false;
        }
        if (tensor.box[dim] == 0 || tensor.box[dim] > 256) {
            return false;
        }
    }
    for (int dim = 0; dim + 1 < tensor.rank; ++dim) {
        const uint64_t stride = tensor.strides_bytes[dim];
        if (stride == 0 || stride % 16 != 0 || stride >= (1ull << 40)) {
            return false;
        }
    }
    const uint64_t inner_bytes = static_cast<uint64_t>(tensor.box[0]) * tensor.element_bytes;
    return inner_bytes % 16 == 0 && inner_bytes <= 128;
}

int encode_tma(const TmaTensor& tensor, CUtensorMap* map) {
    if (!tma_describable(tensor)) {
        return fail(CUVIT_INVALID_ARGUMENT, "tensor cannot be described by a TMA descriptor");
    }
    TensorMapEncodeFn encode = nullptr;
    CUVIT_TRY(tensor_map_encoder(&encode));
    cuuint64_t dims[4];
    cuuint64_t strides[3];
    cuuint32_t box[4];
    cuuint32_t element_strides[4] = {1, 1, 1, 1};
    for (int dim = 0; dim < tensor.rank; ++dim) {
        dims[dim] = tensor.dims[dim];
        box[dim] = tensor.box[dim];
    }
    for (int dim = 0; dim + 1 < tensor.rank; ++dim) {
        strides[dim] = tensor.strides_bytes[dim];
    }
    std::memset(map, 0, sizeof(*map));
    const CUresult result =
        encode(map, tensor.type, static_cast<cuuint32_t>(tensor.rank),
               const_cast<void*>(tensor.base), dims, strides, box, element_strides,
               CU_TENSOR_MAP_INTERLEAVE_NONE, tensor.swizzle,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (result != CUDA_SUCCESS) {
        return fail(CUVIT_CUDA_ERROR,
                    "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(result));
    }
    return CUVIT_OK;
}

// ---- device timeline (instrumented builds only) ---------------------------------------------

#ifdef CUVIT_TIMELINE
namespace {
std::mutex g_timeline_mutex;
std::vector<int (*)(void*)>& timeline_binders() {
    static std::vector<int (*)(void*)> binders;
    return binders;
}
cuvit::dev::TimelineRecord* g_timeline_table = nullptr;

__global__ void timeline_clear_kernel(cuvit::dev::TimelineRecord* records, int count) {
    const int i = static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
    if (i < count) {
        cuvit::dev::TimelineRecord empty{};
        empty.first_ns = ~0ull;
        records[i] = empty;
    }
}
} // namespace

void register_timeline_binder(int (*bind)(void* records)) {
    std::lock_guard<std::mutex> lock(g_timeline_mutex);
    timeline_binders().push_back(bind);
}
#endif

} // namespace cuvit::host

using namespace cuvit::host;

extern "C" {

const char* cuvit_status_string(int status) {
    switch (status) {
    case CUVIT_OK:
        return "ok";
    case CUVIT_INVALID_ARGUMENT:
        return "invalid argument";
    case CUVIT_LENGTH_ERROR:
        return "length error";
    case CUVIT_CUDA_ERROR:
        return "CUDA error";
    case CUVIT_DEVICE_TIMEOUT:
        return "device-side wait timed out";
    case CUVIT_UNSUPPORTED:
        return "unsupported";
    case CUVIT_RUNTIME_ERROR:
        return "runtime error";
    case CUVIT_OUT_OF_MEMORY:
        return "out of memory";
    default:
        return "unknown status";
    }
}

const char* cuvit_last_error_message(void) { return t_last_error.c_str(); }

int cuvit_version(void) { return 100; }

int cuvit_device_status(unsigned* flags) {
    if (flags == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "flags cannot be null");
    }
    const DeviceContext* context = nullptr;
    CUVIT_TRY(current_context(&context));
    CUVIT_TRY_CUDA(cudaDeviceSynchronize());
    unsigned value = 0;
    CUVIT_TRY_CUDA(cudaMemcpy(&value, context->status, sizeof(value), cudaMemcpyDeviceToHost));
    if (value != 0) {
        CUVIT_TRY_CUDA(cudaMemset(context->status, 0, sizeof(unsigned)));
        CUVIT_TRY_CUDA(cudaDeviceSynchronize());
    }
    *flags = value;
    if (value & cuvit::dev::kStatusTimeout) {
        return fail(CUVIT_DEVICE_TIMEOUT, "a kernel gave up on a bounded device-side wait");
    }
    return CUVIT_OK;
}

long long cuvit_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int cuvit_timeline_available(void) {
#ifdef CUVIT_TIMELINE
    return 1;
#else
    return 0;
#endif
}

int cuvit_timeline_reset(void) {
#ifndef CUVIT_TIMELINE
    return fail(CUVIT_UNSUPPORTED, "this build has no device timeline (build with --timeline)");
#else
    const DeviceContext* context = nullptr;
    CUVIT_TRY(current_context(&context));
    std::lock_guard<std::mutex> lock(g_timeline_mutex);
    CUVIT_TRY_CUDA(cudaDeviceSynchronize());
    if (g_timeline_table == nullptr) {
        CUVIT_TRY_CUDA(cudaMalloc(&g_timeline_table,
                                  sizeof(cuvit::dev::TimelineRecord) * cuvit::dev::kTimelineSlots));
        for (int (*bind)(void*) : timeline_binders()) {
            if (bind(g_timeline_table) != 0) {
                return fail(CUVIT_CUDA_ERROR, "binding the device timeline table failed");
            }
        }
    }
    timeline_clear_kernel<<<(cuvit::dev::kTimelineSlots + 255) / 256, 256>>>(
        g_timeline_table, cuvit::dev::kTimelineSlots);
    CUVIT_TRY_CUDA(cudaGetLastError());
    CUVIT_TRY_CUDA(cudaDeviceSynchronize());
    return CUVIT_OK;
#endif
}

int cuvit_timeline_read(cuvit_timeline_record* records, int capacity, int* count) {
#ifndef CUVIT_TIMELINE
    (void)records;
    (void)capacity;
    (void)count;
    return fail(CUVIT_UNSUPPORTED, "this build has no device timeline (build with --timeline)");
#else
    if (count == nullptr || (records == nullptr && capacity > 0)) {
        return fail(CUVIT_INVALID_ARGUMENT, "timeline output cannot be null");
    }
    std::lock_guard<std::mutex> lock(g_timeline_mutex);
    if (g_timeline_table == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "cuvit_timeline_reset() has not been called");
    }
    CUVIT_TRY_CUDA(cudaDeviceSynchronize());
    std::vector<cuvit::dev::TimelineRecord> table(cuvit::dev::kTimelineSlots);
    CUVIT_TRY_CUDA(cudaMemcpy(table.data(), g_timeline_table,
                              sizeof(cuvit::dev::TimelineRecord) * table.size(),
                              cudaMemcpyDeviceToHost));
    std::vector<cuvit::dev::TimelineRecord> used;
    for (const auto& r : table) {
        if (r.grid != 0) {
            used.push_back(r);
        }
    }
    std::sort(used.begin(), used.end(),
              [](const auto& a, const auto& b) { return a.first_ns < b.first_ns; });
    *count = static_cast<int>(used.size());
    for (int i = 0; i < capacity && i < *count; ++i) {
        const auto& r = used[static_cast<size_t>(i)];
        cuvit_timeline_record& out = records[i];
        out.grid = r.grid - 1;
        out.first_ns = r.first_ns;
        out.last_ns = r.last_ns;
        out.warps = r.warps;
        out.cta0_entry_ns = r.cta0_ns[0];
        out.cta0_exit_ns = r.cta0_ns[1];
        out.cta0_entry_clock = r.cta0_clock[0];
        out.cta0_exit_clock = r.cta0_clock[1];
    }
    return CUVIT_OK;
#endif
}

int cuvit_selftest_bounded_wait(unsigned long long limit_ns) {
    if (limit_ns == 0 || limit_ns > 1000000000ull) {
        return fail(CUVIT_INVALID_ARGUMENT, "self-test wait limit must be in (0, 1 s]");
    }
    const DeviceContext* context = nullptr;
    CUVIT_TRY(current_context(&context));
    bounded_wait_selftest_kernel<<<1, 1>>>(context->status, limit_ns);
    return after_launch("bounded_wait_selftest_kernel");
}

} // extern "C"
