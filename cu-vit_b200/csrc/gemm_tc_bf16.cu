// tcgen05 GEMM instantiations with bfloat16 operands (kind::f16, FP32 accumulation): the
// one-CTA kernel for every tile width and layout, and the CTA-pair kernel for large GEMMs
// with a K-major B.
#include "gemm_tc_instances.cuh"
#include "gemm_tc_pair.cuh"

#include <cstdlib>
#include <cstring>

namespace cuvit::gemm {

bool pairs_enabled() {
    static const bool enabled = []() {
        const char* value = std::getenv("CUVIT_GEMM_PAIRS");
        return value == nullptr || std::strcmp(value, "0") != 0;
    }();
    return enabled;
}

int launch_tc_bf16(const Plan& plan, cudaStream_t stream) {
    return launch_by_shape<2, false>(plan, stream);
}

namespace {

// Devices whose resident-pair count each pair instance records.
constexpr int kMaxResidentDevices = 64;

template <int BN>
int launch_pair_instance(const Plan& plan, cudaStream_t stream) {
    using Shape = PairShape<BN>;
    auto* kernel = &tc_gemm_pair_kernel<BN>;
    cudaLaunchAttribute attributes[2]{};
    attributes[0].id = cudaLaunchAttributeClusterDimension;
    attributes[0].val.clusterDim.x = 2;
    attributes[0].val.clusterDim.y = 1;
    attributes[0].val.clusterDim.z = 1;
    attributes[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attributes[1].val.programmaticStreamSerializationAllowed = 1;

    // Shared-memory limit and the number of pairs that can be resident at once (the
    // persistent grid), both once per device.
    static int resident[kMaxResidentDevices] = {};
    int device = 0;
    CUVIT_TRY_CUDA(cudaGetDevice(&device));
    if (device < 0 || device >= kMaxResidentDevices) {
        return host::fail(CUVIT_UNSUPPORTED, "device ordinal out of range");
    }
    CUVIT_TRY_CUDA(host::once_per_device(
        reinterpret_cast<const void*>(kernel), [&](int current) {
            cudaError_t error = cudaFuncSetAttribute(
                kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Shape::kSmemBytes);
            if (error != cudaSuccess) {
                return error;
            }
            cudaLaunchConfig_t probe{};
            probe.gridDim = dim3(2, 1, 1);
            probe.blockDim = dim3(Shape::kThreads, 1, 1);
            probe.dynamicSmemBytes = Shape::kSmemBytes;
            probe.attrs = attributes;
            probe.numAttrs = 1;
            return cudaOccupancyMaxActiveClusters(&resident[current], kernel, &probe);
        }));
    const int resident_pairs = resident[device];
    if (resident_pairs < 1) {
        return host::fail(CUVIT_RUNTIME_ERROR,
                          "no CTA pair of the GEMM kernel fits on this device");
    }
    const int pairs =
        plan.params.total_tiles < resident_pairs ? plan.params.total_tiles : resident_pairs;
    cudaLaunchConfig_t config{};
    config.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
    config.blockDim = dim3(Shape::kThreads, 1, 1);
    config.dynamicSmemBytes = Shape::kSmemBytes;
    config.stream = stream;
    config.attrs = attributes;
    config.numAttrs = host::pdl_enabled() ? 2 : 1;
    cudaLaunchKernelEx(&config, kernel, plan.map_a, plan.map_b, plan.map_c, plan.params);
    return host::after_launch("tc_gemm_pair_kernel");
}

} // namespace

int launch_tc_pair(const Plan& plan, cudaStream_t stream) {
    switch (plan.block_n) {
    case 256:
        return launch_pair_instance<256>(plan, stream);
    default:
        return host::fail(CUVIT_INVALID_ARGUMENT, "unsupported CTA-pair GEMM tile width");
    }
}

} // namespace cuvit::gemm
