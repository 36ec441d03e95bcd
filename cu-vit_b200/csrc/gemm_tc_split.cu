// tcgen05 GEMM instantiations for FP32-faithful products: each operand is split into a
// TF32 head and a TF32 remainder in shared memory and the product is formed as
// hi*hi + hi*lo + lo*hi (the 3xTF32 scheme of Ootomo & Yokota, 2022), accumulated in FP32.
#include "gemm_tc_instances.cuh"

namespace cuvit::gemm {

int launch_tc_split(const Plan& plan, cudaStream_t stream) {
    return launch_by_shape<4, true>(plan, stream);
}

} // namespace cuvit::gemm
