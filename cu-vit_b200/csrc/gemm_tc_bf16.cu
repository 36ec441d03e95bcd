// tcgen05 GEMM instantiations with bfloat16 operands (kind::f16, FP32 accumulation).
#include "gemm_tc_instances.cuh"

namespace cuvit::gemm {

int launch_tc_bf16(const Plan& plan, cudaStream_t stream) {
    return launch_by_shape<2, false>(plan, stream);
}

} // namespace cuvit::gemm
