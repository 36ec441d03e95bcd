// tcgen05 GEMM instantiations with FP32 operands read as TF32 (kind::tf32, one pass).
#include "gemm_tc_instances.cuh"

namespace cuvit::gemm {

int launch_tc_tf32(const Plan& plan, cudaStream_t stream) {
    return launch_by_shape<4, false>(plan, stream);
}

} // namespace cuvit::gemm
