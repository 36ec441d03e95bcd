// Shared body of the per-type launcher translation units: picks the template instantiation
// for (block_n, b_mn_major), raises its dynamic shared memory limit (once per device), and
// launches.
#pragma once

#include "gemm.hpp"

namespace cuvit::gemm {

template <int ElemBytes, int BN, bool BMn, bool Split>
int launch_instance(const Plan& plan, cudaStream_t stream) {
    using Shape = TcShape<ElemBytes, BN, Split>;
    auto* kernel = &tc_gemm_kernel<ElemBytes, BN, BMn, Split>;
    CUVIT_TRY_CUDA(host::allow_dynamic_smem(reinterpret_cast<const void*>(kernel),
                                            Shape::kSmemBytes));
    host::pdl_launch(kernel, plan.grid, Shape::kThreads, Shape::kSmemBytes, stream, plan.map_a,
                     plan.map_b, plan.map_c, plan.params);
    return host::after_launch("tc_gemm_kernel");
}

template <int ElemBytes, bool Split>
int launch_by_shape(const Plan& plan, cudaStream_t stream) {
    const bool mn = plan.b_mn_major;
    switch (plan.block_n) {
    case 64:
        return mn ? launch_instance<ElemBytes, 64, true, Split>(plan, stream)
                  : launch_instance<ElemBytes, 64, false, Split>(plan, stream);
    case 128:
        return mn ? launch_instance<ElemBytes, 128, true, Split>(plan, stream)
                  : launch_instance<ElemBytes, 128, false, Split>(plan, stream);
    default:
        if constexpr (!Split) {
            return mn ? launch_instance<ElemBytes, 256, true, Split>(plan, stream)
                      : launch_instance<ElemBytes, 256, false, Split>(plan, stream);
        }
        return host::fail(CUVIT_INVALID_ARGUMENT, "unsupported GEMM tile width");
    }
}

} // namespace cuvit::gemm
