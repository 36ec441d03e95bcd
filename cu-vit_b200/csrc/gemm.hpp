// GEMM dispatch: validation with the reference launcher's semantics, a prepared "plan"
// (tensor maps + kernel parameters) for the tcgen05 path, and the FP32 SIMT path for
// problems TMA cannot describe.
#pragma once

#include "cuvit_b200.h"
#include "gemm_tc.cuh"
#include "runtime.hpp"

#include <cuda.h>
#include <cuda_runtime.h>

namespace cuvit::gemm {

enum class Path { kNone, kTensorCore, kSimt };

// A fully resolved problem: defaults applied, split batch collapsed, pointers attached.
struct Resolved {
    const void* a = nullptr;
    const void* b = nullptr;
    const float* bias = nullptr;
    void* c = nullptr;
    int c_dtype = CUVIT_DTYPE_F32;
    int math = CUVIT_MATH_FP32;
    cuvit_gemm_problem problem{};
    bool transposed = false;
    int lda = 0, ldb = 0, ldc = 0;
};

struct Plan {
    Path path = Path::kNone;
    // tensor-core path
    CUtensorMap map_a{};
    CUtensorMap map_b{};
    CUtensorMap map_c{}; // output, for TMA stores / reduce-adds (params.c_tma)
    TcParams params{};
    int elem_bytes = 4;
    int block_n = 128;
    bool b_mn_major = false;
    bool split = false;
    bool pair = false; // CTA-pair kernel (256-row tiles, B map boxes of block_n / 2 rows)
    int grid = 0;
    // SIMT path
    Resolved resolved{};
};

// Validates (reference order: src/kernels/gemm.cu:205-231) and resolves defaults. Sets
// *empty when the problem is a no-op.
int resolve(const void* a, const void* b, const float* bias, void* c, int c_dtype, int math,
            const cuvit_gemm_problem& problem, Resolved* out, bool* empty);

// Builds the launch plan for the current device.
int prepare(const Resolved& resolved, Plan* plan);

// Enqueues a prepared plan.
int launch(const Plan& plan, cudaStream_t stream);

// Launchers for the template instantiations (one translation unit per operand type).
int launch_tc_bf16(const Plan& plan, cudaStream_t stream);
int launch_tc_tf32(const Plan& plan, cudaStream_t stream);
int launch_tc_split(const Plan& plan, cudaStream_t stream);
int launch_tc_pair(const Plan& plan, cudaStream_t stream);

// Whether large BF16 GEMMs may use the CTA-pair kernel: on unless the environment sets
// CUVIT_GEMM_PAIRS=0 (which keeps every GEMM on the one-CTA kernel).
bool pairs_enabled();


} // namespace cuvit::gemm
