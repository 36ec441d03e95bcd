// GEMM front end: the reference's validation rules (src/kernels/gemm.cu:199-242), path
// selection (tcgen05 when TMA can describe both operands on an sm_100 device, FP32 SIMT
// otherwise), tensor-map construction, and the C-ABI entry points.
#include "gemm.hpp"

#include <atomic>
#include <cstdint>
#include <string>

namespace cuvit::gemm {
namespace {

std::atomic<int> g_math_mode{CUVIT_MATH_FP32};

// ---------------------------------------------------------------------------------------
// FP32 SIMT path: any strides, any alignment, K = 0. Each output's K reduction is
// sequential, as in the reference's kernel (src/kernels/gemm.cu:117-136).
// ---------------------------------------------------------------------------------------
constexpr int kSimtTile = 64;
constexpr int kSimtK = 16;
constexpr int kSimtThreads = 256;

template <typename T>
__device__ __forceinline__ float load_operand(const T* pointer, long long index) {
    if constexpr (sizeof(T) == 2) {
        return __bfloat162float(pointer[index]);
    } else {
        return pointer[index];
    }
}

template <typename T>
__global__ void __launch_bounds__(kSimtThreads)
    simt_gemm_kernel(const T* __restrict__ a, const T* __restrict__ b,
                     const float* __restrict__ bias, void* c, int c_kind, int m, int n, int k,
                     float alpha, int transposed, long long lda, long long ldb, long long ldc,
                     int count, int inner, long long stride_a, long long stride_b,
                     long long stride_c, long long outer_a, long long outer_b, long long outer_c,
                     int accumulate, int apply_gelu) {
    dev::timeline_enter();
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();
    __shared__ float tile_a[kSimtK][kSimtTile + 4];
    __shared__ float tile_b[kSimtK][kSimtTile + 4];

    const int tx = threadIdx.x % 16;
    const int ty = threadIdx.x / 16;
    const int row0 = blockIdx.y * kSimtTile;
    const int col0 = blockIdx.x * kSimtTile;

    for (int entry = blockIdx.z; entry < count; entry += gridDim.z) {
        long long offset_a, offset_b, offset_c;
        if (inner > 0) {
            const long long outer = entry / inner;
            const long long index = entry % inner;
            offset_a = outer * outer_a + index * stride_a;
            offset_b = outer * outer_b + index * stride_b;
            offset_c = outer * outer_c + index * stride_c;
        } else {
            offset_a = static_cast<long long>(entry) * stride_a;
            offset_b = static_cast<long long>(entry) * stride_b;
            offset_c = static_cast<long long>(entry) * stride_c;
        }
        const T* const ea = a + offset_a;
        const T* const eb = b + offset_b;

        float acc[4][4] = {};
        for (int k0 = 0; k0 < k; k0 += kSimtK) {
            for (int i = threadIdx.x; i < kSimtTile * kSimtK; i += kSimtThreads) {
                const int r = i / kSimtK;
                const int kk = i % kSimtK;
                const int gr = row0 + r;
                const int gk = k0 + kk;
                tile_a[kk][r] = (gr < m && gk < k) ? load_operand(ea, gr * lda + gk) : 0.0F;
            }
            for (int i = threadIdx.x; i < kSimtTile * kSimtK; i += kSimtThreads) {
                int kk, cc;
                if (transposed) {
                    cc = i / kSimtK;
                    kk = i % kSimtK;
                } else {
                    kk = i / kSimtTile;
                    cc = i % kSimtTile;
                }
                const int gk = k0 + kk;
                const int gc = col0 + cc;
                float value = 0.0F;
                if (gk < k && gc < n) {
                    value = transposed ? load_operand(eb, gc * ldb + gk)
                                       : load_operand(eb, gk * ldb + gc);
                }
                tile_b[kk][cc] = value;
            }
            __syncthreads();
#pragma unroll
            for (int kk = 0; kk < kSimtK; ++kk) {
                float fa[4];
                float fb[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    fa[i] = tile_a[kk][ty * 4 + i];
                    fb[i] = tile_b[kk][tx * 4 + i];
                }
#pragma unroll
                for (int i = 0; i < 4; ++i) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        acc[i][j] = fmaf(fa[i], fb[j], acc[i][j]);
                    }
                }
            }
            __syncthreads();
        }

#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = row0 + ty * 4 + i;
            if (row >= m) {
                continue;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int col = col0 + tx * 4 + j;
                if (col >= n) {
                    continue;
                }
                float value = alpha * acc[i][j];
                if (bias != nullptr) {
                    value += bias[col];
                }
                if (apply_gelu) {
                    value = dev::gelu_erf(value);
                }
                const long long at = offset_c + row * ldc + col;
                if (c_kind == 1) {
                    __nv_bfloat16* const out = static_cast<__nv_bfloat16*>(c);
                    out[at] = __float2bfloat16_rn(accumulate ? __bfloat162float(out[at]) + value
                                                             : value);
                } else {
                    float* const out = static_cast<float*>(c);
                    const float stored = accumulate ? out[at] + value : value;
                    out[at] = c_kind == 2 ? dev::round_to_tf32(stored) : stored;
                }
            }
        }
    }
    dev::timeline_exit();
}

int launch_simt(const Resolved& r, cudaStream_t stream) {
    const cuvit_gemm_problem& p = r.problem;
    const long long tiles_n = (p.n + kSimtTile - 1) / kSimtTile;
    const long long tiles_m = (p.m + kSimtTile - 1) / kSimtTile;
    if (tiles_n > 0x7FFFFFFFLL || tiles_m > 65535) {
        return host::fail(CUVIT_LENGTH_ERROR, "GEMM launch exceeds the CUDA grid limit");
    }
    const dim3 grid(static_cast<unsigned>(tiles_n), static_cast<unsigned>(tiles_m),
                    static_cast<unsigned>(p.batch.count < 65535 ? p.batch.count : 65535));
    const int c_kind = r.c_dtype;
    const cuvit_gemm_batch& batch = p.batch;
    if (r.math == CUVIT_MATH_BF16) {
        host::pdl_launch(simt_gemm_kernel<__nv_bfloat16>, grid, kSimtThreads, 0, stream,
                         static_cast<const __nv_bfloat16*>(r.a),
                         static_cast<const __nv_bfloat16*>(r.b), r.bias, r.c, c_kind, p.m, p.n,
                         p.k, p.alpha, r.transposed ? 1 : 0, r.lda, r.ldb, r.ldc, batch.count,
                         batch.inner, batch.stride_a, batch.stride_b, batch.stride_c,
                         batch.outer_stride_a, batch.outer_stride_b, batch.outer_stride_c,
                         p.epilogue.accumulate ? 1 : 0, p.epilogue.gelu ? 1 : 0);
    } else {
        host::pdl_launch(simt_gemm_kernel<float>, grid, kSimtThreads, 0, stream,
                         static_cast<const float*>(r.a), static_cast<const float*>(r.b), r.bias,
                         r.c, c_kind, p.m, p.n, p.k, p.alpha, r.transposed ? 1 : 0, r.lda,
                         r.ldb, r.ldc, batch.count, batch.inner, batch.stride_a, batch.stride_b,
                         batch.stride_c, batch.outer_stride_a, batch.outer_stride_b,
                         batch.outer_stride_c, p.epilogue.accumulate ? 1 : 0,
                         p.epilogue.gelu ? 1 : 0);
    }
    return host::after_launch("simt_gemm_kernel");
}

// Adds the batch dimensions of one operand to a TMA tensor. Returns false when a stride
// is negative (TMA cannot walk backwards).
bool add_batch_dims(const cuvit_gemm_batch& batch, long long stride, long long outer_stride,
                    int element_bytes, host::TmaTensor* tensor, int* has_index, int* has_outer) {
    *has_index = 0;
    *has_outer = 0;
    if (stride < 0 || outer_stride < 0) {
        return false;
    }
    if (batch.inner > 0) {
        if (stride != 0) {
            tensor->dims[tensor->rank] = static_cast<uint64_t>(batch.inner);
            tensor->strides_bytes[tensor->rank - 1] = static_cast<uint64_t>(stride) * element_bytes;
            tensor->box[tensor->rank] = 1;
            ++tensor->rank;
            *has_index = 1;
        }
        if (outer_stride != 0) {
            tensor->dims[tensor->rank] = static_cast<uint64_t>(batch.count / batch.inner);
            tensor->strides_bytes[tensor->rank - 1] =
                static_cast<uint64_t>(outer_stride) * element_bytes;
            tensor->box[tensor->rank] = 1;
            ++tensor->rank;
            *has_outer = 1;
        }
    } else if (batch.count > 1 && stride != 0) {
        tensor->dims[tensor->rank] = static_cast<uint64_t>(batch.count);
        tensor->strides_bytes[tensor->rank - 1] = static_cast<uint64_t>(stride) * element_bytes;
        tensor->box[tensor->rank] = 1;
        ++tensor->rank;
        *has_index = 1;
    }
    return true;
}

// Tile width: the one whose tiles finish soonest, counting whole waves of tiles over the SMs
// (tiles = 128-row blocks x column tiles x batch entries), each wave as long as its tile is
// wide, with a preference for wide tiles (fewer re-reads of A, fewer shared-memory and L2
// bytes per MMA). With many waves this is the width that wastes least padding; with few
// (ViT-Ti/16 at batch 32: M = 6304, 50 row blocks) it avoids a nearly empty last wave. For
// BF16 the preference is stronger: a 128-wide tile needs about 64 FLOP per operand byte, which
// at the BF16 tensor rate asks more of L2 than it gives (ViT-S/16 QKV, N = 1152, K = 384:
// 374 us per pass on 256-wide pair tiles, 11% padding, against 448 on 128-wide tiles).
// N = 384 stays 128 wide (33% padding: its projection measured 350 vs 315 us per pass on
// 256-wide tiles). Per-element results do not depend on the width: every tile reduces K in
// the same order.
int choose_block_n(long long row_blocks, int n, bool split, bool bf16, int sm_count) {
    const int candidates[] = {256, 128, 64};
    const double penalty[] = {1.0, bf16 ? 1.2 : 1.1, 1.4};
    int best = split ? 128 : 256;
    double best_cost = 1e300;
    for (int i = 0; i < 3; ++i) {
        const int bn = candidates[i];
        if (split && bn > 128) {
            continue;
        }
        const long long tiles = row_blocks * ((n + bn - 1) / bn);
        const long long waves = (tiles + sm_count - 1) / sm_count;
        const double cost = static_cast<double>(waves) * bn * penalty[i];
        if (cost < best_cost) {
            best_cost = cost;
            best = bn;
        }
    }
    return best;
}

} // namespace

int resolve(const void* a, const void* b, const float* bias, void* c, int c_dtype, int math,
            const cuvit_gemm_problem& problem, Resolved* out, bool* empty) {
    *empty = false;
    const int m = problem.m;
    const int n = problem.n;
    const int k = problem.k;
    if (m == 0 || n == 0 || problem.batch.count == 0) {
        *empty = true;
        return CUVIT_OK;
    }
    if (m < 0 || n < 0 || k < 0 || problem.batch.count < 0) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "GEMM dimensions cannot be negative");
    }
    if (problem.batch.inner > 0 && problem.batch.count % problem.batch.inner != 0) {
        return host::fail(CUVIT_INVALID_ARGUMENT,
                          "A split GEMM batch must divide into whole inner groups");
    }
    if (a == nullptr || b == nullptr || c == nullptr) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "GEMM operands cannot be null");
    }
    if (problem.layout != CUVIT_LAYOUT_NO_TRANSPOSE && problem.layout != CUVIT_LAYOUT_TRANSPOSED) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "unknown GEMM layout");
    }
    if (c_dtype != CUVIT_DTYPE_F32 && c_dtype != CUVIT_DTYPE_BF16 && c_dtype != CUVIT_DTYPE_TF32) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "unknown output data type");
    }
    if (math != CUVIT_MATH_FP32 && math != CUVIT_MATH_TF32 && math != CUVIT_MATH_BF16) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "unknown GEMM math mode");
    }

    Resolved r;
    r.a = a;
    r.b = b;
    r.bias = bias;
    r.c = c;
    r.c_dtype = c_dtype;
    r.math = math;
    r.problem = problem;
    // One outer group reaches nothing a flat index would not (src/kernels/gemm.cu:218-223).
    if (r.problem.batch.inner >= r.problem.batch.count) {
        r.problem.batch.inner = 0;
    }
    r.transposed = problem.layout == CUVIT_LAYOUT_TRANSPOSED;
    r.lda = problem.lda != 0 ? problem.lda : k;
    r.ldb = problem.ldb != 0 ? problem.ldb : (r.transposed ? k : n);
    r.ldc = problem.ldc != 0 ? problem.ldc : n;
    if (r.lda < k || r.ldc < n || r.ldb < (r.transposed ? k : n)) {
        return host::fail(CUVIT_INVALID_ARGUMENT,
                          "A GEMM leading dimension is smaller than its row");
    }
    *out = r;
    return CUVIT_OK;
}

int prepare(const Resolved& r, Plan* plan) {
    *plan = Plan{};
    plan->resolved = r;
    plan->path = Path::kSimt;

    const cuvit_gemm_problem& p = r.problem;
    const host::DeviceContext* context = nullptr;
    CUVIT_TRY(host::current_context(&context));
    if (!host::is_blackwell(*context) || p.k == 0) {
        return CUVIT_OK;
    }

    const bool bf16 = r.math == CUVIT_MATH_BF16;
    const bool split = r.math == CUVIT_MATH_FP32;
    const int e = bf16 ? 2 : 4;
    const int block_k = kSwizzleBytes / e;
    const int atom = kSwizzleBytes / e;
    const long long row_blocks = (p.m + kBlockM - 1LL) / kBlockM * p.batch.count;
    const int bn = choose_block_n(row_blocks, p.n, split, bf16, context->sm_count);
    // CTA pairs for BF16 with the weights' K-major layout and 256-wide tiles, once there are
    // at least as many 256-row tiles as SMs (two per pair), so the pairs stay busy. A GELU
    // epilogue keeps the one-CTA kernel: its issue slots, not operand traffic, bound it
    // (ViT-B/16 FC1 on B200: 220 us one-CTA, 224 us paired; QKV 153 vs 145 us).
    const long long pair_tiles =
        ((p.m + 2LL * kBlockM - 1) / (2 * kBlockM)) * ((p.n + bn - 1) / bn) * p.batch.count;
    const bool pair = bf16 && r.transposed && bn == 256 && !p.epilogue.gelu &&
                      pairs_enabled() && pair_tiles >= context->sm_count;
    const CUtensorMapDataType type =
        bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;

    host::TmaTensor ta;
    ta.base = r.a;
    ta.type = type;
    ta.element_bytes = e;
    ta.rank = 2;
    ta.dims[0] = static_cast<uint64_t>(p.k);
    ta.dims[1] = static_cast<uint64_t>(p.m);
    ta.strides_bytes[0] = static_cast<uint64_t>(r.lda) * e;
    ta.box[0] = static_cast<uint32_t>(block_k);
    ta.box[1] = kBlockM;
    int a_index = 0, a_outer = 0;
    if (!add_batch_dims(p.batch, p.batch.stride_a, p.batch.outer_stride_a, e, &ta, &a_index,
                        &a_outer)) {
        return CUVIT_OK;
    }

    host::TmaTensor tb;
    tb.base = r.b;
    tb.type = type;
    tb.element_bytes = e;
    tb.rank = 2;
    if (r.transposed) {
        tb.dims[0] = static_cast<uint64_t>(p.k);
        tb.dims[1] = static_cast<uint64_t>(p.n);
        tb.box[0] = static_cast<uint32_t>(block_k);
        tb.box[1] = static_cast<uint32_t>(pair ? bn / 2 : bn);
    } else {
        tb.dims[0] = static_cast<uint64_t>(p.n);
        tb.dims[1] = static_cast<uint64_t>(p.k);
        tb.box[0] = static_cast<uint32_t>(atom);
        tb.box[1] = static_cast<uint32_t>(block_k);
        if (e == 4) {
            tb.swizzle = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
        }
    }
    tb.strides_bytes[0] = static_cast<uint64_t>(r.ldb) * e;
    int b_index = 0, b_outer = 0;
    if (!add_batch_dims(p.batch, p.batch.stride_b, p.batch.outer_stride_b, e, &tb, &b_index,
                        &b_outer)) {
        return CUVIT_OK;
    }
    if (!host::tma_describable(ta) || !host::tma_describable(tb)) {
        return CUVIT_OK;
    }
    if (host::encode_tma(ta, &plan->map_a) != CUVIT_OK ||
        host::encode_tma(tb, &plan->map_b) != CUVIT_OK) {
        host::clear_error();
        return CUVIT_OK; // the driver refused this shape; the SIMT path still serves it
    }

    const int block_m = pair ? 2 * kBlockM : kBlockM;
    const long long m_tiles = (p.m + block_m - 1) / block_m;
    const long long n_tiles = (p.n + bn - 1) / bn;
    const long long total = m_tiles * n_tiles * p.batch.count;
    if (total > 0x7FFFFFFFLL) {
        return CUVIT_OK;
    }

    TcParams& q = plan->params;
    q.m = p.m;
    q.n = p.n;
    q.k = p.k;
    q.m_tiles = static_cast<int>(m_tiles);
    q.n_tiles = static_cast<int>(n_tiles);
    q.k_blocks = (p.k + block_k - 1) / block_k;
    q.total_tiles = static_cast<int>(total);
    q.count = p.batch.count;
    q.inner = p.batch.inner;
    q.a_rank = ta.rank;
    q.b_rank = tb.rank;
    q.a_has_index = a_index;
    q.a_has_outer = a_outer;
    q.b_has_index = b_index;
    q.b_has_outer = b_outer;
    q.alpha = p.alpha;
    q.bias = r.bias;
    q.c = r.c;
    q.ldc = r.ldc;
    q.stride_c = p.batch.stride_c;
    q.outer_stride_c = p.batch.outer_stride_c;
    q.c_kind = r.c_dtype;
    const int ce = r.c_dtype == CUVIT_DTYPE_BF16 ? 2 : 4;
    const auto aligned16 = [ce](long long elements) { return (elements * ce) % 16 == 0; };
    q.c_vector_ok = (reinterpret_cast<uintptr_t>(r.c) % 16 == 0) && aligned16(r.ldc) &&
                            aligned16(p.batch.stride_c) && aligned16(p.batch.outer_stride_c)
                        ? 1
                        : 0;
    q.accumulate = p.epilogue.accumulate ? 1 : 0;
    q.gelu = p.epilogue.gelu ? 1 : 0;
    q.reverse = host::reverse_sweep() ? 1 : 0;
    q.status = context->status;
    q.bias_vector_ok =
        r.bias != nullptr && reinterpret_cast<uintptr_t>(r.bias) % 16 == 0 ? 1 : 0;

    // C through TMA when a descriptor can describe it: 128-byte rows of 32 FP32 or 64 BF16
    // columns, 32 rows per warp. Accumulating into FP32 becomes a TMA reduce-add (one FP32
    // add in L2, the same single rounding as read-add-write); accumulating into BF16 or
    // TF32 storage has to round in that type, so it keeps the direct path.
    q.c_tma = 0;
    const bool reduce_ok = !p.epilogue.accumulate || r.c_dtype == CUVIT_DTYPE_F32;
    const bool chunk_ok = r.c_dtype != CUVIT_DTYPE_BF16 || bn >= 128;
    if (reduce_ok && chunk_ok) {
        host::TmaTensor tc;
        tc.base = r.c;
        tc.type = r.c_dtype == CUVIT_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
        tc.element_bytes = ce;
        tc.rank = 2;
        tc.dims[0] = static_cast<uint64_t>(p.n);
        tc.dims[1] = static_cast<uint64_t>(p.m);
        tc.strides_bytes[0] = static_cast<uint64_t>(r.ldc) * ce;
        tc.box[0] = static_cast<uint32_t>(kSwizzleBytes / ce);
        tc.box[1] = 32;
        int c_index = 0, c_outer = 0;
        if (add_batch_dims(p.batch, p.batch.stride_c, p.batch.outer_stride_c, ce, &tc, &c_index,
                           &c_outer) &&
            host::tma_describable(tc) && host::encode_tma(tc, &plan->map_c) == CUVIT_OK) {
            q.c_tma = 1;
            q.c_rank = tc.rank;
            q.c_has_index = c_index;
            q.c_has_outer = c_outer;
        } else {
            host::clear_error();
        }
    }

    plan->elem_bytes = e;
    plan->block_n = bn;
    plan->b_mn_major = !r.transposed;
    plan->split = split;
    plan->pair = pair;
    plan->grid = static_cast<int>(total < context->sm_count ? total : context->sm_count);
    plan->path = Path::kTensorCore;
    return CUVIT_OK;
}

int launch(const Plan& plan, cudaStream_t stream) {
    switch (plan.path) {
    case Path::kTensorCore:
        if (plan.split) {
            return launch_tc_split(plan, stream);
        }
        if (plan.pair) {
            return launch_tc_pair(plan, stream);
        }
        return plan.elem_bytes == 2 ? launch_tc_bf16(plan, stream) : launch_tc_tf32(plan, stream);
    case Path::kSimt:
        return launch_simt(plan.resolved, stream);
    default:
        return CUVIT_OK;
    }
}

int run(const void* a, const void* b, const float* bias, void* c, int c_dtype, int math,
        const cuvit_gemm_problem* problem, cudaStream_t stream) {
    if (problem == nullptr) {
        return host::fail(CUVIT_INVALID_ARGUMENT, "GEMM problem cannot be null");
    }
    Resolved resolved;
    bool empty = false;
    CUVIT_TRY(resolve(a, b, bias, c, c_dtype, math, *problem, &resolved, &empty));
    if (empty) {
        return CUVIT_OK;
    }
    Plan plan;
    CUVIT_TRY(prepare(resolved, &plan));
    return launch(plan, stream);
}

} // namespace cuvit::gemm

extern "C" {

void cuvit_gemm_problem_init(cuvit_gemm_problem* problem, int m, int n, int k, int layout) {
    if (problem == nullptr) {
        return;
    }
    *problem = cuvit_gemm_problem{};
    problem->m = m;
    problem->n = n;
    problem->k = k;
    problem->layout = layout;
    problem->alpha = 1.0F;
    problem->batch.count = 1;
}

int cuvit_gemm(const float* a, const float* b, const float* bias, float* c,
               const cuvit_gemm_problem* problem, cuvit_stream_t stream) {
    return cuvit::gemm::run(a, b, bias, c, CUVIT_DTYPE_F32,
                            cuvit::gemm::g_math_mode.load(std::memory_order_relaxed), problem,
                            reinterpret_cast<cudaStream_t>(stream));
}

int cuvit_gemm_ex(const void* a, const void* b, const float* bias, void* c, int c_dtype,
                  int math, const cuvit_gemm_problem* problem, cuvit_stream_t stream) {
    return cuvit::gemm::run(a, b, bias, c, c_dtype, math, problem,
                            reinterpret_cast<cudaStream_t>(stream));
}

int cuvit_set_math_mode(int math) {
    if (math != CUVIT_MATH_FP32 && math != CUVIT_MATH_TF32) {
        return cuvit::host::fail(CUVIT_INVALID_ARGUMENT,
                                 "the float GEMM math mode must be FP32 or TF32");
    }
    cuvit::gemm::g_math_mode.store(math, std::memory_order_relaxed);
    return CUVIT_OK;
}

int cuvit_get_math_mode(void) {
    return cuvit::gemm::g_math_mode.load(std::memory_order_relaxed);
}

} // extern "C"
