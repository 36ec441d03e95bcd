// Persistent, warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[e][m][n] = epilogue(alpha * sum_k A[e][m][k] * B[e](k, n) + bias[n])
//
// A is row-major [M, K] (K-major). B is either [N, K] (K-major, the reference's
// kTransposed layout) or [K, N] (MN-major, kNoTranspose). Operands arrive by TMA with
// 128-byte swizzle into a ring of shared-memory stages; one thread issues tcgen05.mma into
// a double-buffered FP32 accumulator in tensor memory; eight epilogue warps drain TMEM,
// apply alpha / bias / GELU, and write C through shared memory with TMA stores -- or TMA
// reduce-adds, which make "accumulate into the residual stream" an FP32 add in L2 without
// the epilogue ever reading C -- while the next tile accumulates.
//
// Roles (one CTA per SM, persistent over output tiles 128 x BN):
//   warp 0         TMA producer (one elected lane)
//   warp 1         MMA issuer (one elected lane)
//   warp 2         TMEM allocator
//   warps 4..11    epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 (= tile rows) and
//                  column half (w-4)/4 of the tile
//   warps 12..15   (Split only) 3xTF32 splitter: rewrites each landed stage as
//                  hi = rn_tf32(x) in place and lo = rn_tf32(x - hi) beside it, so the MMA
//                  warp can issue hi*hi + hi*lo + lo*hi.
//
// Numerics: each output element's K reduction runs in a fixed order that depends only on
// K (no split-K), so results do not depend on M, the batch, or the tile chosen for M.
#pragma once

#include "ptx.cuh"

#include <cuda.h>
#include <cuda_bf16.h>

#include <cstdint>

namespace cuvit::gemm {

constexpr int kBlockM = 128;
constexpr int kSwizzleBytes = 128;  // one swizzle atom row
constexpr int kSmemBudget = 196608; // operand stages per CTA
constexpr int kEpilogueWarps = 8;
constexpr int kEpilogueThreads = 32 * kEpilogueWarps;
constexpr int kSlabBytes = 32 * kSwizzleBytes; // one warp's 32 output rows x 128 bytes

struct TcParams {
    int m, n, k;
    int m_tiles, n_tiles, k_blocks;
    int total_tiles;
    int count, inner; // batch entries; inner > 0 splits entry e into (e / inner, e % inner)
    int a_rank, b_rank, c_rank;
    int a_has_index, a_has_outer, b_has_index, b_has_outer, c_has_index, c_has_outer;
    float alpha;
    const float* bias;
    int bias_vector_ok; // bias is 16-byte aligned
    void* c;
    long long ldc, stride_c, outer_stride_c;
    int c_kind;      // 0: FP32, 1: BF16, 2: FP32 storage rounded to TF32 values
    int c_tma;       // write C with TMA stores (reduce-adds when accumulating)
    int c_vector_ok; // direct path: 16-byte vector stores of whole chunks are aligned
    int accumulate, gelu;
    int reverse; // walk the output tiles from the last to the first
    unsigned* status;
};

// The output tile a CTA's t-th tile index stands for, in the launch's sweep order.
__device__ __forceinline__ int ordered_tile(const TcParams& p, int t) {
    return p.reverse ? p.total_tiles - 1 - t : t;
}

template <int ElemBytes, int BN, bool Split>
struct TcShape {
    static constexpr int kBlockK = kSwizzleBytes / ElemBytes;   // K elements per stage
    static constexpr int kMmaK = 32 / ElemBytes;                 // K per instruction
    static constexpr int kAtomElems = kSwizzleBytes / ElemBytes; // MN elements per atom
    static constexpr int kABytes = kBlockM * kSwizzleBytes;      // 16 KiB
    static constexpr int kBBytes = BN * kSwizzleBytes;
    static constexpr int kStageBytes = (kABytes + kBBytes) * (Split ? 2 : 1);
    static constexpr int kStagesRaw = kSmemBudget / kStageBytes;
    static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
    // Per tile: one FP32 accumulator of BN columns, plus (Split) a second one that collects
    // the small hi*lo and lo*hi cross terms, so the leading product's accumulator takes one
    // rounding per MMA instead of three. Two tiles in flight.
    static constexpr int kAccColumns = Split ? 2 * BN : BN;
    static constexpr int kTmemColumns = 2 * kAccColumns < 32 ? 32 : 2 * kAccColumns;
    static constexpr int kThreads = 32 * (4 + kEpilogueWarps + (Split ? 4 : 0));
    static constexpr int kSlabOffset = kStages * kStageBytes;
    static constexpr int kBarrierOffset = kSlabOffset + kEpilogueWarps * kSlabBytes;
    // barriers: full, empty, converted (split) per stage; tmem full/empty x2; drain
    static constexpr int kBarrierBytes = (3 * kStages + 5) * 8 + 16;
    static constexpr int kSmemBytes = 1024 + kBarrierOffset + kBarrierBytes;
    static_assert(kStages >= 2, "at least two pipeline stages");
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64, 128 or 256");
    static_assert(kSmemBytes <= 232448, "shared memory over the per-block limit");
};

__device__ __forceinline__ void batch_coords(int entry, int inner, int& index, int& outer) {
    if (inner > 0) {
        outer = entry / inner;
        index = entry - outer * inner;
    } else {
        outer = 0;
        index = entry;
    }
}

// Loads Cols accumulator columns of this warp's 32 lanes (adding the cross-term accumulator
// BN columns further on, for Split).
template <int Cols, int BN, bool Split>
__device__ __forceinline__ void load_accumulator(uint32_t taddr, float (&v)[Cols]) {
#pragma unroll
    for (int g = 0; g < Cols / 32; ++g) {
        uint32_t raw[32];
        dev::tmem_load_32(taddr + g * 32, raw);
        if constexpr (Split) {
            uint32_t small[32];
            dev::tmem_load_32(taddr + g * 32 + BN, small);
            dev::tmem_wait_load();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                v[g * 32 + j] = __uint_as_float(raw[j]) + __uint_as_float(small[j]);
            }
        } else {
            dev::tmem_wait_load();
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                v[g * 32 + j] = __uint_as_float(raw[j]);
            }
        }
    }
}

// alpha, bias, GELU on Cols consecutive columns starting at col0 (the reference's order,
// src/kernels/gemm.cu:153-160). Multiplying by alpha == 1 is skipped: it is exact anyway.
template <int Cols>
__device__ __forceinline__ void apply_epilogue(float (&v)[Cols], const TcParams& p, int col0) {
    if (p.alpha != 1.0F) {
#pragma unroll
        for (int j = 0; j < Cols; ++j) {
            v[j] = p.alpha * v[j];
        }
    }
    if (p.bias != nullptr) {
        if (p.bias_vector_ok && col0 + Cols <= p.n) {
            const float4* const b4 = reinterpret_cast<const float4*>(p.bias + col0);
#pragma unroll
            for (int q = 0; q < Cols / 4; ++q) {
                const float4 b = __ldg(b4 + q);
                const float2 lo = dev::f32x2_split(
                    dev::add_f32x2(dev::f32x2(v[4 * q], v[4 * q + 1]), dev::f32x2(b.x, b.y)));
                const float2 hi = dev::f32x2_split(dev::add_f32x2(
                    dev::f32x2(v[4 * q + 2], v[4 * q + 3]), dev::f32x2(b.z, b.w)));
                v[4 * q] = lo.x;
                v[4 * q + 1] = lo.y;
                v[4 * q + 2] = hi.x;
                v[4 * q + 3] = hi.y;
            }
        } else {
#pragma unroll
            for (int j = 0; j < Cols; ++j) {
                if (col0 + j < p.n) {
                    v[j] += __ldg(p.bias + col0 + j);
                }
            }
        }
    }
    if (p.gelu) {
        if (p.c_kind == 1) {
#pragma unroll
            for (int j = 0; j < Cols; j += 2) {
                const float2 g = dev::gelu_bf16_output2(v[j], v[j + 1]);
                v[j] = g.x;
                v[j + 1] = g.y;
            }
        } else {
#pragma unroll
            for (int j = 0; j < Cols; ++j) {
                v[j] = dev::gelu_erf(v[j]);
            }
        }
    }
}

// One 128-byte output row per lane into the warp's slab, in the 128-byte swizzled layout a
// TMA store reads (16-byte chunk j of row r at chunk position j ^ (r % 8)).
template <int Cols>
__device__ __forceinline__ void stage_row(uint8_t* slab, int lane, const float (&v)[Cols],
                                          int c_kind) {
    uint4* const row = reinterpret_cast<uint4*>(slab + lane * kSwizzleBytes);
    if constexpr (Cols == 64) { // bfloat16: 8 values per 16-byte chunk
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            row[j ^ (lane & 7)] =
                make_uint4(dev::pack_bf16x2(v[8 * j], v[8 * j + 1]),
                           dev::pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                           dev::pack_bf16x2(v[8 * j + 4], v[8 * j + 5]),
                           dev::pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
        }
    } else { // FP32 (optionally rounded to TF32 values): 4 values per chunk
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float a = v[4 * j], b = v[4 * j + 1], c = v[4 * j + 2], d = v[4 * j + 3];
            if (c_kind == 2) {
                a = dev::round_to_tf32(a);
                b = dev::round_to_tf32(b);
                c = dev::round_to_tf32(c);
                d = dev::round_to_tf32(d);
            }
            row[j ^ (lane & 7)] = make_uint4(__float_as_uint(a), __float_as_uint(b),
                                             __float_as_uint(c), __float_as_uint(d));
        }
    }
}

// Direct global stores of 32 columns of one row (used when TMA cannot describe C).
__device__ __forceinline__ void store_direct(const TcParams& p, long long row_offset, int col0,
                                             const float (&v)[32]) {
    const bool whole = p.c_vector_ok && (col0 + 32 <= p.n);
    if (p.c_kind != 1) {
        float* const out = static_cast<float*>(p.c) + row_offset + col0;
        if (whole) {
            float4* const out4 = reinterpret_cast<float4*>(out);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                float4 value = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                if (p.accumulate) {
                    const float4 old = out4[q];
                    value.x = old.x + value.x;
                    value.y = old.y + value.y;
                    value.z = old.z + value.z;
                    value.w = old.w + value.w;
                }
                if (p.c_kind == 2) {
                    value.x = dev::round_to_tf32(value.x);
                    value.y = dev::round_to_tf32(value.y);
                    value.z = dev::round_to_tf32(value.z);
                    value.w = dev::round_to_tf32(value.w);
                }
                out4[q] = value;
            }
        } else {
            for (int j = 0; j < 32 && col0 + j < p.n; ++j) {
                const float value = p.accumulate ? out[j] + v[j] : v[j];
                out[j] = p.c_kind == 2 ? dev::round_to_tf32(value) : value;
            }
        }
    } else {
        __nv_bfloat16* const out = static_cast<__nv_bfloat16*>(p.c) + row_offset + col0;
        if (whole) {
            uint4* const out4 = reinterpret_cast<uint4*>(out);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float w[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    w[j] = v[8 * q + j];
                }
                if (p.accumulate) {
                    const uint4 old = out4[q];
                    const __nv_bfloat162* const pairs =
                        reinterpret_cast<const __nv_bfloat162*>(&old);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const float2 f = __bfloat1622float2(pairs[j]);
                        w[2 * j] = f.x + w[2 * j];
                        w[2 * j + 1] = f.y + w[2 * j + 1];
                    }
                }
                out4[q] = make_uint4(dev::pack_bf16x2(w[0], w[1]), dev::pack_bf16x2(w[2], w[3]),
                                     dev::pack_bf16x2(w[4], w[5]), dev::pack_bf16x2(w[6], w[7]));
            }
        } else {
            for (int j = 0; j < 32 && col0 + j < p.n; ++j) {
                const float old = p.accumulate ? __bfloat162float(out[j]) : 0.0F;
                out[j] = __float2bfloat16_rn(p.accumulate ? old + v[j] : v[j]);
            }
        }
    }
}

// Drains Cols columns of the accumulator per step through the warp's slab and TMA.
template <int Cols, int BN, bool Split>
__device__ __forceinline__ void epilogue_tma(const TcParams& p, const CUtensorMap* tma_c,
                                             uint32_t tmem_cols, int first, int last, int col_base,
                                             int row_base, int index, int outer, uint8_t* slab,
                                             uint32_t slab_addr, int lane) {
#pragma unroll 1
    for (int c = first; c < last; c += Cols) {
        const int col0 = col_base + c;
        if (col0 >= p.n) {
            break; // uniform across the warp
        }
        float v[Cols];
        load_accumulator<Cols, BN, Split>(tmem_cols + c, v);
        apply_epilogue<Cols>(v, p, col0);
        // The previous chunk's store must have finished reading the slab.
        if (lane == 0) {
            dev::bulk_wait_group_read0();
        }
        __syncwarp();
        stage_row<Cols>(slab, lane, v, p.c_kind);
        dev::fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
            int coords[4] = {col0, row_base, 0, 0};
            int r = 2;
            if (p.c_has_index) coords[r++] = index;
            if (p.c_has_outer) coords[r++] = outer;
            if (p.accumulate) {
                dev::tma_store<true>(tma_c, slab_addr, p.c_rank, coords);
            } else {
                dev::tma_store<false>(tma_c, slab_addr, p.c_rank, coords);
            }
            dev::bulk_commit_group();
        }
    }
}

template <int ElemBytes, int BN, bool BMnMajor, bool Split>
__global__ void __launch_bounds__(TcShape<ElemBytes, BN, Split>::kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
                   const __grid_constant__ CUtensorMap tma_b,
                   const __grid_constant__ CUtensorMap tma_c, const TcParams p) {
    dev::timeline_enter();
    using Shape = TcShape<ElemBytes, BN, Split>;
    constexpr int kStages = Shape::kStages;
    constexpr dev::MmaKind kKind = ElemBytes == 2 ? dev::MmaKind::kF16 : dev::MmaKind::kTF32;
    constexpr uint32_t kFormat = ElemBytes == 2 ? 1u : 2u; // BF16 or TF32
    constexpr uint32_t kIdesc = dev::make_idesc(kFormat, kBlockM, BN, false, BMnMajor);
    constexpr uint32_t kTxBytes = Shape::kABytes + Shape::kBBytes;
    // An MN-major B of 32-bit elements uses 32-byte swizzle atoms of 4 rows (512 bytes);
    // 16-bit elements use the 8-row (1024-byte) atoms of the ordinary 128-byte swizzle.
    constexpr uint32_t kBLayout =
        ElemBytes == 4 ? dev::kLayoutSwizzle128Atom32 : dev::kLayoutSwizzle128;
    constexpr uint32_t kBAtomBytes = ElemBytes == 4 ? 512u : 1024u;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = dev::smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* const smem = smem_raw + (base - raw_base);

    // Stage s: [A | B | A_lo | B_lo]; then one output slab per epilogue warp; then barriers.
    const auto stage_a = [&](int s) -> uint32_t { return base + s * Shape::kStageBytes; };
    const auto stage_b = [&](int s) -> uint32_t {
        return base + s * Shape::kStageBytes + Shape::kABytes;
    };
    const uint32_t bar_base = base + Shape::kBarrierOffset;
    const auto full_bar = [&](int s) -> uint32_t { return bar_base + 8u * s; };
    const auto empty_bar = [&](int s) -> uint32_t { return bar_base + 8u * (kStages + s); };
    const auto conv_bar = [&](int s) -> uint32_t { return bar_base + 8u * (2 * kStages + s); };
    const auto tfull_bar = [&](int a) -> uint32_t { return bar_base + 8u * (3 * kStages + a); };
    const auto tempty_bar = [&](int a) -> uint32_t {
        return bar_base + 8u * (3 * kStages + 2 + a);
    };
    const uint32_t drain_bar = bar_base + 8u * (3 * kStages + 4);
    uint32_t* const tmem_slot =
        reinterpret_cast<uint32_t*>(smem + Shape::kBarrierOffset + 8 * (3 * kStages + 5));

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            dev::mbar_init(full_bar(s), 1);
            dev::mbar_init(empty_bar(s), 1);
            dev::mbar_init(conv_bar(s), 128);
        }
        for (int a = 0; a < 2; ++a) {
            dev::mbar_init(tfull_bar(a), 1);
            dev::mbar_init(tempty_bar(a), kEpilogueThreads);
        }
        dev::mbar_init(drain_bar, 1);
        dev::fence_barrier_init();
    }
    if (warp == 2) {
        dev::tmem_alloc(dev::smem_u32(tmem_slot), Shape::kTmemColumns);
        dev::tmem_relinquish();
    }
    dev::tc_fence_before();
    __syncthreads();
    dev::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Inputs of this launch may come from the previous one: nothing global is read or
    // written before it has finished.
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();

    const int per_entry = p.m_tiles * p.n_tiles;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer ----------------
        dev::tma_prefetch_descriptor(&tma_a);
        dev::tma_prefetch_descriptor(&tma_b);
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x) {
            const int ordered = ordered_tile(p, tile);
            const int entry = ordered / per_entry;
            const int rest = ordered - entry * per_entry;
            const int m_block = rest / p.n_tiles;
            const int n_block = rest - m_block * p.n_tiles;
            int index, outer;
            batch_coords(entry, p.inner, index, outer);
            for (int kb = 0; kb < p.k_blocks; ++kb) {
                if (!dev::mbar_wait(empty_bar(stage), phase ^ 1u, p.status)) {
                    ok = false;
                    break;
                }
                dev::mbar_arrive_expect_tx(full_bar(stage), kTxBytes);
                const int k0 = kb * Shape::kBlockK;
                int ca[4] = {k0, m_block * kBlockM, 0, 0};
                int r = 2;
                if (p.a_has_index) ca[r++] = index;
                if (p.a_has_outer) ca[r++] = outer;
                dev::tma_load(stage_a(stage), &tma_a, full_bar(stage), p.a_rank, ca);
                if constexpr (!BMnMajor) {
                    int cb[4] = {k0, n_block * BN, 0, 0};
                    int rb = 2;
                    if (p.b_has_index) cb[rb++] = index;
                    if (p.b_has_outer) cb[rb++] = outer;
                    dev::tma_load(stage_b(stage), &tma_b, full_bar(stage), p.b_rank, cb);
                } else {
                    // [K, N] operand: one box per 128-byte atom of N, each BK rows deep.
#pragma unroll
                    for (int atom = 0; atom < BN / Shape::kAtomElems; ++atom) {
                        int cb[4] = {n_block * BN + atom * Shape::kAtomElems, k0, 0, 0};
                        int rb = 2;
                        if (p.b_has_index) cb[rb++] = index;
                        if (p.b_has_outer) cb[rb++] = outer;
                        dev::tma_load(stage_b(stage) + atom * Shape::kBlockK * kSwizzleBytes,
                                      &tma_b, full_bar(stage), p.b_rank, cb);
                    }
                }
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        if (!ok) {
            // Let every load this thread issued land before the CTA can exit.
            for (int s = 0; s < kStages; ++s) {
                dev::mbar_wait(full_bar(s), phase ^ (s < stage ? 0u : 1u), p.status);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---------------- MMA issuer ----------------
        int stage = 0;
        uint32_t phase = 0;
        int local = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < p.total_tiles && ok; tile += gridDim.x, ++local) {
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!dev::mbar_wait(tempty_bar(acc), acc_phase ^ 1u, p.status)) {
                ok = false;
                break;
            }
            dev::tc_fence_after();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * Shape::kAccColumns);
            const uint32_t d_small = d_tmem + BN; // Split: the cross-term accumulator
            for (int kb = 0; kb < p.k_blocks; ++kb) {
                const uint32_t ready = Split ? conv_bar(stage) : full_bar(stage);
                if (!dev::mbar_wait(ready, phase, p.status)) {
                    ok = false;
                    break;
                }
                dev::tc_fence_after();
                const uint32_t a_addr = stage_a(stage);
                const uint32_t b_addr = stage_b(stage);
#pragma unroll
                for (int kk = 0; kk < Shape::kBlockK / Shape::kMmaK; ++kk) {
                    const uint64_t a_desc = dev::smem_desc_sw128(a_addr + kk * 32, 16, 1024);
                    uint64_t b_desc;
                    if constexpr (!BMnMajor) {
                        b_desc = dev::smem_desc_sw128(b_addr + kk * 32, 16, 1024);
                    } else {
                        b_desc = dev::smem_desc(b_addr + kk * Shape::kMmaK * kSwizzleBytes,
                                                Shape::kBlockK * kSwizzleBytes, kBAtomBytes,
                                                kBLayout);
                    }
                    const uint32_t accumulate = (kb > 0 || kk > 0) ? 1u : 0u;
                    if constexpr (Split) {
                        const uint32_t lo_offset = Shape::kABytes + Shape::kBBytes;
                        uint64_t b_lo_desc;
                        if constexpr (!BMnMajor) {
                            b_lo_desc =
                                dev::smem_desc_sw128(b_addr + lo_offset + kk * 32, 16, 1024);
                        } else {
                            b_lo_desc = dev::smem_desc(
                                b_addr + lo_offset + kk * Shape::kMmaK * kSwizzleBytes,
                                Shape::kBlockK * kSwizzleBytes, kBAtomBytes, kBLayout);
                        }
                        const uint64_t a_lo_desc =
                            dev::smem_desc_sw128(a_addr + lo_offset + kk * 32, 16, 1024);
                        dev::mma_ss<kKind>(d_small, a_lo_desc, b_desc, kIdesc, accumulate);
                        dev::mma_ss<kKind>(d_small, a_desc, b_lo_desc, kIdesc, 1u);
                        dev::mma_ss<kKind>(d_tmem, a_desc, b_desc, kIdesc, accumulate);
                    } else {
                        dev::mma_ss<kKind>(d_tmem, a_desc, b_desc, kIdesc, accumulate);
                    }
                }
                dev::tc_commit(empty_bar(stage));
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) {
                break;
            }
            dev::tc_commit(tfull_bar(acc));
        }
        if (!ok) {
            // Drain: the commit arrives once every MMA issued so far has completed, so no
            // MMA still reads shared memory or writes TMEM when the CTA tears down.
            dev::tc_commit(drain_bar);
            dev::mbar_drain_wait(drain_bar, 0);
        }
    } else if (warp >= 4 && warp < 4 + kEpilogueWarps) {
        // ---------------- epilogue ----------------
        const int e = warp - 4;
        const int quarter = warp & 3; // the TMEM lane quarter this warp may access
        constexpr int kHalf = BN / 2;
        const int half = e >> 2;
        uint8_t* const slab = smem + Shape::kSlabOffset + e * kSlabBytes;
        const uint32_t slab_addr = base + Shape::kSlabOffset + e * kSlabBytes;
        const uint32_t lane_field = static_cast<uint32_t>(quarter * 32) << 16;
        if (p.c_tma && lane == 0) {
            dev::tma_prefetch_descriptor(&tma_c);
        }
        int local = 0;
        for (int tile = blockIdx.x; tile < p.total_tiles; tile += gridDim.x, ++local) {
            const int ordered = ordered_tile(p, tile);
            const int entry = ordered / per_entry;
            const int rest = ordered - entry * per_entry;
            const int m_block = rest / p.n_tiles;
            const int n_block = rest - m_block * p.n_tiles;
            int index, outer;
            batch_coords(entry, p.inner, index, outer);
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!dev::mbar_wait_warp(tfull_bar(acc), acc_phase, p.status)) {
                break;
            }
            dev::tc_fence_after();
            const int row_base = m_block * kBlockM + quarter * 32;
            const uint32_t tmem_cols =
                tmem_base + lane_field + static_cast<uint32_t>(acc * Shape::kAccColumns);
            const int first = half * kHalf;
            const int col_base = n_block * BN;
            // A BF16 chunk is 64 columns (128 bytes); with BN = 64 a half tile is narrower,
            // so that combination always takes the direct path (the host never sets c_tma).
            if (p.c_tma && (p.c_kind != 1 || kHalf >= 64)) {
                if (p.c_kind == 1) {
                    epilogue_tma<64, BN, Split>(p, &tma_c, tmem_cols, first, first + kHalf,
                                                col_base, row_base, index, outer, slab,
                                                slab_addr, lane);
                } else {
                    epilogue_tma<32, BN, Split>(p, &tma_c, tmem_cols, first, first + kHalf,
                                                col_base, row_base, index, outer, slab,
                                                slab_addr, lane);
                }
            } else {
                const int row = row_base + lane;
                const long long row_offset = static_cast<long long>(outer) * p.outer_stride_c +
                                             static_cast<long long>(index) * p.stride_c +
                                             static_cast<long long>(row) * p.ldc;
#pragma unroll 1
                for (int c = first; c < first + kHalf; c += 32) {
                    const int col0 = col_base + c;
                    if (col0 >= p.n) {
                        break;
                    }
                    float v[32];
                    load_accumulator<32, BN, Split>(tmem_cols + c, v);
                    apply_epilogue<32>(v, p, col0);
                    if (row < p.m) {
                        store_direct(p, row_offset, col0, v);
                    }
                    __syncwarp();
                }
            }
            dev::tc_fence_before();
            dev::mbar_arrive(tempty_bar(acc));
        }
        if (p.c_tma && lane == 0) {
            dev::bulk_wait_group0();
        }
    } else if (Split && warp >= 4 + kEpilogueWarps) {
        // ---------------- 3xTF32 splitter ----------------
        const int t = threadIdx.x - 32 * (4 + kEpilogueWarps);
        int stage = 0;
        uint32_t phase = 0;
        const int total_blocks =
            ((p.total_tiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
             static_cast<int>(gridDim.x)) *
            p.k_blocks;
        for (int step = 0; step < total_blocks; ++step) {
            if (!dev::mbar_wait_warp(full_bar(stage), phase, p.status)) {
                break;
            }
            // In place: hi = rn_tf32(x) over the landed stage, lo = rn_tf32(x - hi) into the
            // stage's second half. Each thread loads four vectors before converting them, with
            // the rounding done by integer adds and masks, which is exact for |x| < 2^127 (no
            // carry can reach the exponent, and x - hi is exact in FP32); a warp that meets a
            // larger value, an infinity or a NaN redoes its vectors with the checked rounding.
            // Rounding the remainder (rather than letting the MMA truncate it) leaves at most
            // 2^-22 |x| of error per operand.
            const uint32_t hi_addr = stage_a(stage);
            const uint32_t lo_addr = stage_a(stage) + Shape::kABytes + Shape::kBBytes;
            constexpr int kVectors = (Shape::kABytes + Shape::kBBytes) / 16;
            static_assert(kVectors % 512 == 0, "whole rounds of four vectors per thread");
#pragma unroll 1
            for (int first = t; first < kVectors; first += 512) {
                float x[4][4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    dev::ld_shared_v4(hi_addr + 16u * static_cast<uint32_t>(first + 128 * u),
                                      x[u]);
                }
                float h[4][4];
                float l[4][4];
                bool special = false;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t bits = __float_as_uint(x[u][j]);
                        special |= (bits & 0x7FFFFFFFu) >= 0x7F000000u;
                        h[u][j] = __uint_as_float((bits + 0x1000u) & 0xFFFFE000u);
                        l[u][j] = __uint_as_float(
                            (__float_as_uint(x[u][j] - h[u][j]) + 0x1000u) & 0xFFFFE000u);
                    }
                }
                if (__any_sync(0xFFFFFFFFu, special)) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            h[u][j] = dev::round_to_tf32(x[u][j]);
                            const float rest = dev::round_to_tf32(x[u][j] - h[u][j]);
                            l[u][j] = (__float_as_uint(x[u][j]) & 0x7F800000u) == 0x7F800000u
                                          ? 0.0F
                                          : rest;
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const uint32_t offset = 16u * static_cast<uint32_t>(first + 128 * u);
                    dev::st_shared_v4(hi_addr + offset, h[u]);
                    dev::st_shared_v4(lo_addr + offset, l[u]);
                }
            }
            dev::fence_proxy_async_shared();
            dev::mbar_arrive(conv_bar(stage));
            if (++stage == kStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }

    __syncthreads();
    if (warp == 2) {
        dev::tc_fence_after();
        dev::tmem_dealloc(tmem_base, Shape::kTmemColumns);
    }
    dev::timeline_exit();
}

} // namespace cuvit::gemm
