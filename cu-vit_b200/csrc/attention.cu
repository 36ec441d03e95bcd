// Fused multi-head attention for ViT token counts (T <= 256, head_dim 64).
//
// Replaces the reference's three launches per block -- Q.K^T into a [B, h, T, T] logits
// buffer, an in-place row softmax, and P.V (src/model/vit.cu:205-242) -- with one kernel per
// (image, head) that never writes the logits to HBM:
//
//   1. TMA brings Q (two 128-row tiles), K and V of one head into shared memory with
//      128-byte swizzle, straight out of the packed [T, 3, h, d] projection rows.
//   2. One thread issues S = Q.K^T (tcgen05, K-major operands) into tensor memory.
//   3. Four softmax warps, one thread per query row, read their S row from TMEM twice (row
//      max, then exp/sum), and write P back into the same TMEM columns: packed bf16 pairs
//      for BF16, FP32 values (read as TF32) for the FP32 path.
//   4. O = P.V is issued with A = P read from TMEM and B = V (MN-major) from shared memory.
//   5. The softmax warps scale O by 1/rowsum and store it into the [T, h*d] context layout
//      the output projection reads.
//
// All T keys fit one tile, so the softmax is exact (no online rescaling).
#include "cuvit_b200.h"
#include "ptx.cuh"
#include "runtime.hpp"

#include <cuda_bf16.h>

#include <cstdint>

namespace cuvit::attn {
namespace {

constexpr int kHeadDim = 64;
constexpr int kTileQ = 128;
constexpr int kMaxTokens = 256;
constexpr int kThreads = 192; // warp 0 issuer, warp 1 TMEM, warps 2..5 softmax
// The FP32/TF32 instance: 16 softmax warps, the four of each TMEM lane quarter splitting the
// key chunks of its rows (P is stored in place there, so no column remapping is needed).
constexpr int kSplitSoftmaxWarps = 16;
constexpr int kSplitThreads = 64 + 32 * kSplitSoftmaxWarps;
// Row extreme and row sum of the four parts of each row, then the exchange barriers.
constexpr int kSplitExchangeBytes = 2 * 4 * 128 * 4;
// TMEM columns when both query tiles' scores are held at once (FP32 path, at most 224 keys):
// tile 1's scores at 224 and O at 448, after the 224 columns of each tile.
constexpr uint32_t kSecondScores = 224;
constexpr uint32_t kBothTilesO = 448;

template <int ElemBytes>
__host__ __device__ constexpr int softmax_warps() {
    return ElemBytes == 4 ? kSplitSoftmaxWarps : 4;
}

template <int ElemBytes>
__host__ __device__ constexpr int kernel_threads() {
    return ElemBytes == 4 ? kSplitThreads : kThreads;
}

struct Params {
    int tokens;
    int heads;
    int n_keys;  // tokens rounded up to 16 (MMA N)
    int q_tiles; // ceil(tokens / 128)
    float scale_log2; // scale * log2(e)
    float scale;
    void* context;
    int round_output; // FP32 path: store the context rounded to TF32 values
    int reverse;      // walk (image, head) pairs from the last to the first
    unsigned* status;
};

template <int ElemBytes>
struct Layout {
    static constexpr int kAtomElems = 128 / ElemBytes;           // elements per 128-byte row
    static constexpr int kDAtoms = kHeadDim / kAtomElems;        // 1 (bf16) or 2 (fp32)
    static constexpr int kMmaK = 32 / ElemBytes;                 // K per MMA instruction
    static constexpr int kQTileBytes = kDAtoms * kTileQ * 128;   // one 128-row Q tile
    static constexpr uint32_t kTmemColumns = ElemBytes == 2 ? 256 : 512;
    static constexpr int kOColumn = ElemBytes == 2 ? 128 : 256;
    // Minimum dynamic shared memory, chosen so TMEM demand per SM stays within 512 columns.
    static constexpr int kMinSmem = ElemBytes == 2 ? 80 * 1024 : 120 * 1024;
};

template <int ElemBytes>
__global__ void __launch_bounds__(kernel_threads<ElemBytes>())
    attention_kernel(const __grid_constant__ CUtensorMap map_q,
                     const __grid_constant__ CUtensorMap map_kv,
                     const __grid_constant__ CUtensorMap map_v, const Params p) {
    dev::timeline_enter();
    using L = Layout<ElemBytes>;
    using T = typename std::conditional<ElemBytes == 2, __nv_bfloat16, float>::type;
    constexpr dev::MmaKind kKind = ElemBytes == 2 ? dev::MmaKind::kF16 : dev::MmaKind::kTF32;
    constexpr uint32_t kFormat = ElemBytes == 2 ? 1u : 2u;
    // V is the MN-major operand of P.V: 32-bit elements need the 32-byte-atom swizzle.
    constexpr uint32_t kVLayout =
        ElemBytes == 4 ? dev::kLayoutSwizzle128Atom32 : dev::kLayoutSwizzle128;
    constexpr uint32_t kVAtomBytes = ElemBytes == 4 ? 512u : 1024u;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = dev::smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* const smem = smem_raw + (base - raw_base);

    const int kv_region = p.n_keys * 128; // one 128-byte-wide column block of K or V
    const uint32_t q_smem = base;
    const uint32_t k_smem = q_smem + p.q_tiles * L::kQTileBytes;
    const uint32_t v_smem = k_smem + L::kDAtoms * kv_region;
    const uint32_t bar_base = v_smem + L::kDAtoms * kv_region;
    const uint32_t bar_load = bar_base;
    const uint32_t bar_s = bar_base + 8;
    const uint32_t bar_p = bar_base + 16;
    const uint32_t bar_o = bar_base + 24;
    const uint32_t bar_free = bar_base + 32;
    const uint32_t bar_drain = bar_base + 40;
    const uint32_t bar_exchange = bar_base + 48; // {extreme, sum} x lane quarter (split path)
    // Split path with both query tiles' scores in TMEM at once: tile 1's scores and P.
    const uint32_t bar_s1 = bar_base + 112;
    const uint32_t bar_p1 = bar_base + 120;
    uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(smem + (bar_base - base) + 128);
    float* const exchange = reinterpret_cast<float*>(smem + (bar_base - base) + 256);
    constexpr uint32_t kSoftmaxThreads = 32u * softmax_warps<ElemBytes>();

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int job = p.reverse ? static_cast<int>(gridDim.x - 1 - blockIdx.x)
                              : static_cast<int>(blockIdx.x);
    const int image = job / p.heads;
    const int head = job - image * p.heads;
    // FP32/TF32 with two query tiles and at most 224 keys: both tiles' scores fit TMEM at once.
    const bool both_tiles = ElemBytes == 4 && p.q_tiles == 2 && p.n_keys <= kSecondScores;
    const uint32_t o_column = both_tiles ? kBothTilesO : static_cast<uint32_t>(L::kOColumn);

    if (threadIdx.x == 0) {
        dev::mbar_init(bar_load, 1);
        dev::mbar_init(bar_s, 1);
        dev::mbar_init(bar_p, kSoftmaxThreads);
        dev::mbar_init(bar_o, 1);
        dev::mbar_init(bar_free, kSoftmaxThreads);
        dev::mbar_init(bar_drain, 1);
        for (int x = 0; x < 8; ++x) {
            dev::mbar_init(bar_exchange + 8u * x, 4 * 32); // the four warps of a quarter
        }
        dev::mbar_init(bar_s1, 1);
        dev::mbar_init(bar_p1, kSoftmaxThreads);
        dev::fence_barrier_init();
    }
    if (warp == 1) {
        dev::tmem_alloc(dev::smem_u32(tmem_slot), L::kTmemColumns);
        dev::tmem_relinquish();
    }
    dev::tc_fence_before();
    __syncthreads();
    dev::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Inputs of this launch may come from the previous one: nothing global is read or
    // written before it has finished.
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();

    if (warp == 0 && lane == 0) {
        // ---------------- loads and MMA issue ----------------
        dev::tma_prefetch_descriptor(&map_q);
        dev::tma_prefetch_descriptor(&map_kv);
        dev::tma_prefetch_descriptor(&map_v);
        const int hd = p.heads * kHeadDim;
        const uint32_t bytes = static_cast<uint32_t>(p.q_tiles * L::kQTileBytes +
                                                     2 * L::kDAtoms * kv_region);
        dev::mbar_arrive_expect_tx(bar_load, bytes);
        for (int t = 0; t < p.q_tiles; ++t) {
            for (int j = 0; j < L::kDAtoms; ++j) {
                const int c[3] = {head * kHeadDim + j * L::kAtomElems, t * kTileQ, image};
                dev::tma_load(q_smem + t * L::kQTileBytes + j * kTileQ * 128, &map_q, bar_load, 3,
                              c);
            }
        }
        for (int j = 0; j < L::kDAtoms; ++j) {
            const int ck[3] = {hd + head * kHeadDim + j * L::kAtomElems, 0, image};
            dev::tma_load(k_smem + j * kv_region, &map_kv, bar_load, 3, ck);
            const int cv[3] = {2 * hd + head * kHeadDim + j * L::kAtomElems, 0, image};
            dev::tma_load(v_smem + j * kv_region, &map_v, bar_load, 3, cv);
        }
        bool ok = dev::mbar_wait(bar_load, 0, p.status);
        const uint32_t idesc_s = dev::make_idesc(kFormat, kTileQ, p.n_keys, false, false);
        constexpr uint32_t kIdescO = dev::make_idesc(kFormat, kTileQ, kHeadDim, false, true);
        constexpr int kStepsPerAtom = L::kAtomElems / L::kMmaK;
        const auto issue_scores = [&](int t, uint32_t column) {
#pragma unroll
            for (int kk = 0; kk < kHeadDim / L::kMmaK; ++kk) {
                const int atom = kk / kStepsPerAtom;
                const uint32_t offset = (kk % kStepsPerAtom) * 32;
                const uint64_t a_desc = dev::smem_desc_sw128(
                    q_smem + t * L::kQTileBytes + atom * kTileQ * 128 + offset, 16, 1024);
                const uint64_t b_desc =
                    dev::smem_desc_sw128(k_smem + atom * kv_region + offset, 16, 1024);
                dev::mma_ss<kKind>(tmem + column, a_desc, b_desc, idesc_s, kk > 0 ? 1u : 0u);
            }
        };
        const auto issue_context = [&](uint32_t column) {
            // O = P . V, P read from TMEM columns [column, column + n_keys * ElemBytes / 4)
            const int steps = p.n_keys / L::kMmaK;
            for (int kk = 0; kk < steps; ++kk) {
                const uint32_t a_tmem = tmem + column + static_cast<uint32_t>(kk * 8);
                const uint64_t b_desc =
                    dev::smem_desc(v_smem + kk * L::kMmaK * 128, static_cast<uint32_t>(kv_region),
                                   kVAtomBytes, kVLayout);
                dev::mma_ts<kKind>(tmem + o_column, a_tmem, b_desc, kIdescO,
                                   kk > 0 ? 1u : 0u);
            }
        };
        if (ok && both_tiles) {
            // Both tiles' scores at once (tile 1's at column kSecondScores); P.V of tile 0
            // runs while the softmax warps work on tile 1, P.V of tile 1 once O(0) is read.
            dev::tc_fence_after();
            issue_scores(0, 0u);
            dev::tc_commit(bar_s);
            issue_scores(1, kSecondScores);
            dev::tc_commit(bar_s1);
            ok = dev::mbar_wait(bar_p, 0, p.status);
            if (ok) {
                dev::tc_fence_after();
                issue_context(0u);
                dev::tc_commit(bar_o);
                ok = dev::mbar_wait(bar_free, 0, p.status) && dev::mbar_wait(bar_p1, 0, p.status);
            }
            if (ok) {
                dev::tc_fence_after();
                issue_context(kSecondScores);
                dev::tc_commit(bar_o);
            }
        }
        for (int t = 0; t < p.q_tiles && ok && !both_tiles; ++t) {
            // One tile at a time: S(t) reuses the columns of P(t - 1) once O(t - 1) is read.
            if (t > 0 && !dev::mbar_wait(bar_free, (t - 1) & 1, p.status)) {
                ok = false;
                break;
            }
            dev::tc_fence_after();
            issue_scores(t, 0u);
            dev::tc_commit(bar_s);
            if (!dev::mbar_wait(bar_p, t & 1, p.status)) {
                ok = false;
                break;
            }
            dev::tc_fence_after();
            issue_context(0u);
            dev::tc_commit(bar_o);
        }
        if (!ok) {
            // Wait until every MMA issued so far has finished before the CTA tears down.
            dev::tc_commit(bar_drain);
            dev::mbar_drain_wait(bar_drain, 0);
        }
    } else if (ElemBytes == 4 && warp >= 2) {
        // ---------------- softmax and output, split four ways per row ----------------
        // Warp w (2..17) has TMEM lane quarter w & 3 and part (w - 2) >> 2 of the key chunks
        // (32 columns each; parts take chunks / 4, the first chunks % 4 parts one more).
        const int part = (warp - 2) >> 2;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_field = static_cast<uint32_t>(quarter * 32) << 16;
        const int chunks = (p.n_keys + 31) / 32;
        const int c_begin = part * (chunks >> 2) + (part < (chunks & 3) ? part : (chunks & 3));
        const int c_end =
            (part + 1) * (chunks >> 2) + (part + 1 < (chunks & 3) ? part + 1 : (chunks & 3));
        float* const x_extreme = exchange;        // [part][row]
        float* const x_sum = exchange + 4 * kTileQ; // [part][row]
        const uint32_t extreme_bar = bar_exchange + 8u * static_cast<uint32_t>(quarter);
        const uint32_t sum_bar = extreme_bar + 32u;
        // Softmax of query tile t, whose scores start at TMEM column `column`: P (TF32 values)
        // in place, the hand-off on `p_bar`, the row sum into `sum`.
        const auto softmax_tile = [&](int t, uint32_t column, uint32_t s_bar, uint32_t s_parity,
                                      uint32_t p_bar, float& sum) -> bool {
            const uint32_t parity = static_cast<uint32_t>(t & 1);
            if (!dev::mbar_wait_warp(s_bar, s_parity, p.status)) {
                return false;
            }
            dev::tc_fence_after();
            const uint32_t scores = tmem + lane_field + column;
            float maximum = -INFINITY;
            for (int c = c_begin; c < c_end; ++c) {
                uint32_t s[32];
                dev::tmem_load_32(scores + c * 32, s);
                dev::tmem_wait_load();
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (c * 32 + j < p.tokens) {
                        maximum = fmaxf(maximum, __uint_as_float(s[j]) * p.scale);
                    }
                }
            }
            // The maximum is exact in any order; the four parts in a fixed order for the sum.
            x_extreme[part * kTileQ + row] = maximum;
            dev::mbar_arrive(extreme_bar);
            if (!dev::mbar_wait_warp(extreme_bar, parity, p.status)) {
                return false;
            }
            maximum = fmaxf(fmaxf(x_extreme[row], x_extreme[kTileQ + row]),
                            fmaxf(x_extreme[2 * kTileQ + row], x_extreme[3 * kTileQ + row]));
            const float offset = maximum * 1.4426950408889634F;
            float partial = 0.0F;
            for (int c = c_begin; c < c_end; ++c) {
                uint32_t s[32];
                dev::tmem_load_32(scores + c * 32, s);
                dev::tmem_wait_load();
                // P enters the tensor core as TF32: round it here (the MMA would truncate)
                // and normalise by the sum of exactly these values.
                uint32_t lo[16];
                uint32_t hi[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float a =
                        c * 32 + j < p.tokens
                            ? dev::round_to_tf32(
                                  exp2f(__uint_as_float(s[j]) * p.scale_log2 - offset))
                            : 0.0F;
                    const float b =
                        c * 32 + 16 + j < p.tokens
                            ? dev::round_to_tf32(
                                  exp2f(__uint_as_float(s[16 + j]) * p.scale_log2 - offset))
                            : 0.0F;
                    lo[j] = __float_as_uint(a);
                    hi[j] = __float_as_uint(b);
                    partial += a + b;
                }
                dev::tmem_store_16(scores + c * 32, lo);
                dev::tmem_store_16(scores + c * 32 + 16, hi);
            }
            x_sum[part * kTileQ + row] = partial;
            dev::tmem_wait_store();
            dev::tc_fence_before();
            dev::mbar_arrive(p_bar);
            dev::mbar_arrive(sum_bar);
            if (!dev::mbar_wait_warp(sum_bar, parity, p.status)) {
                return false;
            }
            sum = (x_sum[row] + x_sum[kTileQ + row]) +
                  (x_sum[2 * kTileQ + row] + x_sum[3 * kTileQ + row]);
            return true;
        };
        // O of query tile t (this warp's 16 columns), scaled by 1 / rowsum and stored; then O
        // is free for the next P.V.
        const auto readout_tile = [&](int t, float sum) -> bool {
            if (!dev::mbar_wait_warp(bar_o, static_cast<uint32_t>(t & 1), p.status)) {
                return false;
            }
            dev::tc_fence_after();
            uint32_t o[16];
            dev::tmem_load_16(tmem + lane_field + o_column + 16u * static_cast<uint32_t>(part), o);
            dev::tmem_wait_load();
            const float inverse = 1.0F / sum;
            const int query = t * kTileQ + row;
            if (query < p.tokens) {
                float* const out = static_cast<float*>(p.context) +
                                   (static_cast<long long>(image) * p.tokens + query) * p.heads *
                                       kHeadDim +
                                   head * kHeadDim + 16 * part;
                float4* const out4 = reinterpret_cast<float4*>(out);
                const bool round = p.round_output != 0;
                const auto finish = [inverse, round](uint32_t raw) {
                    const float value = __uint_as_float(raw) * inverse;
                    return round ? dev::round_to_tf32(value) : value;
                };
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    out4[q] = make_float4(finish(o[4 * q]), finish(o[4 * q + 1]),
                                          finish(o[4 * q + 2]), finish(o[4 * q + 3]));
                }
            }
            dev::tc_fence_before();
            dev::mbar_arrive(bar_free);
            return true;
        };
        if (both_tiles) {
            // Both softmaxes first (tile 0's P.V runs during tile 1's), then both read-outs.
            float sums[2] = {1.0F, 1.0F};
            if (softmax_tile(0, 0u, bar_s, 0u, bar_p, sums[0]) &&
                softmax_tile(1, kSecondScores, bar_s1, 0u, bar_p1, sums[1]) &&
                readout_tile(0, sums[0])) {
                readout_tile(1, sums[1]);
            }
        } else {
            for (int t = 0; t < p.q_tiles; ++t) {
                float sum = 1.0F;
                if (!softmax_tile(t, 0u, bar_s, static_cast<uint32_t>(t & 1), bar_p, sum) ||
                    !readout_tile(t, sum)) {
                    break;
                }
            }
        }
    } else if (warp >= 2) {
        // ---------------- softmax and output ----------------
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_field = static_cast<uint32_t>(quarter * 32) << 16;
        const int chunks = (p.n_keys + 31) / 32;
        for (int t = 0; t < p.q_tiles; ++t) {
            if (!dev::mbar_wait_warp(bar_s, t & 1, p.status)) {
                break;
            }
            dev::tc_fence_after();
            float maximum = -INFINITY;
            for (int c = 0; c < chunks; ++c) {
                uint32_t s[32];
                dev::tmem_load_32(tmem + lane_field + c * 32, s);
                dev::tmem_wait_load();
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    if (c * 32 + j < p.tokens) {
                        maximum = fmaxf(maximum, __uint_as_float(s[j]) * p.scale);
                    }
                }
            }
            const float offset = maximum * 1.4426950408889634F;
            float sum = 0.0F;
            for (int c = 0; c < chunks; ++c) {
                uint32_t s[32];
                dev::tmem_load_32(tmem + lane_field + c * 32, s);
                dev::tmem_wait_load();
                float e[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    e[j] = c * 32 + j < p.tokens
                               ? exp2f(__uint_as_float(s[j]) * p.scale_log2 - offset)
                               : 0.0F;
                }
                if constexpr (ElemBytes == 2) {
                    uint32_t packed[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        packed[j] = dev::pack_bf16x2(e[2 * j], e[2 * j + 1]);
                        const __nv_bfloat162 pair =
                            *reinterpret_cast<const __nv_bfloat162*>(&packed[j]);
                        const float2 rounded = __bfloat1622float2(pair);
                        sum += rounded.x + rounded.y;
                    }
                    dev::tmem_store_16(tmem + lane_field + c * 16, packed);
                } else {
                    // P enters the tensor core as TF32: round it here (the MMA would
                    // truncate) and normalise by the sum of exactly these values.
                    uint32_t lo[16];
                    uint32_t hi[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float a = dev::round_to_tf32(e[j]);
                        const float b = dev::round_to_tf32(e[16 + j]);
                        lo[j] = __float_as_uint(a);
                        hi[j] = __float_as_uint(b);
                        sum += a + b;
                    }
                    dev::tmem_store_16(tmem + lane_field + c * 32, lo);
                    dev::tmem_store_16(tmem + lane_field + c * 32 + 16, hi);
                }
            }
            dev::tmem_wait_store();
            dev::tc_fence_before();
            dev::mbar_arrive(bar_p);
            if (!dev::mbar_wait_warp(bar_o, t & 1, p.status)) {
                break;
            }
            dev::tc_fence_after();
            uint32_t o0[32];
            uint32_t o1[32];
            dev::tmem_load_32(tmem + lane_field + L::kOColumn, o0);
            dev::tmem_load_32(tmem + lane_field + L::kOColumn + 32, o1);
            dev::tmem_wait_load();
            const float inverse = 1.0F / sum;
            const int query = t * kTileQ + row;
            if (query < p.tokens) {
                T* const out = static_cast<T*>(p.context) +
                               (static_cast<long long>(image) * p.tokens + query) * p.heads *
                                   kHeadDim +
                               head * kHeadDim;
                if constexpr (ElemBytes == 2) {
                    uint4* const out4 = reinterpret_cast<uint4*>(out);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        out4[q] = make_uint4(
                            dev::pack_bf16x2(__uint_as_float(o0[8 * q]) * inverse,
                                             __uint_as_float(o0[8 * q + 1]) * inverse),
                            dev::pack_bf16x2(__uint_as_float(o0[8 * q + 2]) * inverse,
                                             __uint_as_float(o0[8 * q + 3]) * inverse),
                            dev::pack_bf16x2(__uint_as_float(o0[8 * q + 4]) * inverse,
                                             __uint_as_float(o0[8 * q + 5]) * inverse),
                            dev::pack_bf16x2(__uint_as_float(o0[8 * q + 6]) * inverse,
                                             __uint_as_float(o0[8 * q + 7]) * inverse));
                        out4[4 + q] = make_uint4(
                            dev::pack_bf16x2(__uint_as_float(o1[8 * q]) * inverse,
                                             __uint_as_float(o1[8 * q + 1]) * inverse),
                            dev::pack_bf16x2(__uint_as_float(o1[8 * q + 2]) * inverse,
                                             __uint_as_float(o1[8 * q + 3]) * inverse),
                            dev::pack_bf16x2(__uint_as_float(o1[8 * q + 4]) * inverse,
                                             __uint_as_float(o1[8 * q + 5]) * inverse),
                            dev::pack_bf16x2(__uint_as_float(o1[8 * q + 6]) * inverse,
                                             __uint_as_float(o1[8 * q + 7]) * inverse));
                    }
                } else {
                    float4* const out4 = reinterpret_cast<float4*>(out);
                    const bool round = p.round_output != 0;
                    const auto finish = [inverse, round](uint32_t raw) {
                        const float value = __uint_as_float(raw) * inverse;
                        return round ? dev::round_to_tf32(value) : value;
                    };
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        out4[q] = make_float4(finish(o0[4 * q]), finish(o0[4 * q + 1]),
                                              finish(o0[4 * q + 2]), finish(o0[4 * q + 3]));
                        out4[8 + q] = make_float4(finish(o1[4 * q]), finish(o1[4 * q + 1]),
                                                  finish(o1[4 * q + 2]), finish(o1[4 * q + 3]));
                    }
                }
            }
            dev::tc_fence_before();
            dev::mbar_arrive(bar_free);
        }
    }

    __syncthreads();
    if (warp == 1) {
        dev::tc_fence_after();
        dev::tmem_dealloc(tmem, L::kTmemColumns);
    }
    dev::timeline_exit();
}

// ---------------------------------------------------------------------------------------
// BF16: persistent, pipelined variant. One CTA per SM walks (image, head) pairs; Q, K, V of
// the next pair load into the second of two shared-memory buffers while the current pair is
// in softmax. Each 128-row query tile has its own 256-column TMEM region and two softmax
// warpgroups that split its key columns at `split` (a multiple of 32). The row extreme and
// the row sum are combined through shared memory; each warpgroup writes its packed bf16 P
// into the first half of its own score columns, so neither overwrites scores the other still
// reads: keys below `split` land at column key/2, the rest at split + (key - split)/2. O then
// accumulates into 64 columns that neither P occupies (`o_col`). Each softmax warp writes 32
// context rows x 32 features through a shared-memory slab by TMA store.
//
// Roles: warp 0 TMA loads, warps 1 and 3 MMA issue for query tiles 0 and 1, warp 2 TMEM;
// softmax warp w (4..19) has query tile ((w - 4) >> 2) & 1, key half (w - 4) >> 3 and TMEM
// lane quarter w & 3, so every SM sub-partition runs one warp of each (tile, half).
// ---------------------------------------------------------------------------------------
constexpr int kPipeThreads = 640;
constexpr int kPipeSoftmaxWarps = 16;
constexpr int kPipeSlabBytes = 32 * 64; // one warp's 32 context rows x 32 bf16 features
constexpr int kPipeExchangeBytes = 2 * 2 * 2 * kTileQ * 4; // {extreme, sum} x tile x half x row
// buf_full[2], buf_empty[2], s_full[2], p_full[2], o_full[2], o_free[2], drain[2], then the
// partner exchanges: {extreme, sum} x query tile x lane quarter
constexpr int kPipeExchangeBarrier = 14;
constexpr int kPipeBarriers = kPipeExchangeBarrier + 2 * 2 * 4;
// Key pairs of a 32-key chunk whose exponentials run on the FMA pipe (exp2_poly2), as a bit
// mask over the chunk's 16 pairs; the others use the special-function unit. The split
// balances that unit against the issue slots the polynomial takes: with the packed FP32
// polynomial, 6 pairs in 16 (ViT-B/16 at batch 256: 104.4 us per launch, against 106.5 for
// 4 in 16 and for 8 in 16).
constexpr uint32_t kPolyPairs = 0xA4A4u;

struct PipeParams {
    int tokens;
    int heads;
    int n_keys;
    int q_tiles;
    int pairs;        // batch * heads
    int buffer_bytes; // one Q/K/V buffer, 1024-aligned
    int split;        // first key column of the second softmax warpgroup
    int o_col;        // first TMEM column of O within a tile's region
    int reverse;      // walk (image, head) pairs from the last to the first
    float scale;
    float scale_log2;
    unsigned* status;
};

// Shared memory of the pipelined kernel for one Q/K/V buffer size.
constexpr int pipe_smem_bytes(int buffer_bytes) {
    return 1024 + 2 * buffer_bytes + kPipeSoftmaxWarps * kPipeSlabBytes + kPipeExchangeBytes +
           8 * kPipeBarriers + 16;
}

__global__ void __launch_bounds__(kPipeThreads, 1)
    attention_bf16_pipelined(const __grid_constant__ CUtensorMap map_q,
                             const __grid_constant__ CUtensorMap map_kv,
                             const __grid_constant__ CUtensorMap map_ctx, const PipeParams p) {
    dev::timeline_enter();
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = dev::smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* const smem = smem_raw + (base - raw_base);

    const int kv_region = p.n_keys * 128;
    const auto q_smem = [&](int b, int t) -> uint32_t {
        return base + b * p.buffer_bytes + t * kTileQ * 128;
    };
    const auto k_smem = [&](int b) -> uint32_t {
        return base + b * p.buffer_bytes + p.q_tiles * kTileQ * 128;
    };
    const auto v_smem = [&](int b) -> uint32_t { return k_smem(b) + kv_region; };
    const int slab_offset = 2 * p.buffer_bytes;
    const int exchange_offset = slab_offset + kPipeSoftmaxWarps * kPipeSlabBytes;
    const uint32_t bar_base = base + exchange_offset + kPipeExchangeBytes;
    // barriers: buf_full[2], buf_empty[2], s_full[2], p_full[2], o_full[2], o_free[2],
    // drain[2] (one per MMA issuer)
    const auto bar = [&](int kind, int i) -> uint32_t { return bar_base + 8u * (2 * kind + i); };
    constexpr int kBufFull = 0, kBufEmpty = 1, kSFull = 2, kPFull = 3, kOFull = 4, kOFree = 5;
    const uint32_t bar_drain0 = bar_base + 8u * 12;
    const uint32_t bar_drain1 = bar_base + 8u * 13;
    uint32_t* const tmem_slot = reinterpret_cast<uint32_t*>(
        smem + exchange_offset + kPipeExchangeBytes + 8 * kPipeBarriers);

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            dev::mbar_init(bar(kBufFull, i), 1);
            dev::mbar_init(bar(kBufEmpty, i), static_cast<uint32_t>(p.q_tiles));
            dev::mbar_init(bar(kSFull, i), 1);
            dev::mbar_init(bar(kPFull, i), 256);
            dev::mbar_init(bar(kOFull, i), 1);
            dev::mbar_init(bar(kOFree, i), 256);
        }
        dev::mbar_init(bar_drain0, 1);
        dev::mbar_init(bar_drain1, 1);
        for (int x = 0; x < 2 * 2 * 4; ++x) {
            dev::mbar_init(bar_base + 8u * (kPipeExchangeBarrier + x), 64); // two warps
        }
        dev::fence_barrier_init();
    }
    if (warp == 2) {
        dev::tmem_alloc(dev::smem_u32(tmem_slot), 512);
        dev::tmem_relinquish();
    }
    dev::tc_fence_before();
    __syncthreads();
    dev::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Inputs of this launch may come from the previous one: nothing global is read or
    // written before it has finished.
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();

    if (warp == 0 && lane == 0) {
        // ---------------- loads ----------------
        dev::tma_prefetch_descriptor(&map_q);
        dev::tma_prefetch_descriptor(&map_kv);
        const int hd = p.heads * kHeadDim;
        const uint32_t bytes =
            static_cast<uint32_t>(p.q_tiles * kTileQ * 128 + 2 * kv_region);
        int i = 0;
        for (int pair = blockIdx.x; pair < p.pairs; pair += gridDim.x, ++i) {
            const int b = i & 1;
            const uint32_t use = static_cast<uint32_t>(i >> 1);
            if (!dev::mbar_wait(bar(kBufEmpty, b), (use & 1u) ^ 1u, p.status)) {
                break;
            }
            const int job = p.reverse ? p.pairs - 1 - pair : pair;
            const int image = job / p.heads;
            const int head = job - image * p.heads;
            dev::mbar_arrive_expect_tx(bar(kBufFull, b), bytes);
            for (int t = 0; t < p.q_tiles; ++t) {
                const int c[3] = {head * kHeadDim, t * kTileQ, image};
                dev::tma_load(q_smem(b, t), &map_q, bar(kBufFull, b), 3, c);
            }
            const int ck[3] = {hd + head * kHeadDim, 0, image};
            dev::tma_load(k_smem(b), &map_kv, bar(kBufFull, b), 3, ck);
            const int cv[3] = {2 * hd + head * kHeadDim, 0, image};
            dev::tma_load(v_smem(b), &map_kv, bar(kBufFull, b), 3, cv);
        }
    } else if ((warp == 1 || (warp == 3 && p.q_tiles > 1)) && lane == 0) {
        // ---------------- MMA issue: warp 1 for query tile 0, warp 3 for tile 1 ----------------
        // Separate issuers let one tile's MMAs run while the other tile is in softmax, and
        // each commit tracks only its own thread's MMAs.
        const int t = warp == 1 ? 0 : 1;
        const uint32_t idesc_s = dev::make_idesc(1u, kTileQ, p.n_keys, false, false);
        constexpr uint32_t kIdescO = dev::make_idesc(1u, kTileQ, kHeadDim, false, true);
        const int steps = p.n_keys / 16;
        const int split_step = p.split / 16;
        // 16 keys per PV MMA: V advances 16 rows (2048 bytes); P sits at column key/2 below
        // the split and at split/2 + key/2 from it.
        const uint32_t region = tmem + static_cast<uint32_t>(256 * t);
        const uint32_t d_tmem = region + static_cast<uint32_t>(p.o_col);
        const uint32_t a_high = region + static_cast<uint32_t>(p.split / 2);
        const uint32_t bar_drain = t == 0 ? bar_drain0 : bar_drain1;
        bool ok = true;
        int i = 0;
        for (int pair = blockIdx.x; pair < p.pairs && ok; pair += gridDim.x, ++i) {
            const int b = i & 1;
            const uint32_t use = static_cast<uint32_t>(i >> 1);
            const uint32_t parity = static_cast<uint32_t>(i & 1);
            // The buffer's loads have landed and the previous pair's O_t has been read out of
            // this TMEM region.
            if (!dev::mbar_wait(bar(kBufFull, b), use & 1u, p.status) ||
                !dev::mbar_wait(bar(kOFree, t), parity ^ 1u, p.status)) {
                ok = false;
                break;
            }
            dev::tc_fence_after();
            // Descriptors are built once and stepped by adding to their start-address field
            // (16-byte units): 32 bytes per K step.
            const uint64_t q_desc = dev::smem_desc_sw128(q_smem(b, t), 16, 1024);
            const uint64_t k_desc = dev::smem_desc_sw128(k_smem(b), 16, 1024);
#pragma unroll
            for (int kk = 0; kk < kHeadDim / 16; ++kk) {
                dev::mma_ss<dev::MmaKind::kF16>(region, q_desc + 2 * kk, k_desc + 2 * kk,
                                                idesc_s, kk > 0 ? 1u : 0u);
            }
            dev::tc_commit(bar(kSFull, t));
            if (!dev::mbar_wait(bar(kPFull, t), parity, p.status)) {
                ok = false;
                break;
            }
            dev::tc_fence_after();
            const uint64_t v_desc = dev::smem_desc_sw128(v_smem(b), kv_region, 1024);
#pragma unroll
            for (int kk = 0; kk < kMaxTokens / 16; ++kk) {
                if (kk < steps) {
                    const uint32_t a_tmem = (kk < split_step ? region : a_high) + 8u * kk;
                    dev::mma_ts<dev::MmaKind::kF16>(d_tmem, a_tmem, v_desc + 128 * kk, kIdescO,
                                                    kk > 0 ? 1u : 0u);
                }
            }
            dev::tc_commit(bar(kOFull, t));
            dev::tc_commit(bar(kBufEmpty, b)); // one arrival per tile
        }
        if (!ok) {
            dev::tc_commit(bar_drain);
            dev::mbar_drain_wait(bar_drain, 0);
        }
    } else if (warp >= 4) {
        // ---------------- softmax and output ----------------
        const int sw = warp - 4;
        const int t = (sw >> 2) & 1;
        const int h = sw >> 3;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_field = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t region = tmem + lane_field + static_cast<uint32_t>(256 * t);
        uint8_t* const slab = smem + slab_offset + sw * kPipeSlabBytes;
        const uint32_t slab_addr = base + slab_offset + sw * kPipeSlabBytes;
        // Exchange: extreme[t][half][row], then sum[t][half][row].
        float* const x_extreme =
            reinterpret_cast<float*>(smem + exchange_offset) + t * 2 * kTileQ;
        float* const x_sum = x_extreme + 2 * 2 * kTileQ;
        // The two warps (key halves) of one query tile and lane quarter exchange row extreme
        // and row sum over mbarriers, whose waits are bounded like every other wait here: a
        // warp that gave up (another CTA timed out) cannot leave its partner blocked.
        const uint32_t extreme_bar =
            bar_base + 8u * static_cast<uint32_t>(kPipeExchangeBarrier + t * 4 + quarter);
        const uint32_t sum_bar = extreme_bar + 8u * 8u;
        // This warp's 32-column score chunks [c_begin, c_end) and where its P goes.
        const int chunks_all = (p.n_keys + 31) / 32;
        const int c_begin = h == 0 ? 0 : p.split / 32;
        const int c_end = h == 0 ? (p.split / 32 < chunks_all ? p.split / 32 : chunks_all)
                                 : chunks_all;
        const uint32_t p_base = h == 0 ? 0u : static_cast<uint32_t>(p.split);
        if (t < p.q_tiles) {
            if (lane == 0) {
                dev::tma_prefetch_descriptor(&map_ctx);
            }
            // A warp whose 32 query rows all lie past the token count has nothing to compute
            // (both halves of a row quarter agree): its O rows would be clipped by the store.
            const bool live = t * kTileQ + quarter * 32 < p.tokens;
            const bool positive = p.scale >= 0.0F;
            int i = 0;
            for (int pair = blockIdx.x; pair < p.pairs; pair += gridDim.x, ++i) {
                const uint32_t parity = static_cast<uint32_t>(i & 1);
                if (!dev::mbar_wait_warp(bar(kSFull, t), parity, p.status)) {
                    break;
                }
                dev::tc_fence_after();
                float sum = 1.0F;
                if (live) {
                    // The row extreme of the raw scores: the maximum for a positive scale, the
                    // minimum for a negative one; scale is applied once, to the extreme. Four
                    // independent accumulators keep the dependency chains short.
                    float ext[4];
#pragma unroll
                    for (int a = 0; a < 4; ++a) {
                        ext[a] = positive ? -INFINITY : INFINITY;
                    }
                    const auto reduce = [&](const uint32_t(&s)[32], int c) {
                        if ((c + 1) * 32 <= p.tokens) { // whole chunk of real keys
#pragma unroll
                            for (int j = 0; j < 32; j += 2) {
                                const float v0 = __uint_as_float(s[j]);
                                const float v1 = __uint_as_float(s[j + 1]);
                                const int a = (j >> 1) & 3;
                                ext[a] = positive ? dev::max3(ext[a], v0, v1)
                                                  : dev::min3(ext[a], v0, v1);
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j) {
                                if (c * 32 + j < p.tokens) {
                                    const float v = __uint_as_float(s[j]);
                                    ext[j & 3] =
                                        positive ? fmaxf(ext[j & 3], v) : fminf(ext[j & 3], v);
                                }
                            }
                        }
                    };
                    // One 32-column TMEM load per wait (the other warps of the sub-partition
                    // cover its latency); chunk indices relative to c_begin are compile-time,
                    // so the loaded values stay in registers.
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        const int c = c_begin + r;
                        if (c >= c_end) {
                            break;
                        }
                        uint32_t s0[32];
                        dev::tmem_load_32(region + c * 32, s0);
                        dev::tmem_wait_load();
                        reduce(s0, c);
                    }
                    float extreme = positive ? fmaxf(fmaxf(ext[0], ext[1]), fmaxf(ext[2], ext[3]))
                                             : fminf(fminf(ext[0], ext[1]), fminf(ext[2], ext[3]));
                    x_extreme[h * kTileQ + row] = extreme;
                    dev::mbar_arrive(extreme_bar);
                    if (!dev::mbar_wait_warp(extreme_bar, parity, p.status)) {
                        break;
                    }
                    const float other = x_extreme[(h ^ 1) * kTileQ + row];
                    extreme = positive ? fmaxf(extreme, other) : fminf(extreme, other);
                    const float offset = extreme * p.scale_log2;
                    // P = exp(scale * s - max), packed to bf16 pairs in place; the row sum is
                    // taken over the FP32 values. Key pairs go through sm_100's packed FP32
                    // arithmetic (two lanes per instruction).
                    uint64_t sums[4] = {0, 0, 0, 0}; // pairs of +0.0F
                    const uint64_t scale2 = dev::f32x2(p.scale_log2, p.scale_log2);
                    const uint64_t offset2 = dev::f32x2(-offset, -offset);
                    const auto exp_pack = [&](const uint32_t(&s)[32], int c, uint32_t column) {
                        uint32_t packed[16];
                        if ((c + 1) * 32 <= p.tokens) {
                            // The key pairs of kPolyPairs take 2^x on the FMA pipe, the rest
                            // on the special-function unit, which would otherwise bound the
                            // pass.
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                const float2 x = dev::f32x2_split(dev::fma_f32x2(
                                    dev::f32x2(__uint_as_float(s[2 * j]),
                                               __uint_as_float(s[2 * j + 1])),
                                    scale2, offset2));
                                const float2 e = ((kPolyPairs >> j) & 1u) != 0
                                                     ? dev::exp2_poly2(x.x, x.y)
                                                     : make_float2(dev::ex2_approx(x.x),
                                                                   dev::ex2_approx(x.y));
                                sums[j & 3] = dev::add_f32x2(sums[j & 3], dev::f32x2(e.x, e.y));
                                packed[j] = dev::pack_bf16x2(e.x, e.y);
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                const int key = c * 32 + 2 * j;
                                float e0 = 0.0F;
                                float e1 = 0.0F;
                                if (key < p.tokens) {
                                    e0 = dev::ex2_approx(
                                        fmaf(__uint_as_float(s[2 * j]), p.scale_log2, -offset));
                                }
                                if (key + 1 < p.tokens) {
                                    e1 = dev::ex2_approx(fmaf(__uint_as_float(s[2 * j + 1]),
                                                              p.scale_log2, -offset));
                                }
                                sums[j & 3] = dev::add_f32x2(sums[j & 3], dev::f32x2(e0, e1));
                                packed[j] = dev::pack_bf16x2(e0, e1);
                            }
                        }
                        dev::tmem_store_16(region + column, packed);
                    };
#pragma unroll
                    for (int r = 0; r < 8; ++r) {
                        const int c = c_begin + r;
                        if (c >= c_end) {
                            break;
                        }
                        uint32_t s0[32];
                        dev::tmem_load_32(region + c * 32, s0);
                        dev::tmem_wait_load();
                        exp_pack(s0, c, p_base + 16u * r);
                    }
                    const float2 s01 = dev::f32x2_split(dev::add_f32x2(sums[0], sums[1]));
                    const float2 s23 = dev::f32x2_split(dev::add_f32x2(sums[2], sums[3]));
                    const float partial = (s01.x + s01.y) + (s23.x + s23.y);
                    x_sum[h * kTileQ + row] = partial;
                    dev::tmem_wait_store();
                    dev::mbar_arrive(sum_bar);
                    if (!dev::mbar_wait_warp(sum_bar, parity, p.status)) {
                        break;
                    }
                    sum = partial + x_sum[(h ^ 1) * kTileQ + row];
                }
                dev::tc_fence_before();
                dev::mbar_arrive(bar(kPFull, t));
                if (!dev::mbar_wait_warp(bar(kOFull, t), parity, p.status)) {
                    break;
                }
                dev::tc_fence_after();
                uint32_t o[32];
                dev::tmem_load_32(region + static_cast<uint32_t>(p.o_col + 32 * h), o);
                dev::tmem_wait_load();
                dev::tc_fence_before();
                dev::mbar_arrive(bar(kOFree, t)); // this TMEM region may take the next S
                if (!live) {
                    continue;
                }
                const float inverse = 1.0F / sum;
                const uint64_t inverse2 = dev::f32x2(inverse, inverse);
                const auto scaled_pair = [&](int j) {
                    const float2 v = dev::f32x2_split(dev::mul_f32x2(
                        dev::f32x2(__uint_as_float(o[j]), __uint_as_float(o[j + 1])), inverse2));
                    return dev::pack_bf16x2(v.x, v.y);
                };
                if (lane == 0) {
                    dev::bulk_wait_group_read0(); // the slab's previous store has been read
                }
                __syncwarp();
                // 64-byte rows with the 64-byte swizzle of the context tensor map: 16-byte
                // chunk j of row r sits at chunk j ^ ((r >> 1) & 3).
                uint4* const slab_row = reinterpret_cast<uint4*>(slab + lane * 64);
                const int swizzle = (lane >> 1) & 3;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    slab_row[j ^ swizzle] = make_uint4(scaled_pair(8 * j), scaled_pair(8 * j + 2),
                                                       scaled_pair(8 * j + 4),
                                                       scaled_pair(8 * j + 6));
                }
                dev::fence_proxy_async_shared();
                __syncwarp();
                if (lane == 0) {
                    const int job = p.reverse ? p.pairs - 1 - pair : pair;
                    const int image = job / p.heads;
                    const int head = job - image * p.heads;
                    const int coords[3] = {head * kHeadDim + 32 * h,
                                           t * kTileQ + quarter * 32, image};
                    dev::tma_store<false>(&map_ctx, slab_addr, 3, coords);
                    dev::bulk_commit_group();
                }
            }
            if (lane == 0) {
                dev::bulk_wait_group0();
            }
        }
    }

    __syncthreads();
    if (warp == 2) {
        dev::tc_fence_after();
        dev::tmem_dealloc(tmem, 512);
    }
    dev::timeline_exit();
}

// Where the second softmax warpgroup's keys begin and where O accumulates, for n_keys score
// columns: the split (a multiple of 32) that balances the two warpgroups' chunk counts, then
// their real keys, among those that leave 64 TMEM columns free of both P halves. A split at
// the rounded end gives the whole row to the first warpgroup. Returns false if none fits.
bool choose_split(int tokens, int n_keys, int* split, int* o_col) {
    const int end = (n_keys + 31) / 32 * 32;
    const auto place_o = [&](int s) {
        const int first = (s / 2 + 31) / 32 * 32; // free columns [s/2, s) of the first half
        if (first + 64 <= s) {
            return first;
        }
        const int second = (s + (end - s) / 2 + 31) / 32 * 32; // past the second P half
        return second + 64 <= 256 ? second : -1;
    };
    int best_cost = 1 << 30;
    for (int s = 32; s <= end; s += 32) {
        const int o = place_o(s);
        if (o < 0) {
            continue;
        }
        const int chunks = s / 32 > (end - s) / 32 ? s / 32 : (end - s) / 32;
        const int keys_first = s < tokens ? s : tokens;
        const int keys_second = tokens - keys_first;
        const int keys = keys_first > keys_second ? keys_first : keys_second;
        const int cost = chunks * 1024 + keys;
        if (cost < best_cost) {
            best_cost = cost;
            *split = s;
            *o_col = o;
        }
    }
    return best_cost < (1 << 30);
}

template <int ElemBytes>
int launch_typed(const void* qkv, void* context, int batch, int tokens, int heads, float scale,
                 bool round_output, const host::DeviceContext& device, cudaStream_t stream);

int launch_bf16_pipelined(const void* qkv, void* context, int batch, int tokens, int heads,
                          float scale, const host::DeviceContext& device, cudaStream_t stream) {
    const int n_keys = (tokens + 15) / 16 * 16;
    const int q_tiles = (tokens + kTileQ - 1) / kTileQ;
    const int row = 3 * heads * kHeadDim;
    const int e = heads * kHeadDim;
    const int buffer_bytes = (q_tiles * kTileQ * 128 + 2 * n_keys * 128 + 1023) / 1024 * 1024;
    int split = 0;
    int o_col = 0;
    if (pipe_smem_bytes(buffer_bytes) > 227 * 1024 || !choose_split(tokens, n_keys, &split, &o_col)) {
        // Two buffers do not fit next to the slabs (more than 240 tokens): one pair at a time.
        return launch_typed<2>(qkv, context, batch, tokens, heads, scale, false, device, stream);
    }

    host::TmaTensor tq;
    tq.base = qkv;
    tq.type = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    tq.element_bytes = 2;
    tq.rank = 3;
    tq.dims[0] = static_cast<uint64_t>(row);
    tq.dims[1] = static_cast<uint64_t>(tokens);
    tq.dims[2] = static_cast<uint64_t>(batch);
    tq.strides_bytes[0] = static_cast<uint64_t>(row) * 2;
    tq.strides_bytes[1] = static_cast<uint64_t>(row) * tokens * 2;
    tq.box[0] = 64;
    tq.box[1] = kTileQ;
    tq.box[2] = 1;
    host::TmaTensor tkv = tq;
    tkv.box[1] = static_cast<uint32_t>(n_keys);
    host::TmaTensor tc;
    tc.base = context;
    tc.type = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    tc.element_bytes = 2;
    tc.rank = 3;
    tc.dims[0] = static_cast<uint64_t>(e);
    tc.dims[1] = static_cast<uint64_t>(tokens);
    tc.dims[2] = static_cast<uint64_t>(batch);
    tc.strides_bytes[0] = static_cast<uint64_t>(e) * 2;
    tc.strides_bytes[1] = static_cast<uint64_t>(e) * tokens * 2;
    tc.box[0] = 32;
    tc.box[1] = 32;
    tc.box[2] = 1;
    tc.swizzle = CU_TENSOR_MAP_SWIZZLE_64B;

    CUtensorMap map_q;
    CUtensorMap map_kv;
    CUtensorMap map_ctx;
    CUVIT_TRY(host::encode_tma(tq, &map_q));
    CUVIT_TRY(host::encode_tma(tkv, &map_kv));
    CUVIT_TRY(host::encode_tma(tc, &map_ctx));

    PipeParams params;
    params.tokens = tokens;
    params.heads = heads;
    params.n_keys = n_keys;
    params.q_tiles = q_tiles;
    params.pairs = batch * heads;
    params.buffer_bytes = buffer_bytes;
    params.split = split;
    params.o_col = o_col;
    params.reverse = host::reverse_sweep() ? 1 : 0;
    params.scale = scale;
    params.scale_log2 = scale * 1.4426950408889634F;
    params.status = device.status;

    const int smem = pipe_smem_bytes(buffer_bytes);
    auto* kernel = &attention_bf16_pipelined;
    CUVIT_TRY_CUDA(host::allow_dynamic_smem(reinterpret_cast<const void*>(kernel), 227 * 1024));
    const int grid = params.pairs < device.sm_count ? params.pairs : device.sm_count;
    host::pdl_launch(kernel, grid, kPipeThreads, smem, stream, map_q, map_kv, map_ctx, params);
    return host::after_launch("attention_bf16_pipelined");
}

template <int ElemBytes>
int launch_typed(const void* qkv, void* context, int batch, int tokens, int heads, float scale,
                 bool round_output, const host::DeviceContext& device, cudaStream_t stream) {
    using L = Layout<ElemBytes>;
    const int n_keys = (tokens + 15) / 16 * 16;
    const int q_tiles = (tokens + kTileQ - 1) / kTileQ;
    const int row = 3 * heads * kHeadDim;

    host::TmaTensor tq;
    tq.base = qkv;
    tq.type = ElemBytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    tq.element_bytes = ElemBytes;
    tq.rank = 3;
    tq.dims[0] = static_cast<uint64_t>(row);
    tq.dims[1] = static_cast<uint64_t>(tokens);
    tq.dims[2] = static_cast<uint64_t>(batch);
    tq.strides_bytes[0] = static_cast<uint64_t>(row) * ElemBytes;
    tq.strides_bytes[1] = static_cast<uint64_t>(row) * tokens * ElemBytes;
    tq.box[0] = L::kAtomElems;
    tq.box[1] = kTileQ;
    tq.box[2] = 1;
    host::TmaTensor tkv = tq;
    tkv.box[1] = static_cast<uint32_t>(n_keys);
    host::TmaTensor tv = tkv;
    if (ElemBytes == 4) {
        tv.swizzle = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    }

    CUtensorMap map_q;
    CUtensorMap map_kv;
    CUtensorMap map_v;
    CUVIT_TRY(host::encode_tma(tq, &map_q));
    CUVIT_TRY(host::encode_tma(tkv, &map_kv));
    CUVIT_TRY(host::encode_tma(tv, &map_v));

    Params params;
    params.tokens = tokens;
    params.heads = heads;
    params.n_keys = n_keys;
    params.q_tiles = q_tiles;
    params.scale = scale;
    params.scale_log2 = scale * 1.4426950408889634F;
    params.context = context;
    params.round_output = round_output ? 1 : 0;
    params.reverse = host::reverse_sweep() ? 1 : 0;
    params.status = device.status;

    // Operand tiles, then barriers and the TMEM slot (256 bytes), then the row exchange.
    int smem = 1024 + q_tiles * L::kQTileBytes + 2 * L::kDAtoms * n_keys * 128 + 256 +
               kSplitExchangeBytes;
    if (smem < L::kMinSmem) {
        smem = L::kMinSmem;
    }
    auto* kernel = &attention_kernel<ElemBytes>;
    CUVIT_TRY_CUDA(host::allow_dynamic_smem(reinterpret_cast<const void*>(kernel), 227 * 1024));
    host::pdl_launch(kernel, batch * heads, kernel_threads<ElemBytes>(), smem, stream, map_q,
                     map_kv, map_v, params);
    return host::after_launch("attention_kernel");
}

} // namespace
} // namespace cuvit::attn

extern "C" int cuvit_attention(const void* qkv, void* context, int dtype, int batch, int tokens,
                               int heads, int head_dim, float scale, cuvit_stream_t stream) {
    using cuvit::host::fail;
    if (batch == 0) {
        return CUVIT_OK;
    }
    if (batch < 0 || tokens <= 0 || heads <= 0 || head_dim <= 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "attention extents must be positive");
    }
    if (qkv == nullptr || context == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "attention operands cannot be null");
    }
    if (dtype != CUVIT_DTYPE_BF16 && dtype != CUVIT_DTYPE_F32 && dtype != CUVIT_DTYPE_TF32) {
        return fail(CUVIT_INVALID_ARGUMENT, "attention data type must be BF16, F32 or TF32");
    }
    if (head_dim != cuvit::attn::kHeadDim || tokens > cuvit::attn::kMaxTokens) {
        return fail(CUVIT_UNSUPPORTED,
                    "fused attention supports head_dim 64 and at most 256 tokens");
    }
    if (reinterpret_cast<uintptr_t>(qkv) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(context) % 16 != 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "attention operands must be 16-byte aligned");
    }
    if (static_cast<long long>(batch) * heads > 0x7FFFFFFFLL) {
        return fail(CUVIT_LENGTH_ERROR, "attention launch exceeds the CUDA grid limit");
    }
    const cuvit::host::DeviceContext* device = nullptr;
    CUVIT_TRY(cuvit::host::current_context(&device));
    if (!cuvit::host::is_blackwell(*device)) {
        return fail(CUVIT_UNSUPPORTED, "fused attention needs an sm_100 device");
    }
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (dtype == CUVIT_DTYPE_BF16) {
        return cuvit::attn::launch_bf16_pipelined(qkv, context, batch, tokens, heads, scale,
                                                  *device, s);
    }
    return cuvit::attn::launch_typed<4>(qkv, context, batch, tokens, heads, scale,
                                        dtype == CUVIT_DTYPE_TF32, *device, s);
}
