// CTA-pair variant of the tcgen05 GEMM for bfloat16 operands with a K-major B (the weights'
// [N, K] layout): a cluster of two CTAs on neighbouring SMs computes one 256 x BN output tile
// with cta_group::2 MMAs (M = 256). Each CTA stages its own 128 rows of A and its own half
// of B's BN rows, so per output element every SM reads half the B bytes of the one-CTA
// kernel from shared memory and from L2 -- the traffic that bounds the one-CTA kernel.
//
// Protocol (CTA rank 0 of the pair is the leader):
//   warp 0, both CTAs   TMA producer: waits for its own "empty" stage barrier, loads its A
//                       rows and B half into its own stage, completing on its own "full"
//                       barrier
//   warp 3, rank 1      relay: once a stage of rank 1 has landed, arrives on the leader's
//                       "relay" barrier of that stage
//   warp 1, rank 0      MMA issuer: per stage (its own loads and the relay both in), four
//                       256 x BN x 16 MMAs over both CTAs' shared memory; commits free the
//                       stage in both CTAs; after a tile's last stage, commits mark the
//                       accumulator full in both CTAs
//   warps 4..11, both   epilogue of this CTA's 128 accumulator rows (its own TMEM lanes), as
//                       in the one-CTA kernel; one arrival per warp on the leader's
//                       "accumulator empty" barrier
//   warp 2, both        TMEM allocation and release for the pair
// Every wait is bounded; cluster barriers bracket the kernel so neither CTA can exit while
// the other may still touch its shared memory. No TMA load here signals another CTA or uses
// multicast: each CTA's loads complete on that CTA's own barriers.
#pragma once

#include "gemm_tc.cuh"

namespace cuvit::gemm {

template <int BN>
struct PairShape {
    static constexpr int kBlockK = kSwizzleBytes / 2;          // bf16 K elements per stage
    static constexpr int kABytes = kBlockM * kSwizzleBytes;    // this CTA's 128 rows of A
    static constexpr int kBBytes = (BN / 2) * kSwizzleBytes;   // this CTA's half of B
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStagesRaw = kSmemBudget / kStageBytes;
    static constexpr int kStages = kStagesRaw > 8 ? 8 : kStagesRaw;
    static constexpr int kTmemColumns = 2 * BN; // two FP32 accumulators of BN columns
    static constexpr int kThreads = 32 * (4 + kEpilogueWarps);
    static constexpr int kSlabOffset = kStages * kStageBytes;
    static constexpr int kBarrierOffset = kSlabOffset + kEpilogueWarps * kSlabBytes;
    // barriers: full, empty, relay per stage; accumulator full/empty x2; drain
    static constexpr int kBarrierBytes = (3 * kStages + 5) * 8 + 16;
    static constexpr int kSmemBytes = 1024 + kBarrierOffset + kBarrierBytes;
    static_assert(BN == 128 || BN == 256, "pair tiles are 256 x 128 or 256 x 256");
    static_assert(kStages >= 2, "at least two pipeline stages");
    static_assert(kSmemBytes <= 232448, "shared memory over the per-block limit");
};

template <int BN>
__global__ void __launch_bounds__(PairShape<BN>::kThreads, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a,
                        const __grid_constant__ CUtensorMap tma_b,
                        const __grid_constant__ CUtensorMap tma_c, const TcParams p) {
    dev::timeline_enter();
    using Shape = PairShape<BN>;
    constexpr int kStages = Shape::kStages;
    constexpr uint32_t kIdesc = dev::make_idesc(1u, 2 * kBlockM, BN, false, false);
    constexpr uint32_t kTxBytes = Shape::kABytes + Shape::kBBytes;

    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_base = dev::smem_u32(smem_raw);
    const uint32_t base = (raw_base + 1023u) & ~1023u;
    uint8_t* const smem = smem_raw + (base - raw_base);

    // Stage s: [A rows | B half]; then one output slab per epilogue warp; then barriers. Both
    // CTAs use the same offsets, which is what the pair MMA's descriptors assume.
    const auto stage_a = [&](int s) -> uint32_t { return base + s * Shape::kStageBytes; };
    const auto stage_b = [&](int s) -> uint32_t {
        return base + s * Shape::kStageBytes + Shape::kABytes;
    };
    const uint32_t bar_base = base + Shape::kBarrierOffset;
    const auto full_bar = [&](int s) -> uint32_t { return bar_base + 8u * s; };
    const auto empty_bar = [&](int s) -> uint32_t { return bar_base + 8u * (kStages + s); };
    const auto relay_bar = [&](int s) -> uint32_t { return bar_base + 8u * (2 * kStages + s); };
    const auto tfull_bar = [&](int a) -> uint32_t { return bar_base + 8u * (3 * kStages + a); };
    const auto tempty_bar = [&](int a) -> uint32_t {
        return bar_base + 8u * (3 * kStages + 2 + a);
    };
    const uint32_t drain_bar = bar_base + 8u * (3 * kStages + 4);
    uint32_t* const tmem_slot =
        reinterpret_cast<uint32_t*>(smem + Shape::kBarrierOffset + 8 * (3 * kStages + 5));

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const uint32_t rank = dev::cluster_ctarank();
    const bool leader = rank == 0;
    const int pair_id = static_cast<int>(dev::cluster_id_x());
    const int pair_count = static_cast<int>(dev::cluster_count_x());

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            dev::mbar_init(full_bar(s), 1);
            dev::mbar_init(empty_bar(s), 1);
            dev::mbar_init(relay_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            dev::mbar_init(tfull_bar(a), 1);
            dev::mbar_init(tempty_bar(a), 2 * kEpilogueWarps);
        }
        dev::mbar_init(drain_bar, 1);
        dev::fence_barrier_init();
    }
    if (warp == 2) {
        dev::tmem_alloc_pair(dev::smem_u32(tmem_slot), Shape::kTmemColumns);
        dev::tmem_relinquish_pair();
    }
    dev::tc_fence_before();
    __syncwarp();
    // Both CTAs' barriers exist (and the pair's TMEM is allocated) before anything remote.
    dev::cluster_sync();
    dev::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Inputs of this launch may come from the previous one: nothing global is read or
    // written before it has finished.
    dev::grid_dependency_wait();
    dev::grid_launch_dependents();

    const int per_entry = p.m_tiles * p.n_tiles; // m_tiles counts 256-row tiles here
    const int my_tiles =
        pair_id < p.total_tiles ? (p.total_tiles - pair_id + pair_count - 1) / pair_count : 0;

    if (warp == 0 && lane == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        dev::tma_prefetch_descriptor(&tma_a);
        dev::tma_prefetch_descriptor(&tma_b);
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int tile = pair_id; tile < p.total_tiles && ok; tile += pair_count) {
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
                int ca[4] = {k0, (2 * m_block + static_cast<int>(rank)) * kBlockM, 0, 0};
                int r = 2;
                if (p.a_has_index) ca[r++] = index;
                if (p.a_has_outer) ca[r++] = outer;
                dev::tma_load(stage_a(stage), &tma_a, full_bar(stage), p.a_rank, ca);
                int cb[4] = {k0, n_block * BN + static_cast<int>(rank) * (BN / 2), 0, 0};
                int rb = 2;
                if (p.b_has_index) cb[rb++] = index;
                if (p.b_has_outer) cb[rb++] = outer;
                dev::tma_load(stage_b(stage), &tma_b, full_bar(stage), p.b_rank, cb);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        if (!ok) {
            // Let every load this thread issued land before the CTA can exit.
            for (int s = 0; s < kStages; ++s) {
                dev::mbar_drain_wait(full_bar(s), phase ^ (s < stage ? 0u : 1u));
            }
        }
    } else if (warp == 3 && lane == 0 && !leader) {
        // ---------------- relay (rank 1): "this stage of mine has landed" ----------------
        const uint32_t leader_relay0 = dev::map_to_rank(relay_bar(0), 0);
        int stage = 0;
        uint32_t phase = 0;
        const int steps = my_tiles * p.k_blocks;
        for (int step = 0; step < steps; ++step) {
            if (!dev::mbar_wait(full_bar(stage), phase, p.status)) {
                break;
            }
            dev::mbar_arrive_remote(leader_relay0 + 8u * stage);
            if (++stage == kStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
    } else if (warp == 1 && lane == 0 && leader) {
        // ---------------- MMA issuer (rank 0) ----------------
        const uint32_t empty0_local = dev::map_to_rank(empty_bar(0), 0);
        const uint32_t empty0_peer = dev::map_to_rank(empty_bar(0), 1);
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int local = 0; local < my_tiles && ok; ++local) {
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!dev::mbar_wait(tempty_bar(acc), acc_phase ^ 1u, p.status)) {
                ok = false;
                break;
            }
            dev::tc_fence_after();
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
            for (int kb = 0; kb < p.k_blocks; ++kb) {
                if (!dev::mbar_wait(full_bar(stage), phase, p.status) ||
                    !dev::mbar_wait(relay_bar(stage), phase, p.status)) {
                    ok = false;
                    break;
                }
                dev::tc_fence_after();
                // Descriptors are stepped by adding to their start-address field (16-byte
                // units): 32 bytes per K step of 16.
                const uint64_t a_desc = dev::smem_desc_sw128(stage_a(stage), 16, 1024);
                const uint64_t b_desc = dev::smem_desc_sw128(stage_b(stage), 16, 1024);
#pragma unroll
                for (int kk = 0; kk < Shape::kBlockK / 16; ++kk) {
                    dev::mma_pair_f16(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, kIdesc,
                                      (kb > 0 || kk > 0) ? 1u : 0u);
                }
                dev::tc_commit_pair(empty0_local + 8u * stage);
                dev::tc_commit_pair(empty0_peer + 8u * stage);
                if (++stage == kStages) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (!ok) {
                break;
            }
            dev::tc_commit_pair(dev::map_to_rank(tfull_bar(acc), 0));
            dev::tc_commit_pair(dev::map_to_rank(tfull_bar(acc), 1));
        }
        // Every MMA issued has completed (so none still reads either CTA's shared memory or
        // writes TMEM) before this thread reaches the closing cluster barrier.
        dev::tc_commit_pair(dev::map_to_rank(drain_bar, 0));
        dev::mbar_drain_wait(drain_bar, 0);
    } else if (warp >= 4 && warp < 4 + kEpilogueWarps) {
        // ---------------- epilogue (both CTAs, this CTA's 128 rows) ----------------
        const int e = warp - 4;
        const int quarter = warp & 3; // the TMEM lane quarter this warp may access
        constexpr int kHalf = BN / 2;
        const int half = e >> 2;
        uint8_t* const slab = smem + Shape::kSlabOffset + e * kSlabBytes;
        const uint32_t slab_addr = base + Shape::kSlabOffset + e * kSlabBytes;
        const uint32_t lane_field = static_cast<uint32_t>(quarter * 32) << 16;
        const uint32_t leader_tempty0 = dev::map_to_rank(tempty_bar(0), 0);
        if (p.c_tma && lane == 0) {
            dev::tma_prefetch_descriptor(&tma_c);
        }
        int local = 0;
        for (int tile = pair_id; tile < p.total_tiles; tile += pair_count, ++local) {
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
            const int row_base = (2 * m_block + static_cast<int>(rank)) * kBlockM + quarter * 32;
            const uint32_t tmem_cols =
                tmem_base + lane_field + static_cast<uint32_t>(acc * BN);
            const int first = half * kHalf;
            const int col_base = n_block * BN;
            if (p.c_tma && (p.c_kind != 1 || kHalf >= 64)) {
                if (p.c_kind == 1) {
                    epilogue_tma<64, BN, false>(p, &tma_c, tmem_cols, first, first + kHalf,
                                                col_base, row_base, index, outer, slab,
                                                slab_addr, lane);
                } else {
                    epilogue_tma<32, BN, false>(p, &tma_c, tmem_cols, first, first + kHalf,
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
                    load_accumulator<32, BN, false>(tmem_cols + c, v);
                    apply_epilogue<32>(v, p, col0);
                    if (row < p.m) {
                        store_direct(p, row_offset, col0, v);
                    }
                    __syncwarp();
                }
            }
            dev::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                dev::mbar_arrive_remote(leader_tempty0 + 8u * acc);
            }
        }
        if (p.c_tma && lane == 0) {
            dev::bulk_wait_group0();
        }
    }

    dev::tc_fence_before();
    __syncwarp();
    dev::cluster_sync();
    if (warp == 2) {
        dev::tc_fence_after();
        dev::tmem_dealloc_pair(tmem_base, Shape::kTmemColumns);
    }
    dev::timeline_exit();
}

} // namespace cuvit::gemm
