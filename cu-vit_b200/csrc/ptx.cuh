// Inline-PTX building blocks for sm_100a kernels: mbarriers with bounded waits, TMA tile
// loads, and the tcgen05 family (TMEM allocation, MMA issue, commit, TMEM <-> register
// moves). Every wait in this library goes through mbar_wait(), which gives up after
// kWaitLimitNs, records kStatusTimeout in the device status word and returns false so the
// caller can unwind instead of spinning forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "timeline.cuh"

namespace cuvit::dev {

// Device status word bits (read and cleared by cuvit_device_status()).
constexpr unsigned kStatusTimeout = 1u;

// Upper bound on any single wait. Legitimate waits here last microseconds.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* pointer) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(pointer));
}

__device__ __forceinline__ unsigned long long global_timer_ns() {
    unsigned long long value;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(value));
    return value;
}

__device__ __forceinline__ unsigned load_volatile(const unsigned* address) {
    return *reinterpret_cast<const volatile unsigned*>(address);
}

// ---- mbarrier ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t"
        ".reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t"
        "}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase with the given parity to complete. Returns false (and flags the
// status word) when the wait exceeds kWaitLimitNs or another waiter already gave up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, unsigned* status,
                                          unsigned long long limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) {
        return true;
    }
    const unsigned long long start = global_timer_ns();
    while (true) {
#pragma unroll 1
        for (int spin = 0; spin < 32; ++spin) {
            if (mbar_try_wait(bar, parity)) {
                return true;
            }
        }
        if (load_volatile(status) & kStatusTimeout) {
            return false;
        }
        if (global_timer_ns() - start > limit_ns) {
            atomicOr(status, kStatusTimeout);
            return false;
        }
    }
}

// mbar_wait by all 32 lanes of a warp, succeeding or failing for the whole warp, so that a
// warp-wide instruction after it (tcgen05.ld / st are .sync.aligned) never runs with some lanes
// gone: lanes of one warp can disagree when the wait runs out.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, unsigned* status) {
    return __all_sync(0xFFFFFFFFu, mbar_wait(bar, parity, status));
}

// Waits up to limit_ns for a phase regardless of the status word: used after a failure to
// let this thread's own copies in flight land before the CTA exits.
__device__ __forceinline__ bool mbar_drain_wait(uint32_t bar, uint32_t parity,
                                                unsigned long long limit_ns = 100000000ull) {
    const unsigned long long start = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - start > limit_ns) {
            return false;
        }
    }
    return true;
}

// ---- thread-block clusters --------------------------------------------------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t rank;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    return rank;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t id;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(id));
    return id;
}

__device__ __forceinline__ uint32_t cluster_count_x() {
    uint32_t count;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(count));
    return count;
}

// The shared::cluster address of shared-memory offset `addr` in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
    uint32_t mapped;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(mapped) : "r"(addr), "r"(rank));
    return mapped;
}

// Every thread of every CTA in the cluster; orders shared-memory accesses across the cluster.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// One arrival on an mbarrier anywhere in the cluster (a shared::cluster address). As for
// local barriers, the waiting side uses mbar_wait(): data handed over this way lives in
// shared memory or TMEM, and every consumer reaches it through the async proxy or tcgen05
// after that wait.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// Programmatic dependent launch: kernels are launched so that they may start while the
// previous kernel in the stream is still finishing. Each kernel runs its prologue (barrier
// set-up, TMEM allocation, descriptor prefetch), then waits here until the previous grid has
// completed and its writes are visible, before touching any data. Without the launch
// attribute the wait returns at once.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Lets the next kernel in the stream begin launching (its CTAs still wait for this grid to
// complete before reading anything).
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Four floats from / to a 16-byte aligned shared-memory address.
__device__ __forceinline__ void ld_shared_v4(uint32_t address, float (&v)[4]) {
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
                 : "r"(address));
}

__device__ __forceinline__ void st_shared_v4(uint32_t address, const float (&v)[4]) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(address), "f"(v[0]),
                 "f"(v[1]), "f"(v[2]), "f"(v[3])
                 : "memory");
}

// Makes generic-proxy shared-memory writes visible to the async proxy (TMA, tensor core).
__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- TMA --------------------------------------------------------------------------------

__device__ __forceinline__ void tma_prefetch_descriptor(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Tiled load of a box at integer coordinates c[0..rank) into shared memory, completing
// transaction bytes on the mbarrier. Coordinate 0 is the innermost dimension.
__device__ __forceinline__ void tma_load(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                         int rank, const int* c) {
    const uint64_t desc = reinterpret_cast<uint64_t>(map);
    switch (rank) {
    case 2:
        asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::"
                     "bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
                     "l"(desc), "r"(bar), "r"(c[0]), "r"(c[1])
                     : "memory");
        break;
    case 3:
        asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::"
                     "bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
                     "l"(desc), "r"(bar), "r"(c[0]), "r"(c[1]), "r"(c[2])
                     : "memory");
        break;
    default:
        asm volatile("cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::"
                     "bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
                     "l"(desc), "r"(bar), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3])
                     : "memory");
        break;
    }
}

// Tiled store of a shared-memory box to global memory at coordinates c[0..rank) (bulk
// group completion); with Reduce, the box is added into global memory (FP32 add in L2).
template <bool Reduce>
__device__ __forceinline__ void tma_store(const CUtensorMap* map, uint32_t src, int rank,
                                          const int* c) {
    const uint64_t desc = reinterpret_cast<uint64_t>(map);
    if constexpr (Reduce) {
        switch (rank) {
        case 2:
            asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group "
                         "[%0, {%2, %3}], [%1];" ::"l"(desc),
                         "r"(src), "r"(c[0]), "r"(c[1])
                         : "memory");
            break;
        case 3:
            asm volatile("cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group "
                         "[%0, {%2, %3, %4}], [%1];" ::"l"(desc),
                         "r"(src), "r"(c[0]), "r"(c[1]), "r"(c[2])
                         : "memory");
            break;
        default:
            asm volatile("cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group "
                         "[%0, {%2, %3, %4, %5}], [%1];" ::"l"(desc),
                         "r"(src), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3])
                         : "memory");
            break;
        }
    } else {
        switch (rank) {
        case 2:
            asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group "
                         "[%0, {%2, %3}], [%1];" ::"l"(desc),
                         "r"(src), "r"(c[0]), "r"(c[1])
                         : "memory");
            break;
        case 3:
            asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group "
                         "[%0, {%2, %3, %4}], [%1];" ::"l"(desc),
                         "r"(src), "r"(c[0]), "r"(c[1]), "r"(c[2])
                         : "memory");
            break;
        default:
            asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group "
                         "[%0, {%2, %3, %4, %5}], [%1];" ::"l"(desc),
                         "r"(src), "r"(c[0]), "r"(c[1]), "r"(c[2]), "r"(c[3])
                         : "memory");
            break;
        }
    }
}

__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Waits until the shared-memory sources of all committed bulk stores have been read.
__device__ __forceinline__ void bulk_wait_group_read0() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Waits until all committed bulk stores have completed.
__device__ __forceinline__ void bulk_wait_group0() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ---- tcgen05 ----------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t columns) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     dst_smem),
                 "r"(columns)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t columns) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr),
                 "r"(columns)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrives on the mbarrier once all tcgen05 operations this thread issued so far complete.
// ---- CTA pairs (cta_group::2): one MMA spans the tensor memory of both CTAs -------------

// Both CTAs of the pair call these from the same warp index, with the same slot offset.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t columns) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     dst_smem),
                 "r"(columns)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t columns) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr),
                 "r"(columns)
                 : "memory");
}

// D (M = 256: rows 0..127 in this CTA's TMEM, 128..255 in the peer's) (+)= A * B, where each
// CTA holds its own 128 rows of A and half of B's N rows at the same shared-memory offsets.
// Issued by the pair's even CTA only.
__device__ __forceinline__ void mma_pair_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t"
        ".reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t"
        "}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// One arrival on the mbarrier at shared::cluster address `bar` (in either CTA of the pair)
// once every pair MMA this thread has issued so far has completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t cluster_bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            cluster_bar)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}

// Shared-memory layouts a matrix descriptor can name (bits 61..63).
constexpr uint32_t kLayoutSwizzle128 = 2;       // 16-byte chunks over 128-byte rows, 8-row atoms
constexpr uint32_t kLayoutSwizzle128Atom32 = 1; // 32-byte chunks over 128-byte rows, 4-row atoms

// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"): start address, leading and
// stride byte offsets (16-byte units), descriptor version 1, swizzle layout.
__device__ __forceinline__ uint64_t smem_desc(uint32_t address, uint32_t lbo_bytes,
                                              uint32_t sbo_bytes, uint32_t layout) {
    uint64_t desc = 0;
    desc |= static_cast<uint64_t>((address & 0x3FFFFu) >> 4);
    desc |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    desc |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    desc |= 1ull << 46;
    desc |= static_cast<uint64_t>(layout) << 61;
    return desc;
}

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t address, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
    return smem_desc(address, lbo_bytes, sbo_bytes, kLayoutSwizzle128);
}

// Instruction descriptor for kind::f16 / kind::tf32 with FP32 accumulation.
// format: 0 = F16, 1 = BF16, 2 = TF32. mn_major: operand stored MN-major (else K-major).
__host__ __device__ constexpr uint32_t make_idesc(uint32_t format, int m, int n, bool a_mn_major,
                                                  bool b_mn_major) {
    return (1u << 4) | (format << 7) | (format << 10) | (static_cast<uint32_t>(a_mn_major) << 15) |
           (static_cast<uint32_t>(b_mn_major) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

enum class MmaKind { kF16, kTF32 };

// D(tmem) (+)= A(smem desc) * B(smem desc)
template <MmaKind Kind>
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    if constexpr (Kind == MmaKind::kF16) {
        asm volatile(
            "{\n\t"
            ".reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
            "}\n" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t"
            ".reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t"
            "}\n" ::"r"(d_tmem),
            "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// D(tmem) (+)= A(tmem) * B(smem desc)
template <MmaKind Kind>
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    if constexpr (Kind == MmaKind::kF16) {
        asm volatile(
            "{\n\t"
            ".reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
            "}\n" ::"r"(d_tmem),
            "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t"
            ".reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t"
            "}\n" ::"r"(d_tmem),
            "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
            : "memory");
    }
}

// Loads 32 consecutive 32-bit TMEM columns of this warp's 32 lanes (lane i -> thread i).
__device__ __forceinline__ void tmem_load_32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
        "[%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

// Loads 16 consecutive 32-bit TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_load_16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                   "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
}

// Stores 16 consecutive 32-bit TMEM columns of this warp's 32 lanes.
__device__ __forceinline__ void tmem_store_16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_load() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_store() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---- numeric helpers --------------------------------------------------------------------

// The erf form of GELU, matching nn.GELU(approximate='none') and the reference's epilogue
// (src/kernels/gemm.cu:157-160).
__device__ __forceinline__ float gelu_erf(float value) {
    return 0.5F * value * (1.0F + erff(value * 0.7071067811865475F));
}

// Rounds an FP32 value to the nearest TF32 value (10-bit mantissa, ties away from zero in
// magnitude); non-finite values pass through. The tensor core would otherwise truncate the
// low 13 mantissa bits of a TF32 operand, a bias that accumulates over long reductions.
// Written with selects rather than branches: in the 3xTF32 splitter's loop the branches kept
// its shared-memory loads from overlapping and made the conversion six times slower.
__device__ __forceinline__ float round_to_tf32(float x) {
    const uint32_t bits = __float_as_uint(x);
    const uint32_t rounded = (bits + 0x1000u) & 0xFFFFE000u;
    // A carry into an all-ones exponent would turn a finite value into infinity: truncate.
    const uint32_t finite_result =
        (rounded & 0x7F800000u) == 0x7F800000u ? (bits & 0xFFFFE000u) : rounded;
    return __uint_as_float((bits & 0x7F800000u) == 0x7F800000u ? bits : finite_result);
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Two FP32 values in one 64-bit register for sm_100's packed FP32 arithmetic: add, mul and
// fma .rn.f32x2 perform two IEEE round-to-nearest operations per instruction, so code written
// with them gives the results of the scalar operations in half the issue slots.
__device__ __forceinline__ uint64_t f32x2(float low, float high) {
    uint64_t packed;
    asm("mov.b64 %0, {%1, %2};" : "=l"(packed) : "f"(low), "f"(high));
    return packed;
}

__device__ __forceinline__ float2 f32x2_split(uint64_t packed) {
    float2 pair;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(pair.x), "=f"(pair.y) : "l"(packed));
    return pair;
}

__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ uint64_t sub_f32x2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// Three-operand maximum / minimum (sm_100): two new values per instruction in a reduction.
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

__device__ __forceinline__ float min3(float a, float b, float c) {
    float d;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// 2^x for x <= 0 on the FMA pipe, to relieve the special-function unit: x = n + f with n
// the nearest integer (x + 1.5 * 2^23 leaves n in the low mantissa bits) and f in
// [-1/2, 1/2]; 2^f from a degree-3 polynomial fitted here by Remez exchange for minimax
// relative error on [-1/2, 1/2] (7.5e-5, evaluated in FP32); 2^n is added to the exponent
// field. Arguments below -125 are raised to -125 so the exponent stays normal.
__device__ __forceinline__ float exp2_poly(float x) {
    x = fmaxf(x, -125.0F);
    const float shifted = __fadd_rn(x, 12582912.0F);
    const float n = __fadd_rn(shifted, -12582912.0F);
    const float f = __fadd_rn(x, -n);
    float p = fmaf(0.0551716685F, f, 0.2426111251F);
    p = fmaf(p, f, 0.6932609677F);
    p = fmaf(p, f, 0.9999280572F);
    return __int_as_float(__float_as_int(p) + (__float_as_int(shifted) << 23));
}

// exp2_poly on two values, the additions and the polynomial two per instruction: the same
// operations in the same order, so the same results.
__device__ __forceinline__ float2 exp2_poly2(float x0, float x1) {
    const uint64_t x = f32x2(fmaxf(x0, -125.0F), fmaxf(x1, -125.0F));
    const uint64_t shifted = add_f32x2(x, f32x2(12582912.0F, 12582912.0F));
    const uint64_t n = add_f32x2(shifted, f32x2(-12582912.0F, -12582912.0F));
    const uint64_t f = sub_f32x2(x, n);
    uint64_t p = fma_f32x2(f32x2(0.0551716685F, 0.0551716685F), f,
                           f32x2(0.2426111251F, 0.2426111251F));
    p = fma_f32x2(p, f, f32x2(0.6932609677F, 0.6932609677F));
    p = fma_f32x2(p, f, f32x2(0.9999280572F, 0.9999280572F));
    const float2 poly = f32x2_split(p);
    const float2 scale = f32x2_split(shifted);
    return make_float2(__int_as_float(__float_as_int(poly.x) + (__float_as_int(scale.x) << 23)),
                       __int_as_float(__float_as_int(poly.y) + (__float_as_int(scale.y) << 23)));
}

__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// GELU with erf evaluated by Abramowitz & Stegun, Handbook of Mathematical Functions,
// formula 7.1.26 (|error| <= 1.5e-7 on erf), using the hardware reciprocal and exponential.
// For BF16 outputs, whose rounding (2^-9 relative) is far coarser than the approximation;
// FP32 and TF32 outputs keep gelu_erf. Since x * erf(x / sqrt 2) = |x| * erf(|x| / sqrt 2),
//   GELU(x) = max(x, 0) - |x|/2 * erfc(|x| / sqrt 2),  erfc(z) ~= t * P(t) * exp(-z^2),
// which needs no sign handling and never forms 1 - erf (whose cancellation cost up to 15%
// relative error where |GELU| ~ 1e-6): relative error <= 1.7e-3 wherever |GELU| >= 1e-6.
__device__ __forceinline__ float gelu_bf16_output(float x) {
    const float magnitude = fabsf(x);
    const float t = rcp_approx(fmaf(0.3275911F * 0.7071067811865475F, magnitude, 1.0F));
    float poly = fmaf(t, 1.061405429F, -1.453152027F);
    poly = fmaf(t, poly, 1.421413741F);
    poly = fmaf(t, poly, -0.284496736F);
    poly = fmaf(t, poly, 0.254829592F);
    poly *= 0.5F * magnitude * t;
    const float tail = ex2_approx(x * (x * (-0.5F * 1.4426950408889634F)));
    return fmaf(-poly, tail, fmaxf(x, 0.0F));
}

// gelu_bf16_output on two values: the same operations in the same order, with the
// polynomial's coefficients scaled by -1/2 (exact) so its sign and halving need no separate
// steps -- the same results as two scalar calls, the multiply-adds two per instruction.
__device__ __forceinline__ float2 gelu_bf16_output2(float x0, float x1) {
    const float m0 = fabsf(x0);
    const float m1 = fabsf(x1);
    const uint64_t m = f32x2(m0, m1);
    const float2 den = f32x2_split(fma_f32x2(
        f32x2(0.3275911F * 0.7071067811865475F, 0.3275911F * 0.7071067811865475F), m,
        f32x2(1.0F, 1.0F)));
    const uint64_t t = f32x2(rcp_approx(den.x), rcp_approx(den.y));
    uint64_t poly = fma_f32x2(t, f32x2(-0.5F * 1.061405429F, -0.5F * 1.061405429F),
                              f32x2(0.5F * 1.453152027F, 0.5F * 1.453152027F));
    poly = fma_f32x2(t, poly, f32x2(-0.5F * 1.421413741F, -0.5F * 1.421413741F));
    poly = fma_f32x2(t, poly, f32x2(0.5F * 0.284496736F, 0.5F * 0.284496736F));
    poly = fma_f32x2(t, poly, f32x2(-0.5F * 0.254829592F, -0.5F * 0.254829592F));
    poly = mul_f32x2(poly, mul_f32x2(m, t));
    const uint64_t x = f32x2(x0, x1);
    constexpr float kHalfLog2e = -0.5F * 1.4426950408889634F;
    const float2 arg = f32x2_split(mul_f32x2(x, mul_f32x2(x, f32x2(kHalfLog2e, kHalfLog2e))));
    const uint64_t tail = f32x2(ex2_approx(arg.x), ex2_approx(arg.y));
    return f32x2_split(fma_f32x2(poly, tail, f32x2(fmaxf(x0, 0.0F), fmaxf(x1, 0.0F))));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float low, float high) {
    const __nv_bfloat162 pair = __floats2bfloat162_rn(low, high);
    return *reinterpret_cast<const uint32_t*>(&pair);
}

} // namespace cuvit::dev
