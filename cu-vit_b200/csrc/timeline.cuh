// Per-launch device timeline, compiled in only with -DCUVIT_TIMELINE (the instrumented
// library variant, `python cu-vit_b200/build.py --timeline`). Each instrumented kernel stamps
// %globaltimer when its first CTA starts and when its last CTA finishes, into a table keyed
// by the launch's %gridid (one id per launch, or per node of a CUDA graph), plus CTA 0's
// %clock64 at entry and exit so the SM clock each kernel ran at can be read back (cycles /
// nanoseconds). Only thread 0 of a CTA stamps, and only CTAs that can be first (the first
// kTimelineEdge of the grid) or last (the last kTimelineEdge) to run: a stamp from every warp
// of every CTA serialised on one address and tripled the time of the LayerNorm launches. In
// the default build the hooks compile to nothing.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

namespace cuvit::dev {

struct TimelineRecord {
    unsigned long long grid;     // %gridid of the launch; 0 marks a free slot
    unsigned long long first_ns; // earliest CTA entry
    unsigned long long last_ns;  // latest CTA exit
    unsigned long long warps;    // CTAs that stamped their exit
    unsigned long long cta0_ns[2];
    unsigned long long cta0_clock[2];
};

// Hash-table slots; a ViT pass issues at most a few hundred launches.
constexpr int kTimelineSlots = 2048;
// CTAs at each end of a grid that stamp (more than one wave of 148 SMs at 8 CTAs each).
constexpr unsigned kTimelineEdge = 2048;

#ifdef CUVIT_TIMELINE
// One table pointer per translation unit (device symbols do not link across units without
// relocatable device code); runtime.cu binds every unit's pointer to the same table.
static __device__ TimelineRecord* g_timeline_records = nullptr;

__device__ __forceinline__ int timeline_slot(TimelineRecord* records) {
    unsigned long long grid;
    asm volatile("mov.u64 %0, %%gridid;" : "=l"(grid));
    grid += 1; // keep 0 free as the empty mark
    const unsigned start = static_cast<unsigned>((grid * 0x9E3779B97F4A7C15ull) >> 53);
    for (int probe = 0; probe < kTimelineSlots; ++probe) {
        const int slot = static_cast<int>((start + probe) & (kTimelineSlots - 1));
        const unsigned long long seen = atomicCAS(&records[slot].grid, 0ull, grid);
        if (seen == 0ull || seen == grid) {
            return slot;
        }
    }
    return -1;
}

__device__ __forceinline__ unsigned long long timeline_ns() {
    unsigned long long value;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(value));
    return value;
}

__device__ __forceinline__ unsigned timeline_block() {
    return blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
}

__device__ __forceinline__ unsigned timeline_blocks() {
    return gridDim.x * gridDim.y * gridDim.z;
}
#endif

// At kernel entry, before anything else.
__device__ __forceinline__ void timeline_enter() {
#ifdef CUVIT_TIMELINE
    TimelineRecord* const records = g_timeline_records;
    if (records != nullptr && threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0 &&
        timeline_block() < kTimelineEdge) {
        const unsigned long long now = timeline_ns();
        const long long clock = clock64();
        const int slot = timeline_slot(records);
        if (slot >= 0) {
            atomicMin(&records[slot].first_ns, now);
            if (timeline_block() == 0) {
                records[slot].cta0_ns[0] = now;
                records[slot].cta0_clock[0] = static_cast<unsigned long long>(clock);
            }
        }
    }
#endif
}

// At the end of the kernel body. Thread 0 of every CTA reaches it in the instrumented kernels
// (their warp 0 never leaves early), and a CTA's warps end together.
__device__ __forceinline__ void timeline_exit() {
#ifdef CUVIT_TIMELINE
    TimelineRecord* const records = g_timeline_records;
    const unsigned block = timeline_block();
    const unsigned blocks = timeline_blocks();
    if (records != nullptr && threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0 &&
        (block == 0 || block + kTimelineEdge >= blocks)) {
        const long long clock = clock64();
        const unsigned long long now = timeline_ns();
        const int slot = timeline_slot(records);
        if (slot >= 0) {
            atomicMax(&records[slot].last_ns, now);
            atomicAdd(&records[slot].warps, 1ull);
            if (block == 0) {
                records[slot].cta0_ns[1] = now;
                records[slot].cta0_clock[1] = static_cast<unsigned long long>(clock);
            }
        }
    }
#endif
}

} // namespace cuvit::dev

#ifdef CUVIT_TIMELINE
namespace cuvit::host {
// Defined in runtime.cu: every translation unit registers how to point its table at `records`.
void register_timeline_binder(int (*bind)(void* records));
namespace {
int bind_timeline_records(void* records) {
    auto* const typed = static_cast<cuvit::dev::TimelineRecord*>(records);
    return cudaMemcpyToSymbol(cuvit::dev::g_timeline_records, &typed, sizeof(typed)) ==
                   cudaSuccess
               ? 0
               : -1;
}
struct TimelineRegistration {
    TimelineRegistration() { register_timeline_binder(&bind_timeline_records); }
};
const TimelineRegistration g_timeline_registration;
} // namespace
} // namespace cuvit::host
#endif
