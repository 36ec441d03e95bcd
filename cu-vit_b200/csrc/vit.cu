// The model runner: the B200 counterpart of cuvit::VisionTransformer
// (include/cuvit/vit.hpp:63-120, src/model/vit.cu:69-344). Weights are uploaded once into
// one arena (GEMM weights converted to bfloat16 for the BF16 path), activations live in a
// second arena sized for max_batch, and a forward pass is a fixed sequence of this
// library's kernels on one stream -- optionally replayed as a CUDA graph.
//
// Per block (compare src/model/vit.cu:173-261):
//   LN1 -> QKV GEMM (+bias) -> attention -> proj GEMM (+bias, accumulate into tokens)
//   LN2 -> FC1 GEMM (+bias, GELU) -> FC2 GEMM (+bias, accumulate into tokens)
// Attention is the fused kernel for TF32/BF16 and, for the FP32-faithful path, the
// reference's own three steps (scaled Q.K^T GEMM, row softmax, P.V GEMM) on 3xTF32 GEMMs.
// The residual stream (tokens) is FP32 in every precision.
#include "cuvit_b200.h"
#include "elementwise.hpp"
#include "gemm.hpp"
#include "runtime.hpp"

#include <cuda_runtime.h>
#include <sched.h>

#include <algorithm>
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <unordered_map>
#include <vector>

using cuvit::host::fail;

namespace cuvit::model {
namespace {

struct TensorSpec {
    std::string name;
    std::vector<int64_t> extents;
    bool gemm_weight = false; // stored in the compute type
};

std::vector<TensorSpec> tensor_specs(const cuvit_vit_config& c) {
    const int64_t e = c.embed_dim;
    const int64_t side = c.image_size / c.patch_size;
    const int64_t tokens = side * side + 1;
    const int64_t f = c.mlp_hidden;
    std::vector<TensorSpec> specs = {
        {"cls_token", {1, 1, e}, false},
        {"pos_embed", {1, tokens, e}, false},
        {"patch_embed.proj.weight", {e, c.channels, c.patch_size, c.patch_size}, true},
        {"patch_embed.proj.bias", {e}, false},
    };
    for (int i = 0; i < c.depth; ++i) {
        const std::string prefix = "blocks." + std::to_string(i) + ".";
        specs.push_back({prefix + "norm1.weight", {e}, false});
        specs.push_back({prefix + "norm1.bias", {e}, false});
        specs.push_back({prefix + "attn.qkv.weight", {3 * e, e}, true});
        specs.push_back({prefix + "attn.qkv.bias", {3 * e}, false});
        specs.push_back({prefix + "attn.proj.weight", {e, e}, true});
        specs.push_back({prefix + "attn.proj.bias", {e}, false});
        specs.push_back({prefix + "norm2.weight", {e}, false});
        specs.push_back({prefix + "norm2.bias", {e}, false});
        specs.push_back({prefix + "mlp.fc1.weight", {f, e}, true});
        specs.push_back({prefix + "mlp.fc1.bias", {f}, false});
        specs.push_back({prefix + "mlp.fc2.weight", {e, f}, true});
        specs.push_back({prefix + "mlp.fc2.bias", {e}, false});
    }
    specs.push_back({"norm.weight", {e}, false});
    specs.push_back({"norm.bias", {e}, false});
    // The head's weights stay in float storage in every precision (see run_forward).
    specs.push_back({"head.weight", {c.classes, e}, false});
    specs.push_back({"head.bias", {c.classes}, false});
    return specs;
}

int64_t element_count(const std::vector<int64_t>& extents) {
    int64_t count = 1;
    for (const int64_t extent : extents) {
        count *= extent;
    }
    return count;
}

std::string shape_string(const std::vector<int64_t>& extents) {
    std::string text = "[";
    for (size_t i = 0; i < extents.size(); ++i) {
        text += (i ? ", " : "") + std::to_string(extents[i]);
    }
    return text + "]";
}

constexpr size_t kArenaAlignment = 256;

size_t align_up(size_t bytes) { return (bytes + kArenaAlignment - 1) / kArenaAlignment * kArenaAlignment; }

// A fixed set of host threads that split one job: run(job) calls job(part, parts) once per part
// (the calling thread takes part 0) and returns when every part is done.
class HostPool {
  public:
    explicit HostPool(int threads) : parts_(threads < 1 ? 1 : threads) {
        for (int i = 1; i < parts_; ++i) {
            workers_.emplace_back([this, i] { work(i); });
        }
    }
    ~HostPool() {
        {
            std::lock_guard<std::mutex> lock(mutex_);
            stop_ = true;
        }
        start_.notify_all();
        for (std::thread& worker : workers_) {
            worker.join();
        }
    }
    HostPool(const HostPool&) = delete;
    HostPool& operator=(const HostPool&) = delete;

    int parts() const { return parts_; }

    void run(const std::function<void(int, int)>& job) {
        {
            std::lock_guard<std::mutex> lock(mutex_);
            job_ = &job;
            pending_ = parts_ - 1;
            ++generation_;
        }
        start_.notify_all();
        job(0, parts_);
        std::unique_lock<std::mutex> lock(mutex_);
        done_.wait(lock, [this] { return pending_ == 0; });
        job_ = nullptr;
    }

  private:
    void work(int part) {
        uint64_t seen = 0;
        for (;;) {
            const std::function<void(int, int)>* job = nullptr;
            {
                std::unique_lock<std::mutex> lock(mutex_);
                start_.wait(lock, [&] { return stop_ || generation_ != seen; });
                if (stop_) {
                    return;
                }
                seen = generation_;
                job = job_;
            }
            (*job)(part, parts_);
            {
                std::lock_guard<std::mutex> lock(mutex_);
                if (--pending_ == 0) {
                    done_.notify_one();
                }
            }
        }
    }

    const int parts_;
    std::vector<std::thread> workers_;
    std::mutex mutex_;
    std::condition_variable start_;
    std::condition_variable done_;
    const std::function<void(int, int)>* job_ = nullptr;
    uint64_t generation_ = 0;
    int pending_ = 0;
    bool stop_ = false;
};

// CPUs this process may run on.
int process_cpus() {
    cpu_set_t set;
    CPU_ZERO(&set);
    if (sched_getaffinity(0, sizeof(set), &set) == 0) {
        return CPU_COUNT(&set);
    }
    return 1;
}

// Host threads for rounding images: the process's CPUs, at most 8 (the conversion is bound
// by host memory bandwidth well before that).
int host_threads() { return std::clamp(process_cpus(), 1, 8); }

// Whether forward_host_async rounds images to bfloat16 on the host: only with
// CUVIT_HOST_ROUNDING=1. It halves the bytes that cross PCIe but costs ~28 ms of one core per
// 256 ViT images and 1.5x the image bytes in host memory traffic (read 4, write 2, copy 2 per
// pixel, against 4 for copying FP32): on the B200 hosts measured, the FP32 copy already hides
// under the pass (e2e 98% of device-timed at 1, 2 and 8 GPUs) and rounding gained nothing at
// 2 GPUs per host and lost a third of e2e at 8 (8 GPUs sharing 32 CPUs). For PCIe-limited
// hosts with cores to spare.
bool host_rounding_enabled() {
    const char* value = std::getenv("CUVIT_HOST_ROUNDING");
    return value != nullptr && std::strcmp(value, "1") == 0;
}

// count floats -> bfloat16 bit patterns, rounded to nearest even (quiet NaN kept): the
// rounding the BF16 path's patch gather applies to every pixel on the device.
void round_to_bf16(const float* in, uint16_t* out, size_t count) {
    for (size_t i = 0; i < count; ++i) {
        uint32_t u = 0;
        std::memcpy(&u, in + i, sizeof(u));
        const uint32_t rounded = (u + 0x7FFFU + ((u >> 16) & 1U)) >> 16;
        const uint32_t nan = (u >> 16) | 0x40U;
        out[i] = static_cast<uint16_t>((u & 0x7FFFFFFFU) > 0x7F800000U ? nan : rounded);
    }
}

// Restores the caller's current device on scope exit.
class DeviceGuard {
  public:
    explicit DeviceGuard(int device) {
        cudaGetDevice(&previous_);
        if (device != previous_) {
            cudaSetDevice(device);
        }
    }
    ~DeviceGuard() { cudaSetDevice(previous_); }

  private:
    int previous_ = 0;
};

struct BlockWeights {
    const float* norm1_gamma;
    const float* norm1_beta;
    const void* qkv_weight;
    const float* qkv_bias;
    const void* proj_weight;
    const float* proj_bias;
    const float* norm2_gamma;
    const float* norm2_beta;
    const void* fc1_weight;
    const float* fc1_bias;
    const void* fc2_weight;
    const float* fc2_bias;
};

} // namespace
} // namespace cuvit::model

struct cuvit_vit {
    cuvit_vit_config config{};
    int max_batch = 1;
    int precision = CUVIT_MATH_BF16;
    int device = 0;

    void* weight_arena = nullptr;
    size_t weight_used = 0;
    void* activation_arena = nullptr;
    size_t activation_used = 0;

    const float* class_token = nullptr;
    const float* position = nullptr;
    const void* patch_weight = nullptr;
    const float* patch_bias = nullptr;
    std::vector<cuvit::model::BlockWeights> blocks;
    const float* final_gamma = nullptr;
    const float* final_beta = nullptr;
    const void* head_weight = nullptr;
    const float* head_bias = nullptr;

    void* patches = nullptr;
    float* tokens = nullptr;
    void* normalized = nullptr;
    void* qkv = nullptr;
    void* context = nullptr;
    void* hidden = nullptr;
    void* class_rows = nullptr;
    float* scores = nullptr; // FP32 path only: [B*h, T, score_ld]
    int score_ld = 0;
    float* stage_images = nullptr;
    float* stage_images_alt = nullptr; // second image slot of forward_host_async
    float* stage_logits = nullptr;

    cudaStream_t capture_stream = nullptr;
    // (batch, images, logits, images are bfloat16) -> the captured pass
    std::map<std::tuple<int, const void*, float*, bool>, cudaGraphExec_t> graphs;

    // forward_host: images per chunk (0 = automatic), the stream that carries the
    // host-to-device copies, and one event per chunk marking its copy complete.
    int host_chunk = 0;
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t entry_event = nullptr;
    std::vector<cudaEvent_t> chunk_events;

    // forward_host_async: the image slot the next call fills, and per slot the events
    // "its images have landed" and "the pass reading them has finished".
    int async_slot = 0;
    cudaEvent_t slot_loaded[2] = {nullptr, nullptr};
    cudaEvent_t slot_free[2] = {nullptr, nullptr};

    // BF16 path: forward_host_async rounds the host images to bfloat16 on the host (the
    // rounding the device's patch gather would apply) into pinned slots, halving the bytes that
    // cross PCIe; the device slot then holds bfloat16 images.
    bool host_bf16 = false;
    uint16_t* pinned_bf16[2] = {nullptr, nullptr};
    std::unique_ptr<cuvit::model::HostPool> pool;
};

namespace cuvit::model {
namespace {

// Storage of the activations a GEMM or the attention consumes next: bfloat16, TF32-rounded
// floats (so the TF32 tensor core sees round-to-nearest operands, not truncated ones), or
// full floats for the FP32-faithful path.
int compute_dtype(const cuvit_vit& m) {
    switch (m.precision) {
    case CUVIT_MATH_BF16:
        return CUVIT_DTYPE_BF16;
    case CUVIT_MATH_TF32:
        return CUVIT_DTYPE_TF32;
    default:
        return CUVIT_DTYPE_F32;
    }
}

int element_bytes(const cuvit_vit& m) { return m.precision == CUVIT_MATH_BF16 ? 2 : 4; }

int gemm(const cuvit_vit& m, const void* a, const void* b, const float* bias, void* c, int c_dtype,
         const cuvit_gemm_problem& problem, cudaStream_t stream) {
    return cuvit_gemm_ex(a, b, bias, c, c_dtype, m.precision, &problem,
                         reinterpret_cast<cuvit_stream_t>(stream));
}

// Optional per-launch timing: an event pair around each launch plus its algorithmic cost.
class Recorder {
  public:
    explicit Recorder(cudaStream_t stream) : stream_(stream) {}
    Recorder(const Recorder&) = delete;
    Recorder& operator=(const Recorder&) = delete;
    ~Recorder() {
        for (auto& pair : events_) {
            cudaEventDestroy(pair.first);
            cudaEventDestroy(pair.second);
        }
    }

    int begin(int kind, int layer, double flops, double bytes) {
        cudaEvent_t start = nullptr;
        cudaEvent_t stop = nullptr;
        CUVIT_TRY_CUDA(cudaEventCreate(&start));
        CUVIT_TRY_CUDA(cudaEventCreate(&stop));
        events_.emplace_back(start, stop);
        cuvit_launch_record record{};
        record.kind = kind;
        record.layer = layer;
        record.flops = flops;
        record.bytes = bytes;
        records_.push_back(record);
        CUVIT_TRY_CUDA(cudaEventRecord(start, stream_));
        return CUVIT_OK;
    }

    int end() {
        CUVIT_TRY_CUDA(cudaEventRecord(events_.back().second, stream_));
        return CUVIT_OK;
    }

    int finish(cuvit_launch_record* out, int capacity, int* count) {
        CUVIT_TRY_CUDA(cudaStreamSynchronize(stream_));
        for (size_t i = 0; i < records_.size(); ++i) {
            CUVIT_TRY_CUDA(cudaEventElapsedTime(&records_[i].milliseconds, events_[i].first,
                                                events_[i].second));
            if (out != nullptr && static_cast<int>(i) < capacity) {
                out[i] = records_[i];
            }
        }
        *count = static_cast<int>(records_.size());
        return CUVIT_OK;
    }

  private:
    cudaStream_t stream_;
    std::vector<cuvit_launch_record> records_;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> events_;
};

// Runs one launch, bracketed by the recorder's events when one is attached. Consecutive
// launches sweep their tiles / rows / pairs in alternating order (`reverse` flips after each),
// so every kernel starts on what the previous one wrote last, still in L2 (a pass reads or
// writes 0.1-0.3 GB per kernel at batch 256, more than the 126 MB L2).
#define CUVIT_LAUNCH(kind, layer, flops, bytes, expression)                                        \
    do {                                                                                           \
        if (recorder != nullptr) {                                                                 \
            CUVIT_TRY(recorder->begin((kind), (layer), (flops), (bytes)));                         \
        }                                                                                          \
        {                                                                                          \
            const cuvit::host::ReverseSweep sweep_order(reverse);                                  \
            CUVIT_TRY(expression);                                                                 \
        }                                                                                          \
        reverse = !reverse;                                                                        \
        if (recorder != nullptr) {                                                                 \
            CUVIT_TRY(recorder->end());                                                            \
        }                                                                                          \
    } while (0)

int run_block(cuvit_vit& m, const BlockWeights& w, int layer, int batch, cudaStream_t stream,
              Recorder* recorder, bool& reverse) {
    const cuvit_vit_config& c = m.config;
    const int side = c.image_size / c.patch_size;
    const int tokens = side * side + 1;
    const int e = c.embed_dim;
    const int heads = c.heads;
    const int head_dim = e / heads;
    const int f = c.mlp_hidden;
    const int rows = batch * tokens;
    const int dtype = compute_dtype(m);
    const double es = element_bytes(m);
    const double r = rows;
    const cuvit_stream_t s = reinterpret_cast<cuvit_stream_t>(stream);

    CUVIT_LAUNCH(CUVIT_KIND_LAYER_NORM, layer, 0.0, r * e * (4 + es) + 8.0 * e,
                 cuvit_layer_norm_ex(m.tokens, e, w.norm1_gamma, w.norm1_beta, m.normalized,
                                     dtype, e, rows, e, c.layer_norm_epsilon, s));
    cuvit_gemm_problem qkv;
    cuvit_gemm_problem_init(&qkv, rows, 3 * e, e, CUVIT_LAYOUT_TRANSPOSED);
    CUVIT_LAUNCH(CUVIT_KIND_GEMM_QKV, layer, 2.0 * r * 3 * e * e,
                 r * e * es + 3.0 * e * e * es + 12.0 * e + r * 3 * e * es,
                 gemm(m, m.normalized, w.qkv_weight, w.qkv_bias, m.qkv, dtype, qkv, stream));

    const float scale = 1.0F / std::sqrt(static_cast<float>(head_dim));
    const double attention_flops = 4.0 * batch * heads * double(tokens) * tokens * head_dim;
    if (m.precision == CUVIT_MATH_FP32) {
        // The reference's attention steps (src/model/vit.cu:205-242), FP32-faithful.
        const int64_t qkv_per_image = static_cast<int64_t>(tokens) * 3 * e;
        const int64_t per_head = static_cast<int64_t>(tokens) * m.score_ld;
        const double scores = double(batch) * heads * tokens * tokens * 4.0;
        const float* const q = static_cast<const float*>(m.qkv);
        cuvit_gemm_problem logits;
        cuvit_gemm_problem_init(&logits, tokens, tokens, head_dim, CUVIT_LAYOUT_TRANSPOSED);
        logits.alpha = scale;
        logits.lda = 3 * e;
        logits.ldb = 3 * e;
        logits.ldc = m.score_ld;
        logits.batch.count = batch * heads;
        logits.batch.inner = heads;
        logits.batch.stride_a = head_dim;
        logits.batch.stride_b = head_dim;
        logits.batch.stride_c = per_head;
        logits.batch.outer_stride_a = qkv_per_image;
        logits.batch.outer_stride_b = qkv_per_image;
        logits.batch.outer_stride_c = heads * per_head;
        CUVIT_LAUNCH(CUVIT_KIND_ATTENTION, layer, attention_flops / 2, 2.0 * r * e * 4 + scores,
                     gemm(m, q, q + e, nullptr, m.scores, CUVIT_DTYPE_F32, logits, stream));
        CUVIT_LAUNCH(CUVIT_KIND_ATTENTION, layer, 0.0, 2.0 * scores,
                     cuvit_softmax_ex(m.scores, m.scores, batch * heads * tokens, tokens,
                                      m.score_ld, s));
        cuvit_gemm_problem context;
        cuvit_gemm_problem_init(&context, tokens, head_dim, tokens, CUVIT_LAYOUT_NO_TRANSPOSE);
        context.lda = m.score_ld;
        context.ldb = 3 * e;
        context.ldc = e;
        context.batch.count = batch * heads;
        context.batch.inner = heads;
        context.batch.stride_a = per_head;
        context.batch.stride_b = head_dim;
        context.batch.stride_c = head_dim;
        context.batch.outer_stride_a = heads * per_head;
        context.batch.outer_stride_b = qkv_per_image;
        context.batch.outer_stride_c = static_cast<int64_t>(tokens) * e;
        CUVIT_LAUNCH(CUVIT_KIND_ATTENTION, layer, attention_flops / 2, scores + 2.0 * r * e * 4,
                     gemm(m, m.scores, q + 2 * e, nullptr, m.context, CUVIT_DTYPE_F32, context,
                          stream));
    } else {
        CUVIT_LAUNCH(CUVIT_KIND_ATTENTION, layer, attention_flops, r * 3 * e * es + r * e * es,
                     cuvit_attention(m.qkv, m.context, dtype, batch, tokens, heads, head_dim,
                                     scale, s));
    }

    cuvit_gemm_problem projection;
    cuvit_gemm_problem_init(&projection, rows, e, e, CUVIT_LAYOUT_TRANSPOSED);
    projection.epilogue.accumulate = 1;
    CUVIT_LAUNCH(CUVIT_KIND_GEMM_PROJ, layer, 2.0 * r * e * e,
                 r * e * es + double(e) * e * es + 4.0 * e + 8.0 * r * e,
                 gemm(m, m.context, w.proj_weight, w.proj_bias, m.tokens, CUVIT_DTYPE_F32,
                      projection, stream));

    CUVIT_LAUNCH(CUVIT_KIND_LAYER_NORM, layer, 0.0, r * e * (4 + es) + 8.0 * e,
                 cuvit_layer_norm_ex(m.tokens, e, w.norm2_gamma, w.norm2_beta, m.normalized,
                                     dtype, e, rows, e, c.layer_norm_epsilon, s));
    cuvit_gemm_problem first;
    cuvit_gemm_problem_init(&first, rows, f, e, CUVIT_LAYOUT_TRANSPOSED);
    first.epilogue.gelu = 1;
    CUVIT_LAUNCH(CUVIT_KIND_GEMM_FC1, layer, 2.0 * r * f * e,
                 r * e * es + double(f) * e * es + 4.0 * f + r * f * es,
                 gemm(m, m.normalized, w.fc1_weight, w.fc1_bias, m.hidden, dtype, first, stream));
    cuvit_gemm_problem second;
    cuvit_gemm_problem_init(&second, rows, e, f, CUVIT_LAYOUT_TRANSPOSED);
    second.epilogue.accumulate = 1;
    CUVIT_LAUNCH(CUVIT_KIND_GEMM_FC2, layer, 2.0 * r * e * f,
                 r * f * es + double(e) * f * es + 4.0 * e + 8.0 * r * e,
                 gemm(m, m.hidden, w.fc2_weight, w.fc2_bias, m.tokens, CUVIT_DTYPE_F32, second,
                      stream));
    return CUVIT_OK;
}

// Passes below this many GEMM FLOPs launch their kernels with programmatic dependent launch.
constexpr double kDependentLaunchMaxFlops = 2.0e12;

// images: planar FP32 images, or (bf16_images) the same rounded to bfloat16 by the host.
int run_forward(cuvit_vit& m, const void* images, float* logits, int batch, cudaStream_t stream,
                Recorder* recorder = nullptr, bool bf16_images = false) {
    const cuvit_vit_config& c = m.config;
    const int side = c.image_size / c.patch_size;
    const int patch_count = side * side;
    const int tokens = patch_count + 1;
    const int e = c.embed_dim;
    const int patch_elements = c.channels * c.patch_size * c.patch_size;
    const int dtype = compute_dtype(m);
    const double es = element_bytes(m);
    const double b = batch;
    const cuvit_stream_t s = reinterpret_cast<cuvit_stream_t>(stream);
    bool reverse = false;
    // Small passes launch each kernel as a dependent of the previous one (its prologue
    // overlaps the previous tail); large ones do not, since on the power-capped B200 the
    // overlap costs clock (runtime.hpp, pdl_enabled). The measure is the pass's GEMM work:
    // ViT-Ti/16 at batch 32 is 0.07 TFLOP, ViT-S/16 at 128 1.2, ViT-B/16 at 256 9.
    const double per_layer =
        2.0 * tokens * (double(e) * 3 * e + double(e) * e + 2.0 * double(e) * c.mlp_hidden);
    const double pass_flops =
        b * (2.0 * patch_count * double(patch_elements) * e + c.depth * per_layer +
             2.0 * double(e) * c.classes);
    const cuvit::host::DependentLaunch overlap(pass_flops < kDependentLaunchMaxFlops);

    if (bf16_images) {
        CUVIT_LAUNCH(CUVIT_KIND_PATCHES, -1, 0.0, b * patch_count * patch_elements * (2 + es),
                     cuvit::ops::extract_patches_bf16(
                         static_cast<const __nv_bfloat16*>(images),
                         static_cast<__nv_bfloat16*>(m.patches), batch, c.channels,
                         c.image_size, c.image_size, c.patch_size, stream));
    } else {
        CUVIT_LAUNCH(CUVIT_KIND_PATCHES, -1, 0.0, b * patch_count * patch_elements * (4 + es),
                     cuvit_extract_patches_ex(static_cast<const float*>(images), m.patches,
                                              dtype, batch, c.channels, c.image_size,
                                              c.image_size, c.patch_size, s));
    }
    // Class token + positional embedding first; the patch-embedding GEMM then accumulates
    // into rows 1..T-1 (the reference writes the GEMM first and adds after, vit.cu:290-300;
    // each element sees the same two roundings).
    CUVIT_LAUNCH(CUVIT_KIND_TOKENS, -1, 0.0, b * tokens * e * 4 + 4.0 * (tokens + 1) * e,
                 cuvit_init_tokens(m.tokens, m.class_token, m.position, batch, tokens, e, s));
    cuvit_gemm_problem embedding;
    cuvit_gemm_problem_init(&embedding, patch_count, e, patch_elements, CUVIT_LAYOUT_TRANSPOSED);
    embedding.batch.count = batch;
    embedding.batch.stride_a = static_cast<int64_t>(patch_count) * patch_elements;
    embedding.batch.stride_c = static_cast<int64_t>(tokens) * e;
    embedding.epilogue.accumulate = 1;
    CUVIT_LAUNCH(CUVIT_KIND_GEMM_PATCH, -1, 2.0 * b * patch_count * e * patch_elements,
                 b * patch_count * patch_elements * es + double(e) * patch_elements * es +
                     4.0 * e + 8.0 * b * patch_count * e,
                 gemm(m, m.patches, m.patch_weight, m.patch_bias, m.tokens + e, CUVIT_DTYPE_F32,
                      embedding, stream));

    for (size_t i = 0; i < m.blocks.size(); ++i) {
        CUVIT_TRY(
            run_block(m, m.blocks[i], static_cast<int>(i), batch, stream, recorder, reverse));
    }

    // Only the class token feeds the head (src/model/vit.cu:309-316), so only those rows
    // are normalised. The final norm's output and the head's weights stay in float storage
    // and the head runs with TF32 operands rounded to nearest (FP32-faithful in the FP32
    // model): in a BF16 head the bfloat16 roundings of those two added 1.2e-3 RMS straight
    // onto the ViT-B/16 logits, a third of the BF16 path's whole logit error, where the TF32
    // head adds an eighth of that for 0.4 of the 9 TFLOP of a pass at batch 256.
    const int head_math = m.precision == CUVIT_MATH_FP32 ? CUVIT_MATH_FP32 : CUVIT_MATH_TF32;
    const int head_dtype = m.precision == CUVIT_MATH_FP32 ? CUVIT_DTYPE_F32 : CUVIT_DTYPE_TF32;
    CUVIT_LAUNCH(CUVIT_KIND_LAYER_NORM, -1, 0.0, b * e * 8.0 + 8.0 * e,
                 cuvit_layer_norm_ex(m.tokens, static_cast<int64_t>(tokens) * e, m.final_gamma,
                                     m.final_beta, m.class_rows, head_dtype, e, batch, e,
                                     c.layer_norm_epsilon, s));
    cuvit_gemm_problem head;
    cuvit_gemm_problem_init(&head, batch, c.classes, e, CUVIT_LAYOUT_TRANSPOSED);
    CUVIT_LAUNCH(CUVIT_KIND_GEMM_HEAD, -1, 2.0 * b * c.classes * e,
                 b * e * 4.0 + double(c.classes) * e * 4.0 + 4.0 * c.classes + 4.0 * b * c.classes,
                 cuvit_gemm_ex(m.class_rows, m.head_weight, m.head_bias, logits, CUVIT_DTYPE_F32,
                               head_math, &head, s));
    return CUVIT_OK;
}

int check_forward_args(const cuvit_vit* m, const float* images, const float* logits, int batch) {
    if (m == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "model cannot be null");
    }
    if (batch < 0 || batch > m->max_batch) {
        return fail(CUVIT_INVALID_ARGUMENT,
                    "This model was built for at most " + std::to_string(m->max_batch) +
                        " images, but " + std::to_string(batch) + " were given");
    }
    if (batch > 0 && (images == nullptr || logits == nullptr)) {
        return fail(CUVIT_INVALID_ARGUMENT, "Forward pass operands cannot be null");
    }
    return CUVIT_OK;
}

// Builds the model on the current device from FP32 host tensors in load order.
int build(cuvit_vit* m, const float* const* host) {
    const cuvit_vit_config& c = m->config;
    const std::vector<TensorSpec> specs = tensor_specs(c);
    const int ebytes = element_bytes(*m);

    size_t weight_size = 0;
    int64_t largest = 0;
    for (const TensorSpec& spec : specs) {
        const int64_t count = element_count(spec.extents);
        weight_size += align_up(static_cast<size_t>(count) * (spec.gemm_weight ? ebytes : 4));
        largest = count > largest ? count : largest;
    }
    CUVIT_TRY_CUDA(cudaMalloc(&m->weight_arena, weight_size));
    float* staging = nullptr;
    if (ebytes == 2) {
        CUVIT_TRY_CUDA(cudaMalloc(&staging, static_cast<size_t>(largest) * sizeof(float)));
    }
    std::vector<void*> placed(specs.size());
    size_t cursor = 0;
    int status = CUVIT_OK;
    for (size_t i = 0; i < specs.size() && status == CUVIT_OK; ++i) {
        const TensorSpec& spec = specs[i];
        const int64_t count = element_count(spec.extents);
        void* const target = static_cast<uint8_t*>(m->weight_arena) + cursor;
        const bool convert = spec.gemm_weight && ebytes == 2;
        cursor += align_up(static_cast<size_t>(count) * (spec.gemm_weight ? ebytes : 4));
        placed[i] = target;
        if (host[i] == nullptr) {
            status = fail(CUVIT_INVALID_ARGUMENT, "Tensor '" + spec.name + "' is null");
            break;
        }
        if (convert) {
            status = host::check_cuda(cudaMemcpy(staging, host[i], count * sizeof(float),
                                                 cudaMemcpyHostToDevice),
                                      "cudaMemcpy(weights)");
            if (status == CUVIT_OK) {
                status = cuvit_convert_f32_to_bf16(staging, target, count, nullptr);
            }
            if (status == CUVIT_OK) {
                status = host::check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
            }
        } else {
            status = host::check_cuda(
                cudaMemcpy(target, host[i], count * sizeof(float), cudaMemcpyHostToDevice),
                "cudaMemcpy(weights)");
            const bool tf32_operand =
                (spec.gemm_weight && m->precision == CUVIT_MATH_TF32) ||
                (spec.name == "head.weight" && m->precision != CUVIT_MATH_FP32);
            if (status == CUVIT_OK && tf32_operand) {
                // TF32 operands are rounded to nearest once here; the tensor core would
                // otherwise truncate them on every use.
                float* const values = static_cast<float*>(target);
                status = cuvit_round_to_tf32(values, values, count, nullptr);
                if (status == CUVIT_OK) {
                    status = host::check_cuda(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
                }
            }
        }
    }
    if (staging != nullptr) {
        cudaFree(staging);
    }
    CUVIT_TRY(status);
    m->weight_used = cursor;

    size_t index = 0;
    const auto next_f = [&]() { return static_cast<const float*>(placed[index++]); };
    const auto next_w = [&]() { return static_cast<const void*>(placed[index++]); };
    m->class_token = next_f();
    m->position = next_f();
    m->patch_weight = next_w();
    m->patch_bias = next_f();
    m->blocks.resize(static_cast<size_t>(c.depth));
    for (BlockWeights& b : m->blocks) {
        b.norm1_gamma = next_f();
        b.norm1_beta = next_f();
        b.qkv_weight = next_w();
        b.qkv_bias = next_f();
        b.proj_weight = next_w();
        b.proj_bias = next_f();
        b.norm2_gamma = next_f();
        b.norm2_beta = next_f();
        b.fc1_weight = next_w();
        b.fc1_bias = next_f();
        b.fc2_weight = next_w();
        b.fc2_bias = next_f();
    }
    m->final_gamma = next_f();
    m->final_beta = next_f();
    m->head_weight = next_w();
    m->head_bias = next_f();

    // Activations for max_batch images; every buffer is reused by every block, so depth
    // costs no activation memory (compare src/model/vit.cu:145-170).
    const int64_t images = m->max_batch;
    const int side = c.image_size / c.patch_size;
    const int64_t patches = static_cast<int64_t>(side) * side;
    const int64_t tokens = patches + 1;
    const int64_t e = c.embed_dim;
    const int64_t patch_elements = static_cast<int64_t>(c.channels) * c.patch_size * c.patch_size;
    m->score_ld = static_cast<int>((tokens + 3) / 4 * 4);
    struct Piece {
        void** slot;
        size_t bytes;
    };
    std::vector<Piece> pieces = {
        {&m->patches, static_cast<size_t>(images * patches * patch_elements * ebytes)},
        {reinterpret_cast<void**>(&m->tokens), static_cast<size_t>(images * tokens * e * 4)},
        {&m->normalized, static_cast<size_t>(images * tokens * e * ebytes)},
        {&m->qkv, static_cast<size_t>(images * tokens * 3 * e * ebytes)},
        {&m->context, static_cast<size_t>(images * tokens * e * ebytes)},
        {&m->hidden, static_cast<size_t>(images * tokens * c.mlp_hidden * ebytes)},
        {&m->class_rows, static_cast<size_t>(images * e * 4)},
        {reinterpret_cast<void**>(&m->stage_images),
         static_cast<size_t>(images * c.channels * c.image_size * c.image_size * 4)},
        {reinterpret_cast<void**>(&m->stage_images_alt),
         static_cast<size_t>(images * c.channels * c.image_size * c.image_size * 4)},
        {reinterpret_cast<void**>(&m->stage_logits), static_cast<size_t>(images * c.classes * 4)},
    };
    if (m->precision == CUVIT_MATH_FP32) {
        pieces.push_back({reinterpret_cast<void**>(&m->scores),
                          static_cast<size_t>(images * c.heads * tokens * m->score_ld * 4)});
    }
    size_t activation_size = 0;
    for (const Piece& piece : pieces) {
        activation_size += align_up(piece.bytes);
    }
    CUVIT_TRY_CUDA(cudaMalloc(&m->activation_arena, activation_size));
    size_t offset = 0;
    for (const Piece& piece : pieces) {
        *piece.slot = static_cast<uint8_t*>(m->activation_arena) + offset;
        offset += align_up(piece.bytes);
    }
    m->activation_used = activation_size;
    CUVIT_TRY_CUDA(cudaStreamCreateWithFlags(&m->capture_stream, cudaStreamNonBlocking));
    CUVIT_TRY_CUDA(cudaStreamCreateWithFlags(&m->copy_stream, cudaStreamNonBlocking));
    CUVIT_TRY_CUDA(cudaEventCreateWithFlags(&m->entry_event, cudaEventDisableTiming));
    for (int slot = 0; slot < 2; ++slot) {
        CUVIT_TRY_CUDA(cudaEventCreateWithFlags(&m->slot_loaded[slot], cudaEventDisableTiming));
        CUVIT_TRY_CUDA(cudaEventCreateWithFlags(&m->slot_free[slot], cudaEventDisableTiming));
    }
    m->host_bf16 = m->precision == CUVIT_MATH_BF16 && host_rounding_enabled() &&
                   cuvit::ops::bf16_patch_gather_supported(c.image_size, c.image_size,
                                                           c.patch_size);
    if (m->host_bf16) {
        const size_t pinned_bytes = static_cast<size_t>(images) * c.channels * c.image_size *
                                    c.image_size * sizeof(uint16_t);
        for (int slot = 0; slot < 2; ++slot) {
            CUVIT_TRY_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&m->pinned_bf16[slot]),
                                         pinned_bytes, cudaHostAllocDefault));
        }
        m->pool = std::make_unique<HostPool>(host_threads());
    }
    return CUVIT_OK;
}

void release(cuvit_vit* m) {
    m->pool.reset();
    for (int slot = 0; slot < 2; ++slot) {
        if (m->pinned_bf16[slot] != nullptr) {
            cudaFreeHost(m->pinned_bf16[slot]);
            m->pinned_bf16[slot] = nullptr;
        }
    }
    for (auto& entry : m->graphs) {
        cudaGraphExecDestroy(entry.second);
    }
    m->graphs.clear();
    for (cudaEvent_t event : m->chunk_events) {
        cudaEventDestroy(event);
    }
    m->chunk_events.clear();
    if (m->entry_event != nullptr) {
        cudaEventDestroy(m->entry_event);
    }
    for (int slot = 0; slot < 2; ++slot) {
        if (m->slot_loaded[slot] != nullptr) {
            cudaEventDestroy(m->slot_loaded[slot]);
        }
        if (m->slot_free[slot] != nullptr) {
            cudaEventDestroy(m->slot_free[slot]);
        }
    }
    if (m->copy_stream != nullptr) {
        cudaStreamDestroy(m->copy_stream);
    }
    if (m->capture_stream != nullptr) {
        cudaStreamDestroy(m->capture_stream);
    }
    if (m->weight_arena != nullptr) {
        cudaFree(m->weight_arena);
    }
    if (m->activation_arena != nullptr) {
        cudaFree(m->activation_arena);
    }
}

// ---- .cvw v1 reader (layout documented at src/runtime/weights.cpp:13-24) ------------------

struct CvwEntry {
    std::vector<int64_t> extents;
    uint64_t offset = 0;
    uint64_t bytes = 0;
};

int read_cvw(const std::string& path, std::vector<uint8_t>* blob,
             std::unordered_map<std::string, CvwEntry>* entries) {
    std::ifstream stream(path, std::ios::binary | std::ios::ate);
    if (!stream) {
        return fail(CUVIT_RUNTIME_ERROR, "Cannot open weight file: " + path);
    }
    const std::streamoff size = stream.tellg();
    if (size < 0) {
        return fail(CUVIT_RUNTIME_ERROR, "Cannot determine the size of weight file: " + path);
    }
    stream.seekg(0, std::ios::beg);
    blob->resize(static_cast<size_t>(size));
    if (!blob->empty() && !stream.read(reinterpret_cast<char*>(blob->data()), size)) {
        return fail(CUVIT_RUNTIME_ERROR, "Cannot read weight file: " + path);
    }
    uint64_t cursor = 0;
    bool truncated = false;
    const auto read_u32 = [&]() -> uint32_t {
        uint32_t value = 0;
        if (cursor + 4 > blob->size()) {
            truncated = true;
            return 0;
        }
        std::memcpy(&value, blob->data() + cursor, 4);
        cursor += 4;
        return value;
    };
    const auto read_u64 = [&]() -> uint64_t {
        uint64_t value = 0;
        if (cursor + 8 > blob->size()) {
            truncated = true;
            return 0;
        }
        std::memcpy(&value, blob->data() + cursor, 8);
        cursor += 8;
        return value;
    };
    const uint32_t magic = read_u32();
    if (truncated) {
        return fail(CUVIT_RUNTIME_ERROR, "Weight file ends inside a header field");
    }
    if (magic != 0x54495643u) {
        return fail(CUVIT_RUNTIME_ERROR, "Not a Cu-Vit weight file: " + path);
    }
    const uint32_t version = read_u32();
    if (!truncated && version != 1) {
        return fail(CUVIT_RUNTIME_ERROR, "Weight file " + path + " has version " +
                                             std::to_string(version) +
                                             ", but this build reads version 1");
    }
    const uint32_t count = read_u32();
    read_u32(); // reserved
    if (truncated) {
        return fail(CUVIT_RUNTIME_ERROR, "Weight file ends inside a header field");
    }
    for (uint32_t i = 0; i < count; ++i) {
        const uint32_t name_length = read_u32();
        if (truncated || cursor + name_length > blob->size()) {
            return fail(CUVIT_RUNTIME_ERROR, "Weight file ends inside a tensor name");
        }
        const std::string name(reinterpret_cast<const char*>(blob->data() + cursor), name_length);
        cursor += name_length;
        const uint32_t type = read_u32();
        if (!truncated && type != 1) {
            return fail(CUVIT_RUNTIME_ERROR, "Tensor '" + name + "' has unsupported data type " +
                                                 std::to_string(type));
        }
        const uint32_t rank = read_u32();
        if (!truncated && (rank == 0 || rank > 4)) {
            return fail(CUVIT_RUNTIME_ERROR, "Tensor '" + name + "' has rank " +
                                                 std::to_string(rank) + ", outside 1..4");
        }
        CvwEntry entry;
        for (uint32_t axis = 0; axis < rank && !truncated; ++axis) {
            const int64_t extent = static_cast<int64_t>(read_u64());
            if (extent < 0) {
                return fail(CUVIT_RUNTIME_ERROR, "Tensor '" + name + "' has a negative extent");
            }
            entry.extents.push_back(extent);
        }
        entry.offset = read_u64();
        entry.bytes = read_u64();
        if (truncated) {
            return fail(CUVIT_RUNTIME_ERROR, "Weight file ends inside a header field");
        }
        const uint64_t expected = static_cast<uint64_t>(element_count(entry.extents)) * 4;
        if (entry.bytes != expected) {
            return fail(CUVIT_RUNTIME_ERROR, "Tensor '" + name + "' declares " +
                                                 std::to_string(entry.bytes) +
                                                 " bytes but its shape " +
                                                 shape_string(entry.extents) + " needs " +
                                                 std::to_string(expected));
        }
        if (entry.offset > blob->size() || entry.bytes > blob->size() - entry.offset) {
            return fail(CUVIT_RUNTIME_ERROR, "Tensor '" + name + "' lies outside the file");
        }
        if (!entries->emplace(name, entry).second) {
            return fail(CUVIT_RUNTIME_ERROR,
                        "Weight file contains two tensors named '" + name + "'");
        }
    }
    return CUVIT_OK;
}

int create(const cuvit_vit_config* config, const float* const* tensors, int max_batch,
           int precision, int device, cuvit_vit** out) {
    if (out == nullptr || config == nullptr || tensors == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "model creation arguments cannot be null");
    }
    *out = nullptr;
    CUVIT_TRY(cuvit_vit_config_validate(config));
    if (max_batch < 1) {
        return fail(CUVIT_INVALID_ARGUMENT, "The maximum batch size must be at least one");
    }
    if (precision != CUVIT_MATH_FP32 && precision != CUVIT_MATH_TF32 &&
        precision != CUVIT_MATH_BF16) {
        return fail(CUVIT_INVALID_ARGUMENT, "unknown model precision");
    }
    if (precision != CUVIT_MATH_FP32 && (config->embed_dim / config->heads != 64 ||
                                         (config->image_size / config->patch_size) *
                                                     (config->image_size / config->patch_size) +
                                                 1 >
                                             256)) {
        return fail(CUVIT_UNSUPPORTED, "the TF32/BF16 paths need head_dim 64 and at most 256 "
                                       "tokens (fused attention)");
    }
    DeviceGuard guard(device);
    auto model = std::make_unique<cuvit_vit>();
    model->config = *config;
    model->max_batch = max_batch;
    model->precision = precision;
    model->device = device;
    const int status = build(model.get(), tensors);
    if (status != CUVIT_OK) {
        release(model.get());
        return status;
    }
    *out = model.release();
    return CUVIT_OK;
}

// The executable graph of one whole pass for (batch, images, logits), captured on first use.
// Work already queued on `stream` uses the same activation buffers, so the eager warm-up
// pass and the capture start only after it.
int graph_for(cuvit_vit& m, const void* images, float* logits, int batch, cudaStream_t stream,
              cudaGraphExec_t* exec, bool bf16_images = false) {
    const auto key = std::make_tuple(batch, images, logits, bf16_images);
    auto found = m.graphs.find(key);
    if (found == m.graphs.end()) {
        CUVIT_TRY_CUDA(cudaEventRecord(m.entry_event, stream));
        CUVIT_TRY_CUDA(cudaStreamWaitEvent(m.capture_stream, m.entry_event, 0));
        // One eager pass first, so every one-time set-up (device context, kernel attributes,
        // the driver's tensor-map entry point) happens outside the capture, where device
        // synchronisation is allowed.
        CUVIT_TRY(run_forward(m, images, logits, batch, m.capture_stream, nullptr, bf16_images));
        CUVIT_TRY_CUDA(cudaStreamSynchronize(m.capture_stream));
        // Capture on the model's own stream: the caller's may be the legacy default stream,
        // which cannot be captured.
        CUVIT_TRY_CUDA(
            cudaStreamBeginCapture(m.capture_stream, cudaStreamCaptureModeThreadLocal));
        const int status =
            run_forward(m, images, logits, batch, m.capture_stream, nullptr, bf16_images);
        cudaGraph_t graph = nullptr;
        const cudaError_t end = cudaStreamEndCapture(m.capture_stream, &graph);
        CUVIT_TRY(status);
        CUVIT_TRY_CUDA(end);
        cudaGraphExec_t made = nullptr;
        const cudaError_t instantiated = cudaGraphInstantiate(&made, graph, 0);
        cudaGraphDestroy(graph);
        CUVIT_TRY_CUDA(instantiated);
        found = m.graphs.emplace(key, made).first;
    }
    *exec = found->second;
    return CUVIT_OK;
}

// Images per forward_host chunk: halves from 64 images up, a single pass below that. The
// second half's copy hides behind the first half's pass; finer chunks expose less copy time
// but cost more in GEMM wave quantization than they save (ViT-B/16, B=256, on B200: halves
// 12.97 ms, quarters 13.76 ms, one pass 13.56 ms).
int host_chunk_images(const cuvit_vit& m, int batch) {
    if (m.host_chunk > 0) {
        return m.host_chunk < batch ? m.host_chunk : batch;
    }
    return batch >= 64 ? (batch + 1) / 2 : batch;
}

} // namespace
} // namespace cuvit::model

using namespace cuvit::model;

extern "C" {

void cuvit_vit_config_default(cuvit_vit_config* config) {
    if (config == nullptr) {
        return;
    }
    config->image_size = 224;
    config->patch_size = 16;
    config->channels = 3;
    config->embed_dim = 192;
    config->depth = 12;
    config->heads = 3;
    config->mlp_hidden = 768;
    config->classes = 1000;
    config->layer_norm_epsilon = 1.0e-6F;
}

int cuvit_vit_config_validate(const cuvit_vit_config* c) {
    if (c == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "config cannot be null");
    }
    if (c->image_size <= 0 || c->patch_size <= 0 || c->channels <= 0 || c->embed_dim <= 0 ||
        c->depth <= 0 || c->heads <= 0 || c->mlp_hidden <= 0 || c->classes <= 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "Every ViT dimension must be positive");
    }
    if (c->image_size % c->patch_size != 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "The image size must divide into whole patches");
    }
    if (c->embed_dim % c->heads != 0) {
        return fail(CUVIT_INVALID_ARGUMENT,
                    "The embedding dimension must divide across the heads");
    }
    return CUVIT_OK;
}

int cuvit_vit_tensor_count(const cuvit_vit_config* config) {
    if (cuvit_vit_config_validate(config) != CUVIT_OK) {
        return -1;
    }
    return 4 + 12 * config->depth + 4;
}

int cuvit_vit_tensor_info(const cuvit_vit_config* config, int index, char* name,
                          size_t name_capacity, int64_t* extents, int* rank) {
    CUVIT_TRY(cuvit_vit_config_validate(config));
    const std::vector<TensorSpec> specs = tensor_specs(*config);
    if (index < 0 || index >= static_cast<int>(specs.size())) {
        return fail(CUVIT_INVALID_ARGUMENT, "tensor index out of range");
    }
    const TensorSpec& spec = specs[static_cast<size_t>(index)];
    if (name != nullptr && name_capacity > 0) {
        std::snprintf(name, name_capacity, "%s", spec.name.c_str());
    }
    if (rank != nullptr) {
        *rank = static_cast<int>(spec.extents.size());
    }
    if (extents != nullptr) {
        for (size_t i = 0; i < spec.extents.size(); ++i) {
            extents[i] = spec.extents[i];
        }
    }
    return CUVIT_OK;
}

int cuvit_vit_create_from_host(const cuvit_vit_config* config, const float* const* tensors,
                               int tensor_count, int max_batch, int precision, int device,
                               cuvit_vit** model) {
    if (config == nullptr || tensor_count != cuvit_vit_tensor_count(config)) {
        return fail(CUVIT_INVALID_ARGUMENT, "tensor count does not match the configuration");
    }
    return create(config, tensors, max_batch, precision, device, model);
}

int cuvit_vit_create_from_file(const cuvit_vit_config* config, const char* path, int max_batch,
                               int precision, int device, cuvit_vit** model) {
    if (config == nullptr || path == nullptr || model == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "model creation arguments cannot be null");
    }
    CUVIT_TRY(cuvit_vit_config_validate(config));
    std::vector<uint8_t> blob;
    std::unordered_map<std::string, CvwEntry> entries;
    CUVIT_TRY(read_cvw(path, &blob, &entries));
    const std::vector<TensorSpec> specs = tensor_specs(*config);
    std::vector<std::vector<float>> aligned(specs.size());
    std::vector<const float*> pointers(specs.size());
    for (size_t i = 0; i < specs.size(); ++i) {
        const auto found = entries.find(specs[i].name);
        if (found == entries.end()) {
            return fail(CUVIT_RUNTIME_ERROR,
                        "Weight file has no tensor named '" + specs[i].name + "'");
        }
        if (found->second.extents != specs[i].extents) {
            return fail(CUVIT_RUNTIME_ERROR, "Tensor '" + specs[i].name + "' has shape " +
                                                 shape_string(found->second.extents) + ", but " +
                                                 shape_string(specs[i].extents) +
                                                 " was expected");
        }
        aligned[i].resize(found->second.bytes / 4);
        std::memcpy(aligned[i].data(), blob.data() + found->second.offset, found->second.bytes);
        pointers[i] = aligned[i].data();
    }
    return create(config, pointers.data(), max_batch, precision, device, model);
}

int cuvit_vit_destroy(cuvit_vit* model) {
    if (model == nullptr) {
        return CUVIT_OK;
    }
    {
        DeviceGuard guard(model->device);
        cudaDeviceSynchronize();
        release(model);
    }
    delete model;
    return CUVIT_OK;
}

int cuvit_vit_forward(cuvit_vit* model, const float* images, float* logits, int batch,
                      cuvit_stream_t stream) {
    CUVIT_TRY(check_forward_args(model, images, logits, batch));
    if (batch == 0) {
        return CUVIT_OK;
    }
    DeviceGuard guard(model->device);
    return run_forward(*model, images, logits, batch, reinterpret_cast<cudaStream_t>(stream));
}

int cuvit_vit_forward_host(cuvit_vit* model, const float* images, float* logits, int batch,
                           cuvit_stream_t stream) {
    CUVIT_TRY(check_forward_args(model, images, logits, batch));
    if (batch == 0) {
        return CUVIT_OK;
    }
    DeviceGuard guard(model->device);
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const cuvit_vit_config& c = model->config;
    const size_t per_image = static_cast<size_t>(c.channels) * c.image_size * c.image_size;
    const int chunk = host_chunk_images(*model, batch);
    const int chunks = (batch + chunk - 1) / chunk;

    // Graphs for every chunk exist before the first copy is queued: a capture synchronizes
    // the model's capture stream and must not sit between a copy and the pass that reads it.
    std::vector<cudaGraphExec_t> execs(chunks);
    for (int i = 0; i < chunks; ++i) {
        const int images_here = i + 1 < chunks ? chunk : batch - i * chunk;
        CUVIT_TRY(graph_for(*model, model->stage_images + static_cast<size_t>(i) * chunk *
                                                              per_image,
                            model->stage_logits + static_cast<size_t>(i) * chunk * c.classes,
                            images_here, s, &execs[i]));
    }
    while (static_cast<int>(model->chunk_events.size()) < chunks) {
        cudaEvent_t event = nullptr;
        CUVIT_TRY_CUDA(cudaEventCreateWithFlags(&event, cudaEventDisableTiming));
        model->chunk_events.push_back(event);
    }

    // Copies run on the copy stream, chunk after chunk, each pass on the caller's stream once
    // its chunk has landed: chunk i+1 crosses PCIe while chunk i computes. Every chunk owns
    // its slice of the staging buffer, so no copy overwrites images a pass still reads.
    CUVIT_TRY_CUDA(cudaEventRecord(model->entry_event, s));
    CUVIT_TRY_CUDA(cudaStreamWaitEvent(model->copy_stream, model->entry_event, 0));
    for (int i = 0; i < chunks; ++i) {
        const int images_here = i + 1 < chunks ? chunk : batch - i * chunk;
        const size_t offset = static_cast<size_t>(i) * chunk * per_image;
        CUVIT_TRY_CUDA(cudaMemcpyAsync(model->stage_images + offset, images + offset,
                                       images_here * per_image * sizeof(float),
                                       cudaMemcpyHostToDevice, model->copy_stream));
        CUVIT_TRY_CUDA(cudaEventRecord(model->chunk_events[i], model->copy_stream));
    }
    for (int i = 0; i < chunks; ++i) {
        CUVIT_TRY_CUDA(cudaStreamWaitEvent(s, model->chunk_events[i], 0));
        CUVIT_TRY_CUDA(cudaGraphLaunch(execs[i], s));
    }
    const size_t logit_bytes = static_cast<size_t>(batch) * c.classes * sizeof(float);
    CUVIT_TRY_CUDA(
        cudaMemcpyAsync(logits, model->stage_logits, logit_bytes, cudaMemcpyDeviceToHost, s));
    CUVIT_TRY_CUDA(cudaStreamSynchronize(s));
    // The pass is complete: a kernel that gave up on a bounded wait left undefined logits.
    return cuvit::host::peek_device_status();
}

int cuvit_vit_forward_host_async(cuvit_vit* model, const float* images, float* logits,
                                 int batch, cuvit_stream_t stream) {
    CUVIT_TRY(check_forward_args(model, images, logits, batch));
    if (batch == 0) {
        return CUVIT_OK;
    }
    DeviceGuard guard(model->device);
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const cuvit_vit_config& c = model->config;
    const int slot = model->async_slot;
    float* const staged = slot == 0 ? model->stage_images : model->stage_images_alt;
    const bool bf16 = model->host_bf16;
    cudaGraphExec_t exec = nullptr;
    CUVIT_TRY(graph_for(*model, staged, model->stage_logits, batch, s, &exec, bf16));
    model->async_slot = slot ^ 1;
    const size_t count = static_cast<size_t>(batch) * c.channels * c.image_size * c.image_size;
    // The copies wait only for the pass that last read this slot (two calls back), so they
    // overlap the pass of the previous call; the pass waits for the copies.
    CUVIT_TRY_CUDA(cudaStreamWaitEvent(model->copy_stream, model->slot_free[slot], 0));
    if (bf16) {
        // Round the images into this slot's pinned buffer, once the copy that last read it
        // (two calls back) has finished; meanwhile the device runs the previous call's pass.
        // Quarter by quarter, so each quarter's copy overlaps the rounding of the next.
        CUVIT_TRY_CUDA(cudaEventSynchronize(model->slot_loaded[slot]));
        uint16_t* const pinned = model->pinned_bf16[slot];
        uint16_t* const device = reinterpret_cast<uint16_t*>(staged);
        constexpr int kPieces = 4;
        for (int piece = 0; piece < kPieces; ++piece) {
            const size_t first = count * piece / kPieces;
            const size_t last = count * (piece + 1) / kPieces;
            model->pool->run([&](int part, int parts) {
                const size_t begin = first + (last - first) * part / parts;
                const size_t end = first + (last - first) * (part + 1) / parts;
                cuvit::model::round_to_bf16(images + begin, pinned + begin, end - begin);
            });
            CUVIT_TRY_CUDA(cudaMemcpyAsync(device + first, pinned + first,
                                           (last - first) * sizeof(uint16_t),
                                           cudaMemcpyHostToDevice, model->copy_stream));
        }
    } else {
        CUVIT_TRY_CUDA(cudaMemcpyAsync(staged, images, count * sizeof(float),
                                       cudaMemcpyHostToDevice, model->copy_stream));
    }
    CUVIT_TRY_CUDA(cudaEventRecord(model->slot_loaded[slot], model->copy_stream));
    CUVIT_TRY_CUDA(cudaStreamWaitEvent(s, model->slot_loaded[slot], 0));
    CUVIT_TRY_CUDA(cudaGraphLaunch(exec, s));
    CUVIT_TRY_CUDA(cudaEventRecord(model->slot_free[slot], s));
    const size_t logit_bytes = static_cast<size_t>(batch) * c.classes * sizeof(float);
    CUVIT_TRY_CUDA(
        cudaMemcpyAsync(logits, model->stage_logits, logit_bytes, cudaMemcpyDeviceToHost, s));
    return CUVIT_OK;
}

int cuvit_vit_set_host_chunk(cuvit_vit* model, int images) {
    if (model == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "model cannot be null");
    }
    if (images < 0) {
        return fail(CUVIT_INVALID_ARGUMENT, "the host chunk size cannot be negative");
    }
    model->host_chunk = images;
    return CUVIT_OK;
}

int cuvit_vit_forward_graph(cuvit_vit* model, const float* images, float* logits, int batch,
                            cuvit_stream_t stream) {
    CUVIT_TRY(check_forward_args(model, images, logits, batch));
    if (batch == 0) {
        return CUVIT_OK;
    }
    DeviceGuard guard(model->device);
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    cudaGraphExec_t exec = nullptr;
    CUVIT_TRY(graph_for(*model, images, logits, batch, s, &exec));
    CUVIT_TRY_CUDA(cudaGraphLaunch(exec, s));
    return CUVIT_OK;
}

int cuvit_vit_forward_profiled(cuvit_vit* model, const float* images, float* logits, int batch,
                               cuvit_stream_t stream, cuvit_launch_record* records,
                               int capacity, int* count) {
    CUVIT_TRY(check_forward_args(model, images, logits, batch));
    if (count == nullptr) {
        return fail(CUVIT_INVALID_ARGUMENT, "count cannot be null");
    }
    *count = 0;
    if (batch == 0) {
        return CUVIT_OK;
    }
    DeviceGuard guard(model->device);
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    Recorder recorder(s);
    CUVIT_TRY(run_forward(*model, images, logits, batch, s, &recorder));
    return recorder.finish(records, capacity, count);
}

int cuvit_vit_max_batch(const cuvit_vit* model) { return model ? model->max_batch : 0; }
size_t cuvit_vit_weight_bytes(const cuvit_vit* model) { return model ? model->weight_used : 0; }
size_t cuvit_vit_activation_bytes(const cuvit_vit* model) {
    return model ? model->activation_used : 0;
}
size_t cuvit_vit_image_elements(const cuvit_vit* model) {
    if (model == nullptr) {
        return 0;
    }
    return static_cast<size_t>(model->config.channels) * model->config.image_size *
           model->config.image_size;
}
size_t cuvit_vit_host_image_bytes(const cuvit_vit* model) {
    return cuvit_vit_image_elements(model) * (model != nullptr && model->host_bf16 ? 2 : 4);
}

int cuvit_vit_launches_per_forward(const cuvit_vit* model, int batch) {
    if (model == nullptr || batch <= 0) {
        return 0;
    }
    const int attention = model->precision == CUVIT_MATH_FP32 ? 3 : 1;
    return 3 + model->config.depth * (6 + attention) + 2;
}

} // extern "C"
