/*
 * cuvit_b200.h -- C ABI of the B200 (sm_100a) implementation of Cu-Vit's hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream, returns a
 * cuvit_status, and allocates nothing on the calling path (the model runner, the replicas and
 * the communicator allocate once, at creation, like the reference's VisionTransformer
 * constructor; the instrumented build's timeline table is allocated by its first reset). Argument
 * validation happens on the host before any launch, in the same order and with the same
 * outcome classes as the reference's C++ launchers:
 *
 *   reference outcome                          status here
 *   --------------------------------------     --------------------------
 *   silent no-op on an empty problem           CUVIT_OK, nothing launched
 *   std::invalid_argument                      CUVIT_INVALID_ARGUMENT
 *   std::length_error (grid limit)             CUVIT_LENGTH_ERROR
 *   cuvit::CudaError (cudaGetLastError)        CUVIT_CUDA_ERROR
 *   std::runtime_error (weights, shapes)       CUVIT_RUNTIME_ERROR
 *
 * cuvit_last_error_message() returns the detail text of the calling thread's last failure.
 * The C++ header <cuvit/kernels.hpp> wraps these functions with the reference's exact
 * cuvit::launch_* signatures and exception types.
 */
#ifndef CUVIT_B200_H
#define CUVIT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

/* Same handle as cudaStream_t; NULL selects the legacy default stream. */
typedef struct CUstream_st* cuvit_stream_t;

typedef enum cuvit_status {
    CUVIT_OK = 0,
    CUVIT_INVALID_ARGUMENT = 1,
    CUVIT_LENGTH_ERROR = 2,
    CUVIT_CUDA_ERROR = 3,
    /* A bounded device-side wait (mbarrier, TMEM handshake) ran out; the kernel returned
     * early and its outputs are undefined. Reported by cuvit_device_status(). */
    CUVIT_DEVICE_TIMEOUT = 4,
    /* The current device is not an sm_100 part, or a feature is not built. */
    CUVIT_UNSUPPORTED = 5,
    CUVIT_RUNTIME_ERROR = 6,
    CUVIT_OUT_OF_MEMORY = 7
} cuvit_status;

const char* cuvit_status_string(int status);
/* Detail text for the calling thread's most recent non-OK status ("" if none). */
const char* cuvit_last_error_message(void);
/* Library version as major*10000 + minor*100 + patch. */
int cuvit_version(void);

/* ---------------------------------------------------------------------------------------
 * GEMM. Mirrors include/cuvit/kernels.hpp:9-99 of the reference field for field:
 *
 *   C[i][m][n] = epilogue(alpha * sum_k A[i][m][k] * B_layout[i][k][n] + bias[n])
 *
 * epilogue order per element (src/kernels/gemm.cu:153-162): alpha, +bias, GELU (erf form),
 * then store or accumulate into C.
 * ------------------------------------------------------------------------------------- */
typedef enum cuvit_gemm_layout {
    CUVIT_LAYOUT_NO_TRANSPOSE = 0, /* B is [K, N]: C[m][n] = sum_k A[m][k] * B[k][n] */
    CUVIT_LAYOUT_TRANSPOSED = 1    /* B is [N, K]: C[m][n] = sum_k A[m][k] * B[n][k] */
} cuvit_gemm_layout;

/* reference: GemmBatch, include/cuvit/kernels.hpp:46-59 */
typedef struct cuvit_gemm_batch {
    int count;
    int64_t stride_a;
    int64_t stride_b;
    int64_t stride_c;
    /* When positive, entry i is (i / inner, i % inner); the first part advances by the outer
     * strides. inner >= count collapses to a flat batch (src/kernels/gemm.cu:220-223). */
    int inner;
    int64_t outer_stride_a;
    int64_t outer_stride_b;
    int64_t outer_stride_c;
} cuvit_gemm_batch;

/* reference: GemmEpilogue, include/cuvit/kernels.hpp:30-36 */
typedef struct cuvit_gemm_epilogue {
    int accumulate; /* C += value instead of C = value (residual connection) */
    int gelu;       /* GELU (erf form) after the bias */
} cuvit_gemm_epilogue;

/* reference: GemmProblem, include/cuvit/kernels.hpp:74-85. ld* == 0 selects the packed
 * distance: lda = k, ldb = (transposed ? k : n), ldc = n (src/kernels/gemm.cu:226-228). */
typedef struct cuvit_gemm_problem {
    int m;
    int n;
    int k;
    int layout; /* cuvit_gemm_layout */
    float alpha;
    int lda;
    int ldb;
    int ldc;
    cuvit_gemm_batch batch;
    cuvit_gemm_epilogue epilogue;
} cuvit_gemm_problem;

/* Fills *problem like the reference's gemm_problem() (include/cuvit/kernels.hpp:89-96):
 * one un-batched problem, packed operands, alpha 1, no epilogue. */
void cuvit_gemm_problem_init(cuvit_gemm_problem* problem, int m, int n, int k, int layout);

/* Storage types. TF32 is float storage holding values rounded to the nearest TF32 value
 * (10-bit mantissa): what a producer writes for a tensor that a TF32 tensor-core operation
 * consumes next, which would otherwise truncate the low mantissa bits (a bias that
 * accumulates over long reductions). */
typedef enum cuvit_dtype {
    CUVIT_DTYPE_F32 = 0,
    CUVIT_DTYPE_BF16 = 1,
    CUVIT_DTYPE_TF32 = 2
} cuvit_dtype;

/* Arithmetic of a float GEMM.
 *   FP32: FP32-faithful. Tensor-core 3xTF32 split (hi*hi + hi*lo + lo*hi with FP32
 *         accumulation in TMEM) where TMA can describe the operands, FP32 FFMA otherwise.
 *         Holds the reference's FP32 tolerances (tests/gemm_test.cu:83-87).
 *   TF32: one TF32 tensor-core pass (10-bit mantissa products, FP32 accumulation).
 *   BF16: operands in bfloat16, FP32 accumulation. */
typedef enum cuvit_math { CUVIT_MATH_FP32 = 0, CUVIT_MATH_TF32 = 1, CUVIT_MATH_BF16 = 2 } cuvit_math;

/* Replaces cuvit::launch_gemm (include/cuvit/kernels.hpp:98-99, src/kernels/gemm.cu:199-242).
 * FP32 operands; the arithmetic is the process-wide math mode (default CUVIT_MATH_FP32). */
int cuvit_gemm(const float* a, const float* b, const float* bias, float* c,
               const cuvit_gemm_problem* problem, cuvit_stream_t stream);

/* Process-wide arithmetic used by cuvit_gemm(): CUVIT_MATH_FP32 or CUVIT_MATH_TF32. */
int cuvit_set_math_mode(int math);
int cuvit_get_math_mode(void);

/* Typed GEMM: a/b are bfloat16 when math is CUVIT_MATH_BF16 and float otherwise; c is
 * c_dtype (F32, BF16, or TF32-rounded float; accumulate reads it in that type); bias is
 * float. Same problem semantics as cuvit_gemm(). */
int cuvit_gemm_ex(const void* a, const void* b, const float* bias, void* c, int c_dtype,
                  int math, const cuvit_gemm_problem* problem, cuvit_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Memory-bound operators. Each replaces the reference function named beside it.
 * ------------------------------------------------------------------------------------- */

/* cuvit::launch_layer_norm (include/cuvit/kernels.hpp:107-109, normalization.cu:224-239):
 * out = (in - mean) / sqrt(var + eps) * gamma + beta over each row, biased variance. */
int cuvit_layer_norm(const float* input, const float* gamma, const float* beta, float* output,
                     int rows, int columns, float epsilon, cuvit_stream_t stream);

/* Strided/typed layer norm: rows are input_row_stride / output_row_stride elements apart
 * (0 = columns) and the output is out_dtype. Used for the class-token-only final norm. */
int cuvit_layer_norm_ex(const float* input, int64_t input_row_stride, const float* gamma,
                        const float* beta, void* output, int out_dtype,
                        int64_t output_row_stride, int rows, int columns, float epsilon,
                        cuvit_stream_t stream);

/* cuvit::launch_gelu (kernels.hpp:117-118, normalization.cu:257-271): erf-form GELU. */
int cuvit_gelu(const float* input, float* output, int64_t count, cuvit_stream_t stream);

/* cuvit::launch_softmax (kernels.hpp:122-123, normalization.cu:241-255): stable row
 * softmax; input may equal output (the model calls it in place, src/model/vit.cu:225). */
int cuvit_softmax(const float* input, float* output, int rows, int columns,
                  cuvit_stream_t stream);

/* Row-strided softmax: row r starts at r * row_stride (row_stride >= columns). */
int cuvit_softmax_ex(const float* input, float* output, int rows, int columns,
                     int64_t row_stride, cuvit_stream_t stream);

/* cuvit::launch_extract_patches (kernels.hpp:137-138, normalization.cu:273-298):
 * patches[b*P + p][c*patch*patch + r*patch + q] = images[b][c][pr*patch + r][pc*patch + q]. */
int cuvit_extract_patches(const float* images, float* patches, int batch, int channels,
                          int height, int width, int patch, cuvit_stream_t stream);

/* Same gather with the patch matrix written as out_dtype (bfloat16 feeds the BF16 GEMM). */
int cuvit_extract_patches_ex(const float* images, void* patches, int out_dtype, int batch,
                             int channels, int height, int width, int patch,
                             cuvit_stream_t stream);

/* cuvit::launch_add (kernels.hpp:141-142, normalization.cu:300-314): acc += addend. */
int cuvit_add(float* accumulator, const float* addend, int64_t count, cuvit_stream_t stream);

/* cuvit::launch_add_broadcast (kernels.hpp:147-148, normalization.cu:316-332):
 * acc[b*count + i] += addend[i] for b < batch. */
int cuvit_add_broadcast(float* accumulator, const float* addend, int64_t count, int batch,
                        cuvit_stream_t stream);

/* cuvit::launch_broadcast (kernels.hpp:153-154, normalization.cu:334-350):
 * dst[b*dst_stride + i] = src[i] for b < batch. */
int cuvit_broadcast(float* destination, const float* source, int64_t count,
                    int64_t destination_stride, int batch, cuvit_stream_t stream);

/* Class token + positional embedding in one pass (replaces the launch_broadcast +
 * launch_add_broadcast pair at src/model/vit.cu:299-300 when the patch-embedding GEMM then
 * accumulates into rows 1..T-1): tokens[b][0] = cls + pos[0], tokens[b][t] = pos[t]. */
int cuvit_init_tokens(float* tokens, const float* class_token, const float* position,
                      int batch, int tokens_per_image, int embed, cuvit_stream_t stream);

/* Converts count floats to bfloat16 (round to nearest even). */
int cuvit_convert_f32_to_bf16(const float* input, void* output, int64_t count,
                              cuvit_stream_t stream);

/* Rounds count floats to the nearest TF32 value, kept in float storage (CUVIT_DTYPE_TF32);
 * input may equal output. */
int cuvit_round_to_tf32(const float* input, float* output, int64_t count,
                        cuvit_stream_t stream);

/* Top-k report of logits rows (reference: report_top, src/main.cpp:90-114, which the CLI runs
 * on the host): for each of `batch` rows of `classes` device logits, the k largest in
 * descending order -- equal logits by ascending class index, where the reference's
 * partial_sort leaves their order open -- into device arrays [batch, k]: class indices,
 * logits, and softmax probabilities exp(logit - max) / sum_j exp(logit_j - max), summed and
 * divided in double like the reference. NaN logits take no part: they are left out of the
 * maximum and the sum and are never reported; a row with fewer than k other logits reports
 * index -1, value NaN and probability 0 in the remaining places. 1 <= k <= classes. */
int cuvit_logits_top_k(const float* logits, int batch, int classes, int k, int* indices,
                       float* values, float* probabilities, cuvit_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Image preprocessing on the device. Replaces cuvit::preprocess (include/cuvit/image.hpp,
 * src/runtime/image.cpp:90-135), which the reference runs on the host: the shorter side is
 * resized to round(size / crop_fraction) with bilinear sampling and edge clamping, the centre
 * size x size square kept, values scaled to [0, 1] and normalised per channel. Results are
 * bit-identical to the reference's host code.
 * ------------------------------------------------------------------------------------- */
typedef struct cuvit_preprocessing {
    int size;            /* output side (reference default 224) */
    float crop_fraction; /* in (0, 1] (default 0.9) */
    float mean[3];       /* per channel (default 0.5) */
    float stddev[3];     /* per channel, nonzero (default 0.5) */
} cuvit_preprocessing;

/* The reference's Preprocessing defaults (include/cuvit/image.hpp). */
void cuvit_preprocessing_default(cuvit_preprocessing* settings);

/* pixels: device, `batch` interleaved 8-bit RGB images of width x height, image_stride bytes
 * apart (0 = packed, width * height * 3). tensor: device float [batch, 3, size, size], the
 * layout cuvit_vit_forward reads. Rejects what the reference rejects (empty image, size <= 0,
 * crop fraction outside (0, 1], a zero deviation) with CUVIT_INVALID_ARGUMENT and its
 * message, before any launch; images of 2^22 pixels or more a side, sizes above 46340 and
 * batches above 65535 with CUVIT_LENGTH_ERROR (limits of the device kernel, not the
 * reference's). */
int cuvit_preprocess(const uint8_t* pixels, int batch, int width, int height,
                     int64_t image_stride, const cuvit_preprocessing* settings, float* tensor,
                     cuvit_stream_t stream);

/* ---------------------------------------------------------------------------------------
 * Fused attention. Replaces the Q.K^T GEMM -> launch_softmax -> .V GEMM sequence of
 * src/model/vit.cu:198-242 with one kernel that keeps the T x T logits on chip.
 *
 * qkv:     [batch * tokens, 3 * heads * head_dim], each row packed [3][heads][head_dim]
 * context: [batch * tokens, heads * head_dim], head h in columns h*head_dim ..
 * dtype:   CUVIT_DTYPE_BF16 (BF16 tensor cores), CUVIT_DTYPE_F32 (float storage, TF32
 *          tensor cores) or CUVIT_DTYPE_TF32 (the same, context stored rounded to TF32
 *          values); qkv and context share the storage type. Softmax statistics are FP32.
 * Supported: head_dim == 64, 1 <= tokens <= 256, 16-byte aligned rows.
 * ------------------------------------------------------------------------------------- */
int cuvit_attention(const void* qkv, void* context, int dtype, int batch, int tokens,
                    int heads, int head_dim, float scale, cuvit_stream_t stream);

/* Reads and clears the device status word of the current device, after synchronizing it.
 * *flags receives the bits set since the last call (0 = clean). Returns
 * CUVIT_DEVICE_TIMEOUT when a kernel gave up on a bounded wait.
 * The word is one per device and per process: every model, stream and host thread of the
 * process that launches on that device shares it. Once a kernel has timed out, every later
 * wait on that device that does not complete within its first few spins also gives up (so
 * a stuck device drains quickly instead of each kernel waiting out the full limit), until
 * some caller reads the word here; that read clears it for every user of the device. Callers
 * that share a device should therefore agree on who checks it. cuvit_vit_forward_host()
 * checks it (without clearing) after its pass and returns CUVIT_DEVICE_TIMEOUT when set. */
int cuvit_device_status(unsigned* flags);

/* Diagnostic: launches one thread that waits on a barrier nothing will release, with a
 * device-side limit of limit_ns (at most 1 s). The wait gives up, sets the timeout bit of the
 * device status word and the kernel returns, so the next cuvit_device_status() reports
 * CUVIT_DEVICE_TIMEOUT and the context stays usable. Exercises the timeout path without
 * faulting or hanging the GPU. */
int cuvit_selftest_bounded_wait(unsigned long long limit_ns);

/* Number of kernels this library launched from the calling process (all threads). */
long long cuvit_launch_count(void);

/* Device timeline (diagnostic; no reference counterpart). Only the instrumented variant of
 * the library (built with `python cu-vit_b200/build.py --timeline`, file
 * libcuvit_b200_timeline.so) records it; elsewhere cuvit_timeline_available() returns 0 and
 * the other two calls return CUVIT_UNSUPPORTED. Each forward-path kernel stamps the global
 * nanosecond timer when its first CTA starts and when its last CTA ends, and CTA 0 also
 * records its SM's cycle counter at entry and exit (cycles / ns = the SM clock that kernel
 * ran at). One record per launch, keyed by the launch's grid id, current device only. */
typedef struct cuvit_timeline_record {
    unsigned long long grid;        /* per-launch grid identifier */
    unsigned long long first_ns;    /* earliest CTA entry (global timer, ns) */
    unsigned long long last_ns;     /* latest warp exit */
    unsigned long long warps;       /* CTAs that stamped their exit (the grid's last ones) */
    unsigned long long cta0_entry_ns;
    unsigned long long cta0_exit_ns;
    unsigned long long cta0_entry_clock; /* SM cycle counter of CTA 0 */
    unsigned long long cta0_exit_clock;
} cuvit_timeline_record;

int cuvit_timeline_available(void);
/* Synchronizes the device and clears the table (allocating it on first use). */
int cuvit_timeline_reset(void);
/* Synchronizes the device and returns the recorded launches in start order: up to capacity
 * records, *count receives how many there are. */
int cuvit_timeline_read(cuvit_timeline_record* records, int capacity, int* count);

/* ---------------------------------------------------------------------------------------
 * Model runner. Replaces cuvit::VisionTransformer (include/cuvit/vit.hpp:63-120,
 * src/model/vit.cu:69-344): weights and activations live in two arenas allocated at
 * creation; forward() allocates nothing.
 * ------------------------------------------------------------------------------------- */
typedef struct cuvit_vit_config {
    int image_size;
    int patch_size;
    int channels;
    int embed_dim;
    int depth;
    int heads;
    int mlp_hidden;
    int classes;
    float layer_norm_epsilon;
} cuvit_vit_config;

/* ViT-Tiny/16 defaults (include/cuvit/vit.hpp:15-24). */
void cuvit_vit_config_default(cuvit_vit_config* config);
/* reference: VitConfig::validate (src/model/vit.cu:36-47). */
int cuvit_vit_config_validate(const cuvit_vit_config* config);
/* Number of tensors and the timm name / extents of tensor i in load order
 * (reference: VisionTransformer::expected_tensor_names, src/model/vit.cu:49-63).
 * extents receives up to 4 values; *rank their count. */
int cuvit_vit_tensor_count(const cuvit_vit_config* config);
int cuvit_vit_tensor_info(const cuvit_vit_config* config, int index, char* name,
                          size_t name_capacity, int64_t* extents, int* rank);

typedef struct cuvit_vit cuvit_vit;

/* precision: CUVIT_MATH_FP32 (FP32-faithful, unfused attention as in the reference),
 * CUVIT_MATH_TF32 or CUVIT_MATH_BF16 (fused attention). */
int cuvit_vit_create_from_host(const cuvit_vit_config* config, const float* const* tensors,
                               int tensor_count, int max_batch, int precision, int device,
                               cuvit_vit** model);
/* Loads a Cu-Vit .cvw v1 weight file (format of src/runtime/weights.cpp:13-24). */
int cuvit_vit_create_from_file(const cuvit_vit_config* config, const char* path,
                               int max_batch, int precision, int device, cuvit_vit** model);
int cuvit_vit_destroy(cuvit_vit* model);

/* reference: VisionTransformer::forward(images, logits, batch, stream), vit.cu:263-317.
 * images: device [batch, C, H, W] float; logits: device [batch, classes] float. */
int cuvit_vit_forward(cuvit_vit* model, const float* images, float* logits, int batch,
                      cuvit_stream_t stream);
/* Host-memory convenience (reference: forward(std::vector), vit.cu:319-344): copies host
 * images in, runs, copies logits out and synchronizes. Uses staging buffers allocated at
 * creation, so it allocates nothing per call. Batches of 64 images and more run in two
 * halves: the second half's copy runs on a second stream while the first half computes,
 * which needs pinned host memory to overlap. Logits do not depend on the chunking (every
 * image's result is independent of the batch it runs in). Returns CUVIT_DEVICE_TIMEOUT,
 * with undefined logits, when the device status word is set after the pass (it is left set;
 * see cuvit_device_status). */
int cuvit_vit_forward_host(cuvit_vit* model, const float* images, float* logits, int batch,
                           cuvit_stream_t stream);
/* forward_host() without the final synchronisation, for serving loops: queues the copy of
 * the images into one of two staging slots (on a second stream), the pass on `stream`, and
 * the copy of the logits back to `logits`, then returns. The copy of call i+1 overlaps the
 * pass of call i. The host buffers must stay valid and unchanged until `stream` has reached
 * this call's work (synchronize it, or wait on an event recorded after the call); the images
 * must hold their data when the call is made, since the copy is not ordered after earlier
 * work on `stream`. Consecutive calls on one model must use the same stream. BF16 models
 * (patch size and image width multiples of 4) created with CUVIT_HOST_ROUNDING=1 in the
 * environment first round the images to bfloat16 on host threads into pinned buffers the
 * model owns -- the rounding the device would apply to every pixel, so the logits are the
 * same -- and copy half the bytes (for hosts where PCIe, not host memory, limits the copy);
 * the images are then read before the call returns. No reference counterpart (the
 * reference's host-vector forward is synchronous). */
int cuvit_vit_forward_host_async(cuvit_vit* model, const float* images, float* logits,
                                 int batch, cuvit_stream_t stream);
/* Images per forward_host chunk; 0 restores the automatic choice. No reference
 * counterpart (the reference copies the whole batch before running it). */
int cuvit_vit_set_host_chunk(cuvit_vit* model, int images);
/* Replays a CUDA graph of the whole pass for this batch size (captured on first use). */
int cuvit_vit_forward_graph(cuvit_vit* model, const float* images, float* logits, int batch,
                            cuvit_stream_t stream);

/* What one launch of a forward pass does. */
typedef enum cuvit_launch_kind {
    CUVIT_KIND_PATCHES = 0,    /* patch gather */
    CUVIT_KIND_TOKENS = 1,     /* class token + position initialisation */
    CUVIT_KIND_GEMM_PATCH = 2, /* patch-embedding GEMM */
    CUVIT_KIND_LAYER_NORM = 3,
    CUVIT_KIND_GEMM_QKV = 4,
    CUVIT_KIND_ATTENTION = 5,  /* fused attention, or one of the three unfused steps */
    CUVIT_KIND_GEMM_PROJ = 6,
    CUVIT_KIND_GEMM_FC1 = 7,
    CUVIT_KIND_GEMM_FC2 = 8,
    CUVIT_KIND_GEMM_HEAD = 9
} cuvit_launch_kind;

typedef struct cuvit_launch_record {
    int kind;           /* cuvit_launch_kind */
    int layer;          /* block index, -1 outside the blocks */
    double flops;       /* algorithmic FLOPs (2 per multiply-add; 0 for memory-bound kernels) */
    double bytes;       /* algorithmic HBM bytes: every operand read once, results written once */
    float milliseconds; /* device time between CUDA events recorded around the launch */
} cuvit_launch_record;

/* forward() with a CUDA event pair around every launch; synchronizes the stream and fills
 * up to capacity records in launch order (*count receives the number of launches). For
 * per-kernel timing; the events add small gaps, so time whole passes with forward_graph. */
int cuvit_vit_forward_profiled(cuvit_vit* model, const float* images, float* logits, int batch,
                               cuvit_stream_t stream, cuvit_launch_record* records,
                               int capacity, int* count);

int cuvit_vit_max_batch(const cuvit_vit* model);
size_t cuvit_vit_weight_bytes(const cuvit_vit* model);
size_t cuvit_vit_activation_bytes(const cuvit_vit* model);
size_t cuvit_vit_image_elements(const cuvit_vit* model);
/* Bytes one image takes on its way host -> device in forward_host_async: 2 per image element
 * where the model rounds images to bfloat16 on the host (see forward_host_async), else 4.
 * No reference counterpart. */
size_t cuvit_vit_host_image_bytes(const cuvit_vit* model);
/* Kernel launches one forward pass issues for this batch size. */
int cuvit_vit_launches_per_forward(const cuvit_vit* model, int batch);

/* ---------------------------------------------------------------------------------------
 * Several GPUs. No reference counterpart: the reference runs one VisionTransformer on one
 * device. Images are independent, so a batch shards by image across GPUs with the weights
 * replicated, and the logits are the only data exchanged (no per-layer collective).
 * ------------------------------------------------------------------------------------- */

/* The contiguous shard [*first, *first + *count) of `total` images owned by part `index` of
 * `parts`: the first total % parts parts take one extra image. Gathering the parts in index
 * order restores the global image order. */
int cuvit_shard(int total, int parts, int index, int* first, int* count);

/* One process per GPU: an NCCL communicator (NCCL is loaded at run time; these calls return
 * CUVIT_UNSUPPORTED where libnccl.so.2 cannot be loaded). Rank 0 makes the unique id
 * (id_capacity >= 128 bytes) and hands it to every rank by any host channel; every rank then
 * calls cuvit_comm_create, which returns once all `world` ranks have joined. */
typedef struct cuvit_comm cuvit_comm;
int cuvit_comm_unique_id(void* id, size_t id_capacity);
int cuvit_comm_create(const void* id, int world, int rank, int device, cuvit_comm** comm);
int cuvit_comm_destroy(cuvit_comm* comm);
/* Gathers every rank's [rows, classes] device logits to `root` (grouped NCCL send / receive,
 * queued on `stream`): gathered (root only, device) receives world * rows rows in rank order.
 * Every rank calls it with the same rows, classes and root, in the same order relative to its
 * other collectives. */
int cuvit_gather_logits(cuvit_comm* comm, const float* local, float* gathered, int rows,
                        int classes, int root, cuvit_stream_t stream);

/* One process driving several GPUs: a model per device (weights uploaded to each), one host
 * thread per device. devices may repeat a device (two replicas sharing one GPU). */
typedef struct cuvit_replicas cuvit_replicas;
int cuvit_replicas_create(const cuvit_vit_config* config, const float* const* tensors,
                          int tensor_count, int max_batch_per_device, int precision,
                          const int* devices, int device_count, cuvit_replicas** replicas);
int cuvit_replicas_destroy(cuvit_replicas* replicas);
int cuvit_replicas_device_count(const cuvit_replicas* replicas);
/* Host images [batch, C, H, W] in, host logits [batch, classes] out, synchronous: device i
 * runs shard i (cuvit_shard) through cuvit_vit_forward_host and writes its rows of the
 * logits. batch <= device_count * max_batch_per_device. */
int cuvit_replicas_forward_host(cuvit_replicas* replicas, const float* images, float* logits,
                                int batch);
/* Device-resident form: images on device images_device, logits into a buffer on device
 * logits_device; device i copies its shard of the images peer to peer, replays its pass and
 * copies its logits peer to peer into their rows. Synchronous. */
int cuvit_replicas_forward(cuvit_replicas* replicas, const float* images, int images_device,
                           float* logits, int logits_device, int batch);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* CUVIT_B200_H */
