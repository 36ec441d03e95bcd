/*
 * cuvit_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's CPU algorithms for Cu-Vit's hot path, used as the
 * checker for the CUDA library. Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference legs may load it; the product (libcuvit_b200.so) never does.
 *
 * Every function keeps the reference's order of floating-point operations so that, built
 * without FMA contraction (-ffp-contract=off), it reproduces the reference's own CPU code
 * bit for bit; tests/test_oracle.py pins that against golden vectors written by the
 * reference's code itself (tests/golden/make_golden.py) and, when present, against
 * oracle/_ref/libcuvit_ref_cpu.so built from the reference's sources.
 *
 * Reference file:line citations are relative to the Cu-Vit source tree.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* GELU, erf form: tests/reference/linear_algebra.hpp:120-123 (same expression as the GPU
 * epilogue, src/kernels/gemm.cu:157-160). */
float oracle_gelu(float value) { return 0.5F * value * (1.0F + erff(value * 0.7071067811865475F)); }

void oracle_gelu_array(const float* input, float* output, int64_t count) {
    for (int64_t i = 0; i < count; ++i) {
        output[i] = oracle_gelu(input[i]);
    }
}

/*
 * Batched GEMM with the GemmProblem semantics of include/cuvit/kernels.hpp:38-96:
 *   C[e][m][n] = epi(alpha * sum_k A[e][m][k] * B_layout[e][k][n] + bias[n])
 * Per element: float sum over k in order (tests/reference/linear_algebra.hpp:18-48), then
 * alpha, bias, GELU, store or accumulate (src/kernels/gemm.cu:153-162). Batch entry e maps
 * to (e / inner, e % inner) when inner > 0 (src/kernels/gemm.cu:62-72). ld values are the
 * resolved ones (callers apply the packed defaults, src/kernels/gemm.cu:226-228).
 */
void oracle_gemm(const float* a, const float* b, const float* bias, float* c, int m, int n,
                 int k, int transposed, float alpha, int64_t lda, int64_t ldb, int64_t ldc,
                 int count, int inner, int64_t stride_a, int64_t stride_b, int64_t stride_c,
                 int64_t outer_a, int64_t outer_b, int64_t outer_c, int accumulate, int gelu) {
    if (inner >= count) {
        inner = 0;
    }
    for (int entry = 0; entry < count; ++entry) {
        int64_t oa, ob, oc;
        if (inner > 0) {
            const int64_t outer = entry / inner;
            const int64_t index = entry % inner;
            oa = outer * outer_a + index * stride_a;
            ob = outer * outer_b + index * stride_b;
            oc = outer * outer_c + index * stride_c;
        } else {
            oa = (int64_t)entry * stride_a;
            ob = (int64_t)entry * stride_b;
            oc = (int64_t)entry * stride_c;
        }
        for (int row = 0; row < m; ++row) {
            for (int col = 0; col < n; ++col) {
                float sum = 0.0F;
                for (int i = 0; i < k; ++i) {
                    const float left = a[oa + (int64_t)row * lda + i];
                    const float right = transposed ? b[ob + (int64_t)col * ldb + i]
                                                   : b[ob + (int64_t)i * ldb + col];
                    sum += left * right;
                }
                float value = alpha * sum + (bias != NULL ? bias[col] : 0.0F);
                if (gelu) {
                    value = oracle_gelu(value);
                }
                float* const out = c + oc + (int64_t)row * ldc + col;
                *out = accumulate ? *out + value : value;
            }
        }
    }
}

/* Sum of |a_k * b_k| per output: the error scale for a reduction
 * (tests/reference/linear_algebra.hpp:52-68). Packed operands, one problem. */
void oracle_gemm_term_magnitudes(const float* a, const float* b, float* scale, int m, int n,
                                 int k, int transposed, float alpha) {
    for (int row = 0; row < m; ++row) {
        for (int col = 0; col < n; ++col) {
            float total = 0.0F;
            for (int i = 0; i < k; ++i) {
                const float left = a[(int64_t)row * k + i];
                const float right =
                    transposed ? b[(int64_t)col * k + i] : b[(int64_t)i * n + col];
                total += fabsf(left * right);
            }
            scale[(int64_t)row * n + col] = fabsf(alpha) * total;
        }
    }
}

/* Layer norm with double accumulation: tests/reference/linear_algebra.hpp:70-96. Rows are
 * in_stride / out_stride elements apart. */
void oracle_layer_norm(const float* input, int64_t in_stride, const float* gamma,
                       const float* beta, float* output, int64_t out_stride, int rows,
                       int columns, float epsilon) {
    for (int row = 0; row < rows; ++row) {
        const float* const source = input + (int64_t)row * in_stride;
        float* const destination = output + (int64_t)row * out_stride;
        double sum = 0.0;
        for (int c = 0; c < columns; ++c) {
            sum += source[c];
        }
        const double mean = sum / columns;
        double variance = 0.0;
        for (int c = 0; c < columns; ++c) {
            const double centered = source[c] - mean;
            variance += centered * centered;
        }
        variance /= columns;
        const double inverse = 1.0 / sqrt(variance + epsilon);
        for (int c = 0; c < columns; ++c) {
            destination[c] = (float)((source[c] - mean) * inverse) * gamma[c] + beta[c];
        }
    }
}

/* Stable softmax, exponent and sum in double: tests/reference/linear_algebra.hpp:98-118.
 * Rows are stride elements apart; input may equal output. */
void oracle_softmax(const float* input, float* output, int rows, int columns, int64_t stride) {
    for (int row = 0; row < rows; ++row) {
        const float* const source = input + (int64_t)row * stride;
        float* const destination = output + (int64_t)row * stride;
        float maximum = source[0];
        for (int c = 1; c < columns; ++c) {
            maximum = source[c] > maximum ? source[c] : maximum;
        }
        double sum = 0.0;
        for (int c = 0; c < columns; ++c) {
            const double value = exp((double)source[c] - maximum);
            destination[c] = (float)value;
            sum += value;
        }
        for (int c = 0; c < columns; ++c) {
            destination[c] = (float)(destination[c] / sum);
        }
    }
}

/* Top-k report of logits rows: report_top, src/main.cpp:90-114. The k largest logits of each
 * row in descending order (the reference's std::partial_sort leaves equal logits in no
 * particular order; here the lower class index comes first) and their stable-softmax
 * probabilities, exp(logit - max) / sum exp(logit_j - max), in double. */
void oracle_top_k(const float* logits, int batch, int classes, int k, int* indices,
                  float* values, double* probabilities) {
    for (int row = 0; row < batch; ++row) {
        const float* const x = logits + (int64_t)row * classes;
        /* NaN logits take no part in the maximum, the sum or the picks (the reference's
         * partial_sort leaves a row with NaNs unordered, so the rule is this library's). */
        float maximum = -INFINITY;
        for (int c = 0; c < classes; ++c) {
            maximum = x[c] > maximum ? x[c] : maximum;
        }
        double total = 0.0;
        for (int c = 0; c < classes; ++c) {
            if (x[c] == x[c]) {
                total += exp((double)x[c] - maximum);
            }
        }
        float last_value = INFINITY;
        int last_index = -1;
        for (int r = 0; r < k; ++r) {
            int best = -1;
            for (int c = 0; c < classes; ++c) {
                const int after = x[c] < last_value || (x[c] == last_value && c > last_index);
                if (after && (best < 0 || x[c] > x[best])) {
                    best = c;
                }
            }
            const int64_t out = (int64_t)row * k + r;
            indices[out] = best;
            values[out] = best < 0 ? NAN : x[best];
            probabilities[out] = best < 0 ? 0.0 : exp((double)x[best] - maximum) / total;
            if (best >= 0) {
                last_value = x[best];
                last_index = best;
            }
        }
    }
}

/* Patch gather: src/kernels/normalization.cu:159-192, tests/reference/vit.hpp:67-87.
 * patches[b*P + p][ch*pp + r*patch + q] = images[b][ch][pr*patch + r][pc*patch + q]. */
void oracle_extract_patches(const float* images, float* patches, int batch, int channels,
                            int height, int width, int patch) {
    const int across = width / patch;
    const int per_image = (height / patch) * across;
    const int64_t row_length = (int64_t)channels * patch * patch;
    for (int image = 0; image < batch; ++image) {
        for (int p = 0; p < per_image; ++p) {
            const int pr = p / across;
            const int pc = p % across;
            for (int ch = 0; ch < channels; ++ch) {
                for (int r = 0; r < patch; ++r) {
                    for (int q = 0; q < patch; ++q) {
                        const int64_t dst = ((int64_t)image * per_image + p) * row_length +
                                            ((int64_t)ch * patch + r) * patch + q;
                        const int64_t src =
                            (((int64_t)image * channels + ch) * height + pr * patch + r) *
                                width +
                            pc * patch + q;
                        patches[dst] = images[src];
                    }
                }
            }
        }
    }
}

/* src/kernels/normalization.cu:148-154 */
void oracle_add(float* accumulator, const float* addend, int64_t count) {
    for (int64_t i = 0; i < count; ++i) {
        accumulator[i] += addend[i];
    }
}

/* src/kernels/normalization.cu:194-201 */
void oracle_add_broadcast(float* accumulator, const float* addend, int64_t count, int batch) {
    for (int64_t i = 0; i < count * batch; ++i) {
        accumulator[i] += addend[i % count];
    }
}

/* src/kernels/normalization.cu:203-212 */
void oracle_broadcast(float* destination, const float* source, int64_t count,
                      int64_t destination_stride, int batch) {
    for (int b = 0; b < batch; ++b) {
        for (int64_t i = 0; i < count; ++i) {
            destination[b * destination_stride + i] = source[i];
        }
    }
}

/* Attention of one image, all heads: tests/reference/vit.hpp:149-183.
 * qkv: [tokens, 3 * embed] packed [3][heads][head_dim]; context: [tokens, embed]. */
void oracle_attention(const float* qkv, float* context, int tokens, int embed, int heads) {
    const int head_dim = embed / heads;
    const int row = 3 * embed;
    const float scale = 1.0F / sqrtf((float)head_dim);
    float* const logits = (float*)malloc(sizeof(float) * (size_t)tokens * tokens);
    float* const weights = (float*)malloc(sizeof(float) * (size_t)tokens * tokens);
    for (int h = 0; h < heads; ++h) {
        for (int q = 0; q < tokens; ++q) {
            for (int key = 0; key < tokens; ++key) {
                float sum = 0.0F;
                for (int i = 0; i < head_dim; ++i) {
                    sum += qkv[(size_t)q * row + h * head_dim + i] *
                           qkv[(size_t)key * row + embed + h * head_dim + i];
                }
                logits[(size_t)q * tokens + key] = sum * scale;
            }
        }
        oracle_softmax(logits, weights, tokens, tokens, tokens);
        for (int q = 0; q < tokens; ++q) {
            for (int i = 0; i < head_dim; ++i) {
                float sum = 0.0F;
                for (int key = 0; key < tokens; ++key) {
                    sum += weights[(size_t)q * tokens + key] *
                           qkv[(size_t)key * row + 2 * embed + h * head_dim + i];
                }
                context[(size_t)q * embed + h * head_dim + i] = sum;
            }
        }
    }
    free(logits);
    free(weights);
}

/* config: image_size, patch_size, channels, embed_dim, depth, heads, mlp_hidden, classes */
typedef struct {
    int image_size, patch_size, channels, embed, depth, heads, hidden, classes;
} Config;

static void gemm_t(const float* a, const float* b, const float* bias, float* c, int m, int n,
                   int k) {
    oracle_gemm(a, b, bias, c, m, n, k, 1, 1.0F, k, k, n, 1, 0, 0, 0, 0, 0, 0, 0, 0, 0);
}

/*
 * One image through the whole model: tests/reference/vit.hpp:57-112 (forward) and
 * :149-205 (run_block). tensors[] holds the 4 + 12*depth + 4 tensors in the load order of
 * src/model/vit.cu:114-143. Returns 0, or -1 when scratch allocation fails.
 */
int oracle_vit_forward(const int* config_ints, float epsilon, const float* const* tensors,
                       const float* image, float* out_logits) {
    Config c;
    memcpy(&c, config_ints, sizeof(c));
    const int e = c.embed;
    const int across = c.image_size / c.patch_size;
    const int patch_count = across * across;
    const int tokens_n = patch_count + 1;
    const int patch_elements = c.channels * c.patch_size * c.patch_size;
    const size_t te = (size_t)tokens_n * e;

    float* const patches = (float*)malloc(sizeof(float) * (size_t)patch_count * patch_elements);
    float* const tokens = (float*)malloc(sizeof(float) * te);
    float* const normalized = (float*)malloc(sizeof(float) * te);
    float* const qkv = (float*)malloc(sizeof(float) * te * 3);
    float* const context = (float*)malloc(sizeof(float) * te);
    float* const projected = (float*)malloc(sizeof(float) * te);
    float* const hidden = (float*)malloc(sizeof(float) * (size_t)tokens_n * c.hidden);
    if (!patches || !tokens || !normalized || !qkv || !context || !projected || !hidden) {
        free(patches), free(tokens), free(normalized), free(qkv), free(context);
        free(projected), free(hidden);
        return -1;
    }

    const float* const cls = tensors[0];
    const float* const pos = tensors[1];
    oracle_extract_patches(image, patches, 1, c.channels, c.image_size, c.image_size,
                           c.patch_size);
    for (int i = 0; i < e; ++i) {
        tokens[i] = cls[i];
    }
    gemm_t(patches, tensors[2], tensors[3], tokens + e, patch_count, e, patch_elements);
    for (size_t i = 0; i < te; ++i) {
        tokens[i] += pos[i];
    }

    for (int blk = 0; blk < c.depth; ++blk) {
        const float* const* w = tensors + 4 + 12 * blk;
        oracle_layer_norm(tokens, e, w[0], w[1], normalized, e, tokens_n, e, epsilon);
        gemm_t(normalized, w[2], w[3], qkv, tokens_n, 3 * e, e);
        oracle_attention(qkv, context, tokens_n, e, c.heads);
        gemm_t(context, w[4], w[5], projected, tokens_n, e, e);
        for (size_t i = 0; i < te; ++i) {
            tokens[i] += projected[i];
        }
        oracle_layer_norm(tokens, e, w[6], w[7], normalized, e, tokens_n, e, epsilon);
        gemm_t(normalized, w[8], w[9], hidden, tokens_n, c.hidden, e);
        oracle_gelu_array(hidden, hidden, (int64_t)tokens_n * c.hidden);
        gemm_t(hidden, w[10], w[11], projected, tokens_n, e, c.hidden);
        for (size_t i = 0; i < te; ++i) {
            tokens[i] += projected[i];
        }
    }

    const float* const* tail = tensors + 4 + 12 * c.depth;
    oracle_layer_norm(tokens, e, tail[0], tail[1], normalized, e, tokens_n, e, epsilon);
    gemm_t(normalized, tail[2], tail[3], out_logits, 1, c.classes, e);

    free(patches), free(tokens), free(normalized), free(qkv), free(context);
    free(projected), free(hidden);
    return 0;
}

/* Many images spread over worker threads, one image at a time per thread. */
typedef struct {
    const int* config;
    float epsilon;
    const float* const* tensors;
    const float* images;
    float* logits;
    size_t per_image;
    int classes;
    int count;
    int next;
    int failures;
    pthread_mutex_t lock;
} BatchJob;

static void* batch_worker(void* argument) {
    BatchJob* const job = (BatchJob*)argument;
    while (1) {
        pthread_mutex_lock(&job->lock);
        const int index = job->next++;
        pthread_mutex_unlock(&job->lock);
        if (index >= job->count) {
            return NULL;
        }
        const int failed = oracle_vit_forward(job->config, job->epsilon, job->tensors,
                                              job->images + index * job->per_image,
                                              job->logits + (size_t)index * job->classes) != 0;
        if (failed) {
            pthread_mutex_lock(&job->lock);
            job->failures += 1;
            pthread_mutex_unlock(&job->lock);
        }
    }
}

/* Returns the number of images that failed. threads <= 0 uses every online core. */
int oracle_vit_forward_batch(const int* config_ints, float epsilon, const float* const* tensors,
                             const float* images, int count, float* logits, int threads) {
    Config c;
    memcpy(&c, config_ints, sizeof(c));
    BatchJob job;
    job.config = config_ints;
    job.epsilon = epsilon;
    job.tensors = tensors;
    job.images = images;
    job.logits = logits;
    job.per_image = (size_t)c.channels * c.image_size * c.image_size;
    job.classes = c.classes;
    job.count = count;
    job.next = 0;
    job.failures = 0;
    pthread_mutex_init(&job.lock, NULL);
    if (threads <= 0) {
        threads = (int)sysconf(_SC_NPROCESSORS_ONLN);
    }
    if (threads > count) {
        threads = count;
    }
    if (threads < 1) {
        threads = 1;
    }
    pthread_t* const pool = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
    int started = 0;
    for (int i = 0; pool != NULL && i < threads; ++i) {
        started += pthread_create(&pool[i], NULL, batch_worker, &job) == 0;
    }
    if (started == 0) {
        batch_worker(&job);
    }
    for (int i = 0; i < started; ++i) {
        pthread_join(pool[i], NULL);
    }
    free(pool);
    pthread_mutex_destroy(&job.lock);
    return job.failures;
}

int oracle_max_threads(void) { return (int)sysconf(_SC_NPROCESSORS_ONLN); }

/* Image preprocessing: src/runtime/image.cpp:90-135 (preprocess) with its bilinear sampler
 * image.cpp:39-56. The shorter side is resized to round(size / crop_fraction), the centre
 * size x size square is kept, and both steps fold into one sampling pass that maps each
 * output pixel back to a source coordinate; the sample is scaled to [0, 1] and normalised.
 * Interleaved 8-bit RGB in, planar float [3, size, size] out. Every float operation is kept in
 * the reference's order (no contraction). Returns 0, or -1 for arguments the reference
 * rejects (empty image, size <= 0, crop fraction outside (0, 1], zero deviation). */
static float oracle_pixel(const uint8_t* pixels, int width, int height, int column, int row,
                          int channel) {
    column = column < 0 ? 0 : (column > width - 1 ? width - 1 : column);
    row = row < 0 ? 0 : (row > height - 1 ? height - 1 : row);
    return (float)pixels[((size_t)row * (size_t)width + (size_t)column) * 3 + (size_t)channel];
}

static float oracle_bilinear(const uint8_t* pixels, int width, int height, float x, float y,
                             int channel) {
    const int left = (int)floorf(x);
    const int top = (int)floorf(y);
    const float dx = x - (float)left;
    const float dy = y - (float)top;
    const float top_edge = oracle_pixel(pixels, width, height, left, top, channel) * (1.0F - dx) +
                           oracle_pixel(pixels, width, height, left + 1, top, channel) * dx;
    const float bottom_edge =
        oracle_pixel(pixels, width, height, left, top + 1, channel) * (1.0F - dx) +
        oracle_pixel(pixels, width, height, left + 1, top + 1, channel) * dx;
    return top_edge * (1.0F - dy) + bottom_edge * dy;
}

int oracle_preprocess(const uint8_t* pixels, int width, int height, int size,
                      float crop_fraction, const float* mean, const float* stddev, float* out) {
    if (pixels == NULL || width <= 0 || height <= 0 || size <= 0 || !(crop_fraction > 0.0F) ||
        crop_fraction > 1.0F) {
        return -1;
    }
    for (int channel = 0; channel < 3; ++channel) {
        if (stddev[channel] == 0.0F) {
            return -1;
        }
    }
    const float resized = roundf((float)size / crop_fraction);
    const int shorter = width < height ? width : height;
    const float scale = (float)shorter / resized;
    const float crop = (float)size * scale;
    const float origin_x = ((float)width - crop) * 0.5F;
    const float origin_y = ((float)height - crop) * 0.5F;
    const float step = crop / (float)size;
    const size_t plane = (size_t)size * (size_t)size;
    for (int channel = 0; channel < 3; ++channel) {
        for (int row = 0; row < size; ++row) {
            for (int column = 0; column < size; ++column) {
                const float x = origin_x + ((float)column + 0.5F) * step - 0.5F;
                const float y = origin_y + ((float)row + 0.5F) * step - 0.5F;
                const float value = oracle_bilinear(pixels, width, height, x, y, channel) / 255.0F;
                out[(size_t)channel * plane + (size_t)row * (size_t)size + (size_t)column] =
                    (value - mean[channel]) / stddev[channel];
            }
        }
    }
    return 0;
}
