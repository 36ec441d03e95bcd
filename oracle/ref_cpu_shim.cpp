// TEST INFRASTRUCTURE ONLY. A C ABI over the reference's own CPU implementation
// (tests/reference/linear_algebra.hpp, tests/reference/vit.hpp, src/runtime/weights.cpp of
// Cu-Vit), compiled from the reference sources in place by oracle/Makefile into
// oracle/_ref/libcuvit_ref_cpu.so. It validates the C restatement in cuvit_oracle.c and
// serves as the timed CPU baseline ("reference" kind).
#include "cuvit/image.hpp"
#include "cuvit/vit.hpp"
#include "cuvit/weights.hpp"
#include "reference/linear_algebra.hpp"
#include "reference/vit.hpp"

#include <atomic>
#include <cstdint>
#include <exception>
#include <thread>
#include <vector>

namespace {

cuvit::VitConfig make_config(const int* c, float epsilon) {
    cuvit::VitConfig config;
    config.image_size = c[0];
    config.patch_size = c[1];
    config.channels = c[2];
    config.embed_dim = c[3];
    config.depth = c[4];
    config.heads = c[5];
    config.mlp_hidden = c[6];
    config.classes = c[7];
    config.layer_norm_epsilon = epsilon;
    return config;
}

} // namespace

extern "C" {

__attribute__((visibility("default"))) void ref_gemm(const float* a, const float* b,
                                                     const float* bias, float* c, int m, int n,
                                                     int k, int transposed, float alpha) {
    if (transposed) {
        cuvit::reference::gemm_transposed(a, b, bias, c, m, n, k, alpha);
    } else {
        cuvit::reference::gemm(a, b, bias, c, m, n, k, alpha);
    }
}

__attribute__((visibility("default"))) void ref_gemm_term_magnitudes(const float* a,
                                                                     const float* b,
                                                                     float* scale, int m, int n,
                                                                     int k, int transposed,
                                                                     float alpha) {
    const std::vector<float> values =
        cuvit::reference::gemm_term_magnitudes(a, b, m, n, k, transposed != 0, alpha);
    for (size_t i = 0; i < values.size(); ++i) {
        scale[i] = values[i];
    }
}

__attribute__((visibility("default"))) void ref_layer_norm(const float* input,
                                                           const float* gamma,
                                                           const float* beta, float* output,
                                                           int rows, int columns,
                                                           float epsilon) {
    cuvit::reference::layer_norm(input, gamma, beta, output, rows, columns, epsilon);
}

__attribute__((visibility("default"))) void ref_softmax(const float* input, float* output,
                                                        int rows, int columns) {
    cuvit::reference::softmax(input, output, rows, columns);
}

__attribute__((visibility("default"))) void ref_gelu(const float* input, float* output,
                                                     int64_t count) {
    cuvit::reference::gelu(input, output, static_cast<size_t>(count));
}

// cuvit::preprocess (src/runtime/image.cpp:90-135) of one interleaved 8-bit RGB image into a
// planar [3, size, size] tensor. Returns 0, or -1 when the reference throws.
__attribute__((visibility("default"))) int ref_preprocess(const uint8_t* pixels, int width,
                                                          int height, int size,
                                                          float crop_fraction,
                                                          const float* mean,
                                                          const float* stddev, float* out) {
    try {
        cuvit::RgbImage image;
        image.width = width;
        image.height = height;
        image.pixels.assign(pixels, pixels + static_cast<size_t>(width) * height * 3);
        cuvit::Preprocessing settings;
        settings.size = size;
        settings.crop_fraction = crop_fraction;
        for (int c = 0; c < 3; ++c) {
            settings.mean[static_cast<size_t>(c)] = mean[c];
            settings.stddev[static_cast<size_t>(c)] = stddev[c];
        }
        const std::vector<float> tensor = cuvit::preprocess(image, settings);
        for (size_t i = 0; i < tensor.size(); ++i) {
            out[i] = tensor[i];
        }
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

// Runs VitReference::forward over count images with `threads` worker threads, loading the
// weights from a .cvw file. Returns 0, or -1 on any exception.
__attribute__((visibility("default"))) int ref_vit_forward(const char* weights_path,
                                                           const int* config_ints,
                                                           float epsilon, const float* images,
                                                           int count, float* logits,
                                                           int threads) {
    try {
        const cuvit::VitConfig config = make_config(config_ints, epsilon);
        const cuvit::WeightFile file = cuvit::WeightFile::load(weights_path);
        const cuvit::reference::VitReference model(config, file);
        const size_t per_image =
            static_cast<size_t>(config.channels) * config.image_size * config.image_size;
        std::atomic<int> next{0};
        std::atomic<int> failures{0};
        const auto worker = [&]() {
            while (true) {
                const int index = next.fetch_add(1);
                if (index >= count) {
                    return;
                }
                try {
                    const std::vector<float> image(images + index * per_image,
                                                   images + (index + 1) * per_image);
                    const std::vector<float> out = model.forward(image);
                    for (size_t j = 0; j < out.size(); ++j) {
                        logits[static_cast<size_t>(index) * config.classes + j] = out[j];
                    }
                } catch (const std::exception&) {
                    failures.fetch_add(1);
                }
            }
        };
        const int workers = threads > 0 ? threads : 1;
        std::vector<std::thread> pool;
        for (int i = 0; i < workers; ++i) {
            pool.emplace_back(worker);
        }
        for (std::thread& t : pool) {
            t.join();
        }
        return failures.load() == 0 ? 0 : -1;
    } catch (const std::exception&) {
        return -1;
    }
}

} // extern "C"
