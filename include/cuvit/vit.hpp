// The reference's model-runner API (include/cuvit/vit.hpp of Cu-Vit: VitConfig and
// VisionTransformer) as inline wrappers of libcuvit_b200's C ABI, so code written against the
// reference's VisionTransformer builds unchanged against this library. The model runs in the
// FP32-faithful mode (CUVIT_MATH_FP32), the reference's arithmetic; weights come from the host
// project's WeightFile (the reference's include/cuvit/weights.hpp, src/runtime/weights.cpp),
// whose shape checks throw as they do in the reference. Errors map to the reference's
// exception types: std::invalid_argument for arguments and configurations, cuvit::CudaError
// for CUDA failures, std::runtime_error otherwise.
#pragma once

#include "cuvit/kernels.hpp"
#include "cuvit/weights.hpp"
#include "cuvit_b200.h"

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace cuvit {

/// Shape of a Vision Transformer. The defaults describe ViT-Tiny/16 at 224x224
/// (reference: include/cuvit/vit.hpp:14-35).
struct VitConfig {
    int image_size = 224;
    int patch_size = 16;
    int channels = 3;
    int embed_dim = 192;
    int depth = 12;
    int heads = 3;
    int mlp_hidden = 768;
    int classes = 1000;
    float layer_norm_epsilon = 1.0e-6F;

    [[nodiscard]] int patches_per_side() const { return image_size / patch_size; }
    [[nodiscard]] int patch_count() const { return patches_per_side() * patches_per_side(); }
    [[nodiscard]] int token_count() const { return patch_count() + 1; }
    [[nodiscard]] int head_dim() const { return embed_dim / heads; }
    [[nodiscard]] int patch_elements() const { return channels * patch_size * patch_size; }

    /// Throws std::invalid_argument naming the field when the configuration cannot describe
    /// a model (reference: src/model/vit.cu:36-47).
    void validate() const {
        const cuvit_vit_config c = to_c();
        detail::raise_on(cuvit_vit_config_validate(&c));
    }

    [[nodiscard]] cuvit_vit_config to_c() const {
        cuvit_vit_config c{};
        c.image_size = image_size;
        c.patch_size = patch_size;
        c.channels = channels;
        c.embed_dim = embed_dim;
        c.depth = depth;
        c.heads = heads;
        c.mlp_hidden = mlp_hidden;
        c.classes = classes;
        c.layer_norm_epsilon = layer_norm_epsilon;
        return c;
    }
};

/// A ViT ready to run: weights uploaded, activations reserved for max_batch images at
/// construction, no allocation per forward pass (reference: include/cuvit/vit.hpp:49-96).
class VisionTransformer final {
  public:
    VisionTransformer(const VitConfig& config, const WeightFile& file, int max_batch = 1)
        : config_(config), max_batch_(max_batch) {
        config_.validate();
        if (max_batch < 1) {
            throw std::invalid_argument("The maximum batch size must be at least one");
        }
        const cuvit_vit_config c = config_.to_c();
        const int count = cuvit_vit_tensor_count(&c);
        std::vector<const float*> tensors(static_cast<std::size_t>(count));
        for (int index = 0; index < count; ++index) {
            char name[128];
            std::int64_t extents[4];
            int rank = 0;
            detail::raise_on(cuvit_vit_tensor_info(&c, index, name, sizeof(name), extents, &rank));
            std::vector<Extent> expected(extents, extents + rank);
            // The WeightFile checks presence and shape and throws as in the reference.
            tensors[static_cast<std::size_t>(index)] = file.float_data(name, expected);
        }
        int device = 0;
        detail::raise_on(cudaGetDevice(&device) == cudaSuccess ? CUVIT_OK : CUVIT_CUDA_ERROR);
        detail::raise_on(cuvit_vit_create_from_host(&c, tensors.data(), count, max_batch,
                                                     CUVIT_MATH_FP32, device, &model_));
    }

    ~VisionTransformer() { cuvit_vit_destroy(model_); }
    VisionTransformer(const VisionTransformer&) = delete;
    VisionTransformer& operator=(const VisionTransformer&) = delete;
    VisionTransformer(VisionTransformer&& other) noexcept
        : config_(other.config_), max_batch_(other.max_batch_),
          model_(std::exchange(other.model_, nullptr)) {}
    VisionTransformer& operator=(VisionTransformer&& other) noexcept {
        if (this != &other) {
            cuvit_vit_destroy(model_);
            config_ = other.config_;
            max_batch_ = other.max_batch_;
            model_ = std::exchange(other.model_, nullptr);
        }
        return *this;
    }

    /// batch planar [channels, height, width] images in device memory -> batch x classes
    /// logits in device memory, queued on stream.
    void forward(const float* images, float* logits, int batch, cudaStream_t stream = nullptr) {
        detail::raise_on(
            cuvit_vit_forward(model_, images, logits, batch, detail::stream_of(stream)));
    }

    /// Host images in, host logits out, synchronised; the batch is the input size over one
    /// image's elements.
    [[nodiscard]] std::vector<float> forward(const std::vector<float>& images) {
        const std::size_t per_image = image_elements();
        if (per_image == 0 || images.size() % per_image != 0) {
            throw std::invalid_argument(
                "The input is not a whole number of images");
        }
        const std::size_t batch = images.size() / per_image;
        if (batch > static_cast<std::size_t>(max_batch_)) {
            throw std::invalid_argument("This model was built for at most " +
                                        std::to_string(max_batch_) + " images, but " +
                                        std::to_string(batch) + " were given");
        }
        std::vector<float> logits(batch * static_cast<std::size_t>(config_.classes));
        if (batch == 0) {
            return logits;
        }
        detail::raise_on(cuvit_vit_forward_host(model_, images.data(), logits.data(),
                                                static_cast<int>(batch), nullptr));
        return logits;
    }

    [[nodiscard]] const VitConfig& config() const noexcept { return config_; }
    [[nodiscard]] int max_batch() const noexcept { return max_batch_; }
    [[nodiscard]] std::size_t image_elements() const noexcept {
        return static_cast<std::size_t>(cuvit_vit_image_elements(model_));
    }
    [[nodiscard]] std::size_t weight_bytes() const noexcept {
        return static_cast<std::size_t>(cuvit_vit_weight_bytes(model_));
    }
    [[nodiscard]] std::size_t activation_bytes() const noexcept {
        return static_cast<std::size_t>(cuvit_vit_activation_bytes(model_));
    }

    /// The timm tensor names this configuration expects, in load order.
    [[nodiscard]] static std::vector<std::string> expected_tensor_names(const VitConfig& config) {
        const cuvit_vit_config c = config.to_c();
        const int count = cuvit_vit_tensor_count(&c);
        std::vector<std::string> names;
        names.reserve(static_cast<std::size_t>(count > 0 ? count : 0));
        for (int index = 0; index < count; ++index) {
            char name[128];
            std::int64_t extents[4];
            int rank = 0;
            detail::raise_on(cuvit_vit_tensor_info(&c, index, name, sizeof(name), extents, &rank));
            names.emplace_back(name);
        }
        return names;
    }

  private:
    VitConfig config_;
    int max_batch_ = 1;
    cuvit_vit* model_ = nullptr;
};

} // namespace cuvit
