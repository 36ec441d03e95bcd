// TEST INFRASTRUCTURE ONLY. A C ABI over the reference's own FP32 GPU path (src/kernels/
// gemm.cu, src/kernels/normalization.cu, src/model/vit.cu of Cu-Vit), compiled from the
// reference sources in place for sm_100a by oracle/Makefile into
// oracle/_ref/libcuvit_ref_gpu.so. It is the "repo's FP32 GPU path" the TF32 results are
// compared with; it never runs on the product path.
#include "cuvit/kernels.hpp"
#include "cuvit/vit.hpp"
#include "cuvit/weights.hpp"

#include <exception>

#define REF_API extern "C" __attribute__((visibility("default")))

REF_API int ref_gpu_gemm(const float* a, const float* b, const float* bias, float* c, int m,
                         int n, int k, int transposed, float alpha, int accumulate, int gelu) {
    try {
        cuvit::GemmProblem problem = cuvit::gemm_problem(
            m, n, k, transposed ? cuvit::GemmLayout::kTransposed : cuvit::GemmLayout::kNoTranspose);
        problem.alpha = alpha;
        problem.epilogue.accumulate = accumulate != 0;
        problem.epilogue.gelu = gelu != 0;
        cuvit::launch_gemm(a, b, bias, c, problem);
        return cudaDeviceSynchronize() == cudaSuccess ? 0 : -1;
    } catch (const std::exception&) {
        return -1;
    }
}

// The same launch without the synchronisation, on `stream` (so a caller can time it with
// events or capture it in a CUDA graph). Returns 0, or -1 when the reference throws.
REF_API int ref_gpu_gemm_async(const float* a, const float* b, const float* bias, float* c,
                               int m, int n, int k, int transposed, float alpha, int accumulate,
                               int gelu, void* stream) {
    try {
        cuvit::GemmProblem problem = cuvit::gemm_problem(
            m, n, k, transposed ? cuvit::GemmLayout::kTransposed : cuvit::GemmLayout::kNoTranspose);
        problem.alpha = alpha;
        problem.epilogue.accumulate = accumulate != 0;
        problem.epilogue.gelu = gelu != 0;
        cuvit::launch_gemm(a, b, bias, c, problem, static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

REF_API void* ref_gpu_vit_create(const char* weights_path, const int* c, float epsilon,
                                 int max_batch) {
    try {
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
        const cuvit::WeightFile file = cuvit::WeightFile::load(weights_path);
        return new cuvit::VisionTransformer(config, file, max_batch);
    } catch (const std::exception&) {
        return nullptr;
    }
}

// images/logits are device pointers; runs on the given stream.
REF_API int ref_gpu_vit_forward(void* model, const float* images, float* logits, int batch,
                                void* stream) {
    try {
        static_cast<cuvit::VisionTransformer*>(model)->forward(
            images, logits, batch, static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception&) {
        return -1;
    }
}

REF_API void ref_gpu_vit_destroy(void* model) {
    delete static_cast<cuvit::VisionTransformer*>(model);
}
