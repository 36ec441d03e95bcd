// Memory-bound operators the model runner calls directly (no C-ABI counterpart).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace cuvit::ops {

// Whether extract_patches_bf16 takes this image geometry (whole patches, patch and width
// multiples of 4).
bool bf16_patch_gather_supported(int height, int width, int patch);

// The patch gather of cuvit_extract_patches_ex for images already rounded to bfloat16
// (planar [batch, channels, height, width]) into bfloat16 patches: the same values the
// FP32-input gather writes for the same images rounded to nearest even.
int extract_patches_bf16(const __nv_bfloat16* images, __nv_bfloat16* patches, int batch,
                         int channels, int height, int width, int patch, cudaStream_t stream);

} // namespace cuvit::ops
