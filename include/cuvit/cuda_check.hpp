// cuvit/cuda_check.hpp -- the error type and check macro of Cu-Vit's operator API
// (reference: include/cuvit/cuda_check.hpp:11-36), so code written against the reference
// keeps compiling when it switches to this library.
#pragma once

#include <cuda_runtime_api.h>

#include <sstream>
#include <stdexcept>
#include <string>

namespace cuvit {

/// A failed CUDA runtime call, carrying its error code.
class CudaError final : public std::runtime_error {
  public:
    CudaError(cudaError_t code, const std::string& message)
        : std::runtime_error(message), code_(code) {}

    [[nodiscard]] cudaError_t code() const noexcept { return code_; }

  private:
    cudaError_t code_;
};

/// Throws CudaError naming the expression and location when result is not cudaSuccess.
inline void check_cuda(cudaError_t result, const char* expression, const char* file, int line) {
    if (result == cudaSuccess) {
        return;
    }
    std::ostringstream text;
    text << "CUDA call failed: " << expression << " at " << file << ':' << line << " ("
         << cudaGetErrorName(result) << ": " << cudaGetErrorString(result) << ')';
    throw CudaError(result, text.str());
}

} // namespace cuvit

#define CUVIT_CUDA_CHECK(expression) ::cuvit::check_cuda((expression), #expression, __FILE__, __LINE__)
