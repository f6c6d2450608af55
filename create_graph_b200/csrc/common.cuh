// Shared helpers of the sm_100a library: error reporting through the C ABI,
// launch checks and small device utilities.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

namespace cg {

// Last error message of the calling host thread (read through cg_last_error()).
void set_error(const char* fmt, ...);

// Codes returned by every entry point.
enum Status : int {
  kOk = 0,
  kBadArgument = 1,
  kCudaError = 2,
  kUnsupported = 3,
};

#define CG_REQUIRE(cond, ...)                 \
  do {                                        \
    if (!(cond)) {                            \
      ::cg::set_error(__VA_ARGS__);           \
      return ::cg::kBadArgument;              \
    }                                         \
  } while (0)

#define CG_CUDA(call)                                                            \
  do {                                                                           \
    cudaError_t err_ = (call);                                                   \
    if (err_ != cudaSuccess) {                                                   \
      ::cg::set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(err_),  \
                      __FILE__, __LINE__);                                       \
      return ::cg::kCudaError;                                                   \
    }                                                                            \
  } while (0)

// Kernels launched by this library (host-side count, all threads).
void note_launch();

#define CG_LAUNCHED(name)                                                                 \
  do {                                                                                    \
    ::cg::note_launch();                                                                  \
    cudaError_t err_ = cudaGetLastError();                                                \
    if (err_ != cudaSuccess) {                                                            \
      ::cg::set_error("launch of %s failed: %s", name, cudaGetErrorString(err_));         \
      return ::cg::kCudaError;                                                            \
    }                                                                                     \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Number of SMs of the current device (cached per device).
int sm_count();

template <typename T>
__host__ __device__ inline T ceil_div(T a, T b) { return (a + b - 1) / b; }

namespace seg {
// Row chunking of the two-pass column reductions (segment.cu): `chunks`
// partial rows of `cols` floats each.
void colsum_plan(int64_t rows, int64_t cols, int64_t* chunks, int64_t* rows_per);
// 16-byte column sums (b null) or column dot products of contiguous (rows, cols)
// matrices into partial[chunk, c]; false (nothing launched) when not 16-byte aligned
bool colsum4_launch(const float* a, const float* b, int64_t rows, int64_t cols, int64_t chunks, int64_t rows_per,
                    float* partial, cudaStream_t s);
// CSR of element -> row index[e] (rows outside [0, rows) skipped): row_ptr
// (rows + 1) and perm (n: each row's elements ascending, then -1), any size,
// deterministic (segment.cu).
int csr_build_launch(const int32_t* index, int64_t n, int64_t rows, int32_t* row_ptr, int32_t* perm,
                     cudaStream_t s);
}  // namespace seg

}  // namespace cg
