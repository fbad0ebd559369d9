// Common definitions for the B200 CSR SpMV library: status handling, launch
// bookkeeping and small device helpers shared by the kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <cstdio>
#include <cuda_runtime.h>

#include "../../include/prefree_b200.h"

namespace pf {

// Per-thread last-error text, returned by pf_last_error().
void set_error(const char *fmt, ...);

#define PF_CUDA_TRY(call)                                                      \
  do {                                                                         \
    cudaError_t e_ = (call);                                                   \
    if (e_ != cudaSuccess) {                                                   \
      ::pf::set_error("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_),  \
                      __FILE__, __LINE__);                                     \
      return PF_ERR_CUDA;                                                      \
    }                                                                          \
  } while (0)

#define PF_CHECK_ARG(cond, ...)                                                \
  do {                                                                         \
    if (!(cond)) {                                                             \
      ::pf::set_error(__VA_ARGS__);                                            \
      return PF_ERR_INVALID;                                                   \
    }                                                                          \
  } while (0)

// Device-side error bits (written into the handle's error word; never trap).
enum : unsigned {
  PF_DEVERR_WAIT_TIMEOUT = 1u << 0,   // a bounded mbarrier/flag wait gave up
  PF_DEVERR_BOUNDS = 1u << 1,         // a row_ptr/col index outside its range
  PF_DEVERR_ROWPTR = 1u << 2,         // row_ptr not non-decreasing
};

// Count of our kernels launched since library load (bench reports it).
// a 16-bit value from its bit pattern
template <typename H>
__device__ __forceinline__ H half_from_bits(unsigned short b);
template <>
__device__ __forceinline__ __half half_from_bits<__half>(unsigned short b) {
  return __ushort_as_half(b);
}
template <>
__device__ __forceinline__ __nv_bfloat16 half_from_bits<__nv_bfloat16>(unsigned short b) {
  return __ushort_as_bfloat16(b);
}

extern unsigned long long g_launch_count;
// spmv_api.cu: the one-time work of the first multiply with a matrix
pf_status prepare_matrix_i32(pf_handle h, int64_t m, int64_t nnz, const int32_t *row_ptr,
                             cudaStream_t st);
pf_status prepare_matrix_i64(pf_handle h, int64_t m, int64_t nnz, const int64_t *row_ptr,
                             cudaStream_t st);
void count_launches(unsigned long long k);

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) {
  return (a + b - 1) / b;
}

}  // namespace pf
