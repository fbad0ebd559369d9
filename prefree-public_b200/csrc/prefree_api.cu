// preFreeSpMV drop-in: the reference's host driver contract
// (src/spmv_kernel/preFreeSpMV.cu:563-662) on top of the device-pointer core.
//
// Sequence, as in the reference: allocate device arrays, copy CSR + x in,
// run the pre-pass (here: the variant choice from sampled row lengths, wall
// time into *cdPre, once per call), 200 warm-up + 4000 timed launches on the
// legacy default stream timed with events (*cdTime = ms per launch), one clean
// multiply, copy y out, free. Unlike the reference, every launch of the timed
// loop computes the same correct y (alpha = 1, beta = 0 overwrites y), failures
// are returned instead of exit(), and row_ptr is read for rowA+1 entries.
#include <chrono>
#include <cstdlib>
#include <cstdio>

#include "../../include/PreFree.h"
#include "pf_common.cuh"

namespace pf {

static int env_int(const char *name, int dflt) {
  const char *v = std::getenv(name);
  if (!v || !*v) return dflt;
  const int x = std::atoi(v);
  return x >= 0 ? x : dflt;
}

template <typename VT, typename IT>
static pf_status spmv_dispatch(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                               const IT *rp, const int32_t *col, const VT *val,
                               const VT *x, VT *y);

template <>
pf_status spmv_dispatch<double, int32_t>(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                                         const int32_t *rp, const int32_t *col,
                                         const double *val, const double *x, double *y) {
  return pf_spmv_f64_i32(h, m, n, nnz, rp, col, val, 1.0, x, 0.0, y, nullptr);
}
template <>
pf_status spmv_dispatch<double, int64_t>(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                                         const int64_t *rp, const int32_t *col,
                                         const double *val, const double *x, double *y) {
  return pf_spmv_f64_i64(h, m, n, nnz, rp, col, val, 1.0, x, 0.0, y, nullptr);
}
template <>
pf_status spmv_dispatch<float, int32_t>(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                                        const int32_t *rp, const int32_t *col,
                                        const float *val, const float *x, float *y) {
  return pf_spmv_f32_i32(h, m, n, nnz, rp, col, val, 1.0, x, 0.0, y, nullptr);
}

template <typename VT, typename IT>
static pf_status prefree_impl(VT *csrVal, IT *csrRowPtr, int32_t *csrColInd,
                              VT *X_val, VT *Y_val, int64_t m, int64_t n,
                              int64_t nnz, double *cdTime, double *cdPre) {
  PF_CHECK_ARG(cdTime && cdPre, "null timing outputs");
  *cdTime = -1.0;
  *cdPre = -1.0;
  PF_CHECK_ARG(m >= 0 && n >= 0 && nnz >= 0, "negative size");
  PF_CHECK_ARG(m == 0 || (csrRowPtr && Y_val), "null row_ptr / Y");
  PF_CHECK_ARG(nnz == 0 || (csrVal && csrColInd && X_val), "null val/col/X");
  if (m > 0) {
    PF_CHECK_ARG((int64_t)csrRowPtr[0] == 0 && (int64_t)csrRowPtr[m] == nnz,
                 "row_ptr[0] must be 0 and row_ptr[rowA] == nnzA");
  }
  const int warm = env_int("PF_PREFREE_WARMUP", 200);
  const int iters = std::max(1, env_int("PF_PREFREE_ITERS", 4000));

  pf_handle h = nullptr;
  pf_status st = pf_handle_create(&h);
  if (st != PF_OK) return st;
  IT *d_rp = nullptr;
  int32_t *d_col = nullptr;
  VT *d_val = nullptr, *d_x = nullptr, *d_yp = nullptr, *d_y = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  auto cleanup = [&]() {
    cudaFree(d_rp);
    cudaFree(d_col);
    cudaFree(d_val);
    cudaFree(d_x);
    cudaFree(d_yp);
    cudaFree(d_y);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    pf_handle_destroy(h);
  };
#define PF_TRY_CLEAN(call)                                                     \
  do {                                                                         \
    cudaError_t e_ = (call);                                                   \
    if (e_ != cudaSuccess) {                                                   \
      set_error("preFreeSpMV: %s: %s", #call, cudaGetErrorString(e_));         \
      cleanup();                                                               \
      return PF_ERR_CUDA;                                                      \
    }                                                                          \
  } while (0)
  const size_t ms = std::max<int64_t>(m, 1), ns = std::max<int64_t>(n, 1),
               zs = std::max<int64_t>(nnz, 1);
  PF_TRY_CLEAN(cudaMalloc(&d_rp, sizeof(IT) * (ms + 1)));
  PF_TRY_CLEAN(cudaMalloc(&d_col, sizeof(int32_t) * zs));
  PF_TRY_CLEAN(cudaMalloc(&d_val, sizeof(VT) * zs));
  PF_TRY_CLEAN(cudaMalloc(&d_x, sizeof(VT) * ns));
  PF_TRY_CLEAN(cudaMalloc(&d_yp, sizeof(VT) * ms));
  PF_TRY_CLEAN(cudaMalloc(&d_y, sizeof(VT) * ms));
  if (m > 0) PF_TRY_CLEAN(cudaMemcpy(d_rp, csrRowPtr, sizeof(IT) * (m + 1), cudaMemcpyHostToDevice));
  if (nnz > 0) {
    PF_TRY_CLEAN(cudaMemcpy(d_col, csrColInd, sizeof(int32_t) * nnz, cudaMemcpyHostToDevice));
    PF_TRY_CLEAN(cudaMemcpy(d_val, csrVal, sizeof(VT) * nnz, cudaMemcpyHostToDevice));
  }
  if (n > 0) PF_TRY_CLEAN(cudaMemcpy(d_x, X_val, sizeof(VT) * n, cudaMemcpyHostToDevice));

  // pre-pass: variant choice from sampled row lengths
  PF_TRY_CLEAN(cudaDeviceSynchronize());
  const auto t0 = std::chrono::steady_clock::now();
  pf_handle_set_variant(h, PF_VARIANT_AUTO);
  if (sizeof(IT) == 8)
    st = prepare_matrix_i64(h, m, nnz, reinterpret_cast<const int64_t *>(d_rp), nullptr);
  else
    st = prepare_matrix_i32(h, m, nnz, reinterpret_cast<const int32_t *>(d_rp), nullptr);
  if (st != PF_OK) { cleanup(); return st; }
  const auto t1 = std::chrono::steady_clock::now();
  *cdPre = std::chrono::duration<double, std::milli>(t1 - t0).count();

  for (int i = 0; i < warm; ++i) {
    st = spmv_dispatch<VT, IT>(h, m, n, nnz, d_rp, d_col, d_val, d_x, d_yp);
    if (st != PF_OK) { cleanup(); return st; }
  }
  PF_TRY_CLEAN(cudaDeviceSynchronize());
  PF_TRY_CLEAN(cudaEventCreate(&e0));
  PF_TRY_CLEAN(cudaEventCreate(&e1));
  PF_TRY_CLEAN(cudaEventRecord(e0, 0));
  for (int i = 0; i < iters; ++i) {
    st = spmv_dispatch<VT, IT>(h, m, n, nnz, d_rp, d_col, d_val, d_x, d_yp);
    if (st != PF_OK) { cleanup(); return st; }
  }
  PF_TRY_CLEAN(cudaEventRecord(e1, 0));
  PF_TRY_CLEAN(cudaEventSynchronize(e1));
  float total_ms = 0.f;
  PF_TRY_CLEAN(cudaEventElapsedTime(&total_ms, e0, e1));

  st = spmv_dispatch<VT, IT>(h, m, n, nnz, d_rp, d_col, d_val, d_x, d_y);
  if (st != PF_OK) { cleanup(); return st; }
  PF_TRY_CLEAN(cudaDeviceSynchronize());
  uint32_t bits = 0;
  st = pf_handle_device_error(h, &bits, 1);
  if (st != PF_OK) { cleanup(); return st; }
  if (bits) {
    set_error("preFreeSpMV: kernel reported device error bits 0x%x", bits);
    cleanup();
    return PF_ERR_DEVICE;
  }
  if (m > 0) PF_TRY_CLEAN(cudaMemcpy(Y_val, d_y, sizeof(VT) * m, cudaMemcpyDeviceToHost));
  *cdTime = (double)total_ms / iters;
#undef PF_TRY_CLEAN
  cleanup();
  return PF_OK;
}

template <typename VT, typename IT>
static void prefree_cxx(VT *v, IT *rp, int *c, VT *x, VT *y, int64_t m, int64_t n,
                        int64_t z, double *t, double *p) {
  const pf_status st = prefree_impl<VT, IT>(v, rp, c, x, y, m, n, z, t, p);
  if (st != PF_OK) std::fprintf(stderr, "preFreeSpMV failed: %s\n", pf_last_error());
}

}  // namespace pf

// ---- C++ entry points (include/PreFree.h) ------------------------------------
void preFreeSpMV(double *csrVal, int *csrRowPtr, int *csrColInd, double *X_val,
                 double *Y_val, int rowA, int colA, int nnzA, double *cdTime,
                 double *cdPre) {
  pf::prefree_cxx<double, int32_t>(csrVal, csrRowPtr, csrColInd, X_val, Y_val, rowA,
                                   colA, nnzA, cdTime, cdPre);
}

void preFreeSpMV(float *csrVal, int *csrRowPtr, int *csrColInd, float *X_val,
                 float *Y_val, int rowA, int colA, int nnzA, double *cdTime,
                 double *cdPre) {
  pf::prefree_cxx<float, int32_t>(csrVal, csrRowPtr, csrColInd, X_val, Y_val, rowA,
                                  colA, nnzA, cdTime, cdPre);
}

void preFreeSpMV(double *csrVal, int64_t *csrRowPtr, int *csrColInd, double *X_val,
                 double *Y_val, int64_t rowA, int64_t colA, int64_t nnzA,
                 double *cdTime, double *cdPre) {
  pf::prefree_cxx<double, int64_t>(csrVal, csrRowPtr, csrColInd, X_val, Y_val, rowA,
                                   colA, nnzA, cdTime, cdPre);
}

// ---- C linkage (FFI) -----------------------------------------------------------
extern "C" {

pf_status pf_prefree_spmv_f64_i32(double *csrVal, int32_t *csrRowPtr, int32_t *csrColInd,
                                  double *X_val, double *Y_val, int32_t rowA,
                                  int32_t colA, int32_t nnzA, double *cdTime,
                                  double *cdPre) {
  return pf::prefree_impl<double, int32_t>(csrVal, csrRowPtr, csrColInd, X_val, Y_val,
                                           rowA, colA, nnzA, cdTime, cdPre);
}

pf_status pf_prefree_spmv_f64_i64(double *csrVal, int64_t *csrRowPtr, int32_t *csrColInd,
                                  double *X_val, double *Y_val, int64_t rowA,
                                  int64_t colA, int64_t nnzA, double *cdTime,
                                  double *cdPre) {
  return pf::prefree_impl<double, int64_t>(csrVal, csrRowPtr, csrColInd, X_val, Y_val,
                                           rowA, colA, nnzA, cdTime, cdPre);
}

pf_status pf_prefree_spmv_f32_i32(float *csrVal, int32_t *csrRowPtr, int32_t *csrColInd,
                                  float *X_val, float *Y_val, int32_t rowA,
                                  int32_t colA, int32_t nnzA, double *cdTime,
                                  double *cdPre) {
  return pf::prefree_impl<float, int32_t>(csrVal, csrRowPtr, csrColInd, X_val, Y_val,
                                          rowA, colA, nnzA, cdTime, cdPre);
}

}  // extern "C"
