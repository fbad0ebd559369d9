// SpMM: Y = alpha * A * X + beta * Y for a CSR A and KC dense columns per
// pass (X n x k and Y m x k row-major, leading dimensions ldx and ldy).
//
// The ROWVEC layout of the multiply: V lanes per row, each lane covering
// 16-byte-aligned blocks of 4 non-zeros (one 16-byte column load, the value
// pieces holding an element of the row), then for every non-zero the KC
// values X[col][j0 .. j0 + KC) of this pass. A is read once per pass of KC
// columns, so each non-zero's bytes and the line fill of its gather serve KC
// products. The V lanes of a row reduce their KC sums with shuffles; lane
// (j mod V) of the row group stores column j, so the row's KC outputs leave
// together.
//
// Sums are in double (the serial loop's order within a lane, fixed shuffle
// order across lanes); the same bits on every run.
#pragma once

#include "pf_common.cuh"
#include "spmv_nnzsplit.cuh"
#include "spmv_rowvec.cuh"

namespace pf {

template <typename VT, typename IT>
struct SpmmParams {
  int64_t m, n, nnz;
  const IT *__restrict__ row_ptr;
  const int32_t *__restrict__ col;
  const VT *__restrict__ val;
  const VT *__restrict__ X;  // column j0 of this pass at X[r * ldx]
  VT *__restrict__ Y;        // column j0 of this pass at Y[r * ldy]
  int64_t ldx, ldy;
  int kc;                    // columns in this pass (<= KC)
  int64_t ldx_left;          // elements of an X row from column j0 on (host use)
  double alpha, beta;
  unsigned *err;
};

// KC values of an X row: 16-byte loads when the row starts on a 16-byte
// boundary (VX), single elements otherwise; every load asks L2 for a 64-byte
// fill, so a random row gather does not drag in the neighbouring row
template <typename VT, int KC, bool VX>
struct XRow {
  __device__ __forceinline__ static void load(const VT *xr, int kc, double out[KC]) {
#pragma unroll
    for (int j = 0; j < KC; ++j) out[j] = j < kc ? (double)ptx::ldg_x(xr + j) : 0.0;
  }
};
template <int KC>
struct XRow<double, KC, true> {
  __device__ __forceinline__ static void load(const double *xr, int kc, double out[KC]) {
#pragma unroll
    for (int j = 0; j < KC; j += 2) {
      double2 t = make_double2(0.0, 0.0);
      if (j < kc) t = ptx::ldg_x_v2(reinterpret_cast<const double2 *>(xr + j));
      out[j] = t.x;
      if (j + 1 < KC) out[j + 1] = t.y;
    }
  }
};
template <int KC>
struct XRow<float, KC, true> {
  __device__ __forceinline__ static void load(const float *xr, int kc, double out[KC]) {
#pragma unroll
    for (int j = 0; j < KC; j += 4) {
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      if (j < kc) t = ptx::ldg_x_v4(reinterpret_cast<const float4 *>(xr + j));
      const float v[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (j + i < KC) out[j + i] = v[i];
    }
  }
};

// VEC: col and val start on 16-byte boundaries (16-byte block loads);
// otherwise each lane loads single elements s + lig, s + lig + V, ...
// VX: every row of X starts on a 16-byte boundary and holds a whole number
// of 16-byte pieces of the pass's columns (loads past column kc read padding
// of the row or the next column, never past the row's ldx elements).
template <typename VT, typename IT, int V, int KC, int NTB, bool VEC, bool VX>
__global__ void __launch_bounds__(NTB)
spmm_rowvec_kernel(const SpmmParams<VT, IT> P) {
  constexpr int GPW = 32 / V;  // row groups per warp
  const int lane = threadIdx.x & 31;
  const int lig = lane & (V - 1);
  const int gw = lane / V;
  const int64_t warp_global = ((int64_t)blockIdx.x * NTB + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * NTB) >> 5;
  const uint32_t n = (uint32_t)(P.n < 0xffffffffLL ? P.n : 0xffffffffLL);
  const int kc = P.kc;
  bool bad = false;
  for (int64_t rb = warp_global * GPW; rb < P.m; rb += nwarps * GPW) {
    const int64_t r = rb + gw;
    const bool live = r < P.m;
    const int64_t s = live ? (int64_t)__ldg(P.row_ptr + r) : 0;
    const int64_t e = live ? (int64_t)__ldg(P.row_ptr + r + 1) : 0;
    const int64_t q0 = s & ~(int64_t)3;
    const int lo = (int)(s - q0);
    const int64_t l64 = e - q0;
    int len = (int)min(l64, PF_MAX_ROW_SPAN);
    if (l64 > PF_MAX_ROW_SPAN) {
      if (lig == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
      len = 0;
    }
    double acc[KC];
#pragma unroll
    for (int j = 0; j < KC; ++j) acc[j] = 0.0;
    // one non-zero: its KC products
    auto add = [&](int cc, double a) {
      const bool inb = (uint32_t)cc < n;
      bad |= !inb;
      if (inb) {
        double xv[KC];
        XRow<VT, KC, VX>::load(P.X + (int64_t)cc * P.ldx, kc, xv);
#pragma unroll
        for (int j = 0; j < KC; ++j) acc[j] += a * xv[j];
      }
    };
    if (VEC) {
      for (int o = 4 * lig; o < len; o += 4 * V) {
        const int4 c4 = __ldcs(reinterpret_cast<const int4 *>(P.col + q0 + o));
        VT v4[4];
        Block4<VT>::load(P.val, q0 + o, o + 1 >= lo, o + 2 < len, v4);
        const int cc[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (o + i >= lo && o + i < len) add(cc[i], (double)v4[i]);
      }
    } else {
      for (int o = lo + lig; o < len; o += V) add(__ldg(P.col + q0 + o), (double)__ldg(P.val + q0 + o));
    }
#pragma unroll
    for (int j = 0; j < KC; ++j) {
#pragma unroll
      for (int d = V / 2; d > 0; d >>= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], d);
    }
    if (live) {
      VT *yr = P.Y + r * P.ldy;
#pragma unroll
      for (int j = 0; j < KC; ++j) {
        if (j < kc && (j % V) == lig) {
          double out = P.alpha * acc[j];
          if (P.beta != 0.0) out += P.beta * (double)yr[j];
          yr[j] = (VT)out;
        }
      }
    }
  }
  if (bad) atomicOr(P.err, PF_DEVERR_BOUNDS);
}

}  // namespace pf
