// ROWVEC variant: rows split evenly, V lanes per row, each lane covering whole
// 16-byte-aligned blocks of 4 non-zeros (one 16-byte col load, one or two
// 16-byte val loads, four x gathers), U rows per lane group in flight, the
// next rows' bounds prefetched one step ahead. No shared memory, no barriers,
// no carries: a row is finished by the group that owns it (__shfl_xor over
// its V lanes).
//
// The blocks of a row start at floor4(row start); elements outside the row
// are masked. A block is loaded only when it holds an element of the row, and
// each 8-byte-value half only when it holds one, so every load stays inside a
// 16-byte block that contains a valid element. Requires col and val to start
// on 16-byte boundaries (the host falls back to ROWGROUP otherwise).
//
// Selected for regular rows (uniform 16/row, the Laplacian, banded 32/row,
// 2000/row). Correct for any CSR; an unusually long row only slows its group.
#pragma once

#include "pf_common.cuh"
#include "spmv_nnzsplit.cuh"

namespace pf {

template <typename VT>
struct Block4;

template <>
struct Block4<double> {
  // elements q..q+3 (q % 4 == 0): halves loaded only when flagged
  __device__ __forceinline__ static void load(const double *v, int64_t q, bool lo, bool hi,
                                              double out[4]) {
    double2 a = make_double2(0.0, 0.0), b = make_double2(0.0, 0.0);
    if (lo) a = __ldcs(reinterpret_cast<const double2 *>(v + q));
    if (hi) b = __ldcs(reinterpret_cast<const double2 *>(v + q + 2));
    out[0] = a.x;
    out[1] = a.y;
    out[2] = b.x;
    out[3] = b.y;
  }
};

template <>
struct Block4<float> {
  __device__ __forceinline__ static void load(const float *v, int64_t q, bool lo, bool hi,
                                              float out[4]) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (lo || hi) a = __ldcs(reinterpret_cast<const float4 *>(v + q));
    out[0] = a.x;
    out[1] = a.y;
    out[2] = a.z;
    out[3] = a.w;
  }
};

template <typename VT, typename IT, int V, int U, int NTB>
__global__ void __launch_bounds__(NTB)
spmv_rowvec_kernel(const SpmvParams<VT, IT> P) {
  constexpr int GPW = 32 / V;  // row groups per warp
  constexpr int64_t RPW = (int64_t)GPW * U;
  const int lane = threadIdx.x & 31;
  const int lig = lane & (V - 1);
  const int gw = lane / V;
  const int64_t warp_global = (blockIdx.x * (int64_t)NTB + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * NTB) >> 5;
  const int64_t stride = nwarps * RPW;
  const double alpha = P.alpha, beta = P.beta;
  const uint32_t n = (uint32_t)(P.n < 0xffffffffLL ? P.n : 0xffffffffLL);

  int64_t rb = warp_global * RPW;
  int64_t s[U], e[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int64_t r = rb + (int64_t)u * GPW + gw;
    s[u] = r < P.m ? (int64_t)__ldg(P.row_ptr + r) : 0;
    e[u] = r < P.m ? (int64_t)__ldg(P.row_ptr + r + 1) : 0;
  }
  for (; rb < P.m; rb += stride) {
    int64_t ns[U], ne[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t r = rb + stride + (int64_t)u * GPW + gw;
      ns[u] = r < P.m ? (int64_t)__ldg(P.row_ptr + r) : 0;
      ne[u] = r < P.m ? (int64_t)__ldg(P.row_ptr + r + 1) : 0;
    }
    double acc[U];
    int64_t q[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      acc[u] = 0.0;
      q[u] = (s[u] & ~(int64_t)3) + 4 * lig;
    }
    bool bad = false;
    bool more = true;
    while (more) {
      int4 c4[U];
      VT v4[U][4];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const bool act = q[u] < e[u];
        c4[u] = act ? __ldcs(reinterpret_cast<const int4 *>(P.col + q[u])) : make_int4(0, 0, 0, 0);
        Block4<VT>::load(P.val, q[u], act && q[u] + 1 >= s[u], act && q[u] + 2 < e[u], v4[u]);
      }
      VT xv[U][4];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int cc[4] = {c4[u].x, c4[u].y, c4[u].z, c4[u].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int64_t el = q[u] + i;
          const bool use = el >= s[u] && el < e[u];
          const bool inb = (uint32_t)cc[i] < n;
          bad |= use && !inb;
          xv[u][i] = (use && inb) ? __ldg(P.x + cc[i]) : VT(0);
        }
      }
      more = false;
#pragma unroll
      for (int u = 0; u < U; ++u) {
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[u] += (double)v4[u][i] * (double)xv[u][i];
        q[u] += 4 * V;
        more |= q[u] < e[u];
      }
    }
    if (bad) atomicOr(P.err, PF_DEVERR_BOUNDS);
#pragma unroll
    for (int u = 0; u < U; ++u) {
#pragma unroll
      for (int d = V / 2; d > 0; d >>= 1) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], d);
    }
    if (lig == 0) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int64_t r = rb + (int64_t)u * GPW + gw;
        if (r < P.m) {
          double out = alpha * acc[u];
          if (beta != 0.0) out += beta * (double)P.y[r];
          P.y[r] = (VT)out;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      s[u] = ns[u];
      e[u] = ne[u];
    }
  }
}

}  // namespace pf
