// ROWGROUP variant: rows split evenly, V lanes per row, U rows per lane group
// in flight. No row_ptr search, no carries, no shared memory: every row is
// finished by the group that owns it (segmented __shfl_xor reduction).
//
// Chosen by the selector for short, regular rows (uniform 16/row, the
// Laplacian, banded 32/row) and for long rows of equal length, where equal
// rows are equal work. It is correct for any CSR — a long row only makes its
// group slow — so a stale selection never changes results.
//
// Counterpart of the reference's red_row_vector<TILE,BLOCK,4> path
// (src/spmv_kernel/preFreeSpMV.cu:116-150), without its nnz tiles, start_row
// table and boundary atomics: here a group always holds whole rows.
#pragma once

#include "pf_common.cuh"
#include "pf_ptx.cuh"
#include "spmv_nnzsplit.cuh"

namespace pf {

// NTB threads per CTA; V lanes per row (power of two <= 32); U rows per group
// per iteration. A warp covers (32/V)*U consecutive rows per iteration.
template <typename VT, typename IT, int V, int U, int NTB>
__global__ void __launch_bounds__(NTB)
spmv_rowgroup_kernel(const SpmvParams<VT, IT> P) {
  constexpr int GPW = 32 / V;  // groups per warp
  const int lane = threadIdx.x & 31;
  const int lig = lane & (V - 1);
  const int gw = lane / V;
  const int64_t warp_global = (blockIdx.x * (int64_t)NTB + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * NTB) >> 5;
  const uint64_t xpol = ptx::policy_evict_last();
  const uint64_t spol = ptx::policy_evict_first();
  const double alpha = P.alpha, beta = P.beta;
  constexpr int64_t ROWS_PER_WARP = (int64_t)GPW * U;

  const int64_t stride = nwarps * ROWS_PER_WARP;
  // a valid element index: [row_ptr[0], row_ptr[0] + nnz) is readable, nnz > 0
  const int64_t safe = (int64_t)__ldg(P.row_ptr);
  int64_t rb = warp_global * ROWS_PER_WARP;
  // row bounds of the first block; later blocks are prefetched one ahead
  int64_t p[U], pe[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int64_t r = rb + (int64_t)u * GPW + gw;
    const int64_t rc = r < P.m ? r : P.m - 1;
    p[u] = (int64_t)__ldg(P.row_ptr + rc) + lig;
    pe[u] = r < P.m ? (int64_t)__ldg(P.row_ptr + rc + 1) : 0;
  }
  for (; rb < P.m; rb += stride) {
    // prefetch the next block's row bounds
    int64_t np_[U], npe[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t r = rb + stride + (int64_t)u * GPW + gw;
      const int64_t rc = r < P.m ? r : P.m - 1;
      np_[u] = (int64_t)__ldg(P.row_ptr + rc) + lig;
      npe[u] = r < P.m ? (int64_t)__ldg(P.row_ptr + rc + 1) : 0;
    }
    double acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) acc[u] = 0.0;
    bool more = true;
    bool bad = false;
    while (more) {
      // unconditional loads on clamped indices (lanes past their row's end
      // read element row_ptr[0] and discard it)
      int32_t ci[U];
      VT vv[U];
      bool act[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        act[u] = p[u] < pe[u];
        const int64_t q = act[u] ? p[u] : safe;
        ci[u] = ptx::ldg_hint(P.col + q, spol);
        vv[u] = ptx::ldg_hint(P.val + q, spol);
      }
      VT xv[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const bool inb = (uint64_t)(int64_t)ci[u] < (uint64_t)P.n;
        bad |= act[u] && !inb;
        xv[u] = ptx::ldg_hint(P.x + (inb ? ci[u] : 0), xpol);
      }
      more = false;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (act[u] && (uint64_t)(int64_t)ci[u] < (uint64_t)P.n)
          acc[u] += (double)vv[u] * (double)xv[u];
        p[u] += V;
        more |= p[u] < pe[u];
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
      p[u] = np_[u];
      pe[u] = npe[u];
    }
  }
}

}  // namespace pf
