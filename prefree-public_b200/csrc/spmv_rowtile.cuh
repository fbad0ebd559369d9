// ROWTILE variant: row-aligned tiles, coalesced element-per-thread products
// parked in shared memory, then VR lanes per row sum the row from there.
//
// Tile t holds the R = NT / VR rows [t*R, t*R + R). Its non-zeros are the
// contiguous range [a, b) = [row_ptr[t*R], row_ptr[t*R + R]): no search and no
// start-row table is needed to find them, and no row is cut between CTAs, so
// there are no carries and no atomics on y. The range is walked in windows of
// CAP non-zeros. In a window, thread i takes the non-zeros i, i + NT, ... of
// the window (so every warp load of col and val is one contiguous run), issues
// all of its column and value loads, then all of its x gathers, and writes the
// products to shared memory. After a barrier, the VR lanes of row j's group
// add up the products of row j that lie in the window (lane l: positions
// l, l + VR, ...); a row that spans windows keeps its partial in registers. At
// the end the group's lanes combine their partials with __shfl_xor and lane 0
// writes y.
//
// One wave of CTAs strides over the tiles, and each CTA loads the row bounds
// of its next tile while it works on the current one, so that a tile's column
// and value loads start without first waiting on row_ptr.
//
// The reference kernel has the same two stages: a product stage of one
// non-zero per thread per round into shared memory, then row reductions from
// shared memory by a thread, a vector of lanes or the whole block
// (src/spmv_kernel/preFreeSpMV.cu:30-150, 407-437). Its tiles are fixed runs
// of non-zeros, which cut rows (fixed up by fp64 atomicAdd on y) and need the
// start_row pre-pass (:3-28). Here tiles are fixed runs of rows, so the
// product stage's window bounds come straight from two row_ptr entries.
//
// LX (long-row escape): a row of more than `lt` non-zeros is not summed by
// its tile. Its group lists it (one global atomic per row) in the long-row
// chunk list that spmv_longrow_chunks_kernel sums in a second launch, and the
// tile's windows skip its non-zeros. Up to NLR long rows per tile are
// listed; further ones are summed in place (correct, only slower).
//
// Works with any alignment of col and val (element loads). Checks: a tile
// whose range leaves [row_ptr[0], row_ptr[0] + nnz) or holds 2^31 or more
// non-zeros, and a row_ptr that decreases inside a tile, set PF_DEVERR_ROWPTR
// (the tile writes nothing); a column outside [0, n) sets PF_DEVERR_BOUNDS and
// reads as x = 0.
#pragma once

#include "pf_common.cuh"
#include "pf_ptx.cuh"
#include "spmv_nnzsplit.cuh"

namespace pf {

template <typename VT, typename IT, int NT, int VR, int CAP, bool LX, int MINB>
__global__ void __launch_bounds__(NT, MINB)
spmv_rowtile_kernel(const SpmvParams<VT, IT> P, const LongRowScratch L, int64_t lt,
                    int64_t chunk) {
  static_assert(NT % VR == 0 && VR <= 32 && (VR & (VR - 1)) == 0, "VR: power of 2 up to 32");
  static_assert(CAP % NT == 0, "CAP: a multiple of NT");
  constexpr int R = NT / VR;     // rows per tile, one per lane group
  constexpr int K = CAP / NT;    // non-zeros per thread per window
  constexpr int NLR = LX ? 16 : 1;
  __shared__ double prod[CAP];
  __shared__ int rps[R + 1];     // row starts, relative to the tile's first non-zero
  __shared__ int2 lrs[NLR];      // LX: listed long rows [start, end), relative
  __shared__ int nlr;

  const int tid = threadIdx.x;
  const int grp = tid / VR, li = tid & (VR - 1);
  const int64_t base = (int64_t)__ldg(P.row_ptr);
  const int64_t zend = base + P.nnz;
  const uint32_t n = (uint32_t)(P.n < 0xffffffffLL ? P.n : 0xffffffffLL);
  const double alpha = P.alpha, beta = P.beta;
  const int64_t ntiles = ceil_div(P.m, (int64_t)R);
  bool bad = false;

  // row bounds of the CTA's next tile: thread j holds entry j of its R + 1
  // row starts (thread 0 also entry R when R == NT)
  int64_t na = 0, nb = 0, ne = 0;
  auto fetch = [&](int64_t t) {
    if (t >= ntiles) return;
    const int64_t r0 = t * R;
    const int rows = (int)min((int64_t)R, P.m - r0);
    na = (int64_t)__ldg(P.row_ptr + r0);
    nb = (int64_t)__ldg(P.row_ptr + r0 + rows);
    if (tid <= rows) ne = (int64_t)__ldg(P.row_ptr + r0 + tid);
  };
  fetch(blockIdx.x);
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x) {
    const int64_t r0 = t * R;
    const int rows = (int)min((int64_t)R, P.m - r0);
    const int64_t a = na, b = nb, e = ne;
    fetch(t + gridDim.x);
    // the same a and b in every thread: the skip is uniform
    if (a < base || b > zend || b < a || b - a > (int64_t)INT32_MAX) {
      if (tid == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
      continue;
    }
    const int tot = (int)(b - a);
    if (LX && tid == 0) nlr = 0;
    bool clamped = false;
    if (tid <= rows) {
      const int64_t c = min(max(e, a), b);
      clamped = c != e;
      rps[tid] = (int)(c - a);
    }
    if (R == NT && tid == 0) rps[R] = tot;  // entry R is b itself
    bool tile_bad = __syncthreads_or(clamped);
    const bool mine = grp < rows;
    const int rs = mine ? rps[grp] : 0;
    const int re = mine ? max(rps[grp + 1], rs) : 0;
    const bool decreasing = mine && rps[grp + 1] < rs;
    bool is_long = false;
    if (LX) {
      bool lead_long = false;
      if (!tile_bad && mine && li == 0 && (int64_t)(re - rs) > lt) {
        const int p = atomicAdd(&nlr, 1);
        if (p < NLR) {
          lrs[p] = make_int2(rs, re);
          lx_publish_row(L, r0 + grp, a + rs, a + re, chunk, P.err);
          lead_long = true;
        }
      }
      // the group's lanes share a warp: lane 0's decision for all of them
      is_long = __shfl_sync(0xffffffffu, lead_long, (tid & 31) & ~(VR - 1));
    }
    tile_bad |= __syncthreads_or(decreasing);
    if (tile_bad) {
      // a row_ptr entry outside [a, b] or decreasing: nothing is written
      if (tid == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
      continue;
    }
    const int nl = LX ? min(nlr, NLR) : 0;

    double acc = 0.0;
    int w = 0;
    while (true) {
      if (LX) {
        // step over listed long rows that cover w (they may follow each other)
        for (bool moved = true; moved;) {
          moved = false;
          for (int k = 0; k < nl; ++k) {
            const int2 q = lrs[k];
            if (w >= q.x && w < q.y) {
              w = q.y;
              moved = true;
            }
          }
        }
      }
      if (w >= tot) break;
      int w1 = min(w + CAP, tot);
      if (LX) {
        for (int k = 0; k < nl; ++k) {
          const int s = lrs[k].x;
          if (s > w && s < w1) w1 = s;
        }
      }
      const int len = w1 - w;
      const int64_t g0 = a + w;
      // all column and value loads of the window, then all x gathers
      int cc[K];
      VT vv[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int i = tid + k * NT;
        cc[k] = i < len ? __ldcs(P.col + g0 + i) : 0;
        vv[k] = i < len ? __ldcs(P.val + g0 + i) : VT(0);
      }
      VT xv[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int i = tid + k * NT;
        const bool inb = (uint32_t)cc[k] < n;
        bad |= i < len && !inb;
        xv[k] = (i < len && inb) ? ptx::ldg_x(P.x + cc[k]) : VT(0);
      }
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int i = tid + k * NT;
        if (i < len) prod[i] = (double)vv[k] * (double)xv[k];
      }
      __syncthreads();
      if (mine && !is_long) {
        const int lo = max(rs, w) - w, hi = min(re, w1) - w;
        for (int i = lo + li; i < hi; i += VR) acc += prod[i];
      }
      w = w1;
      __syncthreads();  // the products are rewritten by the next window
    }
#pragma unroll
    for (int d = VR / 2; d > 0; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
    if (mine && li == 0 && !is_long) {
      const int64_t r = r0 + grp;
      double out = alpha * acc;
      if (beta != 0.0) out += beta * (double)P.y[r];
      P.y[r] = (VT)out;
    }
    __syncthreads();  // shared state is rewritten by the next tile
  }
  if (bad) atomicOr(P.err, PF_DEVERR_BOUNDS);
}

}  // namespace pf
