// NNZTILE variant: equal-nnz CTA slices walked in tiles of NT * E non-zeros;
// each thread's E consecutive non-zeros stay in registers, the tile's row
// ends are scattered into a bit mask, and one CTA segmented scan finishes
// the rows. Built for many resident CTAs (128 threads, few registers, ~4 KB
// of shared memory): the x gathers of random columns are served by L2, and
// it is the number of warps waiting on them that sets the rate.
//
// Slice c holds the non-zeros [S0, S1) = [base + c*T, min(base + (c+1)*T,
// base + nnz)) (slice geometry and the ownership of cut and empty rows as in
// spmv_nnzsplit.cuh). Its first row is found once by a warp search of
// row_ptr; after that a row cursor r_cur (the first row not yet finished)
// moves forward tile by tile. Tile i covers the absolute positions
// [A + i*TILE, A + (i+1)*TILE) with A = S0 rounded down to a 16-byte block,
// clipped to [S0, S1). Per tile:
//   1. thread t loads the E/4 16-byte column blocks and value pieces holding
//      its positions [tb + E*t, tb + E*t + E), and thread j loads the bounds
//      of row r_cur + j (a coalesced window of NT rows);
//   2. it gathers x for its columns and forms the E products (zero outside
//      [S0, S1));
//   3. every window row that ends inside the tile sets the bit of its last
//      position in the tile's mask and records its row there; empty rows are
//      written at once; a window whose rows all end in the tile is followed
//      by the next window (runs of short rows);
//   4. thread t walks its E products against its E mask bits, writing every
//      row that ends in its range except the first; a CTA segmented scan of
//      (ended a row, sum since its last end) gives the sum flowing into the
//      first one from earlier threads and tiles.
// The sums and their order are fixed by the matrix and the slice size: the
// same bits on every run. A row that starts before the slice or runs past its
// end is finished by contribute_cut_row (partials summed in slice order).
//
// The reference reaches the same per-tile economics (coalesced product loads,
// row sums from the tile, src/spmv_kernel/preFreeSpMV.cu:407-437) through a
// start_row table built by a pre-pass kernel (:3-28) and fp64 atomicAdd on the
// rows cut by its tiles (:67, :91, :142). Here a slice finds its first row by
// one search, carries the row cursor across its tiles, and adds no atomics on
// y. Requires col and val on 16-byte boundaries (the host falls back
// otherwise).
#pragma once

#include "pf_common.cuh"
#include "pf_ptx.cuh"
#include "spmv_nnzsplit.cuh"
#include "spmv_rowvec.cuh"

namespace pf {

template <typename VT, typename IT, int NT, int E, int MINB>
__global__ void __launch_bounds__(NT, MINB)
spmv_nnztile_kernel(const SpmvParams<VT, IT> P) {
  static_assert(E == 4 || E == 8, "E: 4 or 8 non-zeros per thread");
  static_assert(NT % 32 == 0 && NT <= 1024, "NT: whole warps");
  constexpr int TILE = NT * E;
  constexpr int NWARP = NT / 32;
  constexpr int MW = TILE / 32;   // mask words per tile
  constexpr int NB = E / 4;       // 16-byte column blocks per thread
  // double-buffered by tile parity: tile i + 1 scatters while tile i's rows
  // are still being written from its buffer
  __shared__ uint32_t s_mask[2][MW];
  __shared__ int s_row[2][TILE];  // row (relative to the tile's first row) ending at a position
  __shared__ double s_wv[2][NWARP];
  __shared__ int s_wf[2][NWARP];
  __shared__ int64_t s_meta[2];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t c = blockIdx.x;
  const int64_t base = (int64_t)__ldg(P.row_ptr);
  // nnz must equal row_ptr[m] - row_ptr[0], or slices would read outside
  // the arrays: every CTA checks before touching them
  if ((int64_t)__ldg(P.row_ptr + P.m) - base != P.nnz) {
    if (tid == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
    return;
  }
  const int64_t S0 = base + c * P.T;
  const int64_t S1 = min(S0 + P.T, base + P.nnz);
  const bool last = c == P.num_ctas - 1;
  for (int w = tid; w < 2 * MW; w += NT) (&s_mask[0][0])[w] = 0u;
  if (warp == 0) {
    const int64_t lb = warp_lower_bound(P.row_ptr, P.m, S0, lane);
    if (lane == 0) {
      s_meta[0] = lb;
      s_meta[1] = ((int64_t)__ldg(P.row_ptr + lb) != S0) ? 1 : 0;
    }
  }
  __syncthreads();
  if (s_meta[1] != 0 && s_meta[0] == 0) {
    // row_ptr[0] > S0 is impossible for a non-decreasing row_ptr
    if (tid == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
    return;
  }
  const bool head_partial = s_meta[1] != 0;
  int64_t r_cur = head_partial ? s_meta[0] - 1 : s_meta[0];
  const int64_t head_row = head_partial ? r_cur : -1;
  const uint32_t n = (uint32_t)(P.n < 0xffffffffLL ? P.n : 0xffffffffLL);
  const double alpha = P.alpha, beta = P.beta;
  bool bad = false, bad_rows = false;

  auto write_row = [&](int64_t R, double v) {
    double out = alpha * v;
    if (beta != 0.0) out += beta * (double)P.y[R];
    P.y[R] = (VT)out;
  };

  // Positions inside the slice are 32-bit offsets from A, S0 rounded down to
  // a 16-byte block (a slice holds fewer than 2^31 non-zeros); the tile's
  // column and value blocks are addressed from there.
  const int64_t A = S0 & ~(int64_t)3;
  const int lo0 = (int)(S0 - A), hiS = (int)(S1 - A);
  const int4 *__restrict__ colA = reinterpret_cast<const int4 *>(P.col + A);
  const VT *__restrict__ valA = P.val + A;
  // a row_ptr entry as an offset from A, clamped to [-1, hiS + 1] (a row that
  // ends past the slice compares as past it)
  auto rel = [&](int64_t r) -> int {
    const int64_t v = (int64_t)__ldg(P.row_ptr + r) - A;
    return (int)min(max(v, (int64_t)-1), (int64_t)hiS + 1);
  };
  const int ntiles = (hiS + TILE - 1) / TILE;
  double carry = 0.0;  // sum of the open row so far (the same in every thread)
  for (int i = 0; i < ntiles; ++i) {
    const int par = i & 1;
    const int tb = i * TILE;
    const int lo = max(tb, lo0), hi = min(tb + TILE, hiS);
    // ---- 1. this thread's column blocks and value pieces, the row window
    const int q0 = tb + E * tid;
    int cc[E];
    VT vv[E];
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const int q = q0 + 4 * b;
      const bool act = q + 4 > lo && q < hi;
      const int4 c4 = act ? __ldcs(colA + (q >> 2)) : make_int4(0, 0, 0, 0);
      cc[4 * b] = c4.x;
      cc[4 * b + 1] = c4.y;
      cc[4 * b + 2] = c4.z;
      cc[4 * b + 3] = c4.w;
      Block4<VT>::load(valA, q, act && q + 2 > lo, act && q + 2 < hi, vv + 4 * b);
    }
    bool have = r_cur + tid < P.m;
    int rs = 0, re = 0;
    if (have) {
      rs = rel(r_cur + tid);
      re = rel(r_cur + tid + 1);
    }
    // ---- 2. x gathers and products
    double p[E];
#pragma unroll
    for (int k = 0; k < E; ++k) {
      const bool use = q0 + k >= lo && q0 + k < hi;
      const bool inb = (uint32_t)cc[k] < n;
      bad |= use && !inb;
      const VT xv = (use && inb) ? ptx::ldg_x(P.x + cc[k]) : VT(0);
      p[k] = use ? (double)vv[k] * (double)xv : 0.0;
    }
    // ---- 3. row ends of the tile, window by window
    int done = 0;  // rows finished in this tile before the current window
    while (true) {
      // row r_cur + done + tid ends in this tile; an empty row that starts at
      // S1 belongs to the next slice (the last slice takes every row)
      const bool fin = have && re <= hi && !(!last && re == rs && rs == hiS);
      if (fin) {
        if (re > rs && re > lo) {
          const int pos = re - 1 - tb;
          atomicOr(&s_mask[par][pos >> 5], 1u << (pos & 31));
          s_row[par][pos] = done + tid;
        } else if (re == rs) {
          write_row(r_cur + done + tid, 0.0);  // empty row (never the slice's head row)
        } else {
          bad_rows = true;  // row_ptr not non-decreasing
        }
      }
      const int nf = __syncthreads_count(fin);
      done += nf;
      if (nf < NT) break;
      // every row of the window ends here: the next window
      have = r_cur + done + tid < P.m;
      if (have) {
        rs = rel(r_cur + done + tid);
        re = rel(r_cur + done + tid + 1);
      }
    }
    // ---- 4. walk the products against the mask bits: a row that ends and
    // is not the thread's first is written at once
    constexpr uint32_t LMASK = (1u << E) - 1u;
    const uint32_t bits = (s_mask[par][(E * tid) >> 5] >> ((E * tid) & 31)) & LMASK;
    double acc = 0.0, head = 0.0;
    const int first = bits ? __ffs(bits) - 1 : E;
#pragma unroll
    for (int k = 0; k < E; ++k) {
      acc += p[k];
      const bool end = (bits >> k) & 1u;
      if (end && k > first) write_row(r_cur + s_row[par][E * tid + k], acc);
      head = (k == first) ? acc : head;
      acc = end ? 0.0 : acc;
    }
    // segmented scan over the CTA: (ended a row, sum since its last end)
    int f = bits ? 1 : 0;
    double v = acc;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int fu = __shfl_up_sync(0xffffffffu, f, d);
      const double vu = __shfl_up_sync(0xffffffffu, v, d);
      if (lane >= d) {
        if (!f) v = vu + v;
        f |= fu;
      }
    }
    if (lane == 31) {
      s_wf[par][warp] = f;
      s_wv[par][warp] = v;
    }
    __syncthreads();
    // the scan's value entering this warp (from the carry and earlier warps)
    // and leaving the tile (the next carry)
    double pf_v = carry, tot = carry;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) {
      const double wv = s_wv[par][w];
      const bool wf = s_wf[par][w] != 0;
      if (w < warp) pf_v = wf ? wv : pf_v + wv;
      tot = wf ? wv : tot + wv;
    }
    const double incl = f ? v : pf_v + v;
    double excl = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) excl = pf_v;
    if (bits) {
      const int64_t R = r_cur + s_row[par][E * tid + first];
      if (R == head_row) contribute_cut_row(P, base, R, true, c, excl + head);
      else write_row(R, excl + head);
    }
    carry = tot;
    r_cur += done;
    // this parity's mask is set again by tile i + 2: its readers are past
    // the barrier above
    if (tid < MW) s_mask[par][tid] = 0u;
  }
  // the row still open at the slice end runs past S1: hand on its partial
  if (tid == 0 && !last && r_cur < P.m && rel(r_cur) < hiS)
    contribute_cut_row(P, base, r_cur, r_cur == head_row, c, carry);
  if (bad) atomicOr(P.err, PF_DEVERR_BOUNDS);
  if (bad_rows) atomicOr(P.err, PF_DEVERR_ROWPTR);
}

}  // namespace pf
