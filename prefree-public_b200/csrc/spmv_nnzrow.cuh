// NNZROW variant: equal-nnz CTA slices walked in tiles of NT * K non-zeros;
// products parked in shared memory, each row's piece of a tile summed by one
// thread (short pieces) or one warp (long pieces). Shipped with one-warp CTAs
// (NT = 32), whose barriers are warp primitives, and K = 7 non-zeros per
// thread for 8-byte values, 10 for 4- and 2-byte values.
//
// Slice c holds the non-zeros [S0, S1) = [base + c*T, min(base + (c+1)*T,
// base + nnz)) (slice geometry and the ownership of cut and empty rows as in
// spmv_nnzsplit.cuh). Its first row is found once by a warp search of
// row_ptr; a row cursor r_cur (the first row not yet finished) and the
// partial sum of that row (carry) then move forward tile by tile. A tile is
// the positions [tb, te) of the slice, 32-bit offsets from S0. Per tile:
//   1. thread t forms the products of positions tb + t + k*NT (k < K) from
//      the column and value elements it loaded during the previous tile, and
//      parks them in shared memory; it then loads the next tile's elements
//      (coalesced warp loads, in flight while this tile is summed);
//   2. thread j takes row r_cur + done + j of the window of NT rows (the
//      first window's bounds are loaded with the tile's x gathers): the
//      row's piece of the tile is [max(start, tb), min(end, te)). A piece of
//      at most LS products is summed by the thread itself; longer pieces are
//      listed and summed afterwards by a warp each (lane-strided, then
//      __shfl_xor). A row that ends in the tile is written (the cursor's row
//      adds the carry); the row that runs past te leaves its sum as the next
//      carry. A window whose rows all end in the tile is followed by the next.
// The sums and their order are fixed by the matrix and the slice size: the
// same bits on every run. A row that starts before the slice or runs past
// its end is finished by contribute_cut_row (partials summed in slice order).
//
// These are the reference kernel's two stages, a product stage of coalesced
// element-per-thread loads into shared memory and row sums from there by a
// thread, a vector of lanes or the block (src/spmv_kernel/preFreeSpMV.cu:30-150,
// 416-437). Its tiles are likewise fixed runs of non-zeros, so that a tile's
// loads need no row information; it finds each tile's first row in a table
// built by a pre-pass kernel (:3-28) and adds the rows cut by its tiles with
// fp64 atomicAdd (:67, :91). Here a slice finds its first row by one search
// and carries the row cursor and the open row's sum across its tiles: no
// pre-pass and no atomics on y. Works with any alignment of col and val.
#pragma once

#include "pf_common.cuh"
#include "pf_ptx.cuh"
#include "spmv_nnzsplit.cuh"

namespace pf {

template <typename VT, typename IT, int NT, int K, int LS, int MINB>
__global__ void __launch_bounds__(NT, MINB)
spmv_nnzrow_kernel(const SpmvParams<VT, IT> P) {
  constexpr int TILE = NT * K;
  constexpr int NWARP = NT / 32;
  constexpr int LCAP = TILE / (LS + 1) + 2;  // long pieces per tile, at most
  __shared__ double prod[TILE];
  // double-buffered by tile parity: tile i + 1 resets its own copy while
  // tile i's is still being read
  __shared__ int3 s_long[2][LCAP];  // piece [x, y) of window row z (relative to r_cur)
  __shared__ int s_nlong[2];
  __shared__ double s_carry[2];
  __shared__ int64_t s_meta[2];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  // a one-warp CTA synchronises with warp primitives (shared memory is
  // ordered among the warp's lanes by __syncwarp)
  auto cta_sync = [&]() {
    if constexpr (NT == 32) __syncwarp();
    else __syncthreads();
  };
  auto cta_count = [&](bool pred) -> int {
    if constexpr (NT == 32) {
      const int c = __popc(__ballot_sync(0xffffffffu, pred));
      __syncwarp();
      return c;
    } else {
      return __syncthreads_count(pred);
    }
  };
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
  const int L = (int)(S1 - S0);  // positions 0 .. L of the slice
  const bool last = c == P.num_ctas - 1;
  const int32_t *__restrict__ col = P.col + S0;
  const VT *__restrict__ val = P.val + S0;
  const uint32_t n = (uint32_t)(P.n < 0xffffffffLL ? P.n : 0xffffffffLL);
  const double alpha = P.alpha, beta = P.beta;

  // this thread's elements of the first tile: their loads overlap the search
  int cn[K];
  VT vn[K];
  auto load_tile = [&](int tb) {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int pos = tb + tid + k * NT;
      cn[k] = pos < L ? __ldcs(col + pos) : 0;
      vn[k] = pos < L ? __ldcs(val + pos) : VT(0);
    }
  };
  load_tile(0);
  if (warp == 0) {
    const int64_t lb = warp_lower_bound(P.row_ptr, P.m, S0, lane);
    if (lane == 0) {
      s_meta[0] = lb;
      s_meta[1] = ((int64_t)__ldg(P.row_ptr + lb) != S0) ? 1 : 0;
    }
  }
  if (tid < 2) {
    s_nlong[tid] = 0;
    s_carry[tid] = 0.0;
  }
  cta_sync();
  if (s_meta[1] != 0 && s_meta[0] == 0) {
    // row_ptr[0] > S0 is impossible for a non-decreasing row_ptr
    if (tid == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
    return;
  }
  const bool head_partial = s_meta[1] != 0;
  int64_t r_cur = head_partial ? s_meta[0] - 1 : s_meta[0];
  const int64_t head_row = head_partial ? r_cur : -1;
  bool bad = false, bad_rows = false;

  // a row_ptr entry as a position of the slice, clamped to [-1, L + 1]
  // (int32 row_ptr: every entry and S0 are below 2^31, so the difference is
  // exact in 32 bits)
  auto rel = [&](int64_t r) -> int {
    if constexpr (sizeof(IT) == 4) {
      const int v = (int)__ldg(P.row_ptr + r) - (int)S0;
      return min(max(v, -1), L + 1);
    } else {
      const int64_t v = (int64_t)__ldg(P.row_ptr + r) - S0;
      return (int)min(max(v, (int64_t)-1), (int64_t)L + 1);
    }
  };
  auto finish = [&](int64_t R, double sum) {
    if (R == head_row) {
      contribute_cut_row(P, base, R, true, c, sum);
    } else {
      double out = alpha * sum;
      if (beta != 0.0) out += beta * (double)P.y[R];
      P.y[R] = (VT)out;
    }
  };

  double carry = 0.0;  // sum of row r_cur so far (the same in every thread)
  const int ntiles = (L + TILE - 1) / TILE;
  for (int i = 0; i < ntiles; ++i) {
    const int par = i & 1;
    const int tb = i * TILE;
    const int te = min(tb + TILE, L);
    // the bounds of the first window's rows, loaded with the x gathers
    int64_t R = r_cur + tid;
    bool have = R < P.m;
    int rs = have ? rel(R) : L + 1;
    int re = have ? rel(R + 1) : L + 1;
    // ---- 1. products of this tile, then the next tile's loads
    {
      VT xv[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const bool use = tb + tid + k * NT < te;
        const bool inb = (uint32_t)cn[k] < n;
        bad |= use && !inb;
        xv[k] = (use && inb) ? ptx::ldg_x(P.x + cn[k]) : VT(0);
      }
#pragma unroll
      for (int k = 0; k < K; ++k) prod[tid + k * NT] = (double)vn[k] * (double)xv[k];
    }
    if (i + 1 < ntiles) load_tile(tb + TILE);
    cta_sync();
    // the next tile's list and carry: every thread has read the previous
    // tile's carry from that copy before the barrier above
    if (tid == 0) {
      s_nlong[par ^ 1] = 0;
      s_carry[par ^ 1] = 0.0;
    }
    // ---- 2. rows of the tile, window by window
    int done = 0;
    while (true) {
      // an empty row that starts at S1 belongs to the next slice (the last
      // slice takes every row)
      const bool fin = have && re <= te && !(!last && re == rs && rs == L);
      const bool open = have && !fin && rs < te;  // runs past te
      bad_rows |= have && re < rs;
      if (fin || open) {
        const int lo = max(rs, tb) - tb, hi = min(re, te) - tb;
        if (hi - lo > LS) {
          const int e = atomicAdd(&s_nlong[par], 1);
          if (e < LCAP) s_long[par][e] = make_int3(lo, hi, fin ? done + tid : -1 - (done + tid));
          else bad_rows = true;  // more long pieces than a tile can hold
        } else {
          double sum = (done + tid == 0) ? carry : 0.0;
          for (int p = lo; p < hi; ++p) sum += prod[p];
          if (fin) finish(R, sum);
          else s_carry[par] = sum;
        }
      }
      const int nf = cta_count(fin);
      done += nf;
      if (nf < NT) break;
      // every row of the window ends in this tile: the next window
      R = r_cur + done + tid;
      have = R < P.m;
      rs = have ? rel(R) : L + 1;
      re = have ? rel(R + 1) : L + 1;
    }
    // ---- 3. long pieces, one warp each
    const int nlong = min(s_nlong[par], LCAP);
    for (int e = warp; e < nlong; e += NWARP) {
      const int3 q = s_long[par][e];
      double sum = 0.0;
      for (int p = q.x + lane; p < q.y; p += 32) sum += prod[p];
#pragma unroll
      for (int d = 16; d > 0; d >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, d);
      if (lane == 0) {
        const int rel_row = q.z >= 0 ? q.z : -1 - q.z;
        if (rel_row == 0) sum += carry;
        if (q.z >= 0) finish(r_cur + rel_row, sum);
        else s_carry[par] = sum;
      }
    }
    cta_sync();  // the next carry is in place; the products may be rewritten
    carry = s_carry[par];
    r_cur += done;
  }
  // the row still open at the slice end runs past S1: hand on its partial
  if (tid == 0 && !last && r_cur < P.m && rel(r_cur) < L)
    contribute_cut_row(P, base, r_cur, r_cur == head_row, c, carry);
  if (bad) atomicOr(P.err, PF_DEVERR_BOUNDS);
  if (bad_rows) atomicOr(P.err, PF_DEVERR_ROWPTR);
}

}  // namespace pf
