// NNZSPLIT variant: nnz-balanced CTA slices found by binary search of row_ptr,
// thread-sequential row walk + block segmented scan, deterministic cross-CTA
// carry combine for rows cut by a slice boundary.
//
// Replaces the reference's preFreeSpMV_kernel<4,128> + pre_start_rowPerTile
// (src/spmv_kernel/preFreeSpMV.cu:3-28, 407-561). Differences by design:
//   * no start_row table: each CTA finds its first/last row by a 32-ary warp
//     search of row_ptr (the reference builds start_row[] in a separate
//     pre-pass kernel, :583-602);
//   * no atomicAdd on y: a row cut by slice boundaries is finished by whichever
//     participating CTA arrives last, which sums the per-CTA partials in CTA
//     order (the reference uses fp64 atomicAdd at :67, :91, :142, :333, whose
//     order varies run to run);
//   * alpha/beta, fp32 values, int64 row_ptr, row_ptr[0] != 0 (row slices).
//
// Slice geometry (Z = nnz, T = slice size, P = ceil(Z/T) CTAs, base = row_ptr[0]):
//   CTA c owns non-zeros [s, e) = [base + c*T, min(base + (c+1)*T, base + Z)).
//   lb(s) = first r in [0, m] with row_ptr[r] >= s.
//   first_row = lb(s) if row_ptr[lb(s)] == s, else lb(s) - 1 ("head partial":
//   the row started in an earlier CTA). end_row = lb(e) (m for the last CTA),
//   tail partial iff row_ptr[lb(e)] != e (row end_row-1 continues past e).
//   The CTA emits rows [first_row, end_row); empty rows whose start equals a
//   slice start belong to the CTA starting there, trailing empty rows to the
//   last CTA. A cut row R has participants k1-1 .. k2 with
//   k1 = (row_ptr[R]-base)/T + 1, k2 = (row_ptr[R+1]-1-base)/T; its sum is
//   carry_tail[k1-1] + carry_head[k1] + ... + carry_head[k2].
#pragma once

#include "pf_common.cuh"

namespace pf {

template <typename VT, typename IT>
struct SpmvParams {
  int64_t m;
  int64_t n;
  int64_t nnz;  // Z
  int64_t T;    // non-zeros per CTA slice
  int64_t num_ctas;
  const IT *__restrict__ row_ptr;
  const int32_t *__restrict__ col;
  const VT *__restrict__ val;
  const VT *__restrict__ x;
  VT *__restrict__ y;
  double alpha;
  double beta;
  double *carry_head;   // [num_ctas]
  double *carry_tail;   // [num_ctas]
  unsigned *counters;   // [num_ctas], zero between launches (self-resetting)
  unsigned *err;        // device error word
};

// Long-row escape (ROWVEC_LX): rows longer than the short-row
// limit are cut into chunks of at most `chunk` non-zeros by the row kernel,
// which writes one descriptor per chunk; the chunk kernel sums the chunks.
// Chunk ids are reserved with a 64-bit atomic counter. All counters are zero
// between launches (the chunk kernel's last CTA resets them).
struct LongChunk {
  int64_t row;    // the row
  int64_t cs;     // first non-zero of the chunk
  int64_t first;  // chunk id of the row's first chunk (partials, finish counter)
  int32_t len;    // non-zeros in the chunk
  int32_t nch;    // chunks of the row (1: the chunk writes y itself)
};

struct LongRowScratch {
  unsigned long long *alloc;  // chunk ids reserved so far
  LongChunk *chunks;          // [cap_chunks]
  unsigned *cnt;              // [cap_chunks], at a row's first chunk id: chunks finished
  double *part;               // [cap_chunks] chunk partials
  unsigned *done;             // CTAs of the chunk kernel finished
  int64_t cap_chunks;
};

// A row's chunks are the pieces of [s, e) in the aligned windows
// [k * chunk, (k + 1) * chunk) of the absolute non-zero index, so that every
// chunk lies in one window (the chunk kernel covers a window in one pass).
__device__ __forceinline__ int64_t lx_num_chunks(int64_t s, int64_t e, int64_t chunk) {
  return e > s ? (e - 1) / chunk - s / chunk + 1 : 0;
}

// Descriptors of chunks [0, nch) of row `row` = [s, e), first chunk id `first`,
// written by `nthreads` cooperating threads (thread `t` of them).
__device__ __forceinline__ void lx_write_chunks(const LongRowScratch &L, int64_t row, int64_t s,
                                                int64_t e, int64_t first, int64_t chunk, int t,
                                                int nthreads) {
  const int64_t nch = lx_num_chunks(s, e, chunk);
  const int64_t w0 = s / chunk;
  for (int64_t c = t; c < nch; c += nthreads) {
    const int64_t cs = max(s, (w0 + c) * chunk);
    const int64_t ce = min(e, (w0 + c + 1) * chunk);
    L.chunks[first + c] = LongChunk{row, cs, first, (int32_t)(ce - cs), (int32_t)nch};
  }
}

// One thread lists one row directly (one global atomic per row: for rare
// rows, or when a CTA's shared list is full).
__device__ __forceinline__ void lx_publish_row(const LongRowScratch &L, int64_t row, int64_t s,
                                               int64_t e, int64_t chunk, unsigned *err) {
  const int64_t nch = lx_num_chunks(s, e, chunk);
  const int64_t first = (int64_t)atomicAdd(L.alloc, (unsigned long long)nch);
  if (first + nch <= L.cap_chunks) lx_write_chunks(L, row, s, e, first, chunk, 0, 1);
  else atomicOr(err, PF_DEVERR_ROWPTR);
}

// Fused all-gather for the row-sharded iterated multiply: instead of y, each
// finished row is stored straight into every rank's next-x buffer (peer
// pointers over NVLink), and ||y||^2 of this rank's rows is reduced in the
// same kernel and written to slot `rank` of every rank's norm-slot array.
// alpha is taken on the device from the previous iteration's slots:
// alpha = 1 / sqrt(sum of prev[0..nranks)).
struct DistOut {
  double *const *outs;   // [nranks] next-x base pointers (row index: row_offset + r)
  double *const *slots;  // [nranks] norm-slot arrays (this rank writes index `rank`)
  const double *prev;    // this rank's copy of the previous iteration's slots
  double *cta_part;      // [grid] per-CTA partials
  unsigned *counter;     // zero between launches
  // step barrier (optional): flags[p][q] = steps rank q has finished, as seen
  // by rank p. Step `step` waits until this rank's flags reach `step` for
  // every rank and, when done, sets flags[p][rank] = step + 1 on every p.
  unsigned long long *const *flags;
  unsigned long long step;
  int64_t row_offset;
  int nranks, rank;
  // nanoseconds the CTAs spent in the step barrier's wait, summed over CTAs
  // and steps (a diagnostic; null: not counted)
  unsigned long long *wait_ns;
};

// Bound of the step barrier's wait: far above any step (milliseconds); a
// peer that never arrives makes the step flag PF_DEVERR_WAIT_TIMEOUT and go on.
constexpr uint64_t PF_DIST_WAIT_NS = 1000000000ull;  // 1 s

// polling load: no ordering of its own (an acquire load per poll would
// invalidate the SM's L1 under the CTAs that are already computing); the
// waiter orders its later reads with one fence after the wait
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}


// Smallest idx in [0, m] with row_ptr[idx] >= key (row_ptr[m] >= key assumed).
// One warp, 32 probes per step: ~log32(m) dependent loads.
template <typename IT>
__device__ __forceinline__ int64_t warp_lower_bound(const IT *row_ptr, int64_t m,
                                                    int64_t key, int lane) {
  int64_t lo = 0, hi = m;
  while (lo < hi) {
    const int64_t d = hi - lo;
    const int64_t p = lo + (d * lane) / 32;
    const bool pred = (int64_t)__ldg(row_ptr + p) >= key;
    const unsigned b = __ballot_sync(0xffffffffu, pred);
    if (b & 1u) {
      hi = lo;  // answer is lo
      break;
    }
    if (b == 0u) {
      lo = lo + (d * 31) / 32 + 1;
    } else {
      const int f = __ffs(b) - 1;  // first probe with pred true (f >= 1)
      const int64_t pf = lo + (d * f) / 32;
      lo = lo + (d * (f - 1)) / 32 + 1;
      hi = pf;
    }
  }
  return lo;
}

// Deposit this CTA's partial for a cut row and, if it is the last participant
// to arrive, finish the row: sum partials in CTA order and write y.
template <typename VT, typename IT>
__device__ void contribute_cut_row(const SpmvParams<VT, IT> &P, int64_t base,
                                   int64_t R, bool as_head, int64_t c,
                                   double v) {
  if (as_head) P.carry_head[c] = v;
  else P.carry_tail[c] = v;
  __threadfence();
  const int64_t rs = (int64_t)P.row_ptr[R] - base;
  const int64_t re = (int64_t)P.row_ptr[R + 1] - base;
  const int64_t k1 = rs / P.T + 1;
  const int64_t k2 = (re - 1) / P.T;
  if (k1 < 1 || k2 >= P.num_ctas || k1 > k2 || c < k1 - 1 || c > k2) {
    atomicOr(P.err, PF_DEVERR_ROWPTR);
    return;
  }
  const unsigned npart = (unsigned)(k2 - k1 + 2);
  const unsigned old = atomicAdd(P.counters + k1, 1u);
  if (old == npart - 1) {
    __threadfence();
    double sum = __ldcg(P.carry_tail + (k1 - 1));
    for (int64_t cc = k1; cc <= k2; ++cc) sum += __ldcg(P.carry_head + cc);
    double out = P.alpha * sum;
    if (P.beta != 0.0) out += P.beta * (double)P.y[R];
    P.y[R] = (VT)out;
    atomicExch(P.counters + k1, 0u);
  }
}

// V0 loader: the whole CTA copies the tile's val/col with coalesced loads.
template <typename VT, typename IT, int NT, int K, int W>
__global__ void __launch_bounds__(NT)
spmv_nnzsplit_kernel(const SpmvParams<VT, IT> P) {
  constexpr int TILE = NT * K;
  constexpr int NWARP = NT / 32;
  __shared__ VT s_val[TILE];
  __shared__ int32_t s_col[TILE];
  __shared__ IT s_E[W];          // row ends of the window rows
  __shared__ double s_y[W];      // emitted row sums of the window
  __shared__ double s_wv[NWARP];
  __shared__ int s_wf[NWARP];
  __shared__ int64_t s_meta[4];
  __shared__ double s_carry;
  __shared__ int s_jl;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int64_t c = blockIdx.x;
  const int64_t base = (int64_t)__ldg(P.row_ptr);
  // nnz must equal row_ptr[m] - row_ptr[0]: otherwise the slices would read
  // val/col outside the arrays. Every CTA checks and leaves before touching them.
  if ((int64_t)__ldg(P.row_ptr + P.m) - base != P.nnz) {
    if (tid == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
    return;
  }
  const int64_t s = base + c * P.T;
  const int64_t e = min(s + P.T, base + P.nnz);
  const bool last_cta = (c == P.num_ctas - 1);

  if (warp == 0) {
    const int64_t lb = warp_lower_bound(P.row_ptr, P.m, s, lane);
    if (lane == 0) {
      s_meta[0] = lb;
      s_meta[1] = ((int64_t)__ldg(P.row_ptr + lb) != s) ? 1 : 0;
    }
  } else if (warp == 1) {
    if (last_cta) {
      if (lane == 0) { s_meta[2] = P.m; s_meta[3] = 0; }
    } else {
      const int64_t lb2 = warp_lower_bound(P.row_ptr, P.m, e, lane);
      if (lane == 0) {
        s_meta[2] = lb2;
        s_meta[3] = ((int64_t)__ldg(P.row_ptr + lb2) != e) ? 1 : 0;
      }
    }
  }
  __syncthreads();
  if (s_meta[1] != 0 && s_meta[0] == 0) {
    // row_ptr[0] > s is impossible for a non-decreasing row_ptr
    if (tid == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
    return;
  }
  const bool head_partial = s_meta[1] != 0;
  const int64_t first_row = head_partial ? s_meta[0] - 1 : s_meta[0];
  const int64_t end_row = s_meta[2];
  const bool tail_partial = s_meta[3] != 0;
  const double alpha = P.alpha, beta = P.beta;

  int64_t g0 = s;
  int64_t r_cur = first_row;
  double carry = 0.0;

  while (true) {
    const int64_t rows_left = end_row - r_cur;
    const int nw = (int)(rows_left < (int64_t)W ? rows_left : (int64_t)W);
    for (int j = tid; j < nw; j += NT) s_E[j] = __ldg(P.row_ptr + r_cur + 1 + j);
    __syncthreads();

    if (g0 >= e) {
      // Final flush: rows [r_cur, end_row). Only the first can carry a value;
      // the others are empty rows. The last one may be cut at e.
      for (int64_t j = tid; j < rows_left; j += NT) {
        const int64_t R = r_cur + j;
        const double v = (j == 0) ? carry : 0.0;
        const bool is_head = head_partial && R == first_row;
        if (tail_partial && R == end_row - 1) {
          contribute_cut_row(P, base, R, is_head, c, v);
        } else if (is_head) {
          contribute_cut_row(P, base, R, true, c, v);
        } else {
          double out = alpha * v;
          if (beta != 0.0) out += beta * (double)P.y[R];
          P.y[R] = (VT)out;
        }
      }
      break;
    }

    int64_t g1 = min(g0 + TILE, e);
    if (nw == W) g1 = min(g1, (int64_t)s_E[W - 1]);
    if (g1 <= g0) {
      // Window holds W rows that all end at or before g0 (a run of empty
      // rows): emit them; only row 0 carries a value.
      for (int j = tid; j < W; j += NT) {
        const int64_t R = r_cur + j;
        const double v = (j == 0) ? carry : 0.0;
        if (head_partial && R == first_row) {
          contribute_cut_row(P, base, R, true, c, v);
        } else {
          double out = alpha * v;
          if (beta != 0.0) out += beta * (double)P.y[R];
          P.y[R] = (VT)out;
        }
      }
      r_cur += W;
      carry = 0.0;
      __syncthreads();
      continue;
    }

    const int tile_n = (int)(g1 - g0);
    for (int i = tid; i < tile_n; i += NT) {
      s_val[i] = P.val[g0 + i];
      s_col[i] = P.col[g0 + i];
    }
    __syncthreads();

    // ---- per-thread products -------------------------------------------------
    const int i0 = tid * K;
    const int n_items = max(0, min(K, tile_n - i0));
    double p[K];
    {
      int32_t ci[K];
      VT vv[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if (k < n_items) {
          ci[k] = s_col[i0 + k];
          vv[k] = s_val[i0 + k];
        } else {
          ci[k] = 0;
          vv[k] = VT(0);
        }
      }
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if (k < n_items && (uint64_t)(int64_t)ci[k] < (uint64_t)P.n) {
          p[k] = (double)vv[k] * (double)__ldg(P.x + ci[k]);
        } else {
          if (k < n_items) atomicOr(P.err, PF_DEVERR_BOUNDS);
          p[k] = 0.0;
        }
      }
    }

    // ---- entry row: row of item (first item - 1) = first j with E_j >= key --
    const int64_t key = (n_items > 0) ? g0 + i0 : g1;
    int j;
    {
      int lo = 0, hi = nw;  // first j in [0, nw) with s_E[j] >= key
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if ((int64_t)s_E[mid] >= key) hi = mid;
        else lo = mid + 1;
      }
      j = (tid == 0) ? 0 : lo;
    }
    const int j_entry = j;

    // ---- sequential walk over the thread's items ----------------------------
    double acc = 0.0, head_val = 0.0;
    bool has_emit = false;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if (k < n_items) {
        const int64_t g = g0 + i0 + k;
        while (j < nw && (int64_t)s_E[j] <= g) {
          if (!has_emit) {
            head_val = acc;
            has_emit = true;
          } else {
            s_y[j] = acc;
          }
          acc = 0.0;
          ++j;
        }
        acc += p[k];
      }
    }
    if (j >= nw) atomicOr(P.err, PF_DEVERR_ROWPTR);

    // ---- block segmented scan of (has_emit, acc): value after the last reset
    int f = has_emit ? 1 : 0;
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
      s_wf[warp] = f;
      s_wv[warp] = v;
    }
    __syncthreads();
    // prefix of earlier warps, starting from the CTA carry
    int pf_f = 0;
    double pf_v = carry;
    for (int w = 0; w < warp; ++w) {
      if (s_wf[w]) pf_v = s_wv[w];
      else pf_v = pf_v + s_wv[w];
      pf_f |= s_wf[w];
    }
    // inclusive value of this thread with the prefix applied
    const double incl = f ? v : pf_v + v;
    double excl = __shfl_up_sync(0xffffffffu, incl, 1);
    if (lane == 0) excl = pf_v;
    if (tid == NT - 1) {
      s_carry = incl;
      s_jl = j;
    }
    if (has_emit) {
      const int64_t R = r_cur + j_entry;
      const double hv = head_val + excl;
      if (head_partial && R == first_row) {
        contribute_cut_row(P, base, R, true, c, hv);
      } else {
        s_y[j_entry] = hv;
      }
    }
    __syncthreads();

    // ---- coalesced y write of the window rows emitted in this tile ----------
    const int jl = s_jl;
    for (int jj = tid; jj < jl; jj += NT) {
      const int64_t R = r_cur + jj;
      if (head_partial && R == first_row) continue;
      double out = alpha * s_y[jj];
      if (beta != 0.0) out += beta * (double)P.y[R];
      P.y[R] = (VT)out;
    }
    carry = s_carry;
    r_cur += jl;
    g0 = g1;
    __syncthreads();
  }
}

// y = beta*y (all rows empty, Z == 0).
template <typename VT>
__global__ void scale_rows_kernel(int64_t m, double beta, VT *__restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m;
       i += (int64_t)gridDim.x * blockDim.x) {
    y[i] = (beta != 0.0) ? (VT)(beta * (double)y[i]) : VT(0);
  }
}

}  // namespace pf
