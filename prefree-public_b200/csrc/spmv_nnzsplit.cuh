// Pieces shared by the kernels: the multiply's parameters, the geometry of
// equal-nnz slices (NNZROW in spmv_nnzrow.cuh, NNZSPLIT in spmv_tma.cuh) with
// the deterministic finish of rows cut by slice boundaries, the parameters of
// the fused multi-GPU epilogue (spmv_rowvec.cuh), and y = beta*y.
//
// Against the reference's preFreeSpMV_kernel + pre_start_rowPerTile
// (src/spmv_kernel/preFreeSpMV.cu:3-28, 407-561), by design:
//   * no start_row table: a slice finds its first row by a 32-ary warp
//     search of row_ptr (the reference builds start_row[] in a separate
//     pre-pass kernel, :583-602);
//   * no atomicAdd on y: a row cut by slice boundaries is finished by whichever
//     participating slice arrives last, which sums the per-slice partials in
//     slice order (the reference uses fp64 atomicAdd at :67, :91, :142, :333,
//     whose order varies run to run);
//   * alpha/beta, fp32 and 16-bit values, int64 row_ptr, row_ptr[0] != 0.
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

// Longest row (from its first 16-byte block) that the row-vector kernels
// walk with 32-bit offsets: a lane's offset runs up to two steps of 4 * V
// (at most 128 each) past the row's end, which must stay below 2^31. Longer
// rows are flagged PF_DEVERR_ROWPTR and not summed.
constexpr int64_t PF_MAX_ROW_SPAN = (int64_t)INT32_MAX - 512;

// y = beta*y (all rows empty, Z == 0).
template <typename VT>
__global__ void scale_rows_kernel(int64_t m, double beta, VT *__restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m;
       i += (int64_t)gridDim.x * blockDim.x) {
    y[i] = (beta != 0.0) ? (VT)(beta * (double)y[i]) : VT(0);
  }
}

}  // namespace pf
