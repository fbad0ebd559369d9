// ROWSTREAM variant: row tiles streamed into shared memory by a producer
// warp; x gathered into shared memory with asynchronous copies one tile
// ahead of the row sums.
//
// A tile is R consecutive rows (R = (NT/V) * rows_per_group, chosen so that
// an average tile holds ~3/4 of CAP non-zeros). The producer warp's lane 0
// streams the tile's contiguous ranges — row_ptr[r0..r0+R], val and col over
// [row_ptr[r0], row_ptr[r0+R]) — with bulk copies (cp.async.bulk, no tensor
// map, no multicast) into one of three stages, completing on the stage's
// "full" mbarrier.
//
// Consumers, iteration k:
//   A. wait for tile k's stage, then gather x[col] for all its non-zeros
//      (striped over the threads) with 8-byte cp.async copies into a
//      shared-memory buffer: no registers are held while a whole tile's
//      gathers are in flight;
//   B. wait for tile k-1's gathers, one barrier (which also carries the
//      "every wait succeeded" vote), then groups of V lanes sum
//      val*x over their rows of tile k-1 from shared memory and store y
//      (consecutive groups, consecutive rows); rows with more than LT
//      non-zeros are summed afterwards by whole warps; finally the stage is
//      released on its "empty" mbarrier.
// So tile k's gathers are in flight while tile k-1 is summed and tile k+1 is
// being copied in. A tile with more than CAP non-zeros is not staged: its
// groups read col/val/x from global memory, and rows longer than `lx_lt` are
// listed for spmv_longrow_chunks_kernel when the long-row list is enabled.
//
// Whole rows per tile: no carries, no atomics on y, deterministic. Every
// mbarrier wait is bounded; on expiry the kernel sets PF_DEVERR_WAIT_TIMEOUT,
// waits for its own asynchronous copies, and returns.
#pragma once

#include "pf_common.cuh"
#include "pf_ptx.cuh"
#include "spmv_nnzsplit.cuh"
#include "spmv_tma.cuh"

namespace pf {

struct RowStreamCfg {
  static constexpr int NT = 256;      // consumer threads
  static constexpr int NTP = NT + 32; // + producer warp
  static constexpr int CAP = 1536;    // non-zeros per staged tile
  static constexpr int RMAX = 512;    // rows per tile at most
  static constexpr int NSTAGE = 3;    // bulk-copy stages (= gather buffers)
  static constexpr int MAXLONG = 32;  // in-tile long rows listed per tile
};

// One stage. Every bulk copy into it starts 16-byte aligned, so each array
// and the struct itself are multiples of 16 bytes, and each array has room
// for the 16-byte rounding of its copy (up to 15 bytes before the first and
// after the last element).
template <typename VT, typename IT>
struct alignas(128) RowStreamStage {
  VT val[RowStreamCfg::CAP + 32 / sizeof(VT)];
  int32_t col[RowStreamCfg::CAP + 8];
  IT rp[RowStreamCfg::RMAX + 1 + 32 / sizeof(IT) + (sizeof(IT) == 4 ? 3 : 1)];
};
static_assert(sizeof(RowStreamStage<double, int64_t>) % 128 == 0, "stage size");
static_assert(sizeof(((RowStreamStage<float, int32_t> *)0)->val) % 16 == 0, "val size");
static_assert(sizeof(((RowStreamStage<double, int64_t> *)0)->col) % 16 == 0, "col size");
static_assert(sizeof(((RowStreamStage<double, int64_t> *)0)->rp) % 16 == 0, "rp size");
static_assert(sizeof(((RowStreamStage<double, int32_t> *)0)->rp) % 16 == 0, "rp size");

template <typename VT, typename IT>
struct RowStreamSmem {
  RowStreamStage<VT, IT> st[RowStreamCfg::NSTAGE];
  VT sx[RowStreamCfg::NSTAGE][RowStreamCfg::CAP];  // gathered x, per stage
  int lrow[RowStreamCfg::NSTAGE][RowStreamCfg::MAXLONG];
  uint64_t full[RowStreamCfg::NSTAGE];
  uint64_t empty[RowStreamCfg::NSTAGE];
  int64_t a[RowStreamCfg::NSTAGE];     // first non-zero of the tile
  int dv[RowStreamCfg::NSTAGE], dc[RowStreamCfg::NSTAGE], dr[RowStreamCfg::NSTAGE];
  int staged[RowStreamCfg::NSTAGE];    // 1: val/col in shared memory
  int nlong[RowStreamCfg::NSTAGE];
};

template <typename VT>
__device__ __forceinline__ void gather_async(VT *dst, const VT *src, bool valid);
template <>
__device__ __forceinline__ void gather_async<double>(double *dst, const double *src, bool valid) {
  ptx::cp_async8(dst, src, valid);
}
template <>
__device__ __forceinline__ void gather_async<float>(float *dst, const float *src, bool valid) {
  ptx::cp_async4(dst, src, valid);
}

template <typename VT, typename IT, int V, bool LX>
__global__ void __launch_bounds__(RowStreamCfg::NTP)
spmv_rowstream_kernel(const SpmvParams<VT, IT> P, const LongRowScratch L, int rpg, int lt,
                      int64_t lx_lt, int64_t chunk) {
  using C = RowStreamCfg;
  constexpr int NT = C::NT, CAP = C::CAP, NS = C::NSTAGE;
  constexpr int GROUPS = NT / V;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  RowStreamSmem<VT, IT> &S = *reinterpret_cast<RowStreamSmem<VT, IT> *>(smem_raw);
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int R = GROUPS * rpg;
  const int64_t ntiles = ceil_div(P.m, R);
  const uint32_t n = (uint32_t)(P.n < 0xffffffffLL ? P.n : 0xffffffffLL);

  if (tid == NT) {
    for (int i = 0; i < NS; ++i) {
      ptx::mbar_init(&S.full[i], 1);
      ptx::mbar_init(&S.empty[i], NT);
    }
    ptx::fence_mbar_init();
  }
  __syncthreads();

  if (tid >= NT) {
    // ---------------- producer (lane 0 of the last warp) ----------------
    if (tid != NT) return;
    const uint64_t pol = ptx::policy_evict_first();
    int64_t k = 0;
    // the tile's non-zero range is read one tile ahead, before the wait for
    // a free stage, so that load latency overlaps the consumers' work
    int64_t na = 0, nb = 0;
    if (blockIdx.x < ntiles) {
      const int64_t r0 = (int64_t)blockIdx.x * R;
      na = (int64_t)__ldg(P.row_ptr + r0);
      nb = (int64_t)__ldg(P.row_ptr + min(r0 + R, P.m));
    }
    for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++k) {
      const int s = (int)(k % NS);
      const int64_t a = na, b = nb;
      const int64_t tn = t + gridDim.x;
      if (tn < ntiles) {
        na = (int64_t)__ldg(P.row_ptr + tn * R);
        nb = (int64_t)__ldg(P.row_ptr + min(tn * R + R, P.m));
      }
      if (k >= NS &&
          !ptx::mbar_wait_bounded(&S.empty[s], (uint32_t)((k / NS - 1) & 1), PF_WAIT_LIMIT_NS)) {
        atomicOr(P.err, PF_DEVERR_WAIT_TIMEOUT);
        break;
      }
      const int64_t r0 = t * R;
      const int64_t r1 = min(r0 + R, P.m);
      const uintptr_t rl = (uintptr_t)(P.row_ptr + r0) & ~(uintptr_t)15;
      const uintptr_t rh = ((uintptr_t)(P.row_ptr + r1 + 1) + 15) & ~(uintptr_t)15;
      S.dr[s] = (int)(((uintptr_t)(P.row_ptr + r0) & 15) / sizeof(IT));
      S.a[s] = a;
      uint32_t bytes = (uint32_t)(rh - rl);
      const bool stage = (b - a) <= CAP;
      S.staged[s] = stage ? 1 : 0;
      S.nlong[s] = 0;
      uintptr_t vl = 0, vh = 0, cl = 0, ch = 0;
      if (stage && b > a) {
        vl = (uintptr_t)(P.val + a) & ~(uintptr_t)15;
        vh = ((uintptr_t)(P.val + b) + 15) & ~(uintptr_t)15;
        cl = (uintptr_t)(P.col + a) & ~(uintptr_t)15;
        ch = ((uintptr_t)(P.col + b) + 15) & ~(uintptr_t)15;
        S.dv[s] = (int)(((uintptr_t)(P.val + a) & 15) / sizeof(VT));
        S.dc[s] = (int)(((uintptr_t)(P.col + a) & 15) / sizeof(int32_t));
        bytes += (uint32_t)(vh - vl) + (uint32_t)(ch - cl);
      }
      ptx::mbar_arrive_expect_tx(&S.full[s], bytes);
      ptx::bulk_g2s(S.st[s].rp, (const void *)rl, (uint32_t)(rh - rl), &S.full[s], pol);
      if (vh > vl) {
        ptx::bulk_g2s(S.st[s].val, (const void *)vl, (uint32_t)(vh - vl), &S.full[s], pol);
        ptx::bulk_g2s(S.st[s].col, (const void *)cl, (uint32_t)(ch - cl), &S.full[s], pol);
      }
    }
    // wait for the copies of the last stages before shared memory goes away
    for (int64_t j = (k > NS ? k - NS : 0); j < k; ++j)
      if (!ptx::mbar_wait_bounded(&S.full[j % NS], (uint32_t)((j / NS) & 1), PF_WAIT_LIMIT_NS))
        atomicOr(P.err, PF_DEVERR_WAIT_TIMEOUT);
    return;
  }

  // -------------------------- consumers --------------------------------------
  const int g = tid / V;     // group
  const int lig = tid % V;   // lane in group
  const double alpha = P.alpha, beta = P.beta;
  bool bad = false;
  auto store_row = [&](int64_t r, double acc) {
    double out = alpha * acc;
    if (beta != 0.0) out += beta * (double)P.y[r];
    P.y[r] = (VT)out;
  };

  for (int64_t k = 0;; ++k) {
    const int64_t t = (int64_t)blockIdx.x + k * gridDim.x;  // tile gathered now
    const bool have = t < ntiles;
    const bool have_prev = k > 0 && t - (int64_t)gridDim.x < ntiles;  // tile summed now
    if (!have && !have_prev) break;
    bool ok = true;
    // ---- A: tile t's stage, x gathers into shared memory ----------------------
    if (have) {
      const int s = (int)(k % NS);
      ok = ptx::mbar_wait_bounded(&S.full[s], (uint32_t)((k / NS) & 1), PF_WAIT_LIMIT_NS);
      if (ok && S.staged[s]) {
        const RowStreamStage<VT, IT> &B = S.st[s];
        const int64_t r0 = t * R;
        const int nrows = (int)(P.m - r0 < (int64_t)R ? P.m - r0 : (int64_t)R);
        const int tn = (int)((int64_t)B.rp[S.dr[s] + nrows] - S.a[s]);
        const int dc = S.dc[s];
        VT *sx = S.sx[s];
        for (int i = tid; i < tn; i += NT) {
          const int32_t c = B.col[i + dc];
          const bool inb = (uint32_t)c < n;
          bad |= !inb;
          gather_async<VT>(sx + i, P.x + (inb ? c : 0), inb);
        }
      }
    }
    ptx::cp_async_commit();
    if (!have_prev) {
      if (!ptx::named_bar_and(1, NT, ok)) {
        if (tid == 0 && ok) atomicOr(P.err, PF_DEVERR_WAIT_TIMEOUT);
        ptx::cp_async_wait<0>();
        break;
      }
      continue;
    }
    // ---- B: sum tile tp = t - gridDim.x ------------------------------------------
    ptx::cp_async_wait<1>();   // this thread's gathers for tile tp have landed
    if (!ptx::named_bar_and(1, NT, ok)) {
      if (tid == 0 && ok) atomicOr(P.err, PF_DEVERR_WAIT_TIMEOUT);
      ptx::cp_async_wait<0>();
      break;
    }
    const int sp = (int)((k - 1) % NS);
    const int64_t tp = t - gridDim.x;
    const RowStreamStage<VT, IT> &B = S.st[sp];
    const VT *sx = S.sx[sp];
    const bool staged = S.staged[sp] != 0;
    const int64_t a = S.a[sp];
    const int dv = S.dv[sp], dr = S.dr[sp];
    const int64_t r0 = tp * R;
    const int nrows = (int)(P.m - r0 < (int64_t)R ? P.m - r0 : (int64_t)R);

    for (int i = 0; i < rpg; ++i) {
      // every lane of the warp reaches the shuffles below: rows that this
      // group does not sum here just get an empty element range
      const int j = g + GROUPS * i;  // row in tile
      const bool live = j < nrows;
      int64_t rs = live ? (int64_t)B.rp[dr + j] : 0;
      int64_t re = live ? (int64_t)B.rp[dr + j + 1] : 0;
      const int64_t len = re - rs;
      bool store = live;
      if (live && staged && len > lt) {
        if (lig == 0) {
          const int q = atomicAdd(&S.nlong[sp], 1);
          if (q < C::MAXLONG) S.lrow[sp][q] = j;
        }
        re = rs;
        store = false;
      } else if (live && !staged && LX && len > lx_lt) {
        if (lig == 0) lx_publish_row(L, r0 + j, rs, re, chunk, P.err);
        re = rs;
        store = false;
      }
      double acc = 0.0;
      if (staged) {
        const int o0 = (int)(rs - a), o1 = (int)(re - a);
        double a1 = 0.0;
        int o = o0 + lig;
        for (; o + V < o1; o += 2 * V) {
          acc += (double)B.val[o + dv] * (double)sx[o];
          a1 += (double)B.val[o + V + dv] * (double)sx[o + V];
        }
        if (o < o1) acc += (double)B.val[o + dv] * (double)sx[o];
        acc += a1;
      } else {
        for (int64_t e0 = rs + lig; e0 < re; e0 += 8 * V) {
          int32_t cc[8];
          VT vv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int64_t el = e0 + (int64_t)u * V;
            const bool use = el < re;
            cc[u] = use ? __ldg(P.col + el) : 0;
            vv[u] = use ? __ldcs(P.val + el) : VT(0);
          }
          VT xv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const bool use = e0 + (int64_t)u * V < re;
            const bool inb = (uint32_t)cc[u] < n;
            bad |= use && !inb;
            xv[u] = (use && inb) ? __ldg(P.x + cc[u]) : VT(0);
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) acc += (double)vv[u] * (double)xv[u];
        }
      }
#pragma unroll
      for (int d = V / 2; d > 0; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d, V);
      if (lig == 0 && store) store_row(r0 + j, acc);
    }

    // long rows of a staged tile: one warp per row, from shared memory
    if (staged) {
      ptx::named_bar_sync(1, NT);
      const int nl = S.nlong[sp];
      const int nlist = nl < C::MAXLONG ? nl : C::MAXLONG;
      auto warp_row = [&](int j) {
        const int o0 = (int)((int64_t)B.rp[dr + j] - a), o1 = (int)((int64_t)B.rp[dr + j + 1] - a);
        double acc = 0.0;
        for (int o = o0 + lane; o < o1; o += 32) acc += (double)B.val[o + dv] * (double)sx[o];
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
        if (lane == 0) store_row(r0 + j, acc);
      };
      for (int q = warp; q < nlist; q += NT / 32) warp_row(S.lrow[sp][q]);
      if (nl > C::MAXLONG) {
        // more long rows than the list holds: find the unlisted ones
        for (int j = warp; j < nrows; j += NT / 32) {
          if ((int64_t)B.rp[dr + j + 1] - (int64_t)B.rp[dr + j] <= lt) continue;
          bool listed = false;
          for (int q = 0; q < C::MAXLONG; ++q) listed |= (S.lrow[sp][q] == j);
          if (!listed) warp_row(j);
        }
      }
    }
    ptx::mbar_arrive(&S.empty[sp]);
  }
  if (bad) atomicOr(P.err, PF_DEVERR_BOUNDS);
}

}  // namespace pf
