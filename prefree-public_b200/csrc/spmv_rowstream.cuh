// ROWSTREAM variant: row tiles streamed into shared memory by a producer
// warp, summed by lane groups from shared memory.
//
// A tile is R consecutive rows (R = (NT/V) * rows_per_group, chosen so that
// an average tile holds ~3/4 of CAP non-zeros). The producer warp's lane 0
// streams the tile's contiguous ranges — row_ptr[r0..r0+R], val and col over
// [row_ptr[r0], row_ptr[r0+R]) — with bulk copies (cp.async.bulk, no tensor
// map, no multicast) into one of two stages, completing on the stage's
// "full" mbarrier. Consumers: groups of V lanes per row; a group reads its
// rows' col/val from shared memory (lanes on consecutive elements: no bank
// conflicts), issues all of a lane's x gathers before using them, reduces
// with __shfl_xor and stores y (consecutive groups, consecutive rows). Rows
// with more than LT non-zeros are summed afterwards by whole warps (still
// from shared memory). A tile with more than CAP non-zeros is not staged: its
// short rows are read from global memory, and rows longer than `lx_lt` are
// listed for spmv_longrow_chunks_kernel when the long-row list is enabled.
// Consumers release a stage by arriving on its "empty" mbarrier.
//
// Whole rows per tile: no carries, no atomics on y, deterministic. Every
// mbarrier wait is bounded; on expiry the kernel sets PF_DEVERR_WAIT_TIMEOUT
// and returns after waiting (bounded) for its own copies in flight.
#pragma once

#include "pf_common.cuh"
#include "pf_ptx.cuh"
#include "spmv_nnzsplit.cuh"
#include "spmv_tma.cuh"

namespace pf {

struct RowStreamCfg {
  static constexpr int NT = 256;      // consumer threads
  static constexpr int NTP = NT + 32; // + producer warp
  static constexpr int CAP = 4096;    // non-zeros per staged tile
  static constexpr int RMAX = 512;    // rows per tile at most
  static constexpr int NSTAGE = 2;
  static constexpr int MAXLONG = 64;  // in-tile long rows per stage
};

// One stage. Every bulk copy into it starts 16-byte aligned, so each array
// and the struct itself are multiples of 16 bytes, and each array has room
// for the 16-byte rounding of its copy (up to 15 bytes before the first and
// after the last element: 8 extra elements of 4 bytes or 4 of 8 bytes).
template <typename VT, typename IT>
struct alignas(128) RowStreamStage {
  VT val[RowStreamCfg::CAP + 32 / sizeof(VT)];
  int32_t col[RowStreamCfg::CAP + 8];
  IT rp[RowStreamCfg::RMAX + 1 + 32 / sizeof(IT) + (sizeof(IT) == 4 ? 3 : 1)];
};
static_assert(sizeof(RowStreamStage<double, int64_t>) % 128 == 0, "stage size");
static_assert(sizeof(((RowStreamStage<double, int64_t> *)0)->val) % 16 == 0, "val size");
static_assert(sizeof(((RowStreamStage<float, int32_t> *)0)->val) % 16 == 0, "val size");
static_assert(sizeof(((RowStreamStage<double, int64_t> *)0)->col) % 16 == 0, "col size");
static_assert(sizeof(((RowStreamStage<double, int64_t> *)0)->rp) % 16 == 0, "rp size");
static_assert(sizeof(((RowStreamStage<double, int32_t> *)0)->rp) % 16 == 0, "rp size");

template <typename VT, typename IT>
struct RowStreamSmem {
  RowStreamStage<VT, IT> st[RowStreamCfg::NSTAGE];
  int2 lrow[RowStreamCfg::NSTAGE][RowStreamCfg::MAXLONG];  // (row in tile, 0)
  uint64_t full[RowStreamCfg::NSTAGE];
  uint64_t empty[RowStreamCfg::NSTAGE];
  int64_t a[RowStreamCfg::NSTAGE];     // first non-zero of the staged tile
  int dv[RowStreamCfg::NSTAGE], dc[RowStreamCfg::NSTAGE], dr[RowStreamCfg::NSTAGE];
  int staged[RowStreamCfg::NSTAGE];    // 1: val/col in shared memory
  int nlong[RowStreamCfg::NSTAGE];
  int ok[RowStreamCfg::NSTAGE];  // per stage: a flag is rewritten only after its stage is released
};

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
    bool ok = true;
    // the tile's non-zero range is read one tile ahead, before the wait for
    // a free stage, so that load latency overlaps the consumers' work
    int64_t na = 0, nb = 0;
    if (blockIdx.x < ntiles) {
      const int64_t r0 = (int64_t)blockIdx.x * R;
      na = (int64_t)__ldg(P.row_ptr + r0);
      nb = (int64_t)__ldg(P.row_ptr + min(r0 + R, P.m));
    }
    for (int64_t t = blockIdx.x; t < ntiles && ok; t += gridDim.x, ++k) {
      const int s = (int)(k % NS);
      const int64_t a = na, b = nb;
      const int64_t tn = t + gridDim.x;
      if (tn < ntiles) {
        na = (int64_t)__ldg(P.row_ptr + tn * R);
        nb = (int64_t)__ldg(P.row_ptr + min(tn * R + R, P.m));
      }
      if (k >= NS) {
        ok = ptx::mbar_wait_bounded(&S.empty[s], (uint32_t)((k / NS - 1) & 1), PF_WAIT_LIMIT_NS);
        if (!ok) {
          atomicOr(P.err, PF_DEVERR_WAIT_TIMEOUT);
          break;
        }
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
  int64_t k = 0;
  for (int64_t t = blockIdx.x; t < ntiles; t += gridDim.x, ++k) {
    const int s = (int)(k % NS);
    if (tid == 0) {
      const bool ok =
          ptx::mbar_wait_bounded(&S.full[s], (uint32_t)((k / NS) & 1), PF_WAIT_LIMIT_NS);
      if (!ok) atomicOr(P.err, PF_DEVERR_WAIT_TIMEOUT);
      S.ok[s] = ok;
    }
    ptx::named_bar_sync(1, NT);
    if (!S.ok[s]) break;
    const RowStreamStage<VT, IT> &B = S.st[s];
    const bool staged = S.staged[s] != 0;
    const int64_t a = S.a[s];
    const int dv = S.dv[s], dc = S.dc[s], dr = S.dr[s];
    const int64_t r0 = t * R;
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
          const int q = atomicAdd(&S.nlong[s], 1);
          if (q < C::MAXLONG) S.lrow[s][q] = make_int2(j, 0);
        }
        re = rs;
        store = false;
      } else if (live && !staged && LX && len > lx_lt) {
        if (lig == 0) {
          const unsigned long long nch = (unsigned long long)((len + chunk - 1) / chunk);
          const unsigned long long old = atomicAdd(L.alloc, (1ull << 32) | nch);
          const int64_t idx = (int64_t)(old >> 32), base = (int64_t)(old & 0xffffffffull);
          if (idx < L.cap_entries && base + (int64_t)nch <= L.cap_chunks)
            L.ent[idx] = LongRowEntry{r0 + j, rs, re, base};
          else
            atomicOr(P.err, PF_DEVERR_ROWPTR);
        }
        re = rs;
        store = false;
      }
      double acc = 0.0;
      // 8 elements per lane per step, all gathers issued before use
      for (int64_t e0 = rs + lig; e0 < re; e0 += 8 * V) {
        int32_t cc[8];
        VT vv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int64_t el = e0 + (int64_t)u * V;
          const bool use = el < re;
          if (staged) {
            const int o = (int)(el - a);
            cc[u] = use ? B.col[o + dc] : 0;
            vv[u] = use ? B.val[o + dv] : VT(0);
          } else {
            cc[u] = use ? __ldg(P.col + el) : 0;
            vv[u] = use ? __ldcs(P.val + el) : VT(0);
          }
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
#pragma unroll
      for (int d = V / 2; d > 0; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d, V);
      if (lig == 0 && store) {
        const int64_t r = r0 + j;
        double out = alpha * acc;
        if (beta != 0.0) out += beta * (double)P.y[r];
        P.y[r] = (VT)out;
      }
    }

    // long rows of a staged tile: one warp per row, from shared memory
    if (staged) {
      ptx::named_bar_sync(1, NT);
      const int nl = S.nlong[s];
      const int nlist = nl < C::MAXLONG ? nl : C::MAXLONG;
      for (int q = warp; q < nlist; q += NT / 32) {
        const int j = S.lrow[s][q].x;
        const int64_t rs = (int64_t)B.rp[dr + j], re = (int64_t)B.rp[dr + j + 1];
        double acc = 0.0;
        for (int64_t e0 = rs + lane; e0 < re; e0 += 8 * 32) {
          int32_t cc[8];
          VT vv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int64_t el = e0 + (int64_t)u * 32;
            const bool use = el < re;
            const int o = (int)(el - a);
            cc[u] = use ? B.col[o + dc] : 0;
            vv[u] = use ? B.val[o + dv] : VT(0);
          }
          VT xv[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const bool use = e0 + (int64_t)u * 32 < re;
            const bool inb = (uint32_t)cc[u] < n;
            bad |= use && !inb;
            xv[u] = (use && inb) ? __ldg(P.x + cc[u]) : VT(0);
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) acc += (double)vv[u] * (double)xv[u];
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
        if (lane == 0) {
          const int64_t r = r0 + j;
          double out = alpha * acc;
          if (beta != 0.0) out += beta * (double)P.y[r];
          P.y[r] = (VT)out;
        }
      }
      // overflow (more than MAXLONG long rows in the tile): the group pass
      // skipped them, so sum them here by scanning the tile's rows
      if (nl > C::MAXLONG) {
        for (int j = warp; j < nrows; j += NT / 32) {
          const int64_t rs = (int64_t)B.rp[dr + j], re = (int64_t)B.rp[dr + j + 1];
          if (re - rs <= lt) continue;
          bool listed = false;
          for (int q = 0; q < C::MAXLONG; ++q) listed |= (S.lrow[s][q].x == j);
          if (listed) continue;
          double acc = 0.0;
          for (int64_t el = rs + lane; el < re; el += 32) {
            const int o = (int)(el - a);
            const int32_t c = B.col[o + dc];
            const bool inb = (uint32_t)c < n;
            bad |= !inb;
            acc += inb ? (double)B.val[o + dv] * (double)__ldg(P.x + c) : 0.0;
          }
#pragma unroll
          for (int d = 16; d > 0; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
          if (lane == 0) {
            const int64_t r = r0 + j;
            double out = alpha * acc;
            if (beta != 0.0) out += beta * (double)P.y[r];
            P.y[r] = (VT)out;
          }
        }
      }
    }
    ptx::mbar_arrive(&S.empty[s]);
  }
  if (bad) atomicOr(P.err, PF_DEVERR_BOUNDS);
}

}  // namespace pf
