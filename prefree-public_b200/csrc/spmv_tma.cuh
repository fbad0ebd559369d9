// NNZSPLIT variant, TMA-ring form (the default NNZSPLIT kernel on sm_100a).
//
// Same slice geometry, row walk, segmented scan and cut-row combine as
// spmv_nnzsplit.cuh (see the geometry notes there). What changes is how data
// reaches the consumers:
//   * one producer warp (its lane 0) streams the CTA's contiguous val, col and
//     row_ptr ranges with bulk TMA copies (cp.async.bulk, no tensor map, no
//     multicast) into three shared-memory rings, evict-first in L2, completing
//     on per-slot "full" mbarriers;
//   * NC consumer threads take tiles of <= TILE non-zeros and <= W rows from
//     the rings and release slots on per-slot "empty" mbarriers. Per tile:
//     (1) striped products val*x[col] (x evict-last in L2) into a padded
//     shared array, (2) one thread per row sums rows with at most LT items in
//     the tile, (3) one warp per row sums the longer ones; finished rows are
//     stored straight to y (consecutive threads, consecutive rows), the row
//     still open at the tile end carries its partial into the next tile;
//   * val and col have independent 16-byte alignments, each stream starts at
//     the 16-byte block holding its first element and ends at the block
//     holding its last one, so no copy touches another 16-byte block.
// Every mbarrier wait is bounded (PF_WAIT_LIMIT_NS of wall time); on expiry
// the kernel sets PF_DEVERR_WAIT_TIMEOUT, the producer waits (again bounded)
// for the copies it issued, and the CTA returns.
#pragma once

#include "pf_common.cuh"
#include "pf_ptx.cuh"
#include "spmv_nnzsplit.cuh"

namespace pf {

constexpr uint64_t PF_WAIT_LIMIT_NS = 1000000000ull;  // 1 s

struct TmaCfgDefault {
  static constexpr int NC = 256;          // consumer threads (8 warps)
  static constexpr int NT = NC + 32;      // + one producer warp
  static constexpr int K = 7;             // items per consumer thread (odd: no bank conflicts)
  static constexpr int TILE = NC * K;     // 1792 non-zeros per tile
  static constexpr int CE = 512;          // val/col elements per chunk
  static constexpr int NS = 8;            // val/col ring slots
  static constexpr int RING = CE * NS;    // 4096 elements
  static constexpr int CR = 128;          // row_ptr entries per chunk
  static constexpr int NSR = 8;           // row ring slots
  static constexpr int RINGR = CR * NSR;  // 1024 entries
  static constexpr int W = 512;           // rows per tile window
  static constexpr int LT = 24;           // longer in-tile rows go to the warp pass
  static constexpr int PROD = TILE + TILE / 32;  // padded product array
  static constexpr int MAXLONG = TILE / (LT + 1) + 1;  // rows with > LT items
  static constexpr int MINB = 3;          // CTAs per SM the kernel is built for
  static_assert(TILE + 2 * CE <= RING, "tile must fit the ring with one chunk of slack");
  static_assert(W + 2 * CR <= RINGR, "row window must fit the row ring");
};

template <typename VT, typename IT, class C>
struct TmaSmem {
  VT val[C::RING];
  int32_t col[C::RING];
  IT rows[C::RINGR];
  double prod[C::PROD];
  int4 lrow[C::MAXLONG];  // long rows of the tile: (j, a, b, complete)
  uint64_t full_z[C::NS];
  uint64_t empty_z[C::NS];
  uint64_t full_r[C::NSR];
  uint64_t empty_r[C::NSR];
  int64_t meta[4];
  int64_t g1;
  double carry;
  int nlong;
  int ncomp;
  int ok;
};

template <typename VT, typename IT, class C>
__global__ void __launch_bounds__(C::NT, C::MINB)
spmv_tma_kernel(const SpmvParams<VT, IT> P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  TmaSmem<VT, IT, C> &S = *reinterpret_cast<TmaSmem<VT, IT, C> *>(smem_raw);
  constexpr int NC = C::NC, K = C::K, TILE = C::TILE, W = C::W;
  constexpr int CE = C::CE, NS = C::NS, RING = C::RING;
  constexpr int CR = C::CR, NSR = C::NSR, RINGR = C::RINGR;
  constexpr int NWARP = NC / 32;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const bool producer = (warp == NWARP);
  const int64_t c = blockIdx.x;
  const int64_t base = (int64_t)__ldg(P.row_ptr);
  if ((int64_t)__ldg(P.row_ptr + P.m) - base != P.nnz) {
    if (tid == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
    return;
  }
  const int64_t s = base + c * P.T;
  const int64_t e = min(s + P.T, base + P.nnz);
  const bool last_cta = (c == P.num_ctas - 1);

  if (producer && lane == 0) {
    for (int i = 0; i < NS; ++i) {
      ptx::mbar_init(&S.full_z[i], 1);
      ptx::mbar_init(&S.empty_z[i], 1);
    }
    for (int i = 0; i < NSR; ++i) {
      ptx::mbar_init(&S.full_r[i], 1);
      ptx::mbar_init(&S.empty_r[i], 1);
    }
    ptx::fence_mbar_init();
  }
  if (warp == 0) {
    const int64_t lb = warp_lower_bound(P.row_ptr, P.m, s, lane);
    if (lane == 0) {
      S.meta[0] = lb;
      S.meta[1] = ((int64_t)__ldg(P.row_ptr + lb) != s) ? 1 : 0;
    }
  } else if (warp == 1) {
    if (last_cta) {
      if (lane == 0) {
        S.meta[2] = P.m;
        S.meta[3] = 0;
      }
    } else {
      const int64_t lb2 = warp_lower_bound(P.row_ptr, P.m, e, lane);
      if (lane == 0) {
        S.meta[2] = lb2;
        S.meta[3] = ((int64_t)__ldg(P.row_ptr + lb2) != e) ? 1 : 0;
      }
    }
  }
  __syncthreads();
  if (S.meta[1] != 0 && S.meta[0] == 0) {
    if (tid == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
    return;
  }
  const bool head_partial = S.meta[1] != 0;
  const int64_t first_row = head_partial ? S.meta[0] - 1 : S.meta[0];
  const int64_t end_row = S.meta[2];
  const bool tail_partial = S.meta[3] != 0;

  // ---- stream geometry (byte ranges rounded to 16-byte blocks) --------------
  const uintptr_t v_lo = (uintptr_t)(P.val + s) & ~(uintptr_t)15;
  const uintptr_t v_hi = ((uintptr_t)(P.val + e) + 15) & ~(uintptr_t)15;
  const int64_t av = s - (int64_t)(((uintptr_t)(P.val + s) & 15) / sizeof(VT));
  const uintptr_t c_lo = (uintptr_t)(P.col + s) & ~(uintptr_t)15;
  const uintptr_t c_hi = ((uintptr_t)(P.col + e) + 15) & ~(uintptr_t)15;
  const int64_t ac = s - (int64_t)(((uintptr_t)(P.col + s) & 15) / sizeof(int32_t));
  constexpr uint32_t VCB = CE * sizeof(VT), CCB = CE * sizeof(int32_t);
  const int64_t nz_chunks =
      max((int64_t)((v_hi - v_lo + VCB - 1) / VCB), (int64_t)((c_hi - c_lo + CCB - 1) / CCB));
  // row_ptr entries [first_row + 1, end_row] = the ends of rows first_row..end_row-1
  const int64_t r_idx0 = first_row + 1;
  const uintptr_t r_lo = (uintptr_t)(P.row_ptr + r_idx0) & ~(uintptr_t)15;
  const uintptr_t r_hi = ((uintptr_t)(P.row_ptr + end_row + 1) + 15) & ~(uintptr_t)15;
  const int64_t ar = r_idx0 - (int64_t)(((uintptr_t)(P.row_ptr + r_idx0) & 15) / sizeof(IT));
  constexpr uint32_t RCB = CR * sizeof(IT);
  const int64_t nr_chunks = (int64_t)((r_hi - r_lo + RCB - 1) / RCB);

  if (producer) {
    if (lane != 0) return;
    const uint64_t pol = ptx::policy_evict_first();
    int64_t kz = 0, kr = 0;
    bool ok = true;
    uint32_t idle = 0;
    uint64_t t_idle = 0;
    while (ok && (kz < nz_chunks || kr < nr_chunks)) {
      bool progressed = false;
      if (kz < nz_chunks) {
        const int slot = (int)(kz % NS);
        // the val/col ring is the one that fills up: sleep on its next slot
        // for up to ~1 us instead of spinning (the row ring is checked in
        // between, so neither ring can starve the other)
        if (kz < NS ||
            ptx::mbar_try_wait_hint(&S.empty_z[slot], (uint32_t)((kz / NS - 1) & 1), 1000u)) {
          const uintptr_t sv = v_lo + (uintptr_t)kz * VCB;
          const uintptr_t sc = c_lo + (uintptr_t)kz * CCB;
          const uint32_t bv = sv < v_hi ? (uint32_t)min((uintptr_t)VCB, v_hi - sv) : 0u;
          const uint32_t bc = sc < c_hi ? (uint32_t)min((uintptr_t)CCB, c_hi - sc) : 0u;
          ptx::mbar_arrive_expect_tx(&S.full_z[slot], bv + bc);
          if (bv) ptx::bulk_g2s(&S.val[slot * CE], (const void *)sv, bv, &S.full_z[slot], pol);
          if (bc) ptx::bulk_g2s(&S.col[slot * CE], (const void *)sc, bc, &S.full_z[slot], pol);
          ++kz;
          progressed = true;
        }
      }
      if (kr < nr_chunks) {
        const int slot = (int)(kr % NSR);
        const uint32_t par = (uint32_t)((kr / NSR - 1) & 1);
        // once the val/col stream is done, sleep on the row ring instead
        if (kr < NSR || (kz < nz_chunks ? ptx::mbar_test_wait(&S.empty_r[slot], par)
                                        : ptx::mbar_try_wait_hint(&S.empty_r[slot], par, 1000u))) {
          const uintptr_t sr = r_lo + (uintptr_t)kr * RCB;
          const uint32_t br = (uint32_t)min((uintptr_t)RCB, r_hi - sr);
          ptx::mbar_arrive_expect_tx(&S.full_r[slot], br);
          ptx::bulk_g2s(&S.rows[slot * CR], (const void *)sr, br, &S.full_r[slot], pol);
          ++kr;
          progressed = true;
        }
      }
      if (progressed) {
        idle = 0;
      } else if (++idle == 64) {
        t_idle = ptx::globaltimer_ns();
      } else if (idle > 64 && (idle & 63) == 0 &&
                 ptx::globaltimer_ns() - t_idle > PF_WAIT_LIMIT_NS) {
        atomicOr(P.err, PF_DEVERR_WAIT_TIMEOUT);
        ok = false;
      }
    }
    // every issued copy must land before the CTA's shared memory goes away
    for (int64_t k = (kz > NS ? kz - NS : 0); k < kz; ++k)
      if (!ptx::mbar_wait_bounded(&S.full_z[k % NS], (uint32_t)((k / NS) & 1), PF_WAIT_LIMIT_NS))
        atomicOr(P.err, PF_DEVERR_WAIT_TIMEOUT);
    for (int64_t k = (kr > NSR ? kr - NSR : 0); k < kr; ++k)
      if (!ptx::mbar_wait_bounded(&S.full_r[k % NSR], (uint32_t)((k / NSR) & 1), PF_WAIT_LIMIT_NS))
        atomicOr(P.err, PF_DEVERR_WAIT_TIMEOUT);
    return;
  }

  // ---------------------------- consumers ------------------------------------
  constexpr int LT = C::LT;
  const uint64_t xpol = ptx::policy_evict_last();
  const double alpha = P.alpha, beta = P.beta;
  int64_t g0 = s;
  int64_t r_cur = first_row;
  double carry = 0.0;
  int64_t z_ready = 0, r_ready = 0, z_rel = 0, r_rel = 0;  // meaningful in thread 0
  const int64_t z_off = max(av, ac);

  // finished (or still open) row j of the window with its tile value v
  auto emit = [&](int j, double v, bool complete) {
    const int64_t R = r_cur + j;
    if (!complete) {
      S.carry = v;
    } else if (head_partial && R == first_row) {
      contribute_cut_row(P, base, R, true, c, v);
    } else {
      double out = alpha * v;
      if (beta != 0.0) out += beta * (double)P.y[R];
      P.y[R] = (VT)out;
    }
  };
  auto release = [&]() {
    // thread 0: hand fully consumed chunks back to the producer
    while (z_rel < z_ready && z_off + (z_rel + 1) * CE <= g0) {
      ptx::mbar_arrive(&S.empty_z[z_rel % NS]);
      ++z_rel;
    }
    while (r_rel < r_ready && ar + (r_rel + 1) * CR <= r_cur + 1) {
      ptx::mbar_arrive(&S.empty_r[r_rel % NSR]);
      ++r_rel;
    }
  };

  while (true) {
    const int64_t rows_left = end_row - r_cur;
    const int nw = (int)(rows_left < (int64_t)W ? rows_left : (int64_t)W);
    // window row ends: E(j) = row_ptr[r_cur + 1 + j]
    const int rbase = (int)((r_cur + 1 - ar) & (RINGR - 1));
    auto E = [&](int j) -> int64_t { return (int64_t)S.rows[(rbase + j) & (RINGR - 1)]; };

    if (g0 >= e) {
      // rows left: the tail row cut at e (carries a value), then — last CTA
      // only — empty rows starting at e
      for (int64_t j = tid; j < rows_left; j += NC) {
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

    // thread 0 waits for the window's row ends, fixes the tile end g1, then
    // waits for the tile's val/col chunks
    if (tid == 0) {
      bool ok = true;
      const int64_t need_r = (r_cur + nw - ar) / CR;
      while (ok && r_ready <= need_r) {
        ok = ptx::mbar_wait_bounded(&S.full_r[r_ready % NSR], (uint32_t)((r_ready / NSR) & 1),
                                    PF_WAIT_LIMIT_NS);
        if (ok) ++r_ready;
      }
      int64_t g1 = min(g0 + TILE, e);
      if (ok && nw == W) g1 = min(g1, E(W - 1));
      if (ok && g1 > g0) {
        const int64_t need_z = max((g1 - 1 - av) / CE, (g1 - 1 - ac) / CE);
        while (ok && z_ready <= need_z) {
          ok = ptx::mbar_wait_bounded(&S.full_z[z_ready % NS], (uint32_t)((z_ready / NS) & 1),
                                      PF_WAIT_LIMIT_NS);
          if (ok) ++z_ready;
        }
      }
      if (!ok) atomicOr(P.err, PF_DEVERR_WAIT_TIMEOUT);
      S.g1 = g1;
      S.ok = ok;
    }
    ptx::named_bar_sync(1, NC);
    if (!S.ok) break;
    const int64_t g1 = S.g1;

    if (g1 <= g0) {
      // W rows that all end at or before g0 (a run of empty rows)
      for (int j = tid; j < W; j += NC) emit(j, j == 0 ? carry : 0.0, true);
      r_cur += W;
      carry = 0.0;
      ptx::named_bar_sync(1, NC);  // every consumer has read E(W-1)
      if (tid == 0) release();
      continue;
    }

    // ---- (1) products -------------------------------------------------------
    const int tile_n = (int)(g1 - g0);
    {
      const int bv = (int)((g0 - av) & (RING - 1));
      const int bc = (int)((g0 - ac) & (RING - 1));
      int32_t ci[K];
      VT vv[K];
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int i = tid + NC * k;
        const int ii = i < tile_n ? i : 0;  // clamped: always a loaded element
        ci[k] = S.col[(bc + ii) & (RING - 1)];
        vv[k] = S.val[(bv + ii) & (RING - 1)];
      }
      VT xv[K];
      bool bad = false;
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const bool inb = (uint32_t)ci[k] < (uint64_t)P.n;
        bad |= (tid + NC * k < tile_n) && !inb;
        xv[k] = ptx::ldg_hint(P.x + (inb ? ci[k] : 0), xpol);
      }
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int i = tid + NC * k;
        if (i < tile_n) {
          const bool inb = (uint32_t)ci[k] < (uint64_t)P.n;
          S.prod[i + (i >> 5)] = inb ? (double)vv[k] * (double)xv[k] : 0.0;
        }
      }
      if (bad) atomicOr(P.err, PF_DEVERR_BOUNDS);
      if (tid == 0) {
        S.nlong = 0;
        S.carry = 0.0;
      }
    }
    ptx::named_bar_sync(1, NC);

    // ---- (2) one thread per short row -----------------------------------------
    // Rows handled here: those starting before g1, plus empty rows at g1.
    // Completed rows (end <= g1) form a prefix of the window; the thread of
    // its last row records the count (0 when row 0 is still open).
    for (int j = tid; j < nw; j += NC) {
      const int64_t st = (j == 0) ? g0 : E(j - 1);
      const int64_t en = E(j);
      if (st > g1 || (st == g1 && en > g1)) break;  // starts in a later tile
      const bool complete = en <= g1;
      if (complete && (j + 1 == nw || E(j + 1) > g1)) S.ncomp = j + 1;
      if (!complete && j == 0) S.ncomp = 0;
      const int a = (int)((st > g0 ? st : g0) - g0);
      const int b = (int)((en < g1 ? en : g1) - g0);
      if (b - a > LT) {
        const int q = atomicAdd(&S.nlong, 1);
        S.lrow[q] = make_int4(j, a, b, complete ? 1 : 0);
      } else {
        double v0 = 0.0, v1 = 0.0;
        int i = a;
        for (; i + 1 < b; i += 2) {
          v0 += S.prod[i + (i >> 5)];
          v1 += S.prod[(i + 1) + ((i + 1) >> 5)];
        }
        if (i < b) v0 += S.prod[i + (i >> 5)];
        double v = v0 + v1;
        if (j == 0) v += carry;
        emit(j, v, complete);
      }
    }
    ptx::named_bar_sync(1, NC);

    // ---- (3) one warp per long row ---------------------------------------------
    {
      const int nl = S.nlong;
      for (int q = warp; q < nl; q += NWARP) {
        const int4 L = S.lrow[q];
        double v = 0.0;
        for (int i = L.y + lane; i < L.z; i += 32) v += S.prod[i + (i >> 5)];
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
        if (lane == 0) {
          if (L.x == 0) v += carry;
          emit(L.x, v, L.w != 0);
        }
      }
    }
    ptx::named_bar_sync(1, NC);
    carry = S.carry;
    r_cur += S.ncomp;
    g0 = g1;
    if (tid == 0) release();
  }
}

}  // namespace pf
