// WARPSPLIT variant: equal-nnz slices, one warp per slice, no CTA barriers.
//
// The non-zeros [base, base + nnz) are cut into slices of T; warp w takes
// slices w, w + W, ... (W warps in the grid). A warp walks its slice in tiles
// of 32 * EPL non-zeros aligned to absolute multiples of that. Lane 0 streams the
// tiles' columns and values into the warp's own ring of NS shared-memory
// stages with bulk copies (cp.async.bulk, completion on one mbarrier per
// stage, every wait bounded), NS tiles ahead of the tile being summed, so the
// bytes in flight cost no registers. Lane l takes the 8 consecutive
// non-zeros [t0 + 8l, t0 + 8l + 8) of a tile from shared memory and issues
// their 8 x gathers at once.
//
// Row ends come from a window of WIN row_ptr entries in shared memory
// (E[j] = end of row rw + j). Each lane finds its first row by binary search
// in the window, sums its products row by row and writes every row that ends
// inside its range except the first; a warp segmented scan then gives each
// lane the sum flowing into its first row from the lanes before it (and from
// earlier tiles). A tile without a row end is one warp sum. When more than
// WIN rows end inside a tile, the tile is walked in several passes, one per
// window. A whole tile whose row ends are distinct (no empty row ends inside
// it) skips the search: a bit per non-zero marks the row ends, read from the
// window and past it from row_ptr, and every lane walks its products against
// its bits (the same sums in the same order).
//
// A row that starts before the slice (head) or runs past its end (tail) is
// finished by the last of its slices to deposit its partial, summing the
// partials in slice order (contribute_cut_row): the same bits on every run.
// Slice c writes the rows whose first non-zero lies in [S0, S1) and its
// cut head row; the last slice also writes the empty rows at the end.
//
// Follows the reference kernel's division of the non-zeros into equal tiles
// with rows cut at tile boundaries (src/spmv_kernel/preFreeSpMV.cu:30-561),
// without its start-row pre-pass: a slice's first row is found by a search of
// row_ptr. Requires col and val on 16-byte boundaries (the host falls back
// otherwise); each copy covers the 16-byte blocks holding the tile's
// non-zeros, so it never leaves a block that holds one of them.
#pragma once

#include "pf_common.cuh"
#include "pf_ptx.cuh"
#include "spmv_nnzsplit.cuh"
#include "spmv_tma.cuh"

namespace pf {

// first j in [0, WIN) with E[j] > key (WIN if none)
template <int WIN>
__device__ __forceinline__ int window_upper_bound(const int *E, int key) {
  int lo = 0;
#pragma unroll
  for (int step = WIN / 2; step > 0; step >>= 1) {
    if (E[lo + step - 1] <= key) lo += step;
  }
  return (E[lo] <= key) ? lo + 1 : lo;
}

template <typename VT, int WIN, int NS, int EPL = 8>
struct WarpSplitSmem {
  struct Stage {
    alignas(128) int32_t col[32 * EPL];
    alignas(128) VT val[32 * EPL];
  };
  Stage st[NS];
  int win[WIN];
  uint64_t bar[NS];
  // fast tile walk: one bit per non-zero, set where a row ends after it (a
  // row-sum buffer here would cost L1: shared memory and L1 share the SM's
  // 256 KB, and config 3 slowed from 249 to 350 us with 2 KB more per warp)
  uint32_t ends[EPL];
};

// Positions inside a slice are 32-bit offsets from its first non-zero S0
// (a slice holds fewer than 2^31 non-zeros); the window holds row ends as
// such offsets, INT_MAX for rows that never end in this slice.
template <typename VT, typename IT, int NTB, int WIN, int NS, int MINB, int EPL = 8>
__global__ void __launch_bounds__(NTB, MINB)
spmv_warpsplit_kernel(const SpmvParams<VT, IT> P) {
  constexpr int NW = NTB / 32;
  constexpr int TILE = 32 * EPL;  // 32 lanes x EPL non-zeros
  constexpr int NEVER = INT32_MAX;
  constexpr int VB = 16 / (int)sizeof(VT);  // values per 16-byte block
  using Smem = WarpSplitSmem<VT, WIN, NS, EPL>;
  extern __shared__ __align__(128) unsigned char ws_raw[];
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  Smem &S = reinterpret_cast<Smem *>(ws_raw)[wib];
  int *E = S.win;
  const int64_t base = (int64_t)__ldg(P.row_ptr);
  // nnz must equal row_ptr[m] - row_ptr[0], or slices would read outside the
  // arrays: every warp checks before touching them
  if ((int64_t)__ldg(P.row_ptr + P.m) - base != P.nnz) {
    if (threadIdx.x == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
    return;
  }
  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < NS; ++i) ptx::mbar_init(&S.bar[i], 1);
    ptx::fence_mbar_init();
  }
  __syncwarp();
  const uint64_t pol = ptx::policy_evict_first();
  const int64_t nwarps = (int64_t)gridDim.x * NW;
  const uint32_t n = (uint32_t)(P.n < 0xffffffffLL ? P.n : 0xffffffffLL);
  const double alpha = P.alpha, beta = P.beta;
  bool bad = false;
  uint32_t kk = 0;  // tiles this warp has taken from its ring so far

  auto write_row = [&](int64_t R, double v) {
    double out = alpha * v;
    if (beta != 0.0) out += beta * (double)P.y[R];
    P.y[R] = (VT)out;
  };

  for (int64_t c = (int64_t)blockIdx.x * NW + wib; c < P.num_ctas; c += nwarps) {
    const int64_t S0 = base + c * P.T;
    const int64_t S1 = min(S0 + P.T, base + P.nnz);
    const int L = (int)(S1 - S0);  // slice length; positions 0 .. L
    const bool last = c == P.num_ctas - 1;
    const int64_t T0 = S0 & ~(int64_t)(TILE - 1);  // first tile (absolute)
    const int ntiles = (int)((S1 - T0 + TILE - 1) / TILE);

    // tile i of the slice into stage s: the 16-byte blocks holding its non-zeros
    auto issue = [&](int i, int s) {
      const int64_t t0 = T0 + (int64_t)i * TILE;
      const int64_t lo = max(t0, S0), hi = min(t0 + TILE, S1);
      const int64_t ca = lo & ~(int64_t)3, cb = (hi + 3) & ~(int64_t)3;
      const int64_t va = lo & ~(int64_t)(VB - 1), vb = (hi + VB - 1) & ~(int64_t)(VB - 1);
      const uint32_t cbytes = (uint32_t)((cb - ca) * 4), vbytes = (uint32_t)((vb - va) * sizeof(VT));
      ptx::mbar_arrive_expect_tx(&S.bar[s], cbytes + vbytes);
      ptx::bulk_g2s(S.st[s].col + (ca - t0), P.col + ca, cbytes, &S.bar[s], pol);
      ptx::bulk_g2s(S.st[s].val + (va - t0), P.val + va, vbytes, &S.bar[s], pol);
    };
    if (lane == 0) {
      for (int i = 0; i < NS && i < ntiles; ++i) issue(i, (int)((kk + i) % NS));
    }

    const int64_t r0 = warp_lower_bound(P.row_ptr, P.m, S0, lane);
    const int64_t s_r0 = (int64_t)__ldg(P.row_ptr + r0);
    const bool head_partial = s_r0 > S0;  // then r0 >= 1: row r0 - 1 holds S0
    const int64_t head_row = head_partial ? r0 - 1 : -1;
    // window: E[j] = end of row rw + j; rows past m, and rows that start at or
    // after S1 (they belong to the next slice), never end here. The current
    // row (first not yet written) is rw + off.
    int off = WIN;  // nothing loaded yet: the first load starts at rw + off
    int64_t rw = (head_partial ? r0 - 1 : r0) - WIN;
    int rstart = head_partial ? -1 : (int)(s_r0 - S0);  // first non-zero of the current row
    int g = 0;                                           // first non-zero not yet summed
    double carry = 0.0;                                  // sum so far of the current row

    auto load_window = [&]() {
      rw += off;
      off = 0;
      int raw[WIN / 32];
      bool past = false;
#pragma unroll
      for (int k = 0; k < WIN / 32; ++k) {
        const int64_t j = lane + 32 * k;
        const int64_t e = rw + 1 + j <= P.m ? (int64_t)__ldg(P.row_ptr + rw + 1 + j) - S0 : NEVER;
        raw[k] = (int)min(e, (int64_t)NEVER);
        past |= raw[k] >= L;
      }
      __syncwarp();
#pragma unroll
      for (int k = 0; k < WIN / 32; ++k) E[lane + 32 * k] = raw[k];
      __syncwarp();
      if (!last && __any_sync(0xffffffffu, past)) {
        int prev[WIN / 32];
#pragma unroll
        for (int k = 0; k < WIN / 32; ++k) {
          const int j = lane + 32 * k;
          prev[k] = j > 0 ? E[j - 1] : 0;
        }
        __syncwarp();
#pragma unroll
        for (int k = 0; k < WIN / 32; ++k) {
          if (prev[k] >= L) E[lane + 32 * k] = NEVER;
        }
        __syncwarp();
      }
    };

    // One pass over the non-zeros [g, te) of the tile at tb (products p,
    // zero outside the tile's part of the slice): writes the rows whose ends
    // lie in [g, te] (the lane holding g takes the ends at g) and carries the
    // rest. MASK: the pass covers only part of the tile's non-zeros. False if
    // nothing moved (only a decreasing row_ptr).
    auto pass = [&](int tb, int te, const double(&p)[EPL], bool mask) -> bool {
      const int lo = tb + EPL * lane;
      const int a = min(max(lo, g), te), b = min(max(lo + EPL, g), te);
      const bool owner = (g - tb) / EPL == lane;
      int jj = owner ? off : window_upper_bound<WIN>(E, a);
      int nend = jj < WIN ? E[jj] : NEVER;  // next row end
      double acc = 0.0, head = 0.0;
      int first_j = -1;
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const int pos = lo + i;
        if (pos >= a && pos < b) {
          if (nend <= pos) {
            do {
              if (first_j < 0) {
                head = acc;
                first_j = jj;
              } else {
                write_row(rw + jj, acc);
              }
              acc = 0.0;
              ++jj;
              nend = jj < WIN ? E[jj] : NEVER;
            } while (nend <= pos);
          }
          acc += p[i];
        } else if (!mask) {
          acc += p[i];  // zero
        }
      }
      while (nend <= b) {  // the ends after the lane's last non-zero, up to b
        if (first_j < 0) {
          head = acc;
          first_j = jj;
        } else {
          write_row(rw + jj, acc);
        }
        acc = 0.0;
        ++jj;
        nend = jj < WIN ? E[jj] : NEVER;
      }
      // segmented scan over lanes: (ended a row, sum since its last end)
      int f = first_j >= 0 ? 1 : 0;
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
      const double incl = f ? v : carry + v;
      double excl = __shfl_up_sync(0xffffffffu, incl, 1);
      if (lane == 0) excl = carry;
      if (first_j >= 0) {
        const int64_t R = rw + first_j;
        if (R == head_row) contribute_cut_row(P, base, R, true, c, excl + head);
        else write_row(R, excl + head);
      }
      carry = __shfl_sync(0xffffffffu, incl, 31);
      const int noff = __shfl_sync(0xffffffffu, jj, 31);
      const bool moved = noff > off || te > g;
      if (noff > off) rstart = E[noff - 1];
      off = noff;
      g = te;
      return moved;
    };

    // Fast walk of a full tile whose row ends are distinct (no empty row
    // ends inside it): a bit per non-zero marks the row ends, and each lane
    // walks its EPL products without searching the window, writing the rows
    // that end inside its range (a row's number is its rank among the tile's
    // ends). Row ends past the window are read from row_ptr directly (a tile
    // of rows of one non-zero has 32 * EPL ends). The same sums in the same
    // order as pass(). False (nothing changed) when the tile does not qualify.
    auto fast_tile = [&](int tb, const double(&p)[EPL]) -> bool {
      const int tend = tb + TILE;
      if (tb < 0 || tend > L || g != tb || E[off] <= tb) return false;
      uint32_t *M = S.ends;
      if (lane < EPL) M[lane] = 0u;
      __syncwarp();
      int nend = 0;
      int last_e = tb;  // the last row end in the tile
      int prev_hi = tb;  // the end before this step's first
      for (int j0 = off;; j0 += 32) {
        const int j = j0 + lane;
        int e;
        if (j < WIN) {
          e = E[j];
        } else {
          const int64_t r1 = rw + 1 + j;
          e = r1 <= P.m ? (int)max(min((int64_t)__ldg(P.row_ptr + r1) - S0, (int64_t)NEVER),
                                   (int64_t)-1)
                        : NEVER;
        }
        const bool in = e <= tend;
        int prev = __shfl_up_sync(0xffffffffu, e, 1);
        if (lane == 0) prev = prev_hi;
        // an end outside (tb, tend] or not above the one before: not this path
        const bool odd = in && (e <= tb || e <= prev);
        if (in && e > tb) atomicOr(&M[(e - 1 - tb) >> 5], 1u << ((e - 1 - tb) & 31));
        const unsigned inb = __ballot_sync(0xffffffffu, in);
        nend += __popc(inb);
        if (__any_sync(0xffffffffu, odd) || nend > TILE) return false;
        if (inb) last_e = __shfl_sync(0xffffffffu, e, 31 - __clz(inb));
        if (!(inb >> 31)) break;
        prev_hi = __shfl_sync(0xffffffffu, e, 31);
      }
      __syncwarp();
      constexpr uint32_t LMASK = EPL >= 32 ? 0xffffffffu : ((1u << EPL) - 1u);
      const uint32_t bits = (M[(lane * EPL) >> 5] >> ((lane * EPL) & 31)) & LMASK;
      // rank of this lane's first row end among the tile's
      const int cnt = __popc(bits);
      int k = cnt;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, k, d);
        if (lane >= d) k += t;
      }
      k -= cnt;
      const int64_t R0 = rw + off;  // the row of rank 0
      double acc = 0.0, head = 0.0;
      int first = -1;
      // one step of the walk; a row that ends here and is not the lane's
      // first is written at once (its number is R0 + its rank)
      auto step = [&](int i, auto store) {
        acc += p[i];
        const bool e = (bits >> i) & 1u;
        const bool fst = e && first < 0;
        if (e && !fst) store(R0 + k, acc);
        head = fst ? acc : head;
        first = fst ? k : first;
        acc = e ? 0.0 : acc;
        k += e ? 1 : 0;
      };
      // beta is the same for the whole launch: the common beta = 0 walk
      // stores without testing it or reading y
      if (beta == 0.0) {
        VT *const yv = P.y;
#pragma unroll
        for (int i = 0; i < EPL; ++i)
          step(i, [&](int64_t R, double v) { yv[R] = (VT)(alpha * v); });
      } else {
#pragma unroll
        for (int i = 0; i < EPL; ++i) step(i, write_row);
      }
      // segmented scan over lanes, as in pass()
      int f = first >= 0 ? 1 : 0;
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
      const double incl = f ? v : carry + v;
      double excl = __shfl_up_sync(0xffffffffu, incl, 1);
      if (lane == 0) excl = carry;
      // a lane's first row is the only one that can be the slice's cut head
      if (first >= 0) {
        const int64_t R = R0 + first;
        if (R == head_row) contribute_cut_row(P, base, R, true, c, excl + head);
        else write_row(R, excl + head);
      }
      carry = __shfl_sync(0xffffffffu, incl, 31);
      __syncwarp();  // the mask is rewritten by the next tile
      off += nend;  // may pass the window: the next tile reloads it
      rstart = last_e;
      g = tend;
      return true;
    };

    // Wait for tile i of the slice (every lane waits; the outcome is made
    // the same for the whole warp). On a copy that never lands: flag it, wait
    // (bounded) for this warp's other copies in flight, and report false.
    auto wait_tile = [&](int i) -> bool {
      const uint32_t k = kk + (uint32_t)i;
      if (__all_sync(0xffffffffu,
                     ptx::mbar_wait_bounded(&S.bar[k % NS], (k / NS) & 1u, PF_WAIT_LIMIT_NS)))
        return true;
      if (lane == 0) atomicOr(P.err, PF_DEVERR_WAIT_TIMEOUT);
      for (int j = i + 1; j < ntiles && j < i + NS; ++j) {
        const uint32_t kj = kk + (uint32_t)j;
        ptx::mbar_wait_bounded(&S.bar[kj % NS], (kj / NS) & 1u, PF_WAIT_LIMIT_NS);
      }
      return false;
    };
    // x gathers of tile i (columns from its stage), issued a tile ahead of
    // its sum so that they are in flight while the previous tile is walked
    const int tb0 = (int)(T0 - S0);  // first tile base, relative (> -256)
    VT xv[EPL];
    auto gather = [&](int i) {
      const int tb = tb0 + i * TILE, lo = tb + EPL * lane;
      const int ga = max(tb, 0), gb = min(tb + TILE, L);
      const int32_t *cs = S.st[(kk + (uint32_t)i) % NS].col + EPL * lane;
      int cc[EPL];
#pragma unroll
      for (int b = 0; b < EPL / 4; ++b) {
        const int4 c4 = reinterpret_cast<const int4 *>(cs)[b];
        cc[4 * b] = c4.x;
        cc[4 * b + 1] = c4.y;
        cc[4 * b + 2] = c4.z;
        cc[4 * b + 3] = c4.w;
      }
      if (ga == tb && gb == tb + TILE) {
        // the whole tile lies in the slice
#pragma unroll
        for (int q = 0; q < EPL; ++q) {
          const bool inb = (uint32_t)cc[q] < n;
          bad |= !inb;
          xv[q] = inb ? ptx::ldg_x(P.x + cc[q]) : VT(0);
        }
      } else {
#pragma unroll
        for (int q = 0; q < EPL; ++q) {
          const bool use = lo + q >= ga && lo + q < gb;
          const bool inb = (uint32_t)cc[q] < n;
          bad |= use && !inb;
          xv[q] = (use && inb) ? ptx::ldg_x(P.x + cc[q]) : VT(0);
        }
      }
    };
    if (!wait_tile(0)) return;
    gather(0);

    bool ok = true;
    for (int i = 0; i < ntiles; ++i) {
      const int s = (int)((kk + (uint32_t)i) % NS);
      const int tb = tb0 + i * TILE;
      const int tend = min(tb + TILE, L);
      const int lo = tb + EPL * lane;
      // products of tile i (x gathered during the previous tile)
      double p[EPL];
      {
        const int ga = max(tb, 0);
        const bool full = tb >= 0 && tb + TILE <= L;
#pragma unroll
        for (int h = 0; h < EPL / VB; ++h) {
          VT vv[VB];
          if constexpr (VB == 2) {
            const double2 t = reinterpret_cast<const double2 *>(S.st[s].val + EPL * lane)[h];
            vv[0] = t.x;
            vv[1] = t.y;
          } else if constexpr (VB == 8) {
            // 16-bit values: 8 values per 16-byte piece
            const uint4 t = reinterpret_cast<const uint4 *>(S.st[s].val + EPL * lane)[h];
            const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const unsigned short bits = (unsigned short)(w[i >> 1] >> (16 * (i & 1)));
              vv[i] = half_from_bits<VT>(bits);
            }
          } else {
            const float4 t = reinterpret_cast<const float4 *>(S.st[s].val + EPL * lane)[h];
            vv[0] = t.x;
            vv[1] = t.y;
            vv[2] = t.z;
            vv[3] = t.w;
          }
          // values outside the tile's part of the slice are not copied: a
          // partial tile masks them
#pragma unroll
          for (int e = 0; e < VB; ++e) {
            const int q = VB * h + e;
            const bool use = full || (lo + q >= ga && lo + q < tend);
            p[q] = use ? (double)vv[e] * (double)xv[q] : 0.0;
          }
        }
      }
      // the stage is free again: refill it NS tiles ahead
      __syncwarp();
      if (lane == 0 && i + NS < ntiles) {
        ptx::fence_proxy_async_smem();
        issue(i + NS, s);
      }
      if (i + 1 < ntiles) {
        if (!wait_tile(i + 1)) return;
        gather(i + 1);
      }
      if (!ok) continue;  // a decreasing row_ptr: drain the ring only
      if (off >= WIN / 2) load_window();
      if (E[off] > tend) {
        // no row ends in this tile: a plain sum into the current row
        double t = 0.0;
#pragma unroll
        for (int q = 0; q < EPL; q += 8)
          t += ((p[q] + p[q + 1]) + (p[q + 2] + p[q + 3])) + ((p[q + 4] + p[q + 5]) + (p[q + 6] + p[q + 7]));
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) t += __shfl_xor_sync(0xffffffffu, t, d);
        carry += t;
        g = tend;
      } else if (!fast_tile(tb, p)) {
        const int g0 = g;
        while (g < tend) {
          if (off >= WIN / 2) load_window();
          int te = tend;
          if (E[WIN - 1] < te) te = max(E[WIN - 1], g);
          if (!pass(tb, te, p, g != g0 || te != tend)) {
            ok = false;
            break;
          }
        }
      }
    }
    kk += (uint32_t)ntiles;
    // the slice's non-zeros are summed: write the rows that end at its end,
    // hand on a row that runs past it
    while (ok && rw + off < P.m) {
      if (!last && rstart >= L) break;  // the current row belongs to the next slice
      if (off >= WIN / 2) load_window();
      if (E[off] > L) {
        if (lane == 0) contribute_cut_row(P, base, rw + off, rw + off == head_row, c, carry);
        break;
      }
      double z[EPL];
#pragma unroll
      for (int q = 0; q < EPL; ++q) z[q] = 0.0;
      ok = pass((int)((S1 & ~(int64_t)(TILE - 1)) - S0), L, z, false);
    }
    if (!ok && lane == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
  }
  if (bad) atomicOr(P.err, PF_DEVERR_BOUNDS);
}

}  // namespace pf
