// ROWVEC variant: rows split evenly, V lanes per row, each lane covering whole
// 16-byte-aligned blocks of 4 non-zeros (one 16-byte col load, one or two
// 16-byte val loads, four x gathers), U rows per lane group in flight, the
// next rows' bounds prefetched one step ahead. No shared memory, no barriers,
// no carries: a row is finished by the group that owns it (__shfl_xor over
// its V lanes).
//
// The blocks of a row start at floor4(row start); elements outside the row
// are masked. A block is loaded only when it holds an element of the row, and
// each 8-byte-value half only when it holds one, so every load stays inside a
// 16-byte block that contains a valid element. Requires col and val to start
// on 16-byte boundaries (the host falls back to ROWGROUP otherwise).
//
// PIPE (long rows): a lane loads its next block of each row before it
// gathers and sums the current one, so two blocks per row are in flight.
//
// Selected for regular rows (uniform 16/row, the Laplacian, banded 32/row,
// 2000/row). Correct for any CSR; an unusually long row only slows its group.
#pragma once

#include "pf_common.cuh"
#include "pf_ptx.cuh"
#include "spmv_nnzsplit.cuh"

namespace pf {

template <typename VT>
struct Block4;

template <>
struct Block4<double> {
  // elements q..q+3 (q % 4 == 0): halves loaded only when flagged
  __device__ __forceinline__ static void load(const double *v, int64_t q, bool lo, bool hi,
                                              double out[4]) {
    double2 a = make_double2(0.0, 0.0), b = make_double2(0.0, 0.0);
    if (lo) a = __ldcs(reinterpret_cast<const double2 *>(v + q));
    if (hi) b = __ldcs(reinterpret_cast<const double2 *>(v + q + 2));
    out[0] = a.x;
    out[1] = a.y;
    out[2] = b.x;
    out[3] = b.y;
  }
};

// 16-bit values (binary16, bfloat16): the block's 4 values are one 8-byte piece
template <typename H>
struct Block4Half {
  __device__ __forceinline__ static void load(const H *v, int64_t q, bool lo, bool hi, H out[4]) {
    uint2 a = make_uint2(0u, 0u);
    if (lo || hi) a = __ldcs(reinterpret_cast<const uint2 *>(v + q));
    const uint32_t w[2] = {a.x, a.y};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const unsigned short bits = (unsigned short)(w[i >> 1] >> (16 * (i & 1)));
      out[i] = half_from_bits<H>(bits);
    }
  }
};
template <>
struct Block4<__half> : Block4Half<__half> {};
template <>
struct Block4<__nv_bfloat16> : Block4Half<__nv_bfloat16> {};

template <>
struct Block4<float> {
  __device__ __forceinline__ static void load(const float *v, int64_t q, bool lo, bool hi,
                                              float out[4]) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    if (lo || hi) a = __ldcs(reinterpret_cast<const float4 *>(v + q));
    out[0] = a.x;
    out[1] = a.y;
    out[2] = a.z;
    out[3] = a.w;
  }
};

// DIST: the fused all-gather epilogue of DistOut (fp64 only).
// ||y||^2 of the CTA in a fixed order (warp shuffles, then warps in order),
// one partial per CTA; the last CTA to finish sums the partials in CTA order
// and writes the total to slot `rank` of every rank's slots. The same bits on
// every run, whatever the CTA finishing order.
template <int NTB>
__device__ __forceinline__ void dist_norm_epilogue(const DistOut &D, double nsq) {
  __shared__ double part[NTB / 32];
  __shared__ bool last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __threadfence_system();  // this thread's stores to peers before the count
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) nsq += __shfl_xor_sync(0xffffffffu, nsq, d);
  if (lane == 0) part[warp] = nsq;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < NTB / 32; ++w) t += part[w];
    D.cta_part[blockIdx.x] = t;
    __threadfence();
    last = atomicAdd(D.counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // strided partial sums in a fixed order, then the same fixed tree
  double t = 0.0;
  for (unsigned b = threadIdx.x; b < gridDim.x; b += NTB) t += __ldcg(D.cta_part + b);
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) t += __shfl_xor_sync(0xffffffffu, t, d);
  if (lane == 0) part[warp] = t;
  __syncthreads();
  if (threadIdx.x == 0) {
    double tot = 0.0;
    for (int w = 0; w < NTB / 32; ++w) tot += part[w];
    for (int p = 0; p < D.nranks; ++p) D.slots[p][D.rank] = tot;
    *D.counter = 0;
    if (D.flags) {
      // every CTA's stores are visible system-wide (each fenced before the
      // count); announce this step to every rank
      __threadfence_system();
      for (int p = 0; p < D.nranks; ++p) st_release_sys(D.flags[p] + D.rank, D.step + 1);
    }
  }
  __threadfence_system();
}

template <typename VT, typename IT, int V, int U, int NTB, int MINB = 1, bool DIST = false,
          bool PIPE = false>
__global__ void __launch_bounds__(NTB, MINB)
spmv_rowvec_kernel(const SpmvParams<VT, IT> P, const DistOut D = DistOut{}) {
  constexpr int GPW = 32 / V;  // row groups per warp
  constexpr int64_t RPW = (int64_t)GPW * U;
  // DIST: a warp takes KS consecutive steps over 32 consecutive rows (a
  // super-chunk), then jumps ahead by all warps' super-chunks, so that its 32
  // results leave as one 256-byte store per rank instead of many small ones
  // (small NVLink writes cap the all-gather near 150 GB/s per GPU). Without
  // DIST a warp jumps after every step (KS = 1), which keeps every warp busy
  // on matrices with few rows.
  constexpr int KS = (!DIST || RPW >= 32) ? 1 : (int)(32 / RPW);
  constexpr int64_t SUPER = RPW * KS;
  const int lane = threadIdx.x & 31;
  const int lig = lane & (V - 1);
  const int gw = lane / V;
  const int wib = threadIdx.x >> 5;  // warp in block
  const int64_t warp_global = (blockIdx.x * (int64_t)NTB + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * NTB) >> 5;
  const int64_t stride = nwarps * RPW;
  // first row of step k of this warp
  auto step_row = [&](int64_t k) -> int64_t {
    if (KS == 1) return warp_global * RPW + k * stride;
    return ((k / KS) * nwarps + warp_global) * SUPER + (k % KS) * RPW;
  };
  double alpha = P.alpha;
  const double beta = P.beta;
  const uint32_t n = (uint32_t)(P.n < 0xffffffffLL ? P.n : 0xffffffffLL);
  double nsq = 0.0;  // DIST: this thread's share of ||y||^2
  // DIST: the ranks' next-x pointers, read once per CTA (a row store must not
  // wait on a pointer load)
  __shared__ double *s_outs[DIST ? 64 : 1];
  __shared__ double s_wbuf[DIST ? NTB / 32 : 1][DIST ? SUPER : 1];  // a warp's super-chunk
  if (DIST) {
    if (D.flags && D.step > 0) {
      // step barrier: every rank has finished the previous step (its rows of
      // this x and its norm slot are in place), waited on by one thread
      if (threadIdx.x == 0) {
        const unsigned long long *mine = D.flags[D.rank];
        const uint64_t t0 = ptx::globaltimer_ns();
        bool late = false;
        for (int q = 0; q < D.nranks && !late; ++q) {
          while (ld_relaxed_sys(mine + q) < D.step) {
            if (ptx::globaltimer_ns() - t0 > PF_DIST_WAIT_NS) {
              atomicOr(P.err, PF_DEVERR_WAIT_TIMEOUT);
              late = true;
              break;
            }
            __nanosleep(256);
          }
        }
        __threadfence_system();  // the peers' stores before this CTA's reads
        if (D.wait_ns) atomicAdd(D.wait_ns, (unsigned long long)(ptx::globaltimer_ns() - t0));
      }
      __syncthreads();
    }
    double s = 0.0;
    for (int i = 0; i < D.nranks; ++i) s += D.prev[i];
    alpha = s > 0.0 ? 1.0 / sqrt(s) : 1.0;
    if (threadIdx.x < D.nranks) s_outs[threadIdx.x] = D.outs[threadIdx.x] + D.row_offset;
    __syncthreads();
  }

  int64_t kstep = 0;
  int64_t rb = step_row(0);
  // row bounds kept in row_ptr's own type (half the registers for int32)
  IT s[U], e[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int64_t r = rb + (int64_t)u * GPW + gw;
    s[u] = r < P.m ? __ldg(P.row_ptr + r) : IT(0);
    e[u] = r < P.m ? __ldg(P.row_ptr + r + 1) : IT(0);
  }
  for (; rb < P.m; ++kstep, rb = (KS == 1 ? rb + stride : step_row(kstep))) {
    const int64_t rbn = KS == 1 ? rb + stride : step_row(kstep + 1);
    IT ns[U], ne[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t r = rbn + (int64_t)u * GPW + gw;
      ns[u] = r < P.m ? __ldg(P.row_ptr + r) : IT(0);
      ne[u] = r < P.m ? __ldg(P.row_ptr + r + 1) : IT(0);
    }
    // each row from the 16-byte block q0 holding its first non-zero, with
    // 32-bit offsets from it (rows longer than PF_MAX_ROW_SPAN are flagged,
    // not summed)
    double acc[U];
    int64_t q0[U];
    int o[U], lo[U], len[U];
    bool skip[U];
    bool bad = false;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      acc[u] = 0.0;
      skip[u] = false;
      q0[u] = (int64_t)s[u] & ~(int64_t)3;
      lo[u] = (int)((int64_t)s[u] - q0[u]);
      const int64_t l64 = (int64_t)e[u] - q0[u];
      if (l64 > PF_MAX_ROW_SPAN) {
        if (lig == 0) atomicOr(P.err, PF_DEVERR_ROWPTR);
        skip[u] = true;
        len[u] = 0;
      } else {
        len[u] = (int)l64;
      }
      o[u] = 4 * lig;
    }
    // a lane's block at offset oo of row u: the column block and the value
    // halves that hold an element of the row
    auto load_blk = [&](int u, int oo, int4 &cb, VT (&vb)[4]) {
      const bool act = oo < len[u];
      const int64_t q = q0[u] + oo;
      cb = act ? __ldcs(reinterpret_cast<const int4 *>(P.col + q)) : make_int4(0, 0, 0, 0);
      Block4<VT>::load(P.val, q, act && oo + 1 >= lo[u], act && oo + 2 < len[u], vb);
    };
    if constexpr (PIPE) {
      // the next block's loads are issued before this block's gathers, so a
      // lane keeps two blocks of every row in flight
      int4 c4[U];
      VT v4[U][4];
#pragma unroll
      for (int u = 0; u < U; ++u) load_blk(u, o[u], c4[u], v4[u]);
      bool more = true;
      while (more) {
        int4 c4n[U];
        VT v4n[U][4];
#pragma unroll
        for (int u = 0; u < U; ++u) load_blk(u, o[u] + 4 * V, c4n[u], v4n[u]);
        VT xv[U][4];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int cc[4] = {c4[u].x, c4[u].y, c4[u].z, c4[u].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int el = o[u] + i;
            const bool use = el >= lo[u] && el < len[u];
            const bool inb = (uint32_t)cc[i] < n;
            bad |= use && !inb;
            xv[u][i] = (use && inb) ? ptx::ldg_x(P.x + cc[i]) : VT(0);
          }
        }
        more = false;
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[u] += (double)v4[u][i] * (double)xv[u][i];
          o[u] += 4 * V;
          more |= o[u] < len[u];
          c4[u] = c4n[u];
#pragma unroll
          for (int i = 0; i < 4; ++i) v4[u][i] = v4n[u][i];
        }
      }
    } else {
      bool more = true;
      while (more) {
        int4 c4[U];
        VT v4[U][4];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const bool act = o[u] < len[u];
          const int64_t q = q0[u] + o[u];
          c4[u] = act ? __ldcs(reinterpret_cast<const int4 *>(P.col + q)) : make_int4(0, 0, 0, 0);
          Block4<VT>::load(P.val, q, act && o[u] + 1 >= lo[u], act && o[u] + 2 < len[u], v4[u]);
        }
        VT xv[U][4];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int cc[4] = {c4[u].x, c4[u].y, c4[u].z, c4[u].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int el = o[u] + i;
            const bool use = el >= lo[u] && el < len[u];
            const bool inb = (uint32_t)cc[i] < n;
            bad |= use && !inb;
            xv[u][i] = (use && inb) ? ptx::ldg_x(P.x + cc[i]) : VT(0);
          }
        }
        more = false;
#pragma unroll
        for (int u = 0; u < U; ++u) {
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[u] += (double)v4[u][i] * (double)xv[u][i];
          o[u] += 4 * V;
          more |= o[u] < len[u];
        }
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
        if (r < P.m && !skip[u]) {
          if (DIST) {
            const double out = alpha * acc[u];
            nsq += out * out;
            s_wbuf[wib][(kstep % KS) * RPW + u * GPW + gw] = out;
          } else {
            double out = alpha * acc[u];
            if (beta != 0.0) out += beta * (double)P.y[r];
            P.y[r] = (VT)out;
          }
        }
      }
    }
    if (DIST && ((kstep % KS) == KS - 1 || rbn >= P.m)) {
      // the super-chunk is complete (or this warp is done): one 256-byte
      // store per rank (rows past m or not reached are not written)
      __syncwarp();
      const int64_t r0 = rb - (kstep % KS) * RPW;
      const int64_t rows = min((int64_t)SUPER, min(P.m, rb + RPW) - r0);
      for (int64_t i = lane; i < rows; i += 32) {
        const double v = s_wbuf[wib][i];
        for (int p = 0; p < D.nranks; ++p) s_outs[p][r0 + i] = v;
      }
      __syncwarp();
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      s[u] = ns[u];
      e[u] = ne[u];
    }
  }
  if (DIST) dist_norm_epilogue<NTB>(D, nsq);
}

}  // namespace pf
