// C-ABI of the SpMV library: handles, device-pointer entry points, host-buffer
// entry points and the variant selector. The kernels live in spmv_*.cuh.
#include <algorithm>
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "pf_common.cuh"
#include "spmv_nnzsplit.cuh"
#include "spmv_nnzrow.cuh"
#include "spmv_rowgroup.cuh"
#include "spmv_rowvec.cuh"
#include "spmv_tma.cuh"
#include "spmm_rowvec.cuh"

namespace pf {

static thread_local std::string t_last_error;
unsigned long long g_launch_count = 0;
static std::mutex g_count_mu;

void set_error(const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
}

static void count_launch(unsigned long long k = 1) {
  std::lock_guard<std::mutex> g(g_count_mu);
  g_launch_count += k;
}

void count_launches(unsigned long long k) { count_launch(k); }

// Page-locked host memory for the Matrix Market loader's output (mmio.cpp):
// host-to-device copies from it run at full PCIe speed with no staging copy.
void *pinned_alloc(size_t bytes) {
  void *p = nullptr;
  if (cudaHostAlloc(&p, bytes > 0 ? bytes : 1, cudaHostAllocDefault) != cudaSuccess) {
    cudaGetLastError();  // clear the sticky-free error state of the failed call
    return nullptr;
  }
  return p;
}

// Frees p if it is page-locked memory this process allocated through CUDA;
// false (nothing done) for any other pointer, which the caller frees itself.
bool pinned_free(void *p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (a.type != cudaMemoryTypeHost) return false;
  return cudaFreeHost(p) == cudaSuccess;
}

}  // namespace pf

// The selector's decision for one matrix.
struct pf_variant_choice {
  int variant;  // a PF_VARIANT_* other than AUTO
  int lanes;    // lanes per row for the row-group variants (ROWVEC, ROWGROUP)
};

struct pf_select_entry {
  const void *row_ptr;
  int64_t m, nnz;
  int idx_bytes;
  pf_variant_choice choice;
};

// Per-device state: the selector cache, scratch for cut-row carries and the
// long-row chunks, the fused step's norm partials, the device error word, and
// the buffers of the host-buffer entry points.
struct pf_handle_s {
  int device = 0;
  int num_sms = 0;
  int variant = PF_VARIANT_AUTO;
  // selector cache: decision per (row_ptr, m, nnz); any variant is correct
  // for any matrix, so a stale entry can only cost speed
  pf_select_entry cache[16];
  int cache_n = 0, cache_next = 0;
  int64_t *sample_dev = nullptr;
  int64_t *sample_host = nullptr;  // pinned
  int64_t slice_override = 0;  // testing knob: fixed nnz per slice (NNZSPLIT, NNZROW)
  // cut-row scratch
  double *carry = nullptr;     // 2 * cap doubles (head, tail)
  unsigned *counters = nullptr;
  int64_t cap = 0;
  bool scratch_dirty = false;
  unsigned *err = nullptr;
  // fused all-gather: per-CTA norm partials + counter (zeroed when grown)
  double *dist_part = nullptr;
  unsigned *dist_counter = nullptr;
  unsigned long long *dist_wait = nullptr;  // step-barrier wait, ns summed over CTAs
  int64_t dist_grid = 0;                    // CTAs of the last fused launch
  int64_t dist_cap = 0;
  // host-call buffers, and the copy stream and events of the pipelined
  // host call (created on first use)
  void *hbuf[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
  size_t hcap[5] = {0, 0, 0, 0, 0};
  cudaStream_t hcopy = nullptr;
  cudaEvent_t hev[17] = {};
};

namespace pf {

static pf_status ensure_scratch(pf_handle h, int64_t num_ctas, cudaStream_t st) {
  if (num_ctas > h->cap) {
    int64_t cap = std::max<int64_t>(num_ctas, 2 * h->cap);
    if (h->carry) cudaFree(h->carry);
    if (h->counters) cudaFree(h->counters);
    h->carry = nullptr;
    h->counters = nullptr;
    h->cap = 0;
    PF_CUDA_TRY(cudaMalloc(&h->carry, sizeof(double) * 2 * cap));
    PF_CUDA_TRY(cudaMalloc(&h->counters, sizeof(unsigned) * cap));
    h->cap = cap;
    h->scratch_dirty = true;
  }
  if (h->scratch_dirty) {
    PF_CUDA_TRY(cudaMemsetAsync(h->counters, 0, sizeof(unsigned) * h->cap, st));
    h->scratch_dirty = false;
  }
  return PF_OK;
}

// Kernels with more than 48 KB of dynamic shared memory need the attribute
// set on every device they run on: occupancy and attribute are set up once
// per device (0 = not yet).
constexpr int kMaxDevices = 64;

template <typename VT, typename IT>
static int tma_occupancy(int dev, size_t *smem_out) {
  using C = TmaCfgDefault;
  static int occ[kMaxDevices] = {};
  const size_t smem = sizeof(TmaSmem<VT, IT, C>);
  int &o = occ[dev % kMaxDevices];
  if (o == 0) {
    cudaFuncSetAttribute(spmv_tma_kernel<VT, IT, C>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int v = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, spmv_tma_kernel<VT, IT, C>, C::NT, smem);
    o = std::max(1, v);
  }
  *smem_out = smem;
  return o;
}

// ---- variant selection from sampled row lengths ------------------------------
static int rowgroup_lanes(double avg) {
  int v = 4;
  while (v < 32 && v < avg) v *= 2;
  return v;
}

// ROWVEC lanes: two lanes take rows of up to 16 non-zeros (two 4-element
// blocks each: measured faster than four lanes on 16-non-zero rows); longer
// rows get one block per lane up to 16 lanes (measured faster than 32 on
// 2000-non-zero rows: more rows in flight per warp)
static int rowvec_lanes(double avg) {
  if (avg <= 16.0) return 2;
  int v = 4;
  while (v < 16 && 4 * v < avg) v *= 2;
  return v;
}

constexpr int kSampleRows = 1024;

template <typename IT>
__global__ void sample_lengths_kernel(const IT *row_ptr, int64_t m, int S, int64_t *out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < S; i += gridDim.x * blockDim.x) {
    const int64_t r = (int64_t)((__int128)m * (2 * i + 1) / (2 * S));
    out[i] = (int64_t)row_ptr[r + 1] - (int64_t)row_ptr[r];
  }
}

static pf_variant_choice choose_from_stats(int64_t m, int64_t nnz, const int64_t *sample,
                                            int S) {
  const double avg = m > 0 ? (double)nnz / (double)m : 0.0;
  int64_t mx = 0;
  for (int i = 0; i < S; ++i) mx = std::max(mx, sample[i]);
  pf_variant_choice ch;
  // regular rows (the sample never strays far above the mean): whole rows per
  // lane group. Otherwise equal-nnz slices per CTA (NNZROW): on the power-law
  // config 196 us against 216 for per-warp slices walked from a row_ptr
  // window and ~430 for row groups with long rows split off, whose row
  // kernel waits on each step's longest short row.
  if (mx <= 4.0 * avg + 32.0) {
    ch.variant = PF_VARIANT_ROWVEC;
    ch.lanes = rowvec_lanes(avg);
  } else {
    ch.variant = PF_VARIANT_NNZROW;
    ch.lanes = 0;
  }
  return ch;
}

// The selector's choice refined by the value size (every value size takes
// the same kernels today; kept as the one place for such a rule). A forced
// variant is kept as it is.
static pf_variant_choice for_values(pf_handle h, pf_variant_choice ch, int value_bytes) {
  (void)h;
  (void)value_bytes;
  return ch;
}

template <typename IT>
static pf_status select_variant(pf_handle h, int64_t m, int64_t nnz, const IT *row_ptr,
                                cudaStream_t st, pf_variant_choice *out) {
  if (h->variant != PF_VARIANT_AUTO) {
    const double avg = m > 0 ? (double)nnz / (double)m : 0.0;
    *out = pf_variant_choice{h->variant, h->variant == PF_VARIANT_ROWVEC ? rowvec_lanes(avg)
                                                                          : rowgroup_lanes(avg)};
    return PF_OK;
  }
  for (int i = 0; i < h->cache_n; ++i) {
    const pf_select_entry &c = h->cache[i];
    if (c.row_ptr == row_ptr && c.m == m && c.nnz == nnz && c.idx_bytes == (int)sizeof(IT)) {
      *out = c.choice;
      return PF_OK;
    }
  }
  if (!h->sample_dev) {
    PF_CUDA_TRY(cudaMalloc(&h->sample_dev, sizeof(int64_t) * kSampleRows));
    PF_CUDA_TRY(cudaMallocHost(&h->sample_host, sizeof(int64_t) * kSampleRows));
  }
  const int S = (int)std::min<int64_t>(m, kSampleRows);
  sample_lengths_kernel<IT><<<(S + 255) / 256, 256, 0, st>>>(row_ptr, m, S, h->sample_dev);
  count_launch();
  PF_CUDA_TRY(cudaGetLastError());
  PF_CUDA_TRY(cudaMemcpyAsync(h->sample_host, h->sample_dev, sizeof(int64_t) * S,
                              cudaMemcpyDeviceToHost, st));
  PF_CUDA_TRY(cudaStreamSynchronize(st));
  *out = choose_from_stats(m, nnz, h->sample_host, S);
  pf_select_entry &c = h->cache[h->cache_next];
  c = pf_select_entry{row_ptr, m, nnz, (int)sizeof(IT), *out};
  h->cache_next = (h->cache_next + 1) % 16;
  h->cache_n = std::min(16, h->cache_n + 1);
  return PF_OK;
}

template <typename VT, typename IT>
static pf_status launch_nnzrow(pf_handle h, SpmvParams<VT, IT> prm, cudaStream_t st);
template <typename VT, typename IT>
static pf_status launch_nnzsplit_tma(pf_handle h, SpmvParams<VT, IT> prm, cudaStream_t st);

template <typename VT, typename IT, int V>
static pf_status launch_rowgroup(pf_handle h, const SpmvParams<VT, IT> &prm, cudaStream_t st) {
  constexpr int U = 4, NTB = 256;
  const int64_t rows_per_block = (int64_t)(NTB / 32) * (32 / V) * U;
  const int64_t want = ceil_div(prm.m, rows_per_block);
  const int64_t cap = (int64_t)h->num_sms * 32;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min(want, cap));
  spmv_rowgroup_kernel<VT, IT, V, U, NTB><<<grid, NTB, 0, st>>>(prm);
  count_launch();
  PF_CUDA_TRY(cudaGetLastError());
  return PF_OK;
}

// ROWVEC for long rows: 16 lanes per row, one row per lane group, and each
// lane's next block loaded before the current block's gathers (two blocks of
// the row in flight per lane), 4 CTAs per SM. Config 4 (2000 per row):
// 207.8-208.2 us against 215.1-215.9 for two rows per group without the
// early loads; 32 lanes per row, two rows per group with early loads (3
// CTAs per SM, spills) and 3-8 CTAs per SM were slower.
template <typename VT, typename IT>
static pf_status launch_rowvec_long(pf_handle h, const SpmvParams<VT, IT> &prm, cudaStream_t st) {
  constexpr int V = 16, U = 1, NTB = 256, MINB = 4;
  const int64_t rows_per_block = (int64_t)(NTB / 32) * (32 / V) * U;
  const int64_t want = ceil_div(prm.m, rows_per_block);
  const int64_t cap = (int64_t)h->num_sms * 16;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min(want, cap));
  spmv_rowvec_kernel<VT, IT, V, U, NTB, MINB, false, true><<<grid, NTB, 0, st>>>(prm);
  count_launch();
  PF_CUDA_TRY(cudaGetLastError());
  return PF_OK;
}

template <typename VT, typename IT, int V>
static pf_status launch_rowvec(pf_handle h, const SpmvParams<VT, IT> &prm, cudaStream_t st) {
  // U = 2 rows per lane group in flight, built for 4 CTAs per SM (64
  // registers): the best of a sweep over V, U and the CTA bound on configs
  // 1, 2 and 5 (rows of 128 or more non-zeros take launch_rowvec_long)
  constexpr int U = 2, NTB = 256, MINB = 4;
  const int64_t rows_per_block = (int64_t)(NTB / 32) * (32 / V) * U;
  const int64_t want = ceil_div(prm.m, rows_per_block);
  const int64_t cap = (int64_t)h->num_sms * 16;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min(want, cap));
  spmv_rowvec_kernel<VT, IT, V, U, NTB, MINB><<<grid, NTB, 0, st>>>(prm);
  count_launch();
  PF_CUDA_TRY(cudaGetLastError());
  return PF_OK;
}

template <typename IT, int V>
static pf_status launch_rowvec_dist(pf_handle h, const SpmvParams<double, IT> &prm,
                                    const DistOut &D, cudaStream_t st) {
  // 3 CTAs per SM: the fused epilogue's extra state spills at 4 (64 registers)
  constexpr int U = 2, NTB = 256, MINB = 3;
  const int64_t rows_per_block = (int64_t)(NTB / 32) * (32 / V) * U;
  const int64_t want = ceil_div(prm.m, rows_per_block);
  const int64_t cap = (int64_t)h->num_sms * 16;
  const int64_t grid = std::max<int64_t>(1, std::min(want, cap));
  if (grid > h->dist_cap) {
    if (h->dist_part) cudaFree(h->dist_part);
    h->dist_part = nullptr;
    h->dist_cap = 0;
    PF_CUDA_TRY(cudaMalloc(&h->dist_part, sizeof(double) * (size_t)grid + 256));
    h->dist_counter = (unsigned *)(h->dist_part + grid);
    h->dist_wait = (unsigned long long *)(h->dist_part + grid + 1);
    PF_CUDA_TRY(cudaMemsetAsync(h->dist_counter, 0, 16, st));
    h->dist_cap = grid;
  }
  DistOut d = D;
  d.cta_part = h->dist_part;
  d.counter = h->dist_counter;
  d.wait_ns = h->dist_wait;
  h->dist_grid = grid;
  spmv_rowvec_kernel<double, IT, V, U, NTB, MINB, true><<<(unsigned)grid, NTB, 0, st>>>(prm, d);
  count_launch();
  PF_CUDA_TRY(cudaGetLastError());
  return PF_OK;
}

template <typename IT>
static pf_status launch_dist(pf_handle h, int64_t m, int64_t n, int64_t nnz, const IT *row_ptr,
                             const int32_t *col, const double *val, const double *x,
                             const double *prev, int nranks, int rank, double *const *outs,
                             double *const *slots, int64_t row_offset,
                             unsigned long long *const *flags, unsigned long long step,
                             cudaStream_t st) {
  PF_CHECK_ARG(h != nullptr, "null handle");
  PF_CHECK_ARG(m > 0 && n > 0 && nnz > 0, "empty shard");
  PF_CHECK_ARG(row_ptr && col && val && x && prev && outs && slots, "null pointer");
  PF_CHECK_ARG(nranks >= 1 && nranks <= 64 && rank >= 0 && rank < nranks, "bad rank/nranks");
  PF_CHECK_ARG(sizeof(IT) == 8 || nnz <= INT32_MAX, "int32 row_ptr cannot index nnz");
  PF_CHECK_ARG((((uintptr_t)col | (uintptr_t)val) & 15) == 0 && ((uintptr_t)row_ptr % sizeof(IT)) == 0 &&
                   ((uintptr_t)x % 8) == 0,
               "the fused multiply needs 16-byte aligned col/val");
  int cur = 0;
  PF_CUDA_TRY(cudaGetDevice(&cur));
  PF_CHECK_ARG(cur == h->device, "handle bound to device %d, current device is %d", h->device, cur);
  SpmvParams<double, IT> prm{};
  prm.m = m;
  prm.n = n;
  prm.nnz = nnz;
  prm.row_ptr = row_ptr;
  prm.col = col;
  prm.val = val;
  prm.x = x;
  prm.y = nullptr;
  prm.alpha = 1.0;
  prm.beta = 0.0;
  prm.err = h->err;
  DistOut D{};
  D.outs = outs;
  D.slots = slots;
  D.prev = prev;
  D.row_offset = row_offset;
  D.nranks = nranks;
  D.rank = rank;
  D.flags = flags;
  D.step = step;
  switch (rowvec_lanes((double)nnz / (double)m)) {
    case 2: return launch_rowvec_dist<IT, 2>(h, prm, D, st);
    case 4: return launch_rowvec_dist<IT, 4>(h, prm, D, st);
    case 8: return launch_rowvec_dist<IT, 8>(h, prm, D, st);
    default: return launch_rowvec_dist<IT, 16>(h, prm, D, st);
  }
}

template <typename VT, typename IT>
static pf_status launch_spmv(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                             const IT *row_ptr, const int32_t *col,
                             const VT *val, double alpha, const VT *x,
                             double beta, VT *y, cudaStream_t st,
                             const pf_variant_choice *chosen = nullptr) {
  PF_CHECK_ARG(h != nullptr, "null handle");
  PF_CHECK_ARG(m >= 0 && n >= 0 && nnz >= 0, "negative size (m=%lld n=%lld nnz=%lld)",
               (long long)m, (long long)n, (long long)nnz);
  if (m == 0) return PF_OK;
  PF_CHECK_ARG(row_ptr && y, "null row_ptr or y");
  PF_CHECK_ARG(nnz == 0 || (col && val && x), "null col/val/x with nnz > 0");
  PF_CHECK_ARG(sizeof(IT) == 8 || nnz <= INT32_MAX, "int32 row_ptr cannot index nnz=%lld",
               (long long)nnz);
  PF_CHECK_ARG(n <= (int64_t)INT32_MAX + 1, "n must fit int32 column indices");
  PF_CHECK_ARG(nnz == 0 || n > 0, "nnz > 0 needs n > 0 (column indices lie in [0, n))");
  PF_CHECK_ARG(((uintptr_t)row_ptr % sizeof(IT)) == 0 && ((uintptr_t)y % sizeof(VT)) == 0 &&
                   (nnz == 0 || (((uintptr_t)col % 4) == 0 && ((uintptr_t)val % sizeof(VT)) == 0 &&
                                 ((uintptr_t)x % sizeof(VT)) == 0)),
               "arrays must be aligned to their element size");
  int cur = 0;
  PF_CUDA_TRY(cudaGetDevice(&cur));
  PF_CHECK_ARG(cur == h->device, "handle bound to device %d, current device is %d",
               h->device, cur);

  if (nnz == 0) {
    const int threads = 256;
    const int64_t blocks = std::min<int64_t>(ceil_div(m, threads), 4L * h->num_sms * 8);
    scale_rows_kernel<VT><<<(unsigned)blocks, threads, 0, st>>>(m, beta, y);
    count_launch();
    PF_CUDA_TRY(cudaGetLastError());
    return PF_OK;
  }

  pf_variant_choice ch;
  if (chosen) {
    ch = *chosen;
  } else {
    pf_status s = select_variant<IT>(h, m, nnz, row_ptr, st, &ch);
    if (s != PF_OK) return s;
  }
  ch = for_values(h, ch, (int)sizeof(VT));

  SpmvParams<VT, IT> prm;
  prm.m = m;
  prm.n = n;
  prm.nnz = nnz;
  prm.row_ptr = row_ptr;
  prm.col = col;
  prm.val = val;
  prm.x = x;
  prm.y = y;
  prm.alpha = alpha;
  prm.beta = beta;
  prm.err = h->err;
  prm.T = 0;
  prm.num_ctas = 0;
  prm.carry_head = prm.carry_tail = nullptr;
  prm.counters = nullptr;

  const bool aligned = (((uintptr_t)col | (uintptr_t)val) & 15) == 0;
  // NNZSPLIT (bulk copies) takes fp32/fp64 values on 16-byte aligned
  // col/val; NNZROW, which takes any, otherwise
  if (ch.variant == PF_VARIANT_NNZSPLIT) {
    if constexpr (sizeof(VT) >= 4) {
      if (aligned) return launch_nnzsplit_tma<VT, IT>(h, prm, st);
    }
    ch.variant = PF_VARIANT_NNZROW;
  }
  if (ch.variant == PF_VARIANT_NNZROW) return launch_nnzrow<VT, IT>(h, prm, st);
  // ROWVEC needs 16-byte aligned col/val (16-byte block loads); ROWGROUP,
  // its scalar-load form, otherwise
  if (ch.variant == PF_VARIANT_ROWVEC && !aligned) {
    ch.variant = PF_VARIANT_ROWGROUP;
    ch.lanes = rowgroup_lanes(m > 0 ? (double)nnz / (double)m : 0.0);
  }
  if (ch.variant == PF_VARIANT_ROWVEC) {
    switch (ch.lanes) {
      case 2: return launch_rowvec<VT, IT, 2>(h, prm, st);
      case 4: return launch_rowvec<VT, IT, 4>(h, prm, st);
      case 8: return launch_rowvec<VT, IT, 8>(h, prm, st);
      case 16:
        // long rows (every lane walks two blocks or more): one row per lane
        // group with the next block's loads issued ahead
        if (prm.nnz >= 128 * prm.m) return launch_rowvec_long<VT, IT>(h, prm, st);
        return launch_rowvec<VT, IT, 16>(h, prm, st);
      default: return launch_rowvec<VT, IT, 32>(h, prm, st);
    }
  }
  switch (ch.lanes) {  // ROWGROUP
    case 4: return launch_rowgroup<VT, IT, 4>(h, prm, st);
    case 8: return launch_rowgroup<VT, IT, 8>(h, prm, st);
    case 16: return launch_rowgroup<VT, IT, 16>(h, prm, st);
    default: return launch_rowgroup<VT, IT, 32>(h, prm, st);
  }
}

// NNZSPLIT: one CTA per equal-nnz slice, one wave of resident CTAs; a
// producer warp streams the slice with bulk copies (spmv_tma.cuh).
template <typename VT, typename IT>
static pf_status launch_nnzsplit_tma(pf_handle h, SpmvParams<VT, IT> prm, cudaStream_t st) {
  size_t smem = 0;
  const int occ = tma_occupancy<VT, IT>(h->device, &smem);
  const int64_t T = h->slice_override > 0
                        ? h->slice_override
                        : std::max<int64_t>(ceil_div(prm.nnz, (int64_t)h->num_sms * occ),
                                            2 * TmaCfgDefault::TILE);
  const int64_t P = ceil_div(prm.nnz, T);
  PF_CHECK_ARG(P <= INT32_MAX, "too many CTA slices");
  pf_status s = ensure_scratch(h, P, st);
  if (s != PF_OK) return s;
  prm.T = T;
  prm.num_ctas = P;
  prm.carry_head = h->carry;
  prm.carry_tail = h->carry + h->cap;
  prm.counters = h->counters;
  using C = TmaCfgDefault;
  spmv_tma_kernel<VT, IT, C><<<(unsigned)P, C::NT, smem, st>>>(prm);
  count_launch();
  PF_CUDA_TRY(cudaGetLastError());
  return PF_OK;
}

// NNZROW: one wave of resident CTAs, one equal-nnz slice each (at least one
// tile).
template <typename VT, typename IT, int KK>
static pf_status launch_nnzrow_k(pf_handle h, SpmvParams<VT, IT> prm, cudaStream_t st) {
  // one-warp CTAs, KK non-zeros per thread, pieces of more than 64 products
  // to the warp, 32 CTAs per SM: the best of a sweep over 32-256 threads,
  // 4-16 non-zeros per thread, 16-128 products per thread piece, 4-32 CTAs
  // per SM and 1-4 accumulators per piece
  constexpr int NT = 32, K = KK, LS = 64, MINB = 32;
  auto kern = spmv_nnzrow_kernel<VT, IT, NT, K, LS, MINB>;
  static int occ_dev[kMaxDevices] = {};
  int &occ = occ_dev[h->device % kMaxDevices];
  if (occ == 0) {
    int o = 0;
    PF_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kern, NT, 0));
    occ = std::max(1, o);
  }
  const int64_t ctas = (int64_t)h->num_sms * occ;
  // slices of whole 32-element runs: with row_ptr[0] = 0 every warp load of
  // 32 column or value elements then covers whole 32-byte sectors (4 and 8
  // of them) instead of straddling one more
  const int64_t T = h->slice_override > 0
                        ? h->slice_override
                        : std::max<int64_t>(ceil_div(ceil_div(prm.nnz, ctas), 32) * 32, (int64_t)NT * K);
  const int64_t P = ceil_div(prm.nnz, T);
  PF_CHECK_ARG(P <= INT32_MAX, "too many slices");
  PF_CHECK_ARG(T < INT32_MAX, "slice too long");
  pf_status s = ensure_scratch(h, P, st);
  if (s != PF_OK) return s;
  prm.T = T;
  prm.num_ctas = P;
  prm.carry_head = h->carry;
  prm.carry_tail = h->carry + h->cap;
  prm.counters = h->counters;
  kern<<<(unsigned)P, NT, 0, st>>>(prm);
  count_launch();
  PF_CUDA_TRY(cudaGetLastError());
  return PF_OK;
}

// 7 non-zeros per thread for 8-byte values, 10 for 4- and 2-byte values,
// whose next-tile elements take fewer registers (config 3, us: fp64 K = 6
// 180.1, 7 176.1, 8 178.0, 9 182.0; fp32 K = 8 163.7, 10 159.9; fp16 K = 8
// 168.4, 10 162.5; 12 and 16 non-zeros were slower)
template <typename VT, typename IT>
static pf_status launch_nnzrow(pf_handle h, SpmvParams<VT, IT> prm, cudaStream_t st) {
  if constexpr (sizeof(VT) <= 4) return launch_nnzrow_k<VT, IT, 10>(h, prm, st);
  else return launch_nnzrow_k<VT, IT, 7>(h, prm, st);
}

// The one-time work of the first multiply with a matrix: the variant choice
// from sampled row lengths (cached in the handle). Leaves the stream
// synchronised.
template <typename IT>
static pf_status prepare_matrix(pf_handle h, int64_t m, int64_t nnz, const IT *row_ptr,
                                cudaStream_t st) {
  PF_CHECK_ARG(h != nullptr, "null handle");
  if (m <= 0 || nnz <= 0) return PF_OK;
  pf_variant_choice ch;
  pf_status s = select_variant<IT>(h, m, nnz, row_ptr, st, &ch);
  if (s != PF_OK) return s;
  PF_CUDA_TRY(cudaStreamSynchronize(st));
  return PF_OK;
}

pf_status prepare_matrix_i32(pf_handle h, int64_t m, int64_t nnz, const int32_t *row_ptr,
                             cudaStream_t st) {
  return prepare_matrix<int32_t>(h, m, nnz, row_ptr, st);
}
pf_status prepare_matrix_i64(pf_handle h, int64_t m, int64_t nnz, const int64_t *row_ptr,
                             cudaStream_t st) {
  return prepare_matrix<int64_t>(h, m, nnz, row_ptr, st);
}

// ---- SpMM: k dense columns, passes of up to 8 ------------------------------
template <typename VT>
__global__ void scale_block_kernel(int64_t m, int k, double beta, VT *__restrict__ Y, int64_t ldy) {
  const int64_t total = m * (int64_t)k;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    VT *p = Y + (t / k) * ldy + (t % k);
    *p = (beta != 0.0) ? (VT)(beta * (double)*p) : VT(0);
  }
}

template <typename VT, typename IT, int V, int KC>
static void launch_spmm_pass(pf_handle h, const SpmmParams<VT, IT> &p, bool vec, cudaStream_t st) {
  constexpr int NTB = 256;
  constexpr int XB = 16 / (int)sizeof(VT);  // X values per 16-byte piece
  const int64_t rows_per_block = (int64_t)(NTB / 32) * (32 / V);
  const int64_t grid = std::max<int64_t>(1, std::min(ceil_div(p.m, rows_per_block),
                                                     (int64_t)h->num_sms * 16));
  // 16-byte X loads: aligned rows, and the pass's pieces inside each row
  const bool vx = KC >= XB && ((uintptr_t)p.X % 16) == 0 && p.ldx % XB == 0 &&
                  ((p.kc + XB - 1) / XB) * XB <= p.ldx_left;
  if (vec && vx) spmm_rowvec_kernel<VT, IT, V, KC, NTB, true, true><<<(unsigned)grid, NTB, 0, st>>>(p);
  else if (vec) spmm_rowvec_kernel<VT, IT, V, KC, NTB, true, false><<<(unsigned)grid, NTB, 0, st>>>(p);
  else spmm_rowvec_kernel<VT, IT, V, KC, NTB, false, false><<<(unsigned)grid, NTB, 0, st>>>(p);
  count_launch();
}

template <typename VT, typename IT, int V>
static void spmm_pass_kc(pf_handle h, const SpmmParams<VT, IT> &p, bool vec, cudaStream_t st) {
  if (p.kc <= 1) launch_spmm_pass<VT, IT, V, 1>(h, p, vec, st);
  else if (p.kc <= 2) launch_spmm_pass<VT, IT, V, 2>(h, p, vec, st);
  else if (p.kc <= 4) launch_spmm_pass<VT, IT, V, 4>(h, p, vec, st);
  else launch_spmm_pass<VT, IT, V, 8>(h, p, vec, st);
}

template <typename VT, typename IT>
static pf_status launch_spmm(pf_handle h, int64_t m, int64_t n, int64_t nnz, const IT *row_ptr,
                             const int32_t *col, const VT *val, int k, double alpha, const VT *X,
                             int64_t ldx, double beta, VT *Y, int64_t ldy, cudaStream_t st) {
  PF_CHECK_ARG(h != nullptr, "null handle");
  PF_CHECK_ARG(m >= 0 && n >= 0 && nnz >= 0 && k >= 0, "negative size");
  if (m == 0 || k == 0) return PF_OK;
  PF_CHECK_ARG(row_ptr && Y, "null row_ptr or Y");
  PF_CHECK_ARG(nnz == 0 || (col && val && X), "null col/val/X with nnz > 0");
  PF_CHECK_ARG(ldy >= k && (nnz == 0 || ldx >= k), "leading dimension below k");
  PF_CHECK_ARG(((uintptr_t)row_ptr % sizeof(IT)) == 0 && ((uintptr_t)Y % sizeof(VT)) == 0 &&
                   (nnz == 0 || (((uintptr_t)col % 4) == 0 && ((uintptr_t)val % sizeof(VT)) == 0 &&
                                 ((uintptr_t)X % sizeof(VT)) == 0)),
               "arrays must be aligned to their element size");
  int cur = 0;
  PF_CUDA_TRY(cudaGetDevice(&cur));
  PF_CHECK_ARG(cur == h->device, "handle bound to device %d, current device is %d",
               h->device, cur);
  if (nnz == 0) {
    const int64_t blocks = std::min<int64_t>(ceil_div(m * (int64_t)k, (int64_t)256),
                                             (int64_t)h->num_sms * 8);
    scale_block_kernel<VT><<<(unsigned)blocks, 256, 0, st>>>(m, k, beta, Y, ldy);
    count_launch();
    PF_CUDA_TRY(cudaGetLastError());
    return PF_OK;
  }
  // one contiguous column: the SpMV path (its variants and selector)
  if (k == 1 && ldx == 1 && ldy == 1)
    return launch_spmv<VT, IT>(h, m, n, nnz, row_ptr, col, val, alpha, X, beta, Y, st);
  const bool vec = (((uintptr_t)col | (uintptr_t)val) & 15) == 0;
  const int V = rowvec_lanes((double)nnz / (double)m);
  for (int j0 = 0; j0 < k; j0 += 8) {
    SpmmParams<VT, IT> p;
    p.m = m;
    p.n = n;
    p.nnz = nnz;
    p.row_ptr = row_ptr;
    p.col = col;
    p.val = val;
    p.X = X + j0;
    p.Y = Y + j0;
    p.ldx = ldx;
    p.ldy = ldy;
    p.kc = std::min(8, k - j0);
    p.ldx_left = ldx - j0;  // elements of an X row from this pass's first column
    p.alpha = alpha;
    p.beta = beta;
    p.err = h->err;
    switch (V) {
      case 2: spmm_pass_kc<VT, IT, 2>(h, p, vec, st); break;
      case 4: spmm_pass_kc<VT, IT, 4>(h, p, vec, st); break;
      case 8: spmm_pass_kc<VT, IT, 8>(h, p, vec, st); break;
      default: spmm_pass_kc<VT, IT, 16>(h, p, vec, st); break;
    }
    PF_CUDA_TRY(cudaGetLastError());
  }
  return PF_OK;
}

// The selector's choice for a matrix whose row_ptr is in host memory: the
// same evenly spaced sample of row lengths as sample_lengths_kernel.
template <typename IT>
static pf_variant_choice choose_host(pf_handle h, int64_t m, int64_t nnz, const IT *row_ptr) {
  if (h->variant != PF_VARIANT_AUTO) {
    const double avg = m > 0 ? (double)nnz / (double)m : 0.0;
    return pf_variant_choice{h->variant, h->variant == PF_VARIANT_ROWVEC ? rowvec_lanes(avg)
                                                                         : rowgroup_lanes(avg)};
  }
  const int S = (int)std::min<int64_t>(m, kSampleRows);
  int64_t sample[kSampleRows];
  for (int i = 0; i < S; ++i) {
    const int64_t r = (int64_t)((__int128)m * (2 * i + 1) / (2 * S));
    sample[i] = (int64_t)row_ptr[r + 1] - (int64_t)row_ptr[r];
  }
  return choose_from_stats(m, nnz, sample, S);
}

// Host-buffer call. x, row_ptr (and y when beta != 0) are copied first, then
// col/val in row chunks of about equal nnz, all on the handle's copy stream;
// chunk i's multiply and the copy-out of its rows of y run on the caller's
// stream as soon as chunk i has arrived, so the multiplies and the copy-out
// overlap the copy-in of the chunks after it. Returns when y is in place.
constexpr size_t kHostChunkBytes = size_t(256) << 20;
constexpr int kHostMaxChunks = 16;

// col/val bytes per chunk: 256 MB, or PF_HOST_CHUNK_BYTES (tests use small
// chunks to run the pipeline on small matrices)
static size_t host_chunk_bytes() {
  const char *e = std::getenv("PF_HOST_CHUNK_BYTES");
  if (e && *e) {
    const long long v = std::atoll(e);
    if (v > 0) return (size_t)v;
  }
  return kHostChunkBytes;
}

template <typename VT, typename IT>
static pf_status host_spmv(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                           const IT *row_ptr, const int32_t *col, const VT *val,
                           double alpha, const VT *x, double beta, VT *y,
                           cudaStream_t st) {
  PF_CHECK_ARG(h != nullptr, "null handle");
  PF_CHECK_ARG(m >= 0 && n >= 0 && nnz >= 0, "negative size");
  if (m == 0) return PF_OK;
  PF_CHECK_ARG(row_ptr && y, "null row_ptr or y");
  PF_CHECK_ARG(nnz == 0 || (col && val && x), "null col/val/x with nnz > 0");
  const int64_t base = (int64_t)row_ptr[0];
  PF_CHECK_ARG((int64_t)row_ptr[m] - base == nnz, "nnz != row_ptr[m] - row_ptr[0]");
  int cur = 0;
  PF_CUDA_TRY(cudaGetDevice(&cur));
  PF_CHECK_ARG(cur == h->device, "handle bound to device %d, current device is %d", h->device,
               cur);
  const size_t need[5] = {sizeof(IT) * (size_t)(m + 1), sizeof(int32_t) * (size_t)nnz,
                          sizeof(VT) * (size_t)nnz, sizeof(VT) * (size_t)n,
                          sizeof(VT) * (size_t)m};
  for (int i = 0; i < 5; ++i) {
    if (need[i] > h->hcap[i]) {
      if (h->hbuf[i]) cudaFree(h->hbuf[i]);
      h->hbuf[i] = nullptr;
      h->hcap[i] = 0;
      PF_CUDA_TRY(cudaMalloc(&h->hbuf[i], std::max<size_t>(need[i], 256)));
      h->hcap[i] = std::max<size_t>(need[i], 256);
    }
  }
  if (!h->hcopy) {
    PF_CUDA_TRY(cudaStreamCreateWithFlags(&h->hcopy, cudaStreamNonBlocking));
    for (int i = 0; i <= kHostMaxChunks; ++i)
      PF_CUDA_TRY(cudaEventCreateWithFlags(&h->hev[i], cudaEventDisableTiming));
  }
  IT *d_rp = (IT *)h->hbuf[0];
  int32_t *d_col = (int32_t *)h->hbuf[1];
  VT *d_val = (VT *)h->hbuf[2];
  VT *d_x = (VT *)h->hbuf[3];
  VT *d_y = (VT *)h->hbuf[4];
  const cudaStream_t cs = h->hcopy;

  // chunk boundaries: rows [r[i], r[i+1]) starting at the first row whose
  // start reaches i/C of the non-zeros
  const size_t mat_bytes = need[1] + need[2];
  const int C = (int)std::max<size_t>(1, std::min<size_t>(kHostMaxChunks, mat_bytes / host_chunk_bytes()));
  int64_t r[kHostMaxChunks + 1];
  r[0] = 0;
  for (int i = 1; i < C; ++i) {
    const int64_t target = base + (int64_t)((__int128)nnz * i / C);
    int64_t lo = r[i - 1], hi = m;  // first row with row_ptr[row] >= target
    while (lo < hi) {
      const int64_t mid = lo + (hi - lo) / 2;
      if ((int64_t)row_ptr[mid] < target) lo = mid + 1;
      else hi = mid;
    }
    r[i] = lo;
  }
  r[C] = m;
  const pf_variant_choice ch = choose_host<IT>(h, m, nnz, row_ptr);

  // the copy stream starts after the caller's earlier work on st
  PF_CUDA_TRY(cudaEventRecord(h->hev[kHostMaxChunks], st));
  PF_CUDA_TRY(cudaStreamWaitEvent(cs, h->hev[kHostMaxChunks], 0));
  pf_status status = PF_OK;
  auto fail = [&](cudaError_t e, const char *what) {
    if (e != cudaSuccess && status == PF_OK) {
      set_error("%s: %s", what, cudaGetErrorString(e));
      status = PF_ERR_CUDA;
    }
  };
  fail(cudaMemcpyAsync(d_rp, row_ptr, need[0], cudaMemcpyHostToDevice, cs), "copy row_ptr");
  if (n > 0 && nnz > 0) fail(cudaMemcpyAsync(d_x, x, need[3], cudaMemcpyHostToDevice, cs), "copy x");
  if (beta != 0.0) fail(cudaMemcpyAsync(d_y, y, need[4], cudaMemcpyHostToDevice, cs), "copy y");
  for (int i = 0; i < C && status == PF_OK; ++i) {
    const int64_t e0 = (int64_t)row_ptr[r[i]] - base, e1 = (int64_t)row_ptr[r[i + 1]] - base;
    if (e1 > e0) {
      fail(cudaMemcpyAsync(d_col + e0, col + base + e0, sizeof(int32_t) * (size_t)(e1 - e0),
                           cudaMemcpyHostToDevice, cs), "copy col");
      fail(cudaMemcpyAsync(d_val + e0, val + base + e0, sizeof(VT) * (size_t)(e1 - e0),
                           cudaMemcpyHostToDevice, cs), "copy val");
    }
    fail(cudaEventRecord(h->hev[i], cs), "record chunk event");
  }
  // Device arrays hold the slice only: shift so absolute row_ptr values land
  // at element 0 (a chunk's kernel only touches its own [row_ptr[r], row_ptr[r_end])).
  for (int i = 0; i < C && status == PF_OK; ++i) {
    const int64_t mi = r[i + 1] - r[i];
    if (mi == 0) continue;
    const int64_t nz = (int64_t)row_ptr[r[i + 1]] - (int64_t)row_ptr[r[i]];
    fail(cudaStreamWaitEvent(st, h->hev[i], 0), "wait for chunk");
    if (status != PF_OK) break;
    pf_status s = launch_spmv<VT, IT>(h, mi, n, nz, d_rp + r[i], d_col - base, d_val - base,
                                      alpha, d_x, beta, d_y + r[i], st, &ch);
    if (s != PF_OK) {
      status = s;
      break;
    }
    fail(cudaMemcpyAsync(y + r[i], d_y + r[i], sizeof(VT) * (size_t)mi, cudaMemcpyDeviceToHost, st),
         "copy y out");
  }
  // both streams drain before the buffers can be reused or y read
  const cudaError_t e1 = cudaStreamSynchronize(cs);
  const cudaError_t e2 = cudaStreamSynchronize(st);
  fail(e1, "copy stream");
  fail(e2, "stream");
  return status;
}

}  // namespace pf

using namespace pf;

extern "C" {

const char *pf_last_error(void) { return pf::t_last_error.c_str(); }
const char *pf_version(void) { return "prefree-b200 0.1 (sm_100a)"; }
uint64_t pf_launch_count(void) {
  std::lock_guard<std::mutex> g(pf::g_count_mu);
  return pf::g_launch_count;
}

pf_status pf_handle_create(pf_handle *out) {
  PF_CHECK_ARG(out != nullptr, "null out");
  *out = nullptr;
  pf_handle h = new pf_handle_s();
  cudaError_t e = cudaGetDevice(&h->device);
  if (e == cudaSuccess)
    e = cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, h->device);
  if (e == cudaSuccess) e = cudaMalloc(&h->err, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(h->err, 0, sizeof(unsigned));
  if (e != cudaSuccess) {
    set_error("pf_handle_create: %s", cudaGetErrorString(e));
    if (h->err) cudaFree(h->err);
    delete h;
    return PF_ERR_CUDA;
  }
  *out = h;
  return PF_OK;
}

pf_status pf_handle_destroy(pf_handle h) {
  if (!h) return PF_OK;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(h->device);
  if (h->carry) cudaFree(h->carry);
  if (h->counters) cudaFree(h->counters);
  if (h->err) cudaFree(h->err);
  for (int i = 0; i < 5; ++i)
    if (h->hbuf[i]) cudaFree(h->hbuf[i]);
  if (h->hcopy) {
    cudaStreamDestroy(h->hcopy);
    for (int i = 0; i <= kHostMaxChunks; ++i)
      if (h->hev[i]) cudaEventDestroy(h->hev[i]);
  }
  if (h->dist_part) cudaFree(h->dist_part);
  if (h->sample_dev) cudaFree(h->sample_dev);
  if (h->sample_host) cudaFreeHost(h->sample_host);
  cudaSetDevice(cur);
  delete h;
  return PF_OK;
}

pf_status pf_handle_set_variant(pf_handle h, int variant) {
  PF_CHECK_ARG(h != nullptr, "null handle");
  PF_CHECK_ARG(variant == PF_VARIANT_AUTO || variant == PF_VARIANT_NNZSPLIT ||
                   variant == PF_VARIANT_ROWGROUP || variant == PF_VARIANT_ROWVEC ||
                   variant == PF_VARIANT_NNZROW,
               "unknown variant %d", variant);
  h->variant = variant;
  return PF_OK;
}

pf_status pf_handle_set_slice(pf_handle h, int64_t slice_nnz) {
  PF_CHECK_ARG(h != nullptr, "null handle");
  PF_CHECK_ARG(slice_nnz >= 0, "negative slice");
  h->slice_override = slice_nnz;
  return PF_OK;
}

pf_status pf_handle_device_error(pf_handle h, uint32_t *bits, int clear) {
  PF_CHECK_ARG(h != nullptr && bits != nullptr, "null argument");
  PF_CUDA_TRY(cudaDeviceSynchronize());
  unsigned v = 0;
  PF_CUDA_TRY(cudaMemcpy(&v, h->err, sizeof(unsigned), cudaMemcpyDeviceToHost));
  *bits = v;
  if (clear && v) {
    PF_CUDA_TRY(cudaMemset(h->err, 0, sizeof(unsigned)));
    h->scratch_dirty = true;  // a failed launch may leave counters set
  }
  return PF_OK;
}

pf_status pf_handle_dist_wait(pf_handle h, uint64_t *wait_ns, int64_t *ctas, int reset) {
  PF_CHECK_ARG(h != nullptr && wait_ns != nullptr && ctas != nullptr, "null argument");
  *wait_ns = 0;
  *ctas = h->dist_grid;
  if (!h->dist_wait) return PF_OK;
  PF_CUDA_TRY(cudaDeviceSynchronize());
  unsigned long long v = 0;
  PF_CUDA_TRY(cudaMemcpy(&v, h->dist_wait, sizeof(v), cudaMemcpyDeviceToHost));
  *wait_ns = v;
  if (reset) PF_CUDA_TRY(cudaMemset(h->dist_wait, 0, sizeof(v)));
  return PF_OK;
}

pf_status pf_handle_choice_i32(pf_handle h, int64_t m, int64_t nnz, const int32_t *row_ptr,
                               int value_bytes, void *stream, int *variant, int *lanes) {
  PF_CHECK_ARG(h && variant && lanes && row_ptr && m > 0 && nnz > 0, "bad argument");
  PF_CHECK_ARG(value_bytes == 2 || value_bytes == 4 || value_bytes == 8, "bad value size");
  pf_variant_choice ch;
  pf_status s = select_variant<int32_t>(h, m, nnz, row_ptr, (cudaStream_t)stream, &ch);
  if (s != PF_OK) return s;
  ch = for_values(h, ch, value_bytes);
  *variant = ch.variant;
  *lanes = ch.lanes;
  return PF_OK;
}

pf_status pf_handle_choice_i64(pf_handle h, int64_t m, int64_t nnz, const int64_t *row_ptr,
                               int value_bytes, void *stream, int *variant, int *lanes) {
  PF_CHECK_ARG(h && variant && lanes && row_ptr && m > 0 && nnz > 0, "bad argument");
  PF_CHECK_ARG(value_bytes == 2 || value_bytes == 4 || value_bytes == 8, "bad value size");
  pf_variant_choice ch;
  pf_status s = select_variant<int64_t>(h, m, nnz, row_ptr, (cudaStream_t)stream, &ch);
  if (s != PF_OK) return s;
  ch = for_values(h, ch, value_bytes);
  *variant = ch.variant;
  *lanes = ch.lanes;
  return PF_OK;
}

#define PF_DEFINE_SPMV(SUFFIX, VT, IT)                                          \
  pf_status pf_spmv_##SUFFIX(pf_handle h, int64_t m, int64_t n, int64_t nnz,   \
                             const IT *row_ptr, const int32_t *col_idx,         \
                             const VT *val, double alpha, const VT *x,          \
                             double beta, VT *y, void *stream) {                \
    return launch_spmv<VT, IT>(h, m, n, nnz, row_ptr, col_idx, val, alpha, x,  \
                               beta, y, (cudaStream_t)stream);                 \
  }                                                                            \
  pf_status pf_spmv_host_##SUFFIX(pf_handle h, int64_t m, int64_t n,           \
                                  int64_t nnz, const IT *row_ptr,               \
                                  const int32_t *col_idx, const VT *val,        \
                                  double alpha, const VT *x, double beta,       \
                                  VT *y, void *stream) {                        \
    return host_spmv<VT, IT>(h, m, n, nnz, row_ptr, col_idx, val, alpha, x,    \
                             beta, y, (cudaStream_t)stream);                   \
  }

// 16-bit values cross the C ABI as their raw bit patterns (uint16_t)
#define PF_DEFINE_SPMV16(SUFFIX, VT, IT)                                        \
  pf_status pf_spmv_##SUFFIX(pf_handle h, int64_t m, int64_t n, int64_t nnz,   \
                             const IT *row_ptr, const int32_t *col_idx,         \
                             const uint16_t *val, double alpha,                 \
                             const uint16_t *x, double beta, uint16_t *y,       \
                             void *stream) {                                    \
    return launch_spmv<VT, IT>(h, m, n, nnz, row_ptr, col_idx,                 \
                               reinterpret_cast<const VT *>(val), alpha,        \
                               reinterpret_cast<const VT *>(x), beta,           \
                               reinterpret_cast<VT *>(y), (cudaStream_t)stream); \
  }

PF_DEFINE_SPMV16(f16_i32, __half, int32_t)
PF_DEFINE_SPMV16(f16_i64, __half, int64_t)
PF_DEFINE_SPMV16(bf16_i32, __nv_bfloat16, int32_t)
PF_DEFINE_SPMV16(bf16_i64, __nv_bfloat16, int64_t)

#define PF_DEFINE_SPMM(SUFFIX, VT, IT)                                          \
  pf_status pf_spmm_##SUFFIX(pf_handle h, int64_t m, int64_t n, int64_t nnz,   \
                             const IT *row_ptr, const int32_t *col_idx,         \
                             const VT *val, int k, double alpha, const VT *X,   \
                             int64_t ldx, double beta, VT *Y, int64_t ldy,      \
                             void *stream) {                                    \
    return launch_spmm<VT, IT>(h, m, n, nnz, row_ptr, col_idx, val, k, alpha,  \
                               X, ldx, beta, Y, ldy, (cudaStream_t)stream);    \
  }

PF_DEFINE_SPMM(f64_i32, double, int32_t)
PF_DEFINE_SPMM(f64_i64, double, int64_t)
PF_DEFINE_SPMM(f32_i32, float, int32_t)
PF_DEFINE_SPMM(f32_i64, float, int64_t)

pf_status pf_spmv_dist_f64_i64(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                               const int64_t *row_ptr, const int32_t *col_idx,
                               const double *val, const double *x, const double *prev_slots,
                               int nranks, int rank, double *const *out_ptrs,
                               double *const *slot_ptrs, int64_t row_offset,
                               uint64_t *const *flag_ptrs, uint64_t step, void *stream) {
  return launch_dist<int64_t>(h, m, n, nnz, row_ptr, col_idx, val, x, prev_slots, nranks, rank,
                              out_ptrs, slot_ptrs, row_offset,
                              reinterpret_cast<unsigned long long *const *>(flag_ptrs),
                              (unsigned long long)step, (cudaStream_t)stream);
}

pf_status pf_spmv_dist_f64_i32(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                               const int32_t *row_ptr, const int32_t *col_idx,
                               const double *val, const double *x, const double *prev_slots,
                               int nranks, int rank, double *const *out_ptrs,
                               double *const *slot_ptrs, int64_t row_offset,
                               uint64_t *const *flag_ptrs, uint64_t step, void *stream) {
  return launch_dist<int32_t>(h, m, n, nnz, row_ptr, col_idx, val, x, prev_slots, nranks, rank,
                              out_ptrs, slot_ptrs, row_offset,
                              reinterpret_cast<unsigned long long *const *>(flag_ptrs),
                              (unsigned long long)step, (cudaStream_t)stream);
}

PF_DEFINE_SPMV(f64_i32, double, int32_t)
PF_DEFINE_SPMV(f64_i64, double, int64_t)
PF_DEFINE_SPMV(f32_i32, float, int32_t)
PF_DEFINE_SPMV(f32_i64, float, int64_t)

}  // extern "C"
