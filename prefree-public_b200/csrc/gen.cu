// Synthetic CSR generation entry points (host and device). See gen.cuh for the
// per-row definitions shared by both sides.
#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <vector>

#include <cub/device/device_scan.cuh>
#include <cub/device/device_segmented_sort.cuh>

#include "gen.cuh"
#include "pf_common.cuh"

namespace pf {
namespace gen {

// Power-law thresholds thr[l] = floor(2^64 (l - 0.5)^-1.1), l in [2, cap],
// computed once on the host and shared (same bits) with the device.
static std::mutex g_tab_mu;
static std::map<int64_t, std::vector<uint64_t>> g_host_tab;
static std::map<std::pair<int, int64_t>, uint64_t *> g_dev_tab;

static const std::vector<uint64_t> &host_table(int64_t cap) {
  std::lock_guard<std::mutex> g(g_tab_mu);
  auto it = g_host_tab.find(cap);
  if (it != g_host_tab.end()) return it->second;
  std::vector<uint64_t> t((size_t)cap + 1, 0);
  t[0] = ~0ULL;
  t[1] = ~0ULL;
  for (int64_t l = 2; l <= cap; ++l) {
    const double p = std::pow((double)l - 0.5, -1.1);
    t[(size_t)l] = (uint64_t)std::ldexp(p, 64);
  }
  return g_host_tab.emplace(cap, std::move(t)).first->second;
}

static pf_status device_table(int64_t cap, const uint64_t **out) {
  int dev = 0;
  PF_CUDA_TRY(cudaGetDevice(&dev));
  const std::vector<uint64_t> &h = host_table(cap);
  std::lock_guard<std::mutex> g(g_tab_mu);
  auto key = std::make_pair(dev, cap);
  auto it = g_dev_tab.find(key);
  if (it == g_dev_tab.end()) {
    uint64_t *d = nullptr;
    PF_CUDA_TRY(cudaMalloc(&d, sizeof(uint64_t) * h.size()));
    PF_CUDA_TRY(cudaMemcpy(d, h.data(), sizeof(uint64_t) * h.size(), cudaMemcpyHostToDevice));
    it = g_dev_tab.emplace(key, d).first;
  }
  *out = it->second;
  return PF_OK;
}

static int64_t len_cap(const Spec &s) { return s.k < s.n ? s.k : s.n; }

static pf_status check_spec(const pf_gen_spec *spec) {
  PF_CHECK_ARG(spec != nullptr, "null spec");
  PF_CHECK_ARG(spec->cfg >= 1 && spec->cfg <= 5, "unknown config %d", spec->cfg);
  PF_CHECK_ARG(spec->m > 0 && spec->n > 0 && spec->k > 0,
               "unresolved spec (call pf_gen_resolve)");
  PF_CHECK_ARG(spec->n <= INT32_MAX, "n must fit int32 column indices");
  PF_CHECK_ARG(spec->cfg == 3 || spec->cfg == 2 || spec->k <= spec->n,
               "k > n: rows cannot hold k distinct columns");
  return PF_OK;
}

// ---- device kernels ----------------------------------------------------------

__global__ void k_lengths(Spec s, const uint64_t *thr, int64_t r0, int64_t cnt,
                          int64_t *len) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i <= cnt;
       i += (int64_t)gridDim.x * blockDim.x)
    len[i] = (i < cnt) ? row_len(s, thr, r0 + i) : 0;
}

constexpr int kShortMax = 64;

// configs 1, 5 (and any short-row config): draw, sort, finish in registers/local
__global__ void k_cols_short(Spec s, int64_t r0, int64_t cnt, const int64_t *rp,
                             int32_t *col) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < cnt;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = r0 + i;
    const int64_t off = rp[i];
    const int64_t len = rp[i + 1] - off;
    int32_t c[kShortMax];
    for (int64_t j = 0; j < len; ++j) {
      const int32_t v = draw_col(s, r, j, len);
      int64_t q = j;
      while (q > 0 && c[q - 1] > v) {
        c[q] = c[q - 1];
        --q;
      }
      c[q] = v;
    }
    finish_row(s, c, len);
    for (int64_t j = 0; j < len; ++j) col[off + j] = c[j];
  }
}

// long-row configs: unsorted draws (sorted afterwards by a segmented sort)
__global__ void k_cols_draw(Spec s, int64_t r0, int64_t cnt, const int64_t *rp,
                            int32_t *col) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < cnt;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t off = rp[i];
    const int64_t len = rp[i + 1] - off;
    for (int64_t j = 0; j < len; ++j) col[off + j] = draw_col(s, r0 + i, j, len);
  }
}

__global__ void k_cols_finish(Spec s, int64_t cnt, const int64_t *rp,
                              const int32_t *sorted, int32_t *col) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < cnt;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t off = rp[i];
    const int64_t len = rp[i + 1] - off;
    for (int64_t j = 0; j < len; ++j) col[off + j] = (int32_t)(sorted[off + j] + j);
  }
}

template <typename VT>
__global__ void k_fill_values(Spec s, int64_t r0, int64_t cnt, const int64_t *rp,
                              int64_t gbase, int32_t *col, VT *val) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < cnt;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = r0 + i;
    const int64_t off = rp[i];
    const int64_t len = rp[i + 1] - off;
    if (s.cfg == 2) {
      int32_t c[5];
      double v[5];
      laplace_row(s, r, c, v);
      for (int64_t j = 0; j < len; ++j) {
        col[off + j] = c[j];
        val[off + j] = (VT)entry_val(s, r, j, gbase + off + j, v[j]);
      }
    } else {
      for (int64_t j = 0; j < len; ++j)
        val[off + j] = (VT)entry_val(s, r, j, gbase + off + j, 0.0);
    }
  }
}

template <typename IT>
__global__ void k_rowptr_out(int64_t cnt, const int64_t *rp, IT *out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i <= cnt;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (IT)rp[i];
}

template <typename VT>
__global__ void k_x(Spec s, int64_t c0, int64_t cnt, VT *x) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < cnt;
       i += (int64_t)gridDim.x * blockDim.x)
    x[i] = (VT)x_val(s, c0 + i);
}

static unsigned grid_for(int64_t n) {
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, 256), 148 * 64));
}

static int64_t host_count(const Spec &s, const uint64_t *thr, int64_t r0, int64_t r1) {
  if (s.cfg == 1 || s.cfg == 4 || s.cfg == 5) return (r1 - r0) * s.k;
  int64_t t = 0;
  for (int64_t r = r0; r < r1; ++r) t += row_len(s, thr, r);
  return t;
}

}  // namespace gen
}  // namespace pf

using namespace pf;
using namespace pf::gen;

extern "C" {

pf_status pf_gen_resolve(pf_gen_spec *spec) {
  PF_CHECK_ARG(spec != nullptr, "null spec");
  PF_CHECK_ARG(spec->cfg >= 1 && spec->cfg <= 5, "unknown config %d", spec->cfg);
  static const int64_t dm[6] = {0, 100000, 2048LL * 2048, 4000000, 50000, 1LL << 26};
  static const int64_t dk[6] = {0, 16, 5, kPowerLawCap, 2000, 32};
  if (spec->m <= 0) spec->m = dm[spec->cfg];
  if (spec->n <= 0) spec->n = spec->m;
  if (spec->k <= 0) spec->k = dk[spec->cfg];
  if (spec->cfg == 2) {
    const int64_t g = grid_side(spec->m);
    PF_CHECK_ARG(g * g == spec->m && spec->n == spec->m,
                 "config 2 needs a square grid (m = n = G*G)");
  }
  return PF_OK;
}

pf_status pf_gen_count(const pf_gen_spec *spec, int64_t r0, int64_t r1, int64_t *nnz) {
  pf_status st = check_spec(spec);
  if (st != PF_OK) return st;
  PF_CHECK_ARG(nnz && 0 <= r0 && r0 <= r1 && r1 <= spec->m, "bad row range");
  const Spec s = make_spec(*spec);
  const uint64_t *thr = (s.cfg == 3) ? host_table(len_cap(s)).data() : nullptr;
  *nnz = host_count(s, thr, r0, r1);
  return PF_OK;
}

pf_status pf_gen_row_lengths_host(const pf_gen_spec *spec, int64_t r0, int64_t r1,
                                  int64_t *len) {
  pf_status st = check_spec(spec);
  if (st != PF_OK) return st;
  PF_CHECK_ARG(len && 0 <= r0 && r0 <= r1 && r1 <= spec->m, "bad row range");
  const Spec s = make_spec(*spec);
  const uint64_t *thr = (s.cfg == 3) ? host_table(len_cap(s)).data() : nullptr;
  for (int64_t r = r0; r < r1; ++r) len[r - r0] = row_len(s, thr, r);
  return PF_OK;
}

pf_status pf_gen_rows_host(const pf_gen_spec *spec, int64_t r0, int64_t r1,
                           int64_t *row_ptr, int32_t *col, double *val) {
  pf_status st = check_spec(spec);
  if (st != PF_OK) return st;
  PF_CHECK_ARG(row_ptr && col && val && 0 <= r0 && r0 <= r1 && r1 <= spec->m,
               "bad arguments");
  const Spec s = make_spec(*spec);
  const uint64_t *thr = (s.cfg == 3) ? host_table(len_cap(s)).data() : nullptr;
  const int64_t gbase = (s.value_mode == 1) ? host_count(s, thr, 0, r0) : 0;
  int64_t off = 0;
  row_ptr[0] = 0;
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t len = row_len(s, thr, r);
    if (s.cfg == 2) {
      int32_t c[5];
      double v[5];
      laplace_row(s, r, c, v);
      for (int64_t j = 0; j < len; ++j) {
        col[off + j] = c[j];
        val[off + j] = entry_val(s, r, j, gbase + off + j, v[j]);
      }
    } else {
      for (int64_t j = 0; j < len; ++j) col[off + j] = draw_col(s, r, j, len);
      std::sort(col + off, col + off + len);
      finish_row(s, col + off, len);
      for (int64_t j = 0; j < len; ++j) val[off + j] = entry_val(s, r, j, gbase + off + j, 0.0);
    }
    off += len;
    row_ptr[r - r0 + 1] = off;
  }
  return PF_OK;
}

pf_status pf_gen_x_host(const pf_gen_spec *spec, int64_t c0, int64_t c1, double *x) {
  pf_status st = check_spec(spec);
  if (st != PF_OK) return st;
  PF_CHECK_ARG(x && 0 <= c0 && c0 <= c1 && c1 <= spec->n, "bad column range");
  const Spec s = make_spec(*spec);
  for (int64_t c = c0; c < c1; ++c) x[c - c0] = x_val(s, c);
  return PF_OK;
}

pf_status pf_gen_rows_device(const pf_gen_spec *spec, int64_t r0, int64_t r1,
                             int index_bytes, void *row_ptr, int32_t *col,
                             int value_bytes, void *val, void *stream) {
  pf_status st = check_spec(spec);
  if (st != PF_OK) return st;
  PF_CHECK_ARG(row_ptr && 0 <= r0 && r0 <= r1 && r1 <= spec->m, "bad arguments");
  PF_CHECK_ARG(index_bytes == 4 || index_bytes == 8, "index_bytes must be 4 or 8");
  PF_CHECK_ARG(value_bytes == 4 || value_bytes == 8, "value_bytes must be 4 or 8");
  cudaStream_t cs = (cudaStream_t)stream;
  const Spec s = make_spec(*spec);
  const uint64_t *thr_d = nullptr;
  const uint64_t *thr_h = nullptr;
  if (s.cfg == 3) {
    thr_h = host_table(len_cap(s)).data();
    st = device_table(len_cap(s), &thr_d);
    if (st != PF_OK) return st;
  }
  const int64_t cnt = r1 - r0;
  const int64_t nnz = host_count(s, thr_h, r0, r1);
  PF_CHECK_ARG(index_bytes == 8 || nnz <= INT32_MAX, "nnz needs int64 row_ptr");
  PF_CHECK_ARG(nnz == 0 || (col && val), "null col/val");
  const int64_t gbase = (s.value_mode == 1) ? host_count(s, thr_h, 0, r0) : 0;

  int64_t *d_len = nullptr, *d_rp = nullptr;
  void *tmp = nullptr;
  int32_t *sorted = nullptr;
  pf_status ret = PF_OK;
  auto fail = [&](cudaError_t e, const char *what) {
    set_error("pf_gen_rows_device: %s: %s", what, cudaGetErrorString(e));
    ret = PF_ERR_CUDA;
  };
  cudaError_t e = cudaMalloc(&d_len, sizeof(int64_t) * (cnt + 1));
  if (e == cudaSuccess) e = cudaMalloc(&d_rp, sizeof(int64_t) * (cnt + 1));
  if (e != cudaSuccess) {
    fail(e, "cudaMalloc");
  } else {
    k_lengths<<<grid_for(cnt + 1), 256, 0, cs>>>(s, thr_d, r0, cnt, d_len);
    size_t tb = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, tb, d_len, d_rp, cnt + 1, cs);
    e = cudaMalloc(&tmp, std::max<size_t>(tb, 16));
    if (e == cudaSuccess) e = cub::DeviceScan::ExclusiveSum(tmp, tb, d_len, d_rp, cnt + 1, cs);
    if (e != cudaSuccess) fail(e, "scan");
  }
  if (ret == PF_OK && nnz > 0) {
    const int64_t maxlen = (s.cfg == 3) ? len_cap(s) : (s.cfg == 2 ? 5 : s.k);
    if (s.cfg == 2) {
      // columns written together with the values below
    } else if (maxlen <= kShortMax) {
      k_cols_short<<<grid_for(cnt), 256, 0, cs>>>(s, r0, cnt, d_rp, col);
    } else if (nnz > INT32_MAX) {
      set_error("pf_gen_rows_device: long-row config with nnz > 2^31 unsupported");
      ret = PF_ERR_UNSUPPORTED;
    } else {
      k_cols_draw<<<grid_for(cnt), 256, 0, cs>>>(s, r0, cnt, d_rp, col);
      e = cudaMalloc(&sorted, sizeof(int32_t) * nnz);
      size_t sb = 0;
      if (e == cudaSuccess)
        e = cub::DeviceSegmentedSort::SortKeys(nullptr, sb, col, sorted, (int)nnz, (int)cnt,
                                               d_rp, d_rp + 1, cs);
      if (e == cudaSuccess) {
        cudaFree(tmp);
        tmp = nullptr;
        e = cudaMalloc(&tmp, std::max<size_t>(sb, 16));
      }
      if (e == cudaSuccess)
        e = cub::DeviceSegmentedSort::SortKeys(tmp, sb, col, sorted, (int)nnz, (int)cnt,
                                               d_rp, d_rp + 1, cs);
      if (e == cudaSuccess) {
        k_cols_finish<<<grid_for(cnt), 256, 0, cs>>>(s, cnt, d_rp, sorted, col);
      } else {
        fail(e, "segmented sort");
      }
    }
    if (ret == PF_OK) {
      if (value_bytes == 8)
        k_fill_values<double><<<grid_for(cnt), 256, 0, cs>>>(s, r0, cnt, d_rp, gbase, col,
                                                             (double *)val);
      else
        k_fill_values<float><<<grid_for(cnt), 256, 0, cs>>>(s, r0, cnt, d_rp, gbase, col,
                                                            (float *)val);
    }
  }
  if (ret == PF_OK) {
    if (index_bytes == 8)
      k_rowptr_out<int64_t><<<grid_for(cnt + 1), 256, 0, cs>>>(cnt, d_rp, (int64_t *)row_ptr);
    else
      k_rowptr_out<int32_t><<<grid_for(cnt + 1), 256, 0, cs>>>(cnt, d_rp, (int32_t *)row_ptr);
    e = cudaGetLastError();
    if (e != cudaSuccess) fail(e, "launch");
  }
  // temporaries are freed after the stream drains
  cudaStreamSynchronize(cs);
  if (d_len) cudaFree(d_len);
  if (d_rp) cudaFree(d_rp);
  if (tmp) cudaFree(tmp);
  if (sorted) cudaFree(sorted);
  return ret;
}

pf_status pf_gen_x_device(const pf_gen_spec *spec, int64_t c0, int64_t c1,
                          int value_bytes, void *x, void *stream) {
  pf_status st = check_spec(spec);
  if (st != PF_OK) return st;
  PF_CHECK_ARG(x && 0 <= c0 && c0 <= c1 && c1 <= spec->n, "bad column range");
  PF_CHECK_ARG(value_bytes == 4 || value_bytes == 8, "value_bytes must be 4 or 8");
  const Spec s = make_spec(*spec);
  const int64_t cnt = c1 - c0;
  if (cnt == 0) return PF_OK;
  if (value_bytes == 8)
    k_x<double><<<grid_for(cnt), 256, 0, (cudaStream_t)stream>>>(s, c0, cnt, (double *)x);
  else
    k_x<float><<<grid_for(cnt), 256, 0, (cudaStream_t)stream>>>(s, c0, cnt, (float *)x);
  PF_CUDA_TRY(cudaGetLastError());
  return PF_OK;
}

}  // extern "C"
