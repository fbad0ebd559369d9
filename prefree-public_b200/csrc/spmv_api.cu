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

}  // namespace pf

// Per-device state: scratch for cut-row carries, error word, cached buffers
// for the host-buffer entry points.
struct pf_handle_s {
  int device = 0;
  int num_sms = 0;
  int variant = PF_VARIANT_AUTO;
  int64_t slice_override = 0;  // testing knob: fixed nnz per CTA slice
  // cut-row scratch
  double *carry = nullptr;     // 2 * cap doubles (head, tail)
  unsigned *counters = nullptr;
  int64_t cap = 0;
  bool scratch_dirty = false;
  unsigned *err = nullptr;
  // host-call buffers
  void *hbuf[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
  size_t hcap[5] = {0, 0, 0, 0, 0};
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

template <typename VT, typename IT>
struct NnzSplitCfg {
  static constexpr int NT = 256;
  static constexpr int K = 7;
  static constexpr int W = 512;
};

template <typename VT, typename IT>
static int nnzsplit_occupancy() {
  using C = NnzSplitCfg<VT, IT>;
  static int occ = -1;
  if (occ < 0) {
    int o = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &o, spmv_nnzsplit_kernel<VT, IT, C::NT, C::K, C::W>, C::NT, 0);
    occ = std::max(1, o);
  }
  return occ;
}

template <typename VT, typename IT>
static pf_status launch_spmv(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                             const IT *row_ptr, const int32_t *col,
                             const VT *val, double alpha, const VT *x,
                             double beta, VT *y, cudaStream_t st) {
  PF_CHECK_ARG(h != nullptr, "null handle");
  PF_CHECK_ARG(m >= 0 && n >= 0 && nnz >= 0, "negative size (m=%lld n=%lld nnz=%lld)",
               (long long)m, (long long)n, (long long)nnz);
  if (m == 0) return PF_OK;
  PF_CHECK_ARG(row_ptr && y, "null row_ptr or y");
  PF_CHECK_ARG(nnz == 0 || (col && val && x), "null col/val/x with nnz > 0");
  PF_CHECK_ARG(sizeof(IT) == 8 || nnz <= INT32_MAX, "int32 row_ptr cannot index nnz=%lld",
               (long long)nnz);
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

  using C = NnzSplitCfg<VT, IT>;
  constexpr int TILE = C::NT * C::K;
  int64_t T;
  if (h->slice_override > 0) {
    T = h->slice_override;
  } else {
    const int64_t ctas = (int64_t)h->num_sms * nnzsplit_occupancy<VT, IT>();
    T = std::max<int64_t>(ceil_div(nnz, ctas), TILE);
  }
  const int64_t P = ceil_div(nnz, T);
  PF_CHECK_ARG(P <= INT32_MAX, "too many CTA slices");
  pf_status s = ensure_scratch(h, P, st);
  if (s != PF_OK) return s;

  SpmvParams<VT, IT> prm;
  prm.m = m;
  prm.n = n;
  prm.nnz = nnz;
  prm.T = T;
  prm.num_ctas = P;
  prm.row_ptr = row_ptr;
  prm.col = col;
  prm.val = val;
  prm.x = x;
  prm.y = y;
  prm.alpha = alpha;
  prm.beta = beta;
  prm.carry_head = h->carry;
  prm.carry_tail = h->carry + h->cap;
  prm.counters = h->counters;
  prm.err = h->err;
  spmv_nnzsplit_kernel<VT, IT, C::NT, C::K, C::W><<<(unsigned)P, C::NT, 0, st>>>(prm);
  count_launch();
  PF_CUDA_TRY(cudaGetLastError());
  return PF_OK;
}

// Host-buffer call: copy in, one multiply, copy out.
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
  IT *d_rp = (IT *)h->hbuf[0];
  int32_t *d_col = (int32_t *)h->hbuf[1];
  VT *d_val = (VT *)h->hbuf[2];
  VT *d_x = (VT *)h->hbuf[3];
  VT *d_y = (VT *)h->hbuf[4];
  PF_CUDA_TRY(cudaMemcpyAsync(d_rp, row_ptr, need[0], cudaMemcpyHostToDevice, st));
  if (nnz > 0) {
    PF_CUDA_TRY(cudaMemcpyAsync(d_col, col + base, need[1], cudaMemcpyHostToDevice, st));
    PF_CUDA_TRY(cudaMemcpyAsync(d_val, val + base, need[2], cudaMemcpyHostToDevice, st));
  }
  if (n > 0) PF_CUDA_TRY(cudaMemcpyAsync(d_x, x, need[3], cudaMemcpyHostToDevice, st));
  if (beta != 0.0) PF_CUDA_TRY(cudaMemcpyAsync(d_y, y, need[4], cudaMemcpyHostToDevice, st));
  // Device arrays hold the slice only: shift so absolute row_ptr values land
  // at element 0 (the kernel only touches [base, base + nnz)).
  pf_status s = launch_spmv<VT, IT>(h, m, n, nnz, d_rp, d_col - base, d_val - base,
                                    alpha, d_x, beta, d_y, st);
  if (s != PF_OK) return s;
  PF_CUDA_TRY(cudaMemcpyAsync(y, d_y, need[4], cudaMemcpyDeviceToHost, st));
  PF_CUDA_TRY(cudaStreamSynchronize(st));
  return PF_OK;
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
  cudaSetDevice(cur);
  delete h;
  return PF_OK;
}

pf_status pf_handle_set_variant(pf_handle h, int variant) {
  PF_CHECK_ARG(h != nullptr, "null handle");
  PF_CHECK_ARG(variant >= PF_VARIANT_AUTO && variant <= PF_VARIANT_ROWGROUP,
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

PF_DEFINE_SPMV(f64_i32, double, int32_t)
PF_DEFINE_SPMV(f64_i64, double, int64_t)
PF_DEFINE_SPMV(f32_i32, float, int32_t)
PF_DEFINE_SPMV(f32_i64, float, int64_t)

}  // extern "C"
