// pf_spmv_noalloc_f64_i32: the NNZSPLIT (TMA ring) multiply for callers that
// cannot allocate device memory.
//
// Who needs it: code that runs inside an application which has already
// reserved the GPU's memory for itself (a serving process whose allocator
// claims most of HBM at start-up and hands out nothing else), or which must
// not call cudaMalloc/cudaFree mid-run because those calls can synchronize
// the device and can fail under memory pressure. The regular entry points
// allocate their scratch through a pf_handle; this one allocates nothing.
//
// The NNZSPLIT kernel needs scratch beyond its inputs and outputs: one
// head and one tail partial per CTA slice for rows cut by slice boundaries,
// one counter per slice boundary, and a device error word. Here that scratch
// is the file-scope array below, compiled into the library: every GPU that
// loads the library holds it (about 41 KB) until the process exits.
//
// Limits and rules:
//   * at most kNoAllocMaxSlices CTA slices; the slice count is at most the SM
//     count times the kernel's occupancy (444 on a B200), so the limit only
//     binds on a GPU with far more SMs; larger counts are refused with
//     PF_ERR_UNSUPPORTED;
//   * the first call on a device does a one-time set-up with that device
//     current (it looks up the array's device address with
//     cudaGetSymbolAddress and sets the kernel's shared-memory limit); make
//     that first call before any stream capture;
//   * every call shares the one array: calls that overlap on the GPU (two
//     host threads, two streams) race and give wrong results. Each call
//     clears the counters and the error word it uses before its launch;
//   * every call (the nnz = 0 one too) returns once its work has finished on
//     `stream`: it waits for the stream so that it can report the kernel's
//     error word, PF_ERR_DEVICE when a bit is set (for example when
//     row_ptr[m] - row_ptr[0] != nnz; nothing is written then).
#include <mutex>

#include "pf_common.cuh"
#include "spmv_tma.cuh"

namespace {

constexpr int kNoAllocMaxSlices = 2048;

struct NoAllocScratch {
  double carry[2 * kNoAllocMaxSlices];  // head partials, then tail partials
  unsigned counters[kNoAllocMaxSlices];
  unsigned err;
};

// The scratch. In host code this name is only a host-side stand-in for the
// device array; the kernel gets the address from cudaGetSymbolAddress.
static __device__ __align__(256) NoAllocScratch g_noalloc_scratch[1];

struct DeviceSetup {
  bool ready = false;
  NoAllocScratch *scratch = nullptr;  // device address of g_noalloc_scratch
  int num_sms = 0;
  int occupancy = 0;
  size_t smem = 0;
};

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
DeviceSetup g_setup[kMaxDevices];

using Cfg = pf::TmaCfgDefault;

pf_status setup_device(int dev, DeviceSetup **out) {
  PF_CHECK_ARG(dev >= 0 && dev < kMaxDevices, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> g(g_setup_mu);
  DeviceSetup &s = g_setup[dev];
  if (!s.ready) {
    void *p = nullptr;
    PF_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    s.scratch = static_cast<NoAllocScratch *>(p);
    PF_CUDA_TRY(cudaDeviceGetAttribute(&s.num_sms, cudaDevAttrMultiProcessorCount, dev));
    s.smem = sizeof(pf::TmaSmem<double, int32_t, Cfg>);
    PF_CUDA_TRY(cudaFuncSetAttribute(pf::spmv_tma_kernel<double, int32_t, Cfg>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)s.smem));
    PF_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &s.occupancy, pf::spmv_tma_kernel<double, int32_t, Cfg>, Cfg::NT, s.smem));
    if (s.occupancy < 1) s.occupancy = 1;
    s.ready = true;
  }
  *out = &s;
  return PF_OK;
}

}  // namespace

extern "C" pf_status pf_spmv_noalloc_f64_i32(int64_t m, int64_t n, int64_t nnz,
                                             const int32_t *row_ptr, const int32_t *col_idx,
                                             const double *val, double alpha, const double *x,
                                             double beta, double *y, void *stream) {
  using namespace pf;
  PF_CHECK_ARG(m >= 0 && n >= 0 && nnz >= 0, "negative size");
  if (m == 0) return PF_OK;
  PF_CHECK_ARG(row_ptr && y, "null row_ptr or y");
  PF_CHECK_ARG(nnz == 0 || (col_idx && val && x), "null col/val/x with nnz > 0");
  PF_CHECK_ARG(nnz <= INT32_MAX, "int32 row_ptr cannot index nnz=%lld", (long long)nnz);
  PF_CHECK_ARG(nnz == 0 || n > 0, "nnz > 0 needs n > 0");
  PF_CHECK_ARG(n <= (int64_t)INT32_MAX + 1, "n must fit int32 column indices");
  PF_CHECK_ARG(((uintptr_t)row_ptr % 4) == 0 && ((uintptr_t)y % 8) == 0 &&
                   (nnz == 0 || (((uintptr_t)col_idx % 4) == 0 && ((uintptr_t)val % 8) == 0 &&
                                 ((uintptr_t)x % 8) == 0)),
               "arrays must be aligned to their element size");
  cudaStream_t st = (cudaStream_t)stream;
  int dev = 0;
  PF_CUDA_TRY(cudaGetDevice(&dev));
  DeviceSetup *ds = nullptr;
  pf_status s = setup_device(dev, &ds);
  if (s != PF_OK) return s;

  if (nnz == 0) {
    const unsigned blocks = (unsigned)std::min<int64_t>(ceil_div(m, 256), 4L * ds->num_sms * 8);
    scale_rows_kernel<double><<<blocks, 256, 0, st>>>(m, beta, y);
    count_launches(1);
    PF_CUDA_TRY(cudaGetLastError());
    PF_CUDA_TRY(cudaStreamSynchronize(st));  // returns after the work, as every call does
    return PF_OK;
  }

  const int64_t ctas = (int64_t)ds->num_sms * ds->occupancy;
  const int64_t T = std::max<int64_t>(ceil_div(nnz, ctas), 2 * Cfg::TILE);
  const int64_t P = ceil_div(nnz, T);
  if (P > kNoAllocMaxSlices) {
    set_error("pf_spmv_noalloc_f64_i32: %lld CTA slices needed, the built-in scratch holds %d",
              (long long)P, kNoAllocMaxSlices);
    return PF_ERR_UNSUPPORTED;
  }
  NoAllocScratch *sc = ds->scratch;
  // counters must start at zero; the error word is per call
  PF_CUDA_TRY(cudaMemsetAsync(sc->counters, 0, sizeof(unsigned) * (size_t)P, st));
  PF_CUDA_TRY(cudaMemsetAsync(&sc->err, 0, sizeof(unsigned), st));

  SpmvParams<double, int32_t> prm;
  prm.m = m;
  prm.n = n;
  prm.nnz = nnz;
  prm.T = T;
  prm.num_ctas = P;
  prm.row_ptr = row_ptr;
  prm.col = col_idx;
  prm.val = val;
  prm.x = x;
  prm.y = y;
  prm.alpha = alpha;
  prm.beta = beta;
  prm.carry_head = sc->carry;
  prm.carry_tail = sc->carry + kNoAllocMaxSlices;
  prm.counters = sc->counters;
  prm.err = &sc->err;
  spmv_tma_kernel<double, int32_t, Cfg><<<(unsigned)P, Cfg::NT, ds->smem, st>>>(prm);
  count_launches(1);
  PF_CUDA_TRY(cudaGetLastError());

  unsigned bits = 0;
  PF_CUDA_TRY(cudaMemcpyAsync(&bits, &sc->err, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
  PF_CUDA_TRY(cudaStreamSynchronize(st));
  if (bits) {
    set_error("pf_spmv_noalloc_f64_i32: kernel reported device error bits 0x%x", bits);
    return PF_ERR_DEVICE;
  }
  return PF_OK;
}
