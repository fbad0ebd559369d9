/*
 * prefree_b200.h — C ABI of the B200 (sm_100a) CSR SpMV library.
 *
 * y = alpha * A * x + beta * y, A in CSR (0-based), fp64 or fp32 values,
 * int32 column indices, int32 or int64 row pointers. No preprocessing pass:
 * every call works straight from (row_ptr, col_idx, val) as given.
 *
 * Drop-in map onto wang-luhan/preFree-public:
 *   - the C++ entry point `preFreeSpMV` itself (include/PreFree.h:3-5,
 *     defined at src/spmv_kernel/preFreeSpMV.cu:563-662) is declared, with the
 *     identical signature and mangled name, in include/PreFree.h of this repo;
 *   - pf_prefree_spmv_* below are the same calls with C linkage (for ctypes /
 *     FFI callers), one per value/index type;
 *   - pf_spmv_* are the device-pointer core the reference never exposed: its
 *     driver hard-wires allocation + copies + launch (preFreeSpMV.cu:571-648);
 *     these take device pointers, a stream, alpha and beta;
 *   - pf_mmio_read replaces mmio_allinone (utilities/mmio.cpp:1547-1713,
 *     include/mmio.h:177-179), the harness's Matrix Market -> CSR input path.
 *
 * Every function returns a pf_status; none exits the process (the reference's
 * CUDA_CHECK_ERROR calls exit(), include/common.h:49-58). pf_last_error()
 * gives the text of the calling thread's last failure.
 */
#ifndef PREFREE_B200_H
#define PREFREE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum pf_status {
  PF_OK = 0,
  PF_ERR_INVALID = 1,     /* bad argument: size, null pointer, layout       */
  PF_ERR_CUDA = 2,        /* a CUDA runtime call failed                     */
  PF_ERR_DEVICE = 3,      /* a kernel reported an error word (see below)    */
  PF_ERR_UNSUPPORTED = 4, /* valid request this build does not provide      */
  PF_ERR_IO = 5,          /* file could not be opened / read                */
  PF_ERR_FORMAT = 6       /* Matrix Market text could not be parsed         */
} pf_status;

/* Kernel variants (compile-time table, selected per call; AUTO = selector).
 * The missing numbers belonged to variants that measured slower on every
 * configuration and were removed; forcing them is refused. */
typedef enum pf_variant {
  PF_VARIANT_AUTO = 0,
  PF_VARIANT_NNZSPLIT = 1, /* nnz slices streamed by bulk copies (the no-alloc kernel) */
  PF_VARIANT_ROWGROUP = 2, /* row groups, scalar loads: unaligned col/val    */
  PF_VARIANT_ROWVEC = 4,   /* row groups, 16-byte block loads: regular rows    */
  PF_VARIANT_NNZROW = 7    /* nnz slices, row pieces summed: irregular rows   */
} pf_variant;

typedef struct pf_handle_s *pf_handle;

const char *pf_last_error(void);
const char *pf_version(void);
/* Number of this library's kernels launched since it was loaded. */
uint64_t pf_launch_count(void);

/* A handle owns per-device scratch (cross-CTA carries for rows split between
 * CTAs) and the device error word. It is bound to the device current at
 * creation. Calls that share a handle must not overlap on the GPU (use one
 * handle per stream). */
pf_status pf_handle_create(pf_handle *out);
pf_status pf_handle_destroy(pf_handle h);
pf_status pf_handle_set_variant(pf_handle h, int variant);
/* Testing knob: fixed non-zeros per CTA slice for NNZSPLIT and NNZROW
 * (0 = automatic). Small slices force many rows to be cut between CTAs. */
pf_status pf_handle_set_slice(pf_handle h, int64_t slice_nnz);
/* Synchronizes the device, returns the device error bits, optionally clears. */
pf_status pf_handle_device_error(pf_handle h, uint32_t *bits, int clear);
/* The variant (a pf_variant other than AUTO) and lanes per row that a
 * multiply with this handle would run for the device CSR (m, nnz, row_ptr)
 * with values of value_bytes (2, 4 or 8) bytes: the forced variant, or the
 * selector's choice, which it computes (a sample kernel on `stream`,
 * synchronous) and caches as a multiply would. The variant actually
 * launched can still differ for arrays that are not 16-byte aligned (each
 * variant's fallback). */
pf_status pf_handle_choice_i32(pf_handle h, int64_t m, int64_t nnz, const int32_t *row_ptr,
                               int value_bytes, void *stream, int *variant, int *lanes);
pf_status pf_handle_choice_i64(pf_handle h, int64_t m, int64_t nnz, const int64_t *row_ptr,
                               int value_bytes, void *stream, int *variant, int *lanes);

/* ---- device-pointer core: y = alpha*A*x + beta*y ----------------------------
 * row_ptr has m+1 entries; row_ptr[0] may be non-zero (a row slice of a larger
 * CSR): val/col_idx are addressed with the absolute row_ptr values, and nnz
 * must equal row_ptr[m] - row_ptr[0]. x has n entries, y has m. With beta == 0
 * y is not read. `stream` is a cudaStream_t (NULL = legacy default stream).
 * Asynchronous: returns after the launch. Accumulation is in fp64 for both
 * value types; the result is rounded once to the value type. Deterministic:
 * the same inputs give bit-identical y on every call.                         */
pf_status pf_spmv_f64_i32(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                          const int32_t *row_ptr, const int32_t *col_idx,
                          const double *val, double alpha, const double *x,
                          double beta, double *y, void *stream);
pf_status pf_spmv_f64_i64(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                          const int64_t *row_ptr, const int32_t *col_idx,
                          const double *val, double alpha, const double *x,
                          double beta, double *y, void *stream);
pf_status pf_spmv_f32_i32(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                          const int32_t *row_ptr, const int32_t *col_idx,
                          const float *val, double alpha, const float *x,
                          double beta, float *y, void *stream);
pf_status pf_spmv_f32_i64(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                          const int64_t *row_ptr, const int32_t *col_idx,
                          const float *val, double alpha, const float *x,
                          double beta, float *y, void *stream);

/* ---- 16-bit values: binary16 (f16) and bfloat16 (bf16) ------------------------
 * The reference's intended second value type (valT = half, include/common.h:
 * 43-46; that build does not compile, src/spmv_kernel/preFreeSpMV.cu:326).
 * val, x and y hold the 16-bit patterns; products and sums are computed in
 * double and y is rounded once (to nearest). Otherwise as pf_spmv_*.        */
pf_status pf_spmv_f16_i32(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                          const int32_t *row_ptr, const int32_t *col_idx,
                          const uint16_t *val, double alpha, const uint16_t *x,
                          double beta, uint16_t *y, void *stream);
pf_status pf_spmv_f16_i64(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                          const int64_t *row_ptr, const int32_t *col_idx,
                          const uint16_t *val, double alpha, const uint16_t *x,
                          double beta, uint16_t *y, void *stream);
pf_status pf_spmv_bf16_i32(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                           const int32_t *row_ptr, const int32_t *col_idx,
                           const uint16_t *val, double alpha, const uint16_t *x,
                           double beta, uint16_t *y, void *stream);
pf_status pf_spmv_bf16_i64(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                           const int64_t *row_ptr, const int32_t *col_idx,
                           const uint16_t *val, double alpha, const uint16_t *x,
                           double beta, uint16_t *y, void *stream);

/* ---- SpMM: Y = alpha * A * X + beta * Y for k dense columns -----------------
 * No counterpart in the reference (its harness multiplies one vector); the
 * next step beside SpMV in iterative solvers with several right-hand sides.
 * X is n x k and Y is m x k, both row-major on the device with leading
 * dimensions ldx >= k and ldy >= k (elements). Columns are taken in passes
 * of up to 8, each pass reading A once, so a non-zero's bytes and the cache
 * line of its gather serve up to 8 products. Same CSR conventions, status
 * codes and device error word as pf_spmv_*; asynchronous on `stream`.      */
pf_status pf_spmm_f64_i32(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                          const int32_t *row_ptr, const int32_t *col_idx,
                          const double *val, int k, double alpha, const double *X,
                          int64_t ldx, double beta, double *Y, int64_t ldy, void *stream);
pf_status pf_spmm_f64_i64(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                          const int64_t *row_ptr, const int32_t *col_idx,
                          const double *val, int k, double alpha, const double *X,
                          int64_t ldx, double beta, double *Y, int64_t ldy, void *stream);
pf_status pf_spmm_f32_i32(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                          const int32_t *row_ptr, const int32_t *col_idx,
                          const float *val, int k, double alpha, const float *X,
                          int64_t ldx, double beta, float *Y, int64_t ldy, void *stream);
pf_status pf_spmm_f32_i64(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                          const int64_t *row_ptr, const int32_t *col_idx,
                          const float *val, int k, double alpha, const float *X,
                          int64_t ldx, double beta, float *Y, int64_t ldy, void *stream);

/* ---- fused multiply + all-gather for row-sharded iterated multiplies --------
 * No counterpart in the reference (single GPU only). One step of
 * x_{k+1} = A x_k / ||A x_k|| on this rank's row shard (rows
 * [row_offset, row_offset + m) of the full matrix; row_ptr rebased to 0):
 *   alpha = 1 / sqrt(sum of prev_slots[0..nranks));
 *   every finished row value y_r = alpha * (A x)_r is stored straight into
 *   out_ptrs[p][row_offset + r] for every rank p (device array of nranks
 *   pointers: each rank's next-x buffer, peers' reachable over NVLink);
 *   ||y||^2 of this rank's rows is reduced in the same kernel (fixed order:
 *   the same bits every run) and stored to slot_ptrs[p][rank] for every p.
 * Steps must be separated by a cross-rank barrier (peers' stores must land
 * before the next step reads x, and nobody may overwrite a buffer a peer
 * still reads: alternate two x buffers and two slot arrays). With flag_ptrs
 * (device array of nranks pointers to every rank's array of nranks uint64
 * step counters, zero at the start, peer-mapped like out_ptrs) the kernel
 * is that barrier: step `step` (0, 1, ...) waits, one thread per CTA, until
 * its own counters all reach `step`, and when its stores are done it sets
 * counter `rank` to step + 1 on every rank; the host then launches steps
 * back to back. The wait gives up after 1 s with PF_DEVERR_WAIT_TIMEOUT in
 * the device error word. flag_ptrs = NULL: no barrier in the kernel (the
 * caller provides one). fp64 values, col/val 16-byte aligned (ROWVEC
 * kernel). Asynchronous on `stream`.                                        */
pf_status pf_spmv_dist_f64_i64(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                               const int64_t *row_ptr, const int32_t *col_idx,
                               const double *val, const double *x, const double *prev_slots,
                               int nranks, int rank, double *const *out_ptrs,
                               double *const *slot_ptrs, int64_t row_offset,
                               uint64_t *const *flag_ptrs, uint64_t step, void *stream);
pf_status pf_spmv_dist_f64_i32(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                               const int32_t *row_ptr, const int32_t *col_idx,
                               const double *val, const double *x, const double *prev_slots,
                               int nranks, int rank, double *const *out_ptrs,
                               double *const *slot_ptrs, int64_t row_offset,
                               uint64_t *const *flag_ptrs, uint64_t step, void *stream);
/* Nanoseconds the fused steps of this handle spent in their in-kernel step
 * barrier, summed over CTAs and steps since the last reset, and the CTAs of
 * the last fused launch (a diagnostic of how long ranks wait for one
 * another). Synchronizes the device. */
pf_status pf_handle_dist_wait(pf_handle h, uint64_t *wait_ns, int64_t *ctas, int reset);

/* ---- allocation-free multiply (fp64 values, int32 row_ptr) ------------------
 * No counterpart in the reference. For callers that cannot allocate device
 * memory: code running inside an application that has already reserved the
 * GPU's memory for itself, or that must not call cudaMalloc/cudaFree mid-run
 * (they can synchronize the device and fail under memory pressure). Same
 * arguments and result as pf_spmv_f64_i32 without a handle; always uses the
 * NNZSPLIT kernel, whose scratch (cut-row partials, slice counters, error
 * word) is a ~41 KB array built into the library and held by every GPU that
 * loads it until the process exits. At most 2048 CTA slices (the SM count
 * times the kernel's occupancy: 444 on a B200); more are refused with
 * PF_ERR_UNSUPPORTED. The first call on a device sets it up (looks up the
 * array's device address, sets the kernel's shared-memory limit): make it
 * before any stream capture. Calls share the array, so calls that overlap on
 * the GPU race. Returns after the multiply has finished on `stream`, with
 * PF_ERR_DEVICE if the kernel flagged an error.                              */
pf_status pf_spmv_noalloc_f64_i32(int64_t m, int64_t n, int64_t nnz,
                                  const int32_t *row_ptr, const int32_t *col_idx,
                                  const double *val, double alpha, const double *x,
                                  double beta, double *y, void *stream);

/* ---- host-buffer call (one multiply, copies in and out) ---------------------
 * Same arithmetic as pf_spmv_*, on HOST arrays: copies row_ptr/col/val/x in
 * (and y when beta != 0), multiplies once, copies y out, synchronizes. col/val
 * travel in row chunks of about equal nnz (256 MB each, at most 16; the
 * environment variable PF_HOST_CHUNK_BYTES overrides the size) on a copy
 * stream of the handle, and each chunk is multiplied and its rows of y copied
 * out on `stream` while the next chunks are copied in. Device buffers are
 * cached in the handle and reused across calls. Pinned host memory gives full
 * PCIe bandwidth and the overlap; pageable memory works too.                 */
pf_status pf_spmv_host_f64_i32(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                               const int32_t *row_ptr, const int32_t *col_idx,
                               const double *val, double alpha,
                               const double *x, double beta, double *y,
                               void *stream);
pf_status pf_spmv_host_f64_i64(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                               const int64_t *row_ptr, const int32_t *col_idx,
                               const double *val, double alpha,
                               const double *x, double beta, double *y,
                               void *stream);
pf_status pf_spmv_host_f32_i32(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                               const int32_t *row_ptr, const int32_t *col_idx,
                               const float *val, double alpha, const float *x,
                               double beta, float *y, void *stream);
pf_status pf_spmv_host_f32_i64(pf_handle h, int64_t m, int64_t n, int64_t nnz,
                               const int64_t *row_ptr, const int32_t *col_idx,
                               const float *val, double alpha, const float *x,
                               double beta, float *y, void *stream);

/* ---- preFreeSpMV with C linkage ---------------------------------------------
 * Replaces preFreeSpMV (include/PreFree.h:3-5; preFreeSpMV.cu:563-662) for
 * FFI callers. Host arrays in; Y_val is overwritten with A*x; *cdTime = ms per
 * multiply averaged over the timed launches (4000 after 200 warm-up, as at
 * preFreeSpMV.cu:604-650; PF_PREFREE_ITERS / PF_PREFREE_WARMUP override);
 * *cdPre = ms of the pre-pass, which here is only the host-side variant
 * selection (there is no preprocessing kernel). Reads row_ptr[0..rowA] (the
 * reference also copies one entry past it, preFreeSpMV.cu:580; this does not).
 * The fp32 and int64 forms are the same call for the other types.            */
pf_status pf_prefree_spmv_f64_i32(double *csrVal, int32_t *csrRowPtr,
                                  int32_t *csrColInd, double *X_val,
                                  double *Y_val, int32_t rowA, int32_t colA,
                                  int32_t nnzA, double *cdTime, double *cdPre);
pf_status pf_prefree_spmv_f64_i64(double *csrVal, int64_t *csrRowPtr,
                                  int32_t *csrColInd, double *X_val,
                                  double *Y_val, int64_t rowA, int64_t colA,
                                  int64_t nnzA, double *cdTime, double *cdPre);
pf_status pf_prefree_spmv_f32_i32(float *csrVal, int32_t *csrRowPtr,
                                  int32_t *csrColInd, float *X_val,
                                  float *Y_val, int32_t rowA, int32_t colA,
                                  int32_t nnzA, double *cdTime, double *cdPre);

/* ---- Matrix Market -> CSR (the harness input path) --------------------------
 * Replaces mmio_allinone (utilities/mmio.cpp:1547-1713): same banner handling
 * (real / integer / pattern = 1.0 / complex = real part), 1-based -> 0-based,
 * symmetric and Hermitian inputs expanded (off-diagonal entries mirrored),
 * entries of a row kept in file order (no sort), row_ptr has m+1 entries.
 * Differences: 64-bit row_ptr and nnz, a multi-threaded parser, and errors are
 * returned instead of printed. Arrays are malloc'd; free them with pf_free
 * (pf_mmio_read_pinned below returns page-locked arrays instead).            */
pf_status pf_mmio_read(const char *path, int64_t *m, int64_t *n, int64_t *nnz,
                       int *is_symmetric, int64_t **row_ptr, int32_t **col_idx,
                       double **val);
void pf_free(void *p);
/* pf_mmio_read with the three arrays in page-locked (pinned) host memory, so
 * that pf_spmv_host_* (or any cudaMemcpyAsync) copies a file-loaded matrix to
 * the device at full PCIe speed, without a staging copy. Free them with
 * pf_free, which tells pinned arrays from heap ones. Needs the CUDA runtime
 * (no device work). No counterpart in the reference, whose mmio_allinone
 * returns malloc'd arrays (utilities/mmio.cpp:1653-1660). */
pf_status pf_mmio_read_pinned(const char *path, int64_t *m, int64_t *n, int64_t *nnz,
                              int *is_symmetric, int64_t **row_ptr, int32_t **col_idx,
                              double **val);

/* Binary CSR cache: parse a .mtx once, reload its CSR at file-read speed.
 * pf_csr_write / pf_csr_read store and load (m, n, nnz, is_symmetric,
 * row_ptr int64[m+1], col int32[nnz], val double[nnz]); pf_csr_read checks
 * the file's size and the CSR's consistency (row_ptr non-decreasing from 0 to
 * nnz, columns in [0, n)) before returning it. pf_mmio_read_cached reads
 * cache_path when it was written from mtx_path's current size and
 * modification time, else parses mtx_path with pf_mmio_read and (re)writes
 * the cache, best effort. *from_cache (may be NULL) tells which happened.
 * Arrays are malloc'd; free them with pf_free. No counterpart in the
 * reference (its harness parses the text file on every run).                */
pf_status pf_csr_write(const char *path, int64_t m, int64_t n, int64_t nnz, int is_symmetric,
                       const int64_t *row_ptr, const int32_t *col_idx, const double *val);
pf_status pf_csr_read(const char *path, int64_t *m, int64_t *n, int64_t *nnz, int *is_symmetric,
                      int64_t **row_ptr, int32_t **col_idx, double **val);
pf_status pf_mmio_read_cached(const char *mtx_path, const char *cache_path, int64_t *m,
                              int64_t *n, int64_t *nnz, int *is_symmetric, int64_t **row_ptr,
                              int32_t **col_idx, double **val, int *from_cache);
/* pf_mmio_read_cached with the arrays in page-locked host memory (as
 * pf_mmio_read_pinned); free them with pf_free. */
pf_status pf_mmio_read_cached_pinned(const char *mtx_path, const char *cache_path, int64_t *m,
                                     int64_t *n, int64_t *nnz, int *is_symmetric,
                                     int64_t **row_ptr, int32_t **col_idx, double **val,
                                     int *from_cache);

/* ---- row sharding (multi-GPU) -----------------------------------------------
 * Equal-nnz row split: bounds[k] = first row r with row_ptr[r] - row_ptr[0]
 * >= k*nnz/parts (k = 0..parts; bounds[0] = 0, bounds[parts] = m). Host
 * row_ptr. No counterpart in the reference (single GPU only).               */
pf_status pf_shard_bounds_i32(const int32_t *row_ptr, int64_t m, int parts,
                              int64_t *bounds);
pf_status pf_shard_bounds_i64(const int64_t *row_ptr, int64_t m, int parts,
                              int64_t *bounds);

/* ---- synthetic inputs (benchmark configs; no counterpart in the reference,
 * which reads SuiteSparse .mtx files) -----------------------------------------
 * Counter-based: row r of config `cfg` is a pure function of (seed, r), the
 * same bits on host and device. cfg: 1 uniform 16/row 100k^2, 2 5-point
 * Laplacian 2048^2, 3 power-law 4M^2, 4 2000/row 50k^2, 5 banded+uniform
 * 32/row 2^26 (sizes overridable via m for cfg 1,3,4,5: pass m <= 0 for the
 * config's own size). value_mode: 0 = the config's distribution, 1 = i % 15
 * (the reference harness's initVec, include/common.h:126-133).              */
typedef struct pf_gen_spec {
  int cfg;
  int value_mode;
  uint64_t seed;
  int64_t m;     /* rows (0 = config default) */
  int64_t n;     /* cols (0 = config default) */
  int64_t k;     /* nnz per row for fixed-length configs (0 = default) */
} pf_gen_spec;

/* Resolve the defaults of a spec (m, n, k filled in). */
pf_status pf_gen_resolve(pf_gen_spec *spec);
/* Row lengths are needed first: len[r - r0] for rows [r0, r1). Host. */
pf_status pf_gen_row_lengths_host(const pf_gen_spec *spec, int64_t r0,
                                  int64_t r1, int64_t *len);
/* Fill rows [r0, r1) on the HOST: row_ptr (r1-r0+1 entries, starting at 0),
 * col, val (fp64; fp32 callers round). Single thread per call. */
pf_status pf_gen_rows_host(const pf_gen_spec *spec, int64_t r0, int64_t r1,
                           int64_t *row_ptr, int32_t *col, double *val);
pf_status pf_gen_x_host(const pf_gen_spec *spec, int64_t c0, int64_t c1,
                        double *x);
/* Number of non-zeros in rows [r0, r1) (host; sizes the buffers below). */
pf_status pf_gen_count(const pf_gen_spec *spec, int64_t r0, int64_t r1,
                       int64_t *nnz_out);
/* Device generation of rows [r0, r1) into device buffers: row_ptr rebased to
 * start at 0 (r1-r0+1 entries, int32 or int64), col/val sized by
 * pf_gen_count, fp64 or fp32 values. Synchronizes `stream` before returning. */
pf_status pf_gen_rows_device(const pf_gen_spec *spec, int64_t r0, int64_t r1,
                             int index_bytes, void *row_ptr, int32_t *col,
                             int value_bytes, void *val, void *stream);
pf_status pf_gen_x_device(const pf_gen_spec *spec, int64_t c0, int64_t c1,
                          int value_bytes, void *x, void *stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* PREFREE_B200_H */
