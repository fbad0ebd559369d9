/*
 * CPU oracle for the CSR SpMV hot path — TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load this library, and only as the checker or the timed CPU
 * baseline. The product path (the CUDA library under prefree-public_b200/)
 * never calls into it.
 *
 * Pinning: the serial loop below is checked against the reference's own
 * compiled `spmv_serial` (oracle/_ref, built from the reference sources by
 * oracle/Makefile) and against the committed golden fixtures in tests/golden/
 * produced by that build (tests/test_oracle.py).
 *
 * Restated from wang-luhan/preFree-public test/test_cdspmv.cpp:4-20
 * (`spmv_serial`): for each row i, t = 0; t = t + val[j]*x[col[j]] over the
 * row's entries in storage order; Y[i] = Y[i] + t. The reference's `valT` is
 * double under -Dfp64 (include/common.h:39-40) and its offsets are `int`; the
 * variants here add int64 offsets (needed for 2^31 non-zeros) and fp32 inputs
 * widened to double (the reference has no fp32 build), keeping the same order
 * of operations.
 */
#include <stdint.h>
#include <stddef.h>
#include <math.h>

#define ORACLE_SERIAL(NAME, VT, IT)                                            \
  void NAME(const VT *val, const IT *row_ptr, const int32_t *col,              \
            const VT *x, double *y, int64_t m)                                 \
  {                                                                            \
    for (int64_t i = 0; i < m; i++) {                                          \
      double t = 0.0;                                                          \
      IT start = row_ptr[i];                                                   \
      IT len = row_ptr[i + 1] - start;                                         \
      for (IT j = 0; j < len; j++) {                                           \
        int32_t c = col[start + j];                                            \
        t = t + (double)val[start + j] * (double)x[c];                         \
      }                                                                        \
      y[i] = y[i] + t;                                                         \
    }                                                                          \
  }

/* test_cdspmv.cpp:4-20 with int offsets (as in the reference) */
ORACLE_SERIAL(oracle_spmv_serial_f64_i32, double, int32_t)
/* same loop, int64 offsets (config 5: nnz = 2^31) */
ORACLE_SERIAL(oracle_spmv_serial_f64_i64, double, int64_t)
/* same loop on fp32 inputs widened to double */
ORACLE_SERIAL(oracle_spmv_serial_f32_i32, float, int32_t)
ORACLE_SERIAL(oracle_spmv_serial_f32_i64, float, int64_t)

/*
 * Per-row tolerance scale s_i = sum_j |val_ij * x_j| and a Neumaier-compensated
 * row sum (a tie-breaker when the serial sum itself is off by more than the
 * tolerance on very long rows). The north-star tolerance is
 * |y_i - y_ref_i| <= eps * s_i (eps = 1e-12 fp64, 1e-5 fp32).
 */
#define ORACLE_ABS_COMP(NAME, VT, IT)                                          \
  void NAME(const VT *val, const IT *row_ptr, const int32_t *col,              \
            const VT *x, double *abs_sum, double *comp_sum, int64_t m)         \
  {                                                                            \
    for (int64_t i = 0; i < m; i++) {                                          \
      double s = 0.0, sum = 0.0, c = 0.0;                                      \
      for (IT j = row_ptr[i]; j < row_ptr[i + 1]; j++) {                       \
        double p = (double)val[j] * (double)x[col[j]];                         \
        s += fabs(p);                                                          \
        double t = sum + p;                                                    \
        if (fabs(sum) >= fabs(p)) c += (sum - t) + p;                          \
        else c += (p - t) + sum;                                               \
        sum = t;                                                               \
      }                                                                        \
      abs_sum[i] = s;                                                          \
      comp_sum[i] = sum + c;                                                   \
    }                                                                          \
  }

ORACLE_ABS_COMP(oracle_spmv_abs_comp_f64_i32, double, int32_t)
ORACLE_ABS_COMP(oracle_spmv_abs_comp_f64_i64, double, int64_t)
ORACLE_ABS_COMP(oracle_spmv_abs_comp_f32_i32, float, int32_t)
ORACLE_ABS_COMP(oracle_spmv_abs_comp_f32_i64, float, int64_t)

/*
 * Restatement of the reference's CSR construction in mmio_allinone
 * (utilities/mmio.cpp:1547-1713) from already-parsed coordinates: count per
 * row (symmetric inputs add the mirrored off-diagonal entry to the column's
 * row, :1641-1648), exclusive scan (:949-964, :1650), then scatter in file
 * order (:1661-1695) — so column order inside a row is file order, with each
 * symmetric off-diagonal entry placed in row i first and then in row j.
 * Coordinates are already 0-based. Returns nnz of the CSR.
 * Buffers: row_ptr[m+1]; col/val sized for the expanded nnz (<= 2*nnz_in).
 */
int64_t oracle_coo_to_csr(int64_t m, int64_t nnz_in, const int32_t *ri,
                          const int32_t *ci, const double *vi, int symmetric,
                          int64_t *row_ptr, int32_t *col, double *val,
                          int64_t *cursor /* scratch, m entries */)
{
  for (int64_t i = 0; i <= m; i++) row_ptr[i] = 0;
  for (int64_t k = 0; k < nnz_in; k++) {
    row_ptr[ri[k]]++;
    if (symmetric && ri[k] != ci[k]) row_ptr[ci[k]]++;
  }
  /* exclusive scan over m+1 entries */
  int64_t run = 0;
  for (int64_t i = 0; i <= m; i++) {
    int64_t c = row_ptr[i];
    row_ptr[i] = run;
    run += c;
  }
  for (int64_t i = 0; i < m; i++) cursor[i] = 0;
  for (int64_t k = 0; k < nnz_in; k++) {
    int64_t o = row_ptr[ri[k]] + cursor[ri[k]]++;
    col[o] = ci[k];
    val[o] = vi[k];
    if (symmetric && ri[k] != ci[k]) {
      o = row_ptr[ci[k]] + cursor[ci[k]]++;
      col[o] = ri[k];
      val[o] = vi[k];
    }
  }
  return row_ptr[m];
}
