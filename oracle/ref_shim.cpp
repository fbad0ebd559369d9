// C-callable shim around the reference's own CPU code — TEST INFRASTRUCTURE ONLY.
//
// oracle/Makefile compiles this file together with the reference sources where
// they lie (test/test_cdspmv.cpp with its main renamed, utilities/mmio.cpp) into
// oracle/_ref/libref.so. Nothing from the reference is copied here: this file
// only declares the reference functions (valT = double, the -Dfp64 build of
// include/common.h:39-40) and forwards to them with C linkage so Python's ctypes
// can call them.
#include <cstdlib>

// test/test_cdspmv.cpp:4-20
void spmv_serial(double *csrVal, int *csrRowPtr, int *csrColInd,
                 double *X_val, double *Y_val, int rowA, int colA, int nnzA);
// utilities/mmio.cpp:1547-1713 (declared at include/mmio.h:177-179)
int mmio_allinone(int *m, int *n, int *nnz, int *isSymmetric,
                  int **csrRowPtr, int **csrColIdx, double **csrVal,
                  char *filename);

// test_cdspmv.cpp's main calls the GPU driver (include/PreFree.h:3-5); the CPU
// oracle never does, so the GPU library is not linked into this shim.
void preFreeSpMV(double *, int *, int *, double *, double *, int, int, int,
                 double *, double *) { std::abort(); }

extern "C" {

void ref_spmv_serial(double *val, int *row_ptr, int *col, double *x, double *y,
                     int m, int n, int nnz)
{
  spmv_serial(val, row_ptr, col, x, y, m, n, nnz);
}

int ref_mmio_allinone(const char *filename, int *m, int *n, int *nnz, int *sym,
                      int **row_ptr, int **col, double **val)
{
  return mmio_allinone(m, n, nnz, sym, row_ptr, col, val,
                       const_cast<char *>(filename));
}

void ref_free(void *p) { std::free(p); }

}  // extern "C"
