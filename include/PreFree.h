// PreFree.h — drop-in for wang-luhan/preFree-public include/PreFree.h:1-5.
//
// The first declaration is the reference's entry point with valT = double
// (its -Dfp64 build, include/common.h:39-40): same parameter list, same C++
// mangled name (_Z11preFreeSpMVPdPiS0_S_S_iiiS_S_), same meaning — host CSR
// arrays in, Y_val overwritten with A*x, *cdTime = ms per multiply over the
// timed launches, *cdPre = ms of the pre-pass. Linking libprefree_b200.so in
// place of the reference's libPreFreelib.a is the whole integration.
//
// Differences: failures print one line to stderr and set *cdTime = *cdPre = -1
// instead of calling exit() (include/common.h:49-58); row_ptr is read for
// rowA+1 entries, not rowA+2 (src/spmv_kernel/preFreeSpMV.cu:580).
//
// The two overloads are the same call for fp32 values (the reference's second
// type, `half`, does not compile: preFreeSpMV.cu:326) and for int64 row_ptr /
// sizes (nnz >= 2^31, which `int nnzA` cannot hold).
#pragma once

#include <cstdint>

void preFreeSpMV(double *csrVal, int *csrRowPtr, int *csrColInd,
                 double *X_val, double *Y_val, int rowA, int colA, int nnzA,
                 double *cdTime, double *cdPre);

void preFreeSpMV(float *csrVal, int *csrRowPtr, int *csrColInd,
                 float *X_val, float *Y_val, int rowA, int colA, int nnzA,
                 double *cdTime, double *cdPre);

void preFreeSpMV(double *csrVal, int64_t *csrRowPtr, int *csrColInd,
                 double *X_val, double *Y_val, int64_t rowA, int64_t colA,
                 int64_t nnzA, double *cdTime, double *cdPre);
