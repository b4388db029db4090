// oracle/oracle_internal.h -- shared declarations of the CPU parity oracle.
//
// TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); never part
// of the product path.
#pragma once
#include <cstddef>
#include <cstdint>
#include <functional>

namespace orc {
void set_threads(int n);
int get_threads();
void parallel_for(int n, const std::function<void(int)>& f);
// C[m][:] += arow[m] (length K) . B[K][N]   (arow[m] == nullptr means a zero row)
void gemm_rows_acc(int M, int N, int K, const float* const* arow, const float* B, int ldb,
                   float* const* crow);
void gemm_acc(int M, int N, int K, const float* A, int lda, const float* B, int ldb, float* C, int ldc);
}  // namespace orc
