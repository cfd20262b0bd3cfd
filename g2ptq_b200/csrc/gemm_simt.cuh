// fp32 CUDA-core GEMM entry used inside the library.
#pragma once
#include "common.cuh"

namespace g2q {

struct SimtArgs {
  const void* A;
  const void* B;
  float* C;
  long long lda, ldb, ldc;
  long long sA, sB, sC;  // batch strides (elements)
  long long M, N, K;
  float alpha, beta;
  const float* kscale;   // per-k scale applied to B (Gram row scale), nullable
  long long kscale_stride;
  int mask;              // G2Q_MASK_*
  int mirror;            // write C[n][m] too (symmetric Gram, upper tiles)
};

// TA: A stored [K, M]; TB: B stored [N, K].  Types: G2Q_DTYPE_F32 / _BF16.
int simt_gemm(const SimtArgs& a, bool ta, bool tb, int a_dtype, int b_dtype, long long batch,
              cudaStream_t st);

// Convenience wrapper for single fp32 products.
int simt_gemm_f32(float* C, long long ldc, const float* A, long long lda, bool ta,
                  const float* B, long long ldb, bool tb, long long M, long long N, long long K,
                  float alpha, float beta, int mask, cudaStream_t st, long long batch = 1,
                  long long sA = 0, long long sB = 0, long long sC = 0);

}  // namespace g2q
