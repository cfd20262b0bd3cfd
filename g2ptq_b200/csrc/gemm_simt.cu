// fp32 CUDA-core GEMM / Gram kernels.
//
// C <- alpha * C + beta * op(A) op(B) [+ mask], 128x128x8 tiles, 256 threads,
// an 8x8 register tile per thread, double-buffered shared memory.  Used where
// fp32 accuracy is required end to end (Cholesky trailing updates, the G2PTQ
// and GPTAQ precompute products) and as the exact-arithmetic path of the
// Hessian and trailing updates.
#include "gemm_simt.cuh"

namespace g2q {



template <typename T>
__device__ __forceinline__ float ld_elem(const T* p);
template <>
__device__ __forceinline__ float ld_elem<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_elem<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

constexpr int BM = 128, BN = 128, BK = 8;

// TA: A stored [K, M] (element (m,k) at A[k*lda + m]); else [M, K].
// TB: B stored [N, K] (element (k,n) at B[n*ldb + k]); else [K, N].
template <bool TA, bool TB, typename TAe, typename TBe>
__global__ void __launch_bounds__(256) simt_gemm_kernel(SimtArgs p) {
  const long long m0 = (long long)blockIdx.y * BM;
  const long long n0 = (long long)blockIdx.x * BN;
  // Tiles that hold no element of the requested triangle do nothing.
  if ((p.mask == G2Q_MASK_LOWER) && (m0 + BM - 1 < n0)) return;
  if ((p.mask == G2Q_MASK_UPPER || p.mirror) && (n0 + BN - 1 < m0)) return;

  const long long bz = blockIdx.z;
  const TAe* A = reinterpret_cast<const TAe*>(p.A) + bz * p.sA;
  const TBe* B = reinterpret_cast<const TBe*>(p.B) + bz * p.sB;
  float* C = p.C + bz * p.sC;

  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  float ra[4], rb[4];
  // loader coordinates
  // TA: k = tid/32, m = (tid%32)*4 + u ; !TA: m = tid/2, k = (tid%2)*4 + u
  auto load_a = [&](long long k0) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      long long m, k;
      if (TA) { k = tid >> 5; m = (tid & 31) * 4 + u; }
      else    { m = tid >> 1; k = (tid & 1) * 4 + u; }
      long long gm = m0 + m, gk = k0 + k;
      float v = 0.f;
      if (gm < p.M && gk < p.K) v = TA ? ld_elem(A + gk * p.lda + gm) : ld_elem(A + gm * p.lda + gk);
      ra[u] = v;
    }
  };
  auto load_b = [&](long long k0) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      long long n, k;
      if (!TB) { k = tid >> 5; n = (tid & 31) * 4 + u; }
      else     { n = tid >> 1; k = (tid & 1) * 4 + u; }
      long long gn = n0 + n, gk = k0 + k;
      float v = 0.f;
      if (gn < p.N && gk < p.K) {
        v = TB ? ld_elem(B + gn * p.ldb + gk) : ld_elem(B + gk * p.ldb + gn);
        if (p.kscale) v *= __ldg(p.kscale + gk * p.kscale_stride);
      }
      rb[u] = v;
    }
  };
  auto store_ab = [&](int buf) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (TA) As[buf][tid >> 5][(tid & 31) * 4 + u] = ra[u];
      else    As[buf][(tid & 1) * 4 + u][tid >> 1] = ra[u];
      if (!TB) Bs[buf][tid >> 5][(tid & 31) * 4 + u] = rb[u];
      else     Bs[buf][(tid & 1) * 4 + u][tid >> 1] = rb[u];
    }
  };

  const long long nk = (p.K + BK - 1) / BK;
  if (nk > 0) {
    load_a(0);
    load_b(0);
    store_ab(0);
  }
  __syncthreads();
  for (long long kt = 0; kt < nk; ++kt) {
    const int buf = (int)(kt & 1);
    if (kt + 1 < nk) {
      load_a((kt + 1) * BK);
      load_b((kt + 1) * BK);
    }
#pragma unroll
    for (int k = 0; k < BK; ++k) {
      float a[8], b[8];
      float4 a0 = *reinterpret_cast<const float4*>(&As[buf][k][ty * 4]);
      float4 a1 = *reinterpret_cast<const float4*>(&As[buf][k][64 + ty * 4]);
      float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][k][tx * 4]);
      float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][k][64 + tx * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < nk) store_ab(buf ^ 1);
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const long long gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (gm >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const long long gn = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
      if (gn >= p.N) continue;
      bool inside = true;
      if (p.mask == G2Q_MASK_LOWER) inside = gm >= gn;
      else if (p.mask == G2Q_MASK_UPPER || p.mirror) inside = gm <= gn;
      else if (p.mask == G2Q_MASK_STRICT_UPPER) inside = gm < gn;
      float* dst = C + gm * p.ldc + gn;
      if (!inside) {
        if (p.mask == G2Q_MASK_STRICT_UPPER) *dst = 0.f;
        continue;
      }
      float v = p.beta * acc[i][j];
      if (p.alpha != 0.f) v = fmaf(p.alpha, *dst, v);
      *dst = v;
      if (p.mirror && gm != gn) C[gn * p.ldc + gm] = v;
    }
  }
}

template <bool TA, bool TB, typename TAe, typename TBe>
static int launch_simt(const SimtArgs& a, long long batch, cudaStream_t st) {
  if (a.M <= 0 || a.N <= 0 || batch <= 0) return G2Q_OK;
  dim3 grid(cdiv(a.N, BN), cdiv(a.M, BM), (unsigned)batch);
  if (grid.y > 65535u || grid.z > 65535u) return G2Q_ERR_INVALID_ARG;
  simt_gemm_kernel<TA, TB, TAe, TBe><<<grid, 256, 0, st>>>(a);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

int simt_gemm(const SimtArgs& a, bool ta, bool tb, int a_dtype, int b_dtype, long long batch,
              cudaStream_t st) {
  if (a_dtype == G2Q_DTYPE_F32 && b_dtype == G2Q_DTYPE_F32) {
    if (!ta && !tb) return launch_simt<false, false, float, float>(a, batch, st);
    if (!ta && tb) return launch_simt<false, true, float, float>(a, batch, st);
    if (ta && !tb) return launch_simt<true, false, float, float>(a, batch, st);
    return launch_simt<true, true, float, float>(a, batch, st);
  }
  // Gram products over staged tokens: A stored [T, M], B stored [T, N].
  if (ta && !tb) {
    if (a_dtype == G2Q_DTYPE_BF16 && b_dtype == G2Q_DTYPE_BF16)
      return launch_simt<true, false, __nv_bfloat16, __nv_bfloat16>(a, batch, st);
    if (a_dtype == G2Q_DTYPE_F32 && b_dtype == G2Q_DTYPE_BF16)
      return launch_simt<true, false, float, __nv_bfloat16>(a, batch, st);
    if (a_dtype == G2Q_DTYPE_BF16 && b_dtype == G2Q_DTYPE_F32)
      return launch_simt<true, false, __nv_bfloat16, float>(a, batch, st);
  }
  return G2Q_ERR_UNSUPPORTED;
}

int simt_gemm_f32(float* C, long long ldc, const float* A, long long lda, bool ta,
                  const float* B, long long ldb, bool tb, long long M, long long N, long long K,
                  float alpha, float beta, int mask, cudaStream_t st, long long batch,
                  long long sA, long long sB, long long sC) {
  SimtArgs a{};
  a.A = A; a.B = B; a.C = C;
  a.lda = lda; a.ldb = ldb; a.ldc = ldc;
  a.sA = sA; a.sB = sB; a.sC = sC;
  a.M = M; a.N = N; a.K = K;
  a.alpha = alpha; a.beta = beta;
  a.mask = mask;
  return simt_gemm(a, ta, tb, G2Q_DTYPE_F32, G2Q_DTYPE_F32, batch, st);
}

}  // namespace g2q

extern "C" int g2q_gemm(float* C, int64_t ldc, int64_t strideC,
                        const float* A, int64_t lda, int64_t strideA, int transA,
                        const float* B, int64_t ldb, int64_t strideB, int transB,
                        int64_t M, int64_t N, int64_t K, int64_t batch,
                        float alpha, float beta, int out_mask, void* stream) {
  if (!C || (!A && K > 0) || (!B && K > 0) || M < 0 || N < 0 || K < 0 || batch < 0)
    return G2Q_ERR_INVALID_ARG;
  if (out_mask < 0 || out_mask > 3) return G2Q_ERR_INVALID_ARG;
  g2q::SimtArgs a{};
  a.A = A; a.B = B; a.C = C;
  a.lda = lda; a.ldb = ldb; a.ldc = ldc;
  a.sA = strideA; a.sB = strideB; a.sC = strideC;
  a.M = M; a.N = N; a.K = K;
  a.alpha = alpha; a.beta = beta;
  a.kscale = nullptr; a.kscale_stride = 0;
  a.mask = out_mask; a.mirror = 0;
  return g2q::simt_gemm(a, transA != 0, transB != 0, G2Q_DTYPE_F32, G2Q_DTYPE_F32, batch,
                        (cudaStream_t)stream);
}
