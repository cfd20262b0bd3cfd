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

constexpr int BK = 8;

// TILE x TILE output tile per CTA (TILE = 128: 8x8 per thread, 64: 4x4),
// 256 threads, BK = 8, double-buffered shared memory.
// TA: A stored [K, M] (element (m,k) at A[k*lda + m]); else [M, K].
// TB: B stored [N, K] (element (k,n) at B[n*ldb + k]); else [K, N].
template <bool TA, bool TB, typename TAe, typename TBe, int TILE>
__global__ void __launch_bounds__(256) simt_gemm_kernel(SimtArgs p) {
  constexpr int TT = TILE / 16;        // outputs per thread per dimension
  constexpr int LPT = TILE * BK / 256;  // tile elements each thread loads per operand
  const long long m0 = (long long)blockIdx.y * TILE;
  const long long n0 = (long long)blockIdx.x * TILE;
  // Tiles that hold no element of the requested triangle do nothing.
  if ((p.mask == G2Q_MASK_LOWER) && (m0 + TILE - 1 < n0)) return;
  if ((p.mask == G2Q_MASK_UPPER || p.mirror) && (n0 + TILE - 1 < m0)) return;

  const long long bz = blockIdx.z;
  const TAe* A = reinterpret_cast<const TAe*>(p.A) + bz * p.sA;
  const TBe* B = reinterpret_cast<const TBe*>(p.B) + bz * p.sB;
  float* C = p.C + bz * p.sC;

  __shared__ __align__(16) float As[2][BK][TILE];
  __shared__ __align__(16) float Bs[2][BK][TILE];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;

  float acc[TT][TT];
#pragma unroll
  for (int i = 0; i < TT; ++i)
#pragma unroll
    for (int j = 0; j < TT; ++j) acc[i][j] = 0.f;

  float ra[LPT], rb[LPT];
  auto load_a = [&](long long k0) {
#pragma unroll
    for (int u = 0; u < LPT; ++u) {
      const int idx = tid + 256 * u;
      long long m, k;
      if (TA) { k = idx / TILE; m = idx % TILE; }
      else    { m = idx / BK; k = idx % BK; }
      const long long gm = m0 + m, gk = k0 + k;
      float v = 0.f;
      if (gm < p.M && gk < p.K) v = TA ? ld_elem(A + gk * p.lda + gm) : ld_elem(A + gm * p.lda + gk);
      ra[u] = v;
    }
  };
  auto load_b = [&](long long k0) {
#pragma unroll
    for (int u = 0; u < LPT; ++u) {
      const int idx = tid + 256 * u;
      long long n, k;
      if (!TB) { k = idx / TILE; n = idx % TILE; }
      else     { n = idx / BK; k = idx % BK; }
      const long long gn = n0 + n, gk = k0 + k;
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
    for (int u = 0; u < LPT; ++u) {
      const int idx = tid + 256 * u;
      if (TA) As[buf][idx / TILE][idx % TILE] = ra[u];
      else    As[buf][idx % BK][idx / BK] = ra[u];
      if (!TB) Bs[buf][idx / TILE][idx % TILE] = rb[u];
      else     Bs[buf][idx % BK][idx / BK] = rb[u];
    }
  };
  // output rows / columns of this thread: four consecutive at ty*4 (and at
  // TILE/2 + ty*4 for the 8 x 8 case)
  auto off = [](int i, int base) { return i < 4 ? base * 4 + i : TILE / 2 + base * 4 + (i - 4); };

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
      float a[TT], b[TT];
#pragma unroll
      for (int h = 0; h < TT / 4; ++h) {
        const float4 a4 = *reinterpret_cast<const float4*>(&As[buf][k][off(4 * h, ty)]);
        const float4 b4 = *reinterpret_cast<const float4*>(&Bs[buf][k][off(4 * h, tx)]);
        a[4 * h] = a4.x; a[4 * h + 1] = a4.y; a[4 * h + 2] = a4.z; a[4 * h + 3] = a4.w;
        b[4 * h] = b4.x; b[4 * h + 1] = b4.y; b[4 * h + 2] = b4.z; b[4 * h + 3] = b4.w;
      }
#pragma unroll
      for (int i = 0; i < TT; ++i)
#pragma unroll
        for (int j = 0; j < TT; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (kt + 1 < nk) store_ab(buf ^ 1);
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < TT; ++i) {
    const long long gm = m0 + off(i, ty);
    if (gm >= p.M) continue;
#pragma unroll
    for (int j = 0; j < TT; ++j) {
      const long long gn = n0 + off(j, tx);
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
  // 64 x 64 tiles when 128 x 128 tiles would leave most SMs idle
  const long long big = (long long)cdiv(a.N, 128) * cdiv(a.M, 128) * batch;
  if (big < 2 * 148) {
    dim3 grid(cdiv(a.N, 64), cdiv(a.M, 64), (unsigned)batch);
    if (grid.y > 65535u || grid.z > 65535u) return G2Q_ERR_INVALID_ARG;
    simt_gemm_kernel<TA, TB, TAe, TBe, 64><<<grid, 256, 0, st>>>(a);
  } else {
    dim3 grid(cdiv(a.N, 128), cdiv(a.M, 128), (unsigned)batch);
    if (grid.y > 65535u || grid.z > 65535u) return G2Q_ERR_INVALID_ARG;
    simt_gemm_kernel<TA, TB, TAe, TBe, 128><<<grid, 256, 0, st>>>(a);
  }
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
