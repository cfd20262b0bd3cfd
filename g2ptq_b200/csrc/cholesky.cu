// Damped inverse-Cholesky factor U (U^T U = (H + d I)^-1), UL route.
//
// H + dI = V V^T with V upper triangular gives (H + dI)^-1 = V^-T V^-1, so
// U = V^-1.  With the reversal P (index i -> C-1-i), P (H + dI) P = L L^T is an
// ordinary lower Cholesky factorization, V = P L P and U = P L^-1 P.
//
// Blocked right-looking factorization with 128-wide panels that accumulates
// X = L^-1 alongside L (block forward substitution of L X = I):
//   for k:  L_kk = chol(A_kk);  Linv_kk = L_kk^-1                (panel kernel)
//           L_ik = A_ik Linv_kk^T            (i > k)             (GEMM)
//           X_k: = Linv_kk Y_k:                                  (GEMM)
//           A_ij -= L_ik L_jk^T              (i >= j > k)        (GEMM, lower)
//           Y_i: -= L_ik X_k:                (i > k)             (GEMM)
// potrf + trtri = 2C^3/3 flops, where the reference chain
// potrf -> cholesky_inverse -> potrf(upper) costs 4C^3/3.
#include "gemm_simt.cuh"

namespace g2q {

constexpr int NB = 128;

// mean(diag(H)) -> *out (one block).
__global__ void mean_diag_kernel(const float* H, long long C, long long ldh, float* out) {
  __shared__ float red[32];
  float s = 0.f;
  for (long long i = threadIdx.x; i < C; i += blockDim.x) s += H[i * ldh + i];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) *out = s / (float)C;
  }
}

// A[i][j] = H[C-1-i][C-1-j] (+ damp on the diagonal) for j <= i; Y = I.
__global__ void reverse_damp_kernel(const float* H, long long C, long long ldh,
                                    const float* mean_diag, float damp_percent,
                                    float* A, float* Y) {
  const float damp = damp_percent * (*mean_diag);
  long long n = C * C;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    long long i = idx / C, j = idx - i * C;
    float v = 0.f;
    if (j <= i) {
      v = H[(C - 1 - i) * ldh + (C - 1 - j)];
      if (i == j) v += damp;
    }
    A[idx] = v;
    Y[idx] = (i == j) ? 1.f : 0.f;
  }
}

// Factor the nb x nb diagonal block at (k0, k0) of A in place and write its
// lower-triangular inverse to Linv (NB x NB, zero padded).  One pass over the
// pivots computes both: after pivot j scales column j of L, the rows below
// eliminate it from the trailing matrix (a[i][k] -= l_ij l_kj) and from the
// forward substitution of L X = I (x[i][:j+1] -= l_ij x[j][:j+1]).  A 16 x 16
// thread grid covers each trailing triangle.
__global__ void __launch_bounds__(256) panel_kernel(float* A, long long C, long long k0, int nb,
                                                    float* Linv, int* info) {
  extern __shared__ float panel_smem[];
  float (*a)[NB + 1] = reinterpret_cast<float (*)[NB + 1]>(panel_smem);
  float (*x)[NB + 1] = reinterpret_cast<float (*)[NB + 1]>(panel_smem + NB * (NB + 1));
  __shared__ int failed;
  const int t = threadIdx.x;
  const int ty = t >> 4, tx = t & 15;
  for (int idx = t; idx < NB * NB; idx += blockDim.x) {
    const int i = idx / NB, j = idx % NB;
    a[i][j] = (i < nb && j < nb && j <= i) ? A[(k0 + i) * C + k0 + j] : 0.f;
    x[i][j] = (i == j && i < nb) ? 1.f : 0.f;
  }
  if (t == 0) failed = 0;
  __syncthreads();

  for (int j = 0; j < nb; ++j) {
    const float d = a[j][j];
    if (!(d > 0.f)) {  // non-positive or NaN pivot (uniform across the block)
      if (t == 0) {
        failed = 1;
        if (info) atomicCAS(info, 0, (int)(k0 + j + 1));
      }
      break;
    }
    const float l = sqrtf(d);
    __syncthreads();  // every thread has read a[j][j]
    for (int i = j + 1 + t; i < nb; i += blockDim.x) a[i][j] = a[i][j] / l;
    for (int c = t; c <= j; c += blockDim.x) x[j][c] = x[j][c] / l;
    if (t == 0) a[j][j] = l;
    __syncthreads();
    for (int i = j + 1 + ty; i < nb; i += 16) {
      const float lij = a[i][j];
      for (int k = j + 1 + tx; k <= i; k += 16) a[i][k] = fmaf(-lij, a[k][j], a[i][k]);
      for (int c = tx; c <= j; c += 16) x[i][c] = fmaf(-lij, x[j][c], x[i][c]);
    }
    __syncthreads();
  }
  __syncthreads();
  if (failed) {
    // mark the inverse as NaN so downstream products are visibly invalid
    for (int idx = t; idx < NB * NB; idx += blockDim.x) Linv[idx] = __int_as_float(0x7fc00000);
    return;
  }
  for (int idx = t; idx < NB * NB; idx += blockDim.x) {
    const int i = idx / NB, j = idx % NB;
    Linv[idx] = (i < nb && j < nb) ? x[i][j] : 0.f;
    if (i < nb && j <= i) A[(k0 + i) * C + k0 + j] = a[i][j];
  }
}

// U[i][j] = X[C-1-i][C-1-j] for i <= j, 0 below; NaN -> info = -1.
__global__ void extract_u_kernel(const float* X, long long C, float* U, int* info) {
  long long n = C * C;
  bool nan_seen = false;
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    long long i = idx / C, j = idx - i * C;
    float v = 0.f;
    if (i <= j) {
      v = X[(C - 1 - i) * C + (C - 1 - j)];
      if (v != v) nan_seen = true;
    }
    U[idx] = v;
  }
  if (nan_seen && info) atomicCAS(info, 0, -1);
}

static int gemm(float* Cp, long long ldc, const float* Ap, long long lda, bool ta,
                const float* Bp, long long ldb, bool tb, long long M, long long N, long long K,
                float alpha, float beta, int mask, cudaStream_t st) {
  return simt_gemm_f32(Cp, ldc, Ap, lda, ta, Bp, ldb, tb, M, N, K, alpha, beta, mask, st);
}

static constexpr size_t kPanelSmem = 2 * NB * (NB + 1) * sizeof(float);

static int ensure_panel_attr() {
  static int done[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return G2Q_ERR_CUDA;
  if (dev < 64 && done[dev]) return G2Q_OK;
  if (cudaFuncSetAttribute(panel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kPanelSmem) != cudaSuccess)
    return G2Q_ERR_CUDA;
  if (dev < 64) done[dev] = 1;
  return G2Q_OK;
}

int split3(const float* src, long long lds, long long rows, long long cols, __nv_bfloat16* h,
           __nv_bfloat16* m, __nv_bfloat16* l, long long ldd, int transpose, cudaStream_t st);
int tc_update3(float* D, long long ldd, long long M, long long N, long long K,
               __nv_bfloat16* const* a3, long long lda, __nv_bfloat16* const* b3, long long ldb,
               int lower, float alpha, float beta, cudaStream_t st);

// Trailing updates of step k on the tensor cores, fp32-accurate (three-term
// bf16 split, six products): A_ij -= L_ik L_jk^T (lower) and Y_i: -= L_ik X_k:.
// Returns G2Q_ERR_UNSUPPORTED when the shapes do not suit TMA.
static int tc_trailing(float* A, float* Y, long long C, long long k0, int nb, long long rest,
                       __nv_bfloat16* lt, __nv_bfloat16* xk, cudaStream_t st) {
  if (C % 8) return G2Q_ERR_UNSUPPORTED;
  const long long tsz = (long long)NB * C;
  __nv_bfloat16* l3[3] = {lt, lt + tsz, lt + 2 * tsz};
  __nv_bfloat16* x3[3] = {xk, xk + tsz, xk + 2 * tsz};
  // L_ik^T (nb x rest, row stride C) and X_k: (nb x (k0 + nb), row stride C)
  G2Q_TRY(split3(A + (k0 + nb) * C + k0, C, rest, nb, l3[0], l3[1], l3[2], C, 1, st));
  G2Q_TRY(split3(Y + k0 * C, C, nb, k0 + nb, x3[0], x3[1], x3[2], C, 0, st));
  int s = tc_update3(A + (k0 + nb) * C + (k0 + nb), C, rest, rest, nb, l3, C, l3, C, 1, 1.f,
                     -1.f, st);
  if (s != G2Q_OK) return s;
  return tc_update3(Y + (k0 + nb) * C, C, rest, k0 + nb, nb, l3, C, x3, C, 0, 1.f, -1.f, st);
}

static int chol_one(float* U, const float* H, long long C, long long ldh, float damp_percent,
                    int* info, float* ws, int precision, cudaStream_t st) {
  float* A = ws;
  float* Y = A + C * C;
  float* Linv = Y + C * C;
  float* mdiag = Linv + NB * NB;
  __nv_bfloat16* lt = reinterpret_cast<__nv_bfloat16*>(mdiag + 64);
  __nv_bfloat16* xk = lt + 3 * (long long)NB * C;
  G2Q_TRY(ensure_panel_attr());
  if (info && cudaMemsetAsync(info, 0, sizeof(int), st) != cudaSuccess) return G2Q_ERR_CUDA;
  mean_diag_kernel<<<1, 1024, 0, st>>>(H, C, ldh, mdiag);
  G2Q_CHECK_LAUNCH();
  int blocks = (int)((C * C + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  reverse_damp_kernel<<<blocks, 256, 0, st>>>(H, C, ldh, mdiag, damp_percent, A, Y);
  G2Q_CHECK_LAUNCH();
  for (long long k0 = 0; k0 < C; k0 += NB) {
    const int nb = (int)((C - k0) < NB ? (C - k0) : NB);
    const long long rest = C - k0 - nb;
    panel_kernel<<<1, 256, kPanelSmem, st>>>(A, C, k0, nb, Linv, info);
    G2Q_CHECK_LAUNCH();
    // X_k: = Linv_kk Y_k:  (columns 0 .. k0+nb), in place in Y
    G2Q_TRY(gemm(Y + k0 * C, C, Linv, NB, false, Y + k0 * C, C, false, nb, k0 + nb, nb,
                 0.f, 1.f, G2Q_MASK_FULL, st));
    if (rest <= 0) break;
    // L_ik = A_ik Linv_kk^T, in place in A
    G2Q_TRY(gemm(A + (k0 + nb) * C + k0, C, A + (k0 + nb) * C + k0, C, false, Linv, NB, true,
                 rest, nb, nb, 0.f, 1.f, G2Q_MASK_FULL, st));
    if (precision == 1) {
      const int s_tc = tc_trailing(A, Y, C, k0, nb, rest, lt, xk, st);
      if (s_tc == G2Q_OK) continue;
      if (s_tc != G2Q_ERR_UNSUPPORTED) return s_tc;
    }
    // A_ij -= L_ik L_jk^T (lower triangle of the trailing matrix)
    G2Q_TRY(gemm(A + (k0 + nb) * C + (k0 + nb), C, A + (k0 + nb) * C + k0, C, false,
                 A + (k0 + nb) * C + k0, C, true, rest, rest, nb, 1.f, -1.f, G2Q_MASK_LOWER,
                 st));
    // Y_i: -= L_ik X_k:
    G2Q_TRY(gemm(Y + (k0 + nb) * C, C, A + (k0 + nb) * C + k0, C, false, Y + k0 * C, C, false,
                 rest, k0 + nb, nb, 1.f, -1.f, G2Q_MASK_FULL, st));
  }
  extract_u_kernel<<<blocks, 256, 0, st>>>(Y, C, U, info);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

}  // namespace g2q

extern "C" size_t g2q_chol_workspace_bytes(int64_t C) {
  return (size_t)(2 * C * C + g2q::NB * g2q::NB + 64) * sizeof(float) +
         (size_t)6 * g2q::NB * C * sizeof(__nv_bfloat16) + 256;
}

extern "C" int g2q_chol_upper_inverse(float* U, const float* H, int64_t C, int64_t ldh,
                                      int64_t batch, const float* damp_percent_host, int* info,
                                      int precision, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  if (!U || !H || C <= 0 || ldh < C || batch < 0 || !damp_percent_host || !workspace)
    return G2Q_ERR_INVALID_ARG;
  if (workspace_bytes < g2q_chol_workspace_bytes(C)) return G2Q_ERR_INVALID_ARG;
  if (precision != 0 && precision != 1) return G2Q_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  for (int64_t b = 0; b < batch; ++b) {
    G2Q_TRY(g2q::chol_one(U + b * C * C, H + b * C * ldh, C, ldh, damp_percent_host[b],
                          info ? info + b : nullptr, (float*)workspace, precision, st));
  }
  return G2Q_OK;
}
