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
// The factorization (panel, TRSM, SYRK) runs on the caller's stream; the
// inverse chain (X_k, Y update), which no later panel depends on, runs on a
// library-owned side stream ordered by per-step events and joined at the end.
#include <cuda_fp16.h>

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
// lower-triangular inverse to Linv (NB x NB, zero padded).
//
// The block and its inverse live in registers: thread (ty, tx) of a 16 x 16
// grid owns rows 8ty..8ty+7 x columns 8tx..8tx+7 of both L and X = L^-1.
// Blocked right-looking factorization, eight pivots at a time:
//   1. the thread holding diagonal tile jb runs the unblocked factorization of
//      that tile (columns scaled by 1/l_jj, as LAPACK's spotf2);
//   2. the tiles under it apply the same eight pivots to their rows (the strip
//      L_ij), and the tiles of block row jb of X run the forward substitution
//      of L X = I for those eight rows;
//   3. rank-8 updates A_ik -= L_ij L_kj^T of the lower trailing tiles and
//      X_i: -= L_ij X_j: of X.
// Every element sees the same operations in the same order as with one pivot
// at a time, but with two block-wide barriers per eight pivots.
__global__ void __launch_bounds__(256) panel_kernel(float* A, long long C, long long k0, int nb,
                                                    float* Linv, int* info) {
  __shared__ __align__(16) float Ls[8][NB];  // strip L_ij, transposed (column k of the strip)
  __shared__ __align__(16) float Xb[8][NB];  // finished rows of X in block row jb
  __shared__ float Ld[8][8];                 // L_jj (scaled columns)
  __shared__ float Rl[8];                    // 1 / l_jj
  __shared__ int failed;
  const int t = threadIdx.x;
  const int ty = t >> 4, tx = t & 15;
  const int r0 = ty * 8, c0 = tx * 8;
  float a[8][8], x[8][8];
#pragma unroll
  for (int u = 0; u < 8; ++u)
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      const int r = r0 + u, c = c0 + v;
      a[u][v] = (r < nb && c <= r) ? A[(k0 + r) * C + k0 + c] : 0.f;
      x[u][v] = (r == c && r < nb) ? 1.f : 0.f;
    }
  if (t == 0) failed = 0;
  __syncthreads();

  for (int jb = 0; jb * 8 < nb; ++jb) {
    const int j0 = jb * 8;
    const int nbk = (nb - j0) < 8 ? (nb - j0) : 8;
    // ---- 1. diagonal tile
    if (ty == jb && tx == jb) {
      bool ok = true;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float rl = 0.f;
        if (j < nbk && ok) {
          const float d = a[j][j];
          if (!(d > 0.f)) {  // non-positive or NaN pivot
            ok = false;
            failed = 1;
            if (info) atomicCAS(info, 0, (int)(k0 + j0 + j + 1));
          } else {
            const float l = sqrtf(d);
            rl = 1.f / l;
            a[j][j] = l;
#pragma unroll
            for (int u = j + 1; u < 8; ++u) a[u][j] *= rl;
#pragma unroll
            for (int u = j + 1; u < 8; ++u)
#pragma unroll
              for (int v = j + 1; v <= u; ++v) a[u][v] = fmaf(-a[u][j], a[v][j], a[u][v]);
          }
        }
        Rl[j] = rl;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int v = 0; v < 8; ++v) Ld[u][v] = (v < u) ? a[u][v] : 0.f;
    }
    __syncthreads();
    if (failed) break;  // uniform after the barrier
    // ---- 2. the eight pivots on the strip, and on block row jb of X
    if (tx == jb && ty > jb) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j >= nbk) continue;
        const float rl = Rl[j];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float sv = a[u][j] * rl;
          a[u][j] = sv;
          Ls[j][r0 + u] = sv;
#pragma unroll
          for (int v = j + 1; v < 8; ++v) a[u][v] = fmaf(-sv, Ld[v][j], a[u][v]);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j >= nbk) {
#pragma unroll
          for (int u = 0; u < 8; ++u) Ls[j][r0 + u] = 0.f;
        }
    }
    if (ty == jb && tx <= jb) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float rl = Rl[j];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const float xf = (j < nbk) ? x[j][v] * rl : 0.f;
          x[j][v] = xf;
          Xb[j][c0 + v] = xf;
#pragma unroll
          for (int u = j + 1; u < 8; ++u) x[u][v] = fmaf(-Ld[u][j], xf, x[u][v]);
        }
      }
    }
    __syncthreads();
    // ---- 3. rank-8 updates of the trailing lower tiles and of X
    if (ty > jb) {
      float lr[8][8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float4 p0 = *reinterpret_cast<const float4*>(&Ls[k][r0]);
        const float4 p1 = *reinterpret_cast<const float4*>(&Ls[k][r0 + 4]);
        lr[k][0] = p0.x; lr[k][1] = p0.y; lr[k][2] = p0.z; lr[k][3] = p0.w;
        lr[k][4] = p1.x; lr[k][5] = p1.y; lr[k][6] = p1.z; lr[k][7] = p1.w;
      }
      if (tx > jb && tx <= ty) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float4 q0 = *reinterpret_cast<const float4*>(&Ls[k][c0]);
          const float4 q1 = *reinterpret_cast<const float4*>(&Ls[k][c0 + 4]);
          const float lc[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
          for (int u = 0; u < 8; ++u)
#pragma unroll
            for (int v = 0; v < 8; ++v) a[u][v] = fmaf(-lr[k][u], lc[v], a[u][v]);
        }
      } else if (tx <= jb) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float4 q0 = *reinterpret_cast<const float4*>(&Xb[k][c0]);
          const float4 q1 = *reinterpret_cast<const float4*>(&Xb[k][c0 + 4]);
          const float xc[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
          for (int u = 0; u < 8; ++u)
#pragma unroll
            for (int v = 0; v < 8; ++v) x[u][v] = fmaf(-lr[k][u], xc[v], x[u][v]);
        }
      }
    }
  }
  __syncthreads();
  if (failed) {
    // mark the inverse as NaN so downstream products are visibly invalid
    for (int idx = t; idx < NB * NB; idx += blockDim.x) Linv[idx] = __int_as_float(0x7fc00000);
    return;
  }
#pragma unroll
  for (int u = 0; u < 8; ++u)
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      const int r = r0 + u, c = c0 + v;
      Linv[r * NB + c] = (r < nb && c < nb) ? x[u][v] : 0.f;
      if (r < nb && c <= r) A[(k0 + r) * C + k0 + c] = a[u][v];
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



int split2h(const float* src, long long lds, long long n, int K, __half* hi, __half* lo,
            long long ldd, float* scale, int transpose, cudaStream_t st);
int tc_update2h(float* D, long long ldd, long long M, long long N, long long K,
                __half* const* a2, const float* sa, long long lda, __half* const* b2,
                const float* sb, long long ldb, int lower, float alpha, float beta,
                cudaStream_t st);

// Side stream and per-step events of the inverse chain, one set per (device,
// caller stream) so that factorizations issued on different streams overlap.
struct SideState {
  int dev = -1;
  cudaStream_t main = nullptr;
  cudaStream_t side = nullptr;
  cudaEvent_t* ev = nullptr;  // [2 * cap]: factor-step-done, inverse-step-done
  int cap = 0;
};

static int side_state(cudaStream_t main, int steps, SideState** out) {
  constexpr int kSlots = 64;
  static SideState states[kSlots];
  static int next_slot = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return G2Q_ERR_CUDA;
  SideState* s = nullptr;
  for (int i = 0; i < kSlots; ++i)
    if (states[i].side && states[i].dev == dev && states[i].main == main) s = &states[i];
  if (!s) {
    s = &states[next_slot];
    next_slot = (next_slot + 1) % kSlots;
    if (s->side && s->dev != dev) {
      *s = SideState();  // slot held a stream of another device: start over
    }
    // the inverse chain runs at the caller's stream priority
    int prio = 0;
    if (!s->side && (cudaStreamGetPriority(main, &prio) != cudaSuccess ||
                     cudaStreamCreateWithPriority(&s->side, cudaStreamNonBlocking, prio) !=
                         cudaSuccess))
      return G2Q_ERR_CUDA;
    s->dev = dev;
    s->main = main;
  }
  if (s->cap < steps + 1) {
    cudaEvent_t* ev = new cudaEvent_t[2 * (steps + 1)];
    for (int i = 0; i < 2 * (steps + 1); ++i)
      if (cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) != cudaSuccess)
        return G2Q_ERR_CUDA;
    // events of the previous set may still be referenced by queued work; keep them
    s->ev = ev;
    s->cap = steps + 1;
  }
  *out = s;
  return G2Q_OK;
}

static bool tc_ok(long long C) { return C % 8 == 0; }

// Workspace layout (floats unless noted): A [C*C], Y [C*C], diagonal inverses
// [nblk][NB*NB], mean diag [64], then fp16: L21^T splits [2 buffers][2][NB*C],
// X_k splits [2][NB*C], then the splits' scales: L21 [2 buffers][C], X_k [C].
struct CholWs {
  float *A, *Y, *linv, *mdiag;
  __half *lt, *xk;
  float *lsc, *xsc;
};

static CholWs carve(float* ws, long long C) {
  CholWs w;
  const long long nblk = (C + NB - 1) / NB;
  w.A = ws;
  w.Y = w.A + C * C;
  w.linv = w.Y + C * C;
  w.mdiag = w.linv + nblk * NB * NB;
  w.lt = reinterpret_cast<__half*>(w.mdiag + 64);
  w.xk = w.lt + 2 * 2 * (long long)NB * C;
  w.lsc = reinterpret_cast<float*>(w.xk + 2 * (long long)NB * C);
  w.xsc = w.lsc + 2 * C;
  return w;
}

static int chol_one(float* U, const float* H, long long C, long long ldh, float damp_percent,
                    int* info, float* ws, int precision, cudaStream_t st) {
  CholWs w = carve(ws, C);
  float* A = w.A;
  float* Y = w.Y;
  const long long nblk = (C + NB - 1) / NB;
  const bool use_tc = precision == 1 && tc_ok(C);
  SideState* ss = nullptr;
  G2Q_TRY(side_state(st, (int)nblk, &ss));
  cudaStream_t side = ss->side;
  cudaEvent_t* ev = ss->ev;  // ev[2k]: factor step k done, ev[2k+1]: inverse step k done
  if (info && cudaMemsetAsync(info, 0, sizeof(int), st) != cudaSuccess) return G2Q_ERR_CUDA;
  mean_diag_kernel<<<1, 1024, 0, st>>>(H, C, ldh, w.mdiag);
  G2Q_CHECK_LAUNCH();
  int blocks = (int)((C * C + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  reverse_damp_kernel<<<blocks, 256, 0, st>>>(H, C, ldh, w.mdiag, damp_percent, A, Y);
  G2Q_CHECK_LAUNCH();
  const long long tsz = (long long)NB * C;
  for (long long kb = 0; kb < nblk; ++kb) {
    const long long k0 = kb * NB;
    const int nb = (int)((C - k0) < NB ? (C - k0) : NB);
    const long long rest = C - k0 - nb;
    float* linv = w.linv + kb * NB * NB;
    __half* lt = w.lt + (kb & 1) * 2 * tsz;
    __half* l2[2] = {lt, lt + tsz};
    float* lsc = w.lsc + (kb & 1) * C;
    __half* x2[2] = {w.xk, w.xk + tsz};
    // ---- factorization (caller's stream): panel, TRSM, split, SYRK
    panel_kernel<<<1, 256, 0, st>>>(A, C, k0, nb, linv, info);
    G2Q_CHECK_LAUNCH();
    if (rest > 0) {
      // L_ik = A_ik Linv_kk^T, in place in A
      G2Q_TRY(simt_gemm_f32(A + (k0 + nb) * C + k0, C, A + (k0 + nb) * C + k0, C, false, linv,
                            NB, true, rest, nb, nb, 0.f, 1.f, G2Q_MASK_FULL, st));
      if (use_tc) {
        // the inverse chain of step kb-2 used this L21^T buffer
        if (kb >= 2 && cudaStreamWaitEvent(st, ev[2 * (kb - 2) + 1], 0) != cudaSuccess)
          return G2Q_ERR_CUDA;
        G2Q_TRY(split2h(A + (k0 + nb) * C + k0, C, rest, nb, l2[0], l2[1], C, lsc, 1, st));
        G2Q_TRY(tc_update2h(A + (k0 + nb) * C + (k0 + nb), C, rest, rest, nb, l2, lsc, C, l2,
                            lsc, C, 1, 1.f, -1.f, st));
      } else {
        G2Q_TRY(simt_gemm_f32(A + (k0 + nb) * C + (k0 + nb), C, A + (k0 + nb) * C + k0, C, false,
                              A + (k0 + nb) * C + k0, C, true, rest, rest, nb, 1.f, -1.f,
                              G2Q_MASK_LOWER, st));
      }
    }
    if (cudaEventRecord(ev[2 * kb], st) != cudaSuccess) return G2Q_ERR_CUDA;
    // ---- inverse chain (side stream): X_k: = Linv_kk Y_k:, then Y_i: -= L_ik X_k:
    if (cudaStreamWaitEvent(side, ev[2 * kb], 0) != cudaSuccess) return G2Q_ERR_CUDA;
    G2Q_TRY(simt_gemm_f32(Y + k0 * C, C, linv, NB, false, Y + k0 * C, C, false, nb, k0 + nb, nb,
                          0.f, 1.f, G2Q_MASK_FULL, side));
    if (rest > 0) {
      if (use_tc) {
        G2Q_TRY(split2h(Y + k0 * C, C, k0 + nb, nb, x2[0], x2[1], C, w.xsc, 0, side));
        G2Q_TRY(tc_update2h(Y + (k0 + nb) * C, C, rest, k0 + nb, nb, l2, lsc, C, x2, w.xsc, C, 0,
                            1.f, -1.f, side));
      } else {
        G2Q_TRY(simt_gemm_f32(Y + (k0 + nb) * C, C, A + (k0 + nb) * C + k0, C, false, Y + k0 * C,
                              C, false, rest, k0 + nb, nb, 1.f, -1.f, G2Q_MASK_FULL, side));
      }
    }
    if (cudaEventRecord(ev[2 * kb + 1], side) != cudaSuccess) return G2Q_ERR_CUDA;
  }
  if (cudaStreamWaitEvent(st, ev[2 * (nblk - 1) + 1], 0) != cudaSuccess) return G2Q_ERR_CUDA;
  extract_u_kernel<<<blocks, 256, 0, st>>>(Y, C, U, info);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

}  // namespace g2q

extern "C" size_t g2q_chol_workspace_bytes(int64_t C) {
  const int64_t nblk = (C + g2q::NB - 1) / g2q::NB;
  return (size_t)(2 * C * C + nblk * g2q::NB * g2q::NB + 64) * sizeof(float) +
         (size_t)6 * g2q::NB * C * sizeof(__half) + (size_t)3 * C * sizeof(float) + 256;
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
