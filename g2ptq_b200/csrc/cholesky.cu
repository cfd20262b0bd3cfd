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
// The inverse chain (X_k, Y update), which no later panel depends on, runs on a
// library-owned side stream ordered by per-step events and joined at the end.
// On tensor cores the panels and the update of the next panel's column block
// run ahead on a high-priority stream while the rest of each SYRK runs on the
// caller's stream (look-ahead, see chol_batched).
#include <cuda_fp16.h>

#include "gemm_simt.cuh"

namespace g2q {

constexpr int NB = 128;

// mean(diag(H)) -> *out, one block per batch entry (H + b h_bs -> out[b]).
__global__ void mean_diag_kernel(const float* H, long long C, long long ldh, float* out,
                                 long long h_bs) {
  __shared__ float red[32];
  H += blockIdx.x * h_bs;
  out += blockIdx.x;
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

// Damp percentages of up to kDampSlots batch entries, passed by value.
constexpr int kDampSlots = 64;
struct DampSet {
  float pct[kDampSlots];
};

// A[i][j] = H[C-1-i][C-1-j] (+ damp on the diagonal) for j <= i; Y = I.
// Row i over the grid's y loop, columns over the x threads (no per-element
// division); batch entry z = blockIdx.z at H + z h_bs, A / Y + z a_bs, with
// damp percentage d.pct[z] of mean_diag[z].
__global__ void reverse_damp_kernel(const float* H, long long C, long long ldh,
                                    const float* mean_diag, DampSet d, float* A, float* Y,
                                    long long h_bs, long long a_bs) {
  const int z = blockIdx.z;
  H += z * h_bs;
  A += z * a_bs;
  Y += z * a_bs;
  const float damp = d.pct[z] * mean_diag[z];
  for (long long i = blockIdx.y; i < C; i += gridDim.y) {
    const float* h = H + (C - 1 - i) * ldh + (C - 1);
    for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < C;
         j += (long long)gridDim.x * blockDim.x) {
      float v = 0.f;
      if (j <= i) {
        v = h[-j];
        if (i == j) v += damp;
      }
      A[i * C + j] = v;
      Y[i * C + j] = (i == j) ? 1.f : 0.f;
    }
  }
}

static dim3 grid_rows2(long long rows, long long cols) { return wave_grid_2d(rows, cols); }

// Factor the nb x nb diagonal block at (k0, k0) of A in place and write its
// lower-triangular inverse to Linv (NB x NB, zero padded).
//
// One CTA of 256 threads; the block A_kk and the inverse accumulator live in
// shared memory (rows past nb padded with the identity, which factors to
// itself and does not touch the real rows).  Blocked right-looking
// factorization in four 32-column sub-panels s:
//   (a) warp 0 factors the 32 x 32 diagonal sub-block, one row per lane:
//       every lane takes the pivot's sqrt and reciprocal, scales its element
//       of the pivot column by 1/l_jj (as LAPACK's spotf2) and applies the
//       rank-1 update to the rest of its row;
//   (b) forward substitution with that sub-block, one row (or column) per
//       lane: the rows under it become L_is, and block row s of the inverse
//       accumulator Y becomes X_s: = L_ss^-1 Y_s: (L X = I by blocks);
//   (c) rank-32 updates of the trailing lower part, A_ij -= L_is L_js^T, and
//       of the inverse rows below, Y_i: -= L_is X_s:, in 4 x 4 thread tiles.
// Look-ahead: the next diagonal sub-block is updated first, so that warp 0
// factors it while the other seven warps finish the rest of (c).  The pivot
// chain (sqrt, reciprocal, one shared-memory round trip and one fma per
// pivot) is the latency that bounds the kernel.
constexpr int PSUB = 32;          // sub-panel width
constexpr int PLD = NB + 4;       // shared row stride of the block and of Y / X
constexpr int PANEL_THREADS = 256;

__host__ __device__ constexpr int panel_smem_floats() {
  return 2 * NB * PLD + PSUB * PLD + 2 * PSUB * (PSUB + 1) + PSUB + 4;
}

// (a): factor the sub-block at (c0, c0) of As in place (warp 0).  Lane i holds
// row i in registers, shifted four columns after every four pivots, so that
// the pivot loop is a short runtime loop over groups of four (straight-line
// code for all 32 pivots runs once per sub-block and stalls on instruction
// fetch).  The chain from one pivot to the next is a shuffle, sqrt,
// reciprocal, one multiply and one fma (the diagonal element is kept apart);
// the column of l_kj reaches the other rows through shared memory off that
// chain.  Entries of a row at or right of its diagonal are updated too and
// never read (Lc has zero rows past the block, so the reads stay in bounds).
// Lc[k][j] receives l_kj, rls[j] = 1 / l_jj.  A non-positive or NaN pivot sets
// *flag to its 1-based index in A.
__device__ __forceinline__ void panel_factor_sub(float* As, int c0, float* Lc, float* rls,
                                                 volatile int* flag, long long k0, int lane) {
  constexpr int LC = PSUB + 1;
  float d[PSUB];
  const float* row = As + (c0 + lane) * PLD + c0;
#pragma unroll
  for (int m4 = 0; m4 < PSUB; m4 += 4) {
    const float4 v = *reinterpret_cast<const float4*>(row + m4);
    d[m4] = v.x; d[m4 + 1] = v.y; d[m4 + 2] = v.z; d[m4 + 3] = v.w;
  }
  float diag = row[lane];
  bool ok = true;
#pragma unroll 1
  for (int jb = 0; jb < PSUB && ok; jb += 4) {
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = jb + jj;
      const float piv = __shfl_sync(0xffffffffu, diag, j);
      if (!(piv > 0.f)) {  // uniform: every lane holds the same pivot
        if (lane == 0) *flag = (int)(k0 + c0 + j + 1);
        ok = false;
        break;
      }
      const float l = sqrtf(piv);
      const float rl = 1.f / l;
      float lij = 0.f;
      if (lane == j) {
        Lc[j * LC + j] = l;
        rls[j] = rl;
      } else if (lane > j) {
        lij = d[jj] * rl;
        diag = fmaf(-lij, lij, diag);
        Lc[lane * LC + j] = lij;
      }
      __syncwarp();
      // a_ik -= l_ij l_kj for k > j; d[kk] holds column jb + kk
      const float* lcol = Lc + j * (LC + 1);  // lcol[q * LC] = Lc[j + q][j]
#pragma unroll
      for (int kk = jj + 1; kk < PSUB; ++kk) d[kk] = fmaf(-lij, lcol[(kk - jj) * LC], d[kk]);
    }
#pragma unroll
    for (int kk = 0; kk < PSUB - 4; ++kk) d[kk] = d[kk + 4];
  }
  __syncwarp();
  if (ok) {
#pragma unroll 4
    for (int k = 0; k < PSUB; ++k)
      As[(c0 + k) * PLD + c0 + lane] = (lane <= k) ? Lc[k * LC + lane] : 0.f;
  }
  __syncwarp();
}

// Forward substitution with the factored sub-block, one vector per lane:
// x <- L_ss^-1 x, where x[m] = v[m * stride] (shared memory, in place).  The
// vector is held in registers shifted four entries after every four steps
// (runtime loop, compact code); entries past the block are updated from the
// zero rows of Lc and never read.
__device__ __forceinline__ void panel_forward_sub(float* v, int stride, const float* Lc,
                                                  const float* rls, float* lt_col) {
  constexpr int LC = PSUB + 1;
  float x[PSUB];
#pragma unroll
  for (int m = 0; m < PSUB; ++m) x[m] = v[m * stride];
#pragma unroll 1
  for (int mb = 0; mb < PSUB; mb += 4) {
#pragma unroll
    for (int mm = 0; mm < 4; ++mm) {
      const int m = mb + mm;
      const float xm = x[mm] * rls[m];
      v[m * stride] = xm;
      if (lt_col) lt_col[m * PLD] = xm;
      const float* lcol = Lc + m * (LC + 1);  // lcol[q * LC] = Lc[m + q][m]
#pragma unroll
      for (int kk = mm + 1; kk < PSUB; ++kk) x[kk] = fmaf(-xm, lcol[(kk - mm) * LC], x[kk]);
    }
#pragma unroll
    for (int kk = 0; kk < PSUB - 4; ++kk) x[kk] = x[kk + 4];
  }
}

// 4 x 4 tile of D[i0.., j0..] -= sum_m P[m][i0..] Q[m][j0..] over 32 m, where
// P rows are Lt (the transposed strip) and Q rows are Lt or rows of X.
__device__ __forceinline__ void panel_tile_update(float* D, int i0, int j0, const float* P,
                                                  const float* Q, long long ldq, bool lower_only) {
  float acc[4][4];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 4; ++v) acc[u][v] = 0.f;
#pragma unroll 8
  for (int m = 0; m < PSUB; ++m) {
    const float4 p = *reinterpret_cast<const float4*>(P + m * PLD + i0);
    const float4 q = *reinterpret_cast<const float4*>(Q + m * ldq + j0);
    const float pv[4] = {p.x, p.y, p.z, p.w};
    const float qv[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(pv[u], qv[v], acc[u][v]);
  }
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 4; ++v)
      if (!lower_only || j0 + v <= i0 + u) D[(i0 + u) * PLD + j0 + v] -= acc[u][v];
}

__global__ void __launch_bounds__(PANEL_THREADS, 1)
    panel_kernel(float* A, long long C, long long k0, int nb, float* Linv, int* info,
                 long long a_bs, long long linv_bs) {
  extern __shared__ __align__(16) float psm[];
  // batch entry blockIdx.x: its matrix, its diagonal inverses and its info word
  A += blockIdx.x * a_bs;
  Linv += blockIdx.x * linv_bs;
  if (info) info += blockIdx.x;
  float* As = psm;                  // [NB][PLD] block, lower part
  float* Ys = As + NB * PLD;        // [NB][PLD] inverse accumulator Y -> X
  float* Lt = Ys + NB * PLD;        // [PSUB][PLD] strip L_is transposed: Lt[m][i]
  float* Lc = Lt + PSUB * PLD;      // [2 PSUB][PSUB + 1] factored diagonal sub-block + zero rows
  float* rls = Lc + 2 * PSUB * (PSUB + 1);
  volatile int* flag = reinterpret_cast<volatile int*>(rls + PSUB);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int nsub = (nb + PSUB - 1) / PSUB;
  const int rend = nsub * PSUB;     // rows / columns past rend are never touched

  {
    // thread t reads column t % 128 of 64 rows, sixteen loads in flight at a time
    const int c = t & (NB - 1), rb = (t >> 7) * (NB / 2);
#pragma unroll 1
    for (int i0 = 0; i0 < NB / 2; i0 += 16) {
      float v[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int r = rb + i0 + u;
        v[u] = (r < nb && c <= r) ? A[(k0 + r) * C + k0 + c] : (r == c ? 1.f : 0.f);
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int r = rb + i0 + u;
        As[r * PLD + c] = v[u];
        Ys[r * PLD + c] = (r == c) ? 1.f : 0.f;
      }
    }
  }
  for (int idx = t; idx < 2 * PSUB * (PSUB + 1); idx += PANEL_THREADS) Lc[idx] = 0.f;
  if (t == 0) *flag = 0;
  __syncthreads();
  if (warp == 0) panel_factor_sub(As, 0, Lc, rls, flag, k0, lane);
  __syncthreads();

  for (int s = 0; s < nsub; ++s) {
    if (*flag) break;  // uniform: read after a barrier
    const int c0 = s * PSUB;
    // ---- (b) rows under the sub-block: L_is; block row s of Y -> X_s:
    if (warp < 3) {
      const int r = c0 + PSUB + warp * 32 + lane;
      if (r < rend) panel_forward_sub(As + r * PLD + c0, 1, Lc, rls, Lt + r);
    } else if (warp < 7) {
      const int j = (warp - 3) * 32 + lane;
      if (j < c0 + PSUB) panel_forward_sub(Ys + c0 * PLD + j, PLD, Lc, rls, nullptr);
    }
    __syncthreads();
    if (s + 1 >= nsub) break;
    // ---- (c) look-ahead: the next diagonal sub-block first (36 lower 4 x 4 tiles)
    const int n0 = c0 + PSUB;
    if (t < 36) {
      int ti = 0, tt = t;
      while (tt > ti) { tt -= ti + 1; ++ti; }
      panel_tile_update(As, n0 + 4 * ti, n0 + 4 * tt, Lt, Lt, PLD, ti == tt);
    }
    __syncthreads();
    if (warp == 0) {
      panel_factor_sub(As, n0, Lc, rls, flag, k0, lane);
    } else {
      // rest of the trailing lower part (rows from n0 + 32) and the Y rows below s
      const int rows_t = (rend - n0 - PSUB) / 4;        // tile rows under the next sub-block
      const int cols_y = (c0 + PSUB) / 4;               // tile columns of X_s:
      const int rows_y = (rend - n0) / 4;
      // trailing tiles: tile row a (rows n0 + 32 + 4a) has columns n0 .. its diagonal
      const int n_sy = rows_t * 8 + rows_t * (rows_t + 1) / 2;
      const int n_tot = n_sy + rows_y * cols_y;
      for (int id = t - 32; id < n_tot; id += PANEL_THREADS - 32) {
        if (id < n_sy) {
          // walk tile rows: row a holds 8 + a + 1 tiles
          int a = 0, rem = id;
          while (rem >= 9 + a) { rem -= 9 + a; ++a; }
          const int i0 = n0 + PSUB + 4 * a, j0 = n0 + 4 * rem;
          panel_tile_update(As, i0, j0, Lt, Lt, PLD, j0 == i0);
        } else {
          const int q = id - n_sy;
          const int i0 = n0 + 4 * (q / cols_y), j0 = 4 * (q % cols_y);
          panel_tile_update(Ys, i0, j0, Lt, Ys + c0 * PLD, PLD, false);
        }
      }
    }
    __syncthreads();
  }
  __syncthreads();
  if (*flag) {
    if (t == 0 && info) atomicCAS(info, 0, *flag);
    // mark the inverse as NaN so downstream products are visibly invalid
    for (int idx = t; idx < NB * NB; idx += PANEL_THREADS) Linv[idx] = __int_as_float(0x7fc00000);
    return;
  }
  for (int idx = t; idx < NB * NB; idx += PANEL_THREADS) {
    const int r = idx / NB, c = idx % NB;
    Linv[idx] = (r < nb && c < nb) ? Ys[r * PLD + c] : 0.f;
    if (r < nb && c <= r) A[(k0 + r) * C + k0 + c] = As[r * PLD + c];
  }
}

// Products of a 128-wide strip with the panel's lower-triangular inverse Linv
// (NB x NB, zero past nb), in place:
//   RIGHT  S [n x nb] <- S Linv^T   (L_ik = A_ik Linv_kk^T, 64 rows per CTA)
//   LEFT   S [nb x n] <- Linv S     (X_k: = Linv_kk Y_k:,   64 columns per CTA)
// Each CTA stages Linv^T and its part of the strip (k-major) in shared memory
// with all loads in flight, then every thread accumulates a 4 x 8 output tile
// over the nonzero part of Linv from three 16-byte shared loads per k.  K is
// only 128, so a k-tiled GEMM spends its time waiting on one small tile after
// another.
constexpr int LA_ROWS = 64;        // strip rows (RIGHT) or columns (LEFT) per CTA
constexpr int LA_LDT = NB + 4;     // Lt[k][c] = Linv[c][k]
constexpr int LA_LDB = LA_ROWS + 4;  // Bt[k][i]: strip entry i, index k
constexpr int LA_LDO = NB + 1;     // Os[i][c]: results

__host__ __device__ constexpr int linv_apply_smem_floats() {
  return NB * LA_LDT + NB * LA_LDB;
}

template <bool LEFT>
__global__ void __launch_bounds__(256) linv_apply_kernel(float* S, long long lds, long long n,
                                                         const float* __restrict__ Linv, int nb,
                                                         long long s_bs, long long linv_bs) {
  extern __shared__ __align__(16) float lsm[];
  S += blockIdx.z * s_bs;
  Linv += blockIdx.z * linv_bs;
  float* Lt = lsm;                 // [NB][LA_LDT]
  float* Bt = lsm + NB * LA_LDT;   // [NB][LA_LDB]
  float* Os = Bt;                  // [LA_ROWS][LA_LDO], reuses Bt after the products
  const int t = threadIdx.x;
  const long long i0 = (long long)blockIdx.x * LA_ROWS;
  // all loads of a thread in flight before its shared-memory stores: a loop
  // that stores each value before the next load waits for L2 sixty-four times
#pragma unroll 1
  for (int i0l = 0; i0l < NB * NB; i0l += 16 * 256) {
    float v[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) v[u] = Linv[i0l + u * 256 + t];
#pragma unroll
    for (int u = 0; u < 16; ++u) {
      const int idx = i0l + u * 256 + t, c = idx / NB, k = idx % NB;
      Lt[k * LA_LDT + c] = v[u];
    }
  }
  {
    float v[LA_ROWS * NB / 256];
    if (!LEFT) {
      // rows i0 .. i0+63, columns 0 .. nb-1 (consecutive threads: consecutive columns)
#pragma unroll
      for (int u = 0; u < LA_ROWS * NB / 256; ++u) {
        const int idx = u * 256 + t, i = idx / NB, k = idx % NB;
        const long long r = i0 + i;
        v[u] = (r < n && k < nb) ? S[r * lds + k] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < LA_ROWS * NB / 256; ++u) {
        const int idx = u * 256 + t, i = idx / NB, k = idx % NB;
        Bt[k * LA_LDB + i] = v[u];
      }
    } else {
      // rows 0 .. nb-1, columns i0 .. i0+63 (consecutive threads: consecutive columns)
#pragma unroll
      for (int u = 0; u < LA_ROWS * NB / 256; ++u) {
        const int idx = u * 256 + t, k = idx / LA_ROWS, i = idx % LA_ROWS;
        const long long c = i0 + i;
        v[u] = (c < n && k < nb) ? S[k * lds + c] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < LA_ROWS * NB / 256; ++u) {
        const int idx = u * 256 + t, k = idx / LA_ROWS, i = idx % LA_ROWS;
        Bt[k * LA_LDB + i] = v[u];
      }
    }
  }
  __syncthreads();
  // o[i][c] = sum_{k <= c} Bt[k][i] Lt[k][c] for the thread's 4 strip entries i
  // and 8 Linv rows c (output columns for RIGHT, output rows for LEFT)
  const int ti = t & 15, tc = t >> 4;
  const int ib = ti * 4, cb = tc * 8;
  float acc[4][8];
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 8; ++v) acc[u][v] = 0.f;
  const int kend = cb + 8 < nb ? cb + 8 : nb;
#pragma unroll 4
  for (int k = 0; k < kend; ++k) {
    const float4 a4 = *reinterpret_cast<const float4*>(Bt + k * LA_LDB + ib);
    const float4 b0 = *reinterpret_cast<const float4*>(Lt + k * LA_LDT + cb);
    const float4 b1 = *reinterpret_cast<const float4*>(Lt + k * LA_LDT + cb + 4);
    const float a[4] = {a4.x, a4.y, a4.z, a4.w};
    const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int v = 0; v < 8; ++v) acc[u][v] = fmaf(a[u], b[v], acc[u][v]);
  }
  __syncthreads();
#pragma unroll
  for (int u = 0; u < 4; ++u)
#pragma unroll
    for (int v = 0; v < 8; ++v) Os[(ib + u) * LA_LDO + cb + v] = acc[u][v];
  __syncthreads();
  if (!LEFT) {
    for (int idx = t; idx < LA_ROWS * NB; idx += 256) {
      const int i = idx / NB, k = idx % NB;
      const long long r = i0 + i;
      if (r < n && k < nb) S[r * lds + k] = Os[i * LA_LDO + k];
    }
  } else {
    for (int idx = t; idx < LA_ROWS * NB; idx += 256) {
      const int k = idx / LA_ROWS, i = idx % LA_ROWS;
      const long long c = i0 + i;
      if (c < n && k < nb) S[k * lds + c] = Os[i * LA_LDO + k];
    }
  }
}

template <bool LEFT>
static int linv_apply(float* S, long long lds, long long n, const float* Linv, int nb,
                      cudaStream_t st, long long batch = 1, long long s_bs = 0,
                      long long linv_bs = 0) {
  if (n <= 0 || batch <= 0) return G2Q_OK;
  static int done[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return G2Q_ERR_CUDA;
  const size_t smem = linv_apply_smem_floats() * sizeof(float);
  if (dev >= 64 || !done[dev]) {
    if (cudaFuncSetAttribute(linv_apply_kernel<LEFT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
      return G2Q_ERR_CUDA;
    if (dev < 64) done[dev] = 1;
  }
  linv_apply_kernel<LEFT><<<dim3((unsigned)cdiv(n, LA_ROWS), 1, (unsigned)batch), 256, smem,
                            st>>>(S, lds, n, Linv, nb, s_bs, linv_bs);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

// U[i][j] = X[C-1-i][C-1-j] for i <= j, 0 below; NaN -> info = -1.  Batch
// entry z = blockIdx.z at X + z x_bs, U + z u_bs, info + z.
__global__ void extract_u_kernel(const float* X, long long C, float* U, int* info,
                                 long long x_bs, long long u_bs) {
  X += blockIdx.z * x_bs;
  U += blockIdx.z * u_bs;
  if (info) info += blockIdx.z;
  bool nan_seen = false;
  for (long long i = blockIdx.y; i < C; i += gridDim.y) {
    const float* x = X + (C - 1 - i) * C + (C - 1);
    for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < C;
         j += (long long)gridDim.x * blockDim.x) {
      float v = 0.f;
      if (i <= j) {
        v = x[-j];
        if (v != v) nan_seen = true;
      }
      U[i * C + j] = v;
    }
  }
  if (nan_seen && info) atomicCAS(info, 0, -1);
}



int tc_update2h(float* D, long long ldd, long long M, long long N, long long K,
                __half* const* a2, const float* sa, long long lda, __half* const* b2,
                const float* sb, long long ldb, int lower, float alpha, float beta,
                int* status, cudaStream_t st, long long batch = 1, long long k_bs = 0,
                long long d_bs = 0, long long sa_bs = 0, long long sb_bs = 0);
int split2h_strips(const float* src, long long lds, long long n, int K, __half* hi, __half* lo,
                   long long ldd, float* scale, int transpose, int ny, long long src_by,
                   long long dst_by, long long sc_by, int nz, long long src_bz,
                   long long dst_bz, long long sc_bz, cudaStream_t st);

// Side stream and per-step events of the inverse chain, one set per (device,
// caller stream) so that factorizations issued on different streams overlap.
struct SideState {
  int dev = -1;
  cudaStream_t main = nullptr;
  cudaStream_t side = nullptr;
  cudaStream_t crit = nullptr;  // the factorization's critical path, highest priority
  cudaEvent_t* ev = nullptr;    // [4 * cap + 1]: per step four, then one fork event
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
    // the inverse chain runs at the caller's stream priority, the panels and
    // their look-ahead updates at the device's highest, so that their single
    // CTAs take the first SM a trailing update frees
    int prio = 0, least = 0, greatest = 0;
    if (!s->side && (cudaStreamGetPriority(main, &prio) != cudaSuccess ||
                     cudaStreamCreateWithPriority(&s->side, cudaStreamNonBlocking, prio) !=
                         cudaSuccess))
      return G2Q_ERR_CUDA;
    if (!s->crit &&
        (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess ||
         cudaStreamCreateWithPriority(&s->crit, cudaStreamNonBlocking, greatest) != cudaSuccess))
      return G2Q_ERR_CUDA;
    s->dev = dev;
    s->main = main;
  }
  if (s->cap < steps + 1) {
    cudaEvent_t* ev = new cudaEvent_t[4 * (steps + 1) + 1];
    for (int i = 0; i < 4 * (steps + 1) + 1; ++i)
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

// Workspace of the CUDA-core chain (floats): A [C*C], Y [C*C], diagonal
// inverses [nblk][NB*NB], mean diag [64].
struct CholWs {
  float *A, *Y, *linv, *mdiag;
};

static CholWs carve(float* ws, long long C) {
  CholWs w;
  const long long nblk = (C + NB - 1) / NB;
  w.A = ws;
  w.Y = w.A + C * C;
  w.linv = w.Y + C * C;
  w.mdiag = w.linv + nblk * NB * NB;
  return w;
}

static int panel_attr() {
  static int done[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return G2Q_ERR_CUDA;
  if (dev < 64 && done[dev]) return G2Q_OK;
  if (cudaFuncSetAttribute(panel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)(panel_smem_floats() * sizeof(float))) != cudaSuccess)
    return G2Q_ERR_CUDA;
  if (dev < 64) done[dev] = 1;
  return G2Q_OK;
}

// One factorization on fp32 CUDA cores (precision 0, or C not a multiple of 8),
// 128-column steps: the factorization on the caller's stream, the inverse
// chain on the side stream.
static int chol_one(float* U, const float* H, long long C, long long ldh, float damp_percent,
                    int* info, float* ws, cudaStream_t st) {
  G2Q_TRY(panel_attr());
  CholWs w = carve(ws, C);
  float* A = w.A;
  float* Y = w.Y;
  const long long nblk = (C + NB - 1) / NB;
  SideState* ss = nullptr;
  G2Q_TRY(side_state(st, (int)nblk, &ss));
  cudaStream_t side = ss->side;
  cudaEvent_t* ev = ss->ev;  // ev[2k]: factor step k done, ev[2k+1]: inverse step k done
  if (info && cudaMemsetAsync(info, 0, sizeof(int), st) != cudaSuccess) return G2Q_ERR_CUDA;
  mean_diag_kernel<<<1, 1024, 0, st>>>(H, C, ldh, w.mdiag, 0);
  G2Q_CHECK_LAUNCH();
  DampSet ds{};
  ds.pct[0] = damp_percent;
  reverse_damp_kernel<<<grid_rows2(C, C), 256, 0, st>>>(H, C, ldh, w.mdiag, ds, A, Y, 0, 0);
  G2Q_CHECK_LAUNCH();
  for (long long kb = 0; kb < nblk; ++kb) {
    const long long k0 = kb * NB;
    const int nb = (int)((C - k0) < NB ? (C - k0) : NB);
    const long long rest = C - k0 - nb;
    float* linv = w.linv + kb * NB * NB;
    // ---- factorization (caller's stream): panel, TRSM, SYRK
    panel_kernel<<<1, PANEL_THREADS, panel_smem_floats() * sizeof(float), st>>>(A, C, k0, nb,
                                                                                linv, info, 0, 0);
    G2Q_CHECK_LAUNCH();
    if (rest > 0) {
      // L_ik = A_ik Linv_kk^T, in place in A
      G2Q_TRY(linv_apply<false>(A + (k0 + nb) * C + k0, C, rest, linv, nb, st));
      G2Q_TRY(simt_gemm_f32(A + (k0 + nb) * C + (k0 + nb), C, A + (k0 + nb) * C + k0, C, false,
                            A + (k0 + nb) * C + k0, C, true, rest, rest, nb, 1.f, -1.f,
                            G2Q_MASK_LOWER, st));
    }
    if (cudaEventRecord(ev[2 * kb], st) != cudaSuccess) return G2Q_ERR_CUDA;
    // ---- inverse chain (side stream): X_k: = Linv_kk Y_k:, then Y_i: -= L_ik X_k:
    if (cudaStreamWaitEvent(side, ev[2 * kb], 0) != cudaSuccess) return G2Q_ERR_CUDA;
    G2Q_TRY(linv_apply<true>(Y + k0 * C, C, k0 + nb, linv, nb, side));
    if (rest > 0)
      G2Q_TRY(simt_gemm_f32(Y + (k0 + nb) * C, C, A + (k0 + nb) * C + k0, C, false, Y + k0 * C,
                            C, false, rest, k0 + nb, nb, 1.f, -1.f, G2Q_MASK_FULL, side));
    if (cudaEventRecord(ev[2 * kb + 1], side) != cudaSuccess) return G2Q_ERR_CUDA;
  }
  if (cudaStreamWaitEvent(st, ev[2 * (nblk - 1) + 1], 0) != cudaSuccess) return G2Q_ERR_CUDA;
  extract_u_kernel<<<grid_rows2(C, C), 256, 0, st>>>(Y, C, U, info, 0, 0);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

// ---------------------------------------------------------------------------
// Tensor-core chain, n factorizations of one size (n = 1 for a single matrix)
// advancing panel by panel together, every launch of a step covering all n
// (grid z, or one panel CTA each): a layer-batched object (n same-shape
// linears or experts) costs one chain of launches instead of n.
//
// Look-ahead over three streams.  The critical path (library stream at the
// device's highest priority): panel k, L_ik = A_ik Linv_k^T, the split of that
// strip, and the update of column block k+1 alone (the next panel's input).
// The bulk of the trailing update (rows and columns past block k+1) runs on
// the caller's stream, so panel k+1 overlaps the bulk update of step k; the
// inverse chain (X_k: = Linv_k Y_k:, Y_i: -= L_ik X_k:) runs on the side stream.
// Every element receives the same K = 128 products in the same order as with
// one update per step (the same 128 x 128 tiles), so the split changes no bit.
//
// Workspace as arrays over the batch, each 256-byte aligned: A [n][C][C],
// Y [n][C][C], diagonal inverses [n][nblk][NB][NB], mean diagonals [n], then
// fp16: L21^T splits [2 buffers][2][n][NB][C], X_k splits [2][n][NB][C], then
// the splits' scales: L21 [2 buffers][n][C], X_k [n][C].
struct CholWsB {
  float *A, *Y, *linv, *mdiag;
  __half *lt, *xk;
  float *lsc, *xsc;
  size_t bytes;
};

constexpr int kCholArrays = 8;

static CholWsB carve_batched(void* base, long long C, long long n) {
  const long long nblk = (C + NB - 1) / NB;
  CholWsB w{};
  char* p = static_cast<char*>(base);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* q = p ? p + off : nullptr;
    off += (bytes + 255) / 256 * 256;
    return q;
  };
  w.A = reinterpret_cast<float*>(take((size_t)n * C * C * sizeof(float)));
  w.Y = reinterpret_cast<float*>(take((size_t)n * C * C * sizeof(float)));
  w.linv = reinterpret_cast<float*>(take((size_t)n * nblk * NB * NB * sizeof(float)));
  w.mdiag = reinterpret_cast<float*>(take((size_t)n * sizeof(float)));
  w.lt = reinterpret_cast<__half*>(take((size_t)4 * n * NB * C * sizeof(__half)));
  w.xk = reinterpret_cast<__half*>(take((size_t)2 * n * NB * C * sizeof(__half)));
  w.lsc = reinterpret_cast<float*>(take((size_t)2 * n * C * sizeof(float)));
  w.xsc = reinterpret_cast<float*>(take((size_t)n * C * sizeof(float)));
  w.bytes = off;
  return w;
}

// the elementwise grid of one C x C matrix, its y extent shared out over n
static dim3 batch_grid(long long C, long long n) {
  dim3 g = grid_rows2(C, C);
  long long gy = (long long)g.y / n;
  g.y = (unsigned)(gy < 1 ? 1 : gy);
  g.z = (unsigned)n;
  return g;
}

static int chol_batched(float* U, const float* H, long long C, long long ldh, long long n,
                        const float* damp_percent, int* info, void* ws, cudaStream_t st) {
  G2Q_TRY(panel_attr());
  const CholWsB w = carve_batched(ws, C, n);
  const long long nblk = (C + NB - 1) / NB;
  const long long CC = C * C, lbs = nblk * NB * NB;  // batch strides of A / Y / U, Linv
  const long long tsz = n * NB * C;                   // one fp16 term of a strip set
  SideState* ss = nullptr;
  G2Q_TRY(side_state(st, (int)nblk, &ss));
  cudaStream_t side = ss->side, crit = ss->crit;
  // per step k: [4k] strip (or, for the last panel, its inverse) ready, [4k+1]
  // bulk update done, [4k+2] inverse step done, [4k+3] critical step done
  cudaEvent_t* ev = ss->ev;
  auto E = [&](long long k, int which) { return ev[4 * k + which]; };
  cudaEvent_t fork = ev[4 * ss->cap];
  if (info && cudaMemsetAsync(info, 0, n * sizeof(int), st) != cudaSuccess) return G2Q_ERR_CUDA;
  mean_diag_kernel<<<(unsigned)n, 1024, 0, st>>>(H, C, ldh, w.mdiag, C * ldh);
  G2Q_CHECK_LAUNCH();
  for (long long z0 = 0; z0 < n; z0 += kDampSlots) {
    const long long m = n - z0 < kDampSlots ? n - z0 : kDampSlots;
    DampSet ds{};
    for (long long z = 0; z < m; ++z) ds.pct[z] = damp_percent[z0 + z];
    reverse_damp_kernel<<<batch_grid(C, m), 256, 0, st>>>(H + z0 * C * ldh, C, ldh,
                                                          w.mdiag + z0, ds, w.A + z0 * CC,
                                                          w.Y + z0 * CC, C * ldh, CC);
    G2Q_CHECK_LAUNCH();
  }
  if (cudaEventRecord(fork, st) != cudaSuccess || cudaStreamWaitEvent(crit, fork, 0) != cudaSuccess)
    return G2Q_ERR_CUDA;
  const size_t psmem = panel_smem_floats() * sizeof(float);
  for (long long kb = 0; kb < nblk; ++kb) {
    const long long k0 = kb * NB;
    const int nb = (int)((C - k0) < NB ? (C - k0) : NB);
    const long long rest = C - k0 - nb;                 // rows past panel kb
    const long long nbn = rest < NB ? rest : NB;        // width of column block kb + 1
    const long long rest2 = rest - nbn;                 // rows past column block kb + 1
    float* linv = w.linv + kb * NB * NB;
    __half* lt = w.lt + (kb & 1) * 2 * tsz;
    __half* l2[2] = {lt, lt + tsz};
    float* lsc = w.lsc + (kb & 1) * n * C;
    __half* x2[2] = {w.xk, w.xk + tsz};
    // ---- critical path
    // column block kb took its last update from the bulk update of step kb - 2
    // (and from the look-ahead update of step kb - 1, earlier on this stream)
    if (kb >= 2 && cudaStreamWaitEvent(crit, E(kb - 2, 1), 0) != cudaSuccess)
      return G2Q_ERR_CUDA;
    panel_kernel<<<(unsigned)n, PANEL_THREADS, psmem, crit>>>(w.A, C, k0, nb, linv, info, CC,
                                                              lbs);
    G2Q_CHECK_LAUNCH();
    if (rest > 0) {
      G2Q_TRY(linv_apply<false>(w.A + (k0 + nb) * C + k0, C, rest, linv, nb, crit, n, CC, lbs));
      // the inverse step kb - 2 read this strip buffer (the bulk update kb - 2
      // did too: waited for above)
      if (kb >= 2 && cudaStreamWaitEvent(crit, E(kb - 2, 2), 0) != cudaSuccess)
        return G2Q_ERR_CUDA;
      G2Q_TRY(split2h_strips(w.A + (k0 + nb) * C + k0, C, rest, nb, l2[0], l2[1], C, lsc, 1, 1,
                             0, 0, 0, (int)n, CC, (long long)NB * C, C, crit));
    }
    if (cudaEventRecord(E(kb, 0), crit) != cudaSuccess) return G2Q_ERR_CUDA;
    if (rest > 0) {
      // column block kb + 1 next: the bulk update of step kb - 1 adds into it too
      if (kb >= 1 && cudaStreamWaitEvent(crit, E(kb - 1, 1), 0) != cudaSuccess)
        return G2Q_ERR_CUDA;
      G2Q_TRY(tc_update2h(w.A + (k0 + nb) * C + (k0 + nb), C, rest, nbn, nb, l2, lsc, C, l2, lsc,
                          C, 1, 1.f, -1.f, info, crit, n, NB, CC, C, C));
    }
    if (cudaEventRecord(E(kb, 3), crit) != cudaSuccess) return G2Q_ERR_CUDA;
    // ---- bulk trailing update (caller's stream): rows and columns past block kb + 1
    if (rest2 > 0) {
      if (cudaStreamWaitEvent(st, E(kb, 0), 0) != cudaSuccess) return G2Q_ERR_CUDA;
      const long long r2 = k0 + nb + nbn;
      __half* b2[2] = {l2[0] + nbn, l2[1] + nbn};  // the strip from row r2 on
      G2Q_TRY(tc_update2h(w.A + r2 * C + r2, C, rest2, rest2, nb, b2, lsc + nbn, C, b2,
                          lsc + nbn, C, 1, 1.f, -1.f, info, st, n, NB, CC, C, C));
    }
    if (cudaEventRecord(E(kb, 1), st) != cudaSuccess) return G2Q_ERR_CUDA;
    // ---- inverse chain (side stream)
    if (cudaStreamWaitEvent(side, E(kb, 0), 0) != cudaSuccess) return G2Q_ERR_CUDA;
    G2Q_TRY(linv_apply<true>(w.Y + k0 * C, C, k0 + nb, linv, nb, side, n, CC, lbs));
    if (rest > 0) {
      G2Q_TRY(split2h_strips(w.Y + k0 * C, C, k0 + nb, nb, x2[0], x2[1], C, w.xsc, 0, 1, 0, 0, 0,
                             (int)n, CC, (long long)NB * C, C, side));
      G2Q_TRY(tc_update2h(w.Y + (k0 + nb) * C, C, rest, k0 + nb, nb, l2, lsc, C, x2, w.xsc, C, 0,
                          1.f, -1.f, info, side, n, NB, CC, C, C));
    }
    if (cudaEventRecord(E(kb, 2), side) != cudaSuccess) return G2Q_ERR_CUDA;
  }
  if (cudaStreamWaitEvent(st, E(nblk - 1, 2), 0) != cudaSuccess ||
      cudaStreamWaitEvent(st, E(nblk - 1, 3), 0) != cudaSuccess)
    return G2Q_ERR_CUDA;
  extract_u_kernel<<<batch_grid(C, n), 256, 0, st>>>(w.Y, C, U, info, CC, CC);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

}  // namespace g2q

extern "C" size_t g2q_chol_workspace_bytes(int64_t C) {
  if (C <= 0) return 0;
  // one factorization of the tensor-core chain plus the alignment slack its
  // arrays may take in a chain of several (k chains: k times this); covers the
  // CUDA-core chain's layout too
  const size_t b = g2q::carve_batched(nullptr, C, 1).bytes + g2q::kCholArrays * 256;
  return (b + 255) / 256 * 256;  // a multiple of 256: concurrent lanes take aligned slices
}

namespace g2q {
// Up to CHOL_LANES factorizations of one call run side by side, each on a
// library-owned stream forked from and joined back to the caller's stream
// (same priority) with its own slice of the workspace: a chain is a few
// hundred dependent, mostly latency-bound launches, so concurrent chains fill
// the GPU that one chain leaves idle.
constexpr int CHOL_LANES = 4;

struct LaneSet {
  int dev = -1;
  cudaStream_t caller = nullptr;
  cudaStream_t s[CHOL_LANES] = {};
  cudaEvent_t fork = nullptr;
  cudaEvent_t join[CHOL_LANES] = {};
};

static int lane_set(cudaStream_t caller, LaneSet** out) {
  constexpr int kSets = 32;
  static LaneSet sets[kSets];
  static int next = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return G2Q_ERR_CUDA;
  for (int i = 0; i < kSets; ++i)
    if (sets[i].fork && sets[i].dev == dev && sets[i].caller == caller) {
      *out = &sets[i];
      return G2Q_OK;
    }
  LaneSet* ls = &sets[next];
  next = (next + 1) % kSets;
  int prio = 0;
  if (cudaStreamGetPriority(caller, &prio) != cudaSuccess) return G2Q_ERR_CUDA;
  if (!ls->fork || ls->dev != dev) {  // (a reused slot keeps its streams on the same device)
    *ls = LaneSet();
    for (int i = 0; i < CHOL_LANES; ++i) {
      if (cudaStreamCreateWithPriority(&ls->s[i], cudaStreamNonBlocking, prio) != cudaSuccess ||
          cudaEventCreateWithFlags(&ls->join[i], cudaEventDisableTiming) != cudaSuccess)
        return G2Q_ERR_CUDA;
    }
    if (cudaEventCreateWithFlags(&ls->fork, cudaEventDisableTiming) != cudaSuccess)
      return G2Q_ERR_CUDA;
  }
  ls->dev = dev;
  ls->caller = caller;
  *out = ls;
  return G2Q_OK;
}
}  // namespace g2q

extern "C" int g2q_chol_upper_inverse(float* U, const float* H, int64_t C, int64_t ldh,
                                      int64_t batch, const float* damp_percent_host, int* info,
                                      int precision, void* workspace, size_t workspace_bytes,
                                      void* stream) {
  if (!U || !H || C <= 0 || ldh < C || batch < 0 || !damp_percent_host || !workspace)
    return G2Q_ERR_INVALID_ARG;
  const size_t per = g2q_chol_workspace_bytes(C);
  if (workspace_bytes < per) return G2Q_ERR_INVALID_ARG;
  if (precision != 0 && precision != 1) return G2Q_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (precision == 1 && g2q::tc_ok(C)) {
    // tensor-core chains of as many factorizations as the workspace holds
    long long n = (long long)(workspace_bytes / per);
    if (n > batch) n = batch;
    if (n > 65535) n = 65535;
    while (n >= 2 && g2q::carve_batched(nullptr, C, n).bytes > workspace_bytes) --n;
    for (int64_t b = 0; b < batch; b += n) {
      const long long m = batch - b < n ? batch - b : n;
      G2Q_TRY(g2q::chol_batched(U + b * C * C, H + b * C * ldh, C, ldh, m, damp_percent_host + b,
                                info ? info + b : nullptr, workspace, st));
    }
    return G2Q_OK;
  }
  long long lanes = (long long)(workspace_bytes / per);
  if (lanes > g2q::CHOL_LANES) lanes = g2q::CHOL_LANES;
  if (lanes > batch) lanes = batch;
  if (lanes <= 1) {
    for (int64_t b = 0; b < batch; ++b)
      G2Q_TRY(g2q::chol_one(U + b * C * C, H + b * C * ldh, C, ldh, damp_percent_host[b],
                            info ? info + b : nullptr, (float*)workspace, st));
    return G2Q_OK;
  }
  g2q::LaneSet* ls = nullptr;
  G2Q_TRY(g2q::lane_set(st, &ls));
  if (cudaEventRecord(ls->fork, st) != cudaSuccess) return G2Q_ERR_CUDA;
  for (long long l = 0; l < lanes; ++l)
    if (cudaStreamWaitEvent(ls->s[l], ls->fork, 0) != cudaSuccess) return G2Q_ERR_CUDA;
  int status = G2Q_OK;
  for (int64_t b = 0; b < batch && status == G2Q_OK; ++b) {
    const long long l = b % lanes;
    float* ws = (float*)((char*)workspace + l * per);
    status = g2q::chol_one(U + b * C * C, H + b * C * ldh, C, ldh, damp_percent_host[b],
                           info ? info + b : nullptr, ws, ls->s[l]);
  }
  // join every lane, also after an error, so that no lane's work outlives the call's stream
  for (long long l = 0; l < lanes; ++l) {
    if (cudaEventRecord(ls->join[l], ls->s[l]) != cudaSuccess ||
        cudaStreamWaitEvent(st, ls->join[l], 0) != cudaSuccess)
      return G2Q_ERR_CUDA;
  }
  return status;
}
