// Staging, Gram dispatch, permutations, Hessian preparation, export packing
// and the G2PTQ trust region.
#include <cuda_fp16.h>

#include <type_traits>

#include "gemm_simt.cuh"

namespace g2q {

int tc_gram_grouped(float* D, long long ldd, long long d_gstride, long long C, const void* X,
                    int x_dtype, long long ldx, const float* s, long long sstride, int G,
                    long long T, float alpha, float beta, void* workspace,
                    size_t workspace_bytes, int* status, cudaStream_t st);
size_t tc_gram_grouped_workspace_bytes(long long C, long long T, int G);
int tc_gram(float* D, long long ldd, long long M, long long N, const void* A, int a_dtype,
            long long lda, const void* B, int b_dtype, long long ldb, const float* row_scale,
            long long scale_stride, long long T, int symmetric, float alpha, float beta,
            void* workspace, size_t workspace_bytes, int* status, cudaStream_t st);
size_t tc_gram_workspace_bytes(long long M, long long N, long long T);

static int grid_for(long long n, int threads = 256) {
  long long b = (n + threads - 1) / threads;
  if (b > 148 * 64) b = 148 * 64;
  if (b < 1) b = 1;
  return (int)b;
}

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename S, typename D>
__global__ void stage_kernel(D* dst, long long dst_ld, long long row0, const S* src,
                             const S* sub, long long src_ld, long long t, long long C) {
  const long long n = t * C;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long r = idx / C, c = idx - r * C;
    float v = to_f<S>(src[r * src_ld + c]);
    if (sub) v -= to_f<S>(sub[r * src_ld + c]);
    if constexpr (sizeof(D) == 2) dst[(row0 + r) * dst_ld + c] = __float2bfloat16_rn(v);
    else dst[(row0 + r) * dst_ld + c] = v;
  }
}

// Strided row copy in 16-byte words (rows of w16 words; pitches in words).
__global__ void copy_rows16_kernel(uint4* __restrict__ dst, long long dst_pitch,
                                   const uint4* __restrict__ src, long long src_pitch,
                                   long long rows, long long w16) {
  const long long n = rows * w16;
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  // four independent words in flight per thread
  for (; idx + 3 * stride < n; idx += 4 * stride) {
    uint4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const long long i = idx + k * stride;
      const long long r = i / w16, c = i - r * w16;
      v[k] = __ldcs(src + r * src_pitch + c);
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const long long i = idx + k * stride;
      const long long r = i / w16, c = i - r * w16;
      dst[r * dst_pitch + c] = v[k];
    }
  }
  for (; idx < n; idx += stride) {
    const long long r = idx / w16, c = idx - r * w16;
    dst[r * dst_pitch + c] = __ldcs(src + r * src_pitch + c);
  }
}

__global__ void scale_vec_kernel(float* acc, long long C, float keep) {
  const long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c < C) acc[c] *= keep;
}

template <typename S>
__global__ void sq_colsum_kernel(float* acc, float scale, const S* X, long long ldx, long long T,
                                 long long C, long long tchunk) {
  const long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const long long t0 = (long long)blockIdx.y * tchunk;
  const long long t1 = (t0 + tchunk < T) ? t0 + tchunk : T;
  float s = 0.f;
  for (long long t = t0; t < t1; ++t) {
    const float v = to_f<S>(X[t * ldx + c]);
    s = fmaf(v, v, s);
  }
  atomicAdd(acc + c, s * scale);
}

// One CTA per layer: RTN fallback for an all-zero Hessian and dead columns.
// The all-zero test reads the diagonal, which is exact for the positive
// semi-definite Gram matrices the accumulation produces (H_cc = 0 forces row
// and column c to zero).
__global__ void prepare_hessian_kernel(float* H, long long C, float* W, long long rows,
                                       float* extra, long long extra_rows, float* gzero) {
  const long long b = blockIdx.x;
  float* Hb = H + b * C * C;
  __shared__ int nonzero;
  if (threadIdx.x == 0) nonzero = 0;
  __syncthreads();
  for (long long c = threadIdx.x; c < C; c += blockDim.x)
    if (Hb[c * C + c] != 0.f) nonzero = 1;
  __syncthreads();
  if (!nonzero) {
    for (long long c = threadIdx.x; c < C; c += blockDim.x) Hb[c * C + c] = 1.f;
    if (gzero) {
      float* g = gzero + b * rows * C;
      for (long long i = threadIdx.x; i < rows * C; i += blockDim.x) g[i] = 0.f;
    }
    return;
  }
  for (long long c = threadIdx.x; c < C; c += blockDim.x) {
    if (Hb[c * C + c] == 0.f) {
      Hb[c * C + c] = 1.f;
      if (W) {
        float* Wb = W + b * rows * C;
        for (long long r = 0; r < rows; ++r) Wb[r * C + c] = 0.f;
      }
      if (extra) {
        float* Eb = extra + b * extra_rows * C;
        for (long long r = 0; r < extra_rows; ++r) Eb[r * C + c] = 0.f;
      }
    }
  }
}

__global__ void argsort_desc_kernel(long long* perm, const float* key, long long n) {
  __shared__ float tile[1024];
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const float ki = i < n ? key[i] : 0.f;
  long long rank = 0;
  for (long long j0 = 0; j0 < n; j0 += 1024) {
    __syncthreads();
    for (int u = threadIdx.x; u < 1024; u += blockDim.x)
      tile[u] = (j0 + u < n) ? key[j0 + u] : -INFINITY;
    __syncthreads();
    const long long jn = (n - j0) < 1024 ? (n - j0) : 1024;
    for (long long u = 0; u < jn; ++u) {
      const float kj = tile[u];
      const long long j = j0 + u;
      rank += (kj > ki) || (kj == ki && j < i);
    }
  }
  if (i < n) perm[rank] = i;
}

__global__ void mean_diag_kernel(float* key, const float* H, long long nl, long long C) {
  const long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float s = 0.f;
  for (long long b = 0; b < nl; ++b) s += H[b * C * C + c * C + c];
  key[c] = s / (float)nl;
}

// Row r of the grid's y loop, columns over the x threads: no 64-bit division
// per element (the flat-index form of these kernels ran at a sixth of HBM
// bandwidth on the division alone).
template <typename T>
__global__ void permute_cols_kernel(T* dst, const T* src, long long rows, long long C,
                                    const long long* perm, int inverse) {
  for (long long r = blockIdx.y; r < rows; r += gridDim.y) {
    const T* s = src + r * C;
    T* d = dst + r * C;
    for (long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x; c < C;
         c += (long long)gridDim.x * blockDim.x) {
      if (inverse) d[perm[c]] = s[c];
      else d[c] = s[perm[c]];
    }
  }
}

// Column permutation of row-major rows through shared memory: each CTA builds
// the gather index of the output columns once (idx[c] = perm[c]; for the
// inverse idx[perm[c]] = c), then per row stages the source row with
// contiguous (16-byte) loads and writes the permuted row with contiguous
// stores, four columns per thread.  The direct kernel above gathers or
// scatters single elements through 8-byte indices (an int8 row moves at a
// fraction of the bandwidth).  C % 16 == 0 and 16-byte aligned rows.
template <typename T>
__global__ void __launch_bounds__(256) permute_cols_staged_kernel(T* dst, const T* src,
                                                                  long long rows, int C,
                                                                  const long long* perm,
                                                                  int inverse) {
  extern __shared__ __align__(16) unsigned char psm_raw[];
  int* idx = reinterpret_cast<int*>(psm_raw);
  T* row = reinterpret_cast<T*>(psm_raw + (size_t)C * sizeof(int));
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const int p = (int)perm[c];
    if (inverse) idx[p] = c;
    else idx[c] = p;
  }
  constexpr int V = 16 / sizeof(T);  // elements per 16-byte load
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    __syncthreads();  // the index is built; the previous row's reads are done
    const uint4* s = reinterpret_cast<const uint4*>(src + r * C);
    uint4* rs = reinterpret_cast<uint4*>(row);
    for (int v = threadIdx.x; v < C / V; v += blockDim.x) rs[v] = s[v];
    __syncthreads();
    T* d = dst + r * C;
    for (int c4 = threadIdx.x * 4; c4 < C; c4 += blockDim.x * 4) {
      T o[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) o[u] = row[idx[c4 + u]];
      if (sizeof(T) == 4) {
        *reinterpret_cast<float4*>(d + c4) = *reinterpret_cast<const float4*>(o);
      } else {
        *reinterpret_cast<uint32_t*>(d + c4) = *reinterpret_cast<const uint32_t*>(o);
      }
    }
  }
}

template <typename T>
static int permute_cols_staged(T* dst, const T* src, long long rows, long long C,
                               const long long* perm, int inverse, cudaStream_t st, bool* done) {
  *done = false;
  const size_t smem = (size_t)C * (sizeof(int) + sizeof(T));
  if (C % 16 || C > 0x7fffffffLL || smem > 200 * 1024 ||
      (reinterpret_cast<uintptr_t>(dst) & 15) || (reinterpret_cast<uintptr_t>(src) & 15))
    return G2Q_OK;
  if (cudaFuncSetAttribute(permute_cols_staged_kernel<T>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return G2Q_ERR_CUDA;
  long long grid = 148LL * 4;
  if (grid > rows) grid = rows;
  permute_cols_staged_kernel<T><<<(unsigned)grid, 256, smem, st>>>(dst, src, rows, (int)C, perm,
                                                                   inverse);
  G2Q_CHECK_LAUNCH();
  *done = true;
  return G2Q_OK;
}

__global__ void permute_sym_kernel(float* dst, const float* src, long long nl, long long C,
                                   const long long* perm) {
  for (long long row = blockIdx.y; row < nl * C; row += gridDim.y) {
    const long long b = row / C, i = row - b * C;
    const float* s = src + b * C * C + perm[i] * C;
    float* d = dst + row * C;
    for (long long j = (long long)blockIdx.x * blockDim.x + threadIdx.x; j < C;
         j += (long long)gridDim.x * blockDim.x)
      d[j] = s[perm[j]];
  }
}

static dim3 grid_rows(long long rows, long long cols) { return wave_grid_2d(rows, cols); }

// Upper triangle of symmetric matrices, packed row by row: element (i, j),
// i <= j, of matrix b sits at b * C(C+1)/2 + i C - i(i-1)/2 + (j - i).  Rows are
// walked by grid y, columns by thread: reads and writes are both contiguous.
__global__ void pack_upper_kernel(float* dst, const float* H, long long nl, long long C,
                                  long long ldh, long long h_bs, float s) {
  const long long tri = C * (C + 1) / 2;
  for (long long row = blockIdx.y; row < nl * C; row += gridDim.y) {
    const long long b = row / C, i = row - b * C;
    const float* h = H + b * h_bs + i * ldh;
    float* d = dst + b * tri + i * C - i * (i - 1) / 2 - i;
    for (long long j = i + (long long)blockIdx.x * blockDim.x + threadIdx.x; j < C;
         j += (long long)gridDim.x * blockDim.x)
      d[j] = s * h[j];
  }
}

// The inverse of pack_upper_kernel, writing both triangles (the lower one
// mirrored, or zero for a triangular matrix).  One CTA per pair of 32 x 32
// tiles (ti <= tj): the upper tile is read from the packed rows into shared
// memory, then written to (ti, tj) row by row and, transposed, to (tj, ti):
// every global write is a contiguous 32-float run.
__global__ void unpack_upper_kernel(float* H, const float* src, long long C, long long ldh,
                                    long long h_bs, int mirror) {
  const long long ti = blockIdx.y, tj = blockIdx.x;
  if (ti > tj) return;
  __shared__ float tile[32][33];
  const long long b = blockIdx.z;
  const long long tri = C * (C + 1) / 2;
  const float* sb = src + b * tri;
  float* hb = H + b * h_bs;
  const int x = threadIdx.x;
  const long long j = tj * 32 + x;
  for (int y = threadIdx.y; y < 32; y += blockDim.y) {
    const long long i = ti * 32 + y;
    float v = 0.f;
    if (i < C && j < C && j >= i) v = sb[i * C - i * (i - 1) / 2 + (j - i)];
    tile[y][x] = v;
  }
  __syncthreads();
  for (int y = threadIdx.y; y < 32; y += blockDim.y) {
    const long long i = ti * 32 + y;
    if (i < C && j < C && j >= i) hb[i * ldh + j] = tile[y][x];
  }
  // lower triangle: H[jj][ii] = upper (ii, jj) for ii < jj (rows jj of tile
  // tj), or zero for a triangular factor
  const long long ii = ti * 32 + x;
  for (int y = threadIdx.y; y < 32; y += blockDim.y) {
    const long long jj = tj * 32 + y;
    if (ii < C && jj < C && ii < jj) hb[jj * ldh + ii] = mirror ? tile[x][y] : 0.f;
  }
}

template <typename D>
__global__ void cast_check_kernel(D* dst, const float* src, long long n, int* nan_count) {
  int local = 0;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    const float v = src[idx];
    if (v != v) ++local;
    if constexpr (sizeof(D) == 4) dst[idx] = v;
    else if constexpr (std::is_same<D, __half>::value) dst[idx] = __float2half_rn(v);
    else dst[idx] = __float2bfloat16_rn(v);
  }
  if (local && nan_count) atomicAdd(nan_count, local);
}

__global__ void pack_int32_kernel(int32_t* out, const int8_t* codes, long long rows,
                                  long long cols, int bits) {
  const int factor = 32 / bits;
  const long long words = (cols + factor - 1) / factor;
  const long long n = rows * words;
  const int offset = 1 << (bits - 1);
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long r = idx / words, w = idx - r * words;
    uint32_t acc = 0;
    for (int u = 0; u < factor; ++u) {
      const long long c = w * factor + u;
      if (c < cols) {
        const uint32_t v = (uint32_t)(uint8_t)(int8_t)(codes[r * cols + c] + offset);
        acc |= v << (u * bits);
      }
    }
    out[idx] = (int32_t)acc;
  }
}

// One warp per (layer, row).
__global__ void trust_region_kernel(float* beta, const float* grad, const float* GH,
                                    const float* Qs, const float* Ws, const float* dinv,
                                    long long nl, long long rows, long long C, float two_alpha) {
  const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= nl * rows) return;
  const long long b = warp / rows;
  const float* g = grad + warp * C;
  const float* gh = GH + warp * C;
  const float* q = Qs + warp * C;
  const float* w = Ws + warp * C;
  const float* d = dinv + b * C;
  float cs = 0.f;
  for (long long c = lane; c < C; c += 32) cs = fmaf(g[c], gh[c], cs);
  for (int o = 16; o > 0; o >>= 1) cs += __shfl_xor_sync(0xffffffffu, cs, o);
  const float tiny = 1.17549435e-38f;
  float acc = 0.f;
  for (long long c = lane; c < C; c += 32) {
    const float qe = q[c] - w[c];
    const float ghc = gh[c];
    const float dc = d[c];
    const float loss = fabsf((qe * ghc + qe * qe / 2.f) / dc);
    float cc = cs - (ghc * ghc) / dc;
    const float tl = two_alpha * loss;
    cc = fmaxf(cc, tl);
    cc = fmaxf(cc, tiny);
    acc += 1.f - sqrtf(fmaxf(1.f - tl / cc, 0.f));
  }
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) beta[warp] = acc / (float)C;
}

__global__ void diag_utu_kernel(float* dinv, const float* U, long long nl, long long C) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= nl * C) return;
  const long long b = idx / C, c = idx - b * C;
  const float* Ub = U + b * C * C;
  float s = 0.f;
  for (long long k = 0; k <= c; ++k) {
    const float u = Ub[k * C + c];
    s = fmaf(u, u, s);
  }
  dinv[idx] = s;
}

__global__ void scale_rows_kernel(float* X, const float* s, long long nrows, long long C) {
  const long long n = nrows * C;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x)
    X[idx] *= s[idx / C];
}

}  // namespace g2q

#include <atomic>

namespace g2q {
static std::atomic<long long> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace g2q

using namespace g2q;

extern "C" int g2q_abi_version(void) { return 8; }

extern "C" int64_t g2q_launch_count(void) { return g2q::g_launches.load(); }

extern "C" const char* g2q_status_string(int s) {
  switch (s) {
    case G2Q_OK: return "ok";
    case G2Q_ERR_INVALID_ARG: return "invalid argument";
    case G2Q_ERR_CUDA: return "CUDA launch or runtime error";
    case G2Q_ERR_UNSUPPORTED: return "unsupported configuration";
    case G2Q_ERR_NONFINITE: return "non-finite value";
    case G2Q_ERR_TIMEOUT: return "device wait timed out";
    case G2Q_ERR_BAD_SCALE: return "non-positive quantization scale";
    case G2Q_ERR_SCRATCH_LIMIT: return "request exceeds the library-owned static scratch";
  }
  return s > 0 ? "non-positive Cholesky pivot" : "unknown status";
}

extern "C" int g2q_stage_tokens(void* dst, int dst_dtype, int64_t dst_ld, int64_t row0,
                                const void* src, const void* sub, int src_dtype, int64_t src_ld,
                                int64_t t, int64_t C, void* stream) {
  if (!dst || !src || t < 0 || C <= 0 || dst_ld < C || src_ld < C || row0 < 0)
    return G2Q_ERR_INVALID_ARG;
  if (t == 0) return G2Q_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (dst_dtype == src_dtype && !sub) {
    const size_t es = dst_dtype == G2Q_DTYPE_BF16 || dst_dtype == G2Q_DTYPE_F16 ? 2 : 4;
    char* d0 = (char*)dst + (size_t)row0 * dst_ld * es;
    if ((((uintptr_t)d0 | (uintptr_t)src) & 15) == 0 && ((size_t)C * es) % 16 == 0 &&
        ((size_t)dst_ld * es) % 16 == 0 && ((size_t)src_ld * es) % 16 == 0) {
      // 16-byte words on the SMs: reads and writes at HBM speed
      const long long w16 = (long long)((size_t)C * es / 16);
      long long blocks = (t * w16 + 1023) / 1024;
      if (blocks > 148 * 16) blocks = 148 * 16;
      copy_rows16_kernel<<<(int)blocks, 256, 0, st>>>(
          (uint4*)d0, (long long)((size_t)dst_ld * es / 16), (const uint4*)src,
          (long long)((size_t)src_ld * es / 16), t, w16);
      G2Q_CHECK_LAUNCH();
      return G2Q_OK;
    }
    // unaligned rows: a strided device-to-device copy
    if (cudaMemcpy2DAsync((char*)dst + (size_t)row0 * dst_ld * es, (size_t)dst_ld * es, src,
                          (size_t)src_ld * es, (size_t)C * es, (size_t)t,
                          cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      return G2Q_ERR_CUDA;
    return G2Q_OK;
  }
  const int g = grid_for(t * C);
  if (dst_dtype == G2Q_DTYPE_BF16) {
    if (src_dtype != G2Q_DTYPE_BF16 || sub) return G2Q_ERR_INVALID_ARG;
    stage_kernel<__nv_bfloat16, __nv_bfloat16><<<g, 256, 0, st>>>(
        (__nv_bfloat16*)dst, dst_ld, row0, (const __nv_bfloat16*)src,
        (const __nv_bfloat16*)sub, src_ld, t, C);
  } else if (dst_dtype == G2Q_DTYPE_F32) {
    if (src_dtype == G2Q_DTYPE_F32)
      stage_kernel<float, float><<<g, 256, 0, st>>>((float*)dst, dst_ld, row0,
                                                     (const float*)src, (const float*)sub,
                                                     src_ld, t, C);
    else if (src_dtype == G2Q_DTYPE_BF16)
      stage_kernel<__nv_bfloat16, float><<<g, 256, 0, st>>>(
          (float*)dst, dst_ld, row0, (const __nv_bfloat16*)src, (const __nv_bfloat16*)sub,
          src_ld, t, C);
    else if (src_dtype == G2Q_DTYPE_F16)
      stage_kernel<__half, float><<<g, 256, 0, st>>>((float*)dst, dst_ld, row0,
                                                      (const __half*)src, (const __half*)sub,
                                                      src_ld, t, C);
    else
      return G2Q_ERR_INVALID_ARG;
  } else {
    return G2Q_ERR_INVALID_ARG;
  }
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" size_t g2q_gram_grouped_workspace_bytes(int64_t C, int64_t T, int G, int precision) {
  if (precision == 1 && C > 0 && T >= 0 && G > 0) return tc_gram_grouped_workspace_bytes(C, T, G);
  return 0;
}

extern "C" int g2q_gram_update_grouped(float* D, int64_t ldd, int64_t d_gstride, int64_t C,
                                       const void* X, int x_dtype, int64_t ldx, const float* s,
                                       int64_t sstride, int G, int64_t T, float alpha, float beta,
                                       int precision, void* workspace, size_t workspace_bytes,
                                       int* status, void* stream) {
  if (!D || !X || !s || C <= 0 || T < 0 || G <= 0 || ldx < C || ldd < C || sstride < G ||
      d_gstride < C * ldd)
    return G2Q_ERR_INVALID_ARG;
  if (x_dtype != G2Q_DTYPE_BF16 && x_dtype != G2Q_DTYPE_F32) return G2Q_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (precision == 1)
    return tc_gram_grouped(D, ldd, d_gstride, C, X, x_dtype, ldx, s, sstride, G, T, alpha, beta,
                           workspace, workspace_bytes, status, st);
  if (precision != 0) return G2Q_ERR_INVALID_ARG;
  for (int g = 0; g < G; ++g)
    G2Q_TRY(g2q_gram_update(D + g * d_gstride, ldd, C, C, X, x_dtype, ldx, X, x_dtype, ldx, s + g,
                            sstride, T, 1, alpha, beta, 0, nullptr, 0, status, stream));
  return G2Q_OK;
}

extern "C" size_t g2q_gram_workspace_bytes(int64_t M, int64_t N, int64_t T, int precision) {
  if (precision == 1) return tc_gram_workspace_bytes(M, N, T);
  return 0;
}

extern "C" int g2q_gram_update(float* D, int64_t ldd, int64_t M, int64_t N, const void* A,
                               int a_dtype, int64_t lda, const void* B, int b_dtype,
                               int64_t ldb, const float* row_scale, int64_t scale_stride,
                               int64_t T, int symmetric, float alpha, float beta, int precision,
                               void* workspace, size_t workspace_bytes, int* status,
                               void* stream) {
  if (!D || !A || !B || M <= 0 || N <= 0 || T < 0 || lda < M || ldb < N || ldd < N)
    return G2Q_ERR_INVALID_ARG;
  if ((a_dtype != G2Q_DTYPE_BF16 && a_dtype != G2Q_DTYPE_F32) ||
      (b_dtype != G2Q_DTYPE_BF16 && b_dtype != G2Q_DTYPE_F32))
    return G2Q_ERR_INVALID_ARG;
  if (symmetric && M != N) return G2Q_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (precision == 1)
    return tc_gram(D, ldd, M, N, A, a_dtype, lda, B, b_dtype, ldb, row_scale, scale_stride, T,
                   symmetric, alpha, beta, workspace, workspace_bytes, status, st);
  if (precision != 0) return G2Q_ERR_INVALID_ARG;
  SimtArgs a{};
  a.A = A; a.B = B; a.C = D;
  a.lda = lda; a.ldb = ldb; a.ldc = ldd;
  a.M = M; a.N = N; a.K = T;
  a.alpha = alpha; a.beta = beta;
  a.kscale = row_scale; a.kscale_stride = scale_stride;
  a.mask = G2Q_MASK_FULL;
  a.mirror = symmetric ? 1 : 0;
  if (T == 0) {
    // D <- alpha * D (beta term is empty)
    a.K = 0;
  }
  return simt_gemm(a, true, false, a_dtype, b_dtype, 1, st);
}

// acc[c] += scale * sum_t X[t][c]^2 for BF16 X with 16-byte rows: a CTA of
// 32 x 8 threads covers 256 columns (eight per thread, one 16-byte load per
// token) and 128 tokens (eight token lanes), reduces the lanes in shared
// memory and adds one partial per column.
constexpr int SQ_TCHUNK = 128;
__global__ void __launch_bounds__(256) sq_colsum_bf16x8_kernel(float* acc, float scale,
                                                               const __nv_bfloat16* X,
                                                               long long ldx, long long T,
                                                               long long C) {
  __shared__ float part[8][257];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const long long c0 = ((long long)blockIdx.x * 32 + tx) * 8;
  const long long t0 = (long long)blockIdx.y * SQ_TCHUNK;
  const long long t1 = (t0 + SQ_TCHUNK < T) ? t0 + SQ_TCHUNK : T;
  float a[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) a[u] = 0.f;
  if (c0 < C) {
#pragma unroll 4
    for (long long t = t0 + ty; t < t1; t += 8) {
      const uint4 raw = *reinterpret_cast<const uint4*>(X + t * ldx + c0);
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const float v = __bfloat162float(xb[u]);
        a[u] = fmaf(v, v, a[u]);
      }
    }
  }
#pragma unroll
  for (int u = 0; u < 8; ++u) part[ty][tx * 8 + u] = a[u];
  __syncthreads();
  const int c = ty * 32 + tx;  // 256 columns, one per thread
  float sum = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) sum += part[q][c];
  const long long gc = (long long)blockIdx.x * 256 + c;
  if (gc < C) atomicAdd(acc + gc, sum * scale);
}

extern "C" int g2q_sq_colsum(float* acc, float keep, float scale, const void* X, int x_dtype,
                             int64_t ldx, int64_t T, int64_t C, void* stream) {
  if (!acc || !X || C <= 0 || T < 0 || ldx < C) return G2Q_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  scale_vec_kernel<<<cdiv(C, 256), 256, 0, st>>>(acc, C, keep);
  G2Q_CHECK_LAUNCH();
  if (T == 0) return G2Q_OK;
  if (x_dtype == G2Q_DTYPE_BF16 && (C % 8) == 0 && (ldx % 8) == 0 &&
      (reinterpret_cast<uintptr_t>(X) & 15) == 0 && cdiv(T, SQ_TCHUNK) <= 65535) {
    dim3 grid(cdiv(C, 256), cdiv(T, SQ_TCHUNK));
    sq_colsum_bf16x8_kernel<<<grid, dim3(32, 8), 0, st>>>(acc, scale, (const __nv_bfloat16*)X,
                                                         ldx, T, C);
    G2Q_CHECK_LAUNCH();
    return G2Q_OK;
  }
  const long long tchunk = 256;
  dim3 grid(cdiv(C, 256), cdiv(T, tchunk));
  if (grid.y > 65535u) return G2Q_ERR_INVALID_ARG;
  if (x_dtype == G2Q_DTYPE_F32)
    sq_colsum_kernel<float><<<grid, 256, 0, st>>>(acc, scale, (const float*)X, ldx, T, C, tchunk);
  else if (x_dtype == G2Q_DTYPE_BF16)
    sq_colsum_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(acc, scale, (const __nv_bfloat16*)X,
                                                          ldx, T, C, tchunk);
  else if (x_dtype == G2Q_DTYPE_F16)
    sq_colsum_kernel<__half><<<grid, 256, 0, st>>>(acc, scale, (const __half*)X, ldx, T, C,
                                                   tchunk);
  else
    return G2Q_ERR_INVALID_ARG;
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_prepare_hessian(float* H, int64_t nl, int64_t C, float* W, int64_t rows,
                                   float* extra, int64_t extra_rows, float* gzero,
                                   void* stream) {
  if (!H || nl <= 0 || C <= 0 || rows < 0) return G2Q_ERR_INVALID_ARG;
  prepare_hessian_kernel<<<(unsigned)nl, 256, 0, (cudaStream_t)stream>>>(H, C, W, rows, extra,
                                                                         extra_rows, gzero);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_argsort_desc(int64_t* perm, const float* key, int64_t n, void* stream) {
  if (!perm || !key || n <= 0) return G2Q_ERR_INVALID_ARG;
  argsort_desc_kernel<<<cdiv(n, 256), 256, 0, (cudaStream_t)stream>>>((long long*)perm, key, n);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_mean_diag(float* key, const float* H, int64_t nl, int64_t C, void* stream) {
  if (!key || !H || nl <= 0 || C <= 0) return G2Q_ERR_INVALID_ARG;
  mean_diag_kernel<<<cdiv(C, 256), 256, 0, (cudaStream_t)stream>>>(key, H, nl, C);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_permute_cols(void* dst, const void* src, int elem_bytes, int64_t nl,
                                int64_t rows, int64_t C, const int64_t* perm, int inverse,
                                void* stream) {
  if (!dst || !src || !perm || nl < 0 || rows < 0 || C <= 0 || dst == src)
    return G2Q_ERR_INVALID_ARG;
  const long long n = nl * rows * C;
  if (n == 0) return G2Q_OK;
  cudaStream_t st = (cudaStream_t)stream;
  bool done = false;
  if (elem_bytes == 4)
    G2Q_TRY(permute_cols_staged((float*)dst, (const float*)src, nl * rows, C,
                                (const long long*)perm, inverse, st, &done));
  else if (elem_bytes == 1)
    G2Q_TRY(permute_cols_staged((int8_t*)dst, (const int8_t*)src, nl * rows, C,
                                (const long long*)perm, inverse, st, &done));
  if (done) return G2Q_OK;
  if (elem_bytes == 4)
    permute_cols_kernel<float><<<grid_rows(nl * rows, C), 256, 0, st>>>((float*)dst, (const float*)src,
                                                            nl * rows, C, (const long long*)perm,
                                                            inverse);
  else if (elem_bytes == 1)
    permute_cols_kernel<int8_t><<<grid_rows(nl * rows, C), 256, 0, st>>>((int8_t*)dst, (const int8_t*)src,
                                                             nl * rows, C,
                                                             (const long long*)perm, inverse);
  else
    return G2Q_ERR_INVALID_ARG;
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_permute_sym(float* dst, const float* src, int64_t nl, int64_t C,
                               const int64_t* perm, void* stream) {
  if (!dst || !src || !perm || nl <= 0 || C <= 0 || dst == src) return G2Q_ERR_INVALID_ARG;
  permute_sym_kernel<<<grid_rows(nl * C, C), 256, 0, (cudaStream_t)stream>>>(
      dst, src, nl, C, (const long long*)perm);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_pack_upper(float* dst, const float* H, int64_t C, int64_t ldh,
                              int64_t h_bstride, int64_t batch, float scale, void* stream) {
  if (!dst || !H || C <= 0 || ldh < C || batch < 0 || (batch > 1 && h_bstride < C * ldh))
    return G2Q_ERR_INVALID_ARG;
  if (batch == 0) return G2Q_OK;
  pack_upper_kernel<<<grid_rows(batch * C, C), 256, 0, (cudaStream_t)stream>>>(
      dst, H, batch, C, ldh, h_bstride, scale);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_unpack_upper(float* H, const float* src, int64_t C, int64_t ldh,
                                int64_t h_bstride, int64_t batch, int mirror, void* stream) {
  if (!H || !src || C <= 0 || ldh < C || batch < 0 || (batch > 1 && h_bstride < C * ldh) ||
      batch > 65535)
    return G2Q_ERR_INVALID_ARG;
  if (batch == 0) return G2Q_OK;
  const unsigned t = (unsigned)((C + 31) / 32);
  unpack_upper_kernel<<<dim3(t, t, (unsigned)batch), dim3(32, 8), 0, (cudaStream_t)stream>>>(
      H, src, C, ldh, h_bstride, mirror);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_cast_check(void* dst, int dst_dtype, const float* src, int64_t n,
                              int* nan_count, void* stream) {
  if (!dst || !src || n < 0) return G2Q_ERR_INVALID_ARG;
  if (n == 0) return G2Q_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (dst_dtype == G2Q_DTYPE_F32)
    cast_check_kernel<float><<<grid_for(n), 256, 0, st>>>((float*)dst, src, n, nan_count);
  else if (dst_dtype == G2Q_DTYPE_BF16)
    cast_check_kernel<__nv_bfloat16><<<grid_for(n), 256, 0, st>>>((__nv_bfloat16*)dst, src, n,
                                                                  nan_count);
  else if (dst_dtype == G2Q_DTYPE_F16)
    cast_check_kernel<__half><<<grid_for(n), 256, 0, st>>>((__half*)dst, src, n, nan_count);
  else
    return G2Q_ERR_INVALID_ARG;
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_pack_int32(int32_t* out, const int8_t* codes, int64_t rows, int64_t cols,
                              int bits, void* stream) {
  if (!out || !codes || rows < 0 || cols <= 0 || bits < 1 || bits > 8)
    return G2Q_ERR_INVALID_ARG;
  const int factor = 32 / bits;
  const long long n = rows * ((cols + factor - 1) / factor);
  if (n == 0) return G2Q_OK;
  pack_int32_kernel<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(out, codes, rows, cols, bits);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_trust_region_beta(float* beta, const float* grad, const float* GH,
                                     const float* Qsub, const float* Wsub, const float* dinv,
                                     int64_t nl, int64_t rows, int64_t C, float alpha,
                                     void* stream) {
  if (!beta || !grad || !GH || !Qsub || !Wsub || !dinv || nl <= 0 || rows <= 0 || C <= 0)
    return G2Q_ERR_INVALID_ARG;
  const long long warps = nl * rows;
  trust_region_kernel<<<cdiv(warps, 8), 256, 0, (cudaStream_t)stream>>>(
      beta, grad, GH, Qsub, Wsub, dinv, nl, rows, C, (float)(2.0 * (double)alpha));
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_diag_of_utu(float* dinv, const float* U, int64_t nl, int64_t C, void* stream) {
  if (!dinv || !U || nl <= 0 || C <= 0) return G2Q_ERR_INVALID_ARG;
  diag_utu_kernel<<<cdiv(nl * C, 256), 256, 0, (cudaStream_t)stream>>>(dinv, U, nl, C);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_scale_rows(float* X, const float* s, int64_t nl, int64_t rows, int64_t C,
                              void* stream) {
  if (!X || !s || nl <= 0 || rows <= 0 || C <= 0) return G2Q_ERR_INVALID_ARG;
  scale_rows_kernel<<<grid_for(nl * rows * C), 256, 0, (cudaStream_t)stream>>>(X, s, nl * rows,
                                                                              C);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}
