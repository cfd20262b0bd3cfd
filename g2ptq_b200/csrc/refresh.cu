// G2PTQ refresh step: the arithmetic of the saliency and gradient caches and
// the block-loss heads whose backward feeds them.
//
//  * saliency: the per-token group mean of squared output gradients
//    (SaliencyCache.grad_hook, gptq_utils/g2ptq_utils.py:605-618);
//  * running mean of weight gradients (GradientCache.cache_gradient,
//    g2ptq_utils.py:693-702) and the weighted sums over loss types
//    (summarize_saliency / summarize_gradients, g2ptq_utils.py:620-640, 704-711);
//  * block-loss heads, forward and backward in one pass over the rows each:
//    KL(softmax(target) || softmax(x)) summed over rows
//    (compute_kl_grad_hessian, g2ptq_utils.py:969-1001), the sampled-label
//    cross entropy of the same function, and the row-mean squared error of
//    compute_mse_grad_hessian (g2ptq_utils.py:1004-1035).
//
// All of it is HBM-bound: the loss heads read each row once forward
// (an online softmax in base 2 keeps the running maximum and sum) and once
// backward, writing the gradient in the input's dtype.
#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"

namespace g2q {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <typename S>
__device__ __forceinline__ float cvt(S v);
template <>
__device__ __forceinline__ float cvt<float>(float v) { return v; }
template <>
__device__ __forceinline__ float cvt<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float cvt<__half>(__half v) { return __half2float(v); }

template <typename S>
__device__ __forceinline__ S from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// E elements starting at p: one 16-byte load when VEC, else one element.
template <typename S, bool VEC>
struct Lanes {
  static constexpr int E = VEC ? 16 / (int)sizeof(S) : 1;
  __device__ __forceinline__ static void load(float* v, const S* p) {
    if constexpr (VEC) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
      const S* e = reinterpret_cast<const S*>(&raw);
#pragma unroll
      for (int u = 0; u < E; ++u) v[u] = cvt<S>(e[u]);
    } else {
      v[0] = cvt<S>(*p);
    }
  }
  __device__ __forceinline__ static void store(S* p, const float* v) {
    if constexpr (VEC) {
      uint4 raw;
      S* e = reinterpret_cast<S*>(&raw);
#pragma unroll
      for (int u = 0; u < E; ++u) e[u] = from_f<S>(v[u]);
      *reinterpret_cast<uint4*>(p) = raw;
    } else {
      *p = from_f<S>(v[0]);
    }
  }
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// Saliency: out[t][g] = mean over the g-th block of gs columns of grad[t][:]^2.
// One warp per (token, group).
// ---------------------------------------------------------------------------
template <typename S, bool VEC>
__global__ void __launch_bounds__(256) saliency_kernel(float* __restrict__ out,
                                                       const S* __restrict__ grad, long long ld,
                                                       long long T, int G, long long gs,
                                                       float inv_gs) {
  using L = Lanes<S, VEC>;
  const int lane = threadIdx.x & 31;
  const long long nw = (long long)gridDim.x * (blockDim.x >> 5);
  const long long nvec = gs / L::E;
  for (long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < T * G;
       w += nw) {
    const long long t = w / G;
    const long long g = w - t * G;
    const S* p = grad + t * ld + g * gs;
    float acc = 0.f;
#pragma unroll 4
    for (long long i = lane; i < nvec; i += 32) {
      float v[L::E];
      L::load(v, p + i * L::E);
#pragma unroll
      for (int u = 0; u < L::E; ++u) acc = fmaf(v[u], v[u], acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) out[w] = acc * inv_gs;
  }
}

// ---------------------------------------------------------------------------
// out = (first ? 0 : out) + w * x, each product and sum rounded on its own
// (the reference's Python sum over loss types of w * tensor).
// ---------------------------------------------------------------------------
__global__ void scaled_accumulate_kernel(float* __restrict__ out, const float* __restrict__ x,
                                         long long n, float w, int first) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float base = first ? 0.f : out[i];
    out[i] = __fadd_rn(base, __fmul_rn(w, x[i]));
  }
}

__global__ void scaled_accumulate_v4_kernel(float4* __restrict__ out,
                                            const float4* __restrict__ x, long long n4, float w,
                                            int first) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = __ldg(x + i);
    float4 b = first ? make_float4(0.f, 0.f, 0.f, 0.f) : out[i];
    b.x = __fadd_rn(b.x, __fmul_rn(w, v.x));
    b.y = __fadd_rn(b.y, __fmul_rn(w, v.y));
    b.z = __fadd_rn(b.z, __fmul_rn(w, v.z));
    b.w = __fadd_rn(b.w, __fmul_rn(w, v.w));
    out[i] = b;
  }
}

// ---------------------------------------------------------------------------
// cache = (first ? 0 : cache * keep) + grad * inv, each step rounded on its
// own (the reference's cache * (i / (i + 1)) + grad.float() / (n_tok * (i + 1)),
// the division by a host scalar done as torch's CUDA kernels do it: a multiply
// by the fp32 reciprocal).
// ---------------------------------------------------------------------------
template <typename S, bool VEC>
__global__ void __launch_bounds__(256) running_mean_kernel(float* __restrict__ cache,
                                                           const S* __restrict__ grad,
                                                           long long n, float keep, float inv,
                                                           int first) {
  using L = Lanes<S, VEC>;
  const long long nvec = n / L::E;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += stride) {
    float g[L::E];
    L::load(g, grad + i * L::E);
    float* c = cache + i * L::E;
    if constexpr (L::E % 4 == 0) {
#pragma unroll
      for (int q = 0; q < L::E / 4; ++q) {
        float4 b = first ? make_float4(0.f, 0.f, 0.f, 0.f) : reinterpret_cast<float4*>(c)[q];
        b.x = __fadd_rn(first ? 0.f : __fmul_rn(b.x, keep), __fmul_rn(g[4 * q + 0], inv));
        b.y = __fadd_rn(first ? 0.f : __fmul_rn(b.y, keep), __fmul_rn(g[4 * q + 1], inv));
        b.z = __fadd_rn(first ? 0.f : __fmul_rn(b.z, keep), __fmul_rn(g[4 * q + 2], inv));
        b.w = __fadd_rn(first ? 0.f : __fmul_rn(b.w, keep), __fmul_rn(g[4 * q + 3], inv));
        reinterpret_cast<float4*>(c)[q] = b;
      }
    } else {
#pragma unroll
      for (int u = 0; u < L::E; ++u) {
        const float b = first ? 0.f : __fmul_rn(c[u], keep);
        c[u] = __fadd_rn(b, __fmul_rn(g[u], inv));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Block-loss heads.  Row statistics (per row, 3 floats):
//   [0] log2-sum-exp2 of x * log2(e)       (KL, NLL)
//   [1] log2-sum-exp2 of target * log2(e)  (KL)
//   [2] the row's loss                      (all kinds)
// ---------------------------------------------------------------------------
constexpr int LOSS_THREADS = 256;

// 2^v on the SFU (one MUFU op; relative error about 2^-22, results below
// 2^-126 flushed to zero, which no softmax sum notices).
__device__ __forceinline__ float ex2(float v) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

// Running state of one softmax over raw values x: m the largest x seen,
// c = fl(m log2 e) the base-2 offset every term of s was taken against,
// s = sum 2^(x log2 e - c).  Rescales use the stored offsets, so the final
// log2-sum-exp2 c + log2 s matches the terms exactly.
struct Soft {
  float m = -INFINITY;
  float c = -INFINITY;
  float s = 0.f;
};

// Adds E values; returns the offset the terms were taken against (the
// caller's weights for other sums use the same one).
template <int E>
__device__ __forceinline__ bool soft_add(Soft& st, const float* x, float* acc_out = nullptr,
                                         float* rescale_out = nullptr) {
  float mv = x[0];
#pragma unroll
  for (int u = 1; u < E; ++u) mv = fmaxf(mv, x[u]);
  if (!(mv > st.m) && st.m == -INFINITY) return false;  // nothing but -inf so far
  float rs = 1.f;
  if (mv > st.m) {  // the maximum grows: rarely, once the first vectors are in
    const float c = mv * kLog2e;
    rs = ex2(st.c - c);  // 0 on the first vector (st.c = -inf)
    st.s *= rs;
    st.m = mv;
    st.c = c;
  }
  const float nc = -st.c;
  float acc = 0.f;
#pragma unroll
  for (int u = 0; u < E; ++u) {
    const float w = ex2(fmaf(x[u], kLog2e, nc));
    acc += w;
    if (acc_out) acc_out[u] = w;
  }
  st.s += acc;
  if (rescale_out) *rescale_out = rs;
  return true;
}

__device__ __forceinline__ void soft_merge(Soft& a, float m2, float c2, float s2,
                                           float* extra_a = nullptr, float extra_b = 0.f) {
  if (m2 == -INFINITY) return;
  if (a.m == -INFINITY || m2 > a.m) {
    const float r1 = ex2(a.c - c2);
    a.s = a.s * r1 + s2;
    if (extra_a) *extra_a = *extra_a * r1 + extra_b;
    a.m = m2;
    a.c = c2;
  } else {
    const float r2 = ex2(c2 - a.c);
    a.s = a.s + s2 * r2;
    if (extra_a) *extra_a = *extra_a + extra_b * r2;
  }
}

// Block-wide merge of up to two softmax states and one weighted sum carried
// with the second state; thread 0 receives the result.
__device__ __forceinline__ void block_merge(Soft& q, Soft& p, float& a, float& plain) {
  __shared__ float sh[LOSS_THREADS / 32][8];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float qm = __shfl_xor_sync(0xffffffffu, q.m, o);
    const float qc = __shfl_xor_sync(0xffffffffu, q.c, o);
    const float qs = __shfl_xor_sync(0xffffffffu, q.s, o);
    const float pm = __shfl_xor_sync(0xffffffffu, p.m, o);
    const float pc = __shfl_xor_sync(0xffffffffu, p.c, o);
    const float ps = __shfl_xor_sync(0xffffffffu, p.s, o);
    const float pa = __shfl_xor_sync(0xffffffffu, a, o);
    plain += __shfl_xor_sync(0xffffffffu, plain, o);
    soft_merge(q, qm, qc, qs);
    soft_merge(p, pm, pc, ps, &a, pa);
  }
  if (lane == 0) {
    sh[wid][0] = q.m;
    sh[wid][1] = q.c;
    sh[wid][2] = q.s;
    sh[wid][3] = p.m;
    sh[wid][4] = p.c;
    sh[wid][5] = p.s;
    sh[wid][6] = a;
    sh[wid][7] = plain;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < LOSS_THREADS / 32; ++w) {
      soft_merge(q, sh[w][0], sh[w][1], sh[w][2]);
      soft_merge(p, sh[w][3], sh[w][4], sh[w][5], &a, sh[w][6]);
      plain += sh[w][7];
    }
  }
  __syncthreads();
}

__device__ __forceinline__ float log2sum(const Soft& st) {
  return st.m == -INFINITY ? -INFINITY : st.c + log2f(st.s);
}

// One CTA per row (grid-stride).  KIND: 0 KL, 1 NLL, 2 MSE.
template <typename S, bool VEC, int KIND>
__global__ void __launch_bounds__(LOSS_THREADS) loss_forward_kernel(
    float* __restrict__ stats, const S* __restrict__ x, long long ldx, const S* __restrict__ tg,
    long long ldt, const int64_t* __restrict__ labels, long long rows, long long V) {
  using L = Lanes<S, VEC>;
  const long long nvec = V / L::E;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const S* xr = x + r * ldx;
    const S* tr = (KIND != 1) ? tg + r * ldt : nullptr;
    Soft q, p;
    float a = 0.f, plain = 0.f;
#pragma unroll 2
    for (long long i = threadIdx.x; i < nvec; i += LOSS_THREADS) {
      float xv[L::E];
      L::load(xv, xr + i * L::E);
      if constexpr (KIND == 2) {
        float tv[L::E];
        L::load(tv, tr + i * L::E);
#pragma unroll
        for (int u = 0; u < L::E; ++u) {
          const float d = xv[u] - tv[u];
          plain = fmaf(d, d, plain);
        }
      } else {
        soft_add<L::E>(q, xv);
        if constexpr (KIND == 0) {
          float tv[L::E], w[L::E], rs;
          L::load(tv, tr + i * L::E);
          if (soft_add<L::E>(p, tv, w, &rs)) {
            float acca = 0.f;
#pragma unroll
            for (int u = 0; u < L::E; ++u) {
              // a zero weight contributes nothing, as the reference's
              // target * (log target - input) does for target == 0
              acca = (w[u] > 0.f) ? fmaf(w[u], tv[u] - xv[u], acca) : acca;
            }
            a = a * rs + acca;
          }
        }
      }
    }
    block_merge(q, p, a, plain);
    if (threadIdx.x == 0) {
      float* st = stats + 3 * r;
      if constexpr (KIND == 2) {
        st[0] = 0.f;
        st[1] = 0.f;
        st[2] = 0.5f * (plain / (float)V);
      } else {
        const float l2q = log2sum(q);
        st[0] = l2q;
        if constexpr (KIND == 0) {
          const float l2p = log2sum(p);
          st[1] = l2p;
          st[2] = a / p.s - (l2p - l2q) * kLn2;
        } else {
          const long long lab = labels[r];
          st[1] = 0.f;
          if (lab == -100)
            st[2] = 0.f;  // cross entropy's ignore_index
          else if (lab < 0 || lab >= V)
            st[2] = NAN;  // out-of-range label: the loss reports it, nothing is read
          else
            st[2] = l2q * kLn2 - cvt<S>(xr[lab]);
        }
      }
    }
    __syncthreads();
  }
}

// Deterministic sum of the row losses (fixed order) into loss[0].
__global__ void __launch_bounds__(1024) loss_sum_kernel(float* loss, const float* stats,
                                                        long long rows) {
  __shared__ float sh[32];
  float acc = 0.f;
  for (long long r = threadIdx.x; r < rows; r += 1024) acc += stats[3 * r + 2];
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = sh[threadIdx.x];
    v = warp_sum(v);
    if (threadIdx.x == 0) loss[0] = v;
  }
}

template <typename S, bool VEC, int KIND>
__global__ void __launch_bounds__(LOSS_THREADS) loss_backward_kernel(
    S* __restrict__ grad, long long ldg, const float* __restrict__ stats, const S* __restrict__ x,
    long long ldx, const S* __restrict__ tg, long long ldt, const int64_t* __restrict__ labels,
    const float* __restrict__ gscale_ptr, long long rows, long long V) {
  using L = Lanes<S, VEC>;
  const long long nvec = V / L::E;
  const float gs = gscale_ptr ? *gscale_ptr : 1.f;
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    const S* xr = x + r * ldx;
    S* gr = grad + r * ldg;
    const float l2q = stats[3 * r + 0];
    const float l2p = stats[3 * r + 1];
    long long lab = -1;
    float row_gs = gs;
    if constexpr (KIND == 1) {
      lab = labels[r];
      if (lab == -100 || lab < 0 || lab >= V) row_gs = 0.f;  // ignored / invalid rows
    }
    const float invV = 1.f / (float)V;
#pragma unroll 2
    for (long long i = threadIdx.x; i < nvec; i += LOSS_THREADS) {
      float xv[L::E], g[L::E];
      L::load(xv, xr + i * L::E);
      if constexpr (KIND == 0) {
        float tv[L::E];
        L::load(tv, tg + r * ldt + i * L::E);
#pragma unroll
        for (int u = 0; u < L::E; ++u) {
          const float qv = ex2(fmaf(xv[u], kLog2e, -l2q));
          const float pv = ex2(fmaf(tv[u], kLog2e, -l2p));
          g[u] = row_gs * (qv - pv);
        }
      } else if constexpr (KIND == 1) {
#pragma unroll
        for (int u = 0; u < L::E; ++u) {
          const float qv = ex2(fmaf(xv[u], kLog2e, -l2q));
          const long long j = i * L::E + u;
          g[u] = row_gs * (qv - (j == lab ? 1.f : 0.f));
        }
      } else {
        float tv[L::E];
        L::load(tv, tg + r * ldt + i * L::E);
#pragma unroll
        for (int u = 0; u < L::E; ++u) g[u] = row_gs * ((xv[u] - tv[u]) * invV);
      }
      L::store(gr + i * L::E, g);
    }
  }
}

bool aligned16(const void* p) { return p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// One row is the unit of work, so the grid is the number of CTAs that are
// resident at once (rows spread evenly over them; a second partial wave of
// whole rows would leave most SMs idle at the end).
template <typename K>
int loss_grid(K kernel, long long rows) {
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, LOSS_THREADS, 0);
  long long g = (long long)sms * (per_sm > 0 ? per_sm : 1);
  if (rows < g) g = rows;
  return (int)(g < 1 ? 1 : g);
}

template <typename S, bool VEC>
int launch_loss_forward(int kind, float* stats, const S* x, long long ldx, const S* t,
                        long long ldt, const int64_t* labels, long long rows, long long V,
                        cudaStream_t st) {
  if (kind == G2Q_LOSS_KL)
    loss_forward_kernel<S, VEC, 0><<<loss_grid(loss_forward_kernel<S, VEC, 0>, rows),
                                      LOSS_THREADS, 0, st>>>(stats, x, ldx, t, ldt, labels, rows,
                                                             V);
  else if (kind == G2Q_LOSS_NLL)
    loss_forward_kernel<S, VEC, 1><<<loss_grid(loss_forward_kernel<S, VEC, 1>, rows),
                                      LOSS_THREADS, 0, st>>>(stats, x, ldx, t, ldt, labels, rows,
                                                             V);
  else
    loss_forward_kernel<S, VEC, 2><<<loss_grid(loss_forward_kernel<S, VEC, 2>, rows),
                                      LOSS_THREADS, 0, st>>>(stats, x, ldx, t, ldt, labels, rows,
                                                             V);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

template <typename S, bool VEC>
int launch_loss_backward(int kind, S* grad, long long ldg, const float* stats, const S* x,
                         long long ldx, const S* t, long long ldt, const int64_t* labels,
                         const float* gscale, long long rows, long long V, cudaStream_t st) {
  if (kind == G2Q_LOSS_KL)
    loss_backward_kernel<S, VEC, 0><<<loss_grid(loss_backward_kernel<S, VEC, 0>, rows),
                                       LOSS_THREADS, 0, st>>>(grad, ldg, stats, x, ldx, t, ldt,
                                                              labels, gscale, rows, V);
  else if (kind == G2Q_LOSS_NLL)
    loss_backward_kernel<S, VEC, 1><<<loss_grid(loss_backward_kernel<S, VEC, 1>, rows),
                                       LOSS_THREADS, 0, st>>>(grad, ldg, stats, x, ldx, t, ldt,
                                                              labels, gscale, rows, V);
  else
    loss_backward_kernel<S, VEC, 2><<<loss_grid(loss_backward_kernel<S, VEC, 2>, rows),
                                       LOSS_THREADS, 0, st>>>(grad, ldg, stats, x, ldx, t, ldt,
                                                              labels, gscale, rows, V);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

template <typename S>
int dispatch_loss_forward(bool vec, int kind, float* stats, const void* x, long long ldx,
                          const void* t, long long ldt, const int64_t* labels, long long rows,
                          long long V, cudaStream_t st) {
  return vec ? launch_loss_forward<S, true>(kind, stats, (const S*)x, ldx, (const S*)t, ldt,
                                            labels, rows, V, st)
             : launch_loss_forward<S, false>(kind, stats, (const S*)x, ldx, (const S*)t, ldt,
                                             labels, rows, V, st);
}

int elem_bytes(int dtype) {
  return dtype == G2Q_DTYPE_F32 ? 4 : (dtype == G2Q_DTYPE_BF16 || dtype == G2Q_DTYPE_F16) ? 2 : 0;
}

// Whether rows of `n` elements at stride `ld` starting at p can be read in
// 16-byte pieces.
bool vec_ok(const void* p, long long ld, long long n, int eb) {
  const long long per = 16 / eb;
  return aligned16(p) && (ld % per) == 0 && (n % per) == 0;
}

}  // namespace
}  // namespace g2q

using namespace g2q;

extern "C" int g2q_saliency(float* out, const void* grad, int dtype, int64_t ld, int64_t T,
                            int64_t R, int G, void* stream) {
  const int eb = elem_bytes(dtype);
  if (eb == 0 || T < 0 || R <= 0 || G <= 0 || (R % G) != 0 || ld < R)
    return G2Q_ERR_INVALID_ARG;
  if (T == 0) return G2Q_OK;  // nothing to read or write (empty buffers may be NULL)
  if (!out || !grad) return G2Q_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const long long gs = R / G;
  const float inv_gs = 1.f / (float)gs;
  const long long warps = T * (long long)G;
  long long blocks = (warps + 7) / 8;
  if (blocks > 148 * 16) blocks = 148 * 16;
  const bool vec = vec_ok(grad, ld, gs, eb);
#define G2Q_SAL(S)                                                                              \
  if (vec)                                                                                      \
    saliency_kernel<S, true><<<(int)blocks, 256, 0, st>>>(out, (const S*)grad, ld, T, G, gs,    \
                                                          inv_gs);                              \
  else                                                                                          \
    saliency_kernel<S, false><<<(int)blocks, 256, 0, st>>>(out, (const S*)grad, ld, T, G, gs,   \
                                                           inv_gs);
  if (dtype == G2Q_DTYPE_BF16) {
    G2Q_SAL(__nv_bfloat16)
  } else if (dtype == G2Q_DTYPE_F16) {
    G2Q_SAL(__half)
  } else {
    G2Q_SAL(float)
  }
#undef G2Q_SAL
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_scaled_accumulate(float* out, const float* x, int64_t n, float w, int first,
                                     void* stream) {
  if (n < 0 || (n > 0 && (!out || !x))) return G2Q_ERR_INVALID_ARG;
  if (n == 0) return G2Q_OK;
  cudaStream_t st = (cudaStream_t)stream;
  if (aligned16(out) && aligned16(x) && (n % 4) == 0) {
    const long long n4 = n / 4;
    scaled_accumulate_v4_kernel<<<cdiv(n4, 256) < 148 * 8 ? cdiv(n4, 256) : 148 * 8, 256, 0,
                                  st>>>(reinterpret_cast<float4*>(out),
                                        reinterpret_cast<const float4*>(x), n4, w, first);
  } else {
    scaled_accumulate_kernel<<<cdiv(n, 256) < 148 * 8 ? cdiv(n, 256) : 148 * 8, 256, 0, st>>>(
        out, x, n, w, first);
  }
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_running_mean(float* cache, const void* grad, int dtype, int64_t n, float keep,
                                float inv, int first, void* stream) {
  const int eb = elem_bytes(dtype);
  if (eb == 0 || n < 0 || (n > 0 && (!cache || !grad))) return G2Q_ERR_INVALID_ARG;
  if (n == 0) return G2Q_OK;
  cudaStream_t st = (cudaStream_t)stream;
  const bool vec = aligned16(cache) && vec_ok(grad, 0, n, eb);
  const long long units = vec ? n / (16 / eb) : n;
  const int grid = cdiv(units, 256) < 148 * 8 ? cdiv(units, 256) : 148 * 8;
#define G2Q_RM(S)                                                                               \
  if (vec)                                                                                      \
    running_mean_kernel<S, true><<<grid, 256, 0, st>>>(cache, (const S*)grad, n, keep, inv,     \
                                                       first);                                  \
  else                                                                                          \
    running_mean_kernel<S, false><<<grid, 256, 0, st>>>(cache, (const S*)grad, n, keep, inv,    \
                                                        first);
  if (dtype == G2Q_DTYPE_BF16) {
    G2Q_RM(__nv_bfloat16)
  } else if (dtype == G2Q_DTYPE_F16) {
    G2Q_RM(__half)
  } else {
    G2Q_RM(float)
  }
#undef G2Q_RM
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

static int loss_args_ok(int kind, const void* x, const void* target, const int64_t* labels,
                        int dtype, int64_t ldx, int64_t ldt, int64_t rows, int64_t V) {
  if (kind != G2Q_LOSS_KL && kind != G2Q_LOSS_NLL && kind != G2Q_LOSS_MSE) return 0;
  if (elem_bytes(dtype) == 0 || rows < 0 || V <= 0 || ldx < V) return 0;
  if (rows > 0 && !x) return 0;
  if (kind == G2Q_LOSS_NLL) return rows == 0 || labels != nullptr;
  return (rows == 0 || target != nullptr) && ldt >= V;
}

extern "C" int g2q_block_loss_forward(int kind, float* loss, float* row_stats, const void* x,
                                      const void* target, const int64_t* labels, int dtype,
                                      int64_t ldx, int64_t ldt, int64_t rows, int64_t V,
                                      void* stream) {
  if (!loss || (rows > 0 && !row_stats)) return G2Q_ERR_INVALID_ARG;
  if (!loss_args_ok(kind, x, target, labels, dtype, ldx, ldt, rows, V))
    return G2Q_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  if (rows > 0) {
    const int eb = elem_bytes(dtype);
    const bool vec = vec_ok(x, ldx, V, eb) && (kind == G2Q_LOSS_NLL || vec_ok(target, ldt, V, eb));
    int rc;
    if (dtype == G2Q_DTYPE_BF16)
      rc = dispatch_loss_forward<__nv_bfloat16>(vec, kind, row_stats, x, ldx, target, ldt, labels,
                                                rows, V, st);
    else if (dtype == G2Q_DTYPE_F16)
      rc = dispatch_loss_forward<__half>(vec, kind, row_stats, x, ldx, target, ldt, labels, rows,
                                         V, st);
    else
      rc = dispatch_loss_forward<float>(vec, kind, row_stats, x, ldx, target, ldt, labels, rows,
                                        V, st);
    if (rc != G2Q_OK) return rc;
  }
  loss_sum_kernel<<<1, 1024, 0, st>>>(loss, row_stats, rows);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_block_loss_backward(int kind, void* grad, int64_t ldg, const float* row_stats,
                                       const void* x, const void* target, const int64_t* labels,
                                       int dtype, int64_t ldx, int64_t ldt,
                                       const float* grad_scale, int64_t rows, int64_t V,
                                       void* stream) {
  if (!loss_args_ok(kind, x, target, labels, dtype, ldx, ldt, rows, V) || ldg < V)
    return G2Q_ERR_INVALID_ARG;
  if (rows == 0) return G2Q_OK;
  if (!grad || !row_stats) return G2Q_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int eb = elem_bytes(dtype);
  const bool vec = vec_ok(x, ldx, V, eb) && vec_ok(grad, ldg, V, eb) &&
                   (kind == G2Q_LOSS_NLL || vec_ok(target, ldt, V, eb));
#define G2Q_LB(S)                                                                              \
  return vec ? launch_loss_backward<S, true>(kind, (S*)grad, ldg, row_stats, (const S*)x, ldx, \
                                             (const S*)target, ldt, labels, grad_scale, rows,  \
                                             V, st)                                            \
             : launch_loss_backward<S, false>(kind, (S*)grad, ldg, row_stats, (const S*)x,     \
                                              ldx, (const S*)target, ldt, labels, grad_scale,  \
                                              rows, V, st);
  if (dtype == G2Q_DTYPE_BF16) {
    G2Q_LB(__nv_bfloat16)
  } else if (dtype == G2Q_DTYPE_F16) {
    G2Q_LB(__half)
  } else {
    G2Q_LB(float)
  }
#undef G2Q_LB
  return G2Q_ERR_INVALID_ARG;
}
