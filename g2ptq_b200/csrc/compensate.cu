// Lazy-batch column compensation (GPTQ / G2PTQ / GPTAQ) and quantization
// parameters.
//
// Rows of W are independent in the compensation: every row walks the block's
// columns in order, quantizes, and pushes its error onto the remaining
// columns through the shared row U[c, c+1:].  The block of U (and of P for
// GPTAQ) sits in shared memory; the trailing update of the columns after the
// block is a GEMM (gemm_simt.cu or gemm_tc.cu).
#include <cuda_fp16.h>
#include <stdlib.h>

#include "gemm_simt.cuh"

namespace g2q {

constexpr int BLK = 128;  // maximum block width handled by one launch

struct BlockParams {
  float* W;  // row-major rows x ncols per batch entry, updated in place to Q
  long long ldw, w_bs;
  long long rows;
  int ncols;
  const float* hinv;
  long long ldh, h_bs;
  const float* scale;
  const float* zero;
  long long param_ld;
  const int* colmap;
  int maxq;
  int8_t* codes;  // row-major (ldq, q_bs)
  long long ldq, q_bs;
  float* err;  // optional fp32 error, column-major: (c * lde + r) + b * e_bs
  long long lde, e_bs;
  float* erra;  // optional trailing-update operand, column-major (ldea, ea_bs)
  long long ldea, ea_bs;
  // optional fp16 hi/lo copy of the trailing-update operand for the tensor
  // cores: column-major (ldea, eh_bs), each row scaled by a power of two that
  // puts its largest magnitude in [2^14, 2^15); the inverse scale of row r goes
  // to eh_scale[b * rows + r]
  __half* eh_hi;
  __half* eh_lo;
  float* eh_scale;
  long long eh_bs;
  const float* z;  // G2PTQ, row-major (ldz, z_bs)
  float* gh;
  long long ldz, z_bs;
  const float* p;  // GPTAQ, layout (ldh, h_bs)
  int dfact;       // G2PTQ distance factor (the traversal's blocksize)
  // G2PTQ --approx_grad: the traversal's input weights (layout of W) and the
  // shrink factor; wraw == nullptr leaves the standard path
  const float* wraw;
  float beta;
};

// Eight threads share a row and each keeps 16 of the block's columns in
// registers.  At column i the owner of i quantizes it and broadcasts its error
// to the other seven with a shuffle; every thread then applies that error to
// its own columns after i.  The per-column chain is one quantization, one
// shuffle and one update instead of a whole-row sweep per thread, and each
// element still receives its updates in column order, as in the reference.
// Errors are staged in shared memory and written out after the last column.
template <int QT_, int QROWS_>
struct BlockShape {
  static constexpr int QT = QT_;            // threads per row
  static constexpr int SEG = BLK / QT;      // block columns per thread
  static constexpr int LDU = QT * SEG;      // shared-memory row of the U (and P) block
  static constexpr int QROWS = QROWS_;      // rows per CTA
  static constexpr int LDE = BLK + 1;       // staged error row
  static constexpr int THREADS = QT * QROWS;
  static constexpr int smem_floats(int method) {
    return BLK * LDU * (method == G2Q_METHOD_GPTAQ ? 2 : 1) +
           QROWS * LDE * (method == G2Q_METHOD_G2PTQ ? 2 : 1);
  }
};
// Sixteen threads per row (eight columns each), sixteen rows per CTA: twice the
// warps of an eight-thread split for the same rows, which the latency-bound
// column loop needs to hide its dependent chains.  GPTQ's block (64 KB of U,
// 8 KB of errors, 80 registers) fits three CTAs on an SM, G2PTQ's two.
using BlockCfg = BlockShape<16, 16>;

// Offset of column k of thread t's segment in a U (or P) row.  The segment's
// two 4-column halves are swapped when bit 2 of t is set, so that the 16-byte
// loads of eight consecutive segments of one row cover all 32 banks (the same
// as padding each segment by four floats, without the padding's third more
// shared memory).
__device__ __forceinline__ int useg(int t, int k) {
  return t * BlockCfg::SEG + ((((k >> 2) ^ (t >> 2)) & 1) << 2) + (k & 3);
}

// rint(x / s) of the correctly rounded quotient, from a multiply by rs = 1 / s:
// x * rs lies within two units in the last place of the rounded quotient, so
// both round to the same integer unless a half-integer lies within a few
// units; only then the division itself is evaluated.
__device__ __forceinline__ float rint_quot(float x, float s, float rs) {
  const float q0 = x * rs;
  const float h = floorf(q0) + 0.5f;
  if (fabsf(q0 - h) <= fabsf(q0) * 0x1p-20f) return rintf(x / s);
  return rintf(q0);
}

// num / d rounded to nearest from rd = 1 / d: the product num * rd and one
// residual correction, r = num - d q (exact in an fma), q + r rd (Markstein's
// correction step for division with a correctly rounded reciprocal).
__device__ __forceinline__ float div_rn(float num, float d, float rd) {
  const float q = num * rd;
  const float r = fmaf(-q, d, num);
  return fmaf(r, rd, q);
}

template <int METHOD>
__global__ void __launch_bounds__(BlockCfg::THREADS, METHOD == G2Q_METHOD_GPTQ ? 3 : 2)
    block_kernel(BlockParams P) {
  constexpr int QT = BlockCfg::QT, SEG = BlockCfg::SEG;
  constexpr int LDU = BlockCfg::LDU, QROWS = BlockCfg::QROWS, LDE = BlockCfg::LDE;
  extern __shared__ __align__(16) float smem[];
  float* Us = smem;              // [BLK][LDU], segment halves swizzled (useg)
  float* Ps = Us + BLK * LDU;    // GPTAQ P block, same layout
  float* Es = smem + BLK * LDU * (METHOD == G2Q_METHOD_GPTAQ ? 2 : 1);  // [QROWS][LDE] errors
  float* EAs = Es + QROWS * LDE;  // G2PTQ trailing-update errors
  const int b = blockIdx.y;
  const int tid = threadIdx.x;
  const int t = tid & (QT - 1);
  const int lane = tid & 31;
  const int src0 = lane & ~(QT - 1);  // lane holding segment 0 of this row
  const int rl = tid / QT;  // row within the CTA
  const long long r = (long long)blockIdx.x * QROWS + rl;
  const int nc = P.ncols;
  const bool active = r < P.rows;
  const long long rr = active ? r : 0;

  const float* hb = P.hinv + (long long)b * P.h_bs;
  const float* pb = (METHOD == G2Q_METHOD_GPTAQ) ? P.p + (long long)b * P.h_bs : nullptr;
  // 16-byte loads, many in flight, when the block is full width and aligned
  const bool vec = (nc == BLK) && ((P.ldh & 3) == 0) && (((uintptr_t)hb & 15) == 0) &&
                   (METHOD != G2Q_METHOD_GPTAQ || (((uintptr_t)pb & 15) == 0));
  if (vec) {
#pragma unroll 8
    for (int q = tid; q < BLK * BLK / 4; q += QT * QROWS) {
      const int i = q / (BLK / 4), j = (q % (BLK / 4)) * 4;
      const int o = i * LDU + useg(j / SEG, j % SEG);
      *reinterpret_cast<float4*>(&Us[o]) = *reinterpret_cast<const float4*>(hb + i * P.ldh + j);
      if (METHOD == G2Q_METHOD_GPTAQ)
        *reinterpret_cast<float4*>(&Ps[o]) =
            *reinterpret_cast<const float4*>(pb + i * P.ldh + j);
    }
  } else {
#pragma unroll 4
    for (int idx = tid; idx < BLK * BLK; idx += QT * QROWS) {
      const int i = idx / BLK, j = idx % BLK;
      const int o = i * LDU + useg(j / SEG, j % SEG);
      const bool in = i < nc && j < nc;
      Us[o] = in ? hb[i * P.ldh + j] : 0.f;
      if (METHOD == G2Q_METHOD_GPTAQ) Ps[o] = in ? pb[i * P.ldh + j] : 0.f;
    }
  }

  // this thread's 32 columns of W (and of gh / z for G2PTQ) and their parameters
  float wv[SEG], gv[SEG], xv[SEG], sv[SEG], zv[SEG], rv[SEG];
  float* wrow = P.W + (long long)b * P.w_bs + rr * P.ldw + t * SEG;
  float* grow = (METHOD == G2Q_METHOD_G2PTQ)
                    ? P.gh + (long long)b * P.z_bs + rr * P.ldz + t * SEG : nullptr;
  // --approx_grad (G2PTQ): raw weights of this thread's columns
  const bool approx = (METHOD == G2Q_METHOD_G2PTQ) && P.wraw != nullptr;
  const float* rawrow = approx ? P.wraw + (long long)b * P.w_bs + rr * P.ldw + t * SEG : nullptr;
  const float* zrow = (METHOD == G2Q_METHOD_G2PTQ)
                          ? P.z + (long long)b * P.z_bs + rr * P.ldz + t * SEG : nullptr;
  const long long prow = ((long long)b * P.rows + rr) * P.param_ld;
#pragma unroll
  for (int k = 0; k < SEG; ++k) {
    const int col = t * SEG + k;
    const bool in = active && col < nc;
    const int pc = in ? P.colmap[col] : 0;
    wv[k] = in ? wrow[k] : 0.f;
    sv[k] = in ? P.scale[prow + pc] : 1.f;
    zv[k] = in ? P.zero[prow + pc] : 0.f;
    gv[k] = (METHOD == G2Q_METHOD_G2PTQ && in) ? grow[k] : 0.f;
    xv[k] = (METHOD == G2Q_METHOD_G2PTQ && in) ? zrow[k] : 0.f;
    rv[k] = (approx && in) ? rawrow[k] : 0.f;
  }
  __syncthreads();

  // per-column reciprocals (off the column chain): 1 / scale, U's diagonal and
  // its reciprocal for the columns this thread owns
  float rsv[SEG], dv[SEG], rdv[SEG];
#pragma unroll
  for (int k = 0; k < SEG; ++k) {
    const int col = t * SEG + k;
    rsv[k] = 1.f / sv[k];
    dv[k] = col < nc ? Us[col * LDU + useg(t, k)] : 1.f;
    rdv[k] = 1.f / dv[k];
  }

  uint32_t cw[SEG / 4];
#pragma unroll
  for (int k = 0; k < SEG / 4; ++k) cw[k] = 0u;
  const float qlo = -(float)(P.maxq + 1), qhi = (float)P.maxq;

  // The error of column i reaches the other threads one column late: at column
  // i + 1 every thread first quantizes (the owner), then applies column i's
  // shuffled error to its own later columns.  The owner carries its next
  // column's value in `wn` (and `gn`), updated with its own error directly, so
  // the chain from one column to the next holds no shuffle and no shared
  // memory load.  Every element still receives its updates in column order.
  float e_prev = 0.f, aux_prev = 0.f;
#pragma unroll 1
  for (int tw = 0; tw < QT; ++tw) {
    if (tw * SEG >= nc) break;
    const bool after = t >= tw;  // the owner's columns after the current one
    const bool later = t > tw;   // every column of the threads after the owner
    float wn = wv[0], gn = gv[0];
    // --approx_grad: the previous segment's last column of this block pulls
    // this segment's first column toward its raw value after its update
    // (the products rounded apart, as the reference's tensor expression)
    if (approx && tw > 0) wn = __fsub_rn(wn, __fmul_rn(__fsub_rn(wn, rv[0]), P.beta));
    int klast = 0;
#pragma unroll
    for (int k = 0; k < SEG; ++k) {
      const int i = tw * SEG + k;
      if (i >= nc) break;
      klast = k;
      float e = 0.f, aux = 0.f;
      if (t == tw) {
        const float s = sv[k];
        const float zz = zv[k];
        const float wc = wn;
        float q = rint_quot(wc, s, rsv[k]) + zz;
        q = fminf(fmaxf(q, qlo), qhi);
        const float qv = s * (q - zz);
        if (METHOD == G2Q_METHOD_G2PTQ) {
          float num = wc - qv - gn;
          // --approx_grad: the error also shrinks toward the raw weight
          if (approx) num = __fsub_rn(num, __fmul_rn(__fsub_rn(wc, rv[k]), P.beta));
          e = div_rn(num, dv[k], rdv[k]);
          gv[k] = gn;
        } else {
          e = div_rn(wc - qv, dv[k], rdv[k]);
        }
        aux = (METHOD == G2Q_METHOD_G2PTQ) ? xv[k] : wc;
        wv[k] = qv;
        cw[k / 4] |= ((uint32_t)(int)q & 0xffu) << (8 * (k % 4));
        Es[rl * LDE + i] = e;
        if (METHOD == G2Q_METHOD_G2PTQ)
          EAs[rl * LDE + i] = e - xv[k] * (float)(P.dfact - 1 - i);
      }
      const float e_sh = __shfl_sync(0xffffffffu, e, src0 + tw);
      const float aux_sh =
          (METHOD != G2Q_METHOD_GPTQ) ? __shfl_sync(0xffffffffu, aux, src0 + tw) : 0.f;
      // column i - 1's update of this thread's columns after i (the owner's
      // column i received it through wn)
      if (k > 0) {
        const float* urow = Us + (i - 1) * LDU;
        const float* prow_s = Ps + (i - 1) * LDU;
#pragma unroll
        for (int j4 = 0; j4 < SEG; j4 += 4) {
          const float4 u4 = *reinterpret_cast<const float4*>(urow + useg(t, j4));
          const float uu[4] = {u4.x, u4.y, u4.z, u4.w};
          float pp[4] = {0.f, 0.f, 0.f, 0.f};
          if (METHOD == G2Q_METHOD_GPTAQ) {
            const float4 p4 = *reinterpret_cast<const float4*>(prow_s + useg(t, j4));
            pp[0] = p4.x; pp[1] = p4.y; pp[2] = p4.z; pp[3] = p4.w;
          }
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const int j = j4 + m;
            if (j > k ? after : later) {
              if (METHOD == G2Q_METHOD_G2PTQ) {
                wv[j] = fmaf(-e_prev, uu[m], wv[j] - gv[j]);
                gv[j] = fmaf(-aux_prev, uu[m], gv[j]);
              } else if (METHOD == G2Q_METHOD_GPTAQ) {
                wv[j] = fmaf(pp[m], aux_prev, fmaf(-e_prev, uu[m], wv[j]));
              } else {
                wv[j] = fmaf(-e_prev, uu[m], wv[j]);
              }
            }
          }
        }
      }
      // the owner's next column with column i's own update
      if (k + 1 < SEG) {
        const float u1 = Us[i * LDU + useg(tw, k + 1)];
        if (METHOD == G2Q_METHOD_G2PTQ) {
          wn = fmaf(-e, u1, wv[k + 1] - gv[k + 1]);
          if (approx) wn = __fsub_rn(wn, __fmul_rn(__fsub_rn(wn, rv[k + 1]), P.beta));
          gn = fmaf(-aux, u1, gv[k + 1]);
        } else if (METHOD == G2Q_METHOD_GPTAQ) {
          wn = fmaf(Ps[i * LDU + useg(tw, k + 1)], aux, fmaf(-e, u1, wv[k + 1]));
        } else {
          wn = fmaf(-e, u1, wv[k + 1]);
        }
      }
      e_prev = e_sh;
      aux_prev = aux_sh;
    }
    // the segment's last column updates every column of the threads after it
    if (later) {
      const int i = tw * SEG + klast;
      const float* urow = Us + i * LDU;
      const float* prow_s = Ps + i * LDU;
#pragma unroll
      for (int j4 = 0; j4 < SEG; j4 += 4) {
        const float4 u4 = *reinterpret_cast<const float4*>(urow + useg(t, j4));
        const float uu[4] = {u4.x, u4.y, u4.z, u4.w};
        float pp[4] = {0.f, 0.f, 0.f, 0.f};
        if (METHOD == G2Q_METHOD_GPTAQ) {
          const float4 p4 = *reinterpret_cast<const float4*>(prow_s + useg(t, j4));
          pp[0] = p4.x; pp[1] = p4.y; pp[2] = p4.z; pp[3] = p4.w;
        }
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int j = j4 + m;
          if (METHOD == G2Q_METHOD_G2PTQ) {
            wv[j] = fmaf(-e_prev, uu[m], wv[j] - gv[j]);
            gv[j] = fmaf(-aux_prev, uu[m], gv[j]);
          } else if (METHOD == G2Q_METHOD_GPTAQ) {
            wv[j] = fmaf(pp[m], aux_prev, fmaf(-e_prev, uu[m], wv[j]));
          } else {
            wv[j] = fmaf(-e_prev, uu[m], wv[j]);
          }
        }
      }
    }
  }

  if (active) {
    int8_t* qrow = P.codes ? P.codes + (long long)b * P.q_bs + r * P.ldq + t * SEG : nullptr;
#pragma unroll
    for (int k = 0; k < SEG; ++k) {
      if (t * SEG + k >= nc) break;
      wrow[k] = wv[k];
      if (qrow) qrow[k] = (int8_t)((cw[k / 4] >> (8 * (k % 4))) & 0xffu);
      if (METHOD == G2Q_METHOD_G2PTQ) grow[k] = gv[k];
    }
  }
  // errors, column-major: consecutive threads take consecutive rows of a column
  __syncthreads();
  const long long row0 = (long long)blockIdx.x * QROWS;
  // fp16 split of the trailing-update operand: the QT threads of a row find
  // its largest magnitude over the block's columns
  __shared__ float rowf[QROWS];
  if (P.eh_hi) {
    const float* src = (METHOD == G2Q_METHOD_G2PTQ) ? EAs : Es;
    float m = 0.f;
    for (int i = t; i < nc; i += QT) m = fmaxf(m, fabsf(src[rl * LDE + i]));
#pragma unroll
    for (int o = QT / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (t == 0) {
      float f = 1.f, v = 1.f;
      if (m > 0.f && m <= 3.0e38f) {
        int e;
        frexpf(m, &e);
        e = e < -100 ? -100 : e;
        f = ldexpf(1.f, 15 - e);
        v = ldexpf(1.f, e - 15);
      }
      rowf[rl] = f;
      if (active) P.eh_scale[(long long)b * P.rows + r] = v;
    }
    __syncthreads();
  }
  for (int idx = tid; idx < QROWS * nc; idx += QT * QROWS) {
    const int i = idx / QROWS, q = idx % QROWS;
    const long long rq = row0 + q;
    if (rq >= P.rows) continue;
    const float e = Es[q * LDE + i];
    const float ea = (METHOD == G2Q_METHOD_G2PTQ) ? EAs[q * LDE + i] : e;
    if (P.err) P.err[(long long)b * P.e_bs + (long long)i * P.lde + rq] = e;
    const long long ao = (long long)b * P.ea_bs + (long long)i * P.ldea + rq;
    if (P.erra) P.erra[ao] = ea;
    if (P.eh_hi) {
      const float v = ea * rowf[q];
      const __half h = __float2half_rn(v);
      const long long ho = (long long)b * P.eh_bs + (long long)i * P.ldea + rq;
      P.eh_hi[ho] = h;
      P.eh_lo[ho] = __float2half_rn(v - __half2float(h));
    }
  }
}

static size_t block_smem(int method) {
  return (size_t)BlockCfg::smem_floats(method) * sizeof(float);
}

template <int METHOD>
static int launch_block_t(const BlockParams& P, long long batch, cudaStream_t st) {
  static int attr_done[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return G2Q_ERR_CUDA;
  const size_t smem = block_smem(METHOD);
  if (dev >= 64 || !attr_done[dev]) {
    if (cudaFuncSetAttribute(block_kernel<METHOD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess ||
        cudaFuncSetAttribute(block_kernel<METHOD>,
                             cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      return G2Q_ERR_CUDA;
    if (dev < 64) attr_done[dev] = 1;
  }
  dim3 grid(cdiv(P.rows, BlockCfg::QROWS), (unsigned)batch);
  if (grid.y > 65535u) return G2Q_ERR_INVALID_ARG;
  block_kernel<METHOD><<<grid, BlockCfg::THREADS, smem, st>>>(P);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

int launch_block(int method, const BlockParams& P, long long batch, cudaStream_t st) {
  if (P.rows <= 0 || batch <= 0 || P.ncols <= 0) return G2Q_OK;
  switch (method) {
    case G2Q_METHOD_GPTQ: return launch_block_t<G2Q_METHOD_GPTQ>(P, batch, st);
    case G2Q_METHOD_G2PTQ: return launch_block_t<G2Q_METHOD_G2PTQ>(P, batch, st);
    case G2Q_METHOD_GPTAQ: return launch_block_t<G2Q_METHOD_GPTAQ>(P, batch, st);
  }
  return G2Q_ERR_INVALID_ARG;
}

// ---------------------------------------------------------------------------
// Quantization parameters: one warp per (row, group).
// ---------------------------------------------------------------------------

__device__ __forceinline__ void params_from_range(float xmin, float xmax, int bits, int sym,
                                                  float* s_out, float* z_out) {
  const int maxq = (1 << (bits - 1)) - 1;
  const int minq = -(maxq + 1);
  const float bit_range = (float)(maxq - minq);
  xmin = fminf(xmin, 0.f);
  xmax = fmaxf(xmax, 0.f);
  float s, z;
  if (sym) {
    s = fmaxf(fabsf(xmin), xmax) / (bit_range / 2.f);
    z = 0.f;
  } else {
    s = (xmax - xmin) / bit_range;
    z = rintf((float)minq - xmin / s);
    z = fminf(fmaxf(z, (float)minq), (float)maxq);
  }
  *s_out = s;
  *z_out = rintf(z);
}

__global__ void find_params_kernel(float* scale, float* zero, long long param_ld,
                                   const float* W, long long rows, long long cols,
                                   long long ldw, int bits, int sym, int* status,
                                   long long first_start, int groupsize, long long C) {
  const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long r = warp;
  const int gi = blockIdx.y;
  if (r >= rows) return;
  long long c0 = 0, nc = cols;
  long long pc = 0;
  if (first_start >= 0) {
    c0 = first_start + (long long)gi * groupsize;
    nc = (C - c0) < groupsize ? (C - c0) : groupsize;
    pc = c0 / groupsize;
  }
  const float* x = W + r * ldw + c0;
  float mn = INFINITY, mx = -INFINITY;
  for (long long c = lane; c < nc; c += 32) {
    const float v = x[c];
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (lane == 0) {
    float s, z;
    params_from_range(mn, mx, bits, sym, &s, &z);
    scale[r * param_ld + pc] = s;
    zero[r * param_ld + pc] = z;
    if (!(s > 0.f)) record_error(status, G2Q_ERR_BAD_SCALE);
  }
}

// WeightQuantizer.find_params with the clip search (quant_utils.py:406-425):
// the range [xmin, xmax] of a (row, group) is shrunk on a grid,
// xmin * (1 - i / grid) and xmax * (1 - j / grid) for i, j < maxshrink * grid,
// and the first pair with the smallest error is kept; the error is
// sum |fq - x|^norm, or sum (fq - x)^2 h_c with the Hessian diagonal (hclip).
// One warp per (row, group); the group's values sit in registers (8 per lane)
// when it has at most 256 columns, else they are re-read for every candidate.
// For symmetric quantizers the scale of pair (i, j) is max(a_i, b_j) / half,
// so only the 2n distinct values are evaluated and the (i, j) walk then picks
// from them in the reference's order (equal values give equal errors).
constexpr int CLIP_EPL = 8;
constexpr int CLIP_MAXN = 64;

struct ClipArgs {
  int grid;
  float maxshrink;
  float norm;
  const float* hdiag;  // optional, [row blocks][hdiag_ld], column c of the group at c
  long long hdiag_ld;
  long long rows_per_block;
};

__device__ __forceinline__ float clip_err(const float (&xv)[CLIP_EPL], const float (&hv)[CLIP_EPL],
                                          const float* x, const float* hd, int nc, int lane,
                                          bool in_regs, float s, float z, float qlo, float qhi,
                                          float norm) {
  float e = 0.f;
  if (in_regs) {
#pragma unroll
    for (int k = 0; k < CLIP_EPL; ++k) {
      const int c = lane + 32 * k;
      if (c >= nc) break;
      const float q = fminf(fmaxf(rintf(xv[k] / s) + z, qlo), qhi);
      const float d = s * (q - z) - xv[k];
      e += hd ? (d * d) * hv[k] : powf(fabsf(d), norm);
    }
  } else {
    for (int c = lane; c < nc; c += 32) {
      const float q = fminf(fmaxf(rintf(x[c] / s) + z, qlo), qhi);
      const float d = s * (q - z) - x[c];
      e += hd ? (d * d) * hd[c] : powf(fabsf(d), norm);
    }
  }
  for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
  return e;
}

__global__ void find_params_clip_kernel(float* scale, float* zero, long long param_ld,
                                        const float* W, long long rows, long long cols,
                                        long long ldw, int bits, int sym, int* status,
                                        long long first_start, int groupsize, long long C,
                                        ClipArgs ca) {
  __shared__ float ebuf[8][2 * CLIP_MAXN];
  const int wib = threadIdx.x >> 5;
  const long long r = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int gi = blockIdx.y;
  if (r >= rows) return;  // whole warps leave together
  long long c0 = 0, ncl = cols;
  long long pc = 0;
  if (first_start >= 0) {
    c0 = first_start + (long long)gi * groupsize;
    ncl = (C - c0) < groupsize ? (C - c0) : groupsize;
    pc = c0 / groupsize;
  }
  const int nc = (int)ncl;
  const float* x = W + r * ldw + c0;
  const float* hd = ca.hdiag ? ca.hdiag + (r / ca.rows_per_block) * ca.hdiag_ld + c0 : nullptr;
  const bool in_regs = nc <= 32 * CLIP_EPL;
  float xv[CLIP_EPL], hv[CLIP_EPL];
  float mn = INFINITY, mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < CLIP_EPL; ++k) {
    const int c = lane + 32 * k;
    xv[k] = (in_regs && c < nc) ? x[c] : 0.f;
    hv[k] = (in_regs && hd && c < nc) ? hd[c] : 0.f;
  }
  for (int c = lane; c < nc; c += 32) {
    const float v = x[c];
    mn = fminf(mn, v);
    mx = fmaxf(mx, v);
  }
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const int maxq = (1 << (bits - 1)) - 1;
  const int minq = -(maxq + 1);
  const float bit_range = (float)(maxq - minq);
  const float qlo = (float)minq, qhi = (float)maxq;
  const float xmin = fminf(mn, 0.f), xmax = fmaxf(mx, 0.f);
  float s, z;
  params_from_range(xmin, xmax, bits, sym, &s, &z);
  float best = INFINITY;
  const int n = (int)((double)ca.maxshrink * ca.grid);
  if (sym && n <= CLIP_MAXN) {
    float* ea = ebuf[wib];
    float* eb = ea + CLIP_MAXN;
    for (int i = 0; i < n; ++i) {
      const float f = (float)(1.0 - (double)i / ca.grid);
      const float a = fabsf(f * xmin), b = f * xmax;
      const float ia = clip_err(xv, hv, x, hd, nc, lane, in_regs, a / (bit_range / 2.f), 0.f,
                                qlo, qhi, ca.norm);
      const float ib = clip_err(xv, hv, x, hd, nc, lane, in_regs, b / (bit_range / 2.f), 0.f,
                                qlo, qhi, ca.norm);
      if (lane == 0) {
        ea[i] = ia;
        eb[i] = ib;
      }
    }
    __syncwarp();
    for (int i = 0; i < n; ++i) {
      const float a = fabsf((float)(1.0 - (double)i / ca.grid) * xmin);
      for (int j = 0; j < n; ++j) {
        const float b = (float)(1.0 - (double)j / ca.grid) * xmax;
        const float e = a >= b ? ea[i] : eb[j];
        if (e < best) {
          best = e;
          s = fmaxf(a, b) / (bit_range / 2.f);
          z = 0.f;
        }
      }
    }
  } else {
    for (int i = 0; i < n; ++i) {
      const float xmin1 = (float)(1.0 - (double)i / ca.grid) * xmin;
      for (int j = 0; j < n; ++j) {
        const float xmax1 = (float)(1.0 - (double)j / ca.grid) * xmax;
        float s1, z1;
        if (sym) {
          s1 = fmaxf(fabsf(xmin1), xmax1) / (bit_range / 2.f);
          z1 = 0.f;
        } else {
          s1 = (xmax1 - xmin1) / bit_range;
          z1 = fminf(fmaxf(rintf((float)minq - xmin1 / s1), qlo), qhi);
        }
        const float e = clip_err(xv, hv, x, hd, nc, lane, in_regs, s1, z1, qlo, qhi, ca.norm);
        if (e < best) {
          best = e;
          s = s1;
          z = z1;
        }
      }
    }
  }
  if (lane == 0) {
    scale[r * param_ld + pc] = s;
    zero[r * param_ld + pc] = rintf(z);
    if (!(s > 0.f)) record_error(status, G2Q_ERR_BAD_SCALE);
  }
}

static int launch_find_params(float* scale, float* zero, long long param_ld, const float* W,
                              long long rows, long long cols, long long ldw, int bits, int sym,
                              int* status, long long first_start, int ngs, int groupsize,
                              long long C, const g2q_clip_t* clip, cudaStream_t st) {
  if (rows <= 0) return G2Q_OK;
  const int warps_per_block = 8;
  dim3 grid(cdiv(rows, warps_per_block), first_start >= 0 ? ngs : 1);
  if (grid.y > 65535u) return G2Q_ERR_INVALID_ARG;
  if (clip) {
    ClipArgs ca{clip->grid, clip->maxshrink, clip->norm, clip->hdiag, clip->hdiag_ld,
                clip->rows_per_block > 0 ? clip->rows_per_block : rows};
    find_params_clip_kernel<<<grid, 32 * warps_per_block, 0, st>>>(
        scale, zero, param_ld, W, rows, cols, ldw, bits, sym, status, first_start, groupsize, C,
        ca);
  } else {
    find_params_kernel<<<grid, 32 * warps_per_block, 0, st>>>(
        scale, zero, param_ld, W, rows, cols, ldw, bits, sym, status, first_start, groupsize, C);
  }
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

static bool clip_ok(const g2q_clip_t* clip) {
  return !clip || (clip->grid > 0 && clip->maxshrink >= 0.f && clip->maxshrink < 1.f &&
                   (!clip->hdiag || (clip->hdiag_ld >= 0 && clip->rows_per_block > 0)));
}

__global__ void fake_quantize_kernel(float* out, long long ldo, int8_t* codes, long long ldq,
                                     const float* W, long long ldw, long long rows,
                                     long long cols, const float* scale, const float* zero,
                                     long long param_ld, const int* colmap, int maxq) {
  const long long n = rows * cols;
  const float qlo = -(float)(maxq + 1), qhi = (float)maxq;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long r = idx / cols, c = idx - r * cols;
    const long long pi = r * param_ld + (colmap ? colmap[c] : 0);
    const float s = scale[pi], z = zero[pi];
    const float w = W[r * ldw + c];
    float q = rintf(w / s) + z;
    q = fminf(fmaxf(q, qlo), qhi);
    if (out) out[r * ldo + c] = s * (q - z);
    if (codes) codes[r * ldq + c] = (int8_t)(int)q;
  }
}

// W[b][:, c] -= f * G[b][:, c] over a column range (G2PTQ gradient term); row r
// over the grid's y loop, columns over the x threads.
__global__ void sub_scaled_kernel(float* W, const float* G, long long nl_rows, long long C,
                                  long long c0, float f) {
  for (long long r = blockIdx.y; r < nl_rows; r += gridDim.y) {
    float* w = W + r * C;
    const float* g = G + r * C;
    for (long long c = c0 + (long long)blockIdx.x * blockDim.x + threadIdx.x; c < C;
         c += (long long)gridDim.x * blockDim.x)
      w[c] -= f * g[c];
  }
}

static int grid_for(long long n) {
  long long b = (n + 255) / 256;
  if (b > 148 * 64) b = 148 * 64;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace g2q

using namespace g2q;

extern "C" int g2q_find_params(float* scale, float* zero, int64_t param_ld, const float* W,
                               int64_t rows, int64_t cols, int64_t ldw, int bits, int sym,
                               int* status, void* stream) {
  if (!scale || !zero || !W || rows < 0 || cols <= 0 || ldw < cols || bits < 1 || bits > 16)
    return G2Q_ERR_INVALID_ARG;
  return launch_find_params(scale, zero, param_ld, W, rows, cols, ldw, bits, sym, status,
                            -1, 1, 0, cols, nullptr, (cudaStream_t)stream);
}

extern "C" int g2q_find_params_groups(float* scale, float* zero, int64_t param_ld,
                                      const float* W, int64_t rows, int64_t C, int64_t ldw,
                                      int bits, int sym, int64_t first, int count, int groupsize,
                                      int* status, void* stream) {
  if (!scale || !zero || !W || rows < 0 || C <= 0 || ldw < C || bits < 1 || bits > 16 ||
      groupsize <= 0 || count < 0 || first < 0 || first % groupsize != 0 ||
      (count > 0 && first + (int64_t)(count - 1) * groupsize >= C) ||
      param_ld < (first / groupsize) + count)
    return G2Q_ERR_INVALID_ARG;
  if (count == 0) return G2Q_OK;
  return launch_find_params(scale, zero, param_ld, W, rows, 0, ldw, bits, sym, status, first,
                            count, groupsize, C, nullptr, (cudaStream_t)stream);
}

extern "C" int g2q_find_params_clip(float* scale, float* zero, int64_t param_ld, const float* W,
                                    int64_t rows, int64_t cols, int64_t ldw, int bits, int sym,
                                    const g2q_clip_t* clip, int* status, void* stream) {
  if (!scale || !zero || !W || !clip || rows < 0 || cols <= 0 || ldw < cols || bits < 1 ||
      bits > 16 || !clip_ok(clip))
    return G2Q_ERR_INVALID_ARG;
  return launch_find_params(scale, zero, param_ld, W, rows, cols, ldw, bits, sym, status,
                            -1, 1, 0, cols, clip, (cudaStream_t)stream);
}

extern "C" int g2q_fake_quantize(float* out, int64_t ldo, int8_t* codes, int64_t ldq,
                                 const float* W, int64_t ldw, int64_t rows, int64_t cols,
                                 const float* scale, const float* zero, int64_t param_ld,
                                 const int* colmap, int maxq, void* stream) {
  if (!W || !scale || !zero || rows < 0 || cols < 0) return G2Q_ERR_INVALID_ARG;
  if (rows * cols == 0) return G2Q_OK;
  fake_quantize_kernel<<<grid_for(rows * cols), 256, 0, (cudaStream_t)stream>>>(
      out, ldo, codes, ldq, W, ldw, rows, cols, scale, zero, param_ld, colmap, maxq);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

extern "C" int g2q_compensate_block(int method, float* W, int64_t ldw, int64_t w_bstride,
                                    int64_t batch, int64_t rows, int64_t ncols,
                                    const float* hinv, int64_t ldh, int64_t h_bstride,
                                    const float* scale, const float* zero, int64_t param_ld,
                                    const int* colmap, int maxq, int8_t* codes, float* err,
                                    const float* z, float* ghinv, const float* p,
                                    const float* wraw, float approx_beta, void* stream) {
  if (!W || !hinv || !scale || !zero || !colmap || ncols <= 0 || ncols > BLK || rows < 0 ||
      batch < 0 || maxq < 0)
    return G2Q_ERR_INVALID_ARG;
  if ((wraw != nullptr) != (approx_beta != 0.f) || (wraw && method != G2Q_METHOD_G2PTQ))
    return G2Q_ERR_INVALID_ARG;
  if (method == G2Q_METHOD_G2PTQ && (!z || !ghinv)) return G2Q_ERR_INVALID_ARG;
  if (method == G2Q_METHOD_GPTAQ && !p) return G2Q_ERR_INVALID_ARG;
  BlockParams P{};
  P.W = W; P.ldw = ldw; P.w_bs = w_bstride;
  P.rows = rows; P.ncols = (int)ncols;
  P.hinv = hinv; P.ldh = ldh; P.h_bs = h_bstride;
  P.scale = scale; P.zero = zero; P.param_ld = param_ld; P.colmap = colmap; P.maxq = maxq;
  P.codes = codes; P.ldq = ldw; P.q_bs = w_bstride;
  P.err = err; P.lde = rows; P.e_bs = ncols * rows;
  P.z = z; P.gh = ghinv; P.ldz = ldw; P.z_bs = w_bstride;
  P.p = p;
  P.dfact = (int)ncols;
  P.wraw = wraw;
  P.beta = approx_beta;
  return launch_block(method, P, batch, (cudaStream_t)stream);
}


namespace g2q {
size_t gemm_tc_workspace_bytes(long long M, long long N, long long K, long long batch_a,
                               long long batch_b);
int gemm_tc_f32(float* C, long long ldc, long long sC, const float* A, long long lda,
                long long sA, bool ta, const float* B, long long ldb, long long sB, bool tb,
                long long M, long long N, long long K, long long batch, float alpha, float beta,
                int mask, void* workspace, size_t workspace_bytes, int* status, cudaStream_t st);
}  // namespace g2q

// Deferred trailing update of GPTQ: blocks are grouped SUPER at a time; after
// each block only the rest of its group is updated (K = one block), the
// columns after the group once per group (K = SUPER blocks), so the HBM passes
// over W's far columns drop SUPER-fold.  The workspace always has room for
// SUPER blocks; the group size used is G2PTQ_B200_DEFER_BLOCKS (1 to SUPER,
// default 1: measured, the K = 512 updates on the long-K kernel cost more than
// the passes they save).
constexpr int SUPER = 4;

static int defer_blocks() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("G2PTQ_B200_DEFER_BLOCKS");
    v = e ? atoi(e) : 1;
    if (v < 1) v = 1;
    if (v > SUPER) v = SUPER;
  }
  return v;
}

namespace g2q {
int split2h_strips(const float* src, long long lds, long long n, int K, __half* hi, __half* lo,
                   long long ldd, float* scale, int transpose, int ny, long long src_by,
                   long long dst_by, long long sc_by, int nz, long long src_bz,
                   long long dst_bz, long long sc_bz, cudaStream_t st);
int tc_update_f16(float* D, long long ldd, long long d_bs, long long M, long long N, int K,
                  long long batch, __half* const* a2, long long lda, long long a_outer,
                  long long ka_batch, long long ka0, const float* sa, long long sa_bs,
                  __half* const* b2, long long ldb, long long b_inner, long long b_outer,
                  long long kb_batch, long long kb0, long long nb0, const float* sb,
                  long long sb_bs, float beta, int* status, cudaStream_t st);
}  // namespace g2q

// Layout of the workspace (each part 256-byte aligned): the errors of up to
// SUPER blocks (fp32, column-major per block), the fp32-accurate GEMM's own
// operand splits (far updates, and every update where the fused path does not
// apply), and for GPTQ / G2PTQ at precision 1 the fused path's operands: the
// error block's fp16 hi/lo pair and row scales, U cut into 128-row (at most)
// strips as fp16 hi/lo pairs with a scale per strip and column, and for G2PTQ
// Z's block columns transposed the same way with a scale per block and row.
extern "C" size_t g2q_compensate_workspace_bytes(int method, int64_t nl, int64_t rows,
                                                 int64_t C, int precision) {
  const size_t S = (method == G2Q_METHOD_GPTQ && precision == 1) ? SUPER : 1;
  size_t b = (size_t)nl * rows * BLK * S * sizeof(float) + 256;
  if (precision == 1) {
    b += g2q::gemm_tc_workspace_bytes(rows, C, (long long)S * BLK, nl, nl) + 256;
    if (method != G2Q_METHOD_GPTAQ) {
      const size_t strips = (size_t)(C / 64 + 1);  // blocks of >= 64 columns
      b += 2 * ((size_t)nl * BLK * rows * sizeof(__half) + 256);
      b += (size_t)nl * rows * sizeof(float) + 256;
      b += 2 * ((size_t)nl * (C + BLK) * C * sizeof(__half) + 256);
      b += (size_t)nl * strips * C * sizeof(float) + 256;
      if (method == G2Q_METHOD_G2PTQ) {
        b += 2 * ((size_t)nl * (C + BLK) * rows * sizeof(__half) + 256);
        b += (size_t)nl * strips * rows * sizeof(float) + 256;
      }
    }
  }
  return b;
}

static char* align_up(char* p, size_t a) {
  return (char*)(((uintptr_t)p + a - 1) / a * a);
}

extern "C" int g2q_compensate(int method, float* W, int64_t nl, int64_t rows, int64_t C,
                              const float* U, float* scale, float* zero, int64_t ngroups,
                              const int* colgroup, int dynamic_groups, int groupsize, int bits,
                              int sym, int blocksize, int8_t* codes, const float* z, float* gh,
                              const float* p, const float* wraw, float approx_beta,
                              const g2q_clip_t* clip, int precision,
                              void* workspace, size_t workspace_bytes, int* status,
                              void* stream) {
  if (!W || !U || !scale || !zero || !colgroup || !codes || nl <= 0 || rows <= 0 || C <= 0 ||
      blocksize <= 0 || blocksize > BLK || bits < 1 || bits > 8 || !workspace)
    return G2Q_ERR_INVALID_ARG;
  if (dynamic_groups && groupsize <= 0) return G2Q_ERR_INVALID_ARG;
  if (!clip_ok(clip)) return G2Q_ERR_INVALID_ARG;
  if (method == G2Q_METHOD_G2PTQ && (!z || !gh)) return G2Q_ERR_INVALID_ARG;
  if (method == G2Q_METHOD_GPTAQ && !p) return G2Q_ERR_INVALID_ARG;
  if ((wraw != nullptr) != (approx_beta != 0.f) || (wraw && method != G2Q_METHOD_G2PTQ))
    return G2Q_ERR_INVALID_ARG;
  if (precision != 0 && precision != 1) return G2Q_ERR_INVALID_ARG;
  if (workspace_bytes < g2q_compensate_workspace_bytes(method, nl, rows, C, precision))
    return G2Q_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int maxq = (1 << (bits - 1)) - 1;
  const bool use_tc = precision == 1;
  // fused tensor-core updates: operands pre-split once (U, Z) or by the block
  // kernel itself (the error block), one GEMM launch per update
  const bool fused = use_tc && method != G2Q_METHOD_GPTAQ && blocksize % 64 == 0 &&
                     rows % 8 == 0 && C % 8 == 0;
  // GPTQ defers far updates when no group's parameters read columns beyond
  // the block they start in (static groups: found before the traversal)
  const bool defer = fused && method == G2Q_METHOD_GPTQ &&
                     (!dynamic_groups || blocksize % groupsize == 0);
  const int S = defer ? defer_blocks() : 1;
  const int S_ws = (method == G2Q_METHOD_GPTQ && use_tc) ? SUPER : 1;
  char* wsp = align_up((char*)workspace, 256);
  auto take = [&](size_t bytes) {
    char* q = wsp;
    wsp = align_up(wsp + bytes, 256);
    return q;
  };
  float* erra = (float*)take((size_t)nl * rows * BLK * S_ws * sizeof(float));
  const size_t gws = use_tc ? gemm_tc_workspace_bytes(rows, C, (long long)S_ws * BLK, nl, nl)
                            : 0;
  void* gwsp = use_tc ? (void*)take(gws) : nullptr;
  const long long nblk = (C + blocksize - 1) / blocksize;
  const long long nupd = nblk - 1;  // blocks followed by a trailing update (all full)
  __half *eh[2] = {nullptr, nullptr}, *uh[2] = {nullptr, nullptr}, *zh[2] = {nullptr, nullptr};
  float *eh_sc = nullptr, *u_sc = nullptr, *z_sc = nullptr;
  if (fused) {
    eh[0] = (__half*)take((size_t)nl * BLK * rows * sizeof(__half));
    eh[1] = (__half*)take((size_t)nl * BLK * rows * sizeof(__half));
    eh_sc = (float*)take((size_t)nl * rows * sizeof(float));
    uh[0] = (__half*)take((size_t)nl * (C + BLK) * C * sizeof(__half));
    uh[1] = (__half*)take((size_t)nl * (C + BLK) * C * sizeof(__half));
    u_sc = (float*)take((size_t)nl * (C / 64 + 1) * C * sizeof(float));
    if (method == G2Q_METHOD_G2PTQ) {
      zh[0] = (__half*)take((size_t)nl * (C + BLK) * rows * sizeof(__half));
      zh[1] = (__half*)take((size_t)nl * (C + BLK) * rows * sizeof(__half));
      z_sc = (float*)take((size_t)nl * (C / 64 + 1) * rows * sizeof(float));
    }
    if (nupd > 0) {
      // U's strips: strip k = rows [k bs, (k+1) bs), one scale per strip and column
      G2Q_TRY(split2h_strips(U, C, C, blocksize, uh[0], uh[1], C, u_sc, 0, (int)nupd,
                             (long long)blocksize * C, (long long)blocksize * C, C, (int)nl,
                             C * C, nupd * blocksize * C, nupd * C, st));
      // Z's block columns, transposed: [k][row], one scale per block and row
      if (method == G2Q_METHOD_G2PTQ)
        G2Q_TRY(split2h_strips(z, C, rows, blocksize, zh[0], zh[1], rows, z_sc, 1, (int)nupd,
                               blocksize, (long long)blocksize * rows, rows, (int)nl,
                               rows * C, nupd * blocksize * rows, nupd * rows, st));
    }
  }
  // D[:, :, c0:c1] += beta * A @ P[k-rows of the block, c0:c1] on fp32 operands:
  // tensor cores, or CUDA cores where TMA cannot describe them.  A is stored
  // k-major (column-major error) when a_kmajor, else row-major.
  auto update_f32 = [&](float* D, long long c0, long long c1, const float* A, long long lda,
                        long long a_bs, bool a_kmajor, const float* Pm, long long k0, int K,
                        float beta) -> int {
    const long long N = c1 - c0;
    if (N <= 0) return G2Q_OK;
    if (use_tc) {
      const int s = gemm_tc_f32(D + c0, C, rows * C, A, lda, a_bs, a_kmajor, Pm + k0 * C + c0, C,
                                C * C, false, rows, N, K, nl, 1.f, beta, G2Q_MASK_FULL, gwsp, gws,
                                status, st);
      if (s != G2Q_ERR_UNSUPPORTED) return s;
    }
    return simt_gemm_f32(D + c0, C, A, lda, a_kmajor, Pm + k0 * C + c0, C, false, rows, N, K,
                         1.f, beta, G2Q_MASK_FULL, st, nl, a_bs, C * C, rows * C);
  };
  for (long long i1 = 0; i1 < C; i1 += blocksize) {
    const long long i2 = (i1 + blocksize < C) ? i1 + blocksize : C;
    const int nc = (int)(i2 - i1);
    const long long kb = i1 / blocksize;
    const int j = (int)(kb % S);                       // place in its group of S blocks
    const long long s1 = (kb - j) * blocksize;          // the group's first column
    const long long s2 = (s1 + (long long)S * blocksize < C) ? s1 + (long long)S * blocksize : C;
    if (dynamic_groups) {
      // group starts c0 with i1 <= c0 < i2 and c0 % groupsize == 0
      const long long first = (i1 + groupsize - 1) / groupsize * groupsize;
      const int cnt = first < i2 ? (int)((i2 - 1 - first) / groupsize + 1) : 0;
      if (cnt > 0)
        G2Q_TRY(launch_find_params(scale, zero, ngroups, W, nl * rows, 0, C, bits, sym, status,
                                   first, cnt, groupsize, C, clip, st));
    }
    BlockParams P{};
    P.W = W + i1; P.ldw = C; P.w_bs = rows * C;
    P.rows = rows; P.ncols = nc;
    P.hinv = U + i1 * C + i1; P.ldh = C; P.h_bs = C * C;
    P.scale = scale; P.zero = zero; P.param_ld = ngroups; P.colmap = colgroup + i1;
    P.maxq = maxq;
    P.codes = codes + i1; P.ldq = C; P.q_bs = rows * C;
    // block j of its group keeps its errors at k = j * blocksize, so that the
    // group's errors form one contiguous K range for the far update
    P.erra = erra + (size_t)j * blocksize * rows; P.ldea = rows;
    P.ea_bs = (long long)S * BLK * rows;
    if (fused && i2 < C) {
      P.eh_hi = eh[0]; P.eh_lo = eh[1]; P.eh_scale = eh_sc; P.eh_bs = BLK * rows;
    }
    if (method == G2Q_METHOD_G2PTQ) {
      P.z = z + i1; P.gh = gh + i1; P.ldz = C; P.z_bs = rows * C;
    }
    if (method == G2Q_METHOD_GPTAQ) P.p = p + i1 * C + i1;
    P.dfact = blocksize;
    if (wraw) {
      P.wraw = wraw + i1;
      P.beta = approx_beta;
    }
    G2Q_TRY(launch_block(method, P, nl, st));
    if (i2 >= C) break;
    const long long N = C - i2;
    if (method == G2Q_METHOD_G2PTQ) {
      const dim3 grid = wave_grid_2d(nl * rows, N);
      sub_scaled_kernel<<<grid, 256, 0, st>>>(W, gh, nl * rows, C, i2, (float)blocksize);
      G2Q_CHECK_LAUNCH();
    }
    // W[:, i2:] -= Erra @ U[i1:i2, i2:]  (+ G2PTQ: GH[:, i2:] -= Z[:, i1:i2] @ U[i1:i2, i2:];
    // GPTAQ: W[:, i2:] += Q1 @ P[i1:i2, i2:]).  With deferral the block updates
    // only [i2, s2) and the last block of the group the columns after it.
    if (fused) {
      __half* const ub[2] = {uh[0], uh[1]};
      // one fused update of D[:, :, i2:c1] from the block's pre-split error
      auto fused_update = [&](float* D, long long c1, __half* const* a2, long long a_outer,
                              long long ka_batch, long long ka0, const float* sa,
                              long long sa_bs) -> int {
        return tc_update_f16(D + i2, C, rows * C, rows, c1 - i2, nc, nl, a2, rows, a_outer,
                             ka_batch, ka0, sa, sa_bs, ub, C, C, nl * nupd * blocksize,
                             nupd * blocksize, kb * blocksize, i2, u_sc + kb * C + i2, nupd * C,
                             -1.f, status, st);
      };
      if (S == 1 || i2 < s2) {
        // near update: the rest of the group (or, undeferred, every later column)
        const long long c1 = (S == 1) ? C : s2;
        int s_w = fused_update(W, c1, eh, nl * BLK, BLK, 0, eh_sc, rows);
        if (s_w == G2Q_ERR_UNSUPPORTED)
          s_w = update_f32(W, i2, c1, P.erra, rows, (long long)S * BLK * rows, true, U, i1, nc,
                           -1.f);
        G2Q_TRY(s_w);
      } else if (s2 < C) {
        // the group's far update, K = S blocks, from the fp32 errors
        G2Q_TRY(update_f32(W, s2, C, erra, rows, (long long)S * BLK * rows, true, U, s1,
                           (int)(s2 - s1), -1.f));
      }
      if (method == G2Q_METHOD_G2PTQ) {
        int s_g = fused_update(gh, C, zh, nl * nupd * blocksize, nupd * blocksize,
                               kb * blocksize, z_sc + kb * rows, nupd * rows);
        if (s_g == G2Q_ERR_UNSUPPORTED)
          s_g = update_f32(gh, i2, C, z + i1, C, rows * C, false, U, i1, nc, -1.f);
        G2Q_TRY(s_g);
      }
      continue;
    }
    G2Q_TRY(update_f32(W, i2, C, P.erra, rows, (long long)S * BLK * rows, true, U, i1, nc, -1.f));
    if (method == G2Q_METHOD_G2PTQ)
      G2Q_TRY(update_f32(gh, i2, C, z + i1, C, rows * C, false, U, i1, nc, -1.f));
    if (method == G2Q_METHOD_GPTAQ)
      G2Q_TRY(update_f32(W, i2, C, W + i1, C, rows * C, false, p, i1, nc, 1.f));
  }
  return G2Q_OK;
}
