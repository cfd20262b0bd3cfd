// Shared helpers for the g2ptq_b200 CUDA library (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "g2ptq_b200.h"

namespace g2q {
// Counts every kernel launch the library issues (read by g2q_launch_count).
void note_launch();
}  // namespace g2q

#define G2Q_CHECK_LAUNCH()                                   \
  do {                                                       \
    g2q::note_launch();                                      \
    cudaError_t _e = cudaGetLastError();                     \
    if (_e != cudaSuccess) return G2Q_ERR_CUDA;              \
  } while (0)

#define G2Q_TRY(expr)                                        \
  do {                                                       \
    int _s = (expr);                                         \
    if (_s != G2Q_OK) return _s;                             \
  } while (0)

namespace g2q {

static inline int cdiv(long long a, long long b) { return (int)((a + b - 1) / b); }

// 2-D grid for a rows x units elementwise kernel with 256 threads along a row
// (blockIdx.y over rows, blockIdx.x over 256-unit pieces of a row): at most
// 64 CTAs per SM (eight waves of eight), the kernels loop over the rest.  x
// gets as many CTAs as a row has pieces, up to the whole budget when there
// are few rows (a flat array passed as one row), y the rest.  A single wave
// measured 1.3-1.9x slower on these load-store loops (one element in flight
// per thread) and starved flat calls of CTAs.
static inline dim3 wave_grid_2d(long long rows, long long units) {
  const long long wave = 148 * 64;
  long long gx = (units + 255) / 256;
  if (gx < 1) gx = 1;
  long long gy = wave / (gx < wave ? gx : wave);
  if (gy > rows) gy = rows;
  if (gy < 1) gy = 1;
  if (gx > wave / gy) gx = wave / gy;
  return dim3((unsigned)gx, (unsigned)gy);
}

__device__ __forceinline__ float bf16_hi(float x, __nv_bfloat16* hi) {
  __nv_bfloat16 h = __float2bfloat16_rn(x);
  *hi = h;
  return x - __bfloat162float(h);
}

// Splits an fp32 value into a bf16 pair whose sum carries ~16 significant bits.
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16* hi, __nv_bfloat16* lo) {
  float r = bf16_hi(x, hi);
  *lo = __float2bfloat16_rn(r);
}

// Device-side status word: kernels that meet a condition they cannot handle
// record a code here instead of trapping; the host reads it after the stream
// work completes.
__device__ __forceinline__ void record_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

}  // namespace g2q
