// Gram update on tensor cores with library-owned scratch: a variant of
// g2q_gram_update (precision 1) for callers that cannot allocate device memory.
//
// Who needs it: a host that binds only this C ABI and owns no device
// allocator (a C, Go or Rust service with no caching allocator of its own
// cannot hand over the bf16 split buffers that FP32 or row-scaled inputs
// need), and a caller folding activations in the middle of a pipelined step,
// where a fresh cudaMalloc may synchronise the device and stall the streams
// that are still running.  Such callers get their scratch from a fixed
// file-scope device array instead, set up once per device.
//
// The scratch holds the bf16 hi/lo splits of A and B.  Every byte the
// tensor-core kernel reads from it is written earlier on the same stream by
// the split kernel of the same call (the tail of the last token tile is
// zero-filled by TMA from outside the tensor, not read from the scratch), so
// nothing in it has to start at zero.  One array serves the whole device:
// calls that overlap in time (on different streams, or from different host
// threads) race on it; calls on one stream follow one another and are safe.
#include <mutex>

#include "common.cuh"

namespace g2q {

int tc_gram(float* D, long long ldd, long long M, long long N, const void* A, int a_dtype,
            long long lda, const void* B, int b_dtype, long long ldb, const float* row_scale,
            long long scale_stride, long long T, int symmetric, float alpha, float beta,
            void* workspace, size_t workspace_bytes, int* status, cudaStream_t st);
size_t tc_gram_workspace_bytes(long long M, long long N, long long T);

static __device__ __align__(256) unsigned char gram_scratch[G2Q_GRAM_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static std::mutex scratch_mu;
static void* scratch_ptr[kMaxDevices];

// Device address of gram_scratch on the stream's device, looked up once per
// device.  That device must be the current one (the symbol is resolved and
// the kernels launched there); a stream of another device is rejected.  The
// first call on a device does this set-up (it loads the module there); make
// it before any stream capture.
static int scratch_for_stream(cudaStream_t st, void** out) {
  int dev = -1, sdev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return G2Q_ERR_CUDA;
  if (cudaStreamGetDevice(st, &sdev) != cudaSuccess) return G2Q_ERR_INVALID_ARG;
  if (sdev != dev) return G2Q_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lock(scratch_mu);
  if (!scratch_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, gram_scratch) != cudaSuccess || !p) return G2Q_ERR_CUDA;
    scratch_ptr[dev] = p;
  }
  *out = scratch_ptr[dev];
  return G2Q_OK;
}

}  // namespace g2q

extern "C" size_t g2q_gram_static_scratch_bytes(void) { return G2Q_GRAM_STATIC_SCRATCH_BYTES; }

extern "C" int g2q_gram_update_noalloc(float* D, int64_t ldd, int64_t M, int64_t N,
                                       const void* A, int a_dtype, int64_t lda, const void* B,
                                       int b_dtype, int64_t ldb, const float* row_scale,
                                       int64_t scale_stride, int64_t T, int symmetric,
                                       float alpha, float beta, int* status, void* stream) {
  if (!D || !A || !B || M <= 0 || N <= 0 || T < 0 || lda < M || ldb < N || ldd < N)
    return G2Q_ERR_INVALID_ARG;
  if ((a_dtype != G2Q_DTYPE_BF16 && a_dtype != G2Q_DTYPE_F32) ||
      (b_dtype != G2Q_DTYPE_BF16 && b_dtype != G2Q_DTYPE_F32))
    return G2Q_ERR_INVALID_ARG;
  if (symmetric && M != N) return G2Q_ERR_INVALID_ARG;
  // scratch is used when an operand must be split into bf16 terms: FP32 input,
  // or a B side that differs from A (another tensor, or A with a row scale)
  const bool same = (A == B) && (a_dtype == b_dtype) && !row_scale;
  const bool split = a_dtype != G2Q_DTYPE_BF16 ||
                     (!same && (b_dtype != G2Q_DTYPE_BF16 || row_scale != nullptr));
  if (split && g2q::tc_gram_workspace_bytes(M, N, T) > (size_t)G2Q_GRAM_STATIC_SCRATCH_BYTES)
    return G2Q_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  G2Q_TRY(g2q::scratch_for_stream((cudaStream_t)stream, &scratch));
  return g2q::tc_gram(D, ldd, M, N, A, a_dtype, lda, B, b_dtype, ldb, row_scale, scale_stride,
                      T, symmetric, alpha, beta, scratch,
                      (size_t)G2Q_GRAM_STATIC_SCRATCH_BYTES, status, (cudaStream_t)stream);
}
