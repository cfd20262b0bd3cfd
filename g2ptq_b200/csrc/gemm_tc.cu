// Tensor-core (tcgen05) Gram / GEMM path.  Placeholder entry points until the
// sm_100a kernel lands; the fp32 CUDA-core path serves every call meanwhile.
#include "gemm_simt.cuh"

namespace g2q {

size_t tc_gram_workspace_bytes(long long, long long, long long) { return 0; }

int tc_gram(float*, long long, long long, long long, const void*, int, long long, const void*,
            int, long long, const float*, long long, long long, int, float, float, void*, size_t,
            cudaStream_t) {
  return G2Q_ERR_UNSUPPORTED;
}

}  // namespace g2q
