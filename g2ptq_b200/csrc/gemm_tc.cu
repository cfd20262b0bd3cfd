// Tensor-core (tcgen05) Gram / GEMM for sm_100a.
//
//   D[m, n] <- alpha * D[m, n] + beta * sum_k A[k, m] * B[k, n]
//
// Both operands are "MN-major" in global memory: for every k, the m (or n)
// index is contiguous.  That is how the two hot products arrive:
//   * Hessian Gram  H += X^T X  with X token-major [T, C]  (k = token),
//   * GPTQ trailing update  W[:, i2:] -= Err @ U[i1:i2, i2:]  with the block
//     error stored column-major [blk, rows] by the compensation kernel and U
//     row-major (k = block column).
// Tiles of 128 x 64 (MN x K) 16-bit values are fed by TMA (64 x 64 boxes,
// 128-byte swizzle) into a multi-stage shared-memory ring; one thread issues
// tcgen05.mma (M = 128, N = 128 or 256, K = 16, bf16 or fp16 in, fp32
// accumulate in TMEM); the epilogue warps read the accumulator with tcgen05.ld
// and apply alpha / beta, the bounds and the symmetric mirror.
// fp32 operands are carried as a hi/lo pair and multiplied as
// hi*hi + hi*lo + lo*hi (three MMAs per K step): bf16 pairs for the trailing
// update and fp32 Grams, and -- where fp32 accuracy is required (the Cholesky
// updates) -- fp16 pairs of rows scaled by powers of two (22 significant bits,
// the scales applied exactly in the epilogue).

// Accumulator promotion: the tensor core adds each MMA's partial sum into the
// TMEM accumulator with a bias of about one fp32 ulp (measured: the relative
// error of a long Gram product grows linearly with K, every diagonal entry
// too small).  The MMA warp therefore accumulates at most `promote_kb` K
// blocks into one of two TMEM buffers, and the epilogue warps drain each
// finished buffer into an fp32 register accumulator with rounded adds while
// the other buffer fills.  The bias stays below ~1e-6 relative for any K.
//
// Warp roles (192 threads, 320 for 128 x 256 tiles): warp 0 TMA producer,
// warp 1 TMEM owner + MMA issuer, the rest epilogue (TMEM lane quadrant =
// warp % 4).
// Every wait on an mbarrier is bounded (Params::wait_cycles, set from
// g2q_set_wait_limit); on expiry the CTA records G2Q_ERR_TIMEOUT in the
// caller's status word and winds down: the producer waits (with its own fixed
// bound) for the loads it issued to land and the MMA issuer for the MMAs it
// issued to complete before the TMEM is freed and the CTA exits.
#include <cuda.h>
#include <stdlib.h>
#include <cudaTypedefs.h>

#include <cuda_fp16.h>

#include "gemm_simt.cuh"

namespace g2q {
namespace tc {

constexpr int BM = 128, BN = 128, BK = 64;
constexpr int CHUNK_BYTES = 64 * BK * 2;     // one 64 (MN) x 64 (K) bf16 box
constexpr int TILE_BYTES = 2 * CHUNK_BYTES;  // one 128 x 64 operand tile
constexpr long long kWaitCycles = 4000000000LL;   // default bound of one pipeline wait
constexpr long long kDrainCycles = 2000000000LL;  // bound of a wind-down wait after an abort

struct Params {
  float* D;
  long long ldd, d_bs;
  long long M, N;
  int num_kb;
  long long ka_batch, kb_batch;  // per-batch row offset of A / B in their tensor maps
  long long ka0, kb0;            // first K row of A / B
  long long nb0;                 // first N coordinate of B
  float alpha, beta;
  int symmetric;
  int lower;       // write only the lower triangle (m >= n); skip tiles above it
  int promote_kb;  // K blocks accumulated in TMEM before the epilogue drains them
  int raster;      // 1: 1-D grid over the needed tiles in groups of GROUP_M tile rows
  int tiles_m, tiles_n;
  int red;         // short-K epilogue adds beta * acc into D with TMA reduce-add (alpha == 1)
  int f16;         // operands are fp16 (else bf16)
  const float* sa;  // optional per-row (M) and per-column (N) output scales, powers of two
  const float* sb;
  long long sa_bs, sb_bs;  // their batch strides
  int supper;      // write only m < n (strictly upper part)
  int prefetch_kb;  // CTA-pair kernel: L2 prefetch distance in k-blocks (0: none)
  int* status;     // receives G2Q_ERR_TIMEOUT when a wait gives up (may be null)
  long long wait_cycles;  // bound of every pipeline wait (set by the launchers)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t a, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(a), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t a, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(a), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_test(uint32_t a, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(a), "r"(parity)
      : "memory");
  return done != 0;
}

// Pipeline wait: gives up when another warp of the CTA has given up
// (abort_flag) or after `limit` cycles, which sets the flag and records
// G2Q_ERR_TIMEOUT.
__device__ __forceinline__ bool mbar_wait(uint32_t a, uint32_t parity, volatile int* abort_flag,
                                          int* status, long long limit) {
  const long long t0 = clock64();
  while (true) {
    if (mbar_test(a, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > limit) {
      *abort_flag = 1;
      record_error(status, G2Q_ERR_TIMEOUT);
      return false;
    }
  }
}

// Wind-down wait after an abort: the phase completes once asynchronous work
// this thread already issued (loads, MMAs) has finished; bounded by
// kDrainCycles, and it ignores the abort flag.
__device__ __forceinline__ bool mbar_drain(uint32_t a, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_test(a, parity))
    if (clock64() - t0 > kDrainCycles) return false;
  return true;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar)
      : "memory");
}

// D[z][y .. y+31][x .. x+31] += the 32 x 32 fp32 box at smem (128-byte swizzled
// rows), performed by the TMA unit in L2: the SM never reads D.
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, uint32_t src, int x, int y,
                                                  int z) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group"
      " [%0, {%1, %2, %3}], [%4];" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(z), "r"(src)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// wait until at most one committed bulk group still reads shared memory
__device__ __forceinline__ void bulk_wait_read_1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Shared-memory matrix descriptor of an MN-major, 128-byte-swizzled operand:
// 64-element MN chunks 8 KB apart (LBO), groups of 8 K rows 1 KB apart (SBO).
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)(CHUNK_BYTES >> 4) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// The same with MN chunks `lbo` bytes apart (chunks of 64 x BKP for a K depth
// BKP per stage).
__device__ __forceinline__ uint64_t desc_mn_sw128_lbo(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)(lbo >> 4) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kind::f16 instruction descriptor: bf16 x bf16 (or f16 x f16) -> f32, both
// MN-major, M=128, N=n.
__host__ __device__ constexpr uint32_t idesc_bf16_mn(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_f16_mn(int n) {
  return idesc_bf16_mn(n) & ~((7u << 7) | (7u << 10));
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint32_t mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   mbar)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t a) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(a) : "memory");
}

__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// SMALL: short-K variant (K <= 4 blocks, no promotion needed): one accumulator,
// the epilogue reads TMEM directly, and a single pipeline stage (up to three for
// one-term operands) so that two or three CTAs share an SM and overlap one
// CTA's epilogue with another's loads and MMAs.
// WIDE: 128 x 256 output tiles (N = 256 MMAs) for one-term long-K products.
// A k-block then carries 512 tensor cycles of work, enough to hide the
// full/empty barrier round trip that caps 128 x 128 k-blocks near half rate,
// and each SM reads 48 KB per k-block instead of 64 KB for the same work.
// Eight epilogue warps (two per TMEM lane quarter) drain the 256 columns.
template <int NA, int NB, bool SMALL = false, bool WIDE = false>
struct Cfg {
  static constexpr int BN_T = WIDE ? 256 : BN;
  static constexpr int B_BYTES = (BN_T / 64) * CHUNK_BYTES;  // one B term of a stage
  static constexpr int STAGE_BYTES = NA * TILE_BYTES + NB * B_BYTES;
  static constexpr int STAGES =
      SMALL ? ((NA + NB) == 2 ? 3 : 1) : (192 * 1024) / STAGE_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr int MIN_BLOCKS = SMALL ? ((NA + NB) >= 6 ? 2 : 3) : 1;
  static constexpr int EPI_WARPS = WIDE ? 8 : 4;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int ACC_COLS = SMALL ? BN : 2 * BN_T;
  static constexpr int ORDER = (NA > NB ? NA : NB) - 1;  // products a_i b_j with i + j <= ORDER
  static constexpr int PRODUCTS = NA + NB - 1;
  // K blocks per TMEM accumulation group: 16 MMAs for one product, 24 otherwise
  static constexpr int PROMOTE_KB = PRODUCTS == 1 ? 4 : (PRODUCTS <= 3 ? 2 : 1);
};

// Stores four consecutive accumulator columns v[0..3] of row gm starting at
// column gn: alpha/beta, bounds, triangle masks and the symmetric mirror.
#define EPILOGUE_STORE4                                                                        \
  {                                                                                           \
    float* dst = Db + gm * p.ldd + gn;                                                        \
    if (vec_ok && gn + 3 < p.N && (!p.symmetric || gn >= gm) && (!p.lower || gn + 3 <= gm) && \
        (!p.supper || gn > gm)) {                                                             \
      float4* d4 = reinterpret_cast<float4*>(dst);                                            \
      if (p.alpha != 0.f) {                                                                   \
        const float4 o = *d4;                                                                 \
        v[0] = fmaf(p.alpha, o.x, v[0]);                                                      \
        v[1] = fmaf(p.alpha, o.y, v[1]);                                                      \
        v[2] = fmaf(p.alpha, o.z, v[2]);                                                      \
        v[3] = fmaf(p.alpha, o.w, v[3]);                                                      \
      }                                                                                       \
      *d4 = make_float4(v[0], v[1], v[2], v[3]);                                              \
    } else {                                                                                  \
      _Pragma("unroll") for (int u = 0; u < 4; ++u) {                                         \
        if (gn + u >= p.N || (p.symmetric && gn + u < gm) || (p.lower && gn + u > gm) ||      \
            (p.supper && gn + u <= gm))                                                       \
          continue;                                                                           \
        if (p.alpha != 0.f) v[u] = fmaf(p.alpha, dst[u], v[u]);                               \
        dst[u] = v[u];                                                                        \
      }                                                                                       \
    }                                                                                         \
    if (p.symmetric) {                                                                        \
      _Pragma("unroll") for (int u = 0; u < 4; ++u) if (gn + u < p.N && gn + u > gm)         \
          Db[(gn + u) * p.ldd + gm] = v[u];                                                   \
    }                                                                                         \
  }

// Grouped rasterization for long-K products: consecutive CTAs walk GROUP_M tile
// rows together, so a wave of CTAs reads a few dozen distinct operand column
// blocks per K step instead of one per CTA and X stays in L2 between them.
// Symmetric outputs enumerate only tiles with nt >= mt.
constexpr int GROUP_M = 8;
__device__ __forceinline__ bool decode_tile(long long id, int Tm, int Tn, bool sym, int& mt,
                                            int& nt) {
  for (int r0 = 0; r0 < Tm; r0 += GROUP_M) {
    const int gsz = (Tm - r0) < GROUP_M ? (Tm - r0) : GROUP_M;
    const long long tri = (long long)gsz * (gsz + 1) / 2;
    const long long count = sym ? tri + (long long)(Tn - r0 - gsz) * gsz : (long long)gsz * Tn;
    if (id < count) {
      if (!sym) {
        nt = (int)(id / gsz);
        mt = r0 + (int)(id % gsz);
      } else if (id < tri) {
        int c = 0;
        while (id >= c + 1) {
          id -= c + 1;
          ++c;
        }
        nt = r0 + c;
        mt = r0 + (int)id;
      } else {
        id -= tri;
        nt = r0 + gsz + (int)(id / gsz);
        mt = r0 + (int)(id % gsz);
      }
      return true;
    }
    id -= count;
  }
  return false;
}

// Symmetric outputs with 128 x 256 tiles: tile (mt, nt) holds upper-triangle
// elements when mt * 128 <= nt * 256 + 255, i.e. nt >= mt / 2.  Tile rows are
// walked in groups of GROUP_M as above; inside a group the columns where only
// part of the group's rows are needed come first.
__host__ __device__ __forceinline__ long long wide_sym_group_count(int r0, int g, int Tn) {
  long long c = 0;
  for (int i = 0; i < g; ++i) {
    const int lo = (r0 + i) / 2;
    if (lo < Tn) c += Tn - lo;
  }
  return c;
}

__device__ __forceinline__ bool decode_tile_wide_sym(long long id, int Tm, int Tn, int& mt,
                                                     int& nt) {
  for (int r0 = 0; r0 < Tm; r0 += GROUP_M) {
    const int g = (Tm - r0) < GROUP_M ? (Tm - r0) : GROUP_M;
    const long long count = wide_sym_group_count(r0, g, Tn);
    if (id < count) {
      int n = r0 / 2;
      while (true) {
        const int rows = (2 * n + 2 - r0) < g ? (2 * n + 2 - r0) : g;
        if (rows >= g) break;
        if (id < rows) {
          nt = n;
          mt = r0 + (int)id;
          return true;
        }
        id -= rows;
        ++n;
      }
      nt = n + (int)(id / g);
      mt = r0 + (int)(id % g);
      return true;
    }
    id -= count;
  }
  return false;
}

template <int NA, int NB, bool SMALL, bool WIDE>
__global__ void __launch_bounds__((Cfg<NA, NB, SMALL, WIDE>::THREADS),
                                  (Cfg<NA, NB, SMALL, WIDE>::MIN_BLOCKS))
    tc_gemm_kernel(const __grid_constant__ CUtensorMap ma0, const __grid_constant__ CUtensorMap ma1,
                   const __grid_constant__ CUtensorMap ma2, const __grid_constant__ CUtensorMap mb0,
                   const __grid_constant__ CUtensorMap mb1, const __grid_constant__ CUtensorMap mb2,
                   const __grid_constant__ CUtensorMap md, Params p) {
  using K = Cfg<NA, NB, SMALL, WIDE>;
  constexpr int BN_T = K::BN_T;
  int mt = blockIdx.y, nt = blockIdx.x;
  const long long bz = blockIdx.z;
  if (p.raster) {
    const bool found = (WIDE && p.symmetric)
                           ? decode_tile_wide_sym(blockIdx.x, p.tiles_m, p.tiles_n, mt, nt)
                           : decode_tile(blockIdx.x, p.tiles_m, p.tiles_n, p.symmetric, mt, nt);
    if (!found) return;
  }
  // tiles holding no element of the upper (symmetric) / lower triangle
  if (p.symmetric && (long long)nt * BN_T + BN_T - 1 < (long long)mt * BM) return;
  if (p.lower && (long long)nt * BN_T > (long long)mt * BM + BM - 1) return;
  if (p.supper && (long long)mt * BM >= (long long)nt * BN_T + BN_T - 1) return;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + K::STAGES * K::STAGE_BYTES);
  // bars[0..S): full, [S..2S): empty, [2S..2S+2): accumulator full, [2S+2..2S+4): drained,
  // [2S+4]: MMA completion after an abort
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * K::STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + K::STAGES);
  const uint32_t accf0 = smem_u32(bars + 2 * K::STAGES);
  const uint32_t acce0 = smem_u32(bars + 2 * K::STAGES + 2);
  const uint32_t drain0 = smem_u32(bars + 2 * K::STAGES + 4);
  const int ngroups = SMALL ? (p.num_kb > 0 ? 1 : 0)
                            : (p.num_kb + p.promote_kb - 1) / p.promote_kb;
  const int promote_kb = SMALL ? p.num_kb : p.promote_kb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < K::STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, 32 * K::EPI_WARPS);
    }
    mbar_init(drain0, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(K::ACC_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_holder;
  const int m0 = mt * BM, n0 = nt * BN_T;

  int issued = 0;  // k-blocks whose loads the producer issued
  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < p.num_kb; ++kb) {
        const int s = kb % K::STAGES;
        const uint32_t ph = (kb / K::STAGES) & 1;
        if (!mbar_wait(empty0 + 8 * s, ph ^ 1, abort_flag, p.status, p.wait_cycles)) break;
        issued = kb + 1;
        const uint32_t fb = full0 + 8 * s;
        mbar_expect_tx(fb, K::STAGE_BYTES);
        const uint32_t st = smem_u32(smem + s * K::STAGE_BYTES);
        const int ya = (int)(p.ka_batch * bz + p.ka0 + (long long)kb * BK);
        const int yb = (int)(p.kb_batch * bz + p.kb0 + (long long)kb * BK);
        const int xb = (int)(p.nb0 + n0);
#pragma unroll
        for (int i = 0; i < NA; ++i) {
          const CUtensorMap* m = i == 0 ? &ma0 : (i == 1 ? &ma1 : &ma2);
          tma_load_2d(st + i * TILE_BYTES, m, m0, ya, fb);
          tma_load_2d(st + i * TILE_BYTES + CHUNK_BYTES, m, m0 + 64, ya, fb);
        }
        const uint32_t sb = st + NA * TILE_BYTES;
#pragma unroll
        for (int j = 0; j < NB; ++j) {
          const CUtensorMap* m = j == 0 ? &mb0 : (j == 1 ? &mb1 : &mb2);
#pragma unroll
          for (int c = 0; c < BN_T / 64; ++c)
            tma_load_2d(sb + j * K::B_BYTES + c * CHUNK_BYTES, m, xb + 64 * c, yb, fb);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = p.f16 ? idesc_f16_mn(BN_T) : idesc_bf16_mn(BN_T);
      int kb = 0;
      for (int g = 0; g < ngroups; ++g) {
        const int buf = g & 1;
        const uint32_t use_ph = (uint32_t)((g >> 1) & 1);
        if (!mbar_wait(acce0 + 8 * buf, use_ph ^ 1, abort_flag, p.status, p.wait_cycles)) break;
        fence_after();
        const uint32_t acc_t = tmem + (uint32_t)(buf * BN_T);
        const int kend = (kb + promote_kb < p.num_kb) ? kb + promote_kb : p.num_kb;
        const int kstart = kb;
        bool ok = true;
        for (; kb < kend; ++kb) {
          const int s = kb % K::STAGES;
          const uint32_t ph = (kb / K::STAGES) & 1;
          if (!mbar_wait(full0 + 8 * s, ph, abort_flag, p.status, p.wait_cycles)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t sa = smem_u32(smem + s * K::STAGE_BYTES);
          const uint32_t sb = sa + NA * TILE_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint32_t off = kk * 2048;  // 16 K rows = two 8-row swizzle groups
            const uint32_t acc0 = (kb > kstart || kk > 0) ? 1u : 0u;
            // products a_i * b_j with i + j <= ORDER, the leading one first
#pragma unroll
            for (int o = 0; o <= K::ORDER; ++o) {
#pragma unroll
              for (int i = 0; i < NA; ++i) {
                const int j = o - i;
                if (j < 0 || j >= NB) continue;
                umma_bf16(acc_t, desc_mn_sw128(sa + i * TILE_BYTES + off),
                          desc_mn_sw128(sb + j * K::B_BYTES + off), idesc,
                          (o == 0) ? acc0 : 1u);
              }
            }
          }
          umma_commit(empty0 + 8 * s);
        }
        if (!ok) break;
        umma_commit(accf0 + 8 * buf);
      }
    }
  } else if (SMALL) {
    // epilogue warps 2..5, short K: read the single accumulator chunk by chunk
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const long long gm = m0 + row;
    bool ok = true;
    if (ngroups > 0) ok = mbar_wait(accf0, 0, abort_flag, p.status, p.wait_cycles);
    fence_after();
    float* Db = p.D + bz * p.d_bs;
    if (p.red) {
      // Every load has landed and every MMA has read its operands, so the stage
      // buffers are free: each warp stages its 32 rows x 32 columns per chunk in
      // two swizzled 4 KB buffers and the TMA unit adds them into D.
      static_assert(K::STAGES * K::STAGE_BYTES >= 4 * 8192, "staging does not fit");
      uint8_t* stg = smem + q * 8192;
      // the row's operand scale, loaded once; the chunk's 32 column scales,
      // one per lane and passed around by shuffles (no global load per element)
      const float sa_row = (p.sa && gm < p.M) ? p.sa[bz * p.sa_bs + gm] : 1.f;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        if (ngroups > 0) {
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), r);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0u;
        }
        const long long gn_lane = n0 + c * 32 + lane;
        const float sb_lane = (p.sa && gn_lane < p.N) ? p.sb[bz * p.sb_bs + gn_lane] : 1.f;
        if (c >= 2) {
          if (lane == 0) bulk_wait_read_1();
          __syncwarp();
        }
        float* buf = reinterpret_cast<float*>(stg + (c & 1) * 4096);
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          const long long gn = n0 + c * 32 + 4 * j4;
          float v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            v[u] = p.beta * __uint_as_float(r[4 * j4 + u]);
            const float sb_col = __shfl_sync(0xffffffffu, sb_lane, 4 * j4 + u);
            if (p.sa) v[u] *= sa_row * sb_col;
            // leave the other triangle as it is
            if ((p.lower && gn + u > gm) || (p.supper && gn + u <= gm)) v[u] = 0.f;
          }
          *reinterpret_cast<float4*>(buf + lane * 32 + ((j4 ^ (lane & 7)) << 2)) =
              make_float4(v[0], v[1], v[2], v[3]);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          // boxes starting inside D only; TMA clips the parts beyond M and N
          if (ok && n0 + c * 32 < p.N && m0 + q * 32 < p.M)
            tma_reduce_add_3d(&md, smem_u32(buf), n0 + c * 32, m0 + q * 32, (int)bz);
          bulk_commit();
        }
      }
      if (lane == 0) bulk_wait_all();
      __syncwarp();
    } else {
      const bool vec_ok = ((p.ldd & 3) == 0) && ((reinterpret_cast<uintptr_t>(Db) & 15) == 0);
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        if (ngroups > 0) {
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), r);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = 0u;
        }
        if (!ok || gm >= p.M) continue;
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4) {
          const long long gn = n0 + c * 32 + 4 * j4;
          float v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            v[u] = p.beta * __uint_as_float(r[4 * j4 + u]);
            if (p.sa)
              v[u] *= p.sa[bz * p.sa_bs + gm] * (gn + u < p.N ? p.sb[bz * p.sb_bs + gn + u] : 1.f);
          }
          EPILOGUE_STORE4
        }
      }
    }
    if (ngroups > 0) {
      fence_before();
      mbar_arrive(acce0);
    }
  } else {
    // epilogue warps, long K: drain each accumulator buffer into registers.
    // Warp w reads TMEM lanes 32 (w % 4) .. + 31; with eight warps the second
    // four take the upper 128 columns.
    const int q = warp & 3;
    const int half = WIDE ? (warp - 2) / 4 : 0;
    const int row = q * 32 + lane;
    const long long gm = m0 + row;
    float acc[BN];
#pragma unroll
    for (int j = 0; j < BN; ++j) acc[j] = 0.f;
    bool ok = true;
    for (int g = 0; g < ngroups; ++g) {
      const int buf = g & 1;
      const uint32_t use_ph = (uint32_t)((g >> 1) & 1);
      if (ok) ok = mbar_wait(accf0 + 8 * buf, use_ph, abort_flag, p.status, p.wait_cycles);
      fence_after();
      const uint32_t base =
          tmem + (uint32_t)(buf * BN_T + half * BN) + ((uint32_t)(q * 32) << 16);
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(base + (uint32_t)(c * 32), r);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[c * 32 + j] += __uint_as_float(r[j]);
      }
      fence_before();
      mbar_arrive(acce0 + 8 * buf);
    }
    float* Db = p.D + bz * p.d_bs;
    const bool vec_ok = ((p.ldd & 3) == 0) && ((reinterpret_cast<uintptr_t>(Db) & 15) == 0);
    if (ok && gm < p.M) {
#pragma unroll
      for (int j4 = 0; j4 < BN / 4; ++j4) {
        const long long gn = n0 + half * BN + 4 * j4;
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          v[u] = p.beta * acc[4 * j4 + u];
          if (p.sa)
            v[u] *= p.sa[bz * p.sa_bs + gm] * (gn + u < p.N ? p.sb[bz * p.sb_bs + gn + u] : 1.f);
        }
        EPILOGUE_STORE4
      }
    }
  }
  fence_before();
  __syncthreads();
  if (*abort_flag) {
    // a wait gave up: let this CTA's loads land and its MMAs finish before the
    // shared memory and the TMEM are released
    if (warp == 0 && lane == 0) {
      for (int kb = issued > K::STAGES ? issued - K::STAGES : 0; kb < issued; ++kb)
        mbar_drain(full0 + 8 * (kb % K::STAGES), (kb / K::STAGES) & 1);
    } else if (warp == 1 && lane == 0) {
      umma_commit(drain0);
      mbar_drain(drain0, 0);
    }
    __syncthreads();
  }
  if (warp == 1) {
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(K::ACC_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2) for long-K products whose B operand
// is one bf16 term: the Gram folds of add_batch.  A cluster of two CTAs on
// neighbouring SMs computes a 256 x 256 output tile.  CTA r of the pair loads
// rows m0 + 128 r .. + 127 of every A term and columns n0 + 128 r .. + 127 of B
// into its own shared memory; the leader (rank 0) issues M = 256, N = 256 MMAs
// that read both CTAs' operands and write each CTA's TMEM (its 128 rows x all
// 256 columns).  Per SM and 64-token k-block that is 16 KB of A per term plus
// 16 KB of B for 128 x 256 outputs, where a single-CTA 128 x 256 tile reads
// 32 KB of B: operand delivery from L2, which bounds the single-CTA kernel,
// drops by a third for the one-term Gram.
// Barriers: the leader's full[s] counts both CTAs' TMA bytes (the loads use
// the .cta_group::2 form, which may signal the peer's barrier; no multicast);
// one commit with a two-CTA mask frees stage s in both CTAs (empty[s]) and
// announces a finished accumulator buffer to both epilogues (accf[b]); every
// epilogue warp of both CTAs arrives on the leader's acce[b] once it drained b.
// Accumulator promotion as in the single-CTA kernel (PROMOTE_KB k-blocks per
// TMEM buffer, drained into fp32 registers with rounded adds), 32 MMAs per
// buffer.
// ---------------------------------------------------------------------------

template <int NA, int BKP = BK>
struct PairCfg {
  static constexpr int CHUNK = 64 * BKP * 2;                 // one 64 (MN) x BKP (K) box
  static constexpr int TILE = 2 * CHUNK;                     // one 128 x BKP operand tile
  static constexpr int STAGE_BYTES = (NA + 1) * TILE;        // per CTA
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr int EPI_WARPS = 8;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int ACC_COLS = 512;  // two 256-column buffers
  // 32 MMAs per accumulator buffer (measured: 16 MMAs per buffer cost 3-5 %
  // of the fold in drains; the accumulation bias stays near 2e-6 relative)
  static constexpr int PROMOTE_KB = (NA == 1 ? 8 : 4) * BK / BKP;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the variable at shared::cta address a in CTA rank
__device__ __forceinline__ uint32_t mapa_shared(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t mbar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(mbar_cluster)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t a, uint64_t b,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

// arrive on the barrier at shared::cta offset mbar in both CTAs of the pair
// once every MMA issued so far by this thread has completed
__device__ __forceinline__ void umma_commit_pair(uint32_t mbar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(mbar),
      "h"(mask)
      : "memory");
}

// Arrive on a barrier of either CTA of the pair.  The drained-accumulator
// barrier carries no memory data: the TMEM reads before it are ordered against
// the MMAs after it by the tcgen05 fences on both sides, so the default
// (CTA-scope) semantics suffice; a cluster-scope release here costs a memory
// barrier per epilogue warp and drain.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t mbar_cluster) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(mbar_cluster) : "memory");
}

__host__ __device__ constexpr uint32_t idesc_bf16_mn_m256(int n) {
  return (idesc_bf16_mn(n) & ~(31u << 24)) | ((uint32_t)(256 >> 4) << 24);
}

template <int NA, int BKP>
__global__ void __launch_bounds__(PairCfg<NA, BKP>::THREADS, 1)
    tc_pair_kernel(const __grid_constant__ CUtensorMap ma0, const __grid_constant__ CUtensorMap ma1,
                   const __grid_constant__ CUtensorMap mb0, Params p) {
  using K = PairCfg<NA, BKP>;
  constexpr int PT = 256;  // pair tile edge
  const uint32_t rank = cluster_ctarank();
  int mt, nt;
  // both CTAs of a cluster decode the same pair tile, so they leave or stay together
  if (!decode_tile(blockIdx.x >> 1, p.tiles_m, p.tiles_n, p.symmetric, mt, nt)) return;
  const long long bz = blockIdx.z;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + K::STAGES * K::STAGE_BYTES);
  // bars[0..S): full (used in the leader), [S..2S): empty, [2S..2S+2): accumulator
  // full, [2S+2..2S+4): accumulator drained (used in the leader), [2S+4]: MMA completion
  // after an abort (leader)
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * K::STAGES + 5);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + K::STAGES);
  const uint32_t accf0 = smem_u32(bars + 2 * K::STAGES);
  const uint32_t acce0 = smem_u32(bars + 2 * K::STAGES + 2);
  const uint32_t drain0 = smem_u32(bars + 2 * K::STAGES + 4);
  const int ngroups = (p.num_kb + p.promote_kb - 1) / p.promote_kb;
  const int promote_kb = p.promote_kb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < K::STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf0 + 8 * b, 1);
      mbar_init(acce0 + 8 * b, 2 * K::EPI_WARPS);
    }
    mbar_init(drain0, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(K::ACC_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  fence_after();
  const uint32_t tmem = *tmem_holder;
  const int m0 = mt * PT, n0 = nt * PT;

  int issued = 0;  // k-blocks whose loads this CTA's producer issued
  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full_lead = mapa_shared(full0, 0);
      for (int kb = 0; kb < p.num_kb; ++kb) {
        const int s = kb % K::STAGES;
        const uint32_t ph = (kb / K::STAGES) & 1;
        if (!mbar_wait(empty0 + 8 * s, ph ^ 1, abort_flag, p.status, p.wait_cycles)) break;
        issued = kb + 1;
        // the leader's full[s] expects the bytes of both CTAs; the peer's loads
        // may land first (the transaction count goes transiently negative)
        if (rank == 0) mbar_expect_tx(full0 + 8 * s, 2 * K::STAGE_BYTES);
        const uint32_t fb = full_lead + 8 * s;
        const uint32_t st = smem_u32(smem + s * K::STAGE_BYTES);
        const int ya = (int)(p.ka_batch * bz + p.ka0 + (long long)kb * BKP);
        const int yb = (int)(p.kb_batch * bz + p.kb0 + (long long)kb * BKP);
        const int xa = m0 + 128 * (int)rank;
        const int xb = (int)(p.nb0 + n0) + 128 * (int)rank;
#pragma unroll
        for (int i = 0; i < NA; ++i) {
          const CUtensorMap* m = i == 0 ? &ma0 : &ma1;
          tma_load_2d_pair(st + i * K::TILE, m, xa, ya, fb);
          tma_load_2d_pair(st + i * K::TILE + K::CHUNK, m, xa + 64, ya, fb);
        }
        const uint32_t sb = st + NA * K::TILE;
        tma_load_2d_pair(sb, &mb0, xb, yb, fb);
        tma_load_2d_pair(sb + K::CHUNK, &mb0, xb + 64, yb, fb);
        // warm L2 one ring ahead: the first CTA to reach a token slice otherwise
        // waits for DRAM inside the pipeline
        const int kp = kb + p.prefetch_kb;
        if (p.prefetch_kb > 0 && kp < p.num_kb) {
          const int yap = (int)(p.ka_batch * bz + p.ka0 + (long long)kp * BKP);
          const int ybp = (int)(p.kb_batch * bz + p.kb0 + (long long)kp * BKP);
#pragma unroll
          for (int i = 0; i < NA; ++i) {
            const CUtensorMap* m = i == 0 ? &ma0 : &ma1;
            tma_prefetch_2d(m, xa, yap);
            tma_prefetch_2d(m, xa + 64, yap);
          }
          tma_prefetch_2d(&mb0, xb, ybp);
          tma_prefetch_2d(&mb0, xb + 64, ybp);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = idesc_bf16_mn_m256(PT);
      int kb = 0;
      for (int g = 0; g < ngroups; ++g) {
        const int buf = g & 1;
        const uint32_t use_ph = (uint32_t)((g >> 1) & 1);
        if (!mbar_wait(acce0 + 8 * buf, use_ph ^ 1, abort_flag, p.status, p.wait_cycles)) break;
        fence_after();
        const uint32_t acc_t = tmem + (uint32_t)(buf * PT);
        const int kend = (kb + promote_kb < p.num_kb) ? kb + promote_kb : p.num_kb;
        const int kstart = kb;
        bool ok = true;
        for (; kb < kend; ++kb) {
          const int s = kb % K::STAGES;
          const uint32_t ph = (kb / K::STAGES) & 1;
          if (!mbar_wait(full0 + 8 * s, ph, abort_flag, p.status, p.wait_cycles)) {
            ok = false;
            break;
          }
          fence_after();
          const uint32_t sa = smem_u32(smem + s * K::STAGE_BYTES);
          const uint32_t sb = sa + NA * K::TILE;
#pragma unroll
          for (int kk = 0; kk < BKP / 16; ++kk) {
            const uint32_t off = kk * 2048;  // 16 K rows = two 8-row swizzle groups
            const uint32_t acc0 = (kb > kstart || kk > 0) ? 1u : 0u;
#pragma unroll
            for (int i = 0; i < NA; ++i)
              umma_bf16_pair(acc_t, desc_mn_sw128_lbo(sa + i * K::TILE + off, K::CHUNK),
                             desc_mn_sw128_lbo(sb + off, K::CHUNK), idesc, i == 0 ? acc0 : 1u);
          }
          umma_commit_pair(empty0 + 8 * s);
        }
        if (!ok) break;
        umma_commit_pair(accf0 + 8 * buf);
      }
    }
  } else {
    // epilogue warps of both CTAs: warp w reads TMEM lanes 32 (w % 4) .. + 31 of
    // this CTA's 128 rows; the second four warps take the upper 128 columns
    const int q = warp & 3;
    const int half = (warp - 2) / 4;
    const int row = q * 32 + lane;
    const long long gm = m0 + 128 * (long long)rank + row;
    const uint32_t acce_lead = mapa_shared(acce0, 0);
    float acc[BN];
#pragma unroll
    for (int j = 0; j < BN; ++j) acc[j] = 0.f;
    bool ok = true;
    for (int g = 0; g < ngroups; ++g) {
      const int buf = g & 1;
      const uint32_t use_ph = (uint32_t)((g >> 1) & 1);
      if (ok) ok = mbar_wait(accf0 + 8 * buf, use_ph, abort_flag, p.status, p.wait_cycles);
      fence_after();
      const uint32_t base = tmem + (uint32_t)(buf * PT + half * BN) + ((uint32_t)(q * 32) << 16);
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(base + (uint32_t)(c * 32), r);
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[c * 32 + j] += __uint_as_float(r[j]);
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acce_lead + 8 * buf);
    }
    float* Db = p.D + bz * p.d_bs;
    const bool vec_ok = ((p.ldd & 3) == 0) && ((reinterpret_cast<uintptr_t>(Db) & 15) == 0);
    if (ok && gm < p.M) {
#pragma unroll
      for (int j4 = 0; j4 < BN / 4; ++j4) {
        const long long gn = n0 + half * BN + 4 * j4;
        float v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) v[u] = p.beta * acc[4 * j4 + u];
        EPILOGUE_STORE4
      }
    }
  }
  fence_before();
  __syncthreads();
  if (*abort_flag) {
    // a wait gave up: the leader lets the loads of both CTAs into the stages it
    // armed land (its full barriers count both CTAs' bytes) and its MMAs finish;
    // the peer's loads into stages the leader never armed complete no barrier
    // this CTA can wait on, so the peer allows them a fixed settling time
    if (warp == 0 && lane == 0) {
      if (rank == 0) {
        for (int kb = issued > K::STAGES ? issued - K::STAGES : 0; kb < issued; ++kb)
          mbar_drain(full0 + 8 * (kb % K::STAGES), (kb / K::STAGES) & 1);
      } else if (issued > 0) {
        for (int i = 0; i < 200; ++i) __nanosleep(1000);
      }
    } else if (warp == 1 && lane == 0 && rank == 0) {
      umma_commit_pair(drain0);
      mbar_drain(drain0, 0);
    }
    __syncthreads();
  }
  // neither CTA leaves while the other may still touch its shared memory or TMEM
  cluster_sync();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(K::ACC_COLS)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2-D bf16 tensor [outer, inner] with row stride ld (elements), 64 x 64 boxes.
static bool make_map(CUtensorMap* m, const void* base, long long inner, long long outer,
                     long long ld, bool f16 = false, int box_k = BK) {
  auto enc = encode_fn();
  if (!enc) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * 2) & 15) || inner <= 0 || outer <= 0)
    return false;
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {64, (cuuint32_t)box_k};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
             const_cast<void*>(base), dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

struct Maps {
  CUtensorMap a[3], b[3];
  CUtensorMap d;  // fp32 output for the reduce-add epilogue (Params::red)
};

// 3-D fp32 tensor [batch][M][N] (row stride ldd, batch stride d_bs elements),
// 32 x 32 boxes with 128-byte swizzle: the target of the reduce-add epilogue.
static bool make_map_out(CUtensorMap* m, float* D, long long N, long long M, long long batch,
                         long long ldd, long long d_bs) {
  auto enc = encode_fn();
  if (!enc) return false;
  if (batch <= 1) d_bs = M * ldd;
  if ((reinterpret_cast<uintptr_t>(D) & 15) || ((ldd * 4) & 15) || ((d_bs * 4) & 15) || N <= 0 ||
      M <= 0 || batch <= 0 || ldd < N || d_bs < M * ldd)
    return false;
  cuuint64_t dims[3] = {(cuuint64_t)N, (cuuint64_t)M, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ldd * 4), (cuuint64_t)(d_bs * 4)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, D, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Bound of every pipeline wait of the tensor-core kernels, in SM clock cycles
// (g2q_set_wait_limit); read at each launch.
static volatile long long g_wait_cycles = kWaitCycles;

template <int NA, int NB, bool SMALL, bool WIDE = false>
static int launch(const Maps& m, const Params& p, long long batch, cudaStream_t st) {
  using K = Cfg<NA, NB, SMALL, WIDE>;
  static int attr_done[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return G2Q_ERR_CUDA;
  if (dev >= 64 || !attr_done[dev]) {
    if (cudaFuncSetAttribute(tc_gemm_kernel<NA, NB, SMALL, WIDE>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, K::SMEM) != cudaSuccess)
      return G2Q_ERR_CUDA;
    if (dev < 64) attr_done[dev] = 1;
  }
  Params q = p;
  q.wait_cycles = g_wait_cycles;
  q.promote_kb = K::PROMOTE_KB;
  q.tiles_m = cdiv(p.M, BM);
  q.tiles_n = cdiv(p.N, K::BN_T);
  dim3 grid(q.tiles_n, q.tiles_m, (unsigned)batch);
  if (q.raster) {
    const long long tm = q.tiles_m, tn = q.tiles_n;
    long long n = q.symmetric ? tm * (tm + 1) / 2 : tm * tn;
    if (WIDE && q.symmetric) {
      if (p.M != p.N) return G2Q_ERR_INVALID_ARG;
      n = 0;
      for (int r0 = 0; r0 < q.tiles_m; r0 += GROUP_M)
        n += wide_sym_group_count(r0, (q.tiles_m - r0) < GROUP_M ? (q.tiles_m - r0) : GROUP_M,
                                  q.tiles_n);
    } else if (q.symmetric && tm != tn) {
      return G2Q_ERR_INVALID_ARG;
    }
    if (n > 0x7fffffffLL) return G2Q_ERR_INVALID_ARG;
    grid = dim3((unsigned)n, 1, (unsigned)batch);
  }
  if (grid.y > 65535u || grid.z > 65535u) return G2Q_ERR_INVALID_ARG;
  if (!SMALL || q.symmetric || q.alpha != 1.f) q.red = 0;
  tc_gemm_kernel<NA, NB, SMALL, WIDE><<<grid, K::THREADS, K::SMEM, st>>>(
      m.a[0], m.a[1], m.a[2], m.b[0], m.b[1], m.b[2], m.d, q);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

// L2 prefetch of the operands one pipeline ring ahead in the CTA-pair kernel,
// unless G2PTQ_B200_L2_PREFETCH=0.
static bool pair_prefetch_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("G2PTQ_B200_L2_PREFETCH");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <int NA, int BKP = BK>
static int launch_pair(const Maps& m, const Params& p, long long batch, cudaStream_t st) {
  using K = PairCfg<NA, BKP>;
  static int attr_done[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return G2Q_ERR_CUDA;
  if (dev >= 64 || !attr_done[dev]) {
    if (cudaFuncSetAttribute(tc_pair_kernel<NA, BKP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             K::SMEM) != cudaSuccess)
      return G2Q_ERR_CUDA;
    if (dev < 64) attr_done[dev] = 1;
  }
  Params q = p;
  q.wait_cycles = g_wait_cycles;
  q.promote_kb = K::PROMOTE_KB;
  q.prefetch_kb = pair_prefetch_enabled() ? K::STAGES : 0;
  q.tiles_m = cdiv(p.M, 256);
  q.tiles_n = cdiv(p.N, 256);
  q.red = 0;
  if (q.symmetric && q.tiles_m != q.tiles_n) return G2Q_ERR_INVALID_ARG;
  const long long tm = q.tiles_m, tn = q.tiles_n;
  const long long pairs = q.symmetric ? tm * (tm + 1) / 2 : tm * tn;
  if (2 * pairs > 0x7fffffffLL || batch > 65535) return G2Q_ERR_INVALID_ARG;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, (unsigned)batch);
  cfg.blockDim = dim3(K::THREADS, 1, 1);
  cfg.dynamicSmemBytes = K::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e =
      cudaLaunchKernelEx(&cfg, tc_pair_kernel<NA, BKP>, m.a[0], m.a[1], m.b[0], q);
  g2q::note_launch();
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return G2Q_ERR_CUDA;
  }
  return G2Q_OK;
}

// CTA-pair tiles for long-K bf16 products with a one-term B (the Gram folds),
// unless G2PTQ_B200_PAIR_TILES=0 asks for the single-CTA 128 x 256 tiles.
static bool pair_tiles_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("G2PTQ_B200_PAIR_TILES");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

// K depth per pipeline stage of the CTA-pair Gram: 128 tokens (three 64 KB
// stages per CTA), unless G2PTQ_B200_PAIR_BK=64 asks for 64 (six 32 KB stages).
// Measured at 16384 tokens: 250 vs 302 us at C=4096, 2.81 vs 3.22 ms at 14336;
// each k-block then carries 1024 tensor cycles per SM, twice the fixed cost of
// its full / empty barrier round trip and MMA issue.
static int pair_bk() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("G2PTQ_B200_PAIR_BK");
    v = (e && atoi(e) == 64) ? 64 : 128;
  }
  return v;
}

static int dispatch(int na, int nb, Maps& m, const Params& p, long long batch,
                    cudaStream_t st) {
  for (int i = na; i < 3; ++i) m.a[i] = m.a[0];
  for (int j = nb; j < 3; ++j) m.b[j] = m.b[0];
  const bool small = p.num_kb <= 4;
  if (small) {
    if (na == 2 && nb == 2) return launch<2, 2, true>(m, p, batch, st);
  }
  if (!small && nb == 1 && na <= 2 && !p.f16 && !p.sa && !p.lower && !p.supper &&
      p.nb0 == 0 && p.M >= 512 && p.N >= 512 && pair_tiles_enabled()) {
    if (na == 1) return launch_pair<1>(m, p, batch, st);
    return launch_pair<2>(m, p, batch, st);
  }
  if (na == 1 && nb == 1) return launch<1, 1, false, true>(m, p, batch, st);
  if (na == 1 && nb == 2) return launch<1, 2, false>(m, p, batch, st);
  if (na == 2 && nb == 1) return launch<2, 1, false, true>(m, p, batch, st);
  if (na == 2 && nb == 2) return launch<2, 2, false, true>(m, p, batch, st);
  return G2Q_ERR_UNSUPPORTED;
}

template <typename S>
__global__ void split_rows_kernel(const S* X, long long ldx, long long T, long long C,
                                  const float* s, long long sstride, __nv_bfloat16* hi,
                                  __nv_bfloat16* lo, long long ldo) {
  for (long long t = blockIdx.y; t < T; t += gridDim.y) {
    const float f = s ? s[t * sstride] : 1.f;
    for (long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x; c < C;
         c += (long long)gridDim.x * blockDim.x) {
      float v;
      if constexpr (sizeof(S) == 2) v = __bfloat162float(X[t * ldx + c]);
      else v = X[t * ldx + c];
      if (s) v *= f;
      __nv_bfloat16 h, l;
      split_bf16(v, &h, &l);
      hi[t * ldo + c] = h;
      if (lo) lo[t * ldo + c] = l;
    }
  }
}

static int split_rows(const void* X, int dtype, long long ldx, long long T, long long C,
                      const float* s, long long sstride, __nv_bfloat16* hi, __nv_bfloat16* lo,
                      long long ldo, cudaStream_t st) {
  if (T * C == 0) return G2Q_OK;
  const dim3 grid = wave_grid_2d(T, C);
  if (dtype == G2Q_DTYPE_BF16)
    split_rows_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(
        (const __nv_bfloat16*)X, ldx, T, C, s, sstride, hi, lo, ldo);
  else
    split_rows_kernel<float><<<grid, 256, 0, st>>>((const float*)X, ldx, T, C, s, sstride, hi,
                                                   lo, ldo);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

static long long round8(long long v) { return (v + 7) / 8 * 8; }

// hi[g] / lo[g] ([T][ldo] each, group g at offset g * gstride) = bf16 pair of
// X[t][c] * s[t * sstride + g] for all G row groups in one pass over X, eight
// columns (16 bytes of bf16 in, 16 bytes per term out) per thread.
__global__ void __launch_bounds__(256) split_rows_groups_kernel(
    const __nv_bfloat16* __restrict__ X, long long ldx, long long T, long long C,
    const float* __restrict__ s, long long sstride, int G, __nv_bfloat16* hi, __nv_bfloat16* lo,
    long long ldo, long long gstride) {
  const long long nv = C / 8;
  for (long long t = blockIdx.y; t < T; t += gridDim.y) {
    for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < nv;
         v += (long long)gridDim.x * blockDim.x) {
      const uint4 raw = *reinterpret_cast<const uint4*>(X + t * ldx + v * 8);
      const __nv_bfloat16* xb = reinterpret_cast<const __nv_bfloat16*>(&raw);
      float x[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) x[u] = __bfloat162float(xb[u]);
      for (int g = 0; g < G; ++g) {
        const float sg = s[t * sstride + g];
        uint4 h4, l4;
        __nv_bfloat16* hp = reinterpret_cast<__nv_bfloat16*>(&h4);
        __nv_bfloat16* lp = reinterpret_cast<__nv_bfloat16*>(&l4);
#pragma unroll
        for (int u = 0; u < 8; ++u) split_bf16(x[u] * sg, &hp[u], &lp[u]);
        const long long o = g * gstride + t * ldo + v * 8;
        *reinterpret_cast<uint4*>(hi + o) = h4;
        *reinterpret_cast<uint4*>(lo + o) = l4;
      }
    }
  }
}

}  // namespace tc

size_t tc_gram_workspace_bytes(long long M, long long N, long long T) {
  const long long w = tc::round8(M > N ? M : N);
  return (size_t)(4 * T * w * 2 + 4 * 256);
}


// Gram update on tensor cores (see g2q_gram_update).  Falls back to the fp32
// CUDA-core kernel where TMA cannot describe the operands (row strides that
// are not a multiple of 8 elements, misaligned bases) or there is no work.
int tc_gram(float* D, long long ldd, long long M, long long N, const void* A, int a_dtype,
            long long lda, const void* B, int b_dtype, long long ldb, const float* row_scale,
            long long scale_stride, long long T, int symmetric, float alpha, float beta,
            void* workspace, size_t workspace_bytes, int* status, cudaStream_t st) {
  SimtArgs sa{};
  sa.A = A; sa.B = B; sa.C = D;
  sa.lda = lda; sa.ldb = ldb; sa.ldc = ldd;
  sa.M = M; sa.N = N; sa.K = T;
  sa.alpha = alpha; sa.beta = beta;
  sa.kscale = row_scale; sa.kscale_stride = scale_stride;
  sa.mirror = symmetric ? 1 : 0;
  if (T == 0 || !tc::encode_fn()) return simt_gemm(sa, true, false, a_dtype, b_dtype, 1, st);
  const long long w = tc::round8(M > N ? M : N);
  char* ws = (char*)workspace;
  auto take = [&](long long elems) -> __nv_bfloat16* {
    uintptr_t p = ((uintptr_t)ws + 255) & ~(uintptr_t)255;
    ws = (char*)p + elems * 2;
    return (__nv_bfloat16*)p;
  };
  const void* a_terms[2] = {A, nullptr};
  const void* b_terms[2] = {B, nullptr};
  long long lda_t = lda, ldb_t = ldb;
  int na = 1, nb = 1;
  const bool same = (A == B) && (a_dtype == b_dtype) && !row_scale;
  if (symmetric && row_scale && A == B && a_dtype == G2Q_DTYPE_BF16 &&
      b_dtype == G2Q_DTYPE_BF16) {
    // X^T diag(s) X of BF16 tokens: the scaled operand (split into a bf16 pair)
    // goes on the M side and X stays exact on the N side, so the product runs
    // on the 128 x 256 tiles with two MMAs per K step
    if (!workspace || workspace_bytes < tc_gram_workspace_bytes(M, N, T))
      return G2Q_ERR_INVALID_ARG;
    __nv_bfloat16* hi = take(T * w);
    __nv_bfloat16* lo = take(T * w);
    G2Q_TRY(tc::split_rows(A, a_dtype, lda, T, M, row_scale, scale_stride, hi, lo, w, st));
    tc::Maps mp{};
    bool ok = tc::make_map(&mp.a[0], hi, M, T, w) && tc::make_map(&mp.a[1], lo, M, T, w) &&
              tc::make_map(&mp.b[0], B, N, T, ldb);
    if (!ok) return simt_gemm(sa, true, false, a_dtype, b_dtype, 1, st);
    tc::Params p{};
    p.status = status;
    p.D = D; p.ldd = ldd; p.d_bs = 0;
    p.M = M; p.N = N;
    p.num_kb = (int)((T + tc::BK - 1) / tc::BK);
    p.alpha = alpha; p.beta = beta;
    p.symmetric = 1;
    p.raster = 1;
    return tc::dispatch(2, 1, mp, p, 1, st);
  }
  if (a_dtype != G2Q_DTYPE_BF16) {
    if (!workspace || workspace_bytes < tc_gram_workspace_bytes(M, N, T))
      return G2Q_ERR_INVALID_ARG;
    __nv_bfloat16* hi = take(T * w);
    __nv_bfloat16* lo = take(T * w);
    G2Q_TRY(tc::split_rows(A, a_dtype, lda, T, M, nullptr, 0, hi, lo, w, st));
    a_terms[0] = hi;
    a_terms[1] = lo;
    lda_t = w;
    na = 2;
  }
  if (same) {
    b_terms[0] = a_terms[0];
    b_terms[1] = a_terms[1];
    ldb_t = lda_t;
    nb = na;
  } else if (b_dtype != G2Q_DTYPE_BF16 || row_scale) {
    if (!workspace || workspace_bytes < tc_gram_workspace_bytes(M, N, T))
      return G2Q_ERR_INVALID_ARG;
    __nv_bfloat16* hi = take(T * w);
    __nv_bfloat16* lo = take(T * w);
    G2Q_TRY(tc::split_rows(B, b_dtype, ldb, T, N, row_scale, scale_stride, hi, lo, w, st));
    b_terms[0] = hi;
    b_terms[1] = lo;
    ldb_t = w;
    nb = 2;
  }
  if (na == 1 && nb == 1 && M >= 512 && N >= 512 && T > 4 * 128 && tc::pair_tiles_enabled() &&
      tc::pair_bk() == 128) {
    // CTA pairs with 128 tokens per pipeline stage (half the barrier round
    // trips per MMA of the 64-token stages)
    tc::Maps mp{};
    if (tc::make_map(&mp.a[0], a_terms[0], M, T, lda_t, false, 128) &&
        tc::make_map(&mp.b[0], b_terms[0], N, T, ldb_t, false, 128)) {
      mp.a[1] = mp.a[0];
      tc::Params p{};
      p.status = status;
      p.D = D; p.ldd = ldd; p.d_bs = 0;
      p.M = M; p.N = N;
      p.num_kb = (int)((T + 127) / 128);
      p.alpha = alpha; p.beta = beta;
      p.symmetric = symmetric ? 1 : 0;
      p.raster = 1;
      return tc::launch_pair<1, 128>(mp, p, 1, st);
    }
  }
  tc::Maps mp{};
  bool ok = tc::make_map(&mp.a[0], a_terms[0], M, T, lda_t) &&
            tc::make_map(&mp.b[0], b_terms[0], N, T, ldb_t);
  ok = ok && (na == 1 || tc::make_map(&mp.a[1], a_terms[1], M, T, lda_t));
  ok = ok && (nb == 1 || tc::make_map(&mp.b[1], b_terms[1], N, T, ldb_t));
  if (!ok) return simt_gemm(sa, true, false, a_dtype, b_dtype, 1, st);
  tc::Params p{};
  p.status = status;
  p.D = D; p.ldd = ldd; p.d_bs = 0;
  p.M = M; p.N = N;
  p.num_kb = (int)((T + tc::BK - 1) / tc::BK);
  p.alpha = alpha; p.beta = beta;
  p.symmetric = symmetric ? 1 : 0;
  p.raster = 1;
  return tc::dispatch(na, nb, mp, p, 1, st);
}

size_t tc_gram_grouped_workspace_bytes(long long C, long long T, int G) {
  const size_t grouped = (size_t)2 * G * T * tc::round8(C) * 2 + 4 * 256;
  const size_t single = tc_gram_workspace_bytes(C, C, T);
  return grouped > single ? grouped : single;
}

// Row-scaled symmetric Gram updates of G row groups (see g2q_gram_update_grouped):
// BF16 tokens are split for all groups in one pass and the G products run as
// one batched CTA-pair launch (blockIdx.z = group); other inputs take the
// per-group path.
int tc_gram_grouped(float* D, long long ldd, long long d_gstride, long long C, const void* X,
                    int x_dtype, long long ldx, const float* s, long long sstride, int G,
                    long long T, float alpha, float beta, void* workspace,
                    size_t workspace_bytes, int* status, cudaStream_t st) {
  const bool fast = x_dtype == G2Q_DTYPE_BF16 && T > 0 && C >= 512 && (C % 8) == 0 &&
                    (ldx % 8) == 0 && ((reinterpret_cast<uintptr_t>(X) & 15) == 0) && G <= 65535 &&
                    tc::encode_fn() && tc::pair_tiles_enabled() &&
                    workspace_bytes >= tc_gram_grouped_workspace_bytes(C, T, G);
  if (fast) {
    const long long w = tc::round8(C);
    char* ws = (char*)workspace;
    auto take = [&](long long elems) -> __nv_bfloat16* {
      uintptr_t q = ((uintptr_t)ws + 255) & ~(uintptr_t)255;
      ws = (char*)q + elems * 2;
      return (__nv_bfloat16*)q;
    };
    __nv_bfloat16* hi = take((long long)G * T * w);
    __nv_bfloat16* lo = take((long long)G * T * w);
    const long long nv = C / 8;
    const dim3 grid = wave_grid_2d(T, nv);
    tc::split_rows_groups_kernel<<<grid, 256, 0, st>>>((const __nv_bfloat16*)X, ldx, T, C, s,
                                                       sstride, G, hi, lo, w, T * w);
    G2Q_CHECK_LAUNCH();
    tc::Maps mp{};
    // the groups' scaled tokens stacked along K: group g's k-block y sits at
    // row g * T + y; a last partial k-block reads the next group's first rows,
    // which meet X's zero-filled rows past T and add nothing
    if (tc::make_map(&mp.a[0], hi, C, (long long)G * T, w) &&
        tc::make_map(&mp.a[1], lo, C, (long long)G * T, w) &&
        tc::make_map(&mp.b[0], X, C, T, ldx)) {
      tc::Params p{};
      p.status = status;
      p.D = D; p.ldd = ldd; p.d_bs = d_gstride;
      p.M = C; p.N = C;
      p.num_kb = (int)((T + tc::BK - 1) / tc::BK);
      p.ka_batch = T; p.kb_batch = 0;
      p.alpha = alpha; p.beta = beta;
      p.symmetric = 1;
      p.raster = 1;
      return tc::launch_pair<2>(mp, p, G, st);
    }
  }
  for (int g = 0; g < G; ++g)
    G2Q_TRY(tc_gram(D + g * d_gstride, ldd, C, C, X, x_dtype, ldx, X, x_dtype, ldx, s + g, sstride,
                    T, 1, alpha, beta, workspace, workspace_bytes, status, st));
  return G2Q_OK;
}


// ---------------------------------------------------------------------------
// fp32-accurate batched GEMM on tensor cores (the fp32 products of fasterquant:
// G2PTQ's Z / GHinv chain and GPTAQ's P).  Each operand is carried as an fp16
// hi/lo pair, MN-major [batch][Kp][Mp] in the workspace, every output row
// (column) scaled by the power of two that puts its largest magnitude over K in
// [2^14, 2^15); the scales are undone exactly in the epilogue.
// ---------------------------------------------------------------------------

// Largest |x| of every output index of op(X) over K: kmajor != 0 means X is
// stored [n][K] (one row per output index, one warp each), else [K][n] (one
// column each: a CTA takes 32 columns, its eight warps eight interleaved
// slices of K, combined in shared memory).
__global__ void op_absmax_kernel(const float* __restrict__ X, long long ldx, long long xbs,
                                 long long n, long long K, int kmajor, float* fac,
                                 float* inv, long long obs) {
  const int b = blockIdx.y;
  const float* xb = X + (long long)b * xbs;
  float m = 0.f;
  long long i;
  if (kmajor) {
    i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (i < n)
      for (long long k = lane; k < K; k += 32) m = fmaxf(m, fabsf(xb[i * ldx + k]));
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane != 0) return;
  } else {
    __shared__ float part[8][32];
    const int lane = threadIdx.x & 31, ws = threadIdx.x >> 5;
    i = (long long)blockIdx.x * 32 + lane;
    if (i < n)
      for (long long k = ws; k < K; k += 8) m = fmaxf(m, fabsf(xb[k * ldx + i]));
    part[ws][lane] = m;
    __syncthreads();
    if (ws != 0) return;
#pragma unroll
    for (int q = 1; q < 8; ++q) m = fmaxf(m, part[q][lane]);
  }
  if (i >= n) return;
  float f = 1.f, v = 1.f;
  if (m > 0.f && m <= 3.0e38f) {
    int e;
    frexpf(m, &e);
    e = e < -100 ? -100 : e;
    f = ldexpf(1.f, 15 - e);
    v = ldexpf(1.f, e - 15);
  }
  fac[(long long)b * obs + i] = f;
  inv[(long long)b * obs + i] = v;
}

// out[b][k][i] = fp16 hi/lo of op(X)[i][k] * fac[b][i] for k < K, i < n; zero
// padding up to Kp rows (so that one batch's K tiles never read the next's).
__global__ void op_split_kernel(const float* __restrict__ X, long long ldx, long long xbs,
                                long long n, long long K, long long Kp, int kmajor,
                                const float* fac, long long obs, __half* hi, __half* lo,
                                long long ldo, long long out_bs) {
  __shared__ float tile[32][33];
  const int b = blockIdx.z;
  const long long i0 = (long long)blockIdx.x * 32, k0 = (long long)blockIdx.y * 32;
  const float* xb = X + (long long)b * xbs;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    if (kmajor) {  // rows of X are output indices: read along k, transpose
      const long long i = i0 + r, k = k0 + threadIdx.x;
      tile[threadIdx.x][r] = (i < n && k < K) ? xb[i * ldx + k] : 0.f;
    } else {
      const long long k = k0 + r, i = i0 + threadIdx.x;
      tile[r][threadIdx.x] = (i < n && k < K) ? xb[k * ldx + i] : 0.f;
    }
  }
  __syncthreads();
  const long long i = i0 + threadIdx.x;
  if (i >= n) return;
  const float f = fac[(long long)b * obs + i];
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const long long k = k0 + r;
    if (k >= Kp) continue;
    const float v = tile[r][threadIdx.x] * f;
    const __half h = __float2half_rn(v);
    const long long o = (long long)b * out_bs + k * ldo + i;
    hi[o] = h;
    lo[o] = __float2half_rn(v - __half2float(h));
  }
}

// C[b][m][n] = 0 for m >= n (the part a strictly-upper product does not write).
__global__ void zero_lower_kernel(float* C, long long ldc, long long cbs, long long M,
                                  long long N) {
  const int b = blockIdx.y;
  const long long n_el = M * N;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < n_el;
       idx += (long long)gridDim.x * blockDim.x) {
    const long long m = idx / N, nn = idx - m * N;
    if (m >= nn) C[(long long)b * cbs + m * ldc + nn] = 0.f;
  }
}

namespace tc {
static long long round64(long long v) { return (v + 63) / 64 * 64; }

struct OpLayout {
  long long batches, n, Kp, ldo;
  size_t terms_bytes() const { return (size_t)batches * Kp * ldo * sizeof(__half); }
};

static OpLayout op_layout(long long n, long long K, long long batches) {
  return OpLayout{batches, n, round64(K), round8(n)};
}
}  // namespace tc

size_t gemm_tc_workspace_bytes(long long M, long long N, long long K, long long batch_a,
                               long long batch_b) {
  const tc::OpLayout a = tc::op_layout(M, K, batch_a), b = tc::op_layout(N, K, batch_b);
  return 2 * a.terms_bytes() + 2 * b.terms_bytes() +
         (size_t)(2 * batch_a * M + 2 * batch_b * N) * sizeof(float) + 8 * 256;
}

// C <- alpha C + beta op(A) op(B), batched, fp32 in and out, on tensor cores.
// mask: G2Q_MASK_FULL, G2Q_MASK_LOWER or G2Q_MASK_STRICT_UPPER (the rest set to
// zero).  Returns G2Q_ERR_UNSUPPORTED where TMA cannot describe the operands.
int gemm_tc_f32(float* C, long long ldc, long long sC, const float* A, long long lda,
                long long sA, bool ta, const float* B, long long ldb, long long sB, bool tb,
                long long M, long long N, long long K, long long batch, float alpha, float beta,
                int mask, void* workspace, size_t workspace_bytes, int* status, cudaStream_t st) {
  if (M <= 0 || N <= 0 || batch <= 0) return G2Q_OK;
  if (K <= 0 || !tc::encode_fn() || (mask != G2Q_MASK_FULL && mask != G2Q_MASK_LOWER &&
                                     mask != G2Q_MASK_STRICT_UPPER))
    return G2Q_ERR_UNSUPPORTED;
  const long long ba = sA ? batch : 1, bb = sB ? batch : 1;
  if (!workspace || workspace_bytes < gemm_tc_workspace_bytes(M, N, K, ba, bb))
    return G2Q_ERR_INVALID_ARG;
  if (batch > 65535 || ((ldc * 4) & 15) || (reinterpret_cast<uintptr_t>(C) & 15))
    return G2Q_ERR_UNSUPPORTED;
  const tc::OpLayout la = tc::op_layout(M, K, ba), lb = tc::op_layout(N, K, bb);
  char* ws = (char*)workspace;
  auto take = [&](size_t bytes) {
    char* q = (char*)(((uintptr_t)ws + 255) & ~(uintptr_t)255);
    ws = q + bytes;
    return q;
  };
  __half* a_hi = (__half*)take(la.terms_bytes());
  __half* a_lo = (__half*)take(la.terms_bytes());
  __half* b_hi = (__half*)take(lb.terms_bytes());
  __half* b_lo = (__half*)take(lb.terms_bytes());
  float* fa = (float*)take(ba * M * sizeof(float));
  float* ia = (float*)take(ba * M * sizeof(float));
  float* fb = (float*)take(bb * N * sizeof(float));
  float* ib = (float*)take(bb * N * sizeof(float));
  // op(A)[m][k]: A stored [M][K] (k contiguous) unless ta; op(B)[k][n]: B stored
  // [K][N] (n contiguous) unless tb.
  const int a_kmajor = ta ? 0 : 1, b_kmajor = tb ? 1 : 0;
  op_absmax_kernel<<<dim3(a_kmajor ? cdiv(M * 32, 256) : cdiv(M, 32), (unsigned)ba), 256, 0,
                     st>>>(A, lda, sA, M, K, a_kmajor, fa, ia, M);
  G2Q_CHECK_LAUNCH();
  op_absmax_kernel<<<dim3(b_kmajor ? cdiv(N * 32, 256) : cdiv(N, 32), (unsigned)bb), 256, 0,
                     st>>>(B, ldb, sB, N, K, b_kmajor, fb, ib, N);
  G2Q_CHECK_LAUNCH();
  op_split_kernel<<<dim3(cdiv(M, 32), cdiv(la.Kp, 32), (unsigned)ba), dim3(32, 8), 0, st>>>(
      A, lda, sA, M, K, la.Kp, a_kmajor, fa, M, a_hi, a_lo, la.ldo, la.Kp * la.ldo);
  G2Q_CHECK_LAUNCH();
  op_split_kernel<<<dim3(cdiv(N, 32), cdiv(lb.Kp, 32), (unsigned)bb), dim3(32, 8), 0, st>>>(
      B, ldb, sB, N, K, lb.Kp, b_kmajor, fb, N, b_hi, b_lo, lb.ldo, lb.Kp * lb.ldo);
  G2Q_CHECK_LAUNCH();
  if (mask == G2Q_MASK_STRICT_UPPER) {
    long long blocks = (M * N + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    zero_lower_kernel<<<dim3((unsigned)blocks, (unsigned)batch), 256, 0, st>>>(C, ldc, sC, M, N);
    G2Q_CHECK_LAUNCH();
  }
  tc::Maps mp{};
  bool ok = tc::make_map(&mp.a[0], a_hi, M, ba * la.Kp, la.ldo, true) &&
            tc::make_map(&mp.a[1], a_lo, M, ba * la.Kp, la.ldo, true) &&
            tc::make_map(&mp.b[0], b_hi, N, bb * lb.Kp, lb.ldo, true) &&
            tc::make_map(&mp.b[1], b_lo, N, bb * lb.Kp, lb.ldo, true);
  if (!ok) return G2Q_ERR_UNSUPPORTED;
  tc::Params p{};
  p.status = status;
  p.D = C; p.ldd = ldc; p.d_bs = sC;
  p.M = M; p.N = N;
  p.num_kb = (int)(la.Kp / tc::BK);
  p.ka_batch = ba > 1 ? la.Kp : 0;
  p.kb_batch = bb > 1 ? lb.Kp : 0;
  p.alpha = alpha; p.beta = beta;
  p.lower = mask == G2Q_MASK_LOWER;
  p.supper = mask == G2Q_MASK_STRICT_UPPER;
  p.f16 = 1;
  p.sa = ia; p.sb = ib;
  p.sa_bs = ba > 1 ? M : 0;
  p.sb_bs = bb > 1 ? N : 0;
  p.red = (alpha == 1.f && tc::make_map_out(&mp.d, C, N, M, batch, ldc, sC)) ? 1 : 0;
  return tc::dispatch(2, 2, mp, p, batch, st);
}

// Two-term fp16 split of a K x (rows or cols) fp32 block for the fp32-accurate
// updates of the Cholesky chain.  Each output row (M or N index) is scaled by a
// power of two that puts its largest magnitude in [2^14, 2^15), so both terms
// keep 11 significant bits each (22 together) whatever the row's scale; the
// inverse scale is written to `scale` and applied exactly in the epilogue.
//   transpose != 0: src is [rows][K] (row stride lds), dst [K][rows], one scale
//                   per src row (the operand L21 of the SYRK and of the Y update);
//   transpose == 0: src is [K][cols] (row stride lds), dst [K][cols], one scale
//                   per column (the operand X_k of the Y update).
// One block handles 32 rows (or columns) and all K <= 128 of them.
// Batched over grid y and z: block (y, z) reads src + y * src_by + z * src_bz and
// writes hi / lo + y * dst_by + z * dst_bz and scale + y * sc_by + z * sc_bz.
__global__ void __launch_bounds__(256) split2h_kernel(const float* __restrict__ src,
                                                      long long lds, long long n, int K,
                                                      __half* hi, __half* lo, long long ldd,
                                                      float* scale, int transpose,
                                                      long long src_by, long long dst_by,
                                                      long long sc_by, long long src_bz,
                                                      long long dst_bz, long long sc_bz) {
  src += blockIdx.y * src_by + blockIdx.z * src_bz;
  hi += blockIdx.y * dst_by + blockIdx.z * dst_bz;
  lo += blockIdx.y * dst_by + blockIdx.z * dst_bz;
  scale += blockIdx.y * sc_by + blockIdx.z * sc_bz;
  __shared__ float tile[128][33];
  __shared__ float smax[8][32];
  __shared__ float sfac[32];
  const int x = threadIdx.x, y = threadIdx.y;
  const long long n0 = (long long)blockIdx.x * 32;
  const long long ni = n0 + x;
  // sixteen loads of a thread in flight before their shared-memory stores
  if (transpose) {
    // source rows n0..n0+31, K long each: lanes walk k (coalesced), warp y takes
    // rows y, y+8, ...
#pragma unroll 1
    for (int k0 = 0; k0 < K; k0 += 128) {
      float v[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const long long r = n0 + y + 8 * a;
          const int k = k0 + x + 32 * b;
          v[a][b] = (r < n && k < K) ? src[r * lds + k] : 0.f;
        }
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int k = k0 + x + 32 * b;
          if (k < K) tile[k][y + 8 * a] = v[a][b];
        }
    }
  } else {
#pragma unroll 1
    for (int k0 = 0; k0 < K; k0 += 128) {
      float v[16];
#pragma unroll
      for (int a = 0; a < 16; ++a) {
        const int k = k0 + y + 8 * a;
        v[a] = (ni < n && k < K) ? src[(long long)k * lds + ni] : 0.f;
      }
#pragma unroll
      for (int a = 0; a < 16; ++a) {
        const int k = k0 + y + 8 * a;
        if (k < K) tile[k][x] = v[a];
      }
    }
  }
  __syncthreads();
  float m = 0.f;
  for (int k = y; k < K; k += 8) m = fmaxf(m, fabsf(tile[k][x]));
  smax[y][x] = m;
  __syncthreads();
  if (y == 0) {
    float mm = smax[0][x];
#pragma unroll
    for (int q = 1; q < 8; ++q) mm = fmaxf(mm, smax[q][x]);
    float f = 1.f, inv = 1.f;
    if (mm > 0.f && mm <= 3.0e38f) {
      int e;
      frexpf(mm, &e);  // mm in [2^(e-1), 2^e)
      f = ldexpf(1.f, 15 - e);
      inv = ldexpf(1.f, e - 15);
    }
    sfac[x] = f;
    if (ni < n) scale[ni] = inv;
  }
  __syncthreads();
  const float f = sfac[x];
  if (ni < n) {
    for (int k = y; k < K; k += 8) {
      const float v = tile[k][x] * f;
      const __half h = __float2half_rn(v);
      hi[(long long)k * ldd + ni] = h;
      lo[(long long)k * ldd + ni] = __float2half_rn(v - __half2float(h));
    }
  }
}

// The split of ny x nz strips in one launch (strip (y, z) at the given strides).
int split2h_strips(const float* src, long long lds, long long n, int K, __half* hi, __half* lo,
                   long long ldd, float* scale, int transpose, int ny, long long src_by,
                   long long dst_by, long long sc_by, int nz, long long src_bz,
                   long long dst_bz, long long sc_bz, cudaStream_t st) {
  if (n <= 0 || K <= 0 || ny <= 0 || nz <= 0) return G2Q_OK;
  if (K > 128 || ny > 65535 || nz > 65535) return G2Q_ERR_INVALID_ARG;
  split2h_kernel<<<dim3(cdiv(n, 32), ny, nz), dim3(32, 8), 0, st>>>(
      src, lds, n, K, hi, lo, ldd, scale, transpose, src_by, dst_by, sc_by, src_bz, dst_bz,
      sc_bz);
  G2Q_CHECK_LAUNCH();
  return G2Q_OK;
}

// D[b][m][n] += beta sa[b][m] sb[b][n] sum_k A[b][k][m] B[b][k][n] over fp16 hi/lo pairs
// (three products), batched: A's k-rows of batch b start at ka_batch b + ka0 in a
// [a_outer][lda] tensor (M contiguous), B's at kb_batch b + kb0 in [b_outer][ldb]
// (columns from nb0, b_inner wide).  The short-K tensor-core update of the lazy
// compensation on pre-split operands.  Returns G2Q_ERR_UNSUPPORTED where TMA
// cannot describe the operands.
int tc_update_f16(float* D, long long ldd, long long d_bs, long long M, long long N, int K,
                  long long batch, __half* const* a2, long long lda, long long a_outer,
                  long long ka_batch, long long ka0, const float* sa, long long sa_bs,
                  __half* const* b2, long long ldb, long long b_inner, long long b_outer,
                  long long kb_batch, long long kb0, long long nb0, const float* sb,
                  long long sb_bs, float beta, int* status, cudaStream_t st) {
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0) return G2Q_OK;
  if ((K % tc::BK) || !tc::encode_fn()) return G2Q_ERR_UNSUPPORTED;
  tc::Maps mp{};
  bool ok = true;
  for (int i = 0; i < 2 && ok; ++i)
    ok = tc::make_map(&mp.a[i], a2[i], M, a_outer, lda, true) &&
         tc::make_map(&mp.b[i], b2[i], b_inner, b_outer, ldb, true);
  if (!ok) return G2Q_ERR_UNSUPPORTED;
  tc::Params p{};
  p.status = status;
  p.D = D; p.ldd = ldd; p.d_bs = d_bs;
  p.M = M; p.N = N;
  p.num_kb = K / tc::BK;
  p.ka_batch = ka_batch; p.ka0 = ka0;
  p.kb_batch = kb_batch; p.kb0 = kb0; p.nb0 = nb0;
  p.alpha = 1.f; p.beta = beta;
  p.f16 = 1;
  p.sa = sa; p.sb = sb; p.sa_bs = sa_bs; p.sb_bs = sb_bs;
  p.red = tc::make_map_out(&mp.d, D, N, M, batch, ldd, d_bs) ? 1 : 0;
  return tc::dispatch(2, 2, mp, p, batch, st);
}

// fp32-accurate tensor-core update  D <- alpha D + beta * diag(sa) A^T B diag(sb)
// for MN-major two-term fp16 operands A[k][m] (terms a2, row stride lda) and
// B[k][n] (b2, ldb) over K rows (three products: hi*hi, hi*lo, lo*hi); lower != 0
// writes only m >= n.  Batched (batch > 1): entry b's K rows of A and B start at
// row b k_bs of a2 / b2 (k_bs >= K, K a multiple of the K tile), its output at
// D + b d_bs, its scales at sa + b sa_bs and sb + b sb_bs.  Returns
// G2Q_ERR_UNSUPPORTED when TMA cannot describe the operands.
int tc_update2h(float* D, long long ldd, long long M, long long N, long long K,
                __half* const* a2, const float* sa, long long lda, __half* const* b2,
                const float* sb, long long ldb, int lower, float alpha, float beta,
                int* status, cudaStream_t st, long long batch, long long k_bs, long long d_bs,
                long long sa_bs, long long sb_bs) {
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0 || !tc::encode_fn()) return G2Q_ERR_UNSUPPORTED;
  if (batch > 1 && ((K % tc::BK) || k_bs < K || d_bs < M * ldd)) return G2Q_ERR_INVALID_ARG;
  // rows of the operand maps: every batch entry's K rows
  const long long rows = batch > 1 ? (batch - 1) * k_bs + K : K;
  tc::Maps mp{};
  bool ok = true;
  for (int i = 0; i < 2 && ok; ++i)
    ok = tc::make_map(&mp.a[i], a2[i], M, rows, lda, true) &&
         tc::make_map(&mp.b[i], b2[i], N, rows, ldb, true);
  if (!ok) return G2Q_ERR_UNSUPPORTED;
  tc::Params p{};
  p.status = status;
  p.D = D; p.ldd = ldd; p.d_bs = batch > 1 ? d_bs : 0;
  p.M = M; p.N = N;
  p.num_kb = (int)((K + tc::BK - 1) / tc::BK);
  p.ka_batch = batch > 1 ? k_bs : 0;
  p.kb_batch = batch > 1 ? k_bs : 0;
  p.alpha = alpha; p.beta = beta;
  p.lower = lower;
  p.f16 = 1;
  p.sa = sa; p.sb = sb;
  p.sa_bs = batch > 1 ? sa_bs : 0;
  p.sb_bs = batch > 1 ? sb_bs : 0;
  p.red = (alpha == 1.f && tc::make_map_out(&mp.d, D, N, M, batch, ldd, p.d_bs)) ? 1 : 0;
  return tc::dispatch(2, 2, mp, p, batch, st);
}

}  // namespace g2q

extern "C" size_t g2q_gemm_tc_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t batch,
                                              int a_batched, int b_batched) {
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0) return 0;
  return g2q::gemm_tc_workspace_bytes(M, N, K, a_batched ? batch : 1, b_batched ? batch : 1);
}

extern "C" int g2q_gemm_tc(float* C, int64_t ldc, int64_t strideC, const float* A, int64_t lda,
                           int64_t strideA, int transA, const float* B, int64_t ldb,
                           int64_t strideB, int transB, int64_t M, int64_t N, int64_t K,
                           int64_t batch, float alpha, float beta, int out_mask, void* workspace,
                           size_t workspace_bytes, int* status, void* stream) {
  if (!C || (!A && K > 0) || (!B && K > 0) || M < 0 || N < 0 || K < 0 || batch < 0)
    return G2Q_ERR_INVALID_ARG;
  if (out_mask < 0 || out_mask > 3) return G2Q_ERR_INVALID_ARG;
  cudaStream_t st = (cudaStream_t)stream;
  const int s = g2q::gemm_tc_f32(C, ldc, strideC, A, lda, strideA, transA != 0, B, ldb, strideB,
                                 transB != 0, M, N, K, batch, alpha, beta, out_mask, workspace,
                                 workspace_bytes, status, st);
  if (s != G2Q_ERR_UNSUPPORTED) return s;
  // shapes TMA cannot describe, or the inclusive upper mask: fp32 CUDA cores
  g2q::SimtArgs a{};
  a.A = A; a.B = B; a.C = C;
  a.lda = lda; a.ldb = ldb; a.ldc = ldc;
  a.sA = strideA; a.sB = strideB; a.sC = strideC;
  a.M = M; a.N = N; a.K = K;
  a.alpha = alpha; a.beta = beta;
  a.mask = out_mask;
  return g2q::simt_gemm(a, transA != 0, transB != 0, G2Q_DTYPE_F32, G2Q_DTYPE_F32, batch, st);
}

extern "C" int64_t g2q_set_wait_limit(int64_t cycles) {
  const long long prev = g2q::tc::g_wait_cycles;
  g2q::tc::g_wait_cycles = cycles > 0 ? cycles : g2q::tc::kWaitCycles;
  return prev;
}
