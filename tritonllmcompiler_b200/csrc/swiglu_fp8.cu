// FP8 (e4m3) SwiGLU dual GEMM for sm_100a: out = silu(sx*s1 * x@w1) * (sx*s3 * x@w3).
//
// Extension of the reference's fp16 swiglu (python/triton_llm/ops/swiglu.py:54-76; oracle
// python/triton_llm/reference/swiglu.py:12-15) to 8-bit inputs with per-tensor scales, the
// tcgen05 kind::f8f6f4 path (twice the dense fp16 rate on B200). The weights are given
// transposed, w1t/w3t [N, K] with K contiguous (the layout FP8 weights are usually stored
// in), so both UMMA operands are K-major.
//
// Same structure as swiglu.cu: persistent, one CTA per SM; warp 0 TMA (x tile 128 x 128 bytes,
// w1t and w3t tiles 128 x 128 bytes side by side -> one 256-row B operand), warp 1 issues
// 128x256x32 UMMAs into double-buffered TMEM accumulators, warps 2-5 apply the scales,
// silu(g)*u in fp32 and store fp16/bf16. Every wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "common.h"
#include "ptx.cuh"

namespace tllm {

__device__ int g_swiglu8_status = 0;

int swiglu8_read_status(int *out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_swiglu8_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyFromSymbol(swiglu fp8 status)");
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_swiglu8_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyToSymbol(swiglu fp8 status)");
  *out = v;
  return TLLM_OK;
}

namespace swiglu8 {
namespace {

constexpr int BM = 128;
constexpr int BN = 128;   // output columns per tile (each of w1 and w3)
constexpr int BK = 128;   // one 128-byte swizzle row of e4m3
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;          // 16 KB
constexpr int B_BYTES = 2 * BN * BK;      // w1t rows then w3t rows: 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int ACC_COLS = 2 * BN;
constexpr int TMEM_COLS = 512;
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 1024;

enum : int { SITE_EMPTY = 0x41, SITE_FULL = 0x42, SITE_TEMPTY = 0x43, SITE_TFULL = 0x44 };

struct Geom {
  int M, N, K;
  int tiles_m, tiles_n, k_blocks;
  int64_t ldo;
  int vec_store;
  float scale_g, scale_u;  // sx * s1, sx * s3
};

__device__ __forceinline__ void umma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::f8f6f4 instruction descriptor: fp32 accumulator, A and B e4m3 (format 0), both
// K-major; N >> 3 and M >> 4 in their fields (the same bit layout as kind::f16).
constexpr uint32_t idesc_e4m3(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// One row's 32 output columns [nb, nb + 32): silu(scale_g * g) * (scale_u * u) in fp32 from
// the two fp32 accumulators, stored when the row is in range (columns past N are skipped).
template <typename T>
__device__ __forceinline__ void epilogue_chunk(T *orow, int nb, bool row_ok, const Geom &g,
                                               const uint32_t (&gr)[32], const uint32_t (&ur)[32]) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float gv = __uint_as_float(gr[j]) * g.scale_g;
    const float uv = __uint_as_float(ur[j]) * g.scale_u;
    v[j] = (gv / (1.0f + expf(-gv))) * uv;
  }
  if (!row_ok) return;
  if (g.vec_store && nb + 32 <= g.N) {
#pragma unroll
    for (int jj = 0; jj < 32; jj += 8) {
      uint4 raw;
      raw.x = Pack2<T>::pack(v[jj + 0], v[jj + 1]);
      raw.y = Pack2<T>::pack(v[jj + 2], v[jj + 3]);
      raw.z = Pack2<T>::pack(v[jj + 4], v[jj + 5]);
      raw.w = Pack2<T>::pack(v[jj + 6], v[jj + 7]);
      *reinterpret_cast<uint4 *>(orow + nb + jj) = raw;
    }
  } else {
#pragma unroll
    for (int jj = 0; jj < 32; ++jj)
      if (nb + jj < g.N) orow[nb + jj] = from_f32<T>(v[jj]);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    swiglu_fp8_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w1,
                      const __grid_constant__ CUtensorMap tm_w3, T *__restrict__ out, const Geom g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
  uint64_t *full = bars;
  uint64_t *empty = bars + STAGES;
  uint64_t *tfull = bars + 2 * STAGES;
  uint64_t *tempty = bars + 2 * STAGES + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 4);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), kEpiThreads);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(&tm_w1);
    tma_prefetch_desc(&tm_w3);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int num_tiles = g.tiles_m * g.tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile % g.tiles_m) * BM;
        const int n0 = (tile / g.tiles_m) * BN;
        for (int kb = 0; kb < g.k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag, &g_swiglu8_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
          const int k0 = kb * BK;
          tma_load_2d(sa, &tm_x, fb, k0, m0);
          tma_load_2d(sb, &tm_w1, fb, k0, n0);
          tma_load_2d(sb + BN * BK, &tm_w3, fb, k0, n0);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3(BM, 2 * BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, abort_flag, &g_swiglu8_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_TEMPTY)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
        for (int kb = 0; kb < g.k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, &g_swiglu8_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            // Both operands K-major, 128-byte swizzle, 8-row groups 1024 B apart; a k-step
            // of 32 e4m3 elements is 32 bytes along the row.
            const uint64_t adesc = make_sdesc(sa + k * 32, 16, 1024, kSwizzle128B);
            const uint64_t bdesc = make_sdesc(sb + k * 32, 16, 1024, kSwizzle128B);
            umma_f8_ss(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(smem_u32(&empty[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&tfull[acc]));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag, &g_swiglu8_status,
                     TLLM_DEV_WAIT_TIMEOUT + SITE_TFULL))
        break;
      tc_fence_after();
      const int m0 = (tile % g.tiles_m) * BM;
      const int n0 = (tile / g.tiles_m) * BN;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * ACC_COLS;
      const int m = m0 + row;
      T *orow = out + static_cast<int64_t>(m) * g.ldo;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t gr[32], ur[32];
        tmem_ld32(t_row + c, gr);
        tmem_ld32(t_row + BN + c, ur);
        epilogue_chunk<T>(orow, n0 + c, m < g.M, g, gr, ur);
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&tempty[acc]));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// CTA-pair kernel (tcgen05.mma.cta_group::2): a cluster of two CTAs on two SMs computes a
// 256 x 128 output tile. CTA r loads its own 128 rows of x and one weight tile (r = 0: w1t,
// r = 1: w3t), 128 x 128 bytes each, and the pair's leader (r = 0) issues 256 x 256 x 32
// UMMAs whose A rows come from both CTAs' x tiles and whose B rows are the two weight tiles,
// so each CTA's TMEM receives its 128 rows x [x@w1 | x@w3], the layout of the one-CTA
// kernel. A stage is 32 KB per CTA instead of 48 (six stages instead of four), and each SM's
// shared memory feeds 8 KB of operands per 32-deep k-step instead of 12 KB. Each CTA's loads
// complete on the leader's full barrier; the leader's commits arrive on the matching barrier
// in both CTAs; both CTAs' epilogue warps release an accumulator on the leader's tempty
// barrier. Every wait is bounded.
constexpr int PAIR_STAGES = 6;
constexpr int PAIR_STAGE_BYTES = A_BYTES + BN * BK;  // 32 KB: x rows + one weight tile
constexpr int PAIR_SMEM_BYTES = PAIR_STAGES * PAIR_STAGE_BYTES + 1024 + 1024;

__device__ __forceinline__ void umma_f8_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

template <typename T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    swiglu_fp8_pair_kernel(const __grid_constant__ CUtensorMap tm_x,
                           const __grid_constant__ CUtensorMap tm_w1,
                           const __grid_constant__ CUtensorMap tm_w3, T *__restrict__ out,
                           const Geom g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + PAIR_STAGES * PAIR_STAGE_BYTES);
  uint64_t *full = bars;
  uint64_t *empty = bars + PAIR_STAGES;
  uint64_t *tfull = bars + 2 * PAIR_STAGES;
  uint64_t *tempty = bars + 2 * PAIR_STAGES + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * PAIR_STAGES + 4);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int n_pairs = static_cast<int>(gridDim.x >> 1);
  constexpr int kEpiWarps = kEpiThreads / 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PAIR_STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 2 * kEpiWarps);  // both CTAs' epilogue warps
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_x);
    tma_prefetch_desc(rank == 0 ? &tm_w1 : &tm_w3);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_holder), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int num_tiles = g.tiles_m * g.tiles_n;  // tiles_m counts 256-row pair tiles

  if (warp == 0) {
    // ------------------------------ TMA producer (both CTAs) -------------------
    if (lane == 0) {
      const void *tm_w = rank == 0 ? &tm_w1 : &tm_w3;
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += n_pairs) {
        const int m0 = (tile % g.tiles_m) * (2 * BM) + static_cast<int>(rank) * BM;
        const int n0 = (tile / g.tiles_m) * BN;
        for (int kb = 0; kb < g.k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag, &g_swiglu8_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[stage]);
          // The leader's full barrier counts both CTAs' bytes.
          if (rank == 0) mbar_arrive_expect_tx(fb, 2 * PAIR_STAGE_BYTES);
          const uint32_t fb_leader = mapa_shared(fb, 0);
          const uint32_t sa = smem_u32(smem + stage * PAIR_STAGE_BYTES);
          const int k0 = kb * BK;
          tma_load_2d_pair(sa, &tm_x, fb_leader, k0, m0);
          tma_load_2d_pair(sa + A_BYTES, tm_w, fb_leader, k0, n0);
          if (++stage == PAIR_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // The leader's last commits arrive on this CTA's empty barriers: wait for them before
      // the CTA may exit.
      for (int i = 0; ok && i < PAIR_STAGES; ++i) {
        ok = mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag, &g_swiglu8_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_EMPTY);
        if (++stage == PAIR_STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ UMMA issuer (leader) -----------------------
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_e4m3(2 * BM, 2 * BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += n_pairs) {
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, abort_flag, &g_swiglu8_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_TEMPTY)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
        for (int kb = 0; kb < g.k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, &g_swiglu8_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * PAIR_STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 32; ++k) {
            // Both operands K-major, 128-byte swizzle, 8-row groups 1024 B apart, at the same
            // offsets in both CTAs; a k-step of 32 e4m3 elements is 32 bytes along the row.
            const uint64_t adesc = make_sdesc(sa + k * 32, 16, 1024, kSwizzle128B);
            const uint64_t bdesc = make_sdesc(sb + k * 32, 16, 1024, kSwizzle128B);
            umma_f8_ss_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(smem_u32(&empty[stage]));
          if (++stage == PAIR_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(smem_u32(&tfull[acc]));
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------ epilogue (both CTAs) -----------------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t tempty_leader[2] = {mapa_shared(smem_u32(&tempty[0]), 0),
                                       mapa_shared(smem_u32(&tempty[1]), 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < num_tiles; tile += n_pairs) {
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag,
                                             &g_swiglu8_status, TLLM_DEV_WAIT_TIMEOUT + SITE_TFULL)))
        break;
      tc_fence_after();
      const int m0 = (tile % g.tiles_m) * (2 * BM) + static_cast<int>(rank) * BM;
      const int n0 = (tile / g.tiles_m) * BN;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * ACC_COLS;
      const int m = m0 + row;
      T *orow = out + static_cast<int64_t>(m) * g.ldo;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t gr[32], ur[32];
        tmem_ld32(t_row + c, gr);
        tmem_ld32(t_row + BN + c, ur);
        epilogue_chunk<T>(orow, n0 + c, m < g.M, g, gr, ur);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no UMMA, commit or remote arrive of either CTA is still pending
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Kernel choice (tllm_swiglu_fp8_variant): the CTA-pair kernel from two 128-row blocks up,
// or forced.
constexpr int kVariantAuto = 0;
constexpr int kVariantSingleCta = 1;
constexpr int kVariantCtaPair = 2;

template <typename T>
int launch(const void *x, const void *w1t, const void *w3t, void *out, int64_t M, int64_t N,
           int64_t K, int64_t lda, int64_t ldb1, int64_t ldb3, int64_t ldo, float scale_g,
           float scale_u, int variant, cudaStream_t st) {
  CUtensorMap mx, m1, m3;
  const uint32_t box[2] = {BK, 128};
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t str[1] = {static_cast<uint64_t>(lda)};
    int rc = encode_tiled(&mx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(x), dims, str,
                          box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t s1[1] = {static_cast<uint64_t>(ldb1)};
    int rc = encode_tiled(&m1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(w1t), dims, s1,
                          box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const uint64_t s3[1] = {static_cast<uint64_t>(ldb3)};
    rc = encode_tiled(&m3, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(w3t), dims, s3, box,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  Geom g;
  g.M = static_cast<int>(M);
  g.N = static_cast<int>(N);
  g.K = static_cast<int>(K);
  g.tiles_m = static_cast<int>((M + BM - 1) / BM);
  g.tiles_n = static_cast<int>((N + BN - 1) / BN);
  g.k_blocks = static_cast<int>((K + BK - 1) / BK);
  g.ldo = ldo;
  g.vec_store = (ldo % 8 == 0 && aligned16(out)) ? 1 : 0;
  g.scale_g = scale_g;
  g.scale_u = scale_u;
  const int sms = sm_count();
  if (sms >= 2 && variant != kVariantSingleCta && (variant == kVariantCtaPair || M >= 2 * BM)) {
    Geom gp = g;
    gp.tiles_m = static_cast<int>((M + 2 * BM - 1) / (2 * BM));
    const int pair_tiles = gp.tiles_m * gp.tiles_n;
    auto kern = swiglu_fp8_pair_kernel<T>;
    // Persistent grid: as many pairs as can be resident at once.
    KernelLaunchInfo info;
    const int rc = prepare_kernel(reinterpret_cast<const void *>(kern), PAIR_SMEM_BYTES, kThreads, 2, &info);
    if (rc) return rc;
    const int max_clusters = info.resident;
    if (max_clusters < 1) return fail(TLLM_ERR_CUDA, "swiglu_fp8: the CTA-pair kernel cannot be resident");
    const int max_pairs = max_clusters < sms / 2 ? max_clusters : sms / 2;
    const int pairs = pair_tiles < max_pairs ? pair_tiles : max_pairs;
    kern<<<2 * pairs, kThreads, PAIR_SMEM_BYTES, st>>>(mx, m1, m3, static_cast<T *>(out), gp);
    return cuda_status(cudaGetLastError(), "swiglu fp8 pair launch");
  }
  const int num_tiles = g.tiles_m * g.tiles_n;
  const int grid = num_tiles < sms ? num_tiles : sms;
  auto kern = swiglu_fp8_kernel<T>;
  KernelLaunchInfo info;
  const int rc = prepare_kernel(reinterpret_cast<const void *>(kern), SMEM_BYTES, kThreads, 1, &info);
  if (rc) return rc;
  kern<<<grid, kThreads, SMEM_BYTES, st>>>(mx, m1, m3, static_cast<T *>(out), g);
  return cuda_status(cudaGetLastError(), "swiglu fp8 launch");
}

}  // namespace
}  // namespace swiglu8
}  // namespace tllm

extern "C" int tllm_swiglu_fp8_variant(const void *x, const void *w1t, const void *w3t,
                                       void *out, int64_t M, int64_t N, int64_t K, int64_t lda,
                                       int64_t ldb1, int64_t ldb3, int64_t ldo, float scale_x,
                                       float scale_w1, float scale_w3, int out_dtype, int variant,
                                       void *stream) {
  using namespace tllm;
  clear_error();
  TLLM_CHECK_ARG(variant >= swiglu8::kVariantAuto && variant <= swiglu8::kVariantCtaPair,
                 "swiglu_fp8: unknown kernel variant %d", variant);
  TLLM_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "swiglu_fp8: negative dimension");
  TLLM_CHECK_ARG(out_dtype == TLLM_DTYPE_F16 || out_dtype == TLLM_DTYPE_BF16,
                 "swiglu_fp8: unsupported output dtype %d", out_dtype);
  TLLM_CHECK_ARG(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31), "swiglu_fp8: dimension too large");
  if (M == 0 || N == 0) return TLLM_OK;
  TLLM_CHECK_ARG(out && K > 0 && x && w1t && w3t, "swiglu_fp8: null pointer or K == 0");
  TLLM_CHECK_ARG(lda >= K && ldb1 >= K && ldb3 >= K && ldo >= N, "swiglu_fp8: leading dimension too small");
  TLLM_CHECK_ARG(K % 16 == 0 && lda % 16 == 0 && ldb1 % 16 == 0 && ldb3 % 16 == 0,
                 "swiglu_fp8: K and the input leading dimensions must be multiples of 16 bytes");
  TLLM_CHECK_ARG(swiglu8::aligned16(x) && swiglu8::aligned16(w1t) && swiglu8::aligned16(w3t),
                 "swiglu_fp8: inputs must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float sg = scale_x * scale_w1, su = scale_x * scale_w3;
  if (out_dtype == TLLM_DTYPE_F16)
    return swiglu8::launch<__half>(x, w1t, w3t, out, M, N, K, lda, ldb1, ldb3, ldo, sg, su,
                                   variant, st);
  return swiglu8::launch<__nv_bfloat16>(x, w1t, w3t, out, M, N, K, lda, ldb1, ldb3, ldo, sg, su,
                                        variant, st);
}

extern "C" int tllm_swiglu_fp8(const void *x, const void *w1t, const void *w3t, void *out,
                               int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb1,
                               int64_t ldb3, int64_t ldo, float scale_x, float scale_w1,
                               float scale_w3, int out_dtype, void *stream) {
  return tllm_swiglu_fp8_variant(x, w1t, w3t, out, M, N, K, lda, ldb1, ldb3, ldo, scale_x,
                                 scale_w1, scale_w3, out_dtype, 0, stream);
}
