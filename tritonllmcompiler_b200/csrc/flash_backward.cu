// FlashAttention backward for sm_100a (tcgen05 + TMEM + TMA).
//
// The reference has the forward only (python/triton_llm/ops/flash_attention.py:1-7); its
// oracle defines the function being differentiated (python/triton_llm/reference/
// flash_attention.py:12-29: S = q k^T * scale, top-left causal mask, P = softmax(S), O = P v).
// Gradients: dV = P^T dO, dP = dO V^T, dS = P * (dP - rowsum(dO * O)), dQ = scale * dS K,
// dK = scale * dS^T Q. P is recomputed from the forward's per-row log-normaliser
// (tllm_flash_attn_fwd_lse), never stored.
//
// B200 design: one CTA per (b, h, 128-key tile j); it walks the query tiles i that can see
// key tile j (i >= j when causal) and keeps dK_j and dV_j in TMEM for the whole walk.
//   warp 0      TMA: K_j and V_j once; Q_i and dO_i per step (single buffers)
//   warp 1      TMEM (512 columns) and the UMMA-issuing lane, five 128-row GEMMs per step:
//                 S  = Q_i K_j^T      -> TMEM [0,128)    (then reused for dQ_i)
//                 dP = dO_i V_j^T     -> TMEM [128,256)
//                 dV += P^T dO_i      -> TMEM [256,256+D)  (A = P from shared memory, MN-major)
//                 dK += dS^T Q_i      -> TMEM [384,384+D)  (A = dS, MN-major)
//                 dQ = dS K_j         -> TMEM [0,D)        (A = dS, K-major)
//   warps 2-5   one query row per thread: P = 2^(s*scale*log2e - lse) (masked to 0), written
//               to shared memory (fp16/bf16, 128-byte swizzle); dS = P (dP - delta) written
//               likewise; dQ_i staged in shared memory (fp32, in the then free P and dS
//               buffers) and added into an fp32 accumulator by the TMA engine (bulk tensor
//               reduce-add). At the end the same threads hold one key row each and write dK_j
//               and dV_j.
// Every wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "common.h"
#include "ptx.cuh"

namespace tllm {

__device__ int g_fbwd_status = 0;

int fbwd_read_status(int *out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_fbwd_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyFromSymbol(flash bwd status)");
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_fbwd_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyToSymbol(flash bwd status)");
  *out = v;
  return TLLM_OK;
}

namespace fbwd {
namespace {

constexpr int BM = 128;  // query rows per tile
constexpr int BN = 128;  // key rows per tile
constexpr int kThreads = 192;
constexpr int TMEM_COLS = 512;
constexpr int S_COL = 0;    // S_i, then dQ_i
constexpr int DP_COL = 128;
constexpr int DV_COL = 256;
constexpr int DK_COL = 384;
constexpr float kLog2e = 1.4426950408889634f;

enum : int {
  SITE_KV = 0x31,
  SITE_Q = 0x32,
  SITE_QEMPTY = 0x33,
  SITE_DO = 0x34,
  SITE_DOEMPTY = 0x35,
  SITE_S = 0x36,
  SITE_DP = 0x37,
  SITE_P = 0x38,
  SITE_PFREE = 0x39,
  SITE_DS = 0x3a,
  SITE_DQ = 0x3b,
  SITE_DQFREE = 0x3c,
  SITE_ACC = 0x3d,
  SITE_STAGE = 0x3e,
};

// Shared-memory tiles are 128 rows in 128-byte swizzle spans ("chunks" of 64 elements, each
// chunk a contiguous 128 x 128 B block): K, V, Q, dO (D columns) and P, dS (128 columns).
template <int D>
struct Geo {
  static_assert(D == 64 || D == 128, "backward supports head dims 64 and 128");
  static constexpr int CHUNK_BYTES = 128 * 128;
  static constexpr int TILE_D = 128 * D * 2;
  static constexpr int TILE_P = 128 * 128 * 2;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = K_OFF + TILE_D;
  static constexpr int Q_OFF = V_OFF + TILE_D;
  static constexpr int DO_OFF = Q_OFF + TILE_D;
  static constexpr int P_OFF = DO_OFF + TILE_D;
  static constexpr int DS_OFF = P_OFF + TILE_P;
  static constexpr int BAR_OFF = DS_OFF + TILE_P;
  static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory plan");
  static_assert(DS_OFF == P_OFF + TILE_P && 128 * D * 4 <= 2 * TILE_P, "dQ staging spans P and dS");
};

struct Args {
  const float *lse;    // [B, H, Sq]
  const float *delta;  // [B, H, Sq]
  float *dq_acc;       // [B, H, Sq, D], zeroed before the launch
  void *dk, *dv;
  int64_t sdk0, sdk1, sdk2, sdk3;
  int64_t sdv0, sdv1, sdv2, sdv3;
  int H, Sq, Sk;
  int n_qtiles, n_ktiles;
  float scale_log2, scale;
  int causal;
};

// K-major operand (rows = M or N, the reduction dim contiguous): k16 step k.
__device__ __forceinline__ uint64_t kdesc(uint32_t base, int k) {
  const int byte = k * 32;
  return make_sdesc(base + (byte / 128) * (128 * 128) + (byte % 128), 16, 1024, 2u);
}
// MN-major operand (rows = the reduction dim, M or N contiguous in 64-element chunks): k16 step k.
__device__ __forceinline__ uint64_t mndesc(uint32_t base, int k) {
  return make_sdesc(base + k * 16 * 128, 128 * 128, 1024, 2u);
}

// dQ partial tile -> fp32 accumulator in global memory: the TMA engine adds a 128-row x 32-column
// box from shared memory (128-byte swizzle) into the tensor.
__device__ __forceinline__ void tma_reduce_add_2d(const void *map, uint32_t src, int c0, int c1) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until the committed bulk operations have finished reading their shared memory.
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Writes 128 values as one swizzled row of a 128-column tile (thread `row` owns row `row`).
// (`v` holds fp32 bit patterns.)
template <typename T>
__device__ __forceinline__ void store_row128(uint8_t *tile, int row, const uint32_t (&v)[128]) {
#define TLLM_F(i) __uint_as_float(v[i])
#pragma unroll
  for (int u = 0; u < 16; ++u) {
    uint4 pk;
    pk.x = Pack2<T>::pack(TLLM_F(8 * u + 0), TLLM_F(8 * u + 1));
    pk.y = Pack2<T>::pack(TLLM_F(8 * u + 2), TLLM_F(8 * u + 3));
    pk.z = Pack2<T>::pack(TLLM_F(8 * u + 4), TLLM_F(8 * u + 5));
    pk.w = Pack2<T>::pack(TLLM_F(8 * u + 6), TLLM_F(8 * u + 7));
    const int chunk = u >> 3, j = u & 7;
    *reinterpret_cast<uint4 *>(tile + chunk * (128 * 128) + row * 128 + ((j ^ (row & 7)) << 4)) = pk;
  }
#undef TLLM_F
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_dq, const Args a) {
  using G = Geo<D>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int CH = D / 64;  // 128-byte chunks per row of a D-column tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + G::BAR_OFF);
  uint64_t *kv_full = bars + 0;
  uint64_t *q_full = bars + 1;
  uint64_t *q_empty = bars + 2;
  uint64_t *do_full = bars + 3;
  uint64_t *do_empty = bars + 4;
  uint64_t *s_full = bars + 5;
  uint64_t *dp_full = bars + 6;
  uint64_t *p_full = bars + 7;
  uint64_t *p_free = bars + 8;
  uint64_t *ds_full = bars + 9;
  uint64_t *dq_full = bars + 10;
  uint64_t *dq_free = bars + 11;
  uint64_t *acc_done = bars + 12;
  uint64_t *stage_full = bars + 13;  // 128 row threads have staged dQ_i
  uint64_t *stage_free = bars + 14;  // the TMA engine has read the staged dQ tile
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 15);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // (b, h) major; within a head the key tiles with the most query tiles (j = 0 when causal)
  // first.
  const int bh = static_cast<int>(blockIdx.x) / a.n_ktiles;
  const int j = static_cast<int>(blockIdx.x) % a.n_ktiles;
  const int b = bh / a.H;
  const int h = bh % a.H;
  const int i0 = a.causal ? j : 0;
  const int n_it = max(0, a.n_qtiles - i0);

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(kv_full), 1);
    mbar_init(smem_u32(q_full), 1);
    mbar_init(smem_u32(q_empty), 1);
    mbar_init(smem_u32(do_full), 1);
    mbar_init(smem_u32(do_empty), 1);
    mbar_init(smem_u32(s_full), 1);
    mbar_init(smem_u32(dp_full), 1);
    mbar_init(smem_u32(p_full), 128);
    mbar_init(smem_u32(p_free), 1);
    mbar_init(smem_u32(ds_full), 128);
    mbar_init(smem_u32(dq_full), 1);
    mbar_init(smem_u32(dq_free), 128);
    mbar_init(smem_u32(acc_done), 1);
    mbar_init(smem_u32(stage_full), 128);
    mbar_init(smem_u32(stage_free), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint32_t sK = smem_u32(smem + G::K_OFF);
  const uint32_t sV = smem_u32(smem + G::V_OFF);
  const uint32_t sQ = smem_u32(smem + G::Q_OFF);
  const uint32_t sDO = smem_u32(smem + G::DO_OFF);
  const uint32_t sP = smem_u32(smem + G::P_OFF);
  const uint32_t sDS = smem_u32(smem + G::DS_OFF);

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0 && n_it > 0) {
      const uint32_t kvb = smem_u32(kv_full);
      mbar_arrive_expect_tx(kvb, 2 * G::TILE_D);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        tma_load_4d(sK + c * G::CHUNK_BYTES, &tm_k, kvb, c * 64, j * BN, h, b);
        tma_load_4d(sV + c * G::CHUNK_BYTES, &tm_v, kvb, c * 64, j * BN, h, b);
      }
      for (int it = 0; it < n_it; ++it) {
        const int i = i0 + it;
        const uint32_t par = (it & 1) ^ 1;
        if (!mbar_wait(smem_u32(q_empty), par, abort_flag, &g_fbwd_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_QEMPTY))
          break;
        mbar_arrive_expect_tx(smem_u32(q_full), G::TILE_D);
#pragma unroll
        for (int c = 0; c < CH; ++c)
          tma_load_4d(sQ + c * G::CHUNK_BYTES, &tm_q, smem_u32(q_full), c * 64, i * BM, h, b);
        if (!mbar_wait(smem_u32(do_empty), par, abort_flag, &g_fbwd_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_DOEMPTY))
          break;
        mbar_arrive_expect_tx(smem_u32(do_full), G::TILE_D);
#pragma unroll
        for (int c = 0; c < CH; ++c)
          tma_load_4d(sDO + c * G::CHUNK_BYTES, &tm_do, smem_u32(do_full), c * 64, i * BM, h, b);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ UMMA issuer -------------------------------
    if (lane == 0) {
      const uint32_t id_sq = make_idesc_f16(BM, BN, kBF16, false, false);  // S, dP
      const uint32_t id_acc = make_idesc_f16(BN, D, kBF16, true, true);   // dV, dK
      const uint32_t id_dq = make_idesc_f16(BM, D, kBF16, false, true);   // dQ
      bool ok = n_it == 0 || mbar_wait(smem_u32(kv_full), 0, abort_flag, &g_fbwd_status,
                                       TLLM_DEV_WAIT_TIMEOUT + SITE_KV);
      for (int it = 0; it < n_it && ok; ++it) {
        const uint32_t par = it & 1;
        // S = Q K^T into columns the softmax has finished reading dQ_{i-1} from.
        ok = mbar_wait(smem_u32(q_full), par, abort_flag, &g_fbwd_status, TLLM_DEV_WAIT_TIMEOUT + SITE_Q) &&
             (it == 0 || mbar_wait(smem_u32(dq_free), par ^ 1, abort_flag, &g_fbwd_status,
                                   TLLM_DEV_WAIT_TIMEOUT + SITE_DQFREE));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          umma_f16_ss(tmem_base + S_COL, kdesc(sQ, k), kdesc(sK, k), id_sq, k != 0 ? 1u : 0u);
        umma_commit(smem_u32(s_full));
        // dP = dO V^T (its columns were read before the previous step's dS was published).
        if (!mbar_wait(smem_u32(do_full), par, abort_flag, &g_fbwd_status, TLLM_DEV_WAIT_TIMEOUT + SITE_DO)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          umma_f16_ss(tmem_base + DP_COL, kdesc(sDO, k), kdesc(sV, k), id_sq, k != 0 ? 1u : 0u);
        umma_commit(smem_u32(dp_full));
        // dV += P^T dO.
        if (!mbar_wait(smem_u32(p_full), par, abort_flag, &g_fbwd_status, TLLM_DEV_WAIT_TIMEOUT + SITE_P)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < BM / 16; ++k)
          umma_f16_ss(tmem_base + DV_COL, mndesc(sP, k), mndesc(sDO, k), id_acc, (it | k) != 0 ? 1u : 0u);
        umma_commit(smem_u32(p_free));
        umma_commit(smem_u32(do_empty));
        // dK += dS^T Q, then dQ = dS K into S's columns (S was read before P was published).
        if (!mbar_wait(smem_u32(ds_full), par, abort_flag, &g_fbwd_status, TLLM_DEV_WAIT_TIMEOUT + SITE_DS)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < BM / 16; ++k)
          umma_f16_ss(tmem_base + DK_COL, mndesc(sDS, k), mndesc(sQ, k), id_acc, (it | k) != 0 ? 1u : 0u);
#pragma unroll
        for (int k = 0; k < BN / 16; ++k)
          umma_f16_ss(tmem_base + S_COL, kdesc(sDS, k), mndesc(sK, k), id_dq, k != 0 ? 1u : 0u);
        umma_commit(smem_u32(dq_full));
        umma_commit(smem_u32(q_empty));
      }
      umma_commit(smem_u32(acc_done));
    }
  } else {
    // ------------------------- softmax rows / dQ / dK dV ---------------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int64_t rowbase = static_cast<int64_t>(bh) * a.Sq;
    bool ok = true;
    for (int it = 0; it < n_it && ok; ++it) {
      const uint32_t par = it & 1;
      const int i = i0 + it;
      const int qg = i * BM + row;
      const bool rv = qg < a.Sq;
      const float lse = rv ? __ldg(a.lse + rowbase + qg) : 0.f;
      const float dlt = rv ? __ldg(a.delta + rowbase + qg) : 0.f;
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(s_full), par, abort_flag, &g_fbwd_status,
                                             TLLM_DEV_WAIT_TIMEOUT + SITE_S))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // p holds S, then P, then dS (fp32 bits), one row per thread.
      uint32_t p[128];
      tmem_ld4x32(tmem_base + lane_off + S_COL, p);
      const uint64_t scale2 = f2_pack(a.scale_log2, a.scale_log2);
      const uint64_t nlse2 = f2_pack(-lse, -lse);
#pragma unroll
      for (int t = 0; t < 128; t += 2) {
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(__uint_as_float(p[t]), __uint_as_float(p[t + 1])), scale2, nlse2), x0, x1);
        p[t] = __float_as_uint(ex2_approx(x0));
        p[t + 1] = __float_as_uint(ex2_approx(x1));
      }
      // Only tiles on the causal diagonal or at a ragged edge need the mask.
      const bool full = (!a.causal || j * BN + BN - 1 <= i * BM) && (j + 1) * BN <= a.Sk &&
                        (i + 1) * BM <= a.Sq;
      if (!full) {
#pragma unroll
        for (int t = 0; t < 128; ++t) {
          const int kg = j * BN + t;
          if (!(rv && kg < a.Sk && !(a.causal && kg > qg))) p[t] = 0u;
        }
      }
      // P's buffer is free once the previous step's dV GEMM has read it and the TMA engine
      // has read the previous dQ tile staged there.
      if (it > 0 && !__all_sync(0xffffffffu, mbar_wait(smem_u32(p_free), par ^ 1, abort_flag, &g_fbwd_status,
                                                        TLLM_DEV_WAIT_TIMEOUT + SITE_PFREE))) {
        ok = false;
        break;
      }
      if (it > 0) {
        if (threadIdx.x == 64) {
          bulk_wait_read0();
          mbar_arrive(smem_u32(stage_free));
        }
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(stage_free), par ^ 1, abort_flag, &g_fbwd_status,
                                               TLLM_DEV_WAIT_TIMEOUT + SITE_STAGE))) {
          ok = false;
          break;
        }
      }
      store_row128<T>(smem + G::P_OFF, row, p);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(smem_u32(p_full));
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(dp_full), par, abort_flag, &g_fbwd_status,
                                             TLLM_DEV_WAIT_TIMEOUT + SITE_DP))) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 128; c += 32) {
        uint32_t dpr[32];
        tmem_ld32(tmem_base + lane_off + DP_COL + c, dpr);
#pragma unroll
        for (int t = 0; t < 32; ++t)
          p[c + t] = __float_as_uint(__uint_as_float(p[c + t]) * (__uint_as_float(dpr[t]) - dlt));
      }
      // dS's buffer was last read by the previous step's dK and dQ GEMMs, which completed
      // before that step's dQ was published (waited below).
      store_row128<T>(smem + G::DS_OFF, row, p);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(smem_u32(ds_full));
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(dq_full), par, abort_flag, &g_fbwd_status,
                                             TLLM_DEV_WAIT_TIMEOUT + SITE_DQ))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // Stage scale * dQ_i (fp32, zero for rows past Sq) in the P and dS buffers, both free
      // once dQ_i is complete, as D/32 boxes of 128 rows x 32 columns (128-byte swizzle); one
      // thread then has the TMA engine add them into the accumulator.
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_base + lane_off + S_COL + c, r);
        uint8_t *box = smem + G::P_OFF + (c / 32) * (128 * 128) + row * 128;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float4 f;
          f.x = rv ? __uint_as_float(r[4 * u + 0]) * a.scale : 0.f;
          f.y = rv ? __uint_as_float(r[4 * u + 1]) * a.scale : 0.f;
          f.z = rv ? __uint_as_float(r[4 * u + 2]) * a.scale : 0.f;
          f.w = rv ? __uint_as_float(r[4 * u + 3]) * a.scale : 0.f;
          *reinterpret_cast<float4 *>(box + ((u ^ (row & 7)) << 4)) = f;
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(dq_free));
      fence_proxy_async_smem();
      mbar_arrive(smem_u32(stage_full));
      if (threadIdx.x == 64) {
        if (!mbar_wait(smem_u32(stage_full), par, abort_flag, &g_fbwd_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_STAGE)) {
          ok = false;
        } else {
#pragma unroll
          for (int c = 0; c < D / 32; ++c)
            tma_reduce_add_2d(&tm_dq, sP + c * (128 * 128), c * 32, static_cast<int>(rowbase) + i * BM);
          bulk_commit();
        }
      }
      ok = __all_sync(0xffffffffu, ok);
    }
    if (threadIdx.x == 64) bulk_wait_all();
    // ---- dK_j, dV_j: thread `row` holds key row j * BN + row ----
    const int kg = j * BN + row;
    const bool have = ok && n_it > 0 &&
                      __all_sync(0xffffffffu, mbar_wait(smem_u32(acc_done), 0, abort_flag, &g_fbwd_status,
                                                        TLLM_DEV_WAIT_TIMEOUT + SITE_ACC));
    if (have) tc_fence_after();
    if ((have || n_it == 0) && ok) {
      T *dvrow = static_cast<T *>(a.dv) + b * a.sdv0 + h * a.sdv1 + static_cast<int64_t>(kg) * a.sdv2;
      T *dkrow = static_cast<T *>(a.dk) + b * a.sdk0 + h * a.sdk1 + static_cast<int64_t>(kg) * a.sdk2;
#pragma unroll 1
      for (int c = 0; c < D; c += 32) {
        uint32_t rv_[32], rk_[32];
        if (have) {
          tmem_ld32(tmem_base + lane_off + DV_COL + c, rv_);
          tmem_ld32(tmem_base + lane_off + DK_COL + c, rk_);
        } else {
#pragma unroll
          for (int t = 0; t < 32; ++t) rv_[t] = rk_[t] = 0u;
        }
        if (kg < a.Sk) {
#pragma unroll
          for (int t = 0; t < 32; ++t) {
            dvrow[(c + t) * a.sdv3] = from_f32<T>(__uint_as_float(rv_[t]));
            dkrow[(c + t) * a.sdk3] = from_f32<T>(__uint_as_float(rk_[t]) * a.scale);
          }
        }
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

// delta[r] = sum_d dO[r, d] * O[r, d] in fp32, one thread per (b, h, q) row.
template <typename T, int D>
__global__ void __launch_bounds__(256) flash_bwd_delta_kernel(const T *__restrict__ o, const T *__restrict__ dout,
                                                              float *__restrict__ delta, int H, int Sq,
                                                              int64_t so0, int64_t so1, int64_t so2,
                                                              int64_t sd0, int64_t sd1, int64_t sd2,
                                                              int64_t rows) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int64_t q = r % Sq;
  const int64_t bh = r / Sq;
  const int64_t bb = bh / H, hh = bh % H;
  const T *op = o + bb * so0 + hh * so1 + q * so2;
  const T *dp = dout + bb * sd0 + hh * sd1 + q * sd2;
  float acc = 0.f;
#pragma unroll
  for (int d = 0; d < D; d += 8) {
    const uint4 x = __ldg(reinterpret_cast<const uint4 *>(op + d));
    const uint4 y = __ldg(reinterpret_cast<const uint4 *>(dp + d));
    const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 a2 = Pack2<T>::unpack(xs[u]);
      const float2 b2 = Pack2<T>::unpack(ys[u]);
      acc = fmaf(a2.x, b2.x, fmaf(a2.y, b2.y, acc));
    }
  }
  delta[r] = acc;
}

// dq = dq_acc in the I/O dtype.
template <typename T, int D>
__global__ void __launch_bounds__(256) flash_bwd_dq_kernel(const float *__restrict__ acc, T *__restrict__ dq,
                                                           int H, int Sq, int64_t s0, int64_t s1,
                                                           int64_t s2, int64_t s3, int64_t n) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= n) return;
  const int64_t d = e % D;
  const int64_t r = e / D;
  const int64_t q = r % Sq;
  const int64_t bh = r / Sq;
  dq[(bh / H) * s0 + (bh % H) * s1 + q * s2 + d * s3] = from_f32<T>(acc[e]);
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T, int D>
int launch(const void *q, const void *k, const void *v, const void *o, const void *dout,
           const float *lse, void *dq, void *dk, void *dv, float *ws, int64_t B, int64_t H,
           int64_t Sq, int64_t Sk, const int64_t *sq, const int64_t *sk, const int64_t *sv,
           const int64_t *so, const int64_t *sdo, const int64_t *sdq, const int64_t *sdk,
           const int64_t *sdv, float sm_scale, int causal, cudaStream_t st) {
  using Gm = Geo<D>;
  const CUtensorMapDataType dt = std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint32_t box[4] = {64, 128, 1, 1};
  CUtensorMap mq, mk, mv, mdo;
  auto enc = [&](CUtensorMap *m, const void *p, int64_t S, const int64_t *s) {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)(S > 0 ? S : 1), (uint64_t)H, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)s[2] * 2, (uint64_t)s[1] * 2, (uint64_t)s[0] * 2};
    return encode_tiled(m, dt, 4, const_cast<void *>(p), dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
  };
  CUtensorMap mdq;
  {
    // fp32 accumulator [B*H*Sq, D], boxes of 128 rows x 32 columns
    const uint64_t dims[2] = {(uint64_t)D, (uint64_t)(B * H * (Sq > 0 ? Sq : 1))};
    const uint64_t str[1] = {(uint64_t)D * 4};
    const uint32_t box2[2] = {32, 128};
    int rc0 = encode_tiled(&mdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ws, dims, str, box2,
                           CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc0) return rc0;
  }
  int rc = enc(&mq, q, Sq, sq);
  if (!rc) rc = enc(&mk, k, Sk, sk);
  if (!rc) rc = enc(&mv, v, Sk, sv);
  if (!rc) rc = enc(&mdo, dout, Sq, sdo);
  if (rc) return rc;
  const int64_t rows = B * H * Sq;
  float *dq_acc = ws;
  float *delta = rows > 0 ? ws + rows * D : nullptr;
  if (rows > 0) {
    TLLM_CUDA_TRY(cudaMemsetAsync(dq_acc, 0, static_cast<size_t>(rows) * D * sizeof(float), st));
    flash_bwd_delta_kernel<T, D><<<static_cast<unsigned>((rows + 255) / 256), 256, 0, st>>>(
        static_cast<const T *>(o), static_cast<const T *>(dout), delta, static_cast<int>(H),
        static_cast<int>(Sq), so[0], so[1], so[2], sdo[0], sdo[1], sdo[2], rows);
    TLLM_CUDA_TRY(cudaGetLastError());
  }
  Args a{};
  a.lse = lse;
  a.delta = delta;
  a.dq_acc = dq_acc;
  a.dk = dk;
  a.dv = dv;
  a.sdk0 = sdk[0]; a.sdk1 = sdk[1]; a.sdk2 = sdk[2]; a.sdk3 = sdk[3];
  a.sdv0 = sdv[0]; a.sdv1 = sdv[1]; a.sdv2 = sdv[2]; a.sdv3 = sdv[3];
  a.H = static_cast<int>(H);
  a.Sq = static_cast<int>(Sq);
  a.Sk = static_cast<int>(Sk);
  a.n_qtiles = static_cast<int>((Sq + BM - 1) / BM);
  a.n_ktiles = static_cast<int>((Sk + BN - 1) / BN);
  a.scale_log2 = sm_scale * kLog2e;
  a.scale = sm_scale;
  a.causal = causal ? 1 : 0;
  if (a.n_ktiles > 0) {
    auto kern = flash_bwd_kernel<T, D>;
    KernelLaunchInfo info;
    const int rc = prepare_kernel(reinterpret_cast<const void *>(kern), Gm::SMEM_BYTES, kThreads, 1, &info);
    if (rc) return rc;
    const unsigned grid = static_cast<unsigned>(B * H * a.n_ktiles);
    kern<<<grid, kThreads, Gm::SMEM_BYTES, st>>>(mq, mk, mv, mdo, mdq, a);
    TLLM_CUDA_TRY(cudaGetLastError());
  }
  const int64_t n = rows * D;
  if (n > 0)
    flash_bwd_dq_kernel<T, D><<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(
        dq_acc, static_cast<T *>(dq), static_cast<int>(H), static_cast<int>(Sq), sdq[0], sdq[1],
        sdq[2], sdq[3], n);
  return cuda_status(cudaGetLastError(), "flash bwd launch");
}

}  // namespace
}  // namespace fbwd
}  // namespace tllm

extern "C" size_t tllm_flash_attn_bwd_workspace_size(int64_t B, int64_t H, int64_t Sq, int64_t D) {
  if (B <= 0 || H <= 0 || Sq <= 0 || D <= 0) return 0;
  return static_cast<size_t>(B * H * Sq) * static_cast<size_t>(D + 1) * sizeof(float);
}

extern "C" int tllm_flash_attn_bwd(const void *q, const void *k, const void *v, const void *o,
                                   const void *dout, const float *lse, void *dq, void *dk,
                                   void *dv, void *workspace, size_t workspace_bytes, int64_t B,
                                   int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                   const int64_t *sq, const int64_t *sk, const int64_t *sv,
                                   const int64_t *so, const int64_t *sdo, const int64_t *sdq,
                                   const int64_t *sdk, const int64_t *sdv, float sm_scale,
                                   int causal, int dtype, void *stream) {
  using namespace tllm;
  using namespace tllm::fbwd;
  clear_error();
  TLLM_CHECK_ARG(B >= 0 && H >= 0 && Sq >= 0 && Sk >= 0, "flash_attention_backward: negative dimension");
  TLLM_CHECK_ARG(D == 64 || D == 128, "flash_attention_backward: head dim %lld not in {64,128}", (long long)D);
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16,
                 "flash_attention_backward: unsupported dtype %d", dtype);
  TLLM_CHECK_ARG(sq && sk && sv && so && sdo && sdq && sdk && sdv,
                 "flash_attention_backward: null stride array");
  if (B == 0 || H == 0 || (Sq == 0 && Sk == 0)) return TLLM_OK;
  TLLM_CHECK_ARG(q && k && v && o && dout && lse && dq && dk && dv,
                 "flash_attention_backward: null tensor pointer");
  TLLM_CHECK_ARG(Sq < (1LL << 31) && Sk < (1LL << 31) && B * H * ((Sk + 127) / 128) < (1LL << 31) &&
                     B * H * Sq < (1LL << 31),
                 "flash_attention_backward: problem too large");
  const size_t need = tllm_flash_attn_bwd_workspace_size(B, H, Sq, D);
  TLLM_CHECK_ARG(Sq == 0 || (workspace && workspace_bytes >= need),
                 "flash_attention_backward: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  TLLM_CHECK_ARG(Sq == 0 || (reinterpret_cast<uintptr_t>(workspace) & 15u) == 0,
                 "flash_attention_backward: workspace must be 16-byte aligned");
  TLLM_CHECK_ARG(sq[3] == 1 && sk[3] == 1 && sv[3] == 1 && so[3] == 1 && sdo[3] == 1,
                 "flash_attention_backward: q/k/v/o/dout need a unit innermost stride");
  for (int i = 0; i < 3; ++i)
    TLLM_CHECK_ARG(sq[i] % 8 == 0 && sk[i] % 8 == 0 && sv[i] % 8 == 0 && so[i] % 8 == 0 && sdo[i] % 8 == 0,
                   "flash_attention_backward: input strides must be multiples of 8 elements");
  TLLM_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o) && aligned16(dout),
                 "flash_attention_backward: inputs must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // With no queries the kernel writes zero dK and dV (no query tile reaches a key tile).
  float *ws = static_cast<float *>(workspace);
#define TLLM_FBWD(TT, DD)                                                                        \
  return launch<TT, DD>(q, k, v, o, dout, lse, dq, dk, dv, ws, B, H, Sq, Sk, sq, sk, sv, so, sdo, \
                        sdq, sdk, sdv, sm_scale, causal, st)
  if (dtype == TLLM_DTYPE_F16) {
    if (D == 64) TLLM_FBWD(__half, 64);
    TLLM_FBWD(__half, 128);
  }
  if (D == 64) TLLM_FBWD(__nv_bfloat16, 64);
  TLLM_FBWD(__nv_bfloat16, 128);
#undef TLLM_FBWD
}
