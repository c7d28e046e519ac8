// Multi-token, grouped-query attention over the paged KV cache (tcgen05 + TMEM + TMA).
//
// The reference decodes one query token per sequence with as many KV heads as query heads
// (python/triton_llm/ops/paged_attention.py:92-128, asserting Sq == 1 at :105). This operator
// covers the rows either side of it: Sq >= 1 new query tokens per sequence (speculative or
// chunked-prefill decode, prefill) and Hq = G * Hkv query heads sharing each KV head. Query
// token s of sequence b sits at position context_len - Sq + s and, with causal, sees the
// keys at positions <= its own; the cache layout and the attention arithmetic are those of
// python/triton_llm/reference/paged_attention.py:14-40 and flash_attention.py:12-29.
//
// B200 design. A work item is (sequence b, KV head, tile of up to 128 query rows, key split).
// The query rows of a tile are G' heads x S' tokens of one KV head, so every K/V tile loaded
// serves all of them (G * Sq rows per byte of K/V instead of one). K and V blocks are fetched
// by TMA straight from the paged pool (one 4-D box of block_size tokens of one head per cache
// block, coordinates from the block table staged in shared memory a window at a time), 128
// tokens per tile, through rings as deep as shared memory allows (3 stages at D = 128).
//   warp 0      TMA producer (Q tile once, K/V blocks through the block table)
//   warp 1      TMEM allocation and the single UMMA-issuing lane: S_j = Q K_j^T into one of
//               two TMEM S buffers (the next tile's Q K^T overlaps this tile's softmax),
//               O += P_j V_j with P read from TMEM (it overwrites S_j)
//   warps 2-5   softmax, one query row per thread (TMEM lane), lazy O rescale (2^8)
// Long contexts with few items are split over key ranges; each split writes its unnormalised
// O rows with their max and sum, and a merge kernel combines them (log-sum-exp). Keys past the
// context are masked; V rows past the last key of the item's last tile are zeroed in shared
// memory before P V, so unwritten cache memory never reaches the accumulator. Every wait is
// bounded; block-table entries outside the pool are reported (and read as zeros).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "common.h"
#include "paged_attention.cuh"
#include "ptx.cuh"

namespace tllm {

__device__ int g_ppf_status = 0;

int ppf_read_status(int *out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_ppf_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyFromSymbol(paged prefill status)");
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_ppf_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyToSymbol(paged prefill status)");
  *out = v;
  return TLLM_OK;
}

namespace ppf {
namespace {

constexpr int BM = 128;  // query rows per tile
constexpr int BN = 128;  // keys per tile
constexpr int kThreads = 192;
constexpr int kSoftmaxThreads = 128;
constexpr int TMEM_COLS = 512;
constexpr int O_COL = 256;  // S buffers at columns [0,128) and [128,256)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazyRescaleLog2 = 8.0f;
constexpr int kBtWin = 128;  // block-table entries per staged window (two windows)

enum : int {
  SITE_Q = 0x21,
  SITE_KFULL = 0x22,
  SITE_KEMPTY = 0x23,
  SITE_VFULL = 0x24,
  SITE_VEMPTY = 0x25,
  SITE_SFULL = 0x26,
  SITE_PFULL = 0x27,
  SITE_PVDONE = 0x28,
};

template <int D>
struct Geo {
  static constexpr int SWB = D * 2 >= 128 ? 128 : D * 2;  // swizzle span (bytes per row chunk)
  static constexpr int CHUNKS = D * 2 / SWB;
  static constexpr int CHUNK_BYTES = BM * SWB;
  static constexpr int TILE_BYTES = BM * D * 2;
  static constexpr uint32_t LAYOUT = SWB == 128 ? 2u : (SWB == 64 ? 4u : 6u);
  // K/V ring depth: as many stages as 227 KB of shared memory holds (at most 4).
  static constexpr int kSmemMax = 227 * 1024;
  static constexpr int kFixed = 256 + 8 * kBtWin + 1024;  // barriers, block-table windows, align
  static constexpr int NST_FIT = (kSmemMax - kFixed - TILE_BYTES) / (2 * TILE_BYTES);
  static constexpr int NST = NST_FIT > 4 ? 4 : NST_FIT;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + TILE_BYTES;
  static constexpr int V_OFF = K_OFF + NST * TILE_BYTES;
  static constexpr int BAR_OFF = V_OFF + NST * TILE_BYTES;
  static constexpr int BT_OFF = BAR_OFF + 256;
  static constexpr int SMEM_BYTES = BT_OFF + 8 * kBtWin + 1024;
  static_assert(NST >= 2 && SMEM_BYTES <= kSmemMax, "shared memory plan");
};

struct Args {
  void *o;
  int64_t so0, so1, so2, so3;
  float *ws_ml;   // [items, splits, 128, 2] (max in log2 units, sum)
  float *ws_acc;  // [items, splits, 128, D]
  const int32_t *block_tables;
  const int32_t *context_lens;
  int64_t sbt0, sbt1;
  int Hkv, G, Sq;
  int st, gt;      // query tile: st tokens x gt heads
  int n_st, n_rt;  // token tiles, row tiles per KV head
  int splits, tps; // key splits, key tiles per split
  int block_size, max_blocks, num_blocks;
  float scale_log2;
  int causal;
  int vec_store;
};

template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int k) {
  using G = Geo<D>;
  const int byte = k * 32;
  const uint32_t addr = base + (byte / G::SWB) * G::CHUNK_BYTES + (byte % G::SWB);
  return make_sdesc(addr, 16, 8 * G::SWB, G::LAYOUT);
}

__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[32]) { tmem_ld32(taddr, r); }
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[16]) { tmem_ld16(taddr, r); }
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t (&r)[32]) { tmem_st32(taddr, r); }
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t (&r)[16]) { tmem_st16(taddr, r); }

// Keys an item's query rows can see: all of the context, or (causal) up to the position of
// the tile's last query token.
__device__ __forceinline__ int tile_keys(const Args &a, int ctx, int s_last) {
  if (!a.causal) return ctx;
  const int n = ctx - a.Sq + s_last + 1;
  return n < 0 ? 0 : (n > ctx ? ctx : n);
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const Args a) {
  using G = Geo<D>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int OC = D < 32 ? D : 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + G::BAR_OFF);
  constexpr int NST = G::NST;
  uint64_t *q_full = bars + 0;
  uint64_t *k_full = bars + 1;    // [NST]
  uint64_t *k_empty = bars + 5;   // [NST]
  uint64_t *v_full = bars + 9;    // [NST]
  uint64_t *v_empty = bars + 13;  // [NST]
  uint64_t *s_full = bars + 17;   // [2] per S buffer
  uint64_t *p_full = bars + 19;
  uint64_t *pv_done = bars + 20;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 21);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- work item ----
  const int item = static_cast<int>(blockIdx.x) / a.splits;
  const int split = static_cast<int>(blockIdx.x) % a.splits;
  const int rt = item % a.n_rt;
  const int bk = item / a.n_rt;  // b * Hkv + kvh
  const int kvh = bk % a.Hkv;
  const int b = bk / a.Hkv;
  const int g0 = (rt / a.n_st) * a.gt;
  const int s0 = (rt % a.n_st) * a.st;
  const int s_last = min(s0 + a.st, a.Sq) - 1;
  int ctx = __ldg(a.context_lens + b);
  ctx = max(0, min(ctx, a.max_blocks * a.block_size));
  const int n_keys = tile_keys(a, ctx, s_last);  // keys any row of the tile sees
  const int n_tiles_all = (n_keys + BN - 1) / BN;
  const int t_begin = split * a.tps;
  const int t_end = min(n_tiles_all, t_begin + a.tps);
  const int n = max(0, t_end - t_begin);  // key tiles of this CTA
  // The item's last loaded key tile keeps only its first `tail` rows of V.
  const int tail = (t_end == n_tiles_all && n > 0) ? n_keys - (n_tiles_all - 1) * BN : BN;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < NST; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&k_empty[s]), 1);
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 1);
    }
    for (int s = 0; s < 2; ++s) mbar_init(smem_u32(&s_full[s]), 1);
    mbar_init(smem_u32(p_full), kSoftmaxThreads);
    mbar_init(smem_u32(pv_done), 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const uint32_t sQ = smem_u32(smem + G::Q_OFF);
  const uint32_t sK = smem_u32(smem + G::K_OFF);
  const uint32_t sV = smem_u32(smem + G::V_OFF);

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (n > 0) {
      if (lane == 0) {
        const uint32_t qb = smem_u32(q_full);
        mbar_arrive_expect_tx(qb, a.st * a.gt * G::SWB * G::CHUNKS);
#pragma unroll
        for (int c = 0; c < G::CHUNKS; ++c)
          tma_load_4d(sQ + c * G::CHUNK_BYTES, &tm_q, qb, c * (G::SWB / 2), s0,
                      kvh * a.G + g0, b);
      }
      // Block-table entries are staged in shared memory a window at a time by the whole warp
      // (one round trip per window instead of one per tile), in two alternating windows. The
      // copies of a tile are issued by one lane per (cache block, 128-byte chunk), in one
      // warp instruction: a single lane issuing them one after another is the bottleneck.
      // K of tile j goes out one iteration before V of tile j, so waiting for a V slot (which
      // frees after P V) never holds back the next K tile.
      const int32_t *bt = a.block_tables + b * a.sbt0;
      int *bt_s = reinterpret_cast<int *>(smem + G::BT_OFF);  // [2][kBtWin]
      const int bpt = BN / a.block_size;  // cache blocks per key tile
      const int win_tiles = kBtWin / bpt;
      const int blk_bytes = a.block_size * G::SWB;
      const int nblk_all = (n_keys + a.block_size - 1) / a.block_size;
      const int my_i = lane / G::CHUNKS;  // block of the tile this lane copies
      const int my_c = lane % G::CHUNKS;  // 128-byte chunk of the row this lane copies
      // One tile's copies into stage `st` of ring `dst`, completing on `full`.
      auto issue_tile = [&](int j, uint32_t dst, const CUtensorMap *map, uint64_t *full,
                            uint64_t *empty) -> bool {
        const int st = j % NST;
        const int nblk = min(bpt, nblk_all - (t_begin + j) * bpt);
        bool got = true;
        if (lane == 0) {
          got = mbar_wait(smem_u32(&empty[st]), ((j / NST) & 1) ^ 1, abort_flag, &g_ppf_status,
                          TLLM_DEV_WAIT_TIMEOUT + (map == &tm_k ? SITE_KEMPTY : SITE_VEMPTY));
          if (got) mbar_arrive_expect_tx(smem_u32(&full[st]), nblk * blk_bytes * G::CHUNKS);
        }
        if (!__shfl_sync(0xffffffffu, got, 0)) return false;
        if (my_i < nblk) {
          const int phys = bt_s[((j / win_tiles) & 1) * kBtWin + (j % win_tiles) * bpt + my_i];
          tma_load_4d(dst + st * G::TILE_BYTES + my_c * G::CHUNK_BYTES + my_i * blk_bytes, map,
                      smem_u32(&full[st]), my_c * (G::SWB / 2), kvh, 0, phys);
        }
        return true;
      };
      for (int j = 0; j <= n; ++j) {
        if (j < n && j % win_tiles == 0) {
          int *win = bt_s + ((j / win_tiles) & 1) * kBtWin;
          const int e0 = (t_begin + j) * bpt;
          __syncwarp();
          for (int e = lane; e < kBtWin; e += 32) {
            int p = a.num_blocks;  // past the pool: TMA fills zeros
            if (e0 + e < nblk_all) {
              p = __ldg(bt + static_cast<int64_t>(e0 + e) * a.sbt1);
              if (p < 0 || p >= a.num_blocks) {
                atomicCAS(&g_ppf_status, 0, TLLM_DEV_BAD_INDEX);
                p = a.num_blocks;
              }
            }
            win[e] = p;
          }
          __syncwarp();
        }
        if (j < n && !issue_tile(j, sK, &tm_k, k_full, k_empty)) break;
        if (j >= 1 && !issue_tile(j - 1, sV, &tm_v, v_full, v_empty)) break;
      }
    }
  } else if (warp == 1) {
    // ------------------------------ UMMA issuer -------------------------------
    if (lane == 0 && n > 0) {
      const uint32_t idesc_qk = make_idesc_f16(BM, BN, kBF16, false, false);
      const uint32_t idesc_pv = make_idesc_f16(BM, D, kBF16, false, true);
      auto issue_qk = [&](int j) {
        const uint32_t kbase = sK + (j % NST) * G::TILE_BYTES;
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          umma_f16_ss(tmem_base + (j & 1) * BN, kmajor_desc<D>(sQ, k), kmajor_desc<D>(kbase, k),
                      idesc_qk, k != 0 ? 1u : 0u);
        umma_commit(smem_u32(&s_full[j & 1]));
        umma_commit(smem_u32(&k_empty[j % NST]));
      };
      bool ok = mbar_wait(smem_u32(q_full), 0, abort_flag, &g_ppf_status,
                          TLLM_DEV_WAIT_TIMEOUT + SITE_Q);
      for (int j = 0; j < 2 && j < n && ok; ++j) {
        ok = mbar_wait(smem_u32(&k_full[j]), 0, abort_flag, &g_ppf_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_KFULL);
        if (ok) {
          tc_fence_after();
          issue_qk(j);
        }
      }
      for (int j = 0; j < n && ok; ++j) {
        const int s = j % NST;
        if (!mbar_wait(smem_u32(p_full), j & 1, abort_flag, &g_ppf_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_PFULL) ||
            !mbar_wait(smem_u32(&v_full[s]), (j / NST) & 1, abort_flag, &g_ppf_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_VFULL))
          break;
        tc_fence_after();
        const uint32_t vbase = sV + s * G::TILE_BYTES;
        const uint32_t p_tmem = tmem_base + (j & 1) * BN;
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          const uint64_t bdesc =
              make_sdesc(vbase + k * 16 * G::SWB, G::CHUNK_BYTES, 8 * G::SWB, G::LAYOUT);
          umma_f16_ts(tmem_base + O_COL, p_tmem + k * 8, bdesc, idesc_pv, (j | k) != 0 ? 1u : 0u);
        }
        umma_commit(smem_u32(&v_empty[s]));
        umma_commit(smem_u32(pv_done));
        if (j + 2 < n) {
          // S_j's buffer is rewritten only after the P V above (same tensor pipe, in order).
          if (!mbar_wait(smem_u32(&k_full[(j + 2) % NST]), ((j + 2) / NST) & 1, abort_flag,
                         &g_ppf_status, TLLM_DEV_WAIT_TIMEOUT + SITE_KFULL))
            break;
          tc_fence_after();
          issue_qk(j + 2);
        }
      }
    }
  } else {
    // ------------------------------ softmax / epilogue ------------------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int g = g0 + row / a.st;
    const int s = s0 + row % a.st;
    const bool row_valid = row < a.st * a.gt && g < a.G && s < a.Sq;
    const int row_keys = row_valid ? tile_keys(a, ctx, s) : 0;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t o_tm = tmem_base + lane_off + O_COL;
    float m_use = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int sb = j & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&s_full[sb]), (j >> 1) & 1, abort_flag,
                                             &g_ppf_status, TLLM_DEV_WAIT_TIMEOUT + SITE_SFULL))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t s_tm = tmem_base + lane_off + sb * BN;
      const int k0 = (t_begin + j) * BN;
      uint32_t sr[BN];
      tmem_ld4x32(s_tm, sr);
      if (k0 + BN > row_keys) {
#pragma unroll
        for (int t = 0; t < BN; ++t)
          if (k0 + t >= row_keys) sr[t] = __float_as_uint(-INFINITY);
      }
      float mx8[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) mx8[t] = __uint_as_float(sr[t]);
#pragma unroll
      for (int t = 8; t < BN; t += 2)
        mx8[(t >> 1) & 7] =
            max3f(mx8[(t >> 1) & 7], __uint_as_float(sr[t]), __uint_as_float(sr[t + 1]));
      float mx = max3f(max3f(mx8[0], mx8[1], mx8[2]), max3f(mx8[3], mx8[4], mx8[5]),
                       fmaxf(mx8[6], mx8[7]));
      mx *= a.scale_log2;
      // O is stable once the previous tile's P V has completed.
      if (j > 0 && !__all_sync(0xffffffffu,
                               mbar_wait(smem_u32(pv_done), (j - 1) & 1, abort_flag, &g_ppf_status,
                                         TLLM_DEV_WAIT_TIMEOUT + SITE_PVDONE))) {
        ok = false;
        break;
      }
      float alpha = 1.0f;
      bool rescale = false;
      if (m_use == -INFINITY) {
        m_use = mx;  // nothing accumulated yet (every earlier P of this row was 0)
      } else if (mx > m_use + kLazyRescaleLog2) {
        alpha = ex2_approx(m_use - mx);
        m_use = mx;
        rescale = true;
      }
      const float neg_m = m_use == -INFINITY ? 0.f : -m_use;
      const uint64_t scale2 = f2_pack(a.scale_log2, a.scale_log2);
      const uint64_t negm2 = f2_pack(neg_m, neg_m);
      uint64_t ps2[4] = {0ull, 0ull, 0ull, 0ull};
#pragma unroll
      for (int hlf = 0; hlf < 2; ++hlf) {
        uint32_t pk[32];
#pragma unroll
        for (int t = 0; t < 64; t += 2) {
          const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(sr[64 * hlf + t]),
                                             __uint_as_float(sr[64 * hlf + t + 1])),
                                     scale2, negm2);
          float x0, x1;
          f2_unpack(x2, x0, x1);
          const float p0 = ex2_approx(x0);
          const float p1 = ex2_approx(x1);
          ps2[(t >> 1) & 3] = f2_add(ps2[(t >> 1) & 3], f2_pack(p0, p1));
          pk[t >> 1] = Pack2<T>::pack(p0, p1);
        }
        tmem_st32(s_tm + 32 * hlf, pk);
      }
      float psa, psb, psc, psd, pse, psf, psg, psh;
      f2_unpack(ps2[0], psa, psb);
      f2_unpack(ps2[1], psc, psd);
      f2_unpack(ps2[2], pse, psf);
      f2_unpack(ps2[3], psg, psh);
      l_run = l_run * alpha + (((psa + psb) + (psc + psd)) + ((pse + psf) + (psg + psh)));
      if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
        for (int c = 0; c < D; c += OC) {
          uint32_t r[OC];
          tmem_ld_cols(o_tm + c, r);
#pragma unroll
          for (int t = 0; t < OC; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * alpha);
          tmem_st_cols(o_tm + c, r);
        }
      }
      if (j == n - 1 && tail < BN) {
        // Rows of the last V tile past the item's last key are not real tokens: zero them
        // (thread `row` owns V row `row`) before P V reads the tile.
        const int vs = j % NST;
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&v_full[vs]), (j / NST) & 1, abort_flag,
                                               &g_ppf_status, TLLM_DEV_WAIT_TIMEOUT + SITE_VFULL))) {
          ok = false;
          break;
        }
        if (row >= tail) {
          uint8_t *vrow = smem + G::V_OFF + vs * G::TILE_BYTES + row * G::SWB;
#pragma unroll
          for (int c = 0; c < G::CHUNKS; ++c)
#pragma unroll
            for (int x = 0; x < G::SWB; x += 16)
              *reinterpret_cast<uint4 *>(vrow + c * G::CHUNK_BYTES + x) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      tc_fence_before();
      mbar_arrive(smem_u32(p_full));
    }
    // ---- epilogue ----
    bool have_o = false;
    if (ok && n > 0) {
      have_o = __all_sync(0xffffffffu, mbar_wait(smem_u32(pv_done), (n - 1) & 1, abort_flag,
                                                 &g_ppf_status, TLLM_DEV_WAIT_TIMEOUT + SITE_PVDONE));
      if (have_o) tc_fence_after();
    }
    if (ok && (have_o || n == 0)) {
      const int item_split = static_cast<int>(blockIdx.x);
      if (a.splits == 1) {
        const float inv_l = 1.0f / l_run;  // no visible key: 0/0 = NaN, as the reference
        T *orow = static_cast<T *>(a.o) + b * a.so0 + static_cast<int64_t>(kvh * a.G + g) * a.so1 +
                  static_cast<int64_t>(s) * a.so2;
#pragma unroll 1
        for (int c = 0; c < D; c += OC) {
          uint32_t r[OC];
          if (have_o) {
            tmem_ld_cols(o_tm + c, r);
          } else {
#pragma unroll
            for (int t = 0; t < OC; ++t) r[t] = 0u;
          }
          if (row_valid) {
            if (a.vec_store) {
#pragma unroll
              for (int t = 0; t < OC; t += 8) {
                uint4 pk;
                pk.x = Pack2<T>::pack(__uint_as_float(r[t + 0]) * inv_l, __uint_as_float(r[t + 1]) * inv_l);
                pk.y = Pack2<T>::pack(__uint_as_float(r[t + 2]) * inv_l, __uint_as_float(r[t + 3]) * inv_l);
                pk.z = Pack2<T>::pack(__uint_as_float(r[t + 4]) * inv_l, __uint_as_float(r[t + 5]) * inv_l);
                pk.w = Pack2<T>::pack(__uint_as_float(r[t + 6]) * inv_l, __uint_as_float(r[t + 7]) * inv_l);
                *reinterpret_cast<uint4 *>(orow + c + t) = pk;
              }
            } else {
#pragma unroll
              for (int t = 0; t < OC; ++t)
                orow[(c + t) * a.so3] = from_f32<T>(__uint_as_float(r[t]) * inv_l);
            }
          }
        }
      } else {
        const int64_t slot = static_cast<int64_t>(item_split) * BM + row;
        if (row_valid) {
          a.ws_ml[2 * slot] = m_use;
          a.ws_ml[2 * slot + 1] = l_run;
        }
        float *acc = a.ws_acc + slot * D;
#pragma unroll 1
        for (int c = 0; c < D; c += OC) {
          uint32_t r[OC];
          if (have_o) {
            tmem_ld_cols(o_tm + c, r);
          } else {
#pragma unroll
            for (int t = 0; t < OC; ++t) r[t] = 0u;
          }
          if (row_valid) {
#pragma unroll
            for (int t = 0; t < OC; t += 4)
              *reinterpret_cast<float4 *>(acc + c + t) =
                  make_float4(__uint_as_float(r[t]), __uint_as_float(r[t + 1]),
                              __uint_as_float(r[t + 2]), __uint_as_float(r[t + 3]));
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

// One CTA of D threads per (item, valid row): log-sum-exp merge of the item's key splits.
template <typename T, int D>
__global__ void __launch_bounds__(D) paged_prefill_merge_kernel(const Args a) {
  const int row = blockIdx.x;
  const int item = blockIdx.y;
  const int d = threadIdx.x;
  const int rt = item % a.n_rt;
  const int bk = item / a.n_rt;
  const int kvh = bk % a.Hkv;
  const int b = bk / a.Hkv;
  const int g = (rt / a.n_st) * a.gt + row / a.st;
  const int s = (rt % a.n_st) * a.st + row % a.st;
  if (g >= a.G || s >= a.Sq) return;
  const int64_t base = static_cast<int64_t>(item) * a.splits;
  float M = -INFINITY;
  for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, a.ws_ml[2 * ((base + sp) * BM + row)]);
  float L = 0.f, A = 0.f;
  for (int sp = 0; sp < a.splits; ++sp) {
    const int64_t slot = (base + sp) * BM + row;
    const float m = a.ws_ml[2 * slot];
    const float wgt = m == -INFINITY ? 0.f : exp2f(m - M);
    L = fmaf(a.ws_ml[2 * slot + 1], wgt, L);
    A = fmaf(a.ws_acc[slot * D + d], wgt, A);
  }
  T *op = static_cast<T *>(a.o) + b * a.so0 + static_cast<int64_t>(kvh * a.G + g) * a.so1 +
          static_cast<int64_t>(s) * a.so2;
  op[d * a.so3] = from_f32<T>(A / L);
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct Plan {
  int st = 1, gt = 1, n_st = 1, n_gt = 1, n_rt = 1;
  int64_t items = 0;  // (b, kvh, row tile)
  int splits = 1, tps = 1;
  size_t ml_bytes = 0, ws_bytes = 0;
};

Plan make_plan(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t D, int64_t block_size,
               int64_t max_blocks, int sms) {
  Plan p;
  const int64_t G = Hq / Hkv;
  if (Sq >= BM) {
    p.st = BM;
    p.gt = 1;
  } else {
    p.st = static_cast<int>(Sq);
    p.gt = static_cast<int>(std::min<int64_t>(G, BM / Sq));
  }
  p.n_st = static_cast<int>((Sq + p.st - 1) / p.st);
  p.n_gt = static_cast<int>((G + p.gt - 1) / p.gt);
  p.n_rt = p.n_st * p.n_gt;
  p.items = B * Hkv * p.n_rt;
  const int64_t max_tiles = std::max<int64_t>(1, (max_blocks * block_size + BN - 1) / BN);
  int64_t splits = 1;
  const int64_t want = 2LL * (sms > 0 ? sms : 148);
  if (p.items < want) splits = std::min<int64_t>(max_tiles, (want + p.items - 1) / p.items);
  const int64_t tps = (max_tiles + splits - 1) / splits;
  splits = (max_tiles + tps - 1) / tps;
  p.splits = static_cast<int>(splits);
  p.tps = static_cast<int>(tps);
  if (p.splits > 1) {
    p.ml_bytes = (static_cast<size_t>(p.items * p.splits * BM * 2) * sizeof(float) + 255) / 256 * 256;
    p.ws_bytes = p.ml_bytes + static_cast<size_t>(p.items * p.splits * BM * D) * sizeof(float);
  }
  return p;
}

template <typename T, int D>
int launch_d(const void *q, const void *kc, const void *vc, void *o, void *ws, const Plan &pl,
             Args a, int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, const int64_t *sq,
             const int64_t *skc, const int64_t *svc, cudaStream_t st) {
  using G = Geo<D>;
  const CUtensorMapDataType dt = std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUtensorMapSwizzle sw = G::SWB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : (G::SWB == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  CUtensorMap mq, mk, mv;
  {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)Sq, (uint64_t)Hq, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)sq[2] * 2, (uint64_t)sq[1] * 2, (uint64_t)sq[0] * 2};
    const uint32_t box[4] = {static_cast<uint32_t>(G::SWB / 2), static_cast<uint32_t>(pl.st),
                             static_cast<uint32_t>(pl.gt), 1};
    int rc = encode_tiled(&mq, dt, 4, const_cast<void *>(q), dims, str, box, sw);
    if (rc) return rc;
  }
  {
    // Caches [num_blocks, block_size, Hkv, D] as 4-D (D, Hkv, block_size, num_blocks); one box is
    // the block_size tokens of one head in one block.
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)Hkv, (uint64_t)a.block_size, (uint64_t)a.num_blocks};
    const uint32_t box[4] = {static_cast<uint32_t>(G::SWB / 2), 1, static_cast<uint32_t>(a.block_size), 1};
    const uint64_t strk[3] = {(uint64_t)skc[2] * 2, (uint64_t)skc[1] * 2, (uint64_t)skc[0] * 2};
    int rc = encode_tiled(&mk, dt, 4, const_cast<void *>(kc), dims, strk, box, sw);
    if (rc) return rc;
    const uint64_t strv[3] = {(uint64_t)svc[2] * 2, (uint64_t)svc[1] * 2, (uint64_t)svc[0] * 2};
    rc = encode_tiled(&mv, dt, 4, const_cast<void *>(vc), dims, strv, box, sw);
    if (rc) return rc;
  }
  if (pl.splits > 1) {
    a.ws_ml = static_cast<float *>(ws);
    a.ws_acc = reinterpret_cast<float *>(static_cast<char *>(ws) + pl.ml_bytes);
  }
  auto kern = paged_prefill_kernel<T, D>;
  KernelLaunchInfo info;
  const int rc = prepare_kernel(reinterpret_cast<const void *>(kern), G::SMEM_BYTES, kThreads, 1, &info);
  if (rc) return rc;
  cudaError_t e;
  const unsigned grid = static_cast<unsigned>(pl.items * pl.splits);
  kern<<<grid, kThreads, G::SMEM_BYTES, st>>>(mq, mk, mv, a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "paged prefill launch");
  if (pl.splits > 1) {
    dim3 mgrid(static_cast<unsigned>(pl.st * pl.gt), static_cast<unsigned>(pl.items));
    paged_prefill_merge_kernel<T, D><<<mgrid, D, 0, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "paged prefill merge launch");
  }
  return TLLM_OK;
}

}  // namespace
}  // namespace ppf
}  // namespace tllm

namespace tllm {
namespace ppf {
namespace {
// Single-token decode with one query head per KV head is the reference's decode: it goes to
// the CUDA-core split-KV kernel, which reads each token's K/V row with vector loads (this
// kernel is bound by TMA box issue on paged blocks and reaches less there).
bool use_decode_path(int64_t Hq, int64_t Hkv, int64_t Sq, int64_t D) {
  (void)D;
  return Sq == 1 && Hq == Hkv;
}
// Calls with at most 16 query rows per KV head (G = Hq / Hkv heads times Sq new tokens; D 64
// or 128), other than the single-token Hq = Hkv case above, go to the grouped-query split
// kernel, which reads each token's K/V rows once for all those rows.
bool use_gqa_decode_path(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t D,
                         int64_t block_size, int64_t max_blocks) {
  if (Sq == 1 && Hq == Hkv) return false;
  if ((Hq / Hkv) * Sq > 16) return false;
  const paged::Plan pl = paged::plan_gqa(B, Hq, Hkv, Sq, D, block_size, max_blocks, sm_count());
  return paged::gqa_supported(Hq / Hkv, Sq, D, pl);
}
}  // namespace
}  // namespace ppf
}  // namespace tllm

extern "C" size_t tllm_paged_prefill_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq,
                                                    int64_t D, int64_t block_size,
                                                    int64_t max_blocks) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Sq <= 0 || D <= 0 || block_size <= 0 || max_blocks <= 0 ||
      Hq % Hkv != 0)
    return 0;
  if (tllm::ppf::use_decode_path(Hq, Hkv, Sq, D))
    return tllm::paged::plan(B, Hq, D, block_size, max_blocks, tllm::sm_count()).ws_bytes;
  if (tllm::ppf::use_gqa_decode_path(B, Hq, Hkv, Sq, D, block_size, max_blocks))
    return tllm::paged::plan_gqa(B, Hq, Hkv, Sq, D, block_size, max_blocks, tllm::sm_count()).ws_bytes;
  return tllm::ppf::make_plan(B, Hq, Hkv, Sq, D, block_size, max_blocks, tllm::sm_count()).ws_bytes;
}

extern "C" int tllm_paged_prefill(const void *q, const void *k_cache, const void *v_cache,
                                  const int32_t *block_tables, const int32_t *context_lens,
                                  void *o, void *workspace, size_t workspace_bytes, int64_t B,
                                  int64_t Hq, int64_t Hkv, int64_t Sq, int64_t D,
                                  int64_t block_size, int64_t max_blocks, int64_t num_blocks,
                                  const int64_t *sq, const int64_t *skc, const int64_t *svc,
                                  const int64_t *sbt, const int64_t *so, float sm_scale,
                                  int causal, int dtype, void *stream) {
  using namespace tllm;
  using namespace tllm::ppf;
  clear_error();
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16,
                 "paged_prefill: unsupported dtype %d", dtype);
  TLLM_CHECK_ARG(B >= 0 && Hq >= 0 && Hkv >= 0 && Sq >= 0, "paged_prefill: negative dimension");
  TLLM_CHECK_ARG(D == 16 || D == 32 || D == 64 || D == 128,
                 "paged_prefill: head dim %lld not in {16,32,64,128}", (long long)D);
  TLLM_CHECK_ARG(block_size == 16 || block_size == 32 || block_size == 64,
                 "paged_prefill: block_size %lld not in {16,32,64}", (long long)block_size);
  TLLM_CHECK_ARG(sq && skc && svc && sbt && so, "paged_prefill: null stride array");
  if (B == 0 || Hq == 0 || Sq == 0) return TLLM_OK;
  TLLM_CHECK_ARG(Hkv >= 1 && Hq % Hkv == 0, "paged_prefill: %lld query heads do not group over %lld KV heads",
                 (long long)Hq, (long long)Hkv);
  TLLM_CHECK_ARG(q && k_cache && v_cache && block_tables && context_lens && o,
                 "paged_prefill: null tensor pointer");
  TLLM_CHECK_ARG(max_blocks >= 1 && num_blocks >= 1, "paged_prefill: empty block table or pool");
  TLLM_CHECK_ARG(max_blocks * block_size < (1LL << 30) && num_blocks < (1LL << 31) &&
                     Sq < (1LL << 30) && B * Hq < (1LL << 31),
                 "paged_prefill: problem too large");
  TLLM_CHECK_ARG(sq[3] == 1 && skc[3] == 1 && svc[3] == 1,
                 "paged_prefill: q and the caches need a unit innermost stride");
  for (int i = 0; i < 3; ++i)
    TLLM_CHECK_ARG(sq[i] % 8 == 0 && skc[i] % 8 == 0 && svc[i] % 8 == 0,
                   "paged_prefill: q/cache strides must be multiples of 8 elements");
  TLLM_CHECK_ARG(aligned16(q) && aligned16(k_cache) && aligned16(v_cache),
                 "paged_prefill: q and the caches must be 16-byte aligned");
  const bool gqa = use_gqa_decode_path(B, Hq, Hkv, Sq, D, block_size, max_blocks);
  if (use_decode_path(Hq, Hkv, Sq, D) || gqa) {
    const paged::Plan dp = gqa ? paged::plan_gqa(B, Hq, Hkv, Sq, D, block_size, max_blocks, sm_count())
                               : paged::plan(B, Hq, D, block_size, max_blocks, sm_count());
    paged::Params p{};
    p.q = q; p.k_cache = k_cache; p.v_cache = v_cache;
    p.block_tables = block_tables; p.context_lens = context_lens; p.o = o;
    p.B = B; p.H = Hq; p.D = D;
    p.num_blocks = num_blocks;
    p.block_size = static_cast<int>(block_size);
    p.log2_bs = block_size == 16 ? 4 : (block_size == 32 ? 5 : 6);
    p.max_tokens = static_cast<int>(dp.max_tokens);
    p.chunk = static_cast<int>(dp.chunk);
    p.num_splits = static_cast<int>(dp.num_splits);
    p.sq0 = sq[0]; p.sq1 = sq[1]; p.sq3 = sq[3];
    p.skc0 = skc[0]; p.skc1 = skc[1]; p.skc2 = skc[2]; p.skc3 = skc[3];
    p.svc0 = svc[0]; p.svc1 = svc[1]; p.svc2 = svc[2]; p.svc3 = svc[3];
    p.sbt0 = sbt[0]; p.sbt1 = sbt[1];
    p.so0 = so[0]; p.so1 = so[1]; p.so3 = so[3];
    p.sm_scale = sm_scale;
    p.G = static_cast<int>(Hq / Hkv);
    p.Hkv = Hkv;
    p.Sq = static_cast<int>(Sq);
    p.causal = causal ? 1 : 0;
    p.sq2 = sq[2];
    p.so2 = so[2];
    int rc = paged::validate(p);
    if (rc) return rc;
    if (dp.num_splits > 1) {
      if (!workspace || workspace_bytes < dp.ws_bytes)
        return fail(TLLM_ERR_WORKSPACE, "paged_prefill: workspace of %zu bytes needed, %zu given",
                    dp.ws_bytes, workspace_bytes);
      TLLM_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
                     "paged_prefill: workspace must be 256-byte aligned");
      p.ws_ml = static_cast<float *>(workspace);
      p.ws_acc = reinterpret_cast<float *>(static_cast<char *>(workspace) + dp.ws_acc_offset);
    }
    if (gqa) return paged::run_gqa(p, dtype, static_cast<cudaStream_t>(stream));
    return paged::run(p, dtype, static_cast<cudaStream_t>(stream));
  }
  const Plan pl = make_plan(B, Hq, Hkv, Sq, D, block_size, max_blocks, sm_count());
  TLLM_CHECK_ARG(pl.items * pl.splits < (1LL << 31), "paged_prefill: grid too large");
  if (pl.splits > 1) {
    if (!workspace || workspace_bytes < pl.ws_bytes)
      return fail(TLLM_ERR_WORKSPACE, "paged_prefill: workspace of %zu bytes needed, %zu given",
                  pl.ws_bytes, workspace_bytes);
    TLLM_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
                   "paged_prefill: workspace must be 256-byte aligned");
  }
  Args a{};
  a.o = o;
  a.so0 = so[0]; a.so1 = so[1]; a.so2 = so[2]; a.so3 = so[3];
  a.block_tables = block_tables;
  a.context_lens = context_lens;
  a.sbt0 = sbt[0]; a.sbt1 = sbt[1];
  a.Hkv = static_cast<int>(Hkv);
  a.G = static_cast<int>(Hq / Hkv);
  a.Sq = static_cast<int>(Sq);
  a.st = pl.st; a.gt = pl.gt; a.n_st = pl.n_st; a.n_rt = pl.n_rt;
  a.splits = pl.splits; a.tps = pl.tps;
  a.block_size = static_cast<int>(block_size);
  a.max_blocks = static_cast<int>(max_blocks);
  a.num_blocks = static_cast<int>(num_blocks);
  a.scale_log2 = sm_scale * kLog2e;
  a.causal = causal ? 1 : 0;
  a.vec_store = (so[3] == 1 && so[0] % 8 == 0 && so[1] % 8 == 0 && so[2] % 8 == 0 && aligned16(o)) ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TLLM_PPF_LAUNCH(TT, DD) \
  return launch_d<TT, DD>(q, k_cache, v_cache, o, workspace, pl, a, B, Hq, Hkv, Sq, sq, skc, svc, st)
  if (dtype == TLLM_DTYPE_F16) {
    switch (D) {
      case 16: TLLM_PPF_LAUNCH(__half, 16);
      case 32: TLLM_PPF_LAUNCH(__half, 32);
      case 64: TLLM_PPF_LAUNCH(__half, 64);
      default: TLLM_PPF_LAUNCH(__half, 128);
    }
  }
  switch (D) {
    case 16: TLLM_PPF_LAUNCH(__nv_bfloat16, 16);
    case 32: TLLM_PPF_LAUNCH(__nv_bfloat16, 32);
    case 64: TLLM_PPF_LAUNCH(__nv_bfloat16, 64);
    default: TLLM_PPF_LAUNCH(__nv_bfloat16, 128);
  }
#undef TLLM_PPF_LAUNCH
}
