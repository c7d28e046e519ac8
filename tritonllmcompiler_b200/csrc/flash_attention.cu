// FlashAttention forward for sm_100a (tcgen05 + TMEM + TMA).
//
// Reference: python/triton_llm/ops/flash_attention.py:17-133 (Triton FA-2, 64x64 tiles,
// online softmax, causal mask applied to every tile with no tile skipping) and the oracle
// python/triton_llm/reference/flash_attention.py:12-29 (fp32 scores, triu(1) -> -inf mask,
// softmax, P@V, cast to q.dtype).
//
// B200 design: one CTA per (128-row query tile, b, h); grid ordered so the heaviest causal
// query tiles start first.
//   warp 0      TMA producer: Q once, then K_j / V_j tiles [128 x D] through two 2-slot rings.
//   warp 1      allocates 512 TMEM columns; one lane issues the UMMAs:
//                 S_j = Q K_j^T  (128x128, fp32, TMEM columns [0,128) / [128,256) alternately)
//                 O  += P_j V_j  (128xD, fp32, TMEM columns [256, 256+D))
//   warps 2-5   softmax: each thread owns one query row (TMEM lane), reads its S row with
//               tcgen05.ld, applies scale and mask in fp32 (log2 domain), keeps the running
//               max/sum in registers, writes P_j (I/O dtype) to shared memory in the UMMA
//               K-major 128B-swizzle layout and rescales its O row in TMEM when the max grows.
// Causal: only key tiles j <= i are visited for query tile i; only the diagonal tile and a
// ragged key tail are masked. The mask is top-left aligned (key j visible to query i iff
// j <= i), exactly as the reference's offs_m >= offs_n.
// Every CTA loads its own tiles; every mbarrier wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <cmath>
#include <type_traits>

#include "common.h"
#include "ptx.cuh"

namespace tllm {

__device__ int g_flash_status = 0;

int flash_read_status(int *out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_flash_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyFromSymbol(flash status)");
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_flash_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyToSymbol(flash status)");
  *out = v;
  return TLLM_OK;
}

namespace flash {
namespace {

constexpr int BM = 128;  // query rows per CTA
constexpr int BN = 128;  // key rows per tile
constexpr int kThreads = 192;
constexpr int kSoftmaxThreads = 128;
constexpr int TMEM_COLS = 512;
constexpr int S_COL0 = 0;
constexpr int O_COL = 256;
constexpr float kLog2e = 1.4426950408889634f;

enum : int {
  SITE_Q = 1,
  SITE_KFULL = 2,
  SITE_KEMPTY = 3,
  SITE_VFULL = 4,
  SITE_VEMPTY = 5,
  SITE_SFULL = 6,
  SITE_PREADY = 7,
  SITE_PVDONE = 8,
};

// Shared-memory geometry for head dim D: rows of SWB bytes (the swizzle span), D*2/SWB chunks.
template <int D>
struct Geo {
  static constexpr int SWB = D * 2 >= 128 ? 128 : D * 2;
  static constexpr int CHUNKS = D * 2 / SWB;
  static constexpr int CHUNK_BYTES = BM * SWB;  // 128 rows of one swizzle span
  static constexpr int TILE_BYTES = BM * D * 2;
  static constexpr uint32_t LAYOUT = SWB == 128 ? 2u : (SWB == 64 ? 4u : 6u);
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + TILE_BYTES;
  static constexpr int V_OFF = K_OFF + 2 * TILE_BYTES;
  static constexpr int P_OFF = V_OFF + 2 * TILE_BYTES;
  static constexpr int P_BYTES = BM * BN * 2;
  static constexpr int BAR_OFF = P_OFF + P_BYTES;
  static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
};

struct Args {
  void *o;
  int64_t so0, so1, so2, so3;
  int H, Sq, Sk;
  int n_qtiles;
  float scale_log2;
  int causal;
  int vec_store;
  int group;    // heads per scheduling group of the two-tile kernel (see pp_item)
  int n_small;  // groups of `group` heads; the rest have group + 1
  // Packed variable-length sequences (tllm_flash_attn_varlen_fwd): sequence b's query rows
  // are [cu_q[b], cu_q[b+1]) of q/o, its key rows [cu_k[b], cu_k[b+1]) of k/v; query head h
  // reads key/value head h / G. Sq and Sk then hold the maximum lengths.
  const int *cu_q;
  const int *cu_k;
  int G;
  int total_q, total_k;  // rows of q/o and of k/v: cumulative lengths are clamped to them
  // Optional [B, H, Sq] fp32 output (dense batches): log2 of each row's softmax normaliser in
  // the units of s * scale * log2(e), i.e. P = 2^(s * scale * log2(e) - lse). The backward
  // pass recomputes P from it.
  float *lse;
  // e4m3 inputs: the output is (P V) / l times this (the scale of V); the scales of q and k
  // are folded into scale_log2.
  float out_scale;
};

__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[32]) { tmem_ld32(taddr, r); }
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[16]) { tmem_ld16(taddr, r); }
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t (&r)[32]) { tmem_st32(taddr, r); }
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, const uint32_t (&r)[16]) { tmem_st16(taddr, r); }

// K-major operand (Q or K): k16 step `k` of the D reduction.
template <int D>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int k) {
  using G = Geo<D>;
  const int byte = k * 32;
  const uint32_t addr = base + (byte / G::SWB) * G::CHUNK_BYTES + (byte % G::SWB);
  return make_sdesc(addr, 16, 8 * G::SWB, G::LAYOUT);
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const Args a) {
  using G = Geo<D>;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int OC = D < 32 ? D : 32;  // O columns moved per TMEM load/store
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + G::BAR_OFF);
  uint64_t *q_full = bars + 0;
  uint64_t *k_full = bars + 1;   // [2]
  uint64_t *k_empty = bars + 3;  // [2]
  uint64_t *v_full = bars + 5;   // [2]
  uint64_t *v_empty = bars + 7;  // [2]
  uint64_t *s_full = bars + 9;   // [2]
  uint64_t *p_ready = bars + 11;
  uint64_t *pv_done = bars + 12;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 13);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // 1-D grid, head-major: the query tiles of one (b, h) are adjacent in launch order (so the
  // CTAs resident at any time share few heads' K/V in L2), heaviest causal tiles first.
  const int bh = static_cast<int>(blockIdx.x / a.n_qtiles);
  const int b = bh / a.H;
  const int h = bh % a.H;
  const int qt = a.n_qtiles - 1 - static_cast<int>(blockIdx.x % a.n_qtiles);
  const int q0 = qt * BM;
  const int kv_tiles_all = (a.Sk + BN - 1) / BN;
  int n_kv = kv_tiles_all;
  if (a.causal) {
    const int last_q = min(q0 + BM, a.Sq) - 1;
    const int lim = last_q / BN + 1;
    n_kv = min(n_kv, lim);
  }

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&k_empty[s]), 1);
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 1);
      mbar_init(smem_u32(&s_full[s]), 1);
    }
    mbar_init(smem_u32(p_ready), kSoftmaxThreads);
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
  const uint32_t sP = smem_u32(smem + G::P_OFF);

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0 && n_kv > 0) {
      const uint32_t qb = smem_u32(q_full);
      mbar_arrive_expect_tx(qb, G::TILE_BYTES);
#pragma unroll
      for (int c = 0; c < G::CHUNKS; ++c)
        tma_load_4d(sQ + c * G::CHUNK_BYTES, &tm_q, qb, c * (G::SWB / 2), q0, h, b);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        const uint32_t par = ((j >> 1) & 1) ^ 1;
        if (!mbar_wait(smem_u32(&k_empty[s]), par, abort_flag, &g_flash_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_KEMPTY))
          break;
        const uint32_t kb = smem_u32(&k_full[s]);
        mbar_arrive_expect_tx(kb, G::TILE_BYTES);
#pragma unroll
        for (int c = 0; c < G::CHUNKS; ++c)
          tma_load_4d(sK + s * G::TILE_BYTES + c * G::CHUNK_BYTES, &tm_k, kb, c * (G::SWB / 2),
                      j * BN, h, b);
        if (!mbar_wait(smem_u32(&v_empty[s]), par, abort_flag, &g_flash_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_VEMPTY))
          break;
        const uint32_t vb = smem_u32(&v_full[s]);
        mbar_arrive_expect_tx(vb, G::TILE_BYTES);
#pragma unroll
        for (int c = 0; c < G::CHUNKS; ++c)
          tma_load_4d(sV + s * G::TILE_BYTES + c * G::CHUNK_BYTES, &tm_v, vb, c * (G::SWB / 2),
                      j * BN, h, b);
      }
    }
  } else if (warp == 1) {
    // ------------------------------ UMMA issuer -------------------------------
    if (lane == 0 && n_kv > 0) {
      const uint32_t idesc_qk = make_idesc_f16(BM, BN, kBF16, false, false);
      const uint32_t idesc_pv = make_idesc_f16(BM, D, kBF16, false, true);
      bool ok = mbar_wait(smem_u32(q_full), 0, abort_flag, &g_flash_status,
                          TLLM_DEV_WAIT_TIMEOUT + SITE_Q);
      auto issue_qk = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(smem_u32(&k_full[s]), (j >> 1) & 1, abort_flag, &g_flash_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_KFULL))
          return false;
        tc_fence_after();
        const uint32_t kbase = sK + s * G::TILE_BYTES;
        const uint32_t d_tmem = tmem_base + S_COL0 + s * BN;
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          umma_f16_ss(d_tmem, kmajor_desc<D>(sQ, k), kmajor_desc<D>(kbase, k), idesc_qk,
                      k != 0 ? 1u : 0u);
        umma_commit(smem_u32(&k_empty[s]));
        umma_commit(smem_u32(&s_full[s]));
        return true;
      };
      if (ok) ok = issue_qk(0);
      if (ok && n_kv > 1) ok = issue_qk(1);
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        if (!mbar_wait(smem_u32(p_ready), j & 1, abort_flag, &g_flash_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_PREADY))
          break;
        if (!mbar_wait(smem_u32(&v_full[s]), (j >> 1) & 1, abort_flag, &g_flash_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_VFULL))
          break;
        tc_fence_after();
        const uint32_t vbase = sV + s * G::TILE_BYTES;
#pragma unroll
        for (int k = 0; k < BN / 16; ++k) {
          // P: K-major (key index), two 64-key chunks of 16 KB, 128B swizzle.
          const uint64_t adesc =
              make_sdesc(sP + (k >> 2) * (BM * 128) + (k & 3) * 32, 16, 1024, kSwizzle128B);
          // V: N-major (head dim), swizzle-span chunks CHUNK_BYTES apart (LBO), 8-key groups
          // 8*SWB apart (SBO); 16 keys = 16 rows of SWB bytes.
          const uint64_t bdesc =
              make_sdesc(vbase + k * 16 * G::SWB, G::CHUNK_BYTES, 8 * G::SWB, G::LAYOUT);
          umma_f16_ss(tmem_base + O_COL, adesc, bdesc, idesc_pv, (j | k) != 0 ? 1u : 0u);
        }
        umma_commit(smem_u32(&v_empty[s]));
        umma_commit(smem_u32(pv_done));
        if (j + 2 < n_kv) ok = issue_qk(j + 2);
      }
    }
  } else {
    // ------------------------------ softmax / epilogue ------------------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int qg = q0 + row;  // global query index of this thread's row
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    uint8_t *prow = smem + G::P_OFF + row * 128;
    for (int j = 0; j < n_kv; ++j) {
      const int s = j & 1;
      if (!mbar_wait(smem_u32(&s_full[s]), (j >> 1) & 1, abort_flag, &g_flash_status,
                     TLLM_DEV_WAIT_TIMEOUT + SITE_SFULL)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem_base + lane_off + S_COL0 + s * BN + c, r);
#pragma unroll
        for (int t = 0; t < 32; ++t) sv[c + t] = __uint_as_float(r[t]) * a.scale_log2;
      }
      const int k0 = j * BN;
      const bool need_mask = (k0 + BN > a.Sk) || (a.causal && k0 + BN - 1 > q0);
      if (need_mask) {
#pragma unroll
        for (int t = 0; t < BN; ++t) {
          const int kg = k0 + t;
          if (kg >= a.Sk || (a.causal && kg > qg)) sv[t] = -INFINITY;
        }
      }
      float mx = m_run;
#pragma unroll
      for (int t = 0; t < BN; ++t) mx = fmaxf(mx, sv[t]);
      const float m_use = mx == -INFINITY ? 0.f : mx;
      const float alpha = exp2f(m_run - m_use);
      float psum = 0.f;
      // Wait for P_{j-1} V_{j-1} before overwriting P and touching O.
      if (j > 0) {
        if (!mbar_wait(smem_u32(pv_done), (j - 1) & 1, abort_flag, &g_flash_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_PVDONE)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
#pragma unroll
      for (int c = 0; c < BN / 8; ++c) {
        float p[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          p[t] = exp2f(sv[c * 8 + t] - m_use);
          psum += p[t];
        }
        uint4 pk;
        pk.x = Pack2<T>::pack(p[0], p[1]);
        pk.y = Pack2<T>::pack(p[2], p[3]);
        pk.z = Pack2<T>::pack(p[4], p[5]);
        pk.w = Pack2<T>::pack(p[6], p[7]);
        const int half = c >> 3;  // 64-key chunk
        const int piece = c & 7;  // 16-byte piece within the 128-byte row
        *reinterpret_cast<uint4 *>(prow + half * (BM * 128) + ((piece ^ (row & 7)) << 4)) = pk;
      }
      l_run = l_run * alpha + psum;
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        // O row *= alpha, OC columns at a time (OC = 16 for D = 16, else 32).
#pragma unroll 1
        for (int c = 0; c < D; c += OC) {
          uint32_t r[OC];
          tmem_ld_cols(tmem_base + lane_off + O_COL + c, r);
#pragma unroll
          for (int t = 0; t < OC; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * alpha);
          tmem_st_cols(tmem_base + lane_off + O_COL + c, r);
        }
      }
      m_run = mx;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(smem_u32(p_ready));
    }
    // ---- epilogue: O / l -> global ----
    if (ok && n_kv > 0 &&
        mbar_wait(smem_u32(pv_done), (n_kv - 1) & 1, abort_flag, &g_flash_status,
                  TLLM_DEV_WAIT_TIMEOUT + SITE_PVDONE)) {
      tc_fence_after();
      const float inv_l = 1.0f / l_run;
      T *orow = static_cast<T *>(a.o) + b * a.so0 + h * a.so1 + static_cast<int64_t>(qg) * a.so2;
#pragma unroll 1
      for (int c = 0; c < D; c += OC) {
        uint32_t r[OC];
        tmem_ld_cols(tmem_base + lane_off + O_COL + c, r);
        if (qg < a.Sq) {
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
            for (int t = 0; t < OC; ++t) orow[(c + t) * a.so3] = from_f32<T>(__uint_as_float(r[t]) * inv_l);
          }
        }
      }
    } else if (n_kv == 0 && qg < a.Sq) {
      // No keys: softmax over an empty set is 0/0, as in the reference.
      T *orow = static_cast<T *>(a.o) + b * a.so0 + h * a.so1 + static_cast<int64_t>(qg) * a.so2;
      for (int c = 0; c < D; ++c) orow[c * a.so3] = from_f32<T>(NAN);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// =======================================================================================
// Ping-pong kernel: one CTA owns two adjacent 128-row query tiles X = 0 (rows [256t, +128))
// and X = 1 (the next 128 rows) of one (b, h), sharing every K/V tile.
//   warp 0        TMA producer (both Q tiles once, K_j and V_j through 2-slot rings)
//   warp 1        TMEM allocation + UMMA issue (warps 2-3 only hand their registers over)
//   warps 4-7     softmax for tile 0, warps 8-11 softmax for tile 1 (one query row each; a
//                 warp reads TMEM lanes 32*(warp % 4) .. +31, so each group covers 128 rows)
// TMEM (512 columns): S_X at [128X, 128X+128), O_X at [256+128X, 256+128X+D). After the
// softmax of tile X has read S_X(j) it overwrites S_X's first 64 columns with P_X(j) (fp16/
// bf16 pairs), and O_X += P_X V_j is issued with A read from TMEM. Per tile the MMAs run
// QK(j) -> PV(j) -> QK(j+1) in issue order, so S/P reuse needs no extra barrier, while the
// tensor core alternates between the two tiles: the softmax of one tile overlaps the MMAs
// of the other. O is rescaled lazily: the running max used for the exponentials only moves
// when a row's max grows by more than kLazyRescaleLog2 (so P stays below 2^8), which makes
// in-TMEM rescaling rare after the first key tiles.
// =======================================================================================
constexpr int kPPThreads = 384;
constexpr int kPPSoftmaxWarp0 = 4;
// Register hand-off (setmaxnreg): warps 0-3 (TMA, UMMA, two spare) keep 88, enough for the
// fully unrolled UMMA issue loops of the work-stealing kernel without spills; the two softmax
// warpgroups get 208; 88 * 128 + 208 * 256 = 168 * 384, the launch budget.
constexpr int kPPRegsLaunch = 168;
constexpr int kPPRegsLow = 88;
constexpr int kPPRegsHigh = 208;
static_assert(kPPRegsLow * 128 + kPPRegsHigh * 256 <= kPPRegsLaunch * kPPThreads,
              "setmaxnreg split exceeds the launch register budget");
constexpr float kLazyRescaleLog2 = 8.0f;
constexpr int kGroupHeads = 8;


// Shared memory of the two-tile kernel for head dim D and EB-byte inputs. A Q or K tile is
// 128 rows of D * EB bytes in 128-byte-swizzled spans of SWB bytes; with 16-bit inputs a V
// tile has the same shape, with e4m3 inputs it is V transposed (D rows of 128 keys, 128 B).
// kSP (P through shared memory): each query tile also has a P tile (128 rows of 128 keys, in
// the K-major layout of a 128-wide Q tile), and K and V tiles share one ring of NS slots,
// filled and consumed in the order K0, K1, V0, K2, V1, ... (three slots keep the 16-bit
// D = 128 kernel within 227 KB).
template <int D, int EB = 2, bool kSP = false>
struct GeoPP {
  static constexpr int ROWB = D * EB;
  static constexpr int SWB = ROWB >= 128 ? 128 : ROWB;
  static constexpr int CHUNKS = ROWB / SWB;
  static constexpr int CHUNK_ELEMS = SWB / EB;
  static constexpr int CHUNK_BYTES = BM * SWB;
  static constexpr int TILE_BYTES = BM * ROWB;
  static constexpr uint32_t LAYOUT = SWB == 128 ? 2u : (SWB == 64 ? 4u : 6u);
  static_assert(EB == 2 || (D * BN == TILE_BYTES && (D == 64 || D == 128)),
                "e4m3 tiles: head dim 64 or 128");
  static constexpr int NS = (EB == 2 && D == 128) ? 3 : 4;
  static constexpr int Q_OFF = 0;                       // two Q tiles
  static constexpr int K_OFF = Q_OFF + 2 * TILE_BYTES;  // two K slots, or the kSP ring
  static constexpr int V_OFF = K_OFF + 2 * TILE_BYTES;  // two V slots (not kSP)
  static constexpr int P_TILE_BYTES = BM * BN * EB;
  static constexpr int P_OFF = kSP ? K_OFF + NS * TILE_BYTES : V_OFF + 2 * TILE_BYTES;
  static constexpr int BAR_OFF = P_OFF + (kSP ? 2 * P_TILE_BYTES : 0);
  static constexpr int SMEM_BYTES = BAR_OFF + 256 + 1024;
  static_assert(SMEM_BYTES <= 232448, "two-tile kernel: shared memory above the 227 KB limit");
};

enum : int { SITE_PFULL = 9, SITE_ODONE = 10, SITE_QEMPTY = 11, SITE_CLC = 12, SITE_SFREE = 13 };

// One work item of the two-tile kernel: query rows [q0, q0 + 2*BM) of head (b, h) and the
// number of key tiles each of its two query tiles visits.
struct PPItem {
  int b, h, q0;
  int nkv[2];
  int n_kv;
  int Sq, Sk;      // this sequence's lengths
  int qrow, krow;  // first row of the sequence in q/o and in k/v
  int bc, hk;      // batch coordinate of the tensor maps, key/value head
};

// Items are numbered in groups of consecutive (b, h) heads: a.n_small groups of a.group
// heads, then groups of a.group + 1 heads (the last groups are the largest). Within a group
// the heaviest causal pairs of every head come first, then the next heaviest, and so on.
// Dynamic scheduling in that order ends each group, and the grid, with the lightest items (a
// short tail), while the CTAs running at the same time read the K/V of only a few heads
// (they stay in L2).
template <bool kVarlen>
__device__ __forceinline__ PPItem pp_item(const Args &a, int item) {
  PPItem w;
  const int n_pairs = (a.n_qtiles + 1) / 2;
  const int small_items = a.n_small * a.group * n_pairs;
  int heads = a.group, bh0 = 0, r = item;
  if (item < small_items) {
    const int grp = item / (heads * n_pairs);
    r = item - grp * heads * n_pairs;
    bh0 = grp * heads;
  } else {
    heads = a.group + 1;
    const int grp = (item - small_items) / (heads * n_pairs);
    r = item - small_items - grp * heads * n_pairs;
    bh0 = a.n_small * a.group + grp * heads;
  }
  const int bh = bh0 + r % heads;
  w.b = bh / a.H;
  w.h = bh % a.H;
  w.q0 = (n_pairs - 1 - r / heads) * 2 * BM;
  if constexpr (kVarlen) {
    // Clamped to the tensors, so inconsistent offsets cannot move a store out of o.
    w.qrow = min(max(__ldg(a.cu_q + w.b), 0), a.total_q);
    w.krow = min(max(__ldg(a.cu_k + w.b), 0), a.total_k);
    w.Sq = min(max(__ldg(a.cu_q + w.b + 1), w.qrow), a.total_q) - w.qrow;
    w.Sk = min(max(__ldg(a.cu_k + w.b + 1), w.krow), a.total_k) - w.krow;
    w.bc = 0;
    w.hk = w.h / a.G;
  } else {
    w.Sq = a.Sq;
    w.Sk = a.Sk;
    w.qrow = 0;
    w.krow = 0;
    w.bc = w.b;
    w.hk = w.h;
  }
  const int kv_tiles_all = (w.Sk + BN - 1) / BN;
#pragma unroll
  for (int X = 0; X < 2; ++X) {
    const int qx0 = w.q0 + X * BM;
    int n = qx0 < w.Sq ? kv_tiles_all : 0;
    if (a.causal && n > 0) n = min(n, (min(qx0 + BM, w.Sq) - 1) / BN + 1);
    w.nkv[X] = n;
  }
  w.n_kv = max(w.nkv[0], w.nkv[1]);
  return w;
}

// Readers of each work-stealing response: the UMMA lane and one lane per softmax warp.
constexpr int kClcReaders = 1 + 8;

// K-major operand (Q or K) of geometry G: step k of the reduction (32 bytes: 16 elements of
// 16 bits or 32 of 8 bits).
template <class G>
__device__ __forceinline__ uint64_t kmajor_desc_g(uint32_t base, int k) {
  const int byte = k * 32;
  const uint32_t addr = base + (byte / G::SWB) * G::CHUNK_BYTES + (byte % G::SWB);
  return make_sdesc(addr, 16, 8 * G::SWB, G::LAYOUT);
}

__device__ __forceinline__ void umma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 16 bytes to shared memory.
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

// kind::f8f6f4 instruction descriptor: fp32 accumulator, A and B e4m3 (format 0), K-major.
constexpr uint32_t idesc_e4m3(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Four floats to e4m3 (round to nearest even, saturating), the first in the lowest byte.
__device__ __forceinline__ uint32_t pack4_e4m3(float p0, float p1, float p2, float p3) {
  uint32_t r;
  asm("{\n\t.reg .b16 lo, hi;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 lo, %2, %1;\n\t"
      "cvt.rn.satfinite.e4m3x2.f32 hi, %4, %3;\n\t"
      "mov.b32 %0, {lo, hi};\n\t}"
      : "=r"(r)
      : "f"(p0), "f"(p1), "f"(p2), "f"(p3));
  return r;
}

// kSteal: the CTA keeps its TMEM, barriers and descriptors and moves on to further items. While
// an item's last key/value tiles are in flight, the producer cancels the launch of the next CTA
// that has not started (cluster launch control) and the CTA takes over that CTA's item, so
// items still run in launch order, each on the first SM to free up, without a CTA launch and
// set-up between them; the next item's Q tiles, first key tiles and first S overlap the
// current item's epilogue.
// TI: the input element type (T, or __nv_fp8_e4m3 with T the output type). With e4m3 inputs
// tm_v maps V transposed ([.., D, Sk], keys contiguous), so that both UMMA operands of P V are
// K-major, and P goes through shared memory as e4m3 (16 KB per query tile): the softmax frees
// S_X as soon as it has loaded it, so QK_X(j+1) runs on the tensor core while P_X(j) is being
// computed, instead of after PV_X(j).
template <typename T, typename TI, int D, bool kSteal, bool kVarlen, bool kSP>
__global__ void __launch_bounds__(kPPThreads, 1)
    flash_pp_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const Args a) {
  constexpr bool kF8 = std::is_same<TI, __nv_fp8_e4m3>::value;
  static_assert(!kF8 || (!kVarlen && kSP), "e4m3 inputs: dense batches, P in shared memory");
  constexpr int EB = kF8 ? 1 : 2;
  using G = GeoPP<D, EB, kSP>;
  using PG = GeoPP<BN, EB>;  // a P tile has the layout of a Q tile with 128 columns
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr int OC = D < 32 ? D : 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + G::BAR_OFF);
  uint64_t *q_full = bars + 0;
  uint64_t *k_full = bars + 1;     // [2]
  uint64_t *k_empty = bars + 3;    // [2]
  uint64_t *v_full = bars + 5;     // [2]
  uint64_t *v_empty = bars + 7;    // [2]
  uint64_t *s_full = bars + 9;     // [2] per tile
  uint64_t *p_full = bars + 11;    // [2] per tile
  uint64_t *o_done = bars + 13;    // [2] per tile
  uint64_t *q_empty = bars + 15;
  uint64_t *clc_full = bars + 16;  // [2] per response slot
  uint64_t *clc_empty = bars + 18; // [2] per response slot
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 20);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  const uint32_t clc_resp = smem_u32(bars + 22);  // two 16-byte responses
  // kSP: S_X has been read into registers (the next QK_X may overwrite it); o_done then
  // completes after every PV_X (P_X in shared memory and O_X may be reused). The K/V ring uses
  // k_full..v_empty as ring_full[4] and ring_empty[4].
  uint64_t *s_free = bars + 26;    // [2] per tile
  uint64_t *ring_full = bars + 1;  // [NS]
  uint64_t *ring_empty = bars + 5; // [NS]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(q_full), 1);
    mbar_init(smem_u32(q_empty), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&k_empty[s]), 1);
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 1);
      mbar_init(smem_u32(&s_full[s]), 1);
      mbar_init(smem_u32(&p_full[s]), kSoftmaxThreads);
      mbar_init(smem_u32(&o_done[s]), 1);
      mbar_init(smem_u32(&clc_full[s]), 1);
      mbar_init(smem_u32(&clc_empty[s]), kClcReaders);
      mbar_init(smem_u32(&s_free[s]), kSoftmaxThreads);
    }
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
  // Waits for the response to the request made during the it-th item and returns the next
  // item (-1: the grid is exhausted; -2: a wait gave up). With warp_vote the whole warp calls
  // it and gets the same answer.
  auto read_next = [&](int it, bool warp_vote) -> int {
    const int slot = it & 1;
    bool got = mbar_wait(smem_u32(&clc_full[slot]), (it >> 1) & 1, abort_flag, &g_flash_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_CLC);
    if (warp_vote) got = __all_sync(0xffffffffu, got);
    if (!got) return -2;
    const int nxt = clc_cancelled_ctaid_x(clc_resp + 16 * slot);
    // The slot is rewritten by the async proxy two items later.
    fence_proxy_async_smem();
    return nxt;
  };
  if (warp < kPPSoftmaxWarp0) {
  regs_dec<kPPRegsLow>();
  if (warp == 0 && kSP) {
    // ------------------------ TMA producer, one K/V ring ------------------------
    if (lane == 0) {
      int item = static_cast<int>(blockIdx.x);
      int gr = 0;  // ring tiles loaded so far
      int nq = 0;  // Q loads so far
      bool ok = true;
      // Loads key tile j (is_v false) or value tile j into the next ring slot.
      auto load_kv = [&](const PPItem &w, bool is_v, int j) -> bool {
        const int r = gr % G::NS;
        if (!mbar_wait(smem_u32(&ring_empty[r]), ((gr / G::NS) & 1) ^ 1, abort_flag,
                       &g_flash_status, TLLM_DEV_WAIT_TIMEOUT + (is_v ? SITE_VEMPTY : SITE_KEMPTY)))
          return false;
        const uint32_t fb = smem_u32(&ring_full[r]);
        const uint32_t dst = sK + r * G::TILE_BYTES;
        mbar_arrive_expect_tx(fb, G::TILE_BYTES);
        if (kF8 && is_v) {
          // One box of V transposed: 128 keys (x, a multiple of 128) of all D rows.
          tma_load_4d(dst, &tm_v, fb, w.krow + j * BN, 0, w.hk, w.bc);
        } else {
#pragma unroll
          for (int c = 0; c < G::CHUNKS; ++c)
            tma_load_4d(dst + c * G::CHUNK_BYTES, is_v ? &tm_v : &tm_k, fb, c * G::CHUNK_ELEMS,
                        w.krow + j * BN, w.hk, w.bc);
        }
        ++gr;
        return true;
      };
      for (int it = 0; ok && item >= 0; ++it) {
        const PPItem w = pp_item<kVarlen>(a, item);
        if (w.n_kv > 0) {
          // The previous item's last QK has read its Q tiles.
          if (nq > 0 && !mbar_wait(smem_u32(q_empty), (nq - 1) & 1, abort_flag, &g_flash_status,
                                   TLLM_DEV_WAIT_TIMEOUT + SITE_QEMPTY))
            break;
          const uint32_t qb = smem_u32(q_full);
          mbar_arrive_expect_tx(qb, G::TILE_BYTES * ((w.nkv[0] > 0) + (w.nkv[1] > 0)));
#pragma unroll
          for (int X = 0; X < 2; ++X) {
            if (w.nkv[X] == 0) continue;
#pragma unroll
            for (int c = 0; c < G::CHUNKS; ++c)
              tma_load_4d(sQ + X * G::TILE_BYTES + c * G::CHUNK_BYTES, &tm_q, qb,
                          c * G::CHUNK_ELEMS, w.qrow + w.q0 + X * BM, w.h, w.bc);
          }
          ++nq;
          // The order the UMMA warp consumes them in: K0, then K(j+1) before V(j).
          ok = load_kv(w, false, 0);
          for (int j = 0; ok && j < w.n_kv; ++j) {
            if (j + 1 < w.n_kv) ok = load_kv(w, false, j + 1);
            if (ok) ok = load_kv(w, true, j);
          }
        }
        if (!ok || !kSteal) break;
        // Claim the next item while this one's last tiles are in flight.
        const int slot = it & 1;
        if (it >= 2 && !mbar_wait(smem_u32(&clc_empty[slot]), ((it >> 1) - 1) & 1, abort_flag,
                                  &g_flash_status, TLLM_DEV_WAIT_TIMEOUT + SITE_CLC))
          break;
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(smem_u32(&clc_full[slot]), 16);
        clc_try_cancel(clc_resp + 16 * slot, smem_u32(&clc_full[slot]));
        item = read_next(it, false);
      }
    }
  } else if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int item = static_cast<int>(blockIdx.x);
      int g = 0;   // key/value tiles loaded so far (ring position)
      int nq = 0;  // Q loads so far
      bool ok = true;
      for (int it = 0; ok && item >= 0; ++it) {
        const PPItem w = pp_item<kVarlen>(a, item);
        if (w.n_kv > 0) {
          // The previous item's last QK has read its Q tiles.
          if (nq > 0 && !mbar_wait(smem_u32(q_empty), (nq - 1) & 1, abort_flag, &g_flash_status,
                                   TLLM_DEV_WAIT_TIMEOUT + SITE_QEMPTY))
            break;
          const uint32_t qb = smem_u32(q_full);
          mbar_arrive_expect_tx(qb, G::TILE_BYTES * ((w.nkv[0] > 0) + (w.nkv[1] > 0)));
#pragma unroll
          for (int X = 0; X < 2; ++X) {
            if (w.nkv[X] == 0) continue;
#pragma unroll
            for (int c = 0; c < G::CHUNKS; ++c)
              tma_load_4d(sQ + X * G::TILE_BYTES + c * G::CHUNK_BYTES, &tm_q, qb,
                          c * G::CHUNK_ELEMS, w.qrow + w.q0 + X * BM, w.h, w.bc);
          }
          ++nq;
          for (int j = 0; j < w.n_kv; ++j, ++g) {
            const int s = g & 1;
            const uint32_t par = ((g >> 1) & 1) ^ 1;
            if (!mbar_wait(smem_u32(&k_empty[s]), par, abort_flag, &g_flash_status,
                           TLLM_DEV_WAIT_TIMEOUT + SITE_KEMPTY)) {
              ok = false;
              break;
            }
            const uint32_t kb = smem_u32(&k_full[s]);
            mbar_arrive_expect_tx(kb, G::TILE_BYTES);
#pragma unroll
            for (int c = 0; c < G::CHUNKS; ++c)
              tma_load_4d(sK + s * G::TILE_BYTES + c * G::CHUNK_BYTES, &tm_k, kb,
                          c * G::CHUNK_ELEMS, w.krow + j * BN, w.hk, w.bc);
            if (!mbar_wait(smem_u32(&v_empty[s]), par, abort_flag, &g_flash_status,
                           TLLM_DEV_WAIT_TIMEOUT + SITE_VEMPTY)) {
              ok = false;
              break;
            }
            const uint32_t vb = smem_u32(&v_full[s]);
            mbar_arrive_expect_tx(vb, G::TILE_BYTES);
#pragma unroll
            for (int c = 0; c < G::CHUNKS; ++c)
              tma_load_4d(sV + s * G::TILE_BYTES + c * G::CHUNK_BYTES, &tm_v, vb,
                          c * G::CHUNK_ELEMS, w.krow + j * BN, w.hk, w.bc);
          }
        }
        if (!ok || !kSteal) break;
        // Claim the next item while this one's last tiles are in flight.
        const int slot = it & 1;
        if (it >= 2 && !mbar_wait(smem_u32(&clc_empty[slot]), ((it >> 1) - 1) & 1, abort_flag,
                                  &g_flash_status, TLLM_DEV_WAIT_TIMEOUT + SITE_CLC))
          break;
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(smem_u32(&clc_full[slot]), 16);
        clc_try_cancel(clc_resp + 16 * slot, smem_u32(&clc_full[slot]));
        item = read_next(it, false);
      }
    }
  } else if (warp == 1 && kSP) {
    // ------------------------- UMMA issuer, P in shared memory ------------------
    // QK_X(j+1) is issued as soon as the softmax has read S_X(j) and runs while the softmax
    // computes P_X(j); PV_X(j) follows P_X(j). Ring tiles are consumed in load order.
    if (lane == 0) {
      const uint32_t idesc_qk = kF8 ? idesc_e4m3(BM, BN) : make_idesc_f16(BM, BN, kBF16, false, false);
      // 16-bit: B = V [keys, D] MN-major; e4m3: B = V transposed [D, keys] K-major.
      const uint32_t idesc_pv = kF8 ? idesc_e4m3(BM, D) : make_idesc_f16(BM, D, kBF16, false, true);
      const uint32_t sP = smem_u32(smem + G::P_OFF);
      uint32_t nqk[2] = {0u, 0u};  // QK_X issued
      uint32_t npf[2] = {0u, 0u};  // P_X tiles consumed
      int gc = 0;                  // ring tiles consumed
      auto ring_acquire = [&](int site, uint32_t &base) -> bool {
        const int r = gc % G::NS;
        if (!mbar_wait(smem_u32(&ring_full[r]), (gc / G::NS) & 1, abort_flag, &g_flash_status,
                       TLLM_DEV_WAIT_TIMEOUT + site))
          return false;
        tc_fence_after();
        base = sK + r * G::TILE_BYTES;
        return true;
      };
      // The slot is free once the MMAs issued so far (those reading it) have completed.
      auto ring_release = [&]() {
        umma_commit(smem_u32(&ring_empty[gc % G::NS]));
        ++gc;
      };
      // Issues QK_X from the key tile at kbase once the softmax has read the previous S_X.
      auto issue_qk = [&](int X, uint32_t kbase) -> bool {
        if (nqk[X] > 0 && !mbar_wait(smem_u32(&s_free[X]), (nqk[X] - 1) & 1, abort_flag,
                                     &g_flash_status, TLLM_DEV_WAIT_TIMEOUT + SITE_SFREE))
          return false;
        tc_fence_after();
        const uint32_t qbase = sQ + X * G::TILE_BYTES;
#pragma unroll
        for (int k = 0; k < G::ROWB / 32; ++k) {
          if constexpr (kF8)
            umma_f8_ss(tmem_base + X * BN, kmajor_desc_g<G>(qbase, k), kmajor_desc_g<G>(kbase, k),
                       idesc_qk, k != 0 ? 1u : 0u);
          else
            umma_f16_ss(tmem_base + X * BN, kmajor_desc_g<G>(qbase, k), kmajor_desc_g<G>(kbase, k),
                        idesc_qk, k != 0 ? 1u : 0u);
        }
        umma_commit(smem_u32(&s_full[X]));
        ++nqk[X];
        return true;
      };
      int item = static_cast<int>(blockIdx.x);
      int nq = 0;
      bool ok = true;
      for (int it = 0; ok && item >= 0; ++it) {
        const PPItem w = pp_item<kVarlen>(a, item);
        if (w.n_kv > 0) {
          ok = mbar_wait(smem_u32(q_full), nq & 1, abort_flag, &g_flash_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_Q);
          ++nq;
          uint32_t kbase = 0, vbase = 0;
          if (!ok || !(ok = ring_acquire(SITE_KFULL, kbase))) break;
#pragma unroll
          for (int X = 0; X < 2; ++X)
            if (ok && w.nkv[X] > 0) ok = issue_qk(X, kbase);
          if (!ok) break;
          ring_release();
          if (w.n_kv == 1) umma_commit(smem_u32(q_empty));
          for (int j = 0; j < w.n_kv && ok; ++j) {
            if (j + 1 < w.n_kv) {
              if (!(ok = ring_acquire(SITE_KFULL, kbase))) break;
#pragma unroll
              for (int X = 0; X < 2; ++X)
                if (ok && j + 1 < w.nkv[X]) ok = issue_qk(X, kbase);
              if (!ok) break;
              ring_release();
              // The item's last QK has been issued: its Q tiles are free once it completes.
              if (j == w.n_kv - 2) umma_commit(smem_u32(q_empty));
            }
            if (!(ok = ring_acquire(SITE_VFULL, vbase))) break;
#pragma unroll
            for (int X = 0; X < 2; ++X) {
              if (j >= w.nkv[X]) continue;
              if (!mbar_wait(smem_u32(&p_full[X]), npf[X] & 1, abort_flag, &g_flash_status,
                             TLLM_DEV_WAIT_TIMEOUT + SITE_PFULL)) {
                ok = false;
                break;
              }
              ++npf[X];
              tc_fence_after();
              const uint32_t pbase = sP + X * G::P_TILE_BYTES;
              const uint32_t o_tmem = tmem_base + O_COL + X * BN;
              if constexpr (kF8) {
                // A = P_X, B = V transposed (D rows of 128 keys); 32 keys a step.
#pragma unroll
                for (int k = 0; k < BN / 32; ++k)
                  umma_f8_ss(o_tmem, kmajor_desc_g<PG>(pbase, k),
                             make_sdesc(vbase + k * 32, 16, 1024, 2u), idesc_pv, (j | k) != 0 ? 1u : 0u);
              } else {
                // A = P_X, B = V (keys x D, MN-major); 16 keys a step.
#pragma unroll
                for (int k = 0; k < BN / 16; ++k)
                  umma_f16_ss(o_tmem, kmajor_desc_g<PG>(pbase, k),
                              make_sdesc(vbase + k * 16 * G::SWB, G::CHUNK_BYTES, 8 * G::SWB, G::LAYOUT),
                              idesc_pv, (j | k) != 0 ? 1u : 0u);
              }
              umma_commit(smem_u32(&o_done[X]));
            }
            if (!ok) break;
            ring_release();
          }
        }
        if (!ok || !kSteal) break;
        item = read_next(it, false);
        if (item >= -1) mbar_arrive(smem_u32(&clc_empty[it & 1]));
      }
    }
  } else if (warp == 1) {
    // ------------------------------ UMMA issuer -------------------------------
    if (lane == 0) {
      const uint32_t idesc_qk = make_idesc_f16(BM, BN, kBF16, false, false);
      const uint32_t idesc_pv = make_idesc_f16(BM, D, kBF16, false, true);
      auto issue_qk = [&](int X, int kslot) {
        const uint32_t kbase = sK + kslot * G::TILE_BYTES;
        const uint32_t qbase = sQ + X * G::TILE_BYTES;
#pragma unroll
        for (int k = 0; k < D / 16; ++k)
          umma_f16_ss(tmem_base + X * BN, kmajor_desc<D>(qbase, k), kmajor_desc<D>(kbase, k),
                      idesc_qk, k != 0 ? 1u : 0u);
        umma_commit(smem_u32(&s_full[X]));
      };
      int item = static_cast<int>(blockIdx.x);
      int g = 0, nq = 0;
      uint32_t npf[2] = {0u, 0u};  // P tiles consumed per query tile
      bool ok = true;
      for (int it = 0; ok && item >= 0; ++it) {
        const PPItem w = pp_item<kVarlen>(a, item);
        if (w.n_kv > 0) {
          ok = mbar_wait(smem_u32(q_full), nq & 1, abort_flag, &g_flash_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_Q) &&
               mbar_wait(smem_u32(&k_full[g & 1]), (g >> 1) & 1, abort_flag, &g_flash_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_KFULL);
          ++nq;
          if (!ok) break;
          // S_X of the previous item was last read as P by its final PV, issued before this
          // QK; its O_X was read out by the epilogue before the softmax signalled this item's
          // first P, which the first PV below waits for.
          tc_fence_after();
#pragma unroll
          for (int X = 0; X < 2; ++X)
            if (w.nkv[X] > 0) issue_qk(X, g & 1);
          umma_commit(smem_u32(&k_empty[g & 1]));
          if (w.n_kv == 1) umma_commit(smem_u32(q_empty));
          for (int j = 0; j < w.n_kv && ok; ++j) {
            const int gj = g + j;
            const int s = gj & 1;
            if (!mbar_wait(smem_u32(&v_full[s]), (gj >> 1) & 1, abort_flag, &g_flash_status,
                           TLLM_DEV_WAIT_TIMEOUT + SITE_VFULL)) {
              ok = false;
              break;
            }
            const uint32_t vbase = sV + s * G::TILE_BYTES;
            bool next_k_ready = false;
#pragma unroll
            for (int X = 0; X < 2; ++X) {
              if (j >= w.nkv[X]) continue;
              if (!mbar_wait(smem_u32(&p_full[X]), npf[X] & 1, abort_flag, &g_flash_status,
                             TLLM_DEV_WAIT_TIMEOUT + SITE_PFULL)) {
                ok = false;
                break;
              }
              ++npf[X];
              tc_fence_after();
              const uint32_t p_tmem = tmem_base + X * BN;
              const uint32_t o_tmem = tmem_base + O_COL + X * BN;
#pragma unroll
              for (int k = 0; k < BN / 16; ++k) {
                const uint64_t bdesc =
                    make_sdesc(vbase + k * 16 * G::SWB, G::CHUNK_BYTES, 8 * G::SWB, G::LAYOUT);
                umma_f16_ts(o_tmem, p_tmem + k * 8, bdesc, idesc_pv, (j | k) != 0 ? 1u : 0u);
              }
              if (j == w.nkv[X] - 1) {
                umma_commit(smem_u32(&o_done[X]));
              } else {
                if (!next_k_ready) {
                  if (!mbar_wait(smem_u32(&k_full[(gj + 1) & 1]), ((gj + 1) >> 1) & 1, abort_flag,
                                 &g_flash_status, TLLM_DEV_WAIT_TIMEOUT + SITE_KFULL)) {
                    ok = false;
                    break;
                  }
                  tc_fence_after();
                  next_k_ready = true;
                }
                issue_qk(X, (gj + 1) & 1);
              }
            }
            if (!ok) break;
            umma_commit(smem_u32(&v_empty[s]));
            if (next_k_ready) umma_commit(smem_u32(&k_empty[(gj + 1) & 1]));
            // The item's last QK has been issued: its Q tiles are free once it completes.
            if (j == w.n_kv - 2) umma_commit(smem_u32(q_empty));
          }
          g += w.n_kv;
        }
        if (!ok || !kSteal) break;
        item = read_next(it, false);
        if (item >= -1) mbar_arrive(smem_u32(&clc_empty[it & 1]));
      }
    }
  }
  } else {
    regs_inc<kPPRegsHigh>();
    // ------------------------------ softmax / epilogue ------------------------
    const int X = (warp - kPPSoftmaxWarp0) >> 2;
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t s_tm = tmem_base + lane_off + X * BN;
    const uint32_t o_tm = tmem_base + lane_off + O_COL + X * BN;
    int item = static_cast<int>(blockIdx.x);
    uint32_t ns = 0;   // S tiles consumed
    uint32_t nod = 0;  // O tiles finished
    bool ok = true;
    for (int it = 0; ok && item >= 0; ++it) {
      const PPItem w = pp_item<kVarlen>(a, item);
      const int qx0 = w.q0 + X * BM;
      const int qg = qx0 + row;
      const int nk = w.nkv[X];
      float m_use = -INFINITY;  // max the exponentials are taken against (lazily updated)
      float l_run = 0.f;
      for (int j = 0; j < nk; ++j, ++ns) {
        // Waits are voted warp-wide so that a warp leaves together even when a wait gives up.
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&s_full[X]), ns & 1, abort_flag,
                                               &g_flash_status, TLLM_DEV_WAIT_TIMEOUT + SITE_SFULL))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int k0 = j * BN;
        const bool need_mask = (k0 + BN > w.Sk) || (a.causal && k0 + BN - 1 > qx0);
        // The whole S row in one TMEM round trip (four 32-column loads, one wait).
        uint32_t sr[BN];
        tmem_ld4x32(s_tm, sr);
        if constexpr (kSP) {
          // S_X(j) is in registers: QK_X(j+1) may overwrite it while P_X(j) is computed.
          tc_fence_before();
          mbar_arrive(smem_u32(&s_free[X]));
        }
        if (need_mask) {
#pragma unroll
          for (int t = 0; t < BN; ++t) {
            const int kg = k0 + t;
            if (kg >= w.Sk || (a.causal && kg > qg)) sr[t] = __float_as_uint(-INFINITY);
          }
        }
        // Row max on the raw scores (the scale is positive): an 8-way tree of 3-input maxima.
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
        float alpha = 1.0f;
        bool rescale = false;
        if (m_use == -INFINITY) {
          m_use = mx;  // first tile: O not written yet, nothing to rescale
        } else if (mx > m_use + kLazyRescaleLog2) {
          alpha = ex2_approx(m_use - mx);
          m_use = mx;
          rescale = true;
        }
        const float neg_m = m_use == -INFINITY ? 0.f : -m_use;
        const uint64_t scale2 = f2_pack(a.scale_log2, a.scale_log2);
        const uint64_t negm2 = f2_pack(neg_m, neg_m);
        uint64_t ps2[4] = {0ull, 0ull, 0ull, 0ull};
        if constexpr (kSP) {
          // P = 2^(s * scale - m) in the input precision (e4m3: four keys a word; 16-bit: two),
          // kept in registers until PV_X(j-1) has finished with P_X's shared-memory tile and
          // with O_X. Exponent arguments and the row sum use packed fp32 pairs.
          constexpr int PW = BN * EB / 4;  // 32-bit words of a P row
          uint32_t pk[PW];
          if constexpr (kF8) {
#pragma unroll
            for (int t = 0; t < BN; t += 4) {
              float pv[4];
#pragma unroll
              for (int u = 0; u < 4; u += 2) {
                const uint64_t x2 = f2_fma(
                    f2_pack(__uint_as_float(sr[t + u]), __uint_as_float(sr[t + u + 1])), scale2, negm2);
                float x0, x1;
                f2_unpack(x2, x0, x1);
                pv[u] = ex2_approx(x0);
                pv[u + 1] = ex2_approx(x1);
                ps2[((t + u) >> 1) & 3] = f2_add(ps2[((t + u) >> 1) & 3], f2_pack(pv[u], pv[u + 1]));
              }
              pk[t >> 2] = pack4_e4m3(pv[0], pv[1], pv[2], pv[3]);
            }
          } else {
#pragma unroll
            for (int t = 0; t < BN; t += 2) {
              const uint64_t x2 = f2_fma(
                  f2_pack(__uint_as_float(sr[t]), __uint_as_float(sr[t + 1])), scale2, negm2);
              float x0, x1;
              f2_unpack(x2, x0, x1);
              const float p0 = ex2_approx(x0);
              const float p1 = ex2_approx(x1);
              ps2[(t >> 1) & 3] = f2_add(ps2[(t >> 1) & 3], f2_pack(p0, p1));
              pk[t >> 1] = Pack2<T>::pack(p0, p1);
            }
          }
          if (j > 0) {
            if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&o_done[X]), nod & 1, abort_flag,
                                                   &g_flash_status, TLLM_DEV_WAIT_TIMEOUT + SITE_ODONE))) {
              ok = false;
              break;
            }
            ++nod;
            tc_fence_after();
          }
          // Row `row` of P_X in the K-major 128-byte-swizzled layout: 16-byte unit u of a
          // 128-byte span at unit u ^ (row % 8) (eight consecutive rows fill all banks).
          const uint32_t prow = smem_u32(smem + G::P_OFF + X * G::P_TILE_BYTES) + row * 128;
#pragma unroll
          for (int u = 0; u < PW / 4; ++u)
            st_shared_v4(prow + (u >> 3) * PG::CHUNK_BYTES + (((u & 7) ^ (row & 7)) << 4),
                         pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
        } else {
          // P = 2^(s * scale - m), written over S's first 64 columns in packed pairs (S's
          // values are all in registers by now). Exponent arguments and the row sum use packed
          // fp32 pairs (one instruction per pair).
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
            // The first half's store is not waited for on its own: the second half's store
            // waits for both (+1 % in interleaved runs, the same output).
            if (hlf == 0)
              tmem_st32_nowait(s_tm, pk);
            else
              tmem_st32(s_tm + 32 * hlf, pk);
          }
        }
        float psa, psb, psc, psd, pse, psf, psg, psh;
        f2_unpack(ps2[0], psa, psb);
        f2_unpack(ps2[1], psc, psd);
        f2_unpack(ps2[2], pse, psf);
        f2_unpack(ps2[3], psg, psh);
        const float psum = ((psa + psb) + (psc + psd)) + ((pse + psf) + (psg + psh));
        l_run = l_run * alpha + psum;
        // O_X is stable here: with P in TMEM, PV_X(j-1) was issued before QK_X(j), whose
        // completion s_full signalled; with P in shared memory it was waited for above.
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
        // P_X's shared-memory writes become visible to the tensor core (async proxy).
        if constexpr (kSP) fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(smem_u32(&p_full[X]));
      }
      if (!ok) break;
      // ---- epilogue: O / l -> global ----
      if (nk > 0) {
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&o_done[X]), nod & 1, abort_flag,
                                               &g_flash_status, TLLM_DEV_WAIT_TIMEOUT + SITE_ODONE)))
          break;
        ++nod;
        tc_fence_after();
        float inv_l = 1.0f / l_run;
        if constexpr (kF8) inv_l *= a.out_scale;
        if (!kVarlen && a.lse != nullptr && qg < w.Sq)
          a.lse[(static_cast<int64_t>(w.b) * a.H + w.h) * a.Sq + qg] = m_use + log2f(l_run);
        T *orow = static_cast<T *>(a.o) + w.b * a.so0 + w.h * a.so1 +
                  static_cast<int64_t>(w.qrow + qg) * a.so2;
#pragma unroll 1
        for (int c = 0; c < D; c += OC) {
          uint32_t r[OC];
          tmem_ld_cols(o_tm + c, r);
          if (qg < w.Sq) {
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
        // The O_X reads above complete (tcgen05.wait::ld) before this warp's next P store,
        // which the next item's first PV_X waits for.
      } else if (qx0 < w.Sq && qg < w.Sq) {
        // No keys at all (Sk == 0): 0/0, as in the reference.
        T *orow = static_cast<T *>(a.o) + w.b * a.so0 + w.h * a.so1 +
                  static_cast<int64_t>(w.qrow + qg) * a.so2;
        for (int c = 0; c < D; ++c) orow[c * a.so3] = from_f32<T>(NAN);
      }
      if (!kSteal) break;
      item = read_next(it, true);
      __syncwarp();
      if (lane == 0 && item >= -1) mbar_arrive(smem_u32(&clc_empty[it & 1]));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Kernel variants (tllm_flash_attn_fwd_variant): the two-tile kernel with work stealing is
// the default; the single-tile kernel and the two-tile kernel with one item per CTA are kept
// as cross-checks.
constexpr int kVariantPingPong = 0;
constexpr int kVariantSingleTile = 1;
constexpr int kVariantPingPongOneItem = 2;
constexpr int kVariantSmemP = 3;  // P through shared memory, one K/V ring

// Packed variable-length batch: sequence b's rows are [cu_q[b], cu_q[b+1]) of q/o (total_q
// rows) and [cu_k[b], cu_k[b+1]) of k/v (total_k rows, Hkv heads).
struct VarlenDesc {
  const int *cu_q;
  const int *cu_k;
  int64_t total_q, total_k, Hkv;
};

// Scheduling groups of the two-tile kernel: kGroupHeads heads per group, or all heads in one
// group when a causal grid is only a few waves long (its tail then comes from the lightest
// items of all heads); at most 64 MiB of K and V per group; sizes as even as possible.
void set_groups(Args &a, int64_t B, int64_t H, int64_t Sk, int64_t row_bytes, int causal) {
  const int64_t bh = B * H;
  const int64_t n_pairs = (a.n_qtiles + 1) / 2;
  const int64_t sms = sm_count() > 0 ? sm_count() : 148;
  const int64_t kv_head_bytes = 2 * (Sk > 0 ? Sk : 1) * row_bytes;
  int64_t target = (causal && bh * n_pairs <= 4 * sms) ? bh : kGroupHeads;
  target = std::min<int64_t>(target, std::max<int64_t>(1, (64ll << 20) / kv_head_bytes));
  const int64_t n_groups = (bh + target - 1) / target;
  a.group = static_cast<int>(bh / n_groups);
  a.n_small = static_cast<int>(n_groups - bh % n_groups);
}

// Launches a two-tile kernel instance after checking that the register split fits.
template <class GP, typename K>
int launch_pp(K kern, unsigned grid, const CUtensorMap &mq, const CUtensorMap &mk,
              const CUtensorMap &mv, const Args &a, cudaStream_t st) {
  KernelLaunchInfo info;
  const int rc = prepare_kernel(reinterpret_cast<const void *>(kern), GP::SMEM_BYTES, kPPThreads, 1, &info);
  if (rc) return rc;
  // setmaxnreg.inc only completes if the launch holds the registers the split assumes.
  if (info.num_regs != kPPRegsLaunch)
    return fail(TLLM_ERR_CUDA, "flash_attention: kernel built with %d registers, %d expected",
                info.num_regs, kPPRegsLaunch);
  if (info.resident < 1)
    return fail(TLLM_ERR_CUDA, "flash_attention: the two-tile kernel cannot be resident on this device");
  kern<<<grid, kPPThreads, GP::SMEM_BYTES, st>>>(mq, mk, mv, a);
  return cuda_status(cudaGetLastError(), "flash pp launch");
}

template <typename T, int D>
int launch_d(const void *q, const void *k, const void *v, void *o, int64_t B, int64_t H,
             int64_t Sq, int64_t Sk, const int64_t *sq, const int64_t *sk, const int64_t *sv,
             const int64_t *so, float sm_scale, int causal, int variant, cudaStream_t st,
             const VarlenDesc *vl = nullptr, float *lse = nullptr) {
  using G = Geo<D>;
  const CUtensorMapDataType dt = std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUtensorMapSwizzle sw = G::SWB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : (G::SWB == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B);
  const uint32_t box[4] = {static_cast<uint32_t>(G::SWB / 2), static_cast<uint32_t>(BM), 1, 1};
  CUtensorMap mq, mk, mv;
  // Dense: 4-D maps {D, S, H, B}. Packed: {D, total rows, H, 1} (the strides arrays then hold
  // {unused, head, row, 1}).
  const int64_t q_rows = vl ? vl->total_q : Sq;
  const int64_t k_rows = vl ? vl->total_k : Sk;
  const int64_t kv_heads = vl ? vl->Hkv : H;
  const int64_t map_b = vl ? 1 : B;
  {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)q_rows, (uint64_t)H, (uint64_t)map_b};
    const uint64_t str[3] = {(uint64_t)sq[2] * 2, (uint64_t)sq[1] * 2, (uint64_t)sq[0] * 2};
    int rc = encode_tiled(&mq, dt, 4, const_cast<void *>(q), dims, str, box, sw);
    if (rc) return rc;
  }
  {
    // Sk == 0 launches no key loads; the map still needs a non-zero extent.
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)(k_rows > 0 ? k_rows : 1), (uint64_t)kv_heads,
                              (uint64_t)map_b};
    const uint64_t strk[3] = {(uint64_t)sk[2] * 2, (uint64_t)sk[1] * 2, (uint64_t)sk[0] * 2};
    int rc = encode_tiled(&mk, dt, 4, const_cast<void *>(k), dims, strk, box, sw);
    if (rc) return rc;
    const uint64_t strv[3] = {(uint64_t)sv[2] * 2, (uint64_t)sv[1] * 2, (uint64_t)sv[0] * 2};
    rc = encode_tiled(&mv, dt, 4, const_cast<void *>(v), dims, strv, box, sw);
    if (rc) return rc;
  }
  Args a;
  a.o = o;
  a.so0 = so[0];
  a.so1 = so[1];
  a.so2 = so[2];
  a.so3 = so[3];
  a.H = static_cast<int>(H);
  a.Sq = static_cast<int>(Sq);
  a.Sk = static_cast<int>(Sk);
  a.n_qtiles = static_cast<int>((Sq + BM - 1) / BM);
  a.scale_log2 = sm_scale * kLog2e;
  a.causal = causal ? 1 : 0;
  a.vec_store = (so[3] == 1 && so[0] % 8 == 0 && so[1] % 8 == 0 && so[2] % 8 == 0 && aligned16(o)) ? 1 : 0;
  a.lse = lse;
  a.cu_q = vl ? vl->cu_q : nullptr;
  a.cu_k = vl ? vl->cu_k : nullptr;
  a.G = vl ? static_cast<int>(H / vl->Hkv) : 1;
  a.total_q = vl ? static_cast<int>(vl->total_q) : 0;
  a.total_k = vl ? static_cast<int>(vl->total_k) : 0;
  a.out_scale = 1.0f;
  set_groups(a, B, H, Sk, D * 2, causal);
  if (variant == kVariantSingleTile && !vl) {
    auto kern = flash_fwd_kernel<T, D>;
    KernelLaunchInfo info;
    const int rc = prepare_kernel(reinterpret_cast<const void *>(kern), G::SMEM_BYTES, kThreads, 1, &info);
    if (rc) return rc;
    const unsigned grid = static_cast<unsigned>(B * H * a.n_qtiles);
    kern<<<grid, kThreads, G::SMEM_BYTES, st>>>(mq, mk, mv, a);
    return cuda_status(cudaGetLastError(), "flash launch");
  }
  const unsigned grid = static_cast<unsigned>(B * H * ((a.n_qtiles + 1) / 2));
  if (variant == kVariantSmemP && !vl)
    return launch_pp<GeoPP<D, 2, true>>(flash_pp_kernel<T, T, D, true, false, true>, grid, mq, mk,
                                        mv, a, st);
  using GP = GeoPP<D>;
  auto kern = vl ? flash_pp_kernel<T, T, D, true, true, false>
                : (variant == kVariantPingPongOneItem ? flash_pp_kernel<T, T, D, false, false, false>
                                                      : flash_pp_kernel<T, T, D, true, false, false>);
  return launch_pp<GP>(kern, grid, mq, mk, mv, a, st);
}

// e4m3 q, k [B, H, S, D] and V transposed vt [B, H, D, Sk] (keys contiguous); strides in
// elements (= bytes).
template <typename T, int D>
int launch_fp8(const void *q, const void *k, const void *vt, void *o, int64_t B, int64_t H,
               int64_t Sq, int64_t Sk, const int64_t *sq, const int64_t *sk, const int64_t *svt,
               const int64_t *so, float sm_scale, float scale_q, float scale_k, float scale_v,
               int causal, cudaStream_t st) {
  using GP = GeoPP<D, 1, true>;
  const CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_UINT8;
  const CUtensorMapSwizzle sw = GP::SWB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const uint32_t box[4] = {static_cast<uint32_t>(GP::SWB), static_cast<uint32_t>(BM), 1, 1};
  CUtensorMap mq, mk, mv;
  {
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)Sq, (uint64_t)H, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)sq[2], (uint64_t)sq[1], (uint64_t)sq[0]};
    int rc = encode_tiled(&mq, dt, 4, const_cast<void *>(q), dims, str, box, sw);
    if (rc) return rc;
  }
  const uint64_t sk_ext = static_cast<uint64_t>(Sk > 0 ? Sk : 1);
  {
    const uint64_t dims[4] = {(uint64_t)D, sk_ext, (uint64_t)H, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)sk[2], (uint64_t)sk[1], (uint64_t)sk[0]};
    int rc = encode_tiled(&mk, dt, 4, const_cast<void *>(k), dims, str, box, sw);
    if (rc) return rc;
  }
  {
    const uint64_t dims[4] = {sk_ext, (uint64_t)D, (uint64_t)H, (uint64_t)B};
    const uint64_t str[3] = {(uint64_t)svt[2], (uint64_t)svt[1], (uint64_t)svt[0]};
    const uint32_t vbox[4] = {static_cast<uint32_t>(BN), static_cast<uint32_t>(D), 1, 1};
    int rc = encode_tiled(&mv, dt, 4, const_cast<void *>(vt), dims, str, vbox,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  Args a{};
  a.o = o;
  a.so0 = so[0];
  a.so1 = so[1];
  a.so2 = so[2];
  a.so3 = so[3];
  a.H = static_cast<int>(H);
  a.Sq = static_cast<int>(Sq);
  a.Sk = static_cast<int>(Sk);
  a.n_qtiles = static_cast<int>((Sq + BM - 1) / BM);
  a.scale_log2 = sm_scale * scale_q * scale_k * kLog2e;
  a.causal = causal ? 1 : 0;
  a.vec_store = (so[3] == 1 && so[0] % 8 == 0 && so[1] % 8 == 0 && so[2] % 8 == 0 && aligned16(o)) ? 1 : 0;
  a.lse = nullptr;
  a.cu_q = nullptr;
  a.cu_k = nullptr;
  a.G = 1;
  a.out_scale = scale_v;
  set_groups(a, B, H, Sk, D, causal);
  const unsigned grid = static_cast<unsigned>(B * H * ((a.n_qtiles + 1) / 2));
  return launch_pp<GP>(flash_pp_kernel<T, __nv_fp8_e4m3, D, true, false, true>, grid, mq, mk, mv, a, st);
}

template <typename T>
int launch(const void *q, const void *k, const void *v, void *o, int64_t B, int64_t H, int64_t Sq,
           int64_t Sk, int64_t D, const int64_t *sq, const int64_t *sk, const int64_t *sv,
           const int64_t *so, float sm_scale, int causal, int variant, cudaStream_t st,
           const VarlenDesc *vl = nullptr, float *lse = nullptr) {
  switch (D) {
    case 16: return launch_d<T, 16>(q, k, v, o, B, H, Sq, Sk, sq, sk, sv, so, sm_scale, causal, variant, st, vl, lse);
    case 32: return launch_d<T, 32>(q, k, v, o, B, H, Sq, Sk, sq, sk, sv, so, sm_scale, causal, variant, st, vl, lse);
    case 64: return launch_d<T, 64>(q, k, v, o, B, H, Sq, Sk, sq, sk, sv, so, sm_scale, causal, variant, st, vl, lse);
    default: return launch_d<T, 128>(q, k, v, o, B, H, Sq, Sk, sq, sk, sv, so, sm_scale, causal, variant, st, vl, lse);
  }
}

}  // namespace
}  // namespace flash
}  // namespace tllm

namespace tllm {
namespace flash {
namespace {

int entry(const void *q, const void *k, const void *v, void *o, int64_t B, int64_t H, int64_t Sq,
          int64_t Sk, int64_t D, const int64_t *sq, const int64_t *sk, const int64_t *sv,
          const int64_t *so, float sm_scale, int causal, int dtype, int variant, void *stream,
          float *lse = nullptr) {
  clear_error();
  TLLM_CHECK_ARG(B >= 0 && H >= 0 && Sq >= 0 && Sk >= 0, "flash_attention: negative dimension");
  TLLM_CHECK_ARG(D == 16 || D == 32 || D == 64 || D == 128,
                 "flash_attention: head dim %lld not in {16,32,64,128}", (long long)D);
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16,
                 "flash_attention: unsupported dtype %d", dtype);
  TLLM_CHECK_ARG(variant == kVariantPingPong || variant == kVariantSingleTile ||
                     variant == kVariantPingPongOneItem || variant == kVariantSmemP,
                 "flash_attention: unknown kernel variant %d", variant);
  TLLM_CHECK_ARG(sq && sk && sv && so, "flash_attention: null stride array");
  if (B == 0 || H == 0 || Sq == 0) return TLLM_OK;
  if (Sk == 0) {
    // No keys (empty k/v may come as null pointers): every row is 0/0 = NaN, as in the
    // reference kernel. The key/value maps are built over q and never read.
    k = v = q;
    sk = sv = sq;
  }
  TLLM_CHECK_ARG(q && k && v && o, "flash_attention: null tensor pointer");
  TLLM_CHECK_ARG(Sq < (1LL << 31) && Sk < (1LL << 31) && B * H < (1LL << 31),
                 "flash_attention: problem too large");
  TLLM_CHECK_ARG(B * H * ((Sq + 127) / 128) < (1LL << 31), "flash_attention: grid too large");
  TLLM_CHECK_ARG(sq[3] == 1 && sk[3] == 1 && sv[3] == 1,
                 "flash_attention: q/k/v need a unit innermost stride");
  for (int i = 0; i < 3; ++i)
    TLLM_CHECK_ARG(sq[i] % 8 == 0 && sk[i] % 8 == 0 && sv[i] % 8 == 0,
                   "flash_attention: q/k/v strides must be multiples of 8 elements");
  TLLM_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v),
                 "flash_attention: q/k/v must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TLLM_DTYPE_F16)
    return launch<__half>(q, k, v, o, B, H, Sq, Sk, D, sq, sk, sv, so, sm_scale, causal, variant, st,
                          nullptr, lse);
  return launch<__nv_bfloat16>(q, k, v, o, B, H, Sq, Sk, D, sq, sk, sv, so, sm_scale, causal,
                               variant, st, nullptr, lse);
}

}  // namespace
}  // namespace flash
}  // namespace tllm

extern "C" int tllm_flash_attn_fwd(const void *q, const void *k, const void *v, void *o,
                                   int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                   const int64_t *sq, const int64_t *sk, const int64_t *sv,
                                   const int64_t *so, float sm_scale, int causal, int dtype,
                                   void *stream) {
  return tllm::flash::entry(q, k, v, o, B, H, Sq, Sk, D, sq, sk, sv, so, sm_scale, causal, dtype,
                            tllm::flash::kVariantPingPong, stream);
}

extern "C" int tllm_flash_attn_fwd_variant(const void *q, const void *k, const void *v, void *o,
                                           int64_t B, int64_t H, int64_t Sq, int64_t Sk,
                                           int64_t D, const int64_t *sq, const int64_t *sk,
                                           const int64_t *sv, const int64_t *so, float sm_scale,
                                           int causal, int dtype, int variant, void *stream) {
  return tllm::flash::entry(q, k, v, o, B, H, Sq, Sk, D, sq, sk, sv, so, sm_scale, causal, dtype,
                            variant, stream);
}

// tllm_flash_attn_fwd that also writes each query row's softmax log-normaliser (lse, fp32
// [B, H, Sq] contiguous) for the backward pass; no counterpart in the reference, which has the
// forward only.
extern "C" int tllm_flash_attn_fwd_lse(const void *q, const void *k, const void *v, void *o,
                                       float *lse, int64_t B, int64_t H, int64_t Sq, int64_t Sk,
                                       int64_t D, const int64_t *sq, const int64_t *sk,
                                       const int64_t *sv, const int64_t *so, float sm_scale,
                                       int causal, int dtype, void *stream) {
  if (!lse && B > 0 && H > 0 && Sq > 0) {
    tllm::clear_error();
    return tllm::fail(TLLM_ERR_INVALID, "flash_attention: null lse pointer");
  }
  return tllm::flash::entry(q, k, v, o, B, H, Sq, Sk, D, sq, sk, sv, so, sm_scale, causal, dtype,
                            tllm::flash::kVariantPingPong, stream, lse);
}

// Packed variable-length batch (no counterpart in the reference, whose flash_attention takes
// padded [B, H, S, D] tensors): q/o [total_q, H, D], k/v [total_k, Hkv, D] with strides
// {row, head, 1}; sequence b is rows [cu_q[b], cu_q[b+1]) of q/o and [cu_k[b], cu_k[b+1]) of
// k/v (int32, on the device); the causal mask is top-left aligned per sequence, as in
// flash_attention.
extern "C" int tllm_flash_attn_varlen_fwd(const void *q, const void *k, const void *v, void *o,
                                          const int *cu_seqlens_q, const int *cu_seqlens_k,
                                          int64_t B, int64_t H, int64_t Hkv, int64_t total_q,
                                          int64_t total_k, int64_t max_seqlen_q,
                                          int64_t max_seqlen_k, int64_t D, const int64_t *sq,
                                          const int64_t *sk, const int64_t *sv, const int64_t *so,
                                          float sm_scale, int causal, int dtype, void *stream) {
  using namespace tllm;
  using namespace tllm::flash;
  clear_error();
  TLLM_CHECK_ARG(B >= 0 && H >= 0 && Hkv >= 0 && total_q >= 0 && total_k >= 0 &&
                     max_seqlen_q >= 0 && max_seqlen_k >= 0,
                 "flash_attention_varlen: negative dimension");
  TLLM_CHECK_ARG(D == 16 || D == 32 || D == 64 || D == 128,
                 "flash_attention_varlen: head dim %lld not in {16,32,64,128}", (long long)D);
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16,
                 "flash_attention_varlen: unsupported dtype %d", dtype);
  TLLM_CHECK_ARG(sq && sk && sv && so, "flash_attention_varlen: null stride array");
  if (B == 0 || H == 0 || max_seqlen_q == 0 || total_q == 0) return TLLM_OK;
  TLLM_CHECK_ARG(Hkv >= 1 && H % Hkv == 0,
                 "flash_attention_varlen: %lld query heads do not group over %lld key/value heads",
                 (long long)H, (long long)Hkv);
  TLLM_CHECK_ARG(q && k && v && o && cu_seqlens_q && cu_seqlens_k,
                 "flash_attention_varlen: null pointer");
  TLLM_CHECK_ARG(total_q < (1LL << 31) && total_k < (1LL << 31) && B * H < (1LL << 31) &&
                     max_seqlen_q < (1LL << 31) && max_seqlen_k < (1LL << 31),
                 "flash_attention_varlen: problem too large");
  TLLM_CHECK_ARG(B * H * ((max_seqlen_q + 255) / 256) < (1LL << 31),
                 "flash_attention_varlen: grid too large");
  TLLM_CHECK_ARG(sq[2] == 1 && sk[2] == 1 && sv[2] == 1,
                 "flash_attention_varlen: q/k/v need a unit innermost stride");
  for (int i = 0; i < 2; ++i)
    TLLM_CHECK_ARG(sq[i] % 8 == 0 && sk[i] % 8 == 0 && sv[i] % 8 == 0,
                   "flash_attention_varlen: q/k/v strides must be multiples of 8 elements");
  TLLM_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(v),
                 "flash_attention_varlen: q/k/v must be 16-byte aligned");
  // As the dense launcher's {batch, head, row, 1} stride arrays; the batch stride is unused.
  const int64_t sq4[4] = {sq[0], sq[1], sq[0], 1};
  const int64_t sk4[4] = {sk[0], sk[1], sk[0], 1};
  const int64_t sv4[4] = {sv[0], sv[1], sv[0], 1};
  const int64_t so4[4] = {0, so[1], so[0], so[2]};
  const VarlenDesc vl{cu_seqlens_q, cu_seqlens_k, total_q, total_k, Hkv};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TLLM_DTYPE_F16)
    return launch<__half>(q, k, v, o, B, H, max_seqlen_q, max_seqlen_k, D, sq4, sk4, sv4, so4,
                          sm_scale, causal, kVariantPingPong, st, &vl);
  return launch<__nv_bfloat16>(q, k, v, o, B, H, max_seqlen_q, max_seqlen_k, D, sq4, sk4, sv4,
                               so4, sm_scale, causal, kVariantPingPong, st, &vl);
}

// FP8 (e4m3) inputs with per-tensor scales (no counterpart in the reference, whose
// flash_attention is fp16/bf16): softmax(sm_scale * (scale_q q)(scale_k k)^T) (scale_v v),
// causal top-left aligned as in flash_attention. q, k: [B, H, Sq|Sk, D]; vt: V transposed,
// [B, H, D, Sk] (keys contiguous); strides in elements, innermost 1, the others multiples of
// 16; o: [B, H, Sq, D] fp16 or bf16 (out_dtype). P is rounded to e4m3 for the P V product.
extern "C" int tllm_flash_attn_fp8_fwd(const void *q, const void *k, const void *vt, void *o,
                                       int64_t B, int64_t H, int64_t Sq, int64_t Sk, int64_t D,
                                       const int64_t *sq, const int64_t *sk, const int64_t *svt,
                                       const int64_t *so, float sm_scale, float scale_q,
                                       float scale_k, float scale_v, int causal, int out_dtype,
                                       void *stream) {
  using namespace tllm;
  using namespace tllm::flash;
  clear_error();
  TLLM_CHECK_ARG(B >= 0 && H >= 0 && Sq >= 0 && Sk >= 0, "flash_attention_fp8: negative dimension");
  TLLM_CHECK_ARG(D == 64 || D == 128, "flash_attention_fp8: head dim %lld not in {64,128}",
                 (long long)D);
  TLLM_CHECK_ARG(out_dtype == TLLM_DTYPE_F16 || out_dtype == TLLM_DTYPE_BF16,
                 "flash_attention_fp8: unsupported output dtype %d", out_dtype);
  TLLM_CHECK_ARG(sq && sk && svt && so, "flash_attention_fp8: null stride array");
  if (B == 0 || H == 0 || Sq == 0) return TLLM_OK;
  if (Sk == 0) {
    // No keys: NaN rows, as tllm_flash_attn_fwd; the key maps are built over q, never read.
    k = vt = q;
    sk = svt = sq;
  }
  TLLM_CHECK_ARG(q && k && vt && o, "flash_attention_fp8: null tensor pointer");
  TLLM_CHECK_ARG(Sq < (1LL << 31) && Sk < (1LL << 31) && B * H < (1LL << 31) &&
                     B * H * ((Sq + 255) / 256) < (1LL << 31),
                 "flash_attention_fp8: problem too large");
  TLLM_CHECK_ARG(sq[3] == 1 && sk[3] == 1 && svt[3] == 1,
                 "flash_attention_fp8: q/k/vt need a unit innermost stride");
  for (int i = 0; i < 3; ++i)
    TLLM_CHECK_ARG(sq[i] % 16 == 0 && sk[i] % 16 == 0 && svt[i] % 16 == 0,
                   "flash_attention_fp8: q/k/vt strides must be multiples of 16 elements");
  TLLM_CHECK_ARG(aligned16(q) && aligned16(k) && aligned16(vt),
                 "flash_attention_fp8: q/k/vt must be 16-byte aligned");
  TLLM_CHECK_ARG(std::isfinite(scale_q) && std::isfinite(scale_k) && std::isfinite(scale_v) &&
                     scale_q > 0.f && scale_k > 0.f && scale_v > 0.f,
                 "flash_attention_fp8: scales must be positive and finite");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (out_dtype == TLLM_DTYPE_F16)
    return D == 64 ? launch_fp8<__half, 64>(q, k, vt, o, B, H, Sq, Sk, sq, sk, svt, so, sm_scale,
                                            scale_q, scale_k, scale_v, causal, st)
                   : launch_fp8<__half, 128>(q, k, vt, o, B, H, Sq, Sk, sq, sk, svt, so, sm_scale,
                                             scale_q, scale_k, scale_v, causal, st);
  return D == 64 ? launch_fp8<__nv_bfloat16, 64>(q, k, vt, o, B, H, Sq, Sk, sq, sk, svt, so,
                                                 sm_scale, scale_q, scale_k, scale_v, causal, st)
                 : launch_fp8<__nv_bfloat16, 128>(q, k, vt, o, B, H, Sq, Sk, sq, sk, svt, so,
                                                  sm_scale, scale_q, scale_k, scale_v, causal, st);
}
