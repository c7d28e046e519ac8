// SwiGLU dual GEMM for sm_100a: out = silu(x @ w1) * (x @ w3).
//
// Reference: python/triton_llm/ops/swiglu.py:11-76 (Triton, two register accumulators fed
// by shared x tile loads, silu(g)*u epilogue at :47-51) and the oracle
// python/triton_llm/reference/swiglu.py:12-15.
//
// B200 design (persistent, warp-specialised, one CTA per SM):
//   warp 0      TMA producer: per K-step one x tile [128 x 64] (K-major, 128B swizzle) and
//               the matching w1 and w3 tiles [64 x 128] (N-major) into a 4-stage ring; when N
//               is a multiple of 128 the weights are read through 3-D maps {64 columns, K,
//               N / 64} whose outer dimension steps 64 columns, so a whole [64 x 128] tile
//               (two 128-byte-swizzled column chunks) is one TMA box (3 boxes a stage, not 5).
//   warp 1      allocates 512 TMEM columns, then one lane issues tcgen05.mma: the w1 and w3
//               tiles sit side by side in shared memory as ONE N=256 operand, so a single
//               128x256x16 UMMA per k16 step computes [x@w1 | x@w3] into adjacent TMEM
//               columns (the x tile is read once for both products).
//   warps 2-5   epilogue: tcgen05.ld the two fp32 accumulators of a row, silu(g)*u in fp32,
//               one store in the I/O dtype. The accumulator is double-buffered in TMEM
//               (2 x 256 columns) so the epilogue of tile i overlaps the main loop of i+1.
// From M >= 256 (N a multiple of 128) swiglu_pair_kernel below runs instead: two CTAs on two
// SMs share each 256 x 128 output tile through tcgen05.mma.cta_group::2.
// Every CTA loads its own tiles; every mbarrier wait is bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstring>

#include "common.h"
#include "ptx.cuh"

namespace tllm {

__device__ int g_swiglu_status = 0;

int swiglu_read_status(int *out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_swiglu_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyFromSymbol(swiglu status)");
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_swiglu_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyToSymbol(swiglu status)");
  *out = v;
  return TLLM_OK;
}

namespace swiglu {
namespace {

constexpr int BM = 128;
constexpr int BN = 128;  // output columns per tile (each of w1 and w3)
constexpr int BK = 64;   // one 128-byte swizzle row of fp16
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;                 // 16 KB
constexpr int B_CHUNK_BYTES = BK * 64 * 2;           // 8 KB: 64 N-columns x BK rows
constexpr int B_BYTES = 4 * B_CHUNK_BYTES;           // w1[0:64] w1[64:128] w3[0:64] w3[64:128]
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;       // 48 KB
constexpr int ACC_COLS = 2 * BN;                     // G | U
constexpr int TMEM_COLS = 512;                       // two accumulator buffers
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*barriers*/ + 1024 /*alignment*/;
// Column-sharded mode: per epilogue thread, one 256-byte staging slot holding its row of the
// current output tile, which the bulk copies to the destinations read from.
constexpr int PEER_STAGE_BYTES = 128 * BN * 2;
constexpr int SMEM_BYTES_PEERS = SMEM_BYTES + PEER_STAGE_BYTES;

enum : int {
  SITE_EMPTY = 1,
  SITE_FULL = 2,
  SITE_TEMPTY = 3,
  SITE_TFULL = 4,
  SITE_PEER_READY = 5,   // a peer's call did not start
  SITE_PEER_ARRIVE = 6,  // a peer's stores did not complete
};

constexpr int kMaxDst = 8;

struct Geom {
  int M, N, K;
  int tiles_m, tiles_n, k_blocks;
  int64_t ldo;
  int vec_store;  // 16-byte stores allowed (ldo % 8 == 0 and every destination aligned)
  int w3d;        // weight maps are 3-D {64 columns, K, N / 64}: one box per 128-column tile
  // Column-sharded mode (ndst > 0): each output tile is written at column offset col_off
  // of every destination (this rank's [M, N_total] buffer and its peers', over NVLink)
  // instead of to `out`.
  int ndst;
  int64_t col_off;
  void *dst[kMaxDst];
  // Peer handshake of the column-sharded mode (flags[0] == nullptr: none, the caller orders
  // the calls). flags[d] points at rank d's flag words as mapped into this process: words
  // [kFlagReady + s] and [kFlagArrive + s] are written by rank s. rank is this rank's index
  // among the destinations, done counts this launch's finished CTAs (zero between launches),
  // epoch numbers the call (1, 2, ... per set of buffers).
  uint32_t *flags[kMaxDst];
  int rank;
  uint32_t *done;
  uint32_t epoch;
  // CTA-pair column-sharded kernel: the destination maps are 3-D {64 columns, N / 64, M} with
  // boxes of {64, 2, 32}, so every row of a box leaves as one 256-byte span (instead of two
  // 128-byte boxes per row block).
  int store3d;
  // CTA-pair column-sharded kernel: multicast address of the [M, ldo] output bound on every
  // rank (null: none). With it, each warp writes its staged block once through the multicast
  // address instead of once per destination.
  void *mc;
};

// Tensor maps of the destinations' column slices (column-sharded CTA-pair kernel): map d
// covers [M, N] at column offset col_off of destination d, boxes of 64 columns x 32 rows,
// 128-byte swizzle.
struct PeerMaps {
  CUtensorMap m[kMaxDst];
};

constexpr int kFlagReady = 0;
constexpr int kFlagArrive = kMaxDst;
static_assert(2 * kMaxDst == TLLM_SWIGLU_PEER_FLAG_WORDS, "flag words per rank");
// About two seconds at the boost clock: far longer than any peer's launch skew in a healthy
// job, short enough that a rank that never launches is reported instead of hanging.
constexpr long long kPeerWaitLimitCycles = 4000000000LL;

// One thread of CTA 0 at kernel start: tells every peer that this rank's call has begun, so
// every earlier operation on this rank's stream (reads of its previous output included) is
// complete and the peer may store into this rank's buffers.
__device__ __forceinline__ void peer_signal(const Geom &g, int which) {
  for (int d = 0; d < g.ndst; ++d)
    if (d != g.rank) st_release_sys(g.flags[d] + which + g.rank, g.epoch);
}

// Waits until every peer has raised its word `which` of this rank's flags to this call's
// epoch; gives up (records TLLM_DEV_WAIT_TIMEOUT + site, returns false) after the limit.
__device__ __forceinline__ bool peer_wait(const Geom &g, int which, int site) {
  const uint32_t *mine = g.flags[g.rank] + which;
  const long long t0 = clock64();
  for (int s = 0; s < g.ndst; ++s) {
    if (s == g.rank) continue;
    while (static_cast<int>(ld_acquire_sys(mine + s) - g.epoch) < 0) {
      if (clock64() - t0 > kPeerWaitLimitCycles) {
        atomicCAS(&g_swiglu_status, 0, TLLM_DEV_WAIT_TIMEOUT + site);
        return false;
      }
      __nanosleep(128);
    }
  }
  return true;
}

// One thread per CTA once every store of the CTA has completed: the last CTA of the launch
// tells every peer that this rank's stores into it are complete, then waits until every peer
// has said the same, so the launch ends only once this rank's [M, N_total] output is whole.
__device__ __forceinline__ void peer_finish(const Geom &g, int site) {
  __threadfence_system();
  const uint32_t prev = atomicAdd(g.done, 1u);
  if (prev != gridDim.x - 1) return;
  __threadfence_system();
  *g.done = 0u;  // the next launch on this stream starts after this one ends
  peer_signal(g, kFlagArrive);
  peer_wait(g, kFlagArrive, site);
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

template <typename T>
__device__ __forceinline__ void store_row_chunk(T *orow, int n_base, int N, bool vec,
                                                const float (&v)[32]) {
  if (vec && n_base + 32 <= N) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      uint4 raw;
      raw.x = Pack2<T>::pack(v[j + 0], v[j + 1]);
      raw.y = Pack2<T>::pack(v[j + 2], v[j + 3]);
      raw.z = Pack2<T>::pack(v[j + 4], v[j + 5]);
      raw.w = Pack2<T>::pack(v[j + 6], v[j + 7]);
      *reinterpret_cast<uint4 *>(orow + n_base + j) = raw;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (n_base + j < N) orow[n_base + j] = from_f32<T>(v[j]);
  }
}

// Asynchronous bulk copy of `bytes` (a multiple of 16) from shared to global memory, tracked
// in the issuing thread's bulk async-group.
__device__ __forceinline__ void bulk_store(void *dst, uint32_t src_smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(src_smem), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

template <typename T, bool kPeers>
__global__ void __launch_bounds__(kThreads, 1)
    swiglu_tc_kernel(const __grid_constant__ CUtensorMap tm_x,
                     const __grid_constant__ CUtensorMap tm_w1,
                     const __grid_constant__ CUtensorMap tm_w3, T *__restrict__ out,
                     const Geom g) {
  const bool handshake = kPeers && g.flags[0] != nullptr;
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
  volatile int *peer_ok = reinterpret_cast<volatile int *>(tmem_holder + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr bool kBF16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;

  if (handshake && blockIdx.x == 0 && threadIdx.x == 2 * 32) peer_signal(g, kFlagReady);
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
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (tile % g.tiles_m) * BM;
        const int n0 = (tile / g.tiles_m) * BN;
        for (int kb = 0; kb < g.k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag, &g_swiglu_status,
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
          if (g.w3d) {
            tma_load_3d(sb + 0 * B_CHUNK_BYTES, &tm_w1, fb, 0, k0, n0 >> 6);
            tma_load_3d(sb + 2 * B_CHUNK_BYTES, &tm_w3, fb, 0, k0, n0 >> 6);
          } else {
            tma_load_2d(sb + 0 * B_CHUNK_BYTES, &tm_w1, fb, n0, k0);
            tma_load_2d(sb + 1 * B_CHUNK_BYTES, &tm_w1, fb, n0 + 64, k0);
            tma_load_2d(sb + 2 * B_CHUNK_BYTES, &tm_w3, fb, n0, k0);
            tma_load_2d(sb + 3 * B_CHUNK_BYTES, &tm_w3, fb, n0 + 64, k0);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ UMMA issuer -------------------------------
    if (lane == 0) {
      const uint32_t idesc = make_idesc_f16(BM, 2 * BN, kBF16, false, true);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, abort_flag, &g_swiglu_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_TEMPTY)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
        for (int kb = 0; kb < g.k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, &g_swiglu_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // A: K-major, 128B swizzle, 8-row groups 1024 B apart; step 16 elements = 32 B.
            const uint64_t adesc = make_sdesc(sa + k * 32, 16, 1024, kSwizzle128B);
            // B: N-major, 128B swizzle; 64-column atoms 8 KB apart (LBO), 8-row K groups
            // 1024 B apart (SBO); step 16 K rows = 2048 B.
            const uint64_t bdesc = make_sdesc(sb + k * 2048, B_CHUNK_BYTES, 1024, kSwizzle128B);
            umma_f16_ss(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
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
    // ------------------------------ epilogue ----------------------------------
    const int quad = warp & 3;  // TMEM lanes this warp may access
    const int row = quad * 32 + lane;
    uint8_t *peer_stage = smem + SMEM_BYTES - 1024;  // past the barrier block (peer mode only)
    // Peer mode: no store into a peer before the peer's call has begun (its earlier reads of
    // the buffer are complete); the first tile's main loop runs meanwhile.
    bool remote_ok = true;
    if (handshake) {
      if (threadIdx.x == 2 * 32) *peer_ok = peer_wait(g, kFlagReady, SITE_PEER_READY) ? 1 : 0;
      named_bar_sync(1, kEpiThreads);
      remote_ok = *peer_ok != 0;
    }
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag, &g_swiglu_status,
                     TLLM_DEV_WAIT_TIMEOUT + SITE_TFULL))
        break;
      tc_fence_after();
      const int m0 = (tile % g.tiles_m) * BM;
      const int n0 = (tile / g.tiles_m) * BN;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * ACC_COLS;
      const int m = m0 + row;
      T *orow = out + static_cast<int64_t>(m) * g.ldo;
      int staged = 0;  // peer mode: 32-column chunks of this row staged for the bulk copies
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t gr[32], ur[32];
        tmem_ld32(t_row + c, gr);
        tmem_ld32(t_row + BN + c, ur);
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float gv = __uint_as_float(gr[j]);
          const float uv = __uint_as_float(ur[j]);
          v[j] = (gv / (1.0f + expf(-gv))) * uv;
        }
        if (!kPeers) {
          if (m < g.M) store_row_chunk<T>(orow, n0 + c, g.N, g.vec_store != 0, v);
        } else if (m < g.M) {
          if (g.vec_store && n0 + c + 32 <= g.N) {
            // Stage the 64-byte chunk in this thread's row slot; the whole row goes out in one
            // bulk copy per destination after the last chunk.
            if (c == 0) bulk_wait_read<0>();  // the previous tile's copies have read the slot
            uint8_t *slot = peer_stage + row * (BN * 2) + c * 2;
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 raw;
              raw.x = Pack2<T>::pack(v[j + 0], v[j + 1]);
              raw.y = Pack2<T>::pack(v[j + 2], v[j + 3]);
              raw.z = Pack2<T>::pack(v[j + 4], v[j + 5]);
              raw.w = Pack2<T>::pack(v[j + 6], v[j + 7]);
              *reinterpret_cast<uint4 *>(slot + j * 2) = raw;
            }
            ++staged;
          } else {
#pragma unroll 1
            for (int d = 0; d < g.ndst; ++d) {
              if (d != g.rank && !remote_ok) continue;
              T *drow = static_cast<T *>(g.dst[d]) + static_cast<int64_t>(m) * g.ldo + g.col_off;
              store_row_chunk<T>(drow, n0 + c, g.N, false, v);
            }
          }
        }
      }
      if (kPeers && staged > 0) {
        // Staged chunks are the leading ones of the row (only the N tail is stored directly).
        fence_proxy_async_smem();
        const uint32_t src = smem_u32(peer_stage + row * (BN * 2));
        const int64_t off = static_cast<int64_t>(m) * g.ldo + g.col_off + n0;
        // Rotated destination order per row (see the CTA-pair kernel).
        const int dstart = (static_cast<int>(blockIdx.x) + row) % g.ndst;
#pragma unroll 1
        for (int i = 0; i < g.ndst; ++i) {
          const int d = dstart + i < g.ndst ? dstart + i : dstart + i - g.ndst;
          if (d == g.rank || remote_ok) bulk_store(static_cast<T *>(g.dst[d]) + off, src, staged * 64);
        }
        bulk_commit();
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&tempty[acc]));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (kPeers) {
      // This thread's copies have landed; order them (and its direct stores) before the
      // system-scope completion signal.
      bulk_wait_all();
      fence_proxy_async_global();
      __threadfence_system();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
  if (handshake && threadIdx.x == 0) peer_finish(g, SITE_PEER_ARRIVE);
}

// =======================================================================================
// CTA-pair kernel (tcgen05.mma.cta_group::2): a cluster of two CTAs on two SMs computes a
// 256 x 128 output tile. CTA r loads its own 128 rows of x and one weight tile (r = 0: w1,
// r = 1: w3), [64 x 128] each, and the pair's leader (r = 0) issues 256 x 256 x 16 UMMAs
// whose A rows come from both CTAs' x tiles and whose B columns are the two weight tiles, so
// each CTA's TMEM receives its 128 rows x [x@w1 | x@w3], the layout the epilogue above reads.
// A stage is 32 KB per CTA instead of 48, so six stages fit where four did: the loads keep
// 1.7x as much time in flight, and each CTA reads two thirds of the bytes per FLOP.
//   Each CTA's loads land in its own shared memory and complete on the leader's full barrier
//   (the cta_group::2 form of the TMA load); the leader's UMMA commits arrive on the matching
//   barrier in both CTAs
//   (tcgen05.commit with a CTA mask); both CTAs' epilogue warps release an accumulator on
//   the leader's tempty barrier. TMEM is allocated and freed by one warp in each CTA with
//   cta_group::2, between cluster barriers.
// =======================================================================================
constexpr int kPairStageBytes = A_BYTES + 2 * B_CHUNK_BYTES;  // 32 KB: x rows + one weight tile
// Column-sharded mode: each epilogue warp stages its 32 rows x 128 columns of the finished
// tile (two 64-column halves, 128-byte swizzled, 4 KB each) twice over, so the tensor stores
// of one tile into every destination drain while the next tile is staged: 4 warps x 2 x 8 KB.
constexpr int kPairPeerStageBytes = 4 * 2 * 8192;
template <bool kPeers>
struct PairCfg {
  static constexpr int kStages = kPeers ? 5 : 6;  // the staging takes one stage's worth and more
  static constexpr int kSmemBytes =
      kStages * kPairStageBytes + 1024 + (kPeers ? kPairPeerStageBytes : 0) + 1024;
};
static_assert(PairCfg<true>::kSmemBytes <= 232448, "peer-mode pair kernel exceeds shared memory");

template <typename T, bool kPeers>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    swiglu_pair_kernel(const __grid_constant__ CUtensorMap tm_x,
                       const __grid_constant__ CUtensorMap tm_w1,
                       const __grid_constant__ CUtensorMap tm_w3, T *__restrict__ out,
                       const Geom g, const __grid_constant__ PeerMaps pm) {
  constexpr int kPairStages = PairCfg<kPeers>::kStages;
  const bool handshake = kPeers && g.flags[0] != nullptr;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kPairStages * kPairStageBytes);
  uint64_t *full = bars;
  uint64_t *empty = bars + kPairStages;
  uint64_t *tfull = bars + 2 * kPairStages;
  uint64_t *tempty = bars + 2 * kPairStages + 2;
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * kPairStages + 4);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  volatile int *peer_ok = reinterpret_cast<volatile int *>(tmem_holder + 2);
  // Peer mode: staging past the 1 KB barrier block (1024-byte aligned).
  uint8_t *peer_stage = smem + kPairStages * kPairStageBytes + 1024;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int n_pairs = static_cast<int>(gridDim.x >> 1);
  constexpr bool kBF16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;
  constexpr int kEpiWarps = kEpiThreads / 32;

  if (handshake && blockIdx.x == 0 && threadIdx.x == 2 * 32) peer_signal(g, kFlagReady);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) {
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
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag, &g_swiglu_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[stage]);
          // The leader's full barrier counts both CTAs' bytes.
          if (rank == 0) mbar_arrive_expect_tx(fb, 2 * kPairStageBytes);
          const uint32_t fb_leader = mapa_shared(fb, 0);
          const uint32_t sa = smem_u32(smem + stage * kPairStageBytes);
          const int k0 = kb * BK;
          tma_load_2d_pair(sa, &tm_x, fb_leader, k0, m0);
          tma_load_3d_pair(sa + A_BYTES, tm_w, fb_leader, 0, k0, n0 >> 6);
          if (++stage == kPairStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // The leader's last commits arrive on this CTA's empty barriers: wait for them before
      // the CTA may exit.
      for (int i = 0; ok && i < kPairStages; ++i) {
        ok = mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag, &g_swiglu_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_EMPTY);
        if (++stage == kPairStages) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ UMMA issuer (leader) -----------------------
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = make_idesc_f16(2 * BM, 2 * BN, kBF16, false, true);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = pair; tile < num_tiles && ok; tile += n_pairs) {
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, abort_flag, &g_swiglu_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_TEMPTY)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
        for (int kb = 0; kb < g.k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, &g_swiglu_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * kPairStageBytes);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // A: this CTA's (and the peer's) x rows, K-major, 128B swizzle; B: each CTA's
            // weight tile, N-major, two 64-column chunks B_CHUNK_BYTES apart.
            const uint64_t adesc = make_sdesc(sa + k * 32, 16, 1024, kSwizzle128B);
            const uint64_t bdesc = make_sdesc(sb + k * 2048, B_CHUNK_BYTES, 1024, kSwizzle128B);
            umma_f16_ss_pair(d_tmem, adesc, bdesc, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_pair(smem_u32(&empty[stage]));
          if (++stage == kPairStages) {
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
    bool remote_ok = true;
    if (handshake) {
      // No store into a peer before the peer's call has begun; the first main loop runs meanwhile.
      if (threadIdx.x == 2 * 32) *peer_ok = peer_wait(g, kFlagReady, SITE_PEER_READY) ? 1 : 0;
      named_bar_sync(1, kEpiThreads);
      remote_ok = *peer_ok != 0;
    }
    int acc = 0;
    uint32_t acc_phase = 0;
    int it = 0;  // tiles this CTA has finished (peer mode: picks the staging buffer)
    for (int tile = pair; tile < num_tiles; tile += n_pairs, ++it) {
      if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag,
                                             &g_swiglu_status, TLLM_DEV_WAIT_TIMEOUT + SITE_TFULL)))
        break;
      tc_fence_after();
      const int m0 = (tile % g.tiles_m) * (2 * BM) + static_cast<int>(rank) * BM;
      const int n0 = (tile / g.tiles_m) * BN;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * ACC_COLS;
      const int m = m0 + row;
      T *orow = out + static_cast<int64_t>(m) * g.ldo;
      // Peer mode: this warp's staging buffer for this tile; the tensor stores that read it
      // two tiles ago must have finished reading (the last tile's may still be in flight).
      uint8_t *wst = peer_stage + quad * 16384 + (it & 1) * 8192;
      if (kPeers) {
        if (lane == 0 && it >= 2) bulk_wait_read<1>();
        __syncwarp();
      }
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t gr[32], ur[32];
        tmem_ld32(t_row + c, gr);
        tmem_ld32(t_row + BN + c, ur);
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float gv = __uint_as_float(gr[j]);
          const float uv = __uint_as_float(ur[j]);
          v[j] = (gv / (1.0f + expf(-gv))) * uv;
        }
        if (!kPeers) {
          if (m < g.M) store_row_chunk<T>(orow, n0 + c, g.N, g.vec_store != 0, v);
        } else {
          // Row `lane` of the 64-column half c / 64, 16-byte units (c % 64) / 8 .. +3, placed
          // by the 128-byte swizzle (unit ^ row % 8) the tensor maps expect.
          // 3-D boxes: 128-byte row R = 2 * lane + c / 64 of the box, swizzled by R % 8.
          const int srow = g.store3d ? 2 * lane + (c >> 6) : lane;
          uint8_t *hrow = g.store3d ? wst + srow * 128 : wst + (c >> 6) * 4096 + lane * 128;
          const int u0 = (c & 32) >> 3;
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            uint4 raw;
            raw.x = Pack2<T>::pack(v[8 * jj + 0], v[8 * jj + 1]);
            raw.y = Pack2<T>::pack(v[8 * jj + 2], v[8 * jj + 3]);
            raw.z = Pack2<T>::pack(v[8 * jj + 4], v[8 * jj + 5]);
            raw.w = Pack2<T>::pack(v[8 * jj + 6], v[8 * jj + 7]);
            *reinterpret_cast<uint4 *>(hrow + (((u0 + jj) ^ (srow & 7)) << 4)) = raw;
          }
        }
      }
      if (kPeers) fence_proxy_async_smem();  // staged rows visible to the tensor stores
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty_leader[acc]);
      if (kPeers && g.mc != nullptr && remote_ok) {
        // The warp's 32 rows x 128 columns once through the multicast address; the switch
        // writes them into every rank's buffer. A lane stores 16-byte unit uu of row r for
        // idx = 32 k + lane = 16 r + uu, so each half-warp writes 256 contiguous bytes of a row.
        const int y = m0 + quad * 32;
        T *mrow0 = static_cast<T *>(g.mc) + g.col_off + n0;
#pragma unroll 4
        for (int k = 0; k < 16; ++k) {
          const int idx = 32 * k + lane;
          const int r = idx >> 4, uu = idx & 15;
          if (y + r < g.M) {
            const uint4 v = *reinterpret_cast<const uint4 *>(
                wst + (uu >> 3) * 4096 + r * 128 + (((uu & 7) ^ (r & 7)) << 4));
            multimem_st_v4(mrow0 + static_cast<int64_t>(y + r) * g.ldo + uu * 8, v);
          }
        }
      } else if (kPeers && lane == 0) {
        // The warp's 32 rows x 128 columns into every destination's slice; rows past M are
        // clipped by the tensor maps.
        const int y = m0 + quad * 32;
        // Destinations in a rotated order (by CTA and warp), so that at any moment the SMs'
        // stores spread over all peers instead of all targeting the same one.
        const int dstart = (static_cast<int>(blockIdx.x) + quad) % g.ndst;
#pragma unroll 1
        for (int i = 0; i < g.ndst; ++i) {
          const int d = dstart + i < g.ndst ? dstart + i : dstart + i - g.ndst;
          if (d != g.rank && !remote_ok) continue;
          if (g.store3d) {
            tma_store_3d(&pm.m[d], smem_u32(wst), 0, n0 >> 6, y);
          } else {
            tma_store_2d(&pm.m[d], smem_u32(wst), n0, y);
            tma_store_2d(&pm.m[d], smem_u32(wst + 4096), n0 + 64, y);
          }
        }
        bulk_commit();
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (kPeers && lane == 0) {
      bulk_wait_all();  // this warp's stores have landed in every destination
      fence_proxy_async_global();
      __threadfence_system();
    }
    // Multicast stores: every storing thread orders its stores before the flags that the
    // last CTA raises after the barrier below.
    if (kPeers && g.mc != nullptr) __threadfence_system();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no UMMA, commit or remote arrive of either CTA is still pending
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
  if (handshake && threadIdx.x == 0) peer_finish(g, SITE_PEER_ARRIVE);
}

// Layout-agnostic fallback (CUDA cores, fp32 accumulation) for shapes whose strides or
// alignment a TMA descriptor cannot describe: K or N not a multiple of 8, odd strides.
template <typename T>
__global__ void __launch_bounds__(256) swiglu_simt_kernel(const T *__restrict__ x,
                                                          const T *__restrict__ w1,
                                                          const T *__restrict__ w3,
                                                          T *__restrict__ out, int M, int N,
                                                          int K, int64_t lda, int64_t ldb1,
                                                          int64_t ldb3, int64_t ldo) {
  __shared__ float xs[16][17];
  __shared__ float w1s[16][17];
  __shared__ float w3s[16][17];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m = blockIdx.y * 16 + ty;
  const int n = blockIdx.x * 16 + tx;
  float gacc = 0.f, uacc = 0.f;
  for (int k0 = 0; k0 < K; k0 += 16) {
    xs[ty][tx] = (m < M && k0 + tx < K) ? to_f32<T>(x[static_cast<int64_t>(m) * lda + k0 + tx]) : 0.f;
    const int kr = k0 + ty;
    w1s[ty][tx] = (kr < K && n < N) ? to_f32<T>(w1[static_cast<int64_t>(kr) * ldb1 + n]) : 0.f;
    w3s[ty][tx] = (kr < K && n < N) ? to_f32<T>(w3[static_cast<int64_t>(kr) * ldb3 + n]) : 0.f;
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      gacc = fmaf(xs[ty][kk], w1s[kk][tx], gacc);
      uacc = fmaf(xs[ty][kk], w3s[kk][tx], uacc);
    }
    __syncthreads();
  }
  if (m < M && n < N)
    out[static_cast<int64_t>(m) * ldo + n] = from_f32<T>((gacc / (1.0f + expf(-gacc))) * uacc);
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Kernel choice (tllm_swiglu_variant): the CTA-pair kernel whenever it applies, or forced.
constexpr int kVariantAuto = 0;
constexpr int kVariantSingleCta = 1;
constexpr int kVariantCtaPair = 2;
constexpr int kVariantCtaPair3D = 3;  // column-sharded: CTA pairs storing 256-byte rows

// Column-sharded destinations and the peer handshake (see Geom).
struct PeerArgs {
  void *const *dsts = nullptr;
  int ndst = 0;
  int64_t col_off = 0;
  uint32_t *const *flags = nullptr;  // null: no handshake
  int rank = 0;
  uint32_t *done = nullptr;
  uint32_t epoch = 0;
  void *mc = nullptr;  // multicast address of the outputs (CTA-pair kernel only)
};

template <typename T>
int launch(const void *x, const void *w1, const void *w3, void *out, int64_t M, int64_t N,
           int64_t K, int64_t lda, int64_t ldb1, int64_t ldb3, int64_t ldo, cudaStream_t st,
           const PeerArgs &pa = PeerArgs(), int variant = kVariantAuto) {
  const int ndst = pa.ndst;
  void *const *dsts = pa.dsts;
  const int64_t col_off = pa.col_off;
  const bool tma_ok = lda % 8 == 0 && ldb1 % 8 == 0 && ldb3 % 8 == 0 && aligned16(x) &&
                      aligned16(w1) && aligned16(w3) && K % 8 == 0 && N % 8 == 0;
  if (!tma_ok && ndst > 0)
    return fail(TLLM_ERR_INVALID,
                "swiglu column-sharded: K, N and the leading dimensions must be multiples of 8 "
                "and x, w1, w3 16-byte aligned");
  if (!tma_ok) {
    dim3 grid(static_cast<unsigned>((N + 15) / 16), static_cast<unsigned>((M + 15) / 16));
    swiglu_simt_kernel<T><<<grid, 256, 0, st>>>(
        static_cast<const T *>(x), static_cast<const T *>(w1), static_cast<const T *>(w3),
        static_cast<T *>(out), static_cast<int>(M), static_cast<int>(N), static_cast<int>(K),
        lda, ldb1, ldb3, ldo);
    return cuda_status(cudaGetLastError(), "swiglu fallback launch");
  }
  const CUtensorMapDataType dt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap mx, m1, m3;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 2};
    const uint32_t box[2] = {BK, BM};
    int rc = encode_tiled(&mx, dt, 2, const_cast<void *>(x), dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  const bool w3d = N % 128 == 0;
  if (w3d) {
    const uint64_t dims[3] = {64, static_cast<uint64_t>(K), static_cast<uint64_t>(N / 64)};
    const uint32_t box[3] = {64, BK, 2};
    const uint64_t s1[2] = {static_cast<uint64_t>(ldb1) * 2, 128};
    int rc = encode_tiled(&m1, dt, 3, const_cast<void *>(w1), dims, s1, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const uint64_t s3[2] = {static_cast<uint64_t>(ldb3) * 2, 128};
    rc = encode_tiled(&m3, dt, 3, const_cast<void *>(w3), dims, s3, box,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(K)};
    const uint32_t box[2] = {64, BK};
    const uint64_t s1[1] = {static_cast<uint64_t>(ldb1) * 2};
    int rc = encode_tiled(&m1, dt, 2, const_cast<void *>(w1), dims, s1, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const uint64_t s3[1] = {static_cast<uint64_t>(ldb3) * 2};
    rc = encode_tiled(&m3, dt, 2, const_cast<void *>(w3), dims, s3, box,
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
  g.w3d = w3d ? 1 : 0;
  g.ndst = ndst;
  g.col_off = col_off;
  bool dst_aligned = true;
  for (int d = 0; d < kMaxDst; ++d) {
    g.dst[d] = d < ndst ? dsts[d] : nullptr;
    if (d < ndst) dst_aligned = dst_aligned && aligned16(dsts[d]);
    g.flags[d] = (pa.flags && d < ndst) ? pa.flags[d] : nullptr;
  }
  g.rank = pa.rank;
  g.done = pa.done;
  g.epoch = pa.epoch;
  g.store3d = 0;
  g.mc = nullptr;
  g.vec_store = (ldo % 8 == 0 && col_off % 8 == 0 && dst_aligned &&
                 (ndst > 0 || aligned16(out))) ? 1 : 0;
  const int sms = sm_count();
  // The CTA pair needs the one-box weight tiles and pays off from two 128-row blocks up. In
  // the column-sharded mode it writes each destination through a tensor map of its slice.
  const bool peer_maps_ok = ldo % 8 == 0 && col_off % 8 == 0 && dst_aligned;
  const bool pair_ok = w3d && sms >= 2 && (ndst == 0 || peer_maps_ok);
  if (variant == kVariantCtaPair && !pair_ok)
    return fail(TLLM_ERR_INVALID,
                "swiglu: the CTA-pair kernel needs N %% 128 == 0 (and, column-sharded, 16-byte "
                "aligned destinations, column offset and row stride)");
  if (variant == kVariantCtaPair3D && !(pair_ok && ndst > 0))
    return fail(TLLM_ERR_INVALID, "swiglu: variant 3 is the column-sharded CTA-pair kernel");
  if (pair_ok && (variant == kVariantCtaPair || variant == kVariantCtaPair3D ||
                  (variant == kVariantAuto && M >= 2 * BM))) {
    Geom gp = g;
    gp.tiles_m = static_cast<int>((M + 2 * BM - 1) / (2 * BM));
    const int pair_tiles = gp.tiles_m * gp.tiles_n;
    PeerMaps pm;
    memset(&pm, 0, sizeof(pm));
    gp.store3d = variant == kVariantCtaPair3D ? 1 : 0;
    if (pa.mc != nullptr) {
      gp.mc = pa.mc;
      gp.store3d = 0;  // the multicast stores read the 2-D staging layout
    }
    for (int d = 0; d < ndst; ++d) {
      int rc;
      if (gp.store3d) {
        const uint64_t dims[3] = {64, static_cast<uint64_t>(N / 64), static_cast<uint64_t>(M)};
        const uint64_t strides[2] = {128, static_cast<uint64_t>(ldo) * 2};
        const uint32_t box[3] = {64, 2, 32};
        rc = encode_tiled(&pm.m[d], dt, 3, static_cast<T *>(dsts[d]) + col_off, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
      } else {
        const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
        const uint64_t strides[1] = {static_cast<uint64_t>(ldo) * 2};
        const uint32_t box[2] = {64, 32};
        rc = encode_tiled(&pm.m[d], dt, 2, static_cast<T *>(dsts[d]) + col_off, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B);
      }
      if (rc) return rc;
    }
    auto kern = ndst == 0 ? swiglu_pair_kernel<T, false> : swiglu_pair_kernel<T, true>;
    const int smem = ndst == 0 ? PairCfg<false>::kSmemBytes : PairCfg<true>::kSmemBytes;
    // Persistent grid: as many pairs as can be resident at once (clusters are placed on SM
    // pairs of one GPC).
    KernelLaunchInfo info;
    const int rc = prepare_kernel(reinterpret_cast<const void *>(kern), smem, kThreads, 2, &info);
    if (rc) return rc;
    const int max_clusters = info.resident;
    if (max_clusters < 1) return fail(TLLM_ERR_CUDA, "swiglu: the CTA-pair kernel cannot be resident");
    const int max_pairs = max_clusters < sms / 2 ? max_clusters : sms / 2;
    const int pairs = pair_tiles < max_pairs ? pair_tiles : max_pairs;
    kern<<<2 * pairs, kThreads, smem, st>>>(mx, m1, m3, static_cast<T *>(out), gp, pm);
    return cuda_status(cudaGetLastError(), ndst == 0 ? "swiglu pair launch" : "swiglu pair peers launch");
  }
  const int num_tiles = g.tiles_m * g.tiles_n;
  const int grid = num_tiles < sms ? num_tiles : sms;
  if (ndst == 0) {
    auto kern = swiglu_tc_kernel<T, false>;
    KernelLaunchInfo info;
    const int rc = prepare_kernel(reinterpret_cast<const void *>(kern), SMEM_BYTES, kThreads, 1, &info);
    if (rc) return rc;
    kern<<<grid, kThreads, SMEM_BYTES, st>>>(mx, m1, m3, static_cast<T *>(out), g);
    return cuda_status(cudaGetLastError(), "swiglu launch");
  }
  auto kern = swiglu_tc_kernel<T, true>;
  KernelLaunchInfo info;
  const int rc = prepare_kernel(reinterpret_cast<const void *>(kern), SMEM_BYTES_PEERS, kThreads, 1, &info);
  if (rc) return rc;
  kern<<<grid, kThreads, SMEM_BYTES_PEERS, st>>>(mx, m1, m3, static_cast<T *>(out), g);
  return cuda_status(cudaGetLastError(), "swiglu peers launch");
}

}  // namespace
}  // namespace swiglu
}  // namespace tllm

extern "C" int tllm_swiglu(const void *x, const void *w1, const void *w3, void *out, int64_t M,
                           int64_t N, int64_t K, int64_t lda, int64_t ldb1, int64_t ldb3,
                           int64_t ldo, int dtype, void *stream) {
  using namespace tllm;
  clear_error();
  TLLM_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "swiglu: negative dimension");
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16, "swiglu: unsupported dtype %d",
                 dtype);
  TLLM_CHECK_ARG(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31), "swiglu: dimension too large");
  if (M == 0 || N == 0) return TLLM_OK;
  TLLM_CHECK_ARG(out, "swiglu: null output pointer");
  // With K == 0 the inputs are empty (and may be null); the result is silu(0) * 0 = 0.
  TLLM_CHECK_ARG(K == 0 || (x && w1 && w3), "swiglu: null tensor pointer");
  TLLM_CHECK_ARG(lda >= K && ldb1 >= N && ldb3 >= N && ldo >= N, "swiglu: leading dimension too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (K == 0) {
    // x @ w = 0, silu(0) * 0 = 0: a zero fill keeps the contract without a GEMM.
    return cuda_status(cudaMemset2DAsync(out, static_cast<size_t>(ldo) * 2, 0,
                                         static_cast<size_t>(N) * 2, static_cast<size_t>(M), st),
                       "swiglu zero fill");
  }
  if (dtype == TLLM_DTYPE_F16)
    return swiglu::launch<__half>(x, w1, w3, out, M, N, K, lda, ldb1, ldb3, ldo, st);
  return swiglu::launch<__nv_bfloat16>(x, w1, w3, out, M, N, K, lda, ldb1, ldb3, ldo, st);
}

// tllm_swiglu with an explicit kernel choice, for cross-checking: 0 = automatic, 1 = one CTA
// per 128 x 128 tile, 2 = the CTA-pair kernel (N a multiple of 128).
extern "C" int tllm_swiglu_variant(const void *x, const void *w1, const void *w3, void *out,
                                   int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb1,
                                   int64_t ldb3, int64_t ldo, int dtype, int variant, void *stream) {
  using namespace tllm;
  clear_error();
  TLLM_CHECK_ARG(variant >= 0 && variant <= 2, "swiglu: unknown kernel variant %d", variant);
  TLLM_CHECK_ARG(M > 0 && N > 0 && K > 0 && M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31),
                 "swiglu: dimensions must be positive");
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16, "swiglu: unsupported dtype %d",
                 dtype);
  TLLM_CHECK_ARG(x && w1 && w3 && out, "swiglu: null tensor pointer");
  TLLM_CHECK_ARG(lda >= K && ldb1 >= N && ldb3 >= N && ldo >= N, "swiglu: leading dimension too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const swiglu::PeerArgs none;
  if (dtype == TLLM_DTYPE_F16)
    return swiglu::launch<__half>(x, w1, w3, out, M, N, K, lda, ldb1, ldb3, ldo, st, none, variant);
  return swiglu::launch<__nv_bfloat16>(x, w1, w3, out, M, N, K, lda, ldb1, ldb3, ldo, st, none,
                                       variant);
}

extern "C" int tllm_swiglu_colshard(const void *x, const void *w1, const void *w3,
                                    void *const *dsts, int ndst, int64_t col_off, int64_t M,
                                    int64_t N, int64_t K, int64_t lda, int64_t ldb1, int64_t ldb3,
                                    int64_t ldo, int dtype, void *stream) {
  using namespace tllm;
  clear_error();
  TLLM_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "swiglu column-sharded: negative dimension");
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16,
                 "swiglu column-sharded: unsupported dtype %d", dtype);
  TLLM_CHECK_ARG(dsts && ndst >= 1 && ndst <= swiglu::kMaxDst,
                 "swiglu column-sharded: 1..%d destinations required", swiglu::kMaxDst);
  TLLM_CHECK_ARG(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31),
                 "swiglu column-sharded: dimension too large");
  TLLM_CHECK_ARG(col_off >= 0 && ldo >= col_off + N, "swiglu column-sharded: columns outside the row");
  if (M == 0 || N == 0) return TLLM_OK;
  for (int d = 0; d < ndst; ++d)
    TLLM_CHECK_ARG(dsts[d], "swiglu column-sharded: null destination %d", d);
  TLLM_CHECK_ARG(K > 0 && x && w1 && w3, "swiglu column-sharded: K must be positive");
  TLLM_CHECK_ARG(lda >= K && ldb1 >= N && ldb3 >= N, "swiglu column-sharded: leading dimension too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  swiglu::PeerArgs pa;
  pa.dsts = dsts;
  pa.ndst = ndst;
  pa.col_off = col_off;
  if (dtype == TLLM_DTYPE_F16)
    return swiglu::launch<__half>(x, w1, w3, dsts[0], M, N, K, lda, ldb1, ldb3, ldo, st, pa);
  return swiglu::launch<__nv_bfloat16>(x, w1, w3, dsts[0], M, N, K, lda, ldb1, ldb3, ldo, st, pa);
}

namespace tllm {
namespace swiglu {
namespace {
// Shared by the two peer-handshake entries: argument checks, then the launch (mc: the
// multicast address of the outputs, or null).
int colshard_peers(const void *x, const void *w1, const void *w3, void *const *dsts,
                   uint32_t *const *flags, int ndst, int rank, uint32_t *done, uint32_t epoch,
                   int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb1, int64_t ldb3,
                   int64_t ldo, int dtype, int variant, void *mc, void *stream) {
  TLLM_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "swiglu column-sharded: negative dimension");
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16,
                 "swiglu column-sharded: unsupported dtype %d", dtype);
  TLLM_CHECK_ARG(variant >= 0 && variant <= 3, "swiglu column-sharded: unknown kernel variant %d",
                 variant);
  TLLM_CHECK_ARG(dsts && flags && done && ndst >= 1 && ndst <= kMaxDst,
                 "swiglu column-sharded: 1..%d destinations, their flags and a done counter required",
                 kMaxDst);
  TLLM_CHECK_ARG(rank >= 0 && rank < ndst, "swiglu column-sharded: rank %d outside 0..%d", rank,
                 ndst - 1);
  TLLM_CHECK_ARG(epoch != 0, "swiglu column-sharded: epoch 0 is the flags' initial value");
  TLLM_CHECK_ARG(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31),
                 "swiglu column-sharded: dimension too large");
  const int64_t col_off = static_cast<int64_t>(rank) * N;
  TLLM_CHECK_ARG(ldo >= static_cast<int64_t>(ndst) * N, "swiglu column-sharded: row stride below N * ranks");
  for (int d = 0; d < ndst; ++d)
    TLLM_CHECK_ARG(dsts[d] && flags[d], "swiglu column-sharded: null destination or flags %d", d);
  // Every rank takes part in every call, empty or not: a call that returned early here would
  // leave its peers waiting for this rank's flags.
  TLLM_CHECK_ARG(M > 0 && N > 0 && K > 0 && x && w1 && w3,
                 "swiglu column-sharded: M, N and K must be positive");
  TLLM_CHECK_ARG(lda >= K && ldb1 >= N && ldb3 >= N, "swiglu column-sharded: leading dimension too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  PeerArgs pa;
  pa.dsts = dsts;
  pa.ndst = ndst;
  pa.col_off = col_off;
  pa.flags = flags;
  pa.rank = rank;
  pa.done = done;
  pa.epoch = epoch;
  pa.mc = mc;
  if (dtype == TLLM_DTYPE_F16)
    return launch<__half>(x, w1, w3, dsts[rank], M, N, K, lda, ldb1, ldb3, ldo, st, pa,
                                  variant);
  return launch<__nv_bfloat16>(x, w1, w3, dsts[rank], M, N, K, lda, ldb1, ldb3, ldo, st, pa,
                                       variant);
}
}  // namespace
}  // namespace swiglu
}  // namespace tllm

extern "C" int tllm_swiglu_colshard_peers(const void *x, const void *w1, const void *w3,
                                          void *const *dsts, uint32_t *const *flags, int ndst,
                                          int rank, uint32_t *done, uint32_t epoch, int64_t M,
                                          int64_t N, int64_t K, int64_t lda, int64_t ldb1,
                                          int64_t ldb3, int64_t ldo, int dtype, int variant,
                                          void *stream) {
  tllm::clear_error();
  return tllm::swiglu::colshard_peers(x, w1, w3, dsts, flags, ndst, rank, done, epoch, M, N, K, lda,
                                      ldb1, ldb3, ldo, dtype, variant, nullptr, stream);
}

extern "C" int tllm_swiglu_colshard_multicast(const void *x, const void *w1, const void *w3,
                                              void *const *dsts, void *mc,
                                              uint32_t *const *flags, int ndst, int rank,
                                              uint32_t *done, uint32_t epoch, int64_t M,
                                              int64_t N, int64_t K, int64_t lda, int64_t ldb1,
                                              int64_t ldb3, int64_t ldo, int dtype, void *stream) {
  using namespace tllm;
  clear_error();
  TLLM_CHECK_ARG(mc != nullptr && (reinterpret_cast<uintptr_t>(mc) & 15u) == 0,
                 "swiglu column-sharded: the multicast address must be non-null and 16-byte aligned");
  return swiglu::colshard_peers(x, w1, w3, dsts, flags, ndst, rank, done, epoch, M, N, K, lda, ldb1,
                                ldb3, ldo, dtype, 0, mc, stream);
}
