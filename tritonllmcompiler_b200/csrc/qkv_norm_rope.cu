// QKV projection with RMSNorm + RoPE fused into the GEMM epilogue (tcgen05 + TMEM + TMA).
//
// The reference runs the projection and rmsnorm_rope as separate passes
// (python/triton_llm/ops/rmsnorm_rope.py:51-75 reads the projected q/k back from HBM); here the
// GEMM's epilogue applies it per head while the tile is still in TMEM. out = x @ w with w
// [K, N], N = (Hq + 2 * Hkv) * 128 laid out as [q heads | k heads | v heads]; every q head
// (weight wq) and k head (weight wk) of each token row goes through the arithmetic of
// python/triton_llm/reference/norm_rope.py:12-40 on the projection rounded to the I/O dtype,
// with the cos/sin row of that token's position; v heads are stored as projected.
//
// B200 design: the swiglu mainloop (persistent, one CTA per SM; warp 0 TMA of x [128 x 64]
// and two [64 x 128] column blocks of w placed side by side as one N = 256 operand, 4-stage
// ring; warp 1 one 128x256x16 UMMA per k16 step into double-buffered TMEM accumulators), so
// one output tile is two heads of 128 tokens. Warps 2-5: one token row per thread; for each
// head its 128 fp32 values come out of TMEM, the RMSNorm reduction runs over the thread's own
// registers, and the rotate-half pairs (i, i + 64) are both in the thread. Every wait is
// bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.h"
#include "ptx.cuh"

namespace tllm {

__device__ int g_qkv_status = 0;

int qkv_read_status(int *out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_qkv_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyFromSymbol(qkv status)");
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_qkv_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyToSymbol(qkv status)");
  *out = v;
  return TLLM_OK;
}

namespace qkv {
namespace {

constexpr int BM = 128;
constexpr int HD = 128;  // head dim
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_CHUNK_BYTES = BK * 64 * 2;
constexpr int B_BYTES = 4 * B_CHUNK_BYTES;  // 256 output columns (two heads)
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int ACC_COLS = 2 * HD;
constexpr int TMEM_COLS = 512;
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 1024;

enum : int { SITE_EMPTY = 0x51, SITE_FULL = 0x52, SITE_TEMPTY = 0x53, SITE_TFULL = 0x54 };

struct Geom {
  int M, N, K;
  int tiles_m, tiles_n, k_blocks;
  int Hq, Hkv;
  int64_t ldo;
  const void *wq;  // [128] RMSNorm weights of the q heads
  const void *wk;  // [128] of the k heads
  const void *cosb;
  const void *sinb;
  int64_t scos, ssin;
  const int32_t *positions;  // [M]
  int rope_rows;
  float eps;
  // Tiles 0 .. n_wide-1 are 128 rows x 2 heads; the wide tiles that would form a partial last
  // wave are instead split into n_narrow tiles of one head each (half as long), numbered after
  // them.
  int n_wide, n_narrow;
};

// Rows, first head and head count of tile `tile` (0 heads: a one-head tile past the last head,
// skipped by every role).
__device__ __forceinline__ void tile_geo(const Geom &g, int tile, int &m0, int &head0, int &nheads) {
  if (tile < g.n_wide) {
    m0 = (tile % g.tiles_m) * BM;
    head0 = (tile / g.tiles_m) * 2;
    nheads = 2;
    return;
  }
  const int i = tile - g.n_wide;
  const int t = g.n_wide + (i >> 1);
  m0 = (t % g.tiles_m) * BM;
  head0 = (t / g.tiles_m) * 2 + (i & 1);
  nheads = head0 < g.Hq + 2 * g.Hkv ? 1 : 0;
}

template <typename T>
__device__ __forceinline__ float round_io(float v) {
  return to_f32<T>(from_f32<T>(v));
}

template <typename T>
__device__ __forceinline__ void ld8(const T *p, float (&v)[8]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(p));
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = Pack2<T>::unpack(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    qkv_norm_rope_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                         const __grid_constant__ CUtensorMap tm_w1, T *__restrict__ out, const Geom g) {
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
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;

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
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_w1);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_holder), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int num_tiles = g.n_wide + g.n_narrow;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int m0, head0, nheads;
        tile_geo(g, tile, m0, head0, nheads);
        if (nheads == 0) continue;
        for (int kb = 0; kb < g.k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&empty[stage]), phase ^ 1, abort_flag, &g_qkv_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_EMPTY)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_arrive_expect_tx(fb, A_BYTES + nheads * 2 * B_CHUNK_BYTES);
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
          const int k0 = kb * BK;
          tma_load_2d(sa, &tm_x, fb, k0, m0);
          // All 64-column chunks of the [BK x 128 * nheads] weight tile in one box.
          tma_load_3d(sb, nheads == 2 ? &tm_w : &tm_w1, fb, 0, k0, head0 * 2);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc2 = make_idesc_f16(BM, 2 * HD, kBF16, false, true);
      const uint32_t idesc1 = make_idesc_f16(BM, HD, kBF16, false, true);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        int m0, head0, nheads;
        tile_geo(g, tile, m0, head0, nheads);
        if (nheads == 0) continue;
        const uint32_t idesc = nheads == 2 ? idesc2 : idesc1;
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_phase ^ 1, abort_flag, &g_qkv_status,
                       TLLM_DEV_WAIT_TIMEOUT + SITE_TEMPTY)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * ACC_COLS;
        for (int kb = 0; kb < g.k_blocks; ++kb) {
          if (!mbar_wait(smem_u32(&full[stage]), phase, abort_flag, &g_qkv_status,
                         TLLM_DEV_WAIT_TIMEOUT + SITE_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t adesc = make_sdesc(sa + k * 32, 16, 1024, kSwizzle128B);
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
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int heads = g.Hq + 2 * g.Hkv;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int m0, h0, nheads;
      tile_geo(g, tile, m0, h0, nheads);
      if (nheads == 0) continue;
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_phase, abort_flag, &g_qkv_status,
                     TLLM_DEV_WAIT_TIMEOUT + SITE_TFULL))
        break;
      tc_fence_after();
      const int m = m0 + row;
      const bool mv = m < g.M;
      int pos = mv ? __ldg(g.positions + m) : 0;
      pos = min(max(pos, 0), g.rope_rows - 1);
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * ACC_COLS;
#pragma unroll 1
      for (int hh = 0; hh < nheads; ++hh) {
        const int head = h0 + hh;
        if (head >= heads) break;
        // The projection, rounded to the I/O dtype (what a separate GEMM would store).
        float v[HD];
        {
          uint32_t r[32];
#pragma unroll
          for (int c = 0; c < HD; c += 32) {
            tmem_ld32(t_row + hh * HD + c, r);
#pragma unroll
            for (int t = 0; t < 32; ++t) v[c + t] = round_io<T>(__uint_as_float(r[t]));
          }
        }
        T *orow = out + static_cast<int64_t>(m) * g.ldo + head * HD;
        if (head < g.Hq + g.Hkv) {
          const T *w = static_cast<const T *>(head < g.Hq ? g.wq : g.wk);
          float ss = 0.f;
#pragma unroll
          for (int t = 0; t < HD; ++t) ss = fmaf(v[t], v[t], ss);
          const float rstd = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(HD)), g.eps));
          const T *cr = static_cast<const T *>(g.cosb) + static_cast<int64_t>(pos) * g.scos;
          const T *sr = static_cast<const T *>(g.sinb) + static_cast<int64_t>(pos) * g.ssin;
#pragma unroll
          for (int c = 0; c < HD / 2; c += 8) {
            float w1[8], w2[8], c1[8], c2[8], s1[8], s2[8];
            ld8<T>(w + c, w1);
            ld8<T>(w + HD / 2 + c, w2);
            ld8<T>(cr + c, c1);
            ld8<T>(cr + HD / 2 + c, c2);
            ld8<T>(sr + c, s1);
            ld8<T>(sr + HD / 2 + c, s2);
            float o1[8], o2[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              const float y1 = round_io<T>(__fmul_rn(__fmul_rn(v[c + t], rstd), w1[t]));
              const float y2 = round_io<T>(__fmul_rn(__fmul_rn(v[HD / 2 + c + t], rstd), w2[t]));
              o1[t] = __fsub_rn(__fmul_rn(y1, c1[t]), __fmul_rn(y2, s1[t]));
              o2[t] = __fadd_rn(__fmul_rn(y2, c2[t]), __fmul_rn(y1, s2[t]));
            }
            if (mv) {
              uint4 p1, p2;
              p1.x = Pack2<T>::pack(o1[0], o1[1]); p1.y = Pack2<T>::pack(o1[2], o1[3]);
              p1.z = Pack2<T>::pack(o1[4], o1[5]); p1.w = Pack2<T>::pack(o1[6], o1[7]);
              p2.x = Pack2<T>::pack(o2[0], o2[1]); p2.y = Pack2<T>::pack(o2[2], o2[3]);
              p2.z = Pack2<T>::pack(o2[4], o2[5]); p2.w = Pack2<T>::pack(o2[6], o2[7]);
              *reinterpret_cast<uint4 *>(orow + c) = p1;
              *reinterpret_cast<uint4 *>(orow + HD / 2 + c) = p2;
            }
          }
        } else if (mv) {
#pragma unroll
          for (int c = 0; c < HD; c += 8) {
            uint4 pk;
            pk.x = Pack2<T>::pack(v[c + 0], v[c + 1]); pk.y = Pack2<T>::pack(v[c + 2], v[c + 3]);
            pk.z = Pack2<T>::pack(v[c + 4], v[c + 5]); pk.w = Pack2<T>::pack(v[c + 6], v[c + 7]);
            *reinterpret_cast<uint4 *>(orow + c) = pk;
          }
        }
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

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T>
int launch(const void *x, const void *w, void *out, const Geom &g0, int64_t lda, int64_t ldw,
           cudaStream_t st) {
  const CUtensorMapDataType dt =
      std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap mx, mw, mw1;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(g0.K), static_cast<uint64_t>(g0.M)};
    const uint64_t str[1] = {static_cast<uint64_t>(lda) * 2};
    const uint32_t box[2] = {BK, BM};
    int rc = encode_tiled(&mx, dt, 2, const_cast<void *>(x), dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    // 3-D view {64 columns, K, N / 64} of w (N is a multiple of the 128-wide head): the
    // outer dimension steps 64 columns, so one box {64, BK, 4} lands the tile's four
    // 128-byte-swizzled column chunks B_CHUNK_BYTES apart, as the UMMA descriptor expects.
    const uint64_t dims[3] = {64, static_cast<uint64_t>(g0.K), static_cast<uint64_t>(g0.N / 64)};
    const uint64_t str[2] = {static_cast<uint64_t>(ldw) * 2, 128};
    const uint32_t box[3] = {64, BK, 4};
    int rc = encode_tiled(&mw, dt, 3, const_cast<void *>(w), dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    const uint32_t box1[3] = {64, BK, 2};  // one head
    rc = encode_tiled(&mw1, dt, 3, const_cast<void *>(w), dims, str, box1, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  Geom g = g0;
  g.tiles_m = (g.M + BM - 1) / BM;
  g.tiles_n = (g.N + 2 * HD - 1) / (2 * HD);
  g.k_blocks = (g.K + BK - 1) / BK;
  const int wide_all = g.tiles_m * g.tiles_n;
  const int sms = sm_count() > 0 ? sm_count() : 148;
  const int grid = wide_all < sms ? wide_all : sms;
  // A partial last wave of wide tiles would keep a few SMs busy for a whole tile while the
  // rest wait: those tiles run as two one-head tiles each, half as long, on twice the SMs.
  const int rest = wide_all % grid;
  const bool split = wide_all > grid && rest > 0 && 2 * rest <= grid;
  g.n_wide = split ? wide_all - rest : wide_all;
  g.n_narrow = split ? 2 * rest : 0;
  auto kern = qkv_norm_rope_kernel<T>;
  KernelLaunchInfo info;
  const int rc = prepare_kernel(reinterpret_cast<const void *>(kern), SMEM_BYTES, kThreads, 1, &info);
  if (rc) return rc;
  kern<<<grid, kThreads, SMEM_BYTES, st>>>(mx, mw, mw1, static_cast<T *>(out), g);
  return cuda_status(cudaGetLastError(), "qkv norm rope launch");
}

}  // namespace
}  // namespace qkv
}  // namespace tllm

extern "C" int tllm_qkv_norm_rope(const void *x, const void *w, const void *wq, const void *wk,
                                  const void *cos, const void *sin, int64_t rope_rows,
                                  int64_t scos, int64_t ssin, const int32_t *positions, void *out,
                                  int64_t M, int64_t K, int64_t Hq, int64_t Hkv, int64_t D,
                                  int64_t lda, int64_t ldw, int64_t ldo, float eps, int dtype,
                                  void *stream) {
  using namespace tllm;
  clear_error();
  TLLM_CHECK_ARG(M >= 0 && K >= 0 && Hq >= 0 && Hkv >= 0, "qkv_norm_rope: negative dimension");
  TLLM_CHECK_ARG(D == 128, "qkv_norm_rope: head dim %lld, only 128 is supported", (long long)D);
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16, "qkv_norm_rope: unsupported dtype %d",
                 dtype);
  const int64_t N = (Hq + 2 * Hkv) * D;
  if (M == 0 || N == 0) return TLLM_OK;
  TLLM_CHECK_ARG(K > 0 && x && w && wq && wk && cos && sin && positions && out,
                 "qkv_norm_rope: null pointer or K == 0");
  TLLM_CHECK_ARG(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31), "qkv_norm_rope: dimension too large");
  TLLM_CHECK_ARG(rope_rows >= 1, "qkv_norm_rope: empty cos/sin table");
  TLLM_CHECK_ARG(lda >= K && ldw >= N && ldo >= N, "qkv_norm_rope: leading dimension too small");
  TLLM_CHECK_ARG(K % 8 == 0 && lda % 8 == 0 && ldw % 8 == 0 && ldo % 8 == 0 && scos % 8 == 0 && ssin % 8 == 0,
                 "qkv_norm_rope: K and the leading dimensions must be multiples of 8");
  TLLM_CHECK_ARG(qkv::aligned16(x) && qkv::aligned16(w) && qkv::aligned16(out) && qkv::aligned16(wq) &&
                     qkv::aligned16(wk) && qkv::aligned16(cos) && qkv::aligned16(sin),
                 "qkv_norm_rope: pointers must be 16-byte aligned");
  qkv::Geom g{};
  g.M = static_cast<int>(M);
  g.N = static_cast<int>(N);
  g.K = static_cast<int>(K);
  g.Hq = static_cast<int>(Hq);
  g.Hkv = static_cast<int>(Hkv);
  g.ldo = ldo;
  g.wq = wq;
  g.wk = wk;
  g.cosb = cos;
  g.sinb = sin;
  g.scos = scos;
  g.ssin = ssin;
  g.positions = positions;
  g.rope_rows = static_cast<int>(rope_rows);
  g.eps = eps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TLLM_DTYPE_F16) return qkv::launch<__half>(x, w, out, g, lda, ldw, st);
  return qkv::launch<__nv_bfloat16>(x, w, out, g, lda, ldw, st);
}
