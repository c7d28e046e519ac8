// Paged-KV decode attention for sm_100a.
//
// Reference: python/triton_llm/ops/paged_attention.py:11-128 (one Triton program per
// (b, h) walking every block of the sequence serially, with a host .item() sync to size the
// loop) and the oracle python/triton_llm/reference/paged_attention.py:14-40 (gather the
// blocks through block_tables, truncate to context_len, dense softmax attention).
//
// B200 design: decode reads every K/V byte exactly once, so the kernel is an HBM stream.
// Each sequence is cut into fixed token chunks ("splits"); one CTA handles one
// (split, head, sequence). Every token's D-vector is 2*D contiguous bytes, fetched as 16-byte
// vectors by D/8 lanes with 64-bit offsets, many tokens in flight per warp. Scores go to
// shared memory, the chunk's softmax is taken there, and P*V is accumulated in fp32. Each
// split writes its (max, sum, acc[D]) partial to the workspace; a second kernel merges the
// partials with a log-sum-exp rescale. When a launch has a single split the first kernel
// writes the output itself. Context lengths are only read on the device: no host sync.
#include <cuda_bf16.h>
#include <cuda_fp16.h>


#include "common.h"
#include "paged_attention.cuh"
#include "ptx.cuh"

namespace tllm {
namespace paged {

namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr float kLog2e = 1.4426950408889634f;

// Device error word of this file: a block-table entry outside [0, num_blocks) is clamped to
// block 0 (so no out-of-bounds read happens) and reported here.
__device__ int g_paged_status = 0;

__device__ __forceinline__ int64_t checked_block(const int32_t *bt, int64_t idx, int64_t nblocks) {
  int64_t phys = __ldg(bt + idx);
  if (static_cast<uint64_t>(phys) >= static_cast<uint64_t>(nblocks)) {
    atomicCAS(&g_paged_status, 0, TLLM_DEV_BAD_INDEX);
    phys = 0;
  }
  return phys;
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4 &raw, float (&v)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = Pack2<T>::unpack(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

template <typename T, int D, int U>
__global__ void __launch_bounds__(kThreads) paged_split_kernel(const Params p) {
  constexpr int TPT = D / 8;    // lanes per token (16 bytes each)
  constexpr int TPW = 32 / TPT; // tokens per warp step
  constexpr int STEP = kWarps * TPW;
  extern __shared__ float sm[];
  float *scores = sm;                          // [chunk]
  float *red = sm + p.chunk;                   // [kWarps * D]
  __shared__ float s_warp[kWarps];
  __shared__ float s_stat[2];

  const int split = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int sub = lane / TPT;
  const int dpart = (lane % TPT) * 8;

  int len = __ldg(p.context_lens + b);
  len = min(len, p.max_tokens);
  len = max(len, 0);
  const int t0 = split * p.chunk;
  if (split > 0 && t0 >= len) return;  // split 0 always runs so an empty context gives NaN
  const int n = min(len - t0, p.chunk) > 0 ? min(len - t0, p.chunk) : 0;

  // q slice, pre-scaled into the log2 domain in fp32.
  const T *qp = static_cast<const T *>(p.q) + b * p.sq0 + h * p.sq1;
  float qf[8];
  const float qscale = p.sm_scale * kLog2e;
#pragma unroll
  for (int i = 0; i < 8; ++i) qf[i] = to_f32<T>(qp[(dpart + i) * p.sq3]) * qscale;

  const int32_t *bt = p.block_tables + b * p.sbt0;
  const char *kbase = static_cast<const char *>(p.k_cache) + (h * p.skc2 + dpart) * sizeof(T);
  const char *vbase = static_cast<const char *>(p.v_cache) + (h * p.svc2 + dpart) * sizeof(T);

  // ---- scores = (q . k) * scale * log2(e) for the tokens of this split ----
  float wmax = -INFINITY;
  for (int base = warp * TPW; base < n; base += STEP * U) {
    uint4 kv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int tl = base + u * STEP + sub;
      if (tl < n) {
        const int t = t0 + tl;
        const int64_t phys = checked_block(bt, (t >> p.log2_bs) * p.sbt1, p.num_blocks);
        kv[u] = ldg_stream(kbase + (phys * p.skc0 + (t & (p.block_size - 1)) * p.skc1) * sizeof(T));
      } else {
        kv[u] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float kf[8];
      unpack8<T>(kv[u], kf);
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) s = fmaf(qf[i], kf[i], s);
#pragma unroll
      for (int off = TPT / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      const int tl = base + u * STEP + sub;
      if (tl < n) {
        wmax = fmaxf(wmax, s);
        if ((lane % TPT) == 0) scores[tl] = s;
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, off));
  if (lane == 0) s_warp[warp] = wmax;
  __syncthreads();
  float m = s_warp[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) m = fmaxf(m, s_warp[w]);
  __syncthreads();  // everyone has read s_warp before it is reused for the sums

  // ---- p = exp2(s - m), l = sum(p) ----
  float lsum = 0.f;
  for (int i = threadIdx.x; i < n; i += kThreads) {
    const float e = exp2f(scores[i] - m);
    scores[i] = e;
    lsum += e;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
  if (lane == 0) s_warp[warp] = lsum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) l += s_warp[w];
    s_stat[0] = m;
    s_stat[1] = l;
  }

  // ---- acc[d] = sum_t p_t * v_t[d] ----
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int base = warp * TPW; base < n; base += STEP * U) {
    uint4 vv[U];
    float pw[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int tl = base + u * STEP + sub;
      if (tl < n) {
        const int t = t0 + tl;
        const int64_t phys = checked_block(bt, (t >> p.log2_bs) * p.sbt1, p.num_blocks);
        vv[u] = ldg_stream(vbase + (phys * p.svc0 + (t & (p.block_size - 1)) * p.svc1) * sizeof(T));
        pw[u] = scores[tl];
      } else {
        vv[u] = make_uint4(0, 0, 0, 0);
        pw[u] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float vf[8];
      unpack8<T>(vv[u], vf);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(pw[u], vf[i], acc[i]);
    }
  }
  // Reduce over the token sub-slots of the warp (lanes sharing lane % TPT).
#pragma unroll
  for (int off = TPT; off < 32; off <<= 1) {
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], off);
  }
  if (sub == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) red[warp * D + dpart + i] = acc[i];
  }
  __syncthreads();
  const float mm = s_stat[0];
  const float ll = s_stat[1];
  for (int d = threadIdx.x; d < D; d += kThreads) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) a += red[w * D + d];
    if (p.num_splits == 1) {
      T *op = static_cast<T *>(p.o) + b * p.so0 + h * p.so1;
      op[d * p.so3] = from_f32<T>(a / ll);
    } else {
      const int64_t slot = (static_cast<int64_t>(b) * p.H + h) * p.num_splits + split;
      p.ws_acc[slot * D + d] = a;
      if (d == 0) {
        p.ws_ml[2 * slot] = mm;
        p.ws_ml[2 * slot + 1] = ll;
      }
    }
  }
}

// One CTA of D threads per (head, new token, sequence): log-sum-exp merge of the active splits.
template <typename T, int D>
__global__ void __launch_bounds__(D) paged_merge_kernel(const Params p) {
  const int hs = blockIdx.x;  // head * Sq + new token
  const int h = hs / p.Sq;
  const int tok = hs - h * p.Sq;
  const int b = blockIdx.y;
  const int d = threadIdx.x;
  int len = __ldg(p.context_lens + b);
  len = min(len, p.max_tokens);
  len = max(len, 0);
  const int active = len > 0 ? (len + p.chunk - 1) / p.chunk : 1;
  const int64_t slot0 = (static_cast<int64_t>(b) * p.H * p.Sq + hs) * p.num_splits;
  float M = -INFINITY;
  for (int s = 0; s < active; ++s) M = fmaxf(M, p.ws_ml[2 * (slot0 + s)]);
  float L = 0.f, A = 0.f;
  for (int s = 0; s < active; ++s) {
    const float wgt = exp2f(p.ws_ml[2 * (slot0 + s)] - M);
    L = fmaf(p.ws_ml[2 * (slot0 + s) + 1], wgt, L);
    A = fmaf(p.ws_acc[(slot0 + s) * D + d], wgt, A);
  }
  T *op = static_cast<T *>(p.o) + b * p.so0 + h * p.so1 + tok * p.so2;
  op[d * p.so3] = from_f32<T>(A / L);
}

template <typename T, int D>
int launch_typed(const Params &p, cudaStream_t st) {
  constexpr int U = D >= 64 ? 8 : 4;
  const size_t smem = static_cast<size_t>(p.chunk + kWarps * D) * sizeof(float);
  auto kern = paged_split_kernel<T, D, U>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(paged split)");
  }
  dim3 grid(p.num_splits, static_cast<unsigned>(p.H), static_cast<unsigned>(p.B));
  kern<<<grid, kThreads, smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "paged split launch");
  if (p.num_splits > 1) {
    dim3 mgrid(static_cast<unsigned>(p.H), static_cast<unsigned>(p.B));
    paged_merge_kernel<T, D><<<mgrid, D, 0, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e, "paged merge launch");
  }
  return TLLM_OK;
}

template <typename T>
int launch_dtype(const Params &p, cudaStream_t st) {
  switch (p.D) {
    case 16: return launch_typed<T, 16>(p, st);
    case 32: return launch_typed<T, 32>(p, st);
    case 64: return launch_typed<T, 64>(p, st);
    default: return launch_typed<T, 128>(p, st);
  }
}

}  // namespace

int read_status(int *out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_paged_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyFromSymbol(paged status)");
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_paged_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyToSymbol(paged status)");
  *out = v;
  return TLLM_OK;
}

Plan plan(int64_t B, int64_t H, int64_t D, int64_t block_size, int64_t max_blocks, int sms) {
  Plan pl;
  const int64_t max_tokens = max_blocks * block_size;
  pl.max_tokens = max_tokens;
  int64_t chunk = 512;
  auto ctas = [&](int64_t c) { return B * H * ((max_tokens + c - 1) / c); };
  if (max_tokens > 0) {
    // Enough CTAs to cover every SM several times over, but not an excessive number of
    // early-exit CTAs for long maximum lengths.
    while (chunk > 64 && ctas(chunk) < 4LL * (sms > 0 ? sms : 148)) chunk /= 2;
    while (chunk < 16384 && ctas(chunk) > (1LL << 20)) chunk *= 2;
  }
  if (chunk < block_size) chunk = block_size;
  pl.chunk = chunk;
  pl.num_splits = max_tokens > 0 ? (max_tokens + chunk - 1) / chunk : 1;
  if (pl.num_splits < 1) pl.num_splits = 1;
  if (pl.num_splits > 1) {
    pl.ws_ml_floats = B * H * pl.num_splits * 2;
    pl.ws_acc_floats = B * H * pl.num_splits * D;
  }
  // Both arrays start 256-byte aligned.
  const size_t ml_bytes = ((pl.ws_ml_floats * sizeof(float)) + 255) / 256 * 256;
  pl.ws_bytes = ml_bytes + pl.ws_acc_floats * sizeof(float);
  pl.ws_acc_offset = ml_bytes;
  return pl;
}

int validate(const Params &p) {
  TLLM_CHECK_ARG(p.B >= 0 && p.H >= 0, "paged_attention: negative dimension");
  TLLM_CHECK_ARG(p.D == 16 || p.D == 32 || p.D == 64 || p.D == 128,
                 "paged_attention: head dim %lld not in {16,32,64,128}", (long long)p.D);
  TLLM_CHECK_ARG(p.block_size == 16 || p.block_size == 32 || p.block_size == 64,
                 "paged_attention: block_size %d not in {16,32,64}", p.block_size);
  TLLM_CHECK_ARG(p.skc3 == 1 && p.svc3 == 1,
                 "paged_attention: the caches need a unit innermost stride");
  TLLM_CHECK_ARG(p.skc0 % 8 == 0 && p.skc1 % 8 == 0 && p.skc2 % 8 == 0 && p.svc0 % 8 == 0 &&
                     p.svc1 % 8 == 0 && p.svc2 % 8 == 0,
                 "paged_attention: cache strides must be multiples of 8 elements");
  TLLM_CHECK_ARG((reinterpret_cast<uintptr_t>(p.k_cache) & 15u) == 0 &&
                     (reinterpret_cast<uintptr_t>(p.v_cache) & 15u) == 0,
                 "paged_attention: caches must be 16-byte aligned");
  TLLM_CHECK_ARG(p.max_tokens < (1LL << 31), "paged_attention: max_blocks * block_size too large");
  return TLLM_OK;
}

int run(const Params &p, int dtype, cudaStream_t st) {
  if (dtype == TLLM_DTYPE_F16) return launch_dtype<__half>(p, st);
  return launch_dtype<__nv_bfloat16>(p, st);
}

namespace {
template <typename T>
int launch_merge(const Params &p, cudaStream_t st) {
  dim3 mgrid(static_cast<unsigned>(p.H * p.Sq), static_cast<unsigned>(p.B));
  switch (p.D) {
    case 16: paged_merge_kernel<T, 16><<<mgrid, 16, 0, st>>>(p); break;
    case 32: paged_merge_kernel<T, 32><<<mgrid, 32, 0, st>>>(p); break;
    case 64: paged_merge_kernel<T, 64><<<mgrid, 64, 0, st>>>(p); break;
    default: paged_merge_kernel<T, 128><<<mgrid, 128, 0, st>>>(p); break;
  }
  return cuda_status(cudaGetLastError(), "paged merge launch");
}
}  // namespace

int run_merge(const Params &p, int dtype, cudaStream_t st) {
  if (dtype == TLLM_DTYPE_F16) return launch_merge<__half>(p, st);
  return launch_merge<__nv_bfloat16>(p, st);
}

// ---------------------------------------------------------------------------------------
// Grouped-query decode: one CTA per (split, KV head, sequence) computes the G query heads
// that share the KV head, for Sq >= 1 new tokens, so every token's K and V rows cross HBM once
// for all of them.
//   Loads: the split's K tiles and then its V tiles stream through a ring of kGqaStages
//   8 KB tiles in shared memory with 16-byte cp.async copies (consecutive threads copy
//   consecutive 16-byte pieces of one token row; tokens past the context are zero-filled).
//   The copies hold no registers, so three tiles per CTA stay in flight, and the first
//   V tiles are already on their way while the split's softmax is taken.
//   Q.K and P.V: warp-level m16n8k16 MMAs with fp32 accumulation, the R = G * Sq query rows
//   (G heads times Sq new tokens, R <= 16) as the rows of A (q, exact in registers; p rounded
//   to the input type as in the flash kernels) and K / V read from the ring by ldmatrix. With
//   few useful rows the tensor cores do little useful work, but the loop then issues about a
//   quarter of the instructions of the same products on the CUDA cores, which were issue-bound
//   at half of HBM bandwidth. With several new tokens each row has its own causal key limit.
// ---------------------------------------------------------------------------------------
namespace {

constexpr int kGqaStages = 4;
constexpr int kGqaTileBytes = 8192;

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *src, int src_bytes) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// mma.sync m16n8k16 with fp32 accumulation. The warp-level MMA is used here to cut the
// instruction count of a memory-bound loop, not for tensor throughput; with at most 8 query
// rows the caller passes zero for the A registers of rows 8-15 (a1, a3).
template <typename T>
struct Mma16816;
template <>
struct Mma16816<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};
template <>
struct Mma16816<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                             uint32_t a3, uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void *p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a)
               : "memory");
}

// Byte offset of 16-byte chunk c of token row r inside a tile: rows of 2*D bytes, chunks
// XOR-swizzled by the row's low three bits so that the eight rows one ldmatrix reads at the
// same logical chunk fall into eight different bank groups.
template <int D>
__device__ __forceinline__ int tile_off(int r, int c) {
  return r * (2 * D) + ((c ^ (r & 7)) << 4);
}

// Number of the split's keys (local index < the result) that query row r may see: all n with
// causal off; with causal on, query token s of Sq sits at position len - Sq + s and sees the
// keys at positions <= its own.
__device__ __forceinline__ int row_key_limit(const Params &p, int r, int len, int t0, int n) {
  if (!p.causal) return n;
  const int s = r % p.Sq;
  return min(max(len - p.Sq + s + 1 - t0, 0), n);
}

// R = G * Sq query rows (row r = g * Sq + s: query head hk * G + g, new token s); kR16: rows 8-15
// are in use.
template <typename T, int D, bool kR16>
__global__ void __launch_bounds__(kThreads, 4) paged_gqa_split_kernel(const Params p) {
  constexpr int NV = D / 8;                      // 16-byte chunks per token row
  constexpr int TT = kGqaTileBytes / (2 * D);    // tokens per tile: 32 (D 128) or 64 (D 64)
  constexpr int TILE_VEC = TT * NV;
  constexpr int CPT = TILE_VEC / kThreads;       // copies per thread per tile
  constexpr int KS = D / 16;                     // k-steps of Q.K
  constexpr int QK_NT = TT / (8 * kWarps);       // 8-token n-tiles per warp in Q.K
  constexpr int PV_NT = D / (8 * kWarps);        // 8-column n-tiles per warp in P.V
  constexpr int PV_KS = TT / 16;                 // k-steps of P.V per tile
  static_assert(TILE_VEC % kThreads == 0 && NV >= 8, "tile shape");
  static_assert(QK_NT >= 1 && KS % 2 == 0 && PV_NT % 2 == 0, "fragment shape");
  constexpr int TPR = kR16 ? 8 : 16;             // softmax threads per query row
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char *ring = smem;                                                        // [S][TT][2D]
  // Scores [R][SST]: rows padded by TPR floats, so the TPR-thread groups of the softmax that
  // share a warp read different banks.
  const int SST = p.chunk + TPR;
  float *scores = reinterpret_cast<float *>(smem + kGqaStages * kGqaTileBytes);
  const int R = p.G * p.Sq;
  // Byte offsets within the caches: [0] K, [1] V; per block of the split and per row of a block.
  int64_t *s_boff = reinterpret_cast<int64_t *>(scores + R * SST);                 // [2][chunk / 16]
  int64_t *s_roff = s_boff + 2 * (p.chunk / 16);                                    // [2][block_size]
  __shared__ float s_part[16][kWarps];
  __shared__ float s_m[16], s_l[16];
  __shared__ int s_lim[16];

  const int split = blockIdx.x;
  const int hk = blockIdx.y;
  const int b = blockIdx.z;
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int r0 = lane >> 2;  // fragment rows of this lane: r0 and r0 + 8
  const int r1 = r0 + 8;
  const int cq = lane & 3;
  const bool ok0 = r0 < R;
  const bool ok1 = kR16 && r1 < R;

  int len = __ldg(p.context_lens + b);
  len = min(len, p.max_tokens);
  len = max(len, 0);
  const int t0 = split * p.chunk;
  if (split > 0 && t0 >= len) return;  // split 0 always runs so an empty context gives NaN
  const int n = min(len - t0, p.chunk) > 0 ? min(len - t0, p.chunk) : 0;

  // The split's blocks (the chunk is a multiple of the block size) and the rows of a block.
  const int nblk = (n + p.block_size - 1) >> p.log2_bs;
  const int nbs = p.chunk / 16;
  const int32_t *bt = p.block_tables + b * p.sbt0;
  const int64_t kv_off = hk * p.skc2 * static_cast<int64_t>(sizeof(T));
  const int64_t vv_off = hk * p.svc2 * static_cast<int64_t>(sizeof(T));
  for (int i = tid; i < nblk; i += kThreads) {
    const int64_t phys = checked_block(bt, ((t0 >> p.log2_bs) + i) * p.sbt1, p.num_blocks);
    s_boff[i] = phys * p.skc0 * static_cast<int64_t>(sizeof(T)) + kv_off;
    s_boff[nbs + i] = phys * p.svc0 * static_cast<int64_t>(sizeof(T)) + vv_off;
  }
  for (int i = tid; i < p.block_size; i += kThreads) {
    s_roff[i] = i * p.skc1 * static_cast<int64_t>(sizeof(T));
    s_roff[p.block_size + i] = i * p.svc1 * static_cast<int64_t>(sizeof(T));
  }
  if (tid < R) s_lim[tid] = row_key_limit(p, tid, len, t0, n);

  // A fragments of q (the raw input elements; the scale is applied to the fp32 scores):
  // qa[ks][0] = a0 (row r0), [1] = a2 (row r0, upper 8 columns), [2] = a1 (row r1), [3] = a3.
  uint32_t qa[KS][kR16 ? 4 : 2];
  {
    auto qrow = [&](int r) {
      return static_cast<const uint16_t *>(p.q) + b * p.sq0 + (hk * p.G + r / p.Sq) * p.sq1 +
             (r % p.Sq) * p.sq2;
    };
    const uint16_t *q0 = qrow(ok0 ? r0 : 0);
    const uint16_t *q1 = qrow(ok1 ? r1 : 0);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int d0 = 16 * ks + 8 * h + 2 * cq;
        qa[ks][h] = ok0 ? (static_cast<uint32_t>(q0[d0 * p.sq3]) |
                           (static_cast<uint32_t>(q0[(d0 + 1) * p.sq3]) << 16))
                        : 0u;
        if constexpr (kR16)
          qa[ks][2 + h] = ok1 ? (static_cast<uint32_t>(q1[d0 * p.sq3]) |
                                 (static_cast<uint32_t>(q1[(d0 + 1) * p.sq3]) << 16))
                              : 0u;
      }
  }
  __syncthreads();
  const int lim0 = ok0 ? s_lim[r0] : 0;
  const int lim1 = ok1 ? s_lim[r1] : 0;

  const int nt = (n + TT - 1) / TT;
  const int total = 2 * nt;  // K tiles, then V tiles
  // This thread copies chunk c of rows tid / NV + i * (kThreads / NV) of every tile, to fixed
  // places in the tile.
  const int c = tid % NV;
  const char *ksrc = static_cast<const char *>(p.k_cache) + c * 16;
  const char *vsrc = static_cast<const char *>(p.v_cache) + c * 16;

  auto issue = [&](int j) {
    if (j < total) {
      const int isv = j >= nt;
      const int tb = (isv ? j - nt : j) * TT;
      const int64_t *boff = s_boff + isv * nbs;
      const int64_t *roff = s_roff + isv * p.block_size;
      const char *base = isv ? vsrc : ksrc;
      unsigned char *dst = ring + (j % kGqaStages) * kGqaTileBytes;
#pragma unroll
      for (int i = 0; i < CPT; ++i) {
        const int row = tid / NV + i * (kThreads / NV);
        const int tl = tb + row;
        const char *src = base;
        int bytes = 0;
        if (tl < n) {
          src = base + boff[tl >> p.log2_bs] + roff[tl & (p.block_size - 1)];
          bytes = 16;
        }
        cp_async16(dst + tile_off<D>(row, c), src, bytes);
      }
    }
    cp_async_commit();  // empty groups past the end keep the group count uniform
  };

#pragma unroll
  for (int j = 0; j < kGqaStages - 1; ++j) issue(j);

  // ---- scores: S[row][token] = q . k on the tensor cores, one 8-token n-tile per warp step ----
  const float qscale = p.sm_scale * kLog2e;
  float mloc0 = -INFINITY, mloc1 = -INFINITY;
  for (int j = 0; j < nt; ++j) {
    cp_async_wait<kGqaStages - 2>();
    __syncthreads();  // tile j landed for every thread; tile j - 1's slot is free
    issue(j + kGqaStages - 1);
    const unsigned char *tile = ring + (j % kGqaStages) * kGqaTileBytes;
#pragma unroll
    for (int q = 0; q < QK_NT; ++q) {
      const int tok0 = (warp * QK_NT + q) * 8;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kp = 0; kp < KS / 2; ++kp) {
        uint32_t bf[4];
        const int row = tok0 + (lane & 7);
        ldsm_x4(bf, tile + tile_off<D>(row, 4 * kp + (lane >> 3)));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int ks = 2 * kp + h;
          if constexpr (kR16)
            Mma16816<T>::run(acc, qa[ks][0], qa[ks][2], qa[ks][1], qa[ks][3], bf[2 * h], bf[2 * h + 1]);
          else
            Mma16816<T>::run(acc, qa[ks][0], 0u, qa[ks][1], 0u, bf[2 * h], bf[2 * h + 1]);
        }
      }
      const int tl = j * TT + tok0 + 2 * cq;
      if (ok0) {
        const float s0 = acc[0] * qscale, s1 = acc[1] * qscale;
        if (tl < lim0) mloc0 = fmaxf(mloc0, s0);
        if (tl + 1 < lim0) mloc0 = fmaxf(mloc0, s1);
        *reinterpret_cast<float2 *>(scores + r0 * SST + tl) = make_float2(s0, s1);
      }
      if (ok1) {
        const float s0 = acc[2] * qscale, s1 = acc[3] * qscale;
        if (tl < lim1) mloc1 = fmaxf(mloc1, s0);
        if (tl + 1 < lim1) mloc1 = fmaxf(mloc1, s1);
        *reinterpret_cast<float2 *>(scores + r1 * SST + tl) = make_float2(s0, s1);
      }
    }
  }

  // ---- softmax over the split's scores, per row: max, p = exp2(s - max) in place (0 past the
  // row's last visible key, up to the last tile's end), sum. A row that sees no key has sum 0,
  // so its output is NaN as in the reference. ----
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    mloc0 = fmaxf(mloc0, __shfl_xor_sync(0xffffffffu, mloc0, off));
    mloc1 = fmaxf(mloc1, __shfl_xor_sync(0xffffffffu, mloc1, off));
  }
  if (cq == 0) {
    if (ok0) s_part[r0][warp] = mloc0;
    if (ok1) s_part[r1][warp] = mloc1;
  }
  __syncthreads();
  if (tid < R) {
    float mm = s_part[tid][0];
#pragma unroll
    for (int w = 1; w < kWarps; ++w) mm = fmaxf(mm, s_part[tid][w]);
    s_m[tid] = mm;
  }
  __syncthreads();
  {
    // TPR consecutive threads per row (all rows at once).
    const int r = tid / TPR, sub = tid % TPR;
    const int npad = nt * TT;
    float l = 0.f;
    if (r < R) {
      const float mr = s_m[r];
      const int lim = s_lim[r];
      float *row = scores + r * SST;
      for (int i = sub; i < npad; i += TPR) {
        const float e = i < lim ? exp2f(row[i] - mr) : 0.f;
        row[i] = e;
        l += e;
      }
    }
#pragma unroll
    for (int off = TPR / 2; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
    if (r < R && sub == 0) s_l[r] = l;
  }

  // ---- O[row][d] += P . V on the tensor cores; each warp owns D/4 output columns ----
  float acc[PV_NT][4];
#pragma unroll
  for (int q = 0; q < PV_NT; ++q)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[q][i] = 0.f;
  for (int j = nt; j < total; ++j) {
    cp_async_wait<kGqaStages - 2>();
    __syncthreads();
    issue(j + kGqaStages - 1);
    const unsigned char *tile = ring + (j % kGqaStages) * kGqaTileBytes;
    const int tb = (j - nt) * TT + 2 * cq;
#pragma unroll
    for (int ks = 0; ks < PV_KS; ++ks) {
      uint32_t pa0 = 0u, pa1 = 0u, pa2 = 0u, pa3 = 0u;
      if (ok0) {
        const float *pr = scores + r0 * SST + tb + 16 * ks;
        const float2 x = *reinterpret_cast<const float2 *>(pr);
        const float2 y = *reinterpret_cast<const float2 *>(pr + 8);
        pa0 = Pack2<T>::pack(x.x, x.y);
        pa2 = Pack2<T>::pack(y.x, y.y);
      }
      if (ok1) {
        const float *pr = scores + r1 * SST + tb + 16 * ks;
        const float2 x = *reinterpret_cast<const float2 *>(pr);
        const float2 y = *reinterpret_cast<const float2 *>(pr + 8);
        pa1 = Pack2<T>::pack(x.x, x.y);
        pa3 = Pack2<T>::pack(y.x, y.y);
      }
      const int row = 16 * ks + 8 * ((lane >> 3) & 1) + (lane & 7);
#pragma unroll
      for (int np = 0; np < PV_NT / 2; ++np) {
        uint32_t bf[4];
        ldsm_x4_trans(bf, tile + tile_off<D>(row, warp * PV_NT + 2 * np + (lane >> 4)));
        Mma16816<T>::run(acc[2 * np], pa0, pa1, pa2, pa3, bf[0], bf[1]);
        Mma16816<T>::run(acc[2 * np + 1], pa0, pa1, pa2, pa3, bf[2], bf[3]);
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // s_l is visible (also with no tiles)

#pragma unroll
  for (int half = 0; half < (kR16 ? 2 : 1); ++half) {
    const int r = half ? r1 : r0;
    if (half ? !ok1 : !ok0) continue;
    const int g = r / p.Sq, s = r % p.Sq;
    const int h = hk * p.G + g;
    const float inv_l = 1.f / s_l[r];
    const int64_t slot = ((static_cast<int64_t>(b) * p.H + h) * p.Sq + s) * p.num_splits + split;
#pragma unroll
    for (int q = 0; q < PV_NT; ++q) {
      const int d = (warp * PV_NT + q) * 8 + 2 * cq;
      const float v0 = acc[q][2 * half], v1 = acc[q][2 * half + 1];
      if (p.num_splits == 1) {
        T *op = static_cast<T *>(p.o) + b * p.so0 + h * p.so1 + s * p.so2;
        op[d * p.so3] = from_f32<T>(v0 * inv_l);
        op[(d + 1) * p.so3] = from_f32<T>(v1 * inv_l);
      } else {
        *reinterpret_cast<float2 *>(p.ws_acc + slot * D + d) = make_float2(v0, v1);
      }
    }
    if (p.num_splits > 1 && warp == 0 && cq == 0) {
      p.ws_ml[2 * slot] = s_m[r];
      p.ws_ml[2 * slot + 1] = s_l[r];
    }
  }
}

// Ring, scores of the R query rows, and the K and V byte offsets of the split's blocks (block
// size >= 16) and of the rows of a block (block size <= 64).
size_t gqa_smem_bytes(int64_t R, int64_t chunk) {
  const int64_t tpr = R > 8 ? 8 : 16;
  return static_cast<size_t>(kGqaStages) * kGqaTileBytes +
         static_cast<size_t>(R * (chunk + tpr)) * sizeof(float) +
         static_cast<size_t>(2 * (chunk / 16) + 2 * 64) * sizeof(int64_t);
}

template <typename T, int D, bool kR16>
int launch_gqa_typed(const Params &p, cudaStream_t st) {
  const size_t smem = gqa_smem_bytes(static_cast<int64_t>(p.G) * p.Sq, p.chunk);
  auto kern = paged_gqa_split_kernel<T, D, kR16>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(paged gqa split)");
  }
  dim3 grid(p.num_splits, static_cast<unsigned>(p.Hkv), static_cast<unsigned>(p.B));
  kern<<<grid, kThreads, smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e, "paged gqa split launch");
  if (p.num_splits > 1) return launch_merge<T>(p, st);
  return TLLM_OK;
}

template <typename T, int D>
int launch_gqa_d(const Params &p, cudaStream_t st) {
  if (p.G * p.Sq > 8) return launch_gqa_typed<T, D, true>(p, st);
  return launch_gqa_typed<T, D, false>(p, st);
}

}  // namespace

Plan plan_gqa(int64_t B, int64_t H, int64_t Hkv, int64_t Sq, int64_t D, int64_t block_size,
              int64_t max_blocks, int sms) {
  Plan pl = plan(B, Hkv, D, block_size, max_blocks, sms);
  if (pl.num_splits > 1) {
    pl.ws_ml_floats = B * H * Sq * pl.num_splits * 2;
    pl.ws_acc_floats = B * H * Sq * pl.num_splits * D;
  }
  const size_t ml_bytes = ((pl.ws_ml_floats * sizeof(float)) + 255) / 256 * 256;
  pl.ws_bytes = ml_bytes + pl.ws_acc_floats * sizeof(float);
  pl.ws_acc_offset = ml_bytes;
  return pl;
}

bool gqa_supported(int64_t G, int64_t Sq, int64_t D, const Plan &pl) {
  return G >= 1 && Sq >= 1 && G * Sq <= 16 && (D == 64 || D == 128) &&
         gqa_smem_bytes(G * Sq, pl.chunk) <= 200 * 1024;
}

int run_gqa(const Params &p, int dtype, cudaStream_t st) {
  if (dtype == TLLM_DTYPE_F16)
    return p.D == 64 ? launch_gqa_d<__half, 64>(p, st) : launch_gqa_d<__half, 128>(p, st);
  return p.D == 64 ? launch_gqa_d<__nv_bfloat16, 64>(p, st) : launch_gqa_d<__nv_bfloat16, 128>(p, st);
}

}  // namespace paged
}  // namespace tllm

using tllm::paged::Params;
using tllm::paged::Plan;

extern "C" size_t tllm_paged_attn_workspace_size(int64_t B, int64_t H, int64_t D,
                                                 int64_t block_size, int64_t max_blocks) {
  if (B <= 0 || H <= 0 || D <= 0 || block_size <= 0 || max_blocks <= 0) return 0;
  return tllm::paged::plan(B, H, D, block_size, max_blocks, tllm::sm_count()).ws_bytes;
}

extern "C" int tllm_paged_attn_decode(const void *q, const void *k_cache, const void *v_cache,
                                      const int32_t *block_tables, const int32_t *context_lens,
                                      void *o, void *workspace, size_t workspace_bytes,
                                      int64_t B, int64_t H, int64_t D, int64_t block_size,
                                      int64_t max_blocks, int64_t num_blocks,
                                      const int64_t *sq, const int64_t *skc, const int64_t *svc,
                                      const int64_t *sbt, const int64_t *so, float sm_scale,
                                      int dtype, void *stream) {
  using namespace tllm;
  clear_error();
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16,
                 "paged_attention: unsupported dtype %d", dtype);
  TLLM_CHECK_ARG(sq && skc && svc && sbt && so, "paged_attention: null stride array");
  TLLM_CHECK_ARG(max_blocks >= 0 && num_blocks >= 0, "paged_attention: negative table size");
  if (B == 0 || H == 0) return TLLM_OK;
  TLLM_CHECK_ARG(q && k_cache && v_cache && block_tables && context_lens && o,
                 "paged_attention: null tensor pointer");
  TLLM_CHECK_ARG(max_blocks >= 1, "paged_attention: block_tables has no columns");
  TLLM_CHECK_ARG(num_blocks >= 1, "paged_attention: the caches hold no blocks");
  const Plan pl = paged::plan(B, H, D, block_size, max_blocks, sm_count());
  Params p{};
  p.q = q; p.k_cache = k_cache; p.v_cache = v_cache;
  p.block_tables = block_tables; p.context_lens = context_lens; p.o = o;
  p.B = B; p.H = H; p.D = D;
  p.num_blocks = num_blocks;
  p.block_size = static_cast<int>(block_size);
  p.log2_bs = block_size == 16 ? 4 : (block_size == 32 ? 5 : 6);
  p.max_tokens = static_cast<int>(pl.max_tokens < (1LL << 31) ? pl.max_tokens : 0);
  p.chunk = static_cast<int>(pl.chunk);
  p.num_splits = static_cast<int>(pl.num_splits);
  p.sq0 = sq[0]; p.sq1 = sq[1]; p.sq3 = sq[3];
  p.skc0 = skc[0]; p.skc1 = skc[1]; p.skc2 = skc[2]; p.skc3 = skc[3];
  p.svc0 = svc[0]; p.svc1 = svc[1]; p.svc2 = svc[2]; p.svc3 = svc[3];
  p.sbt0 = sbt[0]; p.sbt1 = sbt[1];
  p.so0 = so[0]; p.so1 = so[1]; p.so3 = so[3];
  p.sm_scale = sm_scale;
  int rc = paged::validate(p);
  if (rc) return rc;
  TLLM_CHECK_ARG(pl.max_tokens < (1LL << 31), "paged_attention: max_blocks * block_size too large");
  if (pl.num_splits > 1) {
    if (!workspace || workspace_bytes < pl.ws_bytes)
      return fail(TLLM_ERR_WORKSPACE, "paged_attention: workspace of %zu bytes needed, %zu given",
                  pl.ws_bytes, workspace_bytes);
    TLLM_CHECK_ARG((reinterpret_cast<uintptr_t>(workspace) & 255u) == 0,
                   "paged_attention: workspace must be 256-byte aligned");
    p.ws_ml = static_cast<float *>(workspace);
    p.ws_acc = reinterpret_cast<float *>(static_cast<char *>(workspace) + pl.ws_acc_offset);
  }
  return paged::run(p, dtype, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------------------
// Allocation-free variant of the decode entry point.
//
// Some callers cannot hand this library a device workspace: engines that reserve all device
// memory once at start-up and treat any later cudaMalloc as a fault (cudaMalloc can stall the
// whole device and fragments a pre-planned pool), and foreign-language hosts that reach the
// library through its C ABI with no device allocator of their own. For them the split-KV
// partials live in the fixed array below instead of a caller-provided workspace. Every GPU
// that loads this library keeps the array (TLLM_PAGED_NOALLOC_SCRATCH_BYTES) until the
// process exits.
// ---------------------------------------------------------------------------------------
namespace tllm {
namespace paged {
namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[TLLM_PAGED_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on the current device. In host code the symbol name
// only stands in for the device array, so the address is looked up with the device current.
// It is looked up on every call rather than cached: a cached address would go stale after
// cudaDeviceReset() gives the device a new context, and the lookup costs well under a
// microsecond once the module is loaded (the first call on a device loads it).
int noalloc_scratch(void **out) {
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(paged no-alloc scratch)");
  *out = p;
  return TLLM_OK;
}

}  // namespace
}  // namespace paged
}  // namespace tllm

extern "C" int tllm_paged_attn_decode_noalloc(const void *q, const void *k_cache,
                                              const void *v_cache, const int32_t *block_tables,
                                              const int32_t *context_lens, void *o, int64_t B,
                                              int64_t H, int64_t D, int64_t block_size,
                                              int64_t max_blocks, int64_t num_blocks,
                                              const int64_t *sq, const int64_t *skc,
                                              const int64_t *svc, const int64_t *sbt,
                                              const int64_t *so, float sm_scale, int dtype,
                                              void *stream) {
  using namespace tllm;
  clear_error();
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16,
                 "paged_attention_noalloc: unsupported dtype %d", dtype);
  TLLM_CHECK_ARG(sq && skc && svc && sbt && so, "paged_attention_noalloc: null stride array");
  TLLM_CHECK_ARG(max_blocks >= 0 && num_blocks >= 0, "paged_attention_noalloc: negative table size");
  // Dimensions are checked before the scratch size is planned from them: a negative B or H
  // would otherwise wrap the size around and be reported as a scratch overflow.
  TLLM_CHECK_ARG(B >= 0 && H >= 0, "paged_attention_noalloc: negative dimension");
  TLLM_CHECK_ARG(D == 16 || D == 32 || D == 64 || D == 128,
                 "paged_attention_noalloc: head dim %lld not in {16,32,64,128}", (long long)D);
  TLLM_CHECK_ARG(block_size == 16 || block_size == 32 || block_size == 64,
                 "paged_attention_noalloc: block_size %lld not in {16,32,64}",
                 (long long)block_size);
  if (B == 0 || H == 0) return TLLM_OK;
  TLLM_CHECK_ARG(q && k_cache && v_cache && block_tables && context_lens && o,
                 "paged_attention_noalloc: null tensor pointer");
  TLLM_CHECK_ARG(max_blocks >= 1, "paged_attention_noalloc: block_tables has no columns");
  TLLM_CHECK_ARG(num_blocks >= 1, "paged_attention_noalloc: the caches hold no blocks");
  TLLM_CHECK_ARG(max_blocks * block_size < (1LL << 31),
                 "paged_attention_noalloc: max_blocks * block_size too large");
  const Plan pl = paged::plan(B, H, D, block_size, max_blocks, sm_count());
  if (pl.ws_bytes > TLLM_PAGED_NOALLOC_SCRATCH_BYTES)
    return fail(TLLM_ERR_WORKSPACE,
                "paged_attention_noalloc: this problem needs %zu bytes of split-KV scratch, more "
                "than the library's fixed %zu-byte array; use tllm_paged_attn_decode with a "
                "caller-provided workspace",
                pl.ws_bytes, static_cast<size_t>(TLLM_PAGED_NOALLOC_SCRATCH_BYTES));
  Params p{};
  p.q = q; p.k_cache = k_cache; p.v_cache = v_cache;
  p.block_tables = block_tables; p.context_lens = context_lens; p.o = o;
  p.B = B; p.H = H; p.D = D;
  p.num_blocks = num_blocks;
  p.block_size = static_cast<int>(block_size);
  p.log2_bs = block_size == 16 ? 4 : (block_size == 32 ? 5 : 6);
  p.max_tokens = static_cast<int>(pl.max_tokens);
  p.chunk = static_cast<int>(pl.chunk);
  p.num_splits = static_cast<int>(pl.num_splits);
  p.sq0 = sq[0]; p.sq1 = sq[1]; p.sq3 = sq[3];
  p.skc0 = skc[0]; p.skc1 = skc[1]; p.skc2 = skc[2]; p.skc3 = skc[3];
  p.svc0 = svc[0]; p.svc1 = svc[1]; p.svc2 = svc[2]; p.svc3 = svc[3];
  p.sbt0 = sbt[0]; p.sbt1 = sbt[1];
  p.so0 = so[0]; p.so1 = so[1]; p.so3 = so[3];
  p.sm_scale = sm_scale;
  int rc = paged::validate(p);
  if (rc) return rc;
  if (pl.num_splits > 1) {
    // Every partial slot the merge kernel reads is written earlier in this same call, so the
    // array needs no clearing between calls.
    void *scratch = nullptr;
    rc = paged::noalloc_scratch(&scratch);
    if (rc) return rc;
    p.ws_ml = static_cast<float *>(scratch);
    p.ws_acc = reinterpret_cast<float *>(static_cast<char *>(scratch) + pl.ws_acc_offset);
  }
  return paged::run(p, dtype, static_cast<cudaStream_t>(stream));
}
