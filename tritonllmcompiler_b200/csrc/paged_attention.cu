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

// One CTA of D threads per (head, sequence): log-sum-exp merge of the active splits.
template <typename T, int D>
__global__ void __launch_bounds__(D) paged_merge_kernel(const Params p) {
  const int h = blockIdx.x;
  const int b = blockIdx.y;
  const int d = threadIdx.x;
  int len = __ldg(p.context_lens + b);
  len = min(len, p.max_tokens);
  len = max(len, 0);
  const int active = len > 0 ? (len + p.chunk - 1) / p.chunk : 1;
  const int64_t slot0 = (static_cast<int64_t>(b) * p.H + h) * p.num_splits;
  float M = -INFINITY;
  for (int s = 0; s < active; ++s) M = fmaxf(M, p.ws_ml[2 * (slot0 + s)]);
  float L = 0.f, A = 0.f;
  for (int s = 0; s < active; ++s) {
    const float wgt = exp2f(p.ws_ml[2 * (slot0 + s)] - M);
    L = fmaf(p.ws_ml[2 * (slot0 + s) + 1], wgt, L);
    A = fmaf(p.ws_acc[(slot0 + s) * D + d], wgt, A);
  }
  T *op = static_cast<T *>(p.o) + b * p.so0 + h * p.so1;
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
