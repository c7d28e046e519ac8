// Appending new tokens to the paged KV cache, with the K-side RMSNorm + RoPE fused in.
//
// The reference decodes from a paged cache (python/triton_llm/ops/paged_attention.py) but
// has no operator that fills it. The cache layout is the reference's
// (python/triton_llm/reference/paged_attention.py:29-37): token t of sequence b lives at
// cache[block_tables[b, t // block_size], t % block_size, h, :]. Appending token t of the
// new tokens of sequence b writes position start_pos[b] + t.
//
// B200 design: a pure HBM stream (read the new K/V rows once, write them once), with the
// thread layout of the rmsnorm_rope vector kernel: D / 16 lanes per (token, head) row, each
// owning one 16-byte vector of each half of D, R heads of one token per lane group. With the
// RoPE variant the K row goes through the same norm_rope_vec arithmetic as the plain operator
// (so the cache holds exactly what rmsnorm_rope would return), with the cos/sin row at the
// token's absolute position. A position outside the block table or the RoPE table, or a
// block-table entry outside the pool, is skipped and reported in the device status word.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.h"
#include "ptx.cuh"
#include "rmsnorm_rope.cuh"

namespace tllm {

__device__ int g_pkv_status = 0;

int pkv_read_status(int *out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_pkv_status, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyFromSymbol(paged kv status)");
  const int zero = 0;
  e = cudaMemcpyToSymbol(g_pkv_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpyToSymbol(paged kv status)");
  *out = v;
  return TLLM_OK;
}

namespace pkv {
namespace {

using namespace rr;

struct Geom {
  const int32_t *block_tables;
  const int32_t *start_pos;
  const int32_t *n_new;  // may be null: every one of the T tokens is appended
  int64_t T, H;
  int64_t max_blocks, num_blocks;
  int block_size;
  int64_t rope_rows;
  int64_t skn0, skn1, skn2;  // k_new [B, T, H, D]
  int64_t svn0, svn1, svn2;  // v_new
  int64_t skc0, skc1, skc2;  // k_cache [num_blocks, block_size, H, D]
  int64_t svc0, svc1, svc2;  // v_cache
  int64_t sbt0, sbt1;
  int64_t scos, ssin;
  float eps;
};

// Lane groups of TPR = D / 16 lanes; group gi covers heads [R * (gi % (H / R)), ... + R) of
// token (b, t) = divmod(gi / (H / R), T).
template <typename T, int D, int R, bool kRope>
__global__ void __launch_bounds__(256, 2) paged_append_kernel(
    const T *__restrict__ k_new, const T *__restrict__ v_new, T *__restrict__ k_cache,
    T *__restrict__ v_cache, const T *__restrict__ w, const T *__restrict__ cosb,
    const T *__restrict__ sinb, int64_t groups, Geom g) {
  constexpr int TPR = D / 16;
  constexpr int HALF = D / 2;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t gi_raw = tid / TPR;
  // The TPR lanes of a group sit in one warp; a group past the end recomputes the last
  // group (the RoPE path shuffles inside the group) and writes nothing.
  bool ok = gi_raw < groups;
  const int64_t gi = ok ? gi_raw : groups - 1;
  const int c = static_cast<int>(tid % TPR) * 8;
  const int64_t hg = g.H / R;
  const int64_t h0 = (gi % hg) * R;
  const int64_t bt_idx = gi / hg;
  const int64_t t = bt_idx % g.T;
  const int64_t b = bt_idx / g.T;

  if (g.n_new && t >= __ldg(g.n_new + b)) ok = false;
  const int64_t pos = static_cast<int64_t>(__ldg(g.start_pos + b)) + t;
  const int64_t blk = pos >= 0 ? pos / g.block_size : -1;
  int64_t phys = 0;
  bool in_range = blk >= 0 && blk < g.max_blocks && (!kRope || pos < g.rope_rows);
  if (in_range) {
    phys = __ldg(g.block_tables + b * g.sbt0 + blk * g.sbt1);
    in_range = phys >= 0 && phys < g.num_blocks;
  }
  if (ok && !in_range) atomicCAS(&g_pkv_status, 0, TLLM_DEV_BAD_INDEX);
  ok = ok && in_range;
  const int64_t off = pos - blk * g.block_size;

  const T *kr = k_new + b * g.skn0 + t * g.skn1 + h0 * g.skn2;
  const T *vr = v_new + b * g.svn0 + t * g.svn1 + h0 * g.svn2;
  uint4 k1[R], k2[R], v1[R], v2[R];
#pragma unroll
  for (int u = 0; u < R; ++u) {
    k1[u] = ld_stream(kr + u * g.skn2 + c);
    k2[u] = ld_stream(kr + u * g.skn2 + HALF + c);
    v1[u] = ld_stream(vr + u * g.svn2 + c);
    v2[u] = ld_stream(vr + u * g.svn2 + HALF + c);
  }
  T *kc = k_cache + phys * g.skc0 + off * g.skc1 + h0 * g.skc2;
  T *vc = v_cache + phys * g.svc0 + off * g.svc1 + h0 * g.svc2;
  if constexpr (kRope) {
    const int64_t prow = ok ? pos : 0;
    float w1[8], w2[8], c1[8], c2[8], s1[8], s2[8];
    load8<T>(w + c, w1);
    load8<T>(w + HALF + c, w2);
    load8<T>(cosb + prow * g.scos + c, c1);
    load8<T>(cosb + prow * g.scos + HALF + c, c2);
    load8<T>(sinb + prow * g.ssin + c, s1);
    load8<T>(sinb + prow * g.ssin + HALF + c, s2);
#pragma unroll
    for (int u = 0; u < R; ++u) {
      uint4 o1, o2;
      norm_rope_vec<T, D>(k1[u], k2[u], w1, w2, c1, c2, s1, s2, g.eps, o1, o2);
      k1[u] = o1;
      k2[u] = o2;
    }
  }
  if (ok) {
#pragma unroll
    for (int u = 0; u < R; ++u) {
      st_stream(kc + u * g.skc2 + c, k1[u]);
      st_stream(kc + u * g.skc2 + HALF + c, k2[u]);
      st_stream(vc + u * g.svc2 + c, v1[u]);
      st_stream(vc + u * g.svc2 + HALF + c, v2[u]);
    }
  }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T, int D, bool kRope>
int launch_d(const void *kn, const void *vn, void *kc, void *vc, const void *w, const void *cs,
             const void *sn, int64_t rows, const Geom &g, cudaStream_t st) {
  // Heads per lane group: up to 4, enough bytes in flight per lane for the HBM stream.
  const int R = g.H % 4 == 0 ? 4 : (g.H % 2 == 0 ? 2 : 1);
  const int64_t groups = rows / R;
  const int64_t threads = groups * (D / 16);
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
  const T *knp = static_cast<const T *>(kn);
  const T *vnp = static_cast<const T *>(vn);
  T *kcp = static_cast<T *>(kc);
  T *vcp = static_cast<T *>(vc);
  const T *wp = static_cast<const T *>(w);
  const T *cp = static_cast<const T *>(cs);
  const T *sp = static_cast<const T *>(sn);
  if (R == 4)
    paged_append_kernel<T, D, 4, kRope><<<grid, 256, 0, st>>>(knp, vnp, kcp, vcp, wp, cp, sp, groups, g);
  else if (R == 2)
    paged_append_kernel<T, D, 2, kRope><<<grid, 256, 0, st>>>(knp, vnp, kcp, vcp, wp, cp, sp, groups, g);
  else
    paged_append_kernel<T, D, 1, kRope><<<grid, 256, 0, st>>>(knp, vnp, kcp, vcp, wp, cp, sp, groups, g);
  return cuda_status(cudaGetLastError(), kRope ? "paged append+rope launch" : "paged append launch");
}

template <typename T, bool kRope>
int launch(const void *kn, const void *vn, void *kc, void *vc, const void *w, const void *cs,
           const void *sn, int64_t rows, int64_t D, const Geom &g, cudaStream_t st) {
  switch (D) {
    case 16: return launch_d<T, 16, kRope>(kn, vn, kc, vc, w, cs, sn, rows, g, st);
    case 32: return launch_d<T, 32, kRope>(kn, vn, kc, vc, w, cs, sn, rows, g, st);
    case 64: return launch_d<T, 64, kRope>(kn, vn, kc, vc, w, cs, sn, rows, g, st);
    default: return launch_d<T, 128, kRope>(kn, vn, kc, vc, w, cs, sn, rows, g, st);
  }
}

int entry(const void *k_new, const void *v_new, void *k_cache, void *v_cache,
          const int32_t *block_tables, const int32_t *start_pos, const int32_t *n_new,
          const void *w, const void *cos, const void *sin, int64_t rope_rows, int64_t scos,
          int64_t ssin, float eps, bool rope, int64_t B, int64_t T, int64_t H, int64_t D,
          int64_t block_size, int64_t max_blocks, int64_t num_blocks, const int64_t *skn,
          const int64_t *svn, const int64_t *skc, const int64_t *svc, const int64_t *sbt,
          int dtype, void *stream) {
  const char *op = rope ? "paged_kv_append_rope" : "paged_kv_append";
  clear_error();
  TLLM_CHECK_ARG(B >= 0 && T >= 0 && H >= 0, "%s: negative dimension", op);
  TLLM_CHECK_ARG(D == 16 || D == 32 || D == 64 || D == 128, "%s: head dim %lld not in {16,32,64,128}",
                 op, (long long)D);
  TLLM_CHECK_ARG(block_size >= 1, "%s: block_size must be positive", op);
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16, "%s: unsupported dtype %d", op,
                 dtype);
  TLLM_CHECK_ARG(skn && svn && skc && svc && sbt, "%s: null stride array", op);
  const int64_t rows = B * T * H;
  if (rows == 0) return TLLM_OK;
  TLLM_CHECK_ARG(k_new && v_new && k_cache && v_cache && block_tables && start_pos,
                 "%s: null tensor pointer", op);
  TLLM_CHECK_ARG(max_blocks >= 1 && num_blocks >= 1, "%s: empty block table or pool", op);
  TLLM_CHECK_ARG(skn[3] == 1 && svn[3] == 1 && skc[3] == 1 && svc[3] == 1,
                 "%s: new K/V and caches need a unit innermost stride", op);
  for (int i = 0; i < 3; ++i)
    TLLM_CHECK_ARG(skn[i] % 8 == 0 && svn[i] % 8 == 0 && skc[i] % 8 == 0 && svc[i] % 8 == 0,
                   "%s: strides must be multiples of 8 elements", op);
  TLLM_CHECK_ARG(aligned16(k_new) && aligned16(v_new) && aligned16(k_cache) && aligned16(v_cache),
                 "%s: tensors must be 16-byte aligned", op);
  if (rope) {
    TLLM_CHECK_ARG(w && cos && sin, "%s: null weight/cos/sin pointer", op);
    TLLM_CHECK_ARG(rope_rows >= 1, "%s: empty cos/sin table", op);
    TLLM_CHECK_ARG(scos % 8 == 0 && ssin % 8 == 0 && aligned16(w) && aligned16(cos) && aligned16(sin),
                   "%s: weight/cos/sin rows must be contiguous and 16-byte aligned", op);
  }
  Geom g{};
  g.block_tables = block_tables;
  g.start_pos = start_pos;
  g.n_new = n_new;
  g.T = T;
  g.H = H;
  g.max_blocks = max_blocks;
  g.num_blocks = num_blocks;
  g.block_size = static_cast<int>(block_size);
  g.rope_rows = rope_rows;
  g.skn0 = skn[0]; g.skn1 = skn[1]; g.skn2 = skn[2];
  g.svn0 = svn[0]; g.svn1 = svn[1]; g.svn2 = svn[2];
  g.skc0 = skc[0]; g.skc1 = skc[1]; g.skc2 = skc[2];
  g.svc0 = svc[0]; g.svc1 = svc[1]; g.svc2 = svc[2];
  g.sbt0 = sbt[0]; g.sbt1 = sbt[1];
  g.scos = scos;
  g.ssin = ssin;
  g.eps = eps;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TLLM_DTYPE_F16)
    return rope ? launch<__half, true>(k_new, v_new, k_cache, v_cache, w, cos, sin, rows, D, g, st)
                : launch<__half, false>(k_new, v_new, k_cache, v_cache, w, cos, sin, rows, D, g, st);
  return rope ? launch<__nv_bfloat16, true>(k_new, v_new, k_cache, v_cache, w, cos, sin, rows, D, g, st)
              : launch<__nv_bfloat16, false>(k_new, v_new, k_cache, v_cache, w, cos, sin, rows, D, g, st);
}

}  // namespace
}  // namespace pkv
}  // namespace tllm

extern "C" int tllm_paged_kv_append(const void *k_new, const void *v_new, void *k_cache,
                                    void *v_cache, const int32_t *block_tables,
                                    const int32_t *start_pos, const int32_t *n_new, int64_t B,
                                    int64_t T, int64_t H, int64_t D, int64_t block_size,
                                    int64_t max_blocks, int64_t num_blocks, const int64_t *skn,
                                    const int64_t *svn, const int64_t *skc, const int64_t *svc,
                                    const int64_t *sbt, int dtype, void *stream) {
  return tllm::pkv::entry(k_new, v_new, k_cache, v_cache, block_tables, start_pos, n_new, nullptr,
                          nullptr, nullptr, 0, 0, 0, 0.f, false, B, T, H, D, block_size,
                          max_blocks, num_blocks, skn, svn, skc, svc, sbt, dtype, stream);
}

extern "C" int tllm_paged_kv_append_rope(const void *k_new, const void *v_new, const void *weight,
                                         const void *cos, const void *sin, int64_t rope_rows,
                                         int64_t scos, int64_t ssin, void *k_cache,
                                         void *v_cache, const int32_t *block_tables,
                                         const int32_t *start_pos, const int32_t *n_new,
                                         int64_t B, int64_t T, int64_t H, int64_t D,
                                         int64_t block_size, int64_t max_blocks,
                                         int64_t num_blocks, const int64_t *skn,
                                         const int64_t *svn, const int64_t *skc,
                                         const int64_t *svc, const int64_t *sbt, float eps,
                                         int dtype, void *stream) {
  return tllm::pkv::entry(k_new, v_new, k_cache, v_cache, block_tables, start_pos, n_new, weight,
                          cos, sin, rope_rows, scos, ssin, eps, true, B, T, H, D, block_size,
                          max_blocks, num_blocks, skn, svn, skc, svc, sbt, dtype, stream);
}
