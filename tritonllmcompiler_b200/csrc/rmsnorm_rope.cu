// Fused RMSNorm + rotate-half RoPE for sm_100a.
//
// Reference: python/triton_llm/ops/rmsnorm_rope.py:9-75 (one Triton program per (b,s,h)
// row, 4 warps each) and the oracle python/triton_llm/reference/norm_rope.py:12-40.
//
// B200 design: the op is pure HBM streaming (2 bytes in + 2 bytes out per element plus the
// small cos/sin/weight tables that stay in L2), so a row of D elements is handled by D/16
// threads, each owning one 16-byte vector of the first half and the matching vector of the
// second half; the sum of squares is reduced with warp shuffles inside that thread group and
// the rotate-half pairing (i, i + D/2) never leaves the thread's registers.
//
// Numerics (rmsnorm_rope.cuh) follow the oracle: variance and scaling in fp32, the
// normalised value x * rstd * w rounded to the I/O dtype (norm_rope.py:15), then RoPE in
// fp32 with one rounding per product (norm_rope.py:28-29), stored in the I/O dtype.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.h"
#include "ptx.cuh"
#include "rmsnorm_rope.cuh"

namespace tllm {
namespace {

struct RowGeom {
  int64_t S, H;
  int64_t sxb, sxs, sxh, sxd;
  int64_t sob, sos, soh, sod;
  int64_t scs, scd, sss, ssd, sw;
};

using namespace rr;

// Vector path: unit inner strides, 16-byte aligned rows. A group of TPR = D / 16 threads
// handles R consecutive heads of one (b, s) position: each thread owns one 16-byte vector
// of the first half of D and the matching vector of the second half, requests the x vectors
// of all R rows up front (R * 32 bytes in flight per thread), and loads the weight and the
// cos/sin vectors of position s once for the R rows. H % R == 0.
template <typename T, int D, int R>
__global__ void __launch_bounds__(256, 2) rmsnorm_rope_vec_kernel(
    const T *__restrict__ x, const T *__restrict__ w, const T *__restrict__ cosb,
    const T *__restrict__ sinb, T *__restrict__ out, int64_t groups, RowGeom g, float eps) {
  constexpr int TPR = D / 16;
  constexpr int HALF = D / 2;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t gi_raw = tid / TPR;
  // All TPR lanes of a group sit in one warp (TPR divides 32), so the shuffles below are
  // safe; a group past the end recomputes the last group and skips its stores.
  const bool valid = gi_raw < groups;
  const int64_t gi = valid ? gi_raw : groups - 1;
  const int c = static_cast<int>(tid % TPR) * 8;
  const int64_t row0 = gi * R;
  const int64_t h0 = row0 % g.H;
  const int64_t bs = row0 / g.H;
  const int64_t s = bs % g.S;
  const int64_t b = bs / g.S;
  const T *xr = x + b * g.sxb + s * g.sxs + h0 * g.sxh;
  uint4 x1r[R], x2r[R];
#pragma unroll
  for (int u = 0; u < R; ++u) {
    x1r[u] = ld_stream(xr + u * g.sxh + c);
    x2r[u] = ld_stream(xr + u * g.sxh + HALF + c);
  }
  float w1[8], w2[8], c1[8], c2[8], s1[8], s2[8];
  load8<T>(w + c, w1);
  load8<T>(w + HALF + c, w2);
  load8<T>(cosb + s * g.scs + c, c1);
  load8<T>(cosb + s * g.scs + HALF + c, c2);
  load8<T>(sinb + s * g.sss + c, s1);
  load8<T>(sinb + s * g.sss + HALF + c, s2);
  T *orow = out + b * g.sob + s * g.sos + h0 * g.soh;
#pragma unroll
  for (int u = 0; u < R; ++u) {
    uint4 o1, o2;
    norm_rope_vec<T, D>(x1r[u], x2r[u], w1, w2, c1, c2, s1, s2, eps, o1, o2);
    if (valid) {
      st_stream(orow + u * g.soh + c, o1);
      st_stream(orow + u * g.soh + HALF + c, o2);
    }
  }
}

// General-stride path: one thread per row (any strides, any alignment).
template <typename T>
__global__ void __launch_bounds__(128) rmsnorm_rope_strided_kernel(
    const T *__restrict__ x, const T *__restrict__ w, const T *__restrict__ cosb,
    const T *__restrict__ sinb, T *__restrict__ out, int64_t rows, int D, RowGeom g,
    float eps) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const int64_t h = row % g.H;
  const int64_t bs = row / g.H;
  const int64_t s = bs % g.S;
  const int64_t b = bs / g.S;
  const T *xr = x + b * g.sxb + s * g.sxs + h * g.sxh;
  T *orow = out + b * g.sob + s * g.sos + h * g.soh;
  const int half = D / 2;
  float ss = 0.f;
  for (int i = 0; i < D; ++i) {
    const float v = to_f32<T>(xr[i * g.sxd]);
    ss = fmaf(v, v, ss);
  }
  const float rstd = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(D)), eps));
  for (int i = 0; i < half; ++i) {
    const float y1 =
        round_io<T>(__fmul_rn(__fmul_rn(to_f32<T>(xr[i * g.sxd]), rstd), to_f32<T>(w[i * g.sw])));
    const float y2 = round_io<T>(__fmul_rn(__fmul_rn(to_f32<T>(xr[(i + half) * g.sxd]), rstd),
                                           to_f32<T>(w[(i + half) * g.sw])));
    const float ca = to_f32<T>(cosb[s * g.scs + i * g.scd]);
    const float cb = to_f32<T>(cosb[s * g.scs + (i + half) * g.scd]);
    const float sa = to_f32<T>(sinb[s * g.sss + i * g.ssd]);
    const float sb = to_f32<T>(sinb[s * g.sss + (i + half) * g.ssd]);
    orow[i * g.sod] = from_f32<T>(__fsub_rn(__fmul_rn(y1, ca), __fmul_rn(y2, sa)));
    orow[(i + half) * g.sod] = from_f32<T>(__fadd_rn(__fmul_rn(y2, cb), __fmul_rn(y1, sb)));
  }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T>
int launch(const void *x, const void *w, const void *c, const void *s, void *o, int64_t rows,
           int64_t D, const RowGeom &g, bool vec, float eps, cudaStream_t st) {
  const T *xp = static_cast<const T *>(x);
  const T *wp = static_cast<const T *>(w);
  const T *cp = static_cast<const T *>(c);
  const T *sp = static_cast<const T *>(s);
  T *op = static_cast<T *>(o);
  if (vec) {
    // Heads per thread group: 8 (or 4, 2) when H allows it and there is work for every SM
    // many times over; two 256-thread blocks stay resident per SM (register cap 128).
    const int64_t H = g.H;
    const int64_t sms = sm_count() > 0 ? sm_count() : 148;
    int R = 1;
    if (H % 8 == 0 && rows >= 8LL * sms * 256) R = 8;
    else if (H % 4 == 0 && rows >= 4LL * sms * 256) R = 4;
    else if (H % 2 == 0 && rows >= 2LL * sms * 256) R = 2;
    const int64_t groups = rows / R;
    const int64_t threads = groups * (D / 16);
    const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
#define TLLM_RR_LAUNCH(DD, RR)                                                                \
  rmsnorm_rope_vec_kernel<T, DD, RR><<<grid, 256, 0, st>>>(xp, wp, cp, sp, op, groups, g, eps)
#define TLLM_RR_BY_R(DD)            \
  if (R == 8) TLLM_RR_LAUNCH(DD, 8); \
  else if (R == 4) TLLM_RR_LAUNCH(DD, 4); \
  else if (R == 2) TLLM_RR_LAUNCH(DD, 2); \
  else TLLM_RR_LAUNCH(DD, 1);
    switch (D) {
      case 16: TLLM_RR_BY_R(16) break;
      case 32: TLLM_RR_BY_R(32) break;
      case 64: TLLM_RR_BY_R(64) break;
      default: TLLM_RR_BY_R(128) break;
    }
#undef TLLM_RR_BY_R
#undef TLLM_RR_LAUNCH
  } else {
    const unsigned grid = static_cast<unsigned>((rows + 127) / 128);
    rmsnorm_rope_strided_kernel<T><<<grid, 128, 0, st>>>(xp, wp, cp, sp, op, rows,
                                                         static_cast<int>(D), g, eps);
  }
  return cuda_status(cudaGetLastError(), "rmsnorm_rope launch");
}

}  // namespace
}  // namespace tllm

extern "C" int tllm_rmsnorm_rope(const void *x, const void *w, const void *cos, const void *sin,
                                 void *out, int64_t B, int64_t S, int64_t H, int64_t D,
                                 const int64_t *sx, int64_t sw, const int64_t *scos,
                                 const int64_t *ssin, const int64_t *so, float eps, int dtype,
                                 void *stream) {
  using namespace tllm;
  clear_error();
  TLLM_CHECK_ARG(B >= 0 && S >= 0 && H >= 0, "rmsnorm_rope: negative dimension");
  TLLM_CHECK_ARG(D == 16 || D == 32 || D == 64 || D == 128,
                 "rmsnorm_rope: head dim %lld not in {16,32,64,128}", (long long)D);
  TLLM_CHECK_ARG(dtype == TLLM_DTYPE_F16 || dtype == TLLM_DTYPE_BF16,
                 "rmsnorm_rope: unsupported dtype %d", dtype);
  TLLM_CHECK_ARG(sx && scos && ssin && so, "rmsnorm_rope: null stride array");
  const int64_t rows = B * S * H;
  if (rows == 0) return TLLM_OK;
  TLLM_CHECK_ARG(x && w && cos && sin && out, "rmsnorm_rope: null tensor pointer");
  RowGeom g{S,       H,       sx[0],   sx[1],   sx[2],   sx[3], so[0], so[1],
            so[2],   so[3],   scos[0], scos[1], ssin[0], ssin[1], sw};
  const bool vec = sx[3] == 1 && so[3] == 1 && scos[1] == 1 && ssin[1] == 1 && sw == 1 &&
                   sx[0] % 8 == 0 && sx[1] % 8 == 0 && sx[2] % 8 == 0 && so[0] % 8 == 0 &&
                   so[1] % 8 == 0 && so[2] % 8 == 0 && scos[0] % 8 == 0 && ssin[0] % 8 == 0 &&
                   aligned16(x) && aligned16(out) && aligned16(w) && aligned16(cos) &&
                   aligned16(sin);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TLLM_DTYPE_F16) return launch<__half>(x, w, cos, sin, out, rows, D, g, vec, eps, st);
  return launch<__nv_bfloat16>(x, w, cos, sin, out, rows, D, g, vec, eps, st);
}
