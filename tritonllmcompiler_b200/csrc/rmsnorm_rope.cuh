// Row arithmetic of the fused RMSNorm + rotate-half RoPE, shared by the plain operator
// (rmsnorm_rope.cu) and the paged-cache append (paged_kv.cu) so that both round identically.
//
// Numerics follow python/triton_llm/reference/norm_rope.py:12-40: variance and scaling in
// fp32, the normalised value x * rstd * w rounded to the I/O dtype (:15), then RoPE in fp32
// with one rounding per product (:28-29), stored in the I/O dtype.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace tllm {
namespace rr {

template <typename T>
__device__ __forceinline__ void load8(const T *p, float (&v)[8]) {
  const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(p));
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = Pack2<T>::unpack(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <typename T>
__device__ __forceinline__ void unpack8(const uint4 &raw, float (&v)[8]) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = Pack2<T>::unpack(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <typename T>
__device__ __forceinline__ void store8(T *p, const float (&v)[8]) {
  uint4 raw;
  raw.x = Pack2<T>::pack(v[0], v[1]);
  raw.y = Pack2<T>::pack(v[2], v[3]);
  raw.z = Pack2<T>::pack(v[4], v[5]);
  raw.w = Pack2<T>::pack(v[6], v[7]);
  *reinterpret_cast<uint4 *>(p) = raw;
}

template <typename T>
__device__ __forceinline__ float round_io(float v) {
  return to_f32<T>(from_f32<T>(v));
}

// Streaming global accesses: x is read once (no L1 allocation), out is written once.
__device__ __forceinline__ uint4 ld_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ void st_stream(void *p, const uint4 &v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 raw;
  raw.x = Pack2<T>::pack(v[0], v[1]);
  raw.y = Pack2<T>::pack(v[2], v[3]);
  raw.z = Pack2<T>::pack(v[4], v[5]);
  raw.w = Pack2<T>::pack(v[6], v[7]);
  return raw;
}


// One 16-byte vector of each half of a row, for the TPR = D / 16 lanes that hold the row
// (consecutive lanes of one warp): sum of squares reduced over those lanes, RMSNorm, weight,
// rounding, rotate-half RoPE. x1r/x2r: elements [c, c+8) and [D/2 + c, D/2 + c + 8).
template <typename T, int D>
__device__ __forceinline__ void norm_rope_vec(const uint4 &x1r, const uint4 &x2r,
                                              const float (&w1)[8], const float (&w2)[8],
                                              const float (&c1)[8], const float (&c2)[8],
                                              const float (&s1)[8], const float (&s2)[8],
                                              float eps, uint4 &o1r, uint4 &o2r) {
  constexpr int TPR = D / 16;
  float x1[8], x2[8];
  unpack8<T>(x1r, x1);
  unpack8<T>(x2r, x2);
  float ss2 = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss2 = fmaf(x1[i], x1[i], fmaf(x2[i], x2[i], ss2));
#pragma unroll
  for (int off = TPR / 2; off > 0; off >>= 1) ss2 += __shfl_xor_sync(0xffffffffu, ss2, off);
  const float rstd = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss2, static_cast<float>(D)), eps));
  float o1[8], o2[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float y1 = round_io<T>(__fmul_rn(__fmul_rn(x1[i], rstd), w1[i]));
    const float y2 = round_io<T>(__fmul_rn(__fmul_rn(x2[i], rstd), w2[i]));
    o1[i] = __fsub_rn(__fmul_rn(y1, c1[i]), __fmul_rn(y2, s1[i]));
    o2[i] = __fadd_rn(__fmul_rn(y2, c2[i]), __fmul_rn(y1, s2[i]));
  }
  o1r = pack8<T>(o1);
  o2r = pack8<T>(o2);
}

}  // namespace rr
}  // namespace tllm
