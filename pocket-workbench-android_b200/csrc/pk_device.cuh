// pk_device.cuh -- device helpers shared by the sm_100a kernels.
//
// Float arithmetic that must match the reference bit-for-bit uses the *_rn
// intrinsics, which nvcc never contracts into FMAs; the reference (Rust)
// rounds every multiply and add separately.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pk {

enum : int {
  T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8,
  T_Q8_1 = 9, T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14,
  T_Q8_K = 15, T_BF16 = 30
};

// Exact f16 -> f32 (every f16, subnormals included, is an f32); equals
// util.rs:76-100 for all non-NaN inputs.
__device__ __forceinline__ float f16f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// exp for the f32 paths: computed in double and rounded once, so it is the
// correctly rounded expf except in vanishingly rare cases.  The reference's
// f32::exp resolves to the C library's expf (< 0.51 ulp), so the two agree
// on essentially every input.
__device__ __forceinline__ float expf_cr(float x) { return (float)exp((double)x); }

// Streaming 16-byte load of weights (read once per token): no L1 allocation.
__device__ __forceinline__ uint4 ldw16(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
__device__ __forceinline__ uint32_t byte_of(const uint4 &v, int j) {
  return (word_of(v, j >> 2) >> ((j & 3) * 8)) & 0xFFu;
}

// quant.rs:80-86 get_scale_min_k4 on the 12 scale bytes held in bytes 4..15
// of a Q4_K block header.
__device__ __forceinline__ void scale_min_k4(const uint4 &hdr, int j, int &sc, int &m) {
  if (j < 4) {
    sc = (int)(byte_of(hdr, 4 + j) & 63u);
    m = (int)(byte_of(hdr, 4 + j + 4) & 63u);
  } else {
    sc = (int)((byte_of(hdr, 4 + j + 4) & 0xFu) | ((byte_of(hdr, 4 + j - 4) >> 6) << 4));
    m = (int)((byte_of(hdr, 4 + j + 4) >> 4) | ((byte_of(hdr, 4 + j) >> 6) << 4));
  }
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fadd(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Q8Act::prepare for one 32-element block held one element per lane
// (quant_int.rs:36-53): amax over |x| ignoring NaN, d = amax/127,
// inv = 1/d (0 if d == 0), q = clamp(round_half_away(x*inv), +-127), NaN -> 0.
__device__ __forceinline__ void q8_block_lane(float v, int lane, int8_t *q, float *d, int32_t *sum) {
  float a = fabsf(v);
  float amax = a > 0.0f ? a : 0.0f;
  amax = warp_max(amax);
  float dd = fdiv(amax, 127.0f);
  float inv = dd > 0.0f ? fdiv(1.0f, dd) : 0.0f;
  float r = roundf(fmul(v, inv));
  r = r < -127.0f ? -127.0f : r;
  r = r > 127.0f ? 127.0f : r;
  int iv = isnan(r) ? 0 : (int)r;
  q[lane] = (int8_t)iv;
  int s = warp_sum_i(iv);
  if (lane == 0) {
    *d = dd;
    *sum = s;
  }
}

}  // namespace pk
