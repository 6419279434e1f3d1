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

// K/V cache entries: f32, or f16 when H (each value rounded to nearest even
// at store, converted exactly at load).  i is an element index.
template <bool H>
__device__ __forceinline__ float kv_get(const float *base, size_t i) {
  if (H) return __half2float(reinterpret_cast<const __half *>(base)[i]);
  return base[i];
}
template <bool H>
__device__ __forceinline__ void kv_put(float *base, size_t i, float v) {
  if (H) reinterpret_cast<__half *>(base)[i] = __float2half_rn(v);
  else base[i] = v;
}
// acc + e * v, or acc itself when e == 0 (a zero weight is skipped).
// acc + (-0.0) is acc for every acc, +-0, inf and NaN included, so choosing
// -0.0 for the skipped product gives the skip's bits while the select stays
// off the chain: each step of a chain waits for one add only.
__device__ __forceinline__ float add_weighted(float acc, float e, float v) {
  return fadd(acc, e != 0.0f ? fmul(e, v) : -0.0f);
}

// One staged cache element as f32, and four consecutive ones (p aligned to
// four elements), for kernels templated on the entry type.
__device__ __forceinline__ float kv_f(float v) { return v; }
__device__ __forceinline__ float kv_f(__half v) { return __half2float(v); }
__device__ __forceinline__ float4 kv_f4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ float4 kv_f4(const __half *p) {
  const uint2 u = *reinterpret_cast<const uint2 *>(p);
  const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
  const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

// expf as the C library computes it (the function Rust's f32::exp calls):
// the published table-driven method -- x * 32/ln2 = k + r with |r| <= 1/2,
// 2^(k/32) from a 32-entry table, 2^(r/32) from a cubic, all in double with
// fused multiply-adds, one rounding to float at the end.  The table is
// 2^(i/32) correctly rounded (minus i << 47 in the bit pattern); the cubic's
// coefficients are the method's minimax constants.  This evaluation returns
// the same bits as the host C library for every non-NaN float (checked over
// all 2^32 inputs), which the parity of softmax and SwiGLU depends on.
// The table is global memory read through the read-only data cache: the
// lanes of a warp index it with unrelated k, and a constant-bank read would
// be replayed once per distinct entry, where the L1 serves all 32 entries
// (256 bytes) in two wavefronts.
static __device__ const unsigned long long kExp2Tab[32] = {
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL,
    0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL,
    0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL,
    0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL,
    0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL,
    0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL,
    0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL,
    0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL,
};

__device__ __forceinline__ float expf_lib(float x) {
  if (isnan(x)) return x + x;
  if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);  // overflow
  if (x < -0x1.9fe368p6f) return 0.0f;                       // underflow
  const double kInvLn2N = 0x1.71547652b82fep+0 * 32.0, kShift = 0x1.8p+52;
  const double kC0 = 0x1.c6af84b912394p-5 / 32768.0, kC1 = 0x1.ebfce50fac4f3p-3 / 1024.0,
               kC2 = 0x1.62e42ff0c52d6p-1 / 32.0;
  const double xd = (double)x;
  double kd = __fma_rn(kInvLn2N, xd, kShift);
  const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
  kd = __dsub_rn(kd, kShift);
  const double r = __fma_rn(kInvLn2N, xd, -kd);
  const double s = __longlong_as_double((long long)(__ldg(&kExp2Tab[ki & 31]) + (ki << 47)));
  const double z = __fma_rn(kC0, r, kC1);
  const double r2 = __dmul_rn(r, r);
  double y = __fma_rn(kC2, r, 1.0);
  y = __fma_rn(z, r2, y);
  y = __dmul_rn(y, s);
  return __double2float_rn(y);
}

// Shared-memory accesses by 32-bit shared address (ld/st.shared), for loops
// whose pointers the compiler could otherwise only treat as generic.
__device__ __forceinline__ uint32_t shaddr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint4 sld_v4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 sld_v2(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ int4 sld_v4i(uint32_t a) {
  int4 v;
  asm volatile("ld.shared.v4.s32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ float4 sld_v4f(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ float sld_f(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ int sld_i(uint32_t a) {
  int v;
  asm volatile("ld.shared.s32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint16_t sld_u16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void sst_f(uint32_t a, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}

// Streaming 16-byte load of weights (read once per token): no L1 allocation.
__device__ __forceinline__ uint4 ldw16(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Programmatic dependent launch.  Every kernel calls pdl_trigger() first (so
// the next kernel in the stream may be scheduled once all of this grid's CTAs
// are running) and pdl_wait() before it touches anything an earlier kernel
// wrote.  griddepcontrol.wait returns once the preceding grids have completed
// and their memory is visible; without a programmatic launch it is a no-op.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Hint: stream [p, p + bytes) from HBM into L2 (bytes a multiple of 16, p
// 16-byte aligned, the range inside the allocation).
__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
  if (bytes >= 16) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes & ~15u) : "memory");
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

// q8_block_lane for N independent blocks at once (one value per lane of
// each), their shuffles interleaved so the latencies overlap.  ok[j] must be
// the same on every lane (a block the warp skips still takes part in the
// shuffles and stores nothing).
template <int N>
__device__ __forceinline__ void q8_blocks_lane(const float (&v)[N], const bool (&ok)[N], int lane, int8_t *const (&q)[N],
                                               float *const (&d)[N], int32_t *const (&sum)[N]) {
  float amax[N];
#pragma unroll
  for (int j = 0; j < N; j++) {
    const float a = fabsf(v[j]);
    amax[j] = a > 0.0f ? a : 0.0f;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int j = 0; j < N; j++) {
      const float w = __shfl_xor_sync(0xffffffffu, amax[j], o);
      amax[j] = w > amax[j] ? w : amax[j];
    }
  }
  int iv[N];
  float dd[N];
#pragma unroll
  for (int j = 0; j < N; j++) {
    dd[j] = fdiv(amax[j], 127.0f);
    const float inv = dd[j] > 0.0f ? fdiv(1.0f, dd[j]) : 0.0f;
    float r = roundf(fmul(v[j], inv));
    r = r < -127.0f ? -127.0f : r;
    r = r > 127.0f ? 127.0f : r;
    iv[j] = isnan(r) ? 0 : (int)r;
    if (ok[j]) q[j][lane] = (int8_t)iv[j];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
    for (int j = 0; j < N; j++) iv[j] += __shfl_xor_sync(0xffffffffu, iv[j], o);
  }
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < N; j++)
      if (ok[j]) {
        *d[j] = dd[j];
        *sum[j] = iv[j];
      }
  }
}

// q8_block_lane for a 32-element block held V values per lane by a group of
// L = 32 / V consecutive lanes (l = lane within the group; every group of
// the warp runs it together, each on its own block): value V * l + e is
// v[e].  Same arithmetic, same results.  Every lane of the warp calls it;
// a group with store == false stores nothing.
template <int L, int V>
__device__ __forceinline__ void q8_block_group(const float (&v)[V], int l, bool store, int8_t *q, float *d,
                                               int32_t *sum) {
  static_assert(L * V == 32, "one 32-element block per group");
  float amax = 0.0f;
#pragma unroll
  for (int e = 0; e < V; e++) {
    const float a = fabsf(v[e]);
    amax = a > amax ? a : amax;  // NaN never wins, as in q8_block_lane
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) {
    const float t = __shfl_xor_sync(0xFFFFFFFFu, amax, o);
    amax = t > amax ? t : amax;
  }
  const float dd = fdiv(amax, 127.0f);
  const float inv = dd > 0.0f ? fdiv(1.0f, dd) : 0.0f;
  int s = 0, iv[V];
#pragma unroll
  for (int e = 0; e < V; e++) {
    float r = roundf(fmul(v[e], inv));
    r = r < -127.0f ? -127.0f : r;
    r = r > 127.0f ? 127.0f : r;
    iv[e] = isnan(r) ? 0 : (int)r;
    s += iv[e];
  }
  if (store) {
#pragma unroll
    for (int e = 0; e < V; e++) q[V * l + e] = (int8_t)iv[e];
  }
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  if (store && l == 0) {
    *d = dd;
    *sum = s;
  }
}

}  // namespace pk
