// pk_kernels.cu -- sm_100a kernels for pocketinfer's decode and prefill path.
//
// Reference semantics (Aleinto97/pocket-workbench-android, rust/pocketinfer/src):
//   Q8 activation quantiser       quant_int.rs:17-56
//   int8 k-quant row dots         quant_int.rs:282-419 (lanes::*)
//   dequant (embedding, norms)    quant.rs:102-359
//   rmsnorm / rope / attention / swiglu / residual   model.rs:777-823, 905-1172
//   greedy sampler                sampler.rs:21-36
//
// Exactness.  A row of a k-quant matvec is, in the reference, a sequential
// float sum over per-sub-block terms such as
//     acc += d*da*sc*dot - da*dmin*m*sa          (Q4_K, quant_int.rs:364)
// The kernels below compute every integer dot with dp4a (exact), turn it into
// the same float term with separately rounded multiplies/subtracts (exact),
// park the terms in shared memory, and let one thread per row add them in
// the reference's order.  The matvec output is therefore bit-identical to the
// reference for identical Q8 inputs, not merely within tolerance.
#include <float.h>
#include <limits.h>
#include <math.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>

#include "pk_device.cuh"
#include "pk_quant.cuh"
#include "pk_kernels.h"

namespace pk {

// ------------------------------------------------------------ type table
bool type_block(int t, int *be, int *bb) {  // quant.rs:19-37
  int e, b;
  switch (t) {
    case T_F32: e = 1; b = 4; break;
    case T_F16: case T_BF16: e = 1; b = 2; break;
    case T_Q4_0: e = 32; b = 18; break;
    case T_Q4_1: e = 32; b = 20; break;
    case T_Q5_0: e = 32; b = 22; break;
    case T_Q5_1: e = 32; b = 24; break;
    case T_Q8_0: e = 32; b = 34; break;
    case T_Q8_1: e = 32; b = 36; break;
    case T_Q2_K: e = 256; b = 84; break;
    case T_Q3_K: e = 256; b = 110; break;
    case T_Q4_K: e = 256; b = 144; break;
    case T_Q5_K: e = 256; b = 176; break;
    case T_Q6_K: e = 256; b = 210; break;
    case T_Q8_K: e = 256; b = 292; break;
    default: return false;
  }
  if (be) *be = e;
  if (bb) *bb = b;
  return true;
}

bool type_is_matvec(int t) { return t == T_Q4_K || t == T_Q6_K || t == T_Q4_0 || t == T_Q8_0; }

static inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

size_t packed_q_bytes(int t, int k, int rows) {
  switch (t) {
    case T_Q4_K: return (size_t)rows * (size_t)(k / 256) * 144;
    case T_Q6_K: return (size_t)rows * (size_t)(k / 256) * 208;
    case T_Q8_0: return (size_t)rows * (size_t)k;
    case T_Q4_0: return (size_t)rows * (size_t)(k / 2);
  }
  return 0;
}

static size_t packed_d_bytes(int t, int k, int rows) {
  switch (t) {
    case T_Q6_K: return (size_t)rows * (size_t)(k / 256) * 2;
    case T_Q8_0: case T_Q4_0: return (size_t)rows * (size_t)(k / 32) * 2;
  }
  return 0;
}

size_t packed_bytes(int t, int k, int rows) {
  return align256(packed_q_bytes(t, k, rows)) + align256(packed_d_bytes(t, k, rows));
}

DevTensor packed_view(int t, int k, int rows, const void *packed) {
  DevTensor w;
  w.type = t;
  w.k = k;
  w.rows = rows;
  w.q = (const uint8_t *)packed;
  w.d = packed_d_bytes(t, k, rows) ? (const uint16_t *)((const uint8_t *)packed + align256(packed_q_bytes(t, k, rows)))
                                    : nullptr;
  return w;
}

static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    n = v > 0 ? v : 148;
  }
  return n;
}


// Launch with programmatic stream serialization: the kernel may be scheduled
// while its predecessor in the stream still runs; every kernel here orders its
// dependent reads with pdl_wait() (griddepcontrol.wait).
template <typename... KArgs, typename... Args>
static cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                          Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ------------------------------------------------------------ packing
__global__ void k_pack(int t, const uint8_t *__restrict__ raw, size_t row_bytes, int k, int rows,
                       uint8_t *__restrict__ q, uint16_t *__restrict__ d) {
  pdl_trigger();
  pdl_wait();
  const int be = (t == T_Q4_K || t == T_Q6_K) ? 256 : 32;
  const int nblk = k / be;
  const long n = (long)rows * nblk;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long r = i / nblk;
    const int b = (int)(i - r * nblk);
    switch (t) {
      case T_Q4_K: {
        const uint8_t *s = raw + r * row_bytes + (size_t)b * 144;
        uint8_t *o = q + i * 144;
        for (int j = 0; j < 144; j++) o[j] = s[j];
      } break;
      case T_Q6_K: {
        const uint8_t *s = raw + r * row_bytes + (size_t)b * 210;
        uint8_t *o = q + i * 208;
        for (int j = 0; j < 208; j++) o[j] = s[j];
        d[i] = (uint16_t)(s[208] | (s[209] << 8));
      } break;
      case T_Q8_0: {
        const uint8_t *s = raw + r * row_bytes + (size_t)b * 34;
        uint8_t *o = q + r * (long)k + (long)b * 32;
        for (int j = 0; j < 32; j++) o[j] = s[2 + j];
        d[i] = (uint16_t)(s[0] | (s[1] << 8));
      } break;
      case T_Q4_0: {
        const uint8_t *s = raw + r * row_bytes + (size_t)b * 18;
        uint8_t *o = q + r * (long)(k / 2) + (long)b * 16;
        for (int j = 0; j < 16; j++) o[j] = s[2 + j];
        d[i] = (uint16_t)(s[0] | (s[1] << 8));
      } break;
    }
  }
}

cudaError_t launch_pack(int t, const void *raw, size_t row_bytes, int k, int rows, void *packed, cudaStream_t st) {
  if (!type_is_matvec(t)) return cudaErrorInvalidValue;
  DevTensor w = packed_view(t, k, rows, packed);
  int be = (t == T_Q4_K || t == T_Q6_K) ? 256 : 32;
  long n = (long)rows * (k / be);
  int grid = (int)std::min<long>((n + 255) / 256, (long)num_sms() * 16);
  if (grid < 1) grid = 1;
  return launch(k_pack, dim3(grid), dim3(256), 0, st, t, (const uint8_t *)raw, row_bytes, k, rows, (uint8_t *)w.q, (uint16_t *)w.d);
}

// ------------------------------------------------------------ dequant rows
__global__ void k_dequant_rows(int t, const uint8_t *__restrict__ raw, size_t row_bytes, int k,
                               const uint32_t *__restrict__ ids, float *__restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const long r = ids ? (long)ids[blockIdx.x] : (long)blockIdx.x;
  const uint8_t *row = raw + r * row_bytes;
  for (int j = threadIdx.x; j < k; j += blockDim.x) out[(long)blockIdx.x * k + j] = dequant_elem(t, row, j);
}

cudaError_t launch_dequant_rows(int t, const void *raw, size_t row_bytes, int k, const uint32_t *ids, int n,
                                float *out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  return launch(k_dequant_rows, dim3(n), dim3(256), 0, st, t, (const uint8_t *)raw, row_bytes, k, ids, out);
}

// ------------------------------------------------------------ reductions
// Deterministic block sum: per-warp trees, then warp partials in warp order.
__device__ float block_sum(float v, float *red) {
  v = warp_sum_f(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int i = 0; i < nw; i++) s = fadd(s, red[i]);
    red[32] = s;
  }
  __syncthreads();
  return red[32];
}

__device__ float block_max(float v, float *red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float m = -INFINITY;
    for (int i = 0; i < nw; i++) m = red[i] > m ? red[i] : m;
    red[32] = m;
  }
  __syncthreads();
  return red[32];
}

// A launch gets 48 KB of shared memory, static and dynamic together, unless
// the kernel opts in to more.  The kernels here declare at most 1.2 KB of
// static arrays, so any dynamic size above 44 KB opts in.
template <typename K>
static cudaError_t set_smem(K kernel, size_t smem) {
  if (smem > 44 * 1024) return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return cudaSuccess;
}

// ------------------------------------------------------------ Q8 quantiser
__global__ void k_q8(const float *__restrict__ x, long xs_e, long xs_l, int k, int b, Q8Dev act) {
  pdl_trigger();
  pdl_wait();
  const int nb = k >> 5, lane = threadIdx.x & 31;
  const long nwarp_total = (long)b * nb;
  const long wstride = ((long)gridDim.x * blockDim.x) >> 5;
  for (long w = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5; w < nwarp_total; w += wstride) {
    const int bi = (int)(w / nb), blk = (int)(w - (long)bi * nb);
    float v = x[(long)(blk * 32 + lane) * xs_e + (long)bi * xs_l];
    q8_block_lane(v, lane, act.q + (long)bi * k + blk * 32, act.d + (long)bi * nb + blk, act.s + (long)bi * nb + blk);
  }
}

cudaError_t kernels_binary_version(int *v) {
  cudaFuncAttributes fa{};
  const cudaError_t e = cudaFuncGetAttributes(&fa, k_q8);
  if (e == cudaSuccess) *v = fa.binaryVersion;
  return e;
}

cudaError_t launch_q8(const float *x, long xs_e, long xs_l, int k, int b, Q8Dev act, cudaStream_t st) {
  long warps = (long)b * (k / 32);
  int grid = (int)std::min<long>((warps * 32 + 255) / 256, (long)num_sms() * 8);
  if (grid < 1) grid = 1;
  return launch(k_q8, dim3(grid), dim3(256), 0, st, x, xs_e, xs_l, k, b, act);
}

// Sum of squares in the reference's b == 1 order (simd.rs:47-64 f32_sum_sq):
// eight FMA chains over x[8t + l], lanes l and l + 4 added, then a pairwise
// horizontal add, then an unfused tail.
__device__ float sum_sq_neon(const float *__restrict__ x, int n, float *red) {
  const int tid = threadIdx.x, n8 = n / 8 * 8;
  if (tid < 8) {
    float acc = 0.0f;
    // unrolled so the loads of 32 steps are issued ahead of their FMAs
#pragma unroll 32
    for (int i = tid; i < n8; i += 8) acc = __fmaf_rn(x[i], x[i], acc);
    red[tid] = acc;
  }
  __syncthreads();
  if (tid == 0) {
    const float c0 = fadd(red[0], red[4]), c1 = fadd(red[1], red[5]), c2 = fadd(red[2], red[6]),
                c3 = fadd(red[3], red[7]);
    float s = fadd(fadd(c0, c1), fadd(c2, c3));
    for (int i = n8; i < n; i++) s = fadd(s, fmul(x[i], x[i]));
    red[32] = s;
  }
  __syncthreads();
  return red[32];
}

// Sum of squares in the reference's b > 1 order (model.rs:813-817): one
// sequential unfused chain over the squares sq[] (formed by every thread,
// zero-padded to a multiple of 16).  Thread 0 adds them in order, loading
// the next sixteen while it adds the current sixteen; the padding adds
// +0.0, exact for a sum that starts at +0.0.  Result broadcast through
// red[32].
__device__ float sum_sq_chain(const float *sq, int n, float *red) {
  const int n16 = (n + 15) & ~15;
  if (threadIdx.x == 0) {
    const float4 *s4 = reinterpret_cast<const float4 *>(sq);
    const int g = n16 / 16;
    float ss = 0.0f;
    float4 c0 = s4[0], c1 = s4[1], c2 = s4[2], c3 = s4[3];
    for (int i = 0; i < g; i++) {
      const int nx = i + 1 < g ? 4 * (i + 1) : 4 * i;
      const float4 n0 = s4[nx], n1 = s4[nx + 1], n2 = s4[nx + 2], n3 = s4[nx + 3];
      ss = fadd(ss, c0.x); ss = fadd(ss, c0.y); ss = fadd(ss, c0.z); ss = fadd(ss, c0.w);
      ss = fadd(ss, c1.x); ss = fadd(ss, c1.y); ss = fadd(ss, c1.z); ss = fadd(ss, c1.w);
      ss = fadd(ss, c2.x); ss = fadd(ss, c2.y); ss = fadd(ss, c2.z); ss = fadd(ss, c2.w);
      ss = fadd(ss, c3.x); ss = fadd(ss, c3.y); ss = fadd(ss, c3.z); ss = fadd(ss, c3.w);
      c0 = n0; c1 = n1; c2 = n2; c3 = n3;
    }
    red[32] = ss;
  }
  __syncthreads();
  return red[32];
}

// RMSNorm of token-major x [b][k] (model.rs:812-822) followed by Q8.  The
// token's row, the norm weights and the squares are staged in shared
// memory (dynamic, 3 x k floats, k a multiple of 32); each warp then
// quantises its blocks three at a time.  The weights are constant, so they
// are staged before the wait for the kernel that writes x.
__global__ void k_rmsnorm_q8(const float *__restrict__ x, const float *__restrict__ nw, float eps, int k, Q8Dev act,
                             float *__restrict__ xn, int neon) {
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[40];
  float *ws = xs + k, *sq = ws + k;
  const int bi = blockIdx.x, n4 = k / 4;
  const float4 *x4 = reinterpret_cast<const float4 *>(x + (long)bi * k), *w4 = reinterpret_cast<const float4 *>(nw);
  pdl_trigger();
  for (int i = threadIdx.x; i < n4; i += blockDim.x) reinterpret_cast<float4 *>(ws)[i] = w4[i];
  pdl_wait();
  constexpr int U = 4;  // every load of the row in flight before the first store
  for (int i0 = threadIdx.x; i0 < n4; i0 += U * blockDim.x) {
    float4 v[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int i = i0 + u * blockDim.x;
      v[u] = i < n4 ? x4[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int i = i0 + u * blockDim.x;
      if (i < n4) {
        reinterpret_cast<float4 *>(xs)[i] = v[u];
        reinterpret_cast<float4 *>(sq)[i] =
            make_float4(fmul(v[u].x, v[u].x), fmul(v[u].y, v[u].y), fmul(v[u].z, v[u].z), fmul(v[u].w, v[u].w));
      }
    }
  }
  __syncthreads();
  const float ss = neon ? sum_sq_neon(xs, k, red) : sum_sq_chain(sq, k, red);
  const float s = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(ss, (float)k), eps)));
  const int nb = k >> 5, lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw_ = blockDim.x >> 5;
  for (int b0 = w; b0 < nb; b0 += 3 * nw_) {
    float v[3];
    bool ok[3];
    int8_t *qp[3];
    float *dp[3];
    int32_t *sp[3];
#pragma unroll
    for (int j = 0; j < 3; j++) {
      const int blk = b0 + j * nw_;
      ok[j] = blk < nb;
      const int bc = ok[j] ? blk : 0, i = bc * 32 + lane;
      v[j] = fmul(fmul(xs[i], s), ws[i]);
      if (ok[j] && xn) xn[(long)bi * k + i] = v[j];
      qp[j] = act.q + (long)bi * k + bc * 32;
      dp[j] = act.d + (long)bi * nb + bc;
      sp[j] = act.s + (long)bi * nb + bc;
    }
    q8_blocks_lane<3>(v, ok, lane, qp, dp, sp);
  }
}

cudaError_t launch_rmsnorm_q8(const float *x, const float *nw, float eps, int k, int b, Q8Dev act, float *xn,
                              cudaStream_t st, bool neon) {
  if (k % 32 != 0 || ((uintptr_t)x | (uintptr_t)nw) % 16 != 0) return cudaErrorInvalidValue;
  const size_t smem = (size_t)3 * k * 4;
  cudaError_t e = set_smem(k_rmsnorm_q8, smem);
  if (e != cudaSuccess) return e;
  return launch(k_rmsnorm_q8, dim3(b), dim3(256), smem, st, x, nw, eps, k, act, xn, neon ? 1 : 0);
}

// SwiGLU (model.rs:1105-1115: h = g / (1 + exp(-g)) * u) of token-major g, u [b][k], then Q8 of
// the product; h (optional) gets the floats.  One warp per 32-element block.
__global__ void k_swiglu_q8(const float *__restrict__ g, const float *__restrict__ u, int k, int b, Q8Dev act,
                            float *__restrict__ h) {
  pdl_trigger();
  pdl_wait();
  const int nb = k >> 5, lane = threadIdx.x & 31;
  const long nwarp_total = (long)b * nb;
  const long wstride = ((long)gridDim.x * blockDim.x) >> 5;
  for (long w = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5; w < nwarp_total; w += wstride) {
    const int bi = (int)(w / nb), blk = (int)(w - (long)bi * nb);
    const long i = (long)bi * k + blk * 32 + lane;
    const float gg = g[i];
    const float v = fmul(fdiv(gg, fadd(1.0f, expf_lib(-gg))), u[i]);
    if (h) h[i] = v;
    q8_block_lane(v, lane, act.q + (long)bi * k + blk * 32, act.d + (long)bi * nb + blk, act.s + (long)bi * nb + blk);
  }
}

cudaError_t launch_swiglu_q8(const float *g, const float *u, int k, int b, Q8Dev act, float *h, cudaStream_t st) {
  if (k % 32 != 0 || b < 1) return cudaErrorInvalidValue;
  long warps = (long)b * (k / 32);
  int grid = (int)std::min<long>((warps * 32 + 255) / 256, (long)num_sms() * 8);
  return launch(k_swiglu_q8, dim3(std::max(grid, 1)), dim3(256), 0, st, g, u, k, b, act, h);
}

// ------------------------------------------------------------ matvec core
// A "group" is the unit one thread handles: 64 weights of Q4_K / Q6_K or a
// 32-weight block of Q8_0 / Q4_0.  It yields TPG consecutive terms of the
// row's reference accumulation order (term index = group * TPG + s).
// ------------------------------------------------------------ single-lane tile
constexpr int B1_THREADS = 256;
constexpr int B1_RT = 16;   // rows per tile
constexpr int B1_TW = 256;  // terms per wave per row
constexpr int B1_MIN_CTAS = 3;  // resident CTAs per SM the register budget must allow

// Rows [r0, r0+nr) of W against one activation held in shared memory.
// Returns the row's reference-ordered sum in threads [0, nr).  Each thread
// issues the weight loads of U items before it computes any of them (an
// item past the end loads a valid one again and stores nothing), so a wave
// waits for about one global round trip instead of one per item.
template <int T>
__device__ float tile_b1(const DevTensor &W, int r0, int nr, const ActRef &A, float *Tsm) {
  constexpr int GE = Geo<T>::GE, TPG = Geo<T>::TPG, GW = B1_TW / TPG;
  constexpr int U = TPG == 1 ? 4 : 2;
  const int G = W.k / GE;
  const int tid = threadIdx.x;
  float acc = 0.0f;
  for (int g0 = 0; g0 < G; g0 += GW) {
    const int gw = min(GW, G - g0);
    const int items = nr * gw;
    for (int it0 = tid; it0 < items; it0 += U * B1_THREADS) {
      GroupW<T> gwt[U];
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int it = min(it0 + u * B1_THREADS, items - 1);
        const int rl = it / gw, gl = it - rl * gw;
        gwt[u].load(W, r0 + rl, g0 + gl);
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int it = it0 + u * B1_THREADS;
        if (it < items) {
          const int rl = it / gw, gl = it - rl * gw;
          float t[TPG];
          gwt[u].terms(A, t);
#pragma unroll
          for (int s = 0; s < TPG; s++) Tsm[(gl * TPG + s) * B1_RT + rl] = t[s];
        }
      }
    }
    __syncthreads();
    if (tid < nr) {
      const int nt = gw * TPG;
#pragma unroll 8
      for (int j = 0; j < nt; j++) acc = fadd(acc, Tsm[j * B1_RT + tid]);
    }
    __syncthreads();
  }
  return acc;
}

// L2 prefetch of rows [r0, r0+nr) of W (quant bytes and per-block scales).
// Tile byte ranges of the device layout start on 16-byte boundaries.
__device__ void prefetch_rows(const DevTensor &W, int r0, int nr) {
  size_t rq = 0, rd = 0;
  switch (W.type) {
    case T_Q4_K: rq = (size_t)(W.k >> 8) * 144; break;
    case T_Q6_K: rq = (size_t)(W.k >> 8) * 208; rd = (size_t)(W.k >> 8) * 2; break;
    case T_Q8_0: rq = (size_t)W.k; rd = (size_t)(W.k >> 5) * 2; break;
    case T_Q4_0: rq = (size_t)(W.k >> 1); rd = (size_t)(W.k >> 5) * 2; break;
    default: return;
  }
  const uint8_t *q = W.q + (size_t)r0 * rq;
  if (((uintptr_t)q & 15) == 0) prefetch_l2(q, (uint32_t)(rq * nr));
  if (rd) {
    const uint8_t *d = reinterpret_cast<const uint8_t *>(W.d) + (size_t)r0 * rd;
    if (((uintptr_t)d & 15) == 0) prefetch_l2(d, (uint32_t)(rd * nr));
  }
}

__device__ float tile_b1_any(const DevTensor &W, int r0, int nr, const ActRef &A, float *Tsm) {
  switch (W.type) {
    case T_Q4_K: return tile_b1<T_Q4_K>(W, r0, nr, A, Tsm);
    case T_Q6_K: return tile_b1<T_Q6_K>(W, r0, nr, A, Tsm);
    case T_Q8_0: return tile_b1<T_Q8_0>(W, r0, nr, A, Tsm);
    default: return tile_b1<T_Q4_0>(W, r0, nr, A, Tsm);
  }
}

struct B1Smem {
  int8_t *q;
  float *d;
  int32_t *s;
  float *T;
  float *red;
  float *xv;
};

static size_t b1_smem_bytes(int k) {
  const size_t nb = (size_t)k / 32;
  return ((size_t)k + 15) / 16 * 16 + nb * 4 + nb * 4 + (size_t)B1_TW * B1_RT * 4 + 40 * 4 + B1_RT * 4 * 2;
}

__device__ B1Smem b1_carve(uint8_t *base, int k) {
  B1Smem m;
  const int nb = k >> 5;
  m.q = (int8_t *)base;
  size_t off = ((size_t)k + 15) / 16 * 16;
  m.d = (float *)(base + off);
  off += (size_t)nb * 4;
  m.s = (int32_t *)(base + off);
  off += (size_t)nb * 4;
  m.T = (float *)(base + off);
  off += (size_t)B1_TW * B1_RT * 4;
  m.red = (float *)(base + off);
  off += 40 * 4;
  m.xv = (float *)(base + off);
  return m;
}

// Fill the CTA's shared Q8 activation from a float vector (optionally RMS
// normalised, model.rs:795-809 / 812-822) or from a precomputed Q8Act.
__device__ void act_prologue(const B1Src &src, int k, const B1Smem &m) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nb = k >> 5;
  if (src.x == nullptr) {
    const int4 *sq = reinterpret_cast<const int4 *>(src.act.q);
    for (int i = tid; i < k / 16; i += blockDim.x) reinterpret_cast<int4 *>(m.q)[i] = sq[i];
    for (int i = tid; i < nb; i += blockDim.x) {
      m.d[i] = src.act.d[i];
      m.s[i] = src.act.s[i];
    }
    __syncthreads();
    return;
  }
  float scale = 1.0f;
  if (src.nw) {  // model.rs:791-810: the b == 1 rmsnorm
    const float ss = sum_sq_neon(src.x, k, m.red);
    scale = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(ss, (float)k), src.eps)));
  }
  for (int blk = warp; blk < nb; blk += blockDim.x >> 5) {
    float v = src.x[blk * 32 + lane];
    if (src.nw) v = fmul(fmul(v, scale), src.nw[blk * 32 + lane]);
    q8_block_lane(v, lane, m.q + blk * 32, m.d + blk, m.s + blk);
  }
  __syncthreads();
}

__global__ void __launch_bounds__(B1_THREADS, B1_MIN_CTAS) k_mv_b1(DevTensor W, B1Src src, float *__restrict__ out, int add) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int tiles = (W.rows + B1_RT - 1) / B1_RT;
  if (threadIdx.x == 0)  // weights are constant: stream them in while the previous kernel runs
    for (int t = blockIdx.x, i = 0; t < tiles && i < 2; t += gridDim.x, i++)
      prefetch_rows(W, t * B1_RT, min(B1_RT, W.rows - t * B1_RT));
  pdl_trigger();
  pdl_wait();
  const B1Smem m = b1_carve(smem_raw, W.k);
  act_prologue(src, W.k, m);
  const ActRef A{m.q, m.d, m.s};
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int r0 = t * B1_RT, nr = min(B1_RT, W.rows - r0);
    const int tn = t + 2 * gridDim.x;  // two tiles ahead of this CTA's current one
    if (threadIdx.x == 0 && tn < tiles) prefetch_rows(W, tn * B1_RT, min(B1_RT, W.rows - tn * B1_RT));
    const float acc = tile_b1_any(W, r0, nr, A, m.T);
    if ((int)threadIdx.x < nr) {
      const float v = fadd(0.0f, acc);  // Pool::matmul zero-fills, then out += acc
      const int r = r0 + threadIdx.x;
      out[r] = add ? fadd(out[r], v) : v;
    }
  }
}

// One CTA per tile, at most as many as fit on the GPU at once (the kernel's
// registers and shared memory, from the occupancy calculator, cached per
// kernel and size).
template <typename K>
static int b1_grid(K kernel, int tiles, size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<const void *, size_t>, int> per_sm_of;
  int per_sm = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = per_sm_of.find({(const void *)kernel, smem});
    if (it != per_sm_of.end()) per_sm = it->second;
  }
  if (per_sm == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, B1_THREADS, smem) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    std::lock_guard<std::mutex> lock(mu);
    per_sm_of[{(const void *)kernel, smem}] = per_sm;
  }
  return std::max(1, std::min(tiles, num_sms() * per_sm));
}

cudaError_t launch_mv_b1(const DevTensor &w, const B1Src &src, float *out, bool add, cudaStream_t st) {
  if (!type_is_matvec(w.type)) return cudaErrorInvalidValue;
  const size_t smem = b1_smem_bytes(w.k);
  cudaError_t e = set_smem(k_mv_b1, smem);
  if (e != cudaSuccess) return e;
  const int tiles = (w.rows + B1_RT - 1) / B1_RT;
  return launch(k_mv_b1, dim3(b1_grid(k_mv_b1, tiles, smem)), dim3(B1_THREADS), smem, st, w, src, out, add ? 1 : 0);
}

// q/k/v for one token + RoPE (model.rs:953-979) + KV write (model.rs:984-992).
__global__ void __launch_bounds__(B1_THREADS, B1_MIN_CTAS) k_qkv_b1(QkvArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int tq = (a.wq.rows + B1_RT - 1) / B1_RT, tk = (a.wk.rows + B1_RT - 1) / B1_RT,
            tv = (a.wv.rows + B1_RT - 1) / B1_RT;
  if (threadIdx.x == 0)
    for (int t = blockIdx.x, i = 0; t < tq + tk + tv && i < 2; t += gridDim.x, i++) {
      const int seg = t < tq ? 0 : (t < tq + tk ? 1 : 2);
      const int tt = seg == 0 ? t : (seg == 1 ? t - tq : t - tq - tk);
      const DevTensor &W = seg == 0 ? a.wq : (seg == 1 ? a.wk : a.wv);
      prefetch_rows(W, tt * B1_RT, min(B1_RT, W.rows - tt * B1_RT));
    }
  pdl_trigger();
  pdl_wait();
  const B1Smem m = b1_carve(smem_raw, a.wq.k);
  act_prologue(a.src, a.wq.k, m);
  const ActRef A{m.q, m.d, m.s};
  const int pos = *a.pos;
  const int tid = threadIdx.x;
  for (int t = blockIdx.x; t < tq + tk + tv; t += gridDim.x) {
    const int seg = t < tq ? 0 : (t < tq + tk ? 1 : 2);
    const int tt = seg == 0 ? t : (seg == 1 ? t - tq : t - tq - tk);
    const DevTensor &W = seg == 0 ? a.wq : (seg == 1 ? a.wk : a.wv);
    const int r0 = tt * B1_RT, nr = min(B1_RT, W.rows - r0);
    const float acc = tile_b1_any(W, r0, nr, A, m.T);
    const float val = fadd(0.0f, acc);
    if (tid < nr) m.xv[tid] = val;
    __syncthreads();
    if (tid < nr) {
      const int r = r0 + tid, hd = r / a.dh, d = r - hd * a.dh;
      float o = val;
      if (seg < 2 && d < 2 * a.half) {
        const int i = d >> 1;
        const float c = a.rope_cos[(size_t)pos * a.half + i], s = a.rope_sin[(size_t)pos * a.half + i];
        if ((d & 1) == 0) o = fsub(fmul(val, c), fmul(m.xv[tid + 1], s));
        else o = fadd(fmul(m.xv[tid - 1], s), fmul(val, c));
      }
      const size_t ki = ((size_t)hd * a.dh + d) * a.n_ctx + pos, vi = ((size_t)hd * a.n_ctx + pos) * a.dh + d;
      if (seg == 0) a.qout[r] = o;
      else if (a.kv16) {
        if (seg == 1) kv_put<true>(a.kcache, ki, o);  // K is d-major
        else kv_put<true>(a.vcache, vi, o);
      } else {
        if (seg == 1) a.kcache[ki] = o;
        else a.vcache[vi] = o;
      }
    }
    __syncthreads();
  }
}

cudaError_t launch_qkv_b1(const QkvArgs &a, cudaStream_t st) {
  if (!type_is_matvec(a.wq.type) || !type_is_matvec(a.wk.type) || !type_is_matvec(a.wv.type)) return cudaErrorInvalidValue;
  const size_t smem = b1_smem_bytes(a.wq.k);
  cudaError_t e = set_smem(k_qkv_b1, smem);
  if (e != cudaSuccess) return e;
  const int tiles = (a.wq.rows + B1_RT - 1) / B1_RT + (a.wk.rows + B1_RT - 1) / B1_RT + (a.wv.rows + B1_RT - 1) / B1_RT;
  return launch(k_qkv_b1, dim3(b1_grid(k_qkv_b1, tiles, smem)), dim3(B1_THREADS), smem, st, a);
}

// gate/up for one token + SwiGLU (model.rs:1105-1115).
__global__ void __launch_bounds__(B1_THREADS, B1_MIN_CTAS) k_gateup_b1(DevTensor wg, DevTensor wu, B1Src src, float *__restrict__ h) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int tiles = (wg.rows + B1_RT - 1) / B1_RT;
  if (threadIdx.x == 0)
    for (int t = blockIdx.x, i = 0; t < tiles && i < 2; t += gridDim.x, i++) {
      prefetch_rows(wg, t * B1_RT, min(B1_RT, wg.rows - t * B1_RT));
      prefetch_rows(wu, t * B1_RT, min(B1_RT, wu.rows - t * B1_RT));
    }
  pdl_trigger();
  pdl_wait();
  const B1Smem m = b1_carve(smem_raw, wg.k);
  act_prologue(src, wg.k, m);
  const ActRef A{m.q, m.d, m.s};
  for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int r0 = t * B1_RT, nr = min(B1_RT, wg.rows - r0);
    const float ag = tile_b1_any(wg, r0, nr, A, m.T);
    const float au = tile_b1_any(wu, r0, nr, A, m.T);
    if ((int)threadIdx.x < nr) {
      const float g = fadd(0.0f, ag), u = fadd(0.0f, au);
      const float s = fdiv(g, fadd(1.0f, expf_lib(-g)));
      h[r0 + threadIdx.x] = fmul(s, u);
    }
  }
}

cudaError_t launch_gateup_b1(const DevTensor &wg, const DevTensor &wu, const B1Src &src, float *h, cudaStream_t st) {
  if (!type_is_matvec(wg.type) || !type_is_matvec(wu.type) || wg.rows != wu.rows || wg.k != wu.k)
    return cudaErrorInvalidValue;
  const size_t smem = b1_smem_bytes(wg.k);
  cudaError_t e = set_smem(k_gateup_b1, smem);
  if (e != cudaSuccess) return e;
  const int tiles = (wg.rows + B1_RT - 1) / B1_RT;
  return launch(k_gateup_b1, dim3(b1_grid(k_gateup_b1, tiles, smem)), dim3(B1_THREADS), smem, st, wg, wu, src, h);
}

// ------------------------------------------------- multi-lane matvec, tensor cores
// b > 1 (prefill chunks, Pool::matmul with several lanes).  The reference adds
// one float term per (row, lane, sub-block) in sub-block order
// (quant_int.rs:282-419).  Each sub-block's integer dot is one element of an
// int8 mma.sync tile (m16n8k32 per 32-element sub-block, m16n8k16 per
// 16-element Q6_K piece), exact in int32; every thread turns its four tile
// elements into the reference's float terms (operand order as in the scalar
// path) and adds them, sub-block after sub-block, to the running sums.  A
// tile is 16 rows x 32 lanes (four lane groups of 8); the tile's rows and
// the lanes' activation scales are staged in shared memory one k-chunk at a
// time.  mv_tile below has the details.
constexpr int MM_WARPS = 4;
constexpr int MM_ROWS = 16;
constexpr int MM_LANES = 8 * MM_WARPS;

// Integer tile products.  The accumulator starts at DOT_BIAS, the bit
// pattern of 1.5 * 2^23, so each result is the float 12582912 + dot exactly
// (|dot| < 2^20 here) and unbias() turns it into the float dot.
constexpr int DOT_BIAS = 0x4B400000;
__device__ __forceinline__ float unbias(int d) { return fsub(__int_as_float(d), 12582912.0f); }
__device__ __forceinline__ void mma_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(DOT_BIAS));
}
__device__ __forceinline__ void mma_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%7,%7,%7};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0), "r"(DOT_BIAS));
}
__device__ __forceinline__ uint32_t ldg_u32(const int8_t *p) { return __ldg(reinterpret_cast<const uint32_t *>(p)); }
// Asynchronous global -> shared copies (completed by cp_async_wait_all).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_all;" ::: "memory");
}

template <int T> struct MmGeo;
template <> struct MmGeo<T_Q4_K> { static constexpr int BE = 256, QB = 144; static constexpr bool D = false; };
template <> struct MmGeo<T_Q6_K> { static constexpr int BE = 256, QB = 208; static constexpr bool D = true; };
template <> struct MmGeo<T_Q8_0> { static constexpr int BE = 32, QB = 32; static constexpr bool D = true; };
template <> struct MmGeo<T_Q4_0> { static constexpr int BE = 32, QB = 16; static constexpr bool D = true; };

// Lane stride (in float2) of the staged activation scales: odd, so the four
// lane pairs a warp reads at once fall in different banks.
__host__ __device__ inline int mm_lane_stride(int sbc) { return sbc | 1; }
constexpr int MM_RELAY_BYTES = 4 * 32 * 16;  // one float4 per thread of each lane group
// Storage blocks per staged chunk of a matrix of nblk blocks, so that the
// chunk's rows and lane scales fit in smem_bytes of shared memory; Q8_0 /
// Q4_0 chunks hold whole 8-block units.
template <int T>
__host__ __device__ inline int mm_nbc(int nblk, int smem_bytes) {
  const int per_block = MM_ROWS * (MmGeo<T>::QB + (MmGeo<T>::D ? 4 : 0)) + MM_LANES * (MmGeo<T>::BE / 32) * 8;
  int n = (smem_bytes - MM_RELAY_BYTES - MM_LANES * 8) / per_block;
  if (MmGeo<T>::BE == 32) n &= ~7;
  return nblk < n ? nblk : n;
}
template <int T>
__host__ __device__ inline size_t mm_smem_bytes(int nbc) {
  return (size_t)MM_ROWS * nbc * (MmGeo<T>::QB + (MmGeo<T>::D ? 4 : 0)) +
         (size_t)MM_LANES * mm_lane_stride(nbc * MmGeo<T>::BE / 32) * 8 + MM_RELAY_BYTES;
}

// Exact int -> float conversions on the integer/FP32 pipes: x + 1.5*2^23 as
// a float bit pattern is exact for |x| < 2^22, and a byte placed under the
// exponent of 2^23 is 2^23 + byte.
__device__ __forceinline__ float dotf(int x) { return fsub(__int_as_float(x + 0x4B400000), 12582912.0f); }
template <int B>
__device__ __forceinline__ float bytef(uint32_t w) {  // byte B of w (a value below 256)
  return fsub(__int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7540u + B)), 8388608.0f);
}
__device__ __forceinline__ uint2 ldg_u2(const int8_t *p) { return __ldg(reinterpret_cast<const uint2 *>(p)); }
// Named barriers 1 + s (s < 8) with immediate ids, so the kernel holds only
// the barriers it uses.
__device__ __forceinline__ void mm_bar_sync(int s, int n) {
  switch (s) {
    case 0: asm volatile("bar.sync 1, %0;" ::"r"(n) : "memory"); break;
    case 1: asm volatile("bar.sync 2, %0;" ::"r"(n) : "memory"); break;
    case 2: asm volatile("bar.sync 3, %0;" ::"r"(n) : "memory"); break;
    case 3: asm volatile("bar.sync 4, %0;" ::"r"(n) : "memory"); break;
    case 4: asm volatile("bar.sync 5, %0;" ::"r"(n) : "memory"); break;
    case 5: asm volatile("bar.sync 6, %0;" ::"r"(n) : "memory"); break;
    case 6: asm volatile("bar.sync 7, %0;" ::"r"(n) : "memory"); break;
    default: asm volatile("bar.sync 8, %0;" ::"r"(n) : "memory"); break;
  }
}
__device__ __forceinline__ void mm_bar_arrive(int s, int n) {
  switch (s) {
    case 0: asm volatile("bar.arrive 1, %0;" ::"r"(n) : "memory"); break;
    case 1: asm volatile("bar.arrive 2, %0;" ::"r"(n) : "memory"); break;
    case 2: asm volatile("bar.arrive 3, %0;" ::"r"(n) : "memory"); break;
    case 3: asm volatile("bar.arrive 4, %0;" ::"r"(n) : "memory"); break;
    case 4: asm volatile("bar.arrive 5, %0;" ::"r"(n) : "memory"); break;
    case 5: asm volatile("bar.arrive 6, %0;" ::"r"(n) : "memory"); break;
    case 6: asm volatile("bar.arrive 7, %0;" ::"r"(n) : "memory"); break;
    default: asm volatile("bar.arrive 8, %0;" ::"r"(n) : "memory"); break;
  }
}

// One 16-row x 8LG-lane tile (row tile bx, lane tile blockIdx.y) of out = W * act.
//
// Work unit: eight consecutive float terms of every (row, lane) of the tile
// (a Q4_K superblock, half a Q6_K superblock, eight Q8_0 / Q4_0 blocks).
// Warp w is lane group lw = w % LG (lanes 8lw .. 8lw+7) and k slice
// ks = w / LG of KS: units are dealt to the slices round robin, each slice
// forms its unit's terms in registers, then adds them to the running sums
// of the (row, lane) pairs, which pass from slice to slice through shared
// memory (named barrier 1 + s is the hand-off into slice s).  So every sum
// is still the reference's sequential one, term after term.
//
// Integer dots are independent of the order of the 32 products, so for
// Q4_K / Q8_0 the k slots of a sub-block are permuted: thread t's A and B
// fragment slots 4t..4t+3 and 16+4t..16+4t+3 carry elements 8t..8t+7 of
// the weight row and of the activation lane (one 64-bit load each).
template <int T, int KS, int LG>
__device__ __forceinline__ void mv_tile(const DevTensor &W, const Q8Dev &act, float *out, long os_row, long os_lane,
                                        int add, int bx, int NBC, uint8_t *mm_smem) {
  using G = MmGeo<T>;
  constexpr int UPB = T == T_Q6_K ? 2 : 1;             // units per storage block (K-quants)
  constexpr bool KQ = G::BE == 256;
  const int SBC = NBC * G::BE / 32;                     // 32-element activation blocks per chunk
  const int LS = mm_lane_stride(SBC);
  uint8_t *wq = mm_smem;                                // [16 rows][NBC][QB]
  float *wd = (float *)(mm_smem + MM_ROWS * NBC * G::QB);  // [16 rows][NBC] (types with a separate d)
  float2 *asf = (float2 *)(mm_smem + MM_ROWS * NBC * (G::QB + (G::D ? 4 : 0)));  // [32 lanes][LS] {da, sa}
  float4 *relay = (float4 *)(asf + MM_LANES * LS);     // [lane groups][32]
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
  const int lw = w % LG, ks = w / LG;
  const int r0 = bx * MM_ROWS, nr = min(MM_ROWS, W.rows - r0);
  const int L0 = blockIdx.y * 8 * LG, nl = min(8 * LG, act.b - L0);
  const int nact = (nl + 7) >> 3;                      // lane groups with lanes
  const bool active = lw < nact;
  const int k = W.k, nblk = k / G::BE, nb32 = k >> 5;
  const int units = KQ ? nblk * UPB : (nblk + 7) >> 3;  // units of the whole row
  const int lbc = min(L0 + 8 * lw + g, act.b - 1);     // lane of this thread's B fragment loads
  const int lc0 = 8 * lw + 2 * t, lc1 = lc0 + 1;        // local lanes of this thread's accumulators
  const int8_t *aq = act.q + (long)lbc * k;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};             // (row g, lc0), (g, lc1), (g + 8, lc0), (g + 8, lc1)
  const size_t row_q = (size_t)nblk * G::QB;
  for (int c0 = 0; c0 < nblk; c0 += NBC) {
    const int nbc = min(NBC, nblk - c0);
    __syncthreads();  // the previous chunk is consumed
    // stage: the tile's rows and the lanes' activation scales by asynchronous
    // copies (every copy in flight at once), the f16 row scales by plain loads;
    // warps take rows (lanes), lanes take pieces, so no index is divided
    constexpr int NW = LG * KS;
    const int v16 = nbc * G::QB / 16;
    for (int r = w; r < nr; r += NW)
      for (int j = lane; j < v16; j += 32)
        cp_async16(wq + (size_t)r * NBC * G::QB + 16 * j, W.q + (size_t)(r0 + r) * row_q + (size_t)c0 * G::QB + 16 * j);
    const int s0 = c0 * (G::BE / 32), nsb = nbc * (G::BE / 32);
    for (int l = w; l < nl; l += NW) {
      const long o = (long)(L0 + l) * nb32 + s0;
      for (int j = lane; j < nsb; j += 32) {
        cp_async4(&asf[l * LS + j].x, act.d + o + j);
        cp_async4(&asf[l * LS + j].y, act.s + o + j);
      }
    }
    if (G::D)
      for (int r = w; r < nr; r += NW)
        for (int j = lane; j < nbc; j += 32) wd[r * NBC + j] = f16f(__ldg(W.d + (size_t)(r0 + r) * nblk + c0 + j));
    cp_async_wait_all();
    // the block sums as floats (each thread converts the entries it copied)
    for (int l = w; l < nl; l += NW)
      for (int j = lane; j < nsb; j += 32) {
        float *sp = &asf[l * LS + j].y;
        *sp = (float)__float_as_int(*sp);
      }
    __syncthreads();
    if (!active) continue;  // no lanes for this warp (it still meets every __syncthreads)
    const uint8_t *qa = wq + (size_t)g * NBC * G::QB, *qb = wq + (size_t)(g + 8) * NBC * G::QB;
    const float2 *as0 = asf + lc0 * LS, *as1 = asf + lc1 * LS;
    const int ubase = KQ ? c0 * UPB : c0 >> 3;            // global index of the chunk's first unit
    const int nu = KQ ? nbc * UPB : (nbc + 7) >> 3;       // units in this chunk
    // B fragments of unit u of this chunk (16 words; 8 for a Q6_K half)
    auto load_b = [&](int u, uint32_t (&bw)[16]) {
      if (T == T_Q6_K) {
        const int8_t *ap = aq + (size_t)(c0 + (u >> 1)) * 256 + (u & 1) * 128;
#pragma unroll
        for (int e = 0; e < 8; e++) bw[e] = ldg_u32(ap + (e & 3) * 32 + (e >> 2) * 16 + 4 * t);  // piece (4h+s, g2), e = 4 g2 + s
      } else if (T == T_Q4_K) {
        const int8_t *ap = aq + (size_t)(c0 + u) * 256;
#pragma unroll
        for (int e = 0; e < 8; e++) {  // sub-block e, permuted slots
          const uint2 v = ldg_u2(ap + e * 32 + 8 * t);
          bw[2 * e] = v.x;
          bw[2 * e + 1] = v.y;
        }
      } else {
        const int8_t *ap = aq + (size_t)(c0 + 8 * u) * 32;
        const int nv = min(8, nbc - 8 * u);
#pragma unroll
        for (int e = 0; e < 8; e++) {
          if (T == T_Q8_0) {
            const uint2 v = e < nv ? ldg_u2(ap + e * 32 + 8 * t) : make_uint2(0u, 0u);
            bw[2 * e] = v.x;
            bw[2 * e + 1] = v.y;
          } else {
            bw[2 * e] = e < nv ? ldg_u32(ap + e * 32 + 4 * t) : 0u;
            bw[2 * e + 1] = e < nv ? ldg_u32(ap + e * 32 + 16 + 4 * t) : 0u;
          }
        }
      }
    };
    // the eight terms of unit u for this thread's four (row, lane) pairs
    auto unit_terms = [&](int u, const uint32_t (&bc)[16], float (&tm)[8][4]) {
      if (T == T_Q4_K) {
        const int i = u;
        const uint4 ha = *reinterpret_cast<const uint4 *>(qa + i * 144), hb = *reinterpret_cast<const uint4 *>(qb + i * 144);
        const float da_r = f16f((uint16_t)(ha.x & 0xFFFFu)), dm_r = f16f((uint16_t)(ha.x >> 16));
        const float db_r = f16f((uint16_t)(hb.x & 0xFFFFu)), dmb_r = f16f((uint16_t)(hb.x >> 16));
        // get_scale_min_k4 (quant.rs:80-86), a byte per sub-block
        const uint32_t sca_lo = ha.y & 0x3F3F3F3Fu, ma_lo = ha.z & 0x3F3F3F3Fu;
        const uint32_t sca_hi = (ha.w & 0x0F0F0F0Fu) | ((ha.y >> 2) & 0x30303030u);
        const uint32_t ma_hi = ((ha.w >> 4) & 0x0F0F0F0Fu) | ((ha.z >> 2) & 0x30303030u);
        const uint32_t scb_lo = hb.y & 0x3F3F3F3Fu, mb_lo = hb.z & 0x3F3F3F3Fu;
        const uint32_t scb_hi = (hb.w & 0x0F0F0F0Fu) | ((hb.y >> 2) & 0x30303030u);
        const uint32_t mb_hi = ((hb.w >> 4) & 0x0F0F0F0Fu) | ((hb.z >> 2) & 0x30303030u);
#pragma unroll
        for (int p = 0; p < 4; p++) {
          const uint2 wa = *reinterpret_cast<const uint2 *>(qa + i * 144 + 16 + 32 * p + 8 * t);
          const uint2 wb = *reinterpret_cast<const uint2 *>(qb + i * 144 + 16 + 32 * p + 8 * t);
#pragma unroll
          for (int h = 0; h < 2; h++) {
            const int j = 2 * p + h, sl = i * 8 + j;
            const uint32_t M = 0x0F0F0F0Fu;
            const uint32_t x0 = h ? (wa.x >> 4) & M : wa.x & M, x1 = h ? (wb.x >> 4) & M : wb.x & M;
            const uint32_t x2 = h ? (wa.y >> 4) & M : wa.y & M, x3 = h ? (wb.y >> 4) & M : wb.y & M;
            int dot[4];
            mma_k32(dot, x0, x1, x2, x3, bc[2 * j], bc[2 * j + 1]);
            const float2 a0 = as0[sl], a1 = as1[sl];
            const uint32_t sa_w = j < 4 ? sca_lo : sca_hi, ma_w = j < 4 ? ma_lo : ma_hi;
            const uint32_t sb_w = j < 4 ? scb_lo : scb_hi, mb_w = j < 4 ? mb_lo : mb_hi;
            float sca, mma_, scb, mmb;
            switch (j & 3) {
              case 0: sca = bytef<0>(sa_w); mma_ = bytef<0>(ma_w); scb = bytef<0>(sb_w); mmb = bytef<0>(mb_w); break;
              case 1: sca = bytef<1>(sa_w); mma_ = bytef<1>(ma_w); scb = bytef<1>(sb_w); mmb = bytef<1>(mb_w); break;
              case 2: sca = bytef<2>(sa_w); mma_ = bytef<2>(ma_w); scb = bytef<2>(sb_w); mmb = bytef<2>(mb_w); break;
              default: sca = bytef<3>(sa_w); mma_ = bytef<3>(ma_w); scb = bytef<3>(sb_w); mmb = bytef<3>(mb_w); break;
            }
            tm[j][0] = fsub(fmul(fmul(fmul(da_r, a0.x), sca), unbias(dot[0])), fmul(fmul(fmul(a0.x, dm_r), mma_), a0.y));
            tm[j][1] = fsub(fmul(fmul(fmul(da_r, a1.x), sca), unbias(dot[1])), fmul(fmul(fmul(a1.x, dm_r), mma_), a1.y));
            tm[j][2] = fsub(fmul(fmul(fmul(db_r, a0.x), scb), unbias(dot[2])), fmul(fmul(fmul(a0.x, dmb_r), mmb), a0.y));
            tm[j][3] = fsub(fmul(fmul(fmul(db_r, a1.x), scb), unbias(dot[3])), fmul(fmul(fmul(a1.x, dmb_r), mmb), a1.y));
          }
        }
      } else if (T == T_Q6_K) {
        // half h of superblock i: pieces (sub-block 4h+s, 16-half g2) in the
        // reference's order g2 = 0, 1, then s = 0..3 (quant_int.rs:380-405)
        const int i = u >> 1, h = u & 1;
        const float dra = wd[g * NBC + i], drb = wd[(g + 8) * NBC + i];
        const uint8_t *ba = qa + i * 208, *bb = qb + i * 208;
        const uint2 sa2 = *reinterpret_cast<const uint2 *>(ba + 192 + 8 * h);
        const uint2 sb2 = *reinterpret_cast<const uint2 *>(bb + 192 + 8 * h);
#pragma unroll
        for (int g2 = 0; g2 < 2; g2++) {
          const uint32_t la0 = *reinterpret_cast<const uint32_t *>(ba + h * 64 + g2 * 16 + 4 * t);
          const uint32_t la1 = *reinterpret_cast<const uint32_t *>(ba + h * 64 + 32 + g2 * 16 + 4 * t);
          const uint32_t lha = *reinterpret_cast<const uint32_t *>(ba + 128 + h * 32 + g2 * 16 + 4 * t);
          const uint32_t lb0 = *reinterpret_cast<const uint32_t *>(bb + h * 64 + g2 * 16 + 4 * t);
          const uint32_t lb1 = *reinterpret_cast<const uint32_t *>(bb + h * 64 + 32 + g2 * 16 + 4 * t);
          const uint32_t lhb = *reinterpret_cast<const uint32_t *>(bb + 128 + h * 32 + g2 * 16 + 4 * t);
#pragma unroll
          for (int s = 0; s < 4; s++) {
            // quant_int.rs:386-394 unpacking, four bytes at a time, minus 32
            auto unpack = [&](uint32_t l0w, uint32_t l1w, uint32_t hw) {
              const uint32_t lo = s & 1 ? l1w : l0w;
              const uint32_t q = ((s & 2 ? lo >> 4 : lo) & 0x0F0F0F0Fu) |
                                 ((s == 0 ? hw << 4 : s == 1 ? hw << 2 : s == 2 ? hw : hw >> 2) & 0x30303030u);
              return __vsub4(q, 0x20202020u);
            };
            int dot[4];
            mma_k16(dot, unpack(la0, la1, lha), unpack(lb0, lb1, lhb), bc[4 * g2 + s]);
            const float2 a0 = as0[i * 8 + 4 * h + s], a1 = as1[i * 8 + 4 * h + s];
            // the signed scale byte (g2 + 2s) of this half, exactly, on the integer pipe
            const int sh = 8 * (g2 + 2 * s);
            const uint32_t swa = sh < 32 ? sa2.x : sa2.y, swb = sh < 32 ? sb2.x : sb2.y;
            const float sca = dotf((int)(int8_t)(uint8_t)(swa >> (sh & 31)));
            const float scb = dotf((int)(int8_t)(uint8_t)(swb >> (sh & 31)));
            tm[4 * g2 + s][0] = fmul(fmul(fmul(dra, sca), a0.x), unbias(dot[0]));
            tm[4 * g2 + s][1] = fmul(fmul(fmul(dra, sca), a1.x), unbias(dot[1]));
            tm[4 * g2 + s][2] = fmul(fmul(fmul(drb, scb), a0.x), unbias(dot[2]));
            tm[4 * g2 + s][3] = fmul(fmul(fmul(drb, scb), a1.x), unbias(dot[3]));
          }
        }
      } else {  // Q8_0 / Q4_0: one 32-element block per term
        const int nv = min(8, nbc - 8 * u);
#pragma unroll
        for (int e = 0; e < 8; e++) {
          if (e >= nv) {  // past the row's last block: +0.0 terms (adding them is exact)
            tm[e][0] = tm[e][1] = tm[e][2] = tm[e][3] = 0.0f;
            continue;
          }
          const int i = 8 * u + e;
          const float dra = wd[g * NBC + i], drb = wd[(g + 8) * NBC + i];
          uint32_t x0, x1, x2, x3;
          if (T == T_Q8_0) {  // permuted slots: elements 8t..8t+7
            const uint2 wa = *reinterpret_cast<const uint2 *>(qa + i * 32 + 8 * t);
            const uint2 wb = *reinterpret_cast<const uint2 *>(qb + i * 32 + 8 * t);
            x0 = wa.x;
            x2 = wa.y;
            x1 = wb.x;
            x3 = wb.y;
          } else {  // low nibbles = elements 0-15, high = 16-31
            const uint32_t wa = *reinterpret_cast<const uint32_t *>(qa + i * 16 + 4 * t);
            const uint32_t wb = *reinterpret_cast<const uint32_t *>(qb + i * 16 + 4 * t);
            x0 = wa & 0x0F0F0F0Fu;
            x2 = (wa >> 4) & 0x0F0F0F0Fu;
            x1 = wb & 0x0F0F0F0Fu;
            x3 = (wb >> 4) & 0x0F0F0F0Fu;
          }
          int dot[4];
          mma_k32(dot, x0, x1, x2, x3, bc[2 * e], bc[2 * e + 1]);
          const float2 a0 = as0[i], a1 = as1[i];
          if (T == T_Q8_0) {  // quant_int.rs:291-296
            tm[e][0] = fmul(fmul(dra, a0.x), unbias(dot[0]));
            tm[e][1] = fmul(fmul(dra, a1.x), unbias(dot[1]));
            tm[e][2] = fmul(fmul(drb, a0.x), unbias(dot[2]));
            tm[e][3] = fmul(fmul(drb, a1.x), unbias(dot[3]));
          } else {  // quant_int.rs:316-323
            tm[e][0] = fmul(fmul(dra, a0.x), fsub(unbias(dot[0]), fmul(8.0f, a0.y)));
            tm[e][1] = fmul(fmul(dra, a1.x), fsub(unbias(dot[1]), fmul(8.0f, a1.y)));
            tm[e][2] = fmul(fmul(drb, a0.x), fsub(unbias(dot[2]), fmul(8.0f, a0.y)));
            tm[e][3] = fmul(fmul(drb, a1.x), fsub(unbias(dot[3]), fmul(8.0f, a1.y)));
          }
        }
      }
    };
    const int nbar = 64 * nact;  // one hand-off: the active lane groups' sender and receiver warps
    int u = ((ks - ubase) % KS + KS) % KS;  // this slice's first unit of the chunk
    // With four or more slices each unit's B fragments are loaded one unit
    // ahead; with one, the other resident warps cover the load.
    constexpr bool AHEAD = KS >= 4;
    uint32_t bc[16], bn[16];
    if (AHEAD && u < nu) load_b(u, bc);
    for (; u < nu; u += KS) {
      if (AHEAD && u + KS < nu) load_b(u + KS, bn);
      if (!AHEAD) load_b(u, bc);
      float tm[8][4];
      unit_terms(u, bc, tm);
      const int gu = ubase + u;
      if (KS > 1 && gu > 0) {  // take the running sums from the previous unit's slice
        mm_bar_sync(ks, nbar);
        const float4 r = relay[lw * 32 + lane];
        acc[0] = r.x; acc[1] = r.y; acc[2] = r.z; acc[3] = r.w;
      }
#pragma unroll
      for (int j = 0; j < 8; j++) {
#pragma unroll
        for (int e = 0; e < 4; e++) acc[e] = fadd(acc[e], tm[j][e]);
      }
      if (KS > 1 && gu + 1 < units) {  // and hand them to the next unit's slice
        relay[lw * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        mm_bar_arrive((ks + 1) % KS, nbar);
      }
      if (AHEAD) {
#pragma unroll
        for (int e = 0; e < 16; e++) bc[e] = bn[e];
      }
    }
  }
  // the slice of the last unit holds the final sums:
  // out = 0.0 + acc (Pool::matmul zero-fills, then adds), or x += that
  if (!active || ks != (units - 1) % KS) return;
#pragma unroll
  for (int e = 0; e < 4; e++) {
    const int r = g + (e >> 1) * 8, l = (e & 1) ? lc1 : lc0;
    if (r < nr && l < nl) {
      float *o = out + (long)(r0 + r) * os_row + (long)(L0 + l) * os_lane;
      const float v = fadd(0.0f, acc[e]);
      *o = add ? fadd(*o, v) : v;
    }
  }
}

// Up to three matrices against one activation in one launch (q/k/v,
// gate/up): CTA x-index ranges [cta0, next cta0) belong to segment s.
struct MvSeg {
  DevTensor W;
  float *out;
  long os_row, os_lane;
  int add, cta0, nbc;
};
constexpr int MV_MAX_SEGS = 3;
struct MvSegs {
  MvSeg s[MV_MAX_SEGS];
  int n;
};

// KS k slices of LG lane groups: (1, 4) and (4, 4) for b > 8, (4, 1) and
// (8, 1) for b <= 8, where one lane group holds every lane and the slices
// keep all warps busy.
template <int KS, int LG>
__global__ void __launch_bounds__(32 * LG * KS, KS == 1 ? 5 : KS * LG == 4 ? 4 : 1) k_mv_mma(MvSegs ss, Q8Dev act) {
  extern __shared__ __align__(16) uint8_t mm_smem[];
  const int bx = blockIdx.x;
  const MvSeg &S = (ss.n > 2 && bx >= ss.s[2].cta0) ? ss.s[2] : (ss.n > 1 && bx >= ss.s[1].cta0) ? ss.s[1] : ss.s[0];
  const int tb = bx - S.cta0;
  // the tile's rows are constant: bring them into L2 while the previous kernel runs
  if (threadIdx.x == 0 && blockIdx.y == 0) prefetch_rows(S.W, tb * MM_ROWS, min(MM_ROWS, S.W.rows - tb * MM_ROWS));
  pdl_trigger();
  pdl_wait();
  switch (S.W.type) {
    case T_Q4_K: mv_tile<T_Q4_K, KS, LG>(S.W, act, S.out, S.os_row, S.os_lane, S.add, tb, S.nbc, mm_smem); break;
    case T_Q6_K: mv_tile<T_Q6_K, KS, LG>(S.W, act, S.out, S.os_row, S.os_lane, S.add, tb, S.nbc, mm_smem); break;
    case T_Q8_0: mv_tile<T_Q8_0, KS, LG>(S.W, act, S.out, S.os_row, S.os_lane, S.add, tb, S.nbc, mm_smem); break;
    default: mv_tile<T_Q4_0, KS, LG>(S.W, act, S.out, S.os_row, S.os_lane, S.add, tb, S.nbc, mm_smem); break;
  }
}

// Blocks per chunk and shared memory of one matrix for a weight budget.
static int mv_seg_nbc(const DevTensor &w, int wbytes) {
  switch (w.type) {
    case T_Q4_K: return mm_nbc<T_Q4_K>(w.k / 256, wbytes);
    case T_Q6_K: return mm_nbc<T_Q6_K>(w.k / 256, wbytes);
    case T_Q8_0: return mm_nbc<T_Q8_0>(w.k / 32, wbytes);
    default: return mm_nbc<T_Q4_0>(w.k / 32, wbytes);
  }
}
static size_t mv_seg_smem(const DevTensor &w, int nbc) {
  switch (w.type) {
    case T_Q4_K: return mm_smem_bytes<T_Q4_K>(nbc);
    case T_Q6_K: return mm_smem_bytes<T_Q6_K>(nbc);
    case T_Q8_0: return mm_smem_bytes<T_Q8_0>(nbc);
    default: return mm_smem_bytes<T_Q4_0>(nbc);
  }
}

// Tile shape: b > 8 uses four lane groups (32 lanes a tile) with four k
// slices when the tiles are at most one per SM (a 16-warp CTA per SM with a
// larger staged chunk), else one; b <= 8 uses one lane group with eight
// slices (at most one tile per SM) or four.
// The b > 8 matvec kernel: mma.sync tiles (0) or tcgen05 (1); the
// environment variable PK_PREFILL_MMA=tc sets 1 at load.
static std::atomic<int> g_mv_path{-1};
static int mv_path() {
  int v = g_mv_path.load();
  if (v < 0) {
    const char *e = std::getenv("PK_PREFILL_MMA");
    int want = (e && std::strcmp(e, "tc") == 0) ? 1 : 0;
    g_mv_path.compare_exchange_strong(v, want);
    v = g_mv_path.load();
  }
  return v;
}
void set_mv_path(int path) { g_mv_path.store(path ? 1 : 0); }

cudaError_t launch_mv_multi(int n, const MvOut *outs, const Q8Dev &act, cudaStream_t st) {
  if (n < 1 || n > MV_MAX_SEGS || act.b < 1) return cudaErrorInvalidValue;
  if (act.b > 8 && mv_path() == 1) {
    bool tc = true;
    for (int i = 0; i < n; i++) tc = tc && mv_tc_supports(outs[i].w, act);
    if (tc) return launch_mv_tc(n, outs, act, st);
  }
  int tiles = 0;
  for (int i = 0; i < n; i++) {
    const MvOut &o = outs[i];
    if (!type_is_matvec(o.w.type) || act.k != o.w.k || o.w.rows < 1) return cudaErrorInvalidValue;
    tiles += (o.w.rows + MM_ROWS - 1) / MM_ROWS;
  }
  const int LG = act.b <= 8 ? 1 : 4;
  const int lane_tiles = (act.b + 8 * LG - 1) / (8 * LG), sms = num_sms();
  const long ctas = (long)tiles * lane_tiles;
  const bool big = ctas <= sms;  // at most one tile per SM: one wide CTA each
  const int KS = LG == 4 ? (big ? 4 : 1) : (big ? 8 : 4);
  // shared memory per CTA: one CTA per SM (wide), else up to five
  const int wbytes = big ? 200 * 1024 : 44 * 1024;
  MvSegs ss{};
  ss.n = n;
  int cta = 0;
  size_t smem = 0;
  for (int i = 0; i < n; i++) {
    const MvOut &o = outs[i];
    const int nbc = mv_seg_nbc(o.w, wbytes);
    ss.s[i] = MvSeg{o.w, o.out, o.os_row, o.os_lane, o.add ? 1 : 0, cta, nbc};
    cta += (o.w.rows + MM_ROWS - 1) / MM_ROWS;
    smem = std::max(smem, mv_seg_smem(o.w, nbc));
  }
  const dim3 grid(tiles, lane_tiles);
  cudaError_t e;
  void (*kern)(MvSegs, Q8Dev) = LG == 4 ? (KS == 4 ? k_mv_mma<4, 4> : k_mv_mma<1, 4>)
                                        : (KS == 8 ? k_mv_mma<8, 1> : k_mv_mma<4, 1>);
  if ((e = set_smem(kern, smem)) != cudaSuccess) return e;
  return launch(kern, grid, dim3(32 * LG * KS), smem, st, ss, act);
}

cudaError_t launch_mv_lanes(const DevTensor &w, const Q8Dev &act, float *out, long os_row, long os_lane, bool add,
                            cudaStream_t st) {
  const MvOut o{w, out, os_row, os_lane, add};
  return launch_mv_multi(1, &o, act, st);
}

// ------------------------------------------------------------ RoPE + KV, SwiGLU
// One thread per element: threads [0, n_head*half) rotate one q pair in
// place; the rest write one K element (rotated) and one V element to the
// cache.  grid = (b, element blocks).
__global__ void k_rope_kv(float *q, const float *k, const float *v, const int *pos, const float *rc, const float *rs,
                          int half, int dh, int n_head, int n_kv, int n_ctx, float *kc, float *vc, size_t lane_stride,
                          int kv16) {
  pdl_trigger();
  pdl_wait();
  const int bi = blockIdx.x;
  const int i = blockIdx.y * blockDim.x + threadIdx.x;
  const int nq = n_head * half, kdim = n_kv * dh;
  if (i >= nq + kdim) return;
  const int p = pos[bi];
  if (i < nq) {
    const int h = i / half, j = i - h * half;
    float *qr = q + (long)bi * n_head * dh + h * dh + 2 * j;
    const float x0 = qr[0], x1 = qr[1];
    const float c = rc[(size_t)p * half + j], s = rs[(size_t)p * half + j];
    qr[0] = fsub(fmul(x0, c), fmul(x1, s));
    qr[1] = fadd(fmul(x0, s), fmul(x1, c));
    return;
  }
  const int e = i - nq, h = e / dh, d = e - h * dh;
  const size_t ls = (size_t)bi * lane_stride;  // this token's own cache when every token has one
  const float *kr = k + (long)bi * kdim;
  float o = kr[e];
  if (d < 2 * half) {
    const int j = d >> 1;
    const float c = rc[(size_t)p * half + j], s = rs[(size_t)p * half + j];
    if ((d & 1) == 0) o = fsub(fmul(kr[e], c), fmul(kr[e + 1], s));
    else o = fadd(fmul(kr[e - 1], s), fmul(kr[e], c));
  }
  const size_t ki = ls + ((size_t)h * dh + d) * n_ctx + p, vi = ls + ((size_t)h * n_ctx + p) * dh + d;
  const float vv = v[(long)bi * kdim + e];
  if (kv16) {  // K is d-major: [kv head][d][position]
    kv_put<true>(kc, ki, o);
    kv_put<true>(vc, vi, vv);
  } else {
    kc[ki] = o;
    vc[vi] = vv;
  }
}

cudaError_t launch_rope_kv(float *q, const float *k, const float *v, int b, const int *pos, const float *rc,
                           const float *rs, int half, int dh, int n_head, int n_kv, int n_ctx, float *kc, float *vc,
                           cudaStream_t st, size_t lane_stride, bool kv16) {
  const int total = n_head * half + n_kv * dh;
  return launch(k_rope_kv, dim3(b, (total + 127) / 128), dim3(128), 0, st, q, k, v, pos, rc, rs, half, dh, n_head,
                n_kv, n_ctx, kc, vc, lane_stride, kv16 ? 1 : 0);
}

__global__ void k_expf(const float *x, float *out, long n) {
  pdl_trigger();
  pdl_wait();
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    out[i] = expf_lib(x[i]);
}

cudaError_t launch_expf(const float *x, float *out, long n, cudaStream_t st) {
  int grid = (int)std::min<long>((n + 255) / 256, (long)num_sms() * 16);
  return launch(k_expf, dim3(std::max(grid, 1)), dim3(256), 0, st, x, out, n);
}


// ------------------------------------------------------------ attention
// One CTA per (token, head), the reference's exact arithmetic
// (model.rs:993-1087, aarch64 build):
//   s_p = dot(q, k_p) * scale; for b == 1 the dot is f32_dot's order (two
//         4-lane unfused accumulators reduced pairwise, simd.rs:19-43), for
//         b > 1 one sequential chain (model.rs:1028-1033);
//   M   = max_p s_p (order-free);  e_p = exp(s_p - M);
//   sum = sequential over p;  inv = sum > 0 ? 1/sum : 0;
//   out[d] = (sequential over p, zero weights skipped, of e_p * v_p[d]) * inv.
// Every thread below dh owns one d and runs its chain over p; one more
// thread runs the sum chain.  Scores live in the per-(token, head) scratch
// row, so any context length fits.
template <bool KV16>
__global__ void k_attn(AttnArgs a, int dot8) {
  __shared__ float qs[256];
  __shared__ float red[40];
  __shared__ float s_inv;
  const int h = blockIdx.x, bi = blockIdx.y, tid = threadIdx.x, dh = a.dh;
  const int kh = h / (a.n_head / a.n_kv);
  pdl_trigger();
  pdl_wait();
  const int pos = a.pos[bi];
  const long hb = (long)bi * a.n_head + h;
  for (int d = tid; d < dh; d += blockDim.x) qs[d] = a.q[hb * dh + d];
  __syncthreads();
  // element offsets of this token's and head's K and V (f32 or f16 entries)
  const size_t kb = (size_t)bi * a.lane_stride + (size_t)kh * a.n_ctx * dh, vb = kb;
  float *sc = a.scores + hb * a.n_ctx;
  float mx = -INFINITY;
  const size_t nc = (size_t)a.n_ctx;
  for (int p = tid; p <= pos; p += blockDim.x) {
    const size_t kcol = kb + p;  // K is d-major: element d of position p at kcol + d * n_ctx
    float s;
    if (dot8) {
      float c[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
      int d = 0;
      for (; d + 8 <= dh; d += 8) {
#pragma unroll
        for (int u = 0; u < 8; u++) c[u] = fadd(c[u], fmul(qs[d + u], kv_get<KV16>(a.kcache, kcol + (size_t)(d + u) * nc)));
      }
      s = fadd(fadd(c[0], c[1]), fadd(c[2], c[3]));
      s = fadd(s, fadd(fadd(c[4], c[5]), fadd(c[6], c[7])));
      for (; d < dh; d++) s = fadd(s, fmul(qs[d], kv_get<KV16>(a.kcache, kcol + (size_t)d * nc)));
    } else {
      s = 0.0f;
      for (int d = 0; d < dh; d++) s = fadd(s, fmul(qs[d], kv_get<KV16>(a.kcache, kcol + (size_t)d * nc)));
    }
    s = fmul(s, a.scale);
    sc[p] = s;
    mx = s > mx ? s : mx;
  }
  const float M = block_max(mx, red);
  for (int p = tid; p <= pos; p += blockDim.x) sc[p] = expf_lib(fsub(sc[p], M));
  __syncthreads();
  float acc = 0.0f;
  if (tid < dh) {
    const size_t vr = vb + tid;
#pragma unroll 8
    for (int p = 0; p <= pos; p++) {
      const float e = sc[p];
      const float v = kv_get<KV16>(a.vcache, vr + (size_t)p * dh);
      acc = add_weighted(acc, e, v);
    }
  }
  if (tid == (dh < (int)blockDim.x ? dh : 0)) {
    float sum = 0.0f;
#pragma unroll 8
    for (int p = 0; p <= pos; p++) sum = fadd(sum, sc[p]);
    s_inv = sum > 0.0f ? fdiv(1.0f, sum) : 0.0f;
  }
  __syncthreads();
  if (tid < dh) {
    const float o = fmul(acc, s_inv);
    a.out[hb * dh + tid] = o;
    if (a.q8.q) {  // dh % 32 == 0: warp w holds block (h * dh + 32 w) / 32 of the token's row
      const int qk = a.n_head * dh, blk = (h * dh + tid) >> 5;
      q8_block_lane(o, tid & 31, a.q8.q + (long)bi * qk + blk * 32, a.q8.d + (long)bi * (qk >> 5) + blk,
                    a.q8.s + (long)bi * (qk >> 5) + blk);
    }
  }
}

// Chunk attention (b > 1): the same arithmetic as k_attn's b > 1 branch, one
// CTA per (group of AC_G tokens, head), the head's K and V brought into
// shared memory tile by tile (AC_P positions, double-buffered asynchronous
// copies) and shared by the group's tokens.
//   pass 1: thread (token, 4 positions) runs four score chains over d
//           (sequential, unfused) against the K tile [d][position];
//   pass 2: the tile's weights e = exp(s - M) (0 past the token's position,
//           which the V chain skips and which adds +0.0 exactly to a sum that
//           starts at +0.0), then thread (token, 4 dims) runs four V chains
//           and the token's sum chain over the tile in position order.
// KT is the cache entry type (float, or __half converted exactly when read).
constexpr int AC_THREADS = 256;
__host__ __device__ constexpr int ac_group(int dh) { return 512 / dh < 8 ? 512 / dh : 8; }
__host__ __device__ constexpr int ac_tile(int dh) { return dh <= 64 ? 128 : 64; }
static size_t ac_smem(int dh, size_t esz) {
  const int G = ac_group(dh), P = ac_tile(dh);
  return esz * 2 * P * dh + sizeof(float) * ((size_t)G * (P + 4) + (size_t)G * dh + AC_THREADS + 16);
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_ns() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// DHC: the head dimension as a compile-time constant (64, 128), or 0 for any.
template <int DHC, typename KT>
__global__ void __launch_bounds__(AC_THREADS) k_attn_chunk(AttnArgs a) {
  extern __shared__ __align__(16) float acs[];
  constexpr int EPC = 16 / sizeof(KT);  // entries per 16-byte copy
  const int dh = DHC ? DHC : a.dh, G = ac_group(dh), P = ac_tile(dh), QP = P / 4, tid = threadIdx.x;
  const int h = blockIdx.y, kh = h / (a.n_head / a.n_kv), t0 = blockIdx.x * G;
  KT *buf0 = reinterpret_cast<KT *>(acs), *buf1 = buf0 + P * dh;
  float *E = reinterpret_cast<float *>(buf1 + P * dh), *qs = E + G * (P + 4), *red = qs + G * dh;
  float *Ms = red + AC_THREADS;
  int *posv = (int *)(Ms + 8);
  pdl_trigger();
  pdl_wait();
  if (tid < G) {
    const int bi = t0 + tid;
    posv[tid] = bi < a.b ? min(a.pos[bi], a.n_ctx - 1) : -1;
  }
  for (int i = tid; i < G * dh; i += AC_THREADS) {
    const int t = i / dh, bi = t0 + t;
    qs[i] = bi < a.b ? a.q[((long)bi * a.n_head + h) * dh + (i - t * dh)] : 0.0f;
  }
  __syncthreads();
  int maxpos = -1;
  for (int t = 0; t < G; t++) maxpos = max(maxpos, posv[t]);
  if (maxpos < 0) return;
  const int nt = maxpos / P + 1;
  const KT *kc = reinterpret_cast<const KT *>(a.kcache) + (size_t)kh * dh * a.n_ctx;
  const KT *vc = reinterpret_cast<const KT *>(a.vcache) + (size_t)kh * a.n_ctx * dh;
  auto stage_k = [&](int i, KT *dst) {
    const int p0 = i * P, nq = (min(P, maxpos + 1 - p0) + EPC - 1) / EPC, CP = P / EPC;
    for (int c = tid; c < dh * CP; c += AC_THREADS) {
      const int d = c / CP, j = c - d * CP;
      if (j < nq) cp_async16(dst + d * P + EPC * j, kc + (size_t)d * a.n_ctx + p0 + EPC * j);
    }
  };
  auto stage_v = [&](int i, KT *dst) {
    const int p0 = i * P, nq = min(P, maxpos + 1 - p0) * dh / EPC;
    for (int c = tid; c < nq; c += AC_THREADS) cp_async16(dst + EPC * c, vc + (size_t)p0 * dh + EPC * c);
  };
  // ---- pass 1: scores
  const int st = tid / QP, sq = tid - st * QP;
  const int spos = st < G ? posv[st] : -1;
  float *sc = a.scores + ((long)(t0 + st) * a.n_head + h) * a.n_ctx;
  float mx = -INFINITY;
  stage_k(0, buf0);
  cp_async_commit();
  for (int i = 0; i < nt; i++) {
    if (i + 1 < nt) stage_k(i + 1, (i & 1) ? buf0 : buf1);
    else stage_v(0, (i & 1) ? buf0 : buf1);
    cp_async_commit();
    cp_async_wait1();
    __syncthreads();
    const int p = i * P + 4 * sq;
    if (p <= spos) {
      const KT *kt = ((i & 1) ? buf1 : buf0) + 4 * sq;
      const float *qv = qs + st * dh;
      float c0 = 0.0f, c1 = 0.0f, c2 = 0.0f, c3 = 0.0f;
#pragma unroll 8
      for (int d = 0; d < dh; d++) {
        const float4 k = kv_f4(kt + d * P);
        const float qq = qv[d];
        c0 = fadd(c0, fmul(qq, k.x));
        c1 = fadd(c1, fmul(qq, k.y));
        c2 = fadd(c2, fmul(qq, k.z));
        c3 = fadd(c3, fmul(qq, k.w));
      }
      const float sv[4] = {fmul(c0, a.scale), fmul(c1, a.scale), fmul(c2, a.scale), fmul(c3, a.scale)};
#pragma unroll
      for (int u = 0; u < 4; u++)
        if (p + u <= spos) {
          sc[p + u] = sv[u];
          mx = sv[u] > mx ? sv[u] : mx;
        }
    }
    __syncthreads();
  }
  red[tid] = mx;
  __syncthreads();
  if (tid < G) {
    float m = -INFINITY;
    for (int i = 0; i < QP; i++) m = red[tid * QP + i] > m ? red[tid * QP + i] : m;
    Ms[tid] = m;
  }
  __syncthreads();
  // ---- pass 2: weights, V chains and sum chains (thread: token vt, dims 4 vd .. 4 vd + 3)
  const int H4 = dh / 4, vt = tid / H4, vd = tid - vt * H4;
  const bool vact = vt < G;
  const float *Et = E + (vact ? vt : 0) * (P + 4);
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sum = 0.0f;
  for (int j = 0; j < nt; j++) {
    const KT *vb = ((nt + j) & 1) ? buf1 : buf0;
    if (j + 1 < nt) stage_v(j + 1, ((nt + j) & 1) ? buf0 : buf1);
    cp_async_commit();
    const int p0 = j * P;
    for (int i = tid; i < G * P; i += AC_THREADS) {
      const int t = i / P, pl = i - t * P, p = p0 + pl;
      float e = 0.0f;
      if (p <= posv[t]) {
        const float *srow = a.scores + ((long)(t0 + t) * a.n_head + h) * a.n_ctx;
        e = expf_lib(fsub(srow[p], Ms[t]));
      }
      E[t * (P + 4) + pl] = e;
    }
    cp_async_wait1();
    __syncthreads();
    if (vact) {
      const int npr = (min(P, maxpos + 1 - p0) + 3) & ~3;
      const KT *vv = vb + 4 * vd;
      for (int pl = 0; pl < npr; pl += 4) {
        const float4 e4 = *(const float4 *)(Et + pl);
        const float ev[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
        for (int u = 0; u < 4; u++) {
          const float4 v = kv_f4(vv + (pl + u) * dh);
          acc[0] = add_weighted(acc[0], ev[u], v.x);
          acc[1] = add_weighted(acc[1], ev[u], v.y);
          acc[2] = add_weighted(acc[2], ev[u], v.z);
          acc[3] = add_weighted(acc[3], ev[u], v.w);
          sum = fadd(sum, ev[u]);
        }
      }
    }
    __syncthreads();
  }
  const bool valid = vact && t0 + vt < a.b;
  const long bi = t0 + vt;
  float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (valid) {
    const float inv = sum > 0.0f ? fdiv(1.0f, sum) : 0.0f;
#pragma unroll
    for (int e = 0; e < 4; e++) o[e] = fmul(acc[e], inv);
    *(float4 *)(a.out + (bi * a.n_head + h) * dh + 4 * vd) = make_float4(o[0], o[1], o[2], o[3]);
  }
  if (a.q8.q && tid < ((G * H4 + 31) & ~31)) {
    // dh % 32 == 0, so H4 is a multiple of 8 and each group of eight threads
    // holds one 32-element block of one token's row, or no valid token at
    // all (it still takes part in the shuffles, which stay inside the group,
    // and stores nothing).  Whole warps take part.
    const int qk = a.n_head * dh, blk = (h * dh + 4 * vd) >> 5;
    const long qo = valid ? bi * qk + blk * 32 : 0, so = valid ? bi * (qk >> 5) + blk : 0;
    q8_block_group<8, 4>(o, tid & 7, valid, a.q8.q + qo, a.q8.d + so, a.q8.s + so);
  }
}

static cudaError_t launch_attention_k(const AttnArgs &a, cudaStream_t st);

// b == 1 order attention (k_attn with dot8) for one token per CTA with the
// head's K and V brought through shared memory in 128-position tiles, three
// stages of cp.async (two tiles in flight while one is used), so the score
// dots and the per-d chains read shared memory instead of waiting on global
// loads:
//   pass 1: thread t scores position p0 + t of the tile: eight chains over d
//           (d = 8j + u in chain u), reduced ((c0+c1)+(c2+c3))+((c4+c5)+(c6+c7));
//   pass 2: the tile's V rows and scores; thread p turns score p into
//           e_p = exp(s_p - M) in shared memory, then thread d < DH runs its
//           chain over the tile's positions in order (zero weights skipped)
//           and thread DH the sum chain.
// Same operations in the same order as k_attn, so the same bits.  KT is the
// cache entry type (float, or __half converted exactly when read).  Needs
// n_ctx and the lane stride multiples of 16 bytes' worth of entries, and
// 16-byte aligned K, V and score rows.
constexpr int AB_P = 128, AB_NS = 3;
__host__ __device__ constexpr size_t ab_smem(int dh, size_t esz) {
  return (size_t)AB_NS * (dh * AB_P * esz + AB_P * 4) + (esz == 4 ? 0 : (size_t)AB_P * dh * 4);
}

template <int DH, typename KT>
__global__ void __launch_bounds__(DH == 64 ? 128 : 256) k_attn_b1t(AttnArgs a) {
  constexpr int P = AB_P, NS = AB_NS, NT = DH == 64 ? 128 : 256, TILE = DH * P, EPC = 16 / sizeof(KT);
  extern __shared__ __align__(16) float at_sm[];
  KT *const tiles = reinterpret_cast<KT *>(at_sm);
  // NS tiles of TILE entries, then e: [NS][P], then (f16) the V products [P][DH]
  float *const es = reinterpret_cast<float *>(tiles + NS * TILE);
  float *const prod_buf = es + NS * P;
  __shared__ float qs[DH];
  __shared__ float red[40];
  __shared__ float s_inv;
  const int h = blockIdx.x, bi = blockIdx.y, tid = threadIdx.x;
  const int kh = h / (a.n_head / a.n_kv);
  const KT *kb = reinterpret_cast<const KT *>(a.kcache) + (size_t)bi * a.lane_stride + (size_t)kh * a.n_ctx * DH;
  const KT *vb = reinterpret_cast<const KT *>(a.vcache) + (size_t)bi * a.lane_stride + (size_t)kh * a.n_ctx * DH;
  {
    // The history below this token's position is not written by the kernels
    // this launch waits for: ask L2 for it while they run.  pos may not be
    // final yet, so it is clamped to the cache and only sizes the hint.
    const int hist = min(max(a.pos[bi], 0), a.n_ctx - 1);
    if (tid < DH) prefetch_l2(kb + (size_t)tid * a.n_ctx, (uint32_t)(hist * sizeof(KT)));  // K row d = tid
    else if (tid == DH) prefetch_l2(vb, (uint32_t)((size_t)hist * DH * sizeof(KT)));
  }
  pdl_trigger();
  pdl_wait();
  const int pos = a.pos[bi], n = pos + 1, nt = (n + P - 1) / P;
  const long hb = (long)bi * a.n_head + h;
  if (tid < DH) qs[tid] = a.q[hb * DH + tid];
  float *sc = a.scores + hb * a.n_ctx;
  // K tile t into stage t % NS: [d][P] from the d-major cache, 16-byte chunks
  // holding a position <= pos.  Every call commits one group (empty past the
  // last tile), so "wait until NS - 1 groups are pending" completes tile t.
  auto load_k = [&](int t) {
    if (t < nt) {
      KT *dst = tiles + (t % NS) * TILE;
      constexpr int CP = P / EPC;
      const int p0 = t * P, nq = (min(P, n - p0) + EPC - 1) / EPC;
      for (int c = tid; c < DH * CP; c += NT) {
        const int d = c / CP, j = c % CP;
        if (j < nq) cp_async16(dst + d * P + EPC * j, kb + (size_t)d * a.n_ctx + p0 + EPC * j);
      }
    }
    cp_async_commit();
  };
  for (int t = 0; t < NS - 1; t++) load_k(t);
  float mx = -INFINITY;
  for (int t = 0; t < nt; t++) {
    load_k(t + NS - 1);
    cp_async_wait_ns<NS - 1>();
    __syncthreads();
    const KT *cur = tiles + (t % NS) * TILE;
    const int p = t * P + tid;
    if (tid < P && p <= pos) {
      float c[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int d = 0; d < DH; d += 8) {
#pragma unroll
        for (int u = 0; u < 8; u++) c[u] = fadd(c[u], fmul(qs[d + u], kv_f(cur[(d + u) * P + tid])));
      }
      float sv = fadd(fadd(c[0], c[1]), fadd(c[2], c[3]));
      sv = fadd(sv, fadd(fadd(c[4], c[5]), fadd(c[6], c[7])));
      sv = fmul(sv, a.scale);
      sc[p] = sv;
      mx = sv > mx ? sv : mx;
    }
    __syncthreads();
  }
  cp_async_wait_all();  // only empty groups are left
  const float M = block_max(mx, red);  // (its barriers also order the score stores before pass 2)
  // V tile t into stage t % NS: P rows of DH entries (contiguous), and the scores of its positions
  auto load_v = [&](int t) {
    if (t < nt) {
      KT *dst = tiles + (t % NS) * TILE;
      float *edst = es + (t % NS) * P;
      const int p0 = t * P, nv = min(P, n - p0);
      const KT *src = vb + (size_t)p0 * DH;
      for (int c = tid; c < nv * (DH / EPC); c += NT) cp_async16(dst + EPC * c, src + EPC * c);
      if (tid < ((nv + 3) >> 2)) cp_async16(edst + 4 * tid, sc + p0 + 4 * tid);
    }
    cp_async_commit();
  };
  for (int t = 0; t < NS - 1; t++) load_v(t);
  float acc = 0.0f, sum = 0.0f;
  for (int t = 0; t < nt; t++) {
    load_v(t + NS - 1);
    cp_async_wait_ns<NS - 1>();
    __syncthreads();
    const KT *cur = tiles + (t % NS) * TILE;
    float *ec = es + (t % NS) * P;
    const int nv = min(P, n - t * P);
    bool zero = false;  // a weight of this tile underflowed to 0
    if (tid < nv) {
      ec[tid] = expf_lib(fsub(ec[tid], M));
      zero = ec[tid] == 0.0f;
    }
    const bool any_zero = __syncthreads_or(zero) != 0;  // uniform over the CTA
    // the tile's products e_p * v_p[d] by every thread (-0.0 for a zero
    // weight, which the chain then adds exactly as a skip), so that each
    // chain step below waits for one add; f32 products overwrite the tile
    float *const pr = sizeof(KT) == 4 ? reinterpret_cast<float *>(tiles + (t % NS) * TILE) : prod_buf;
    if (!any_zero) {  // no weight is 0: the plain products
      for (int i = tid; i < nv * (DH / 4); i += NT) {
        const int j = i / (DH / 4), d4 = 4 * (i % (DH / 4));
        const float e = ec[j];
        const float4 v = kv_f4(cur + j * DH + d4);
        *reinterpret_cast<float4 *>(pr + j * DH + d4) = make_float4(fmul(e, v.x), fmul(e, v.y), fmul(e, v.z), fmul(e, v.w));
      }
    } else {
      for (int i = tid; i < nv * (DH / 4); i += NT) {
        const int j = i / (DH / 4), d4 = 4 * (i % (DH / 4));
        const float e = ec[j];
        const float4 v = kv_f4(cur + j * DH + d4);
        const bool z = e == 0.0f;
        *reinterpret_cast<float4 *>(pr + j * DH + d4) =
            make_float4(z ? -0.0f : fmul(e, v.x), z ? -0.0f : fmul(e, v.y), z ? -0.0f : fmul(e, v.z),
                        z ? -0.0f : fmul(e, v.w));
      }
    }
    __syncthreads();
    if (tid < DH) {
#pragma unroll 8
      for (int j = 0; j < nv; j++) acc = fadd(acc, pr[j * DH + tid]);
    } else if (tid == DH) {
#pragma unroll 8
      for (int j = 0; j < nv; j++) sum = fadd(sum, ec[j]);
    }
    __syncthreads();
  }
  cp_async_wait_all();
  if (tid == DH) s_inv = sum > 0.0f ? fdiv(1.0f, sum) : 0.0f;
  __syncthreads();
  if (tid < DH) {
    const float o = fmul(acc, s_inv);
    a.out[hb * DH + tid] = o;
    if (a.q8.q) {  // warp w holds block (h * DH + 32 w) / 32 of the token's row
      const int qk = a.n_head * DH, blk = (h * DH + tid) >> 5;
      q8_block_lane(o, tid & 31, a.q8.q + (long)bi * qk + blk * 32, a.q8.d + (long)bi * (qk >> 5) + blk,
                    a.q8.s + (long)bi * (qk >> 5) + blk);
    }
  }
}

cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st) {
  if (a.dh > 256 || a.dh % 4 != 0 || a.n_head % a.n_kv != 0) return cudaErrorInvalidValue;
  if (a.q8.q && a.dh % 32 != 0) {  // quantise separately
    AttnArgs b = a;
    b.q8 = Q8Dev{};
    cudaError_t e = launch_attention_k(b, st);
    if (e != cudaSuccess) return e;
    return launch_q8(a.out, 1, (long)a.n_head * a.dh, a.n_head * a.dh, a.b, a.q8, st);
  }
  return launch_attention_k(a, st);
}

// The b == 1 order for long histories, split so that many more CTAs
// stream K and V (same values, same order, so the same bits as k_attn_b1t):
//   k_attn_sc: CTA (head, token, c) scores positions [c * pchunk, ...) as
//              k_attn_b1t's pass 1 and writes their maximum (-inf if none);
//   k_attn_pv: CTA (head, token, part) takes M as the maximum of those
//              (order-free), turns each 128-position tile's scores into e_p
//              in shared memory and runs the chains of d = 32 part .. +31
//              over V's matching 128-byte row pieces, plus its own copy of
//              the sum chain; its 32 outputs are one Q8 block.
template <int DH, typename KT>
__global__ void __launch_bounds__(DH == 64 ? 128 : 256) k_attn_sc(AttnArgs a) {
  constexpr int P = AB_P, NS = AB_NS, NT = DH == 64 ? 128 : 256, TILE = DH * P, EPC = 16 / sizeof(KT);
  extern __shared__ __align__(16) float at_sm[];
  KT *const tiles = reinterpret_cast<KT *>(at_sm);
  __shared__ float qs[DH];
  __shared__ float red[40];
  const int h = blockIdx.x, bi = blockIdx.y, c = blockIdx.z, tid = threadIdx.x;
  const int kh = h / (a.n_head / a.n_kv);
  pdl_trigger();
  pdl_wait();
  const int pos = a.pos[bi];
  const long hb = (long)bi * a.n_head + h;
  const int p_lo = c * a.pchunk, p_hi = min(p_lo + a.pchunk, pos + 1);
  float *pm = a.pmax + hb * gridDim.z + c;
  if (p_lo >= p_hi) {  // the whole CTA: no position of this token in the chunk
    if (tid == 0) *pm = -INFINITY;
    return;
  }
  if (tid < DH) qs[tid] = a.q[hb * DH + tid];
  const KT *kb = reinterpret_cast<const KT *>(a.kcache) + (size_t)bi * a.lane_stride + (size_t)kh * a.n_ctx * DH;
  float *sc = a.scores + hb * a.n_ctx;
  const int nt = (p_hi - p_lo + P - 1) / P;
  auto load_k = [&](int t) {
    if (t < nt) {
      KT *dst = tiles + (t % NS) * TILE;
      constexpr int CP = P / EPC;
      const int p0 = p_lo + t * P, nq = (min(P, p_hi - p0) + EPC - 1) / EPC;
      for (int i = tid; i < DH * CP; i += NT) {
        const int d = i / CP, j = i % CP;
        if (j < nq) cp_async16(dst + d * P + EPC * j, kb + (size_t)d * a.n_ctx + p0 + EPC * j);
      }
    }
    cp_async_commit();
  };
  for (int t = 0; t < NS - 1; t++) load_k(t);
  float mx = -INFINITY;
  for (int t = 0; t < nt; t++) {
    load_k(t + NS - 1);
    cp_async_wait_ns<NS - 1>();
    __syncthreads();
    const KT *cur = tiles + (t % NS) * TILE;
    const int p = p_lo + t * P + tid;
    if (tid < P && p < p_hi) {
      float cc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int d = 0; d < DH; d += 8) {
#pragma unroll
        for (int u = 0; u < 8; u++) cc[u] = fadd(cc[u], fmul(qs[d + u], kv_f(cur[(d + u) * P + tid])));
      }
      float sv = fadd(fadd(cc[0], cc[1]), fadd(cc[2], cc[3]));
      sv = fadd(sv, fadd(fadd(cc[4], cc[5]), fadd(cc[6], cc[7])));
      sv = fmul(sv, a.scale);
      sc[p] = sv;
      mx = sv > mx ? sv : mx;
    }
    __syncthreads();
  }
  cp_async_wait_all();
  const float M = block_max(mx, red);
  if (tid == 0) *pm = M;
}

// The value pass: one CTA of 256 threads per (stream, head, 64 of the head's
// dims), three stages of V pieces and scores.  Per 128-position tile every
// thread takes part in the exps and in the products e_p * v_p[d] (four dims
// at a time, -0.0 for a zero weight: adding it leaves the chain as skipping
// would), then each of the 64 chain threads only loads and adds, in
// position order, with the loads unrolled ahead of the adds, while one more
// thread runs the sum chain.  f32 products overwrite their V piece; f16 ones
// (twice the size) go to a separate [P][W] buffer.
constexpr int PV_P = 128, PV_W = 64, PV_NT = 256, PV_NS = 3;
constexpr size_t pv_smem(size_t esz) {
  return (size_t)PV_NS * (PV_P * PV_W * esz + PV_P * 4) + (esz == 4 ? 0 : (size_t)PV_P * PV_W * 4);
}

template <int DH, typename KT>
__global__ void __launch_bounds__(PV_NT) k_attn_pv(AttnArgs a, int nch) {
  constexpr int P = PV_P, NS = PV_NS, W = PV_W, NT = PV_NT, EPC = 16 / sizeof(KT), CW = W / EPC;
  static_assert(DH % W == 0 && W % 32 == 0, "whole Q8 blocks per CTA");
  extern __shared__ __align__(16) float pv_sm[];
  KT *const pieces = reinterpret_cast<KT *>(pv_sm);
  // NS V pieces of P x W entries, then e: [NS][P], then (f16) the products [P][W]
  float *const es = reinterpret_cast<float *>(pieces + NS * P * W);
  float *const prod_buf = es + NS * P;
  __shared__ float s_m, s_inv;
  const int h = blockIdx.x, bi = blockIdx.y, part = blockIdx.z, tid = threadIdx.x;
  const int kh = h / (a.n_head / a.n_kv);
  pdl_trigger();
  pdl_wait();
  const int pos = a.pos[bi], n = pos + 1, nt = (n + P - 1) / P;
  const long hb = (long)bi * a.n_head + h;
  if (tid == 0) {
    const float *pm = a.pmax + hb * nch;
    float m = -INFINITY;
    for (int c = 0; c < nch; c++) m = pm[c] > m ? pm[c] : m;
    s_m = m;
  }
  __syncthreads();
  const float M = s_m;
  const KT *vb = reinterpret_cast<const KT *>(a.vcache) + (size_t)bi * a.lane_stride + (size_t)kh * a.n_ctx * DH + part * W;
  const float *sc = a.scores + hb * a.n_ctx;
  auto load = [&](int t) {
    if (t < nt) {
      KT *dst = pieces + (t % NS) * P * W;
      float *edst = es + (t % NS) * P;
      const int p0 = t * P, nv = min(P, n - p0);
      for (int i = tid; i < nv * CW; i += NT) {
        const int r = i / CW, j = i % CW;
        cp_async16(dst + r * W + EPC * j, vb + (size_t)(p0 + r) * DH + EPC * j);
      }
      for (int i = tid; i < ((nv + 3) >> 2); i += NT) cp_async16(edst + 4 * i, sc + p0 + 4 * i);
    }
    cp_async_commit();
  };
  for (int t = 0; t < NS - 1; t++) load(t);
  float acc = 0.0f, sum = 0.0f;
  for (int t = 0; t < nt; t++) {
    load(t + NS - 1);
    cp_async_wait_ns<NS - 1>();
    __syncthreads();
    const KT *cur = pieces + (t % NS) * P * W;
    float *ec = es + (t % NS) * P;
    const int nv = min(P, n - t * P);
    bool zero = false;  // a weight of this tile underflowed to 0
    for (int j = tid; j < nv; j += NT) {
      ec[j] = expf_lib(fsub(ec[j], M));
      zero = zero || ec[j] == 0.0f;
    }
    const bool any_zero = __syncthreads_or(zero) != 0;  // uniform over the CTA
    float *const pr = sizeof(KT) == 4 ? reinterpret_cast<float *>(pieces + (t % NS) * P * W) : prod_buf;
    if (!any_zero) {  // no weight is 0: the plain products
      for (int i = tid; i < nv * (W / 4); i += NT) {
        const int j = i / (W / 4), d4 = 4 * (i % (W / 4));
        const float e = ec[j];
        const float4 v = kv_f4(cur + j * W + d4);
        *reinterpret_cast<float4 *>(pr + j * W + d4) = make_float4(fmul(e, v.x), fmul(e, v.y), fmul(e, v.z), fmul(e, v.w));
      }
    } else {
      for (int i = tid; i < nv * (W / 4); i += NT) {
        const int j = i / (W / 4), d4 = 4 * (i % (W / 4));
        const float e = ec[j];
        const float4 v = kv_f4(cur + j * W + d4);
        const bool z = e == 0.0f;
        *reinterpret_cast<float4 *>(pr + j * W + d4) =
            make_float4(z ? -0.0f : fmul(e, v.x), z ? -0.0f : fmul(e, v.y), z ? -0.0f : fmul(e, v.z),
                        z ? -0.0f : fmul(e, v.w));
      }
    }
    __syncthreads();
    if (tid < W) {
#pragma unroll 16
      for (int j = 0; j < nv; j++) acc = fadd(acc, pr[j * W + tid]);
    } else if (tid == W) {
#pragma unroll 16
      for (int j = 0; j < nv; j++) sum = fadd(sum, ec[j]);
    }
    __syncthreads();
  }
  cp_async_wait_all();
  if (tid == W) s_inv = sum > 0.0f ? fdiv(1.0f, sum) : 0.0f;
  __syncthreads();
  if (tid < W) {  // warp w holds Q8 block (h * DH + part * W) / 32 + w of the token's row
    const float o = fmul(acc, s_inv);
    a.out[hb * DH + part * W + tid] = o;
    if (a.q8.q) {
      const int qk = a.n_head * DH, blk = (h * DH + part * W + tid) >> 5;
      q8_block_lane(o, tid & 31, a.q8.q + (long)bi * qk + blk * 32, a.q8.d + (long)bi * (qk >> 5) + blk,
                    a.q8.s + (long)bi * (qk >> 5) + blk);
    }
  }
}

// KT: the cache entry type.  The tiled kernels copy 16-byte pieces, so they
// need n_ctx, the lane stride and (for the chunk kernel) dh in whole pieces
// and 16-byte aligned caches; otherwise k_attn reads entries one at a time.
template <typename KT>
static cudaError_t launch_attention_t(const AttnArgs &a, cudaStream_t st) {
  constexpr int EPC = 16 / sizeof(KT);
  constexpr size_t ESZ = sizeof(KT);
  const bool aligned = (((uintptr_t)a.kcache | (uintptr_t)a.vcache) & 15) == 0 && a.n_ctx % EPC == 0;
  if (a.b > 1 && !a.b1_order && a.lane_stride == 0 && aligned && a.dh % EPC == 0) {
    const size_t smem = ac_smem(a.dh, ESZ);
    const int G = ac_group(a.dh);
    const dim3 grid((a.b + G - 1) / G, a.n_head);
    void (*kern)(AttnArgs) = a.dh == 64    ? k_attn_chunk<64, KT>
                             : a.dh == 128 ? k_attn_chunk<128, KT>
                                           : k_attn_chunk<0, KT>;
    cudaError_t e = set_smem(kern, smem);
    if (e != cudaSuccess) return e;
    return launch(kern, grid, dim3(AC_THREADS), smem, st, a);
  }
  const bool dot8 = a.b == 1 || a.b1_order;
  const bool tiles = dot8 && (a.dh == 64 || a.dh == 128) && aligned && a.lane_stride % EPC == 0 &&
                     ((uintptr_t)a.scores & 15) == 0;
  if (tiles && a.pmax && a.pchunk > 0) {
    if (a.pchunk % AB_P != 0) return cudaErrorInvalidValue;
    const int nch = (a.n_ctx + a.pchunk - 1) / a.pchunk;
    void (*ks)(AttnArgs) = a.dh == 64 ? k_attn_sc<64, KT> : k_attn_sc<128, KT>;
    void (*kv)(AttnArgs, int) = a.dh == 64 ? k_attn_pv<64, KT> : k_attn_pv<128, KT>;
    const size_t s1 = (size_t)AB_NS * a.dh * AB_P * ESZ;
    cudaError_t e = set_smem(ks, s1);
    if (e == cudaSuccess) e = set_smem(kv, pv_smem(ESZ));
    if (e == cudaSuccess)
      e = launch(ks, dim3(a.n_head, a.b, nch), dim3(a.dh == 64 ? 128 : 256), s1, st, a);
    if (e != cudaSuccess) return e;
    return launch(kv, dim3(a.n_head, a.b, a.dh / PV_W), dim3(PV_NT), pv_smem(ESZ), st, a, nch);
  }
  if (tiles) {
    const size_t smem = ab_smem(a.dh, ESZ);
    void (*kern)(AttnArgs) = a.dh == 64 ? k_attn_b1t<64, KT> : k_attn_b1t<128, KT>;
    cudaError_t e = set_smem(kern, smem);
    if (e != cudaSuccess) return e;
    return launch(kern, dim3(a.n_head, a.b), dim3(a.dh == 64 ? 128 : 256), smem, st, a);
  }
  const int threads = a.dh < 128 ? 128 : 256;
  return launch(k_attn<(sizeof(KT) == 2)>, dim3(a.n_head, a.b), dim3(threads), 0, st, a, dot8 ? 1 : 0);
}

static cudaError_t launch_attention_k(const AttnArgs &a, cudaStream_t st) {
  return a.kv16 ? launch_attention_t<__half>(a, st) : launch_attention_t<float>(a, st);
}

// ------------------------------------------------------------ temperature / top-p sampling
// sampler.rs:21-92 for temp > 0, on one CTA of 1024 threads, with the
// reference's arithmetic and order:
//   M = max (strict '>', NaN never wins); e_i = exp((l_i - M) * (1 / temp));
//   sum = sequential over i; 0 (no draw) unless sum > 0;
//   top_p in (0, 1): indices sorted by e descending, equal e by index (the
//   oracle's tie order; Rust's sort_unstable leaves it open), acc += e / sum
//   in that order until acc >= top_p; e of the others set to 0 and
//   sum = sequential over the kept ones in index order;
//   r = rng.next_f32() * sum, the first i whose running sum of e reaches r
//   (n - 1 if none).
// Elementwise steps run on all threads; each sum is one thread's sequential
// chain.  The sort is a bitonic network on 64-bit keys (~bits(e) << 32 | i)
// in the scratch buffer.
constexpr int SMP_THREADS = 1024;
static int smp_pow2(int n) {
  int p = 1;
  while (p < n) p <<= 1;
  return p;
}
size_t sample_scratch_bytes(int n) {
  const size_t a = ((size_t)n * 4 + 255) & ~(size_t)255;
  return 2 * a + (size_t)smp_pow2(n) * 8 + (((size_t)n + 255) & ~(size_t)255);
}

__device__ float rng_next_f32(unsigned long long *state) {  // sampler.rs:6-19 (splitmix64)
  unsigned long long z = *state + 0x9E3779B97F4A7C15ULL;
  *state = z;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  z ^= z >> 31;
  return (float)(unsigned)(z >> 40) * (1.0f / 16777216.0f);
}

__global__ void __launch_bounds__(SMP_THREADS) k_sample(const float *__restrict__ logits, int n, int p2, float temp,
                                                        float top_p, unsigned long long *rng, uint8_t *scratch,
                                                        uint32_t *tok) {
  __shared__ float redf[32];
  __shared__ float s_val;
  __shared__ int s_cut;
  pdl_trigger();
  pdl_wait();
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const size_t fa = ((size_t)n * 4 + 255) & ~(size_t)255;
  float *E = (float *)scratch, *P = (float *)(scratch + fa);
  unsigned long long *K = (unsigned long long *)(scratch + 2 * fa);
  uint8_t *keep = scratch + 2 * fa + (size_t)p2 * 8;
  // the maximum (order-free: NaN never wins)
  float mx = -INFINITY;
  for (int i = tid; i < n; i += SMP_THREADS) {
    const float v = logits[i];
    mx = v > mx ? v : mx;
  }
  mx = warp_max(mx);
  if (lane == 0) redf[w] = mx;
  __syncthreads();
  if (tid == 0) {
    float m = -INFINITY;
    for (int i = 0; i < SMP_THREADS / 32; i++) m = redf[i] > m ? redf[i] : m;
    s_val = m;
  }
  __syncthreads();
  const float M = s_val, inv = fdiv(1.0f, temp);
  for (int i = tid; i < n; i += SMP_THREADS) E[i] = expf_lib(fmul(fsub(logits[i], M), inv));
  __syncthreads();
  if (tid == 0) {
    float sum = 0.0f;
#pragma unroll 8
    for (int i = 0; i < n; i++) sum = fadd(sum, E[i]);
    s_val = sum;
  }
  __syncthreads();
  float sum = s_val;
  if (!(sum > 0.0f)) {
    if (tid == 0) *tok = 0u;
    return;
  }
  if (top_p > 0.0f && top_p < 1.0f) {
    for (int i = tid; i < p2; i += SMP_THREADS)
      K[i] = i < n ? ((unsigned long long)(~__float_as_uint(E[i])) << 32) | (unsigned)i : ~0ULL;
    __syncthreads();
    for (int k = 2; k <= p2; k <<= 1)
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < p2; i += SMP_THREADS) {
          const int l = i ^ j;
          if (l > i) {
            const unsigned long long a = K[i], b = K[l];
            if ((a > b) == ((i & k) == 0)) {
              K[i] = b;
              K[l] = a;
            }
          }
        }
        __syncthreads();
      }
    for (int k = tid; k < n; k += SMP_THREADS) {
      P[k] = fdiv(E[(unsigned)(K[k] & 0xFFFFFFFFULL)], sum);
      keep[k] = 0;
    }
    __syncthreads();
    if (tid == 0) {
      float acc = 0.0f;
      int cut = n;
      for (int k = 0; k < n; k++) {
        acc = fadd(acc, P[k]);
        if (acc >= top_p) {
          cut = k + 1;
          break;
        }
      }
      s_cut = cut;
    }
    __syncthreads();
    for (int k = tid; k < s_cut; k += SMP_THREADS) keep[(unsigned)(K[k] & 0xFFFFFFFFULL)] = 1;
    __syncthreads();
    for (int i = tid; i < n; i += SMP_THREADS)
      if (!keep[i]) E[i] = 0.0f;
    __syncthreads();
    if (tid == 0) {
      float ns = 0.0f;
      for (int i = 0; i < n; i++)
        if (keep[i]) ns = fadd(ns, E[i]);
      s_val = ns;
    }
    __syncthreads();
    sum = s_val;
  }
  if (tid == 0) {
    const float r = fmul(rng_next_f32(rng), sum);
    float acc = 0.0f;
    unsigned t = (unsigned)(n - 1);
    for (int i = 0; i < n; i++) {
      acc = fadd(acc, E[i]);
      if (acc >= r) {
        t = (unsigned)i;
        break;
      }
    }
    *tok = t;
  }
}

cudaError_t launch_sample(const float *logits, int n, float temp, float top_p, unsigned long long *rng, void *scratch,
                          uint32_t *tok, cudaStream_t st) {
  if (n < 1 || !(temp > 0.0f) || (((uintptr_t)scratch) & 255)) return cudaErrorInvalidValue;
  return launch(k_sample, dim3(1), dim3(SMP_THREADS), 0, st, logits, n, smp_pow2(n), temp, top_p, rng,
                (uint8_t *)scratch, tok);
}

// ------------------------------------------------------------ argmax / feedback
__global__ void __launch_bounds__(1024) k_argmax(const float *__restrict__ x, int n, uint32_t *out) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_trigger();
  pdl_wait();
  x += (size_t)blockIdx.x * n;  // one row per CTA
  out += blockIdx.x;
  float bv = -INFINITY;
  int bi = INT_MAX;
  const int nt = blockDim.x;
  for (int i0 = threadIdx.x; i0 < n; i0 += 8 * nt) {  // eight loads in flight, then compared in index order
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) v[u] = i0 + u * nt < n ? x[i0 + u * nt] : -INFINITY;
#pragma unroll
    for (int u = 0; u < 8; u++)
      if (v[u] > bv) { bv = v[u]; bi = i0 + u * nt; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
    *out = bi == INT_MAX ? 0u : (uint32_t)bi;  // nothing above -inf: the reference keeps index 0
  }
}

cudaError_t launch_argmax(const float *x, int n, uint32_t *out_idx, cudaStream_t st, int rows) {
  if (rows < 1) return cudaErrorInvalidValue;
  return launch(k_argmax, dim3(rows), dim3(1024), 0, st, x, n, out_idx);
}

// Row r: ids[r] = tok[r], pos[r] += 1, hist[r * hist_stride + step[r]] = tok[r], step[r] += 1.
__global__ void k_advance(const uint32_t *tok, uint32_t *ids, int *pos, uint32_t *hist, int *step, int rows,
                          size_t hist_stride) {
  pdl_trigger();
  pdl_wait();
  const int r = threadIdx.x;
  if (r >= rows) return;
  const uint32_t t = tok[r];
  ids[r] = t;
  pos[r] += 1;
  hist[(size_t)r * hist_stride + step[r]] = t;
  step[r] += 1;
}

cudaError_t launch_advance(const uint32_t *tok, uint32_t *ids, int *pos, uint32_t *hist, int *step, cudaStream_t st,
                           int rows, size_t hist_stride) {
  if (rows < 1 || rows > 1024) return cudaErrorInvalidValue;
  return launch(k_advance, dim3(1), dim3(rows <= 32 ? 32 : (rows + 31) & ~31), 0, st, tok, ids, pos, hist, step,
                rows, hist_stride);
}

}  // namespace pk
