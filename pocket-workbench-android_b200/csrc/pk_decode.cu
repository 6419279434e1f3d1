// pk_decode.cu -- persistent single-token decode kernel for sm_100a.
//
// Reference semantics (Aleinto97/pocket-workbench-android, rust/pocketinfer/src):
//   forward_inner, one token       model.rs:833-1170
//   Q8Act::prepare                 quant_int.rs:17-56
//   lanes::* row dots              quant_int.rs:282-419
//   rmsnorm (b == 1, f32_sum_sq)   model.rs:791-810, simd.rs:47-64
//   rope                           model.rs:953-979
//   attention (b == 1, f32_dot)    model.rs:993-1087, simd.rs:19-43
//   swiglu / residuals             model.rs:1095-1125
//   greedy sample                  sampler.rs:26-36
//
// Work split.  The grid has one CTA per SM (fewer for small models: every
// CTA owns rows of every matrix) and every CTA owns a fixed slice of rows of
// every matrix (host-built chunk list).  Per CTA:
//   warp 0           producer: walks the chunk list (plus the K/V history of
//                    the attention heads this CTA owns) and bulk-copies each
//                    chunk into the next free ring slot (mbarrier complete_tx);
//   warps 3..11      term warps: integer dots + float terms of a chunk into a
//                    term buffer (DK_NB buffers, in turn);
//   warps 1, 2       chain warps: one lane per row adds that row's terms in
//                    the reference's order and runs the epilogue; each row
//                    group is assigned to one of them by the plan.
// Phase hand-off (qkv | attention | o | gate+up | down): the epilogues
// publish their rows as tagged 8-byte words (value + epoch/phase tag) and
// the next phase's readers poll the words they need until every tag is the
// previous phase's, so no grid barrier separates the phases.  No CTA can get
// two phases ahead of another: each phase reads all of the previous phase's
// output (attention reads its heads' q/k/v, and the o phase then reads every
// head), and every CTA writes rows of every phase; the residual alternates
// between two buffers.  The producer streams on regardless.
//
// Every wait is bounded (2 s); a wait that runs out records PK_ERR_TIMEOUT in
// the error word, the CTA's consumers stop together at the end of the phase,
// and the producer waits for its own copies in flight before it returns.
#include <float.h>
#include <limits.h>
#include <math.h>

#include <algorithm>
#include <string>
#include <vector>

#include "pk.h"
#include "pk_decode.h"
#include "pk_device.cuh"
#include "pk_quant.cuh"

namespace pk {
namespace {

constexpr int CONS = DK_THREADS - 32;  // consumer threads (warps 1..)
// Warp roles: warp 0 the producer, warps 1 .. DK_CHAINS the chain warps, the
// rest term warps.
__host__ __device__ constexpr int chain_of_warp(int w) { return (w >= 1 && w <= DK_CHAINS) ? w - 1 : -1; }
__host__ __device__ constexpr bool term_warp(int w) { return w > DK_CHAINS; }
__host__ __device__ constexpr int term_rank(int w) { return w - 1 - DK_CHAINS; }  // among the term warps
constexpr int TERM_T = DK_THREADS - 32 - 32 * DK_CHAINS;  // term threads

// Named barriers: all consumers; per (term buffer, chain warp) "terms ready"
// and "buffer free" pairs (a barrier id is only ever shared by the term warps
// and ONE chain warp, so generations cannot mix); the value-chain warps.
constexpr int NB_CONS = 1, NB_FULLT = 2, NB_EMPTYT = 2 + DK_NB * DK_CHAINS, NB_V = 2 + 2 * DK_NB * DK_CHAINS;
static_assert(NB_V < 16, "named barrier ids");
// The term warps form two groups that take alternate chunks (chunk mv: group
// mv & 1), so two chunks' items are in flight at once.
constexpr int TG0 = 32 * ((TERM_T / 32 + 1) / 2), TG1 = TERM_T - TG0;  // threads per group
static_assert(TG1 > 0 && TG0 % 32 == 0 && TG1 % 32 == 0, "two whole-warp term groups");
// A term-buffer barrier's participants: the chunk's group and one chain warp.
__host__ __device__ constexpr int nb_pair(int mv) { return ((mv & 1) ? TG1 : TG0) + 32; }
constexpr unsigned long long WAIT_NS = 2000000000ull;
// Waiting threads yield their issue slots: consumers waiting for ring data
// suspend in mbarrier.try_wait (woken when the phase completes), and pollers
// of another SM's tagged words sleep between reads.
constexpr uint32_t DATA_SLEEP_NS = 4000, POLL_SLEEP_NS = 128;

__device__ __forceinline__ uint32_t saddr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
__device__ __forceinline__ void bar_arrive(int id, int n) { asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// Named barrier that also ORs a predicate over the participating threads:
// every thread gets the same answer (a decision to stop cannot diverge).
__device__ __forceinline__ bool bar_or(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Like mbar_test, but the thread may sleep up to `ns` in the hardware until the
// phase completes (it wakes as soon as it does).
__device__ __forceinline__ bool mbar_test_sleep(uint64_t *b, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// Bounded wait for the completion of phase `parity`; false on timeout or abort.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, const volatile int *abort,
                                          uint32_t sleep_ns = 0) {
  if (mbar_test(b, parity)) return true;
  const unsigned long long t0 = gtime();
  for (;;) {
    if (sleep_ns ? mbar_test_sleep(b, parity, sleep_ns) : mbar_test(b, parity)) return true;
    if (abort && *abort) return false;
    if (gtime() - t0 > WAIT_NS) return false;
  }
}
// Untiled bulk copy global -> this CTA's shared memory (16-byte aligned
// addresses, size a multiple of 16), completion counted on mbarrier b.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   saddr(dst)),
               "l"(src), "r"(bytes), "r"(saddr(b))
               : "memory");
}
// Tiled 2-D tensor copy global -> this CTA's own shared memory only:
// the box of tensor map `map` at element coordinates (x, y), completion
// counted on mbarrier b.  x * element size is a multiple of 16 bytes at
// every call site, dst is box-size aligned.
__device__ __forceinline__ void tma_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *b) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          saddr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(saddr(b))
      : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Tagged words (see DecodeArgs): single-copy atomic 8-byte accesses at GPU
// scope, so a reader sees a value together with the tag it was written with.
__device__ __forceinline__ void st_ll(unsigned long long *p, float v, uint32_t tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_ll(const unsigned long long *p) {
  unsigned long long w;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}
// Two consecutive tagged words in one 16-byte load (p 16-byte aligned); each
// word is still read single-copy atomically.
__device__ __forceinline__ void ld_ll2(const unsigned long long *p, unsigned long long &a, unsigned long long &b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ bool ll_ok(unsigned long long w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
__device__ __forceinline__ float ll_val(unsigned long long w) { return __uint_as_float((uint32_t)w); }

__device__ __forceinline__ void prefetch_l1(const void *p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}
__device__ __forceinline__ const uint8_t *align16_down(const uint8_t *p) {
  return (const uint8_t *)((uintptr_t)p & ~(uintptr_t)15);
}

// Shared memory layout (host and device agree through dk_layout).
struct Layout {
  size_t ring, full, empty, desc, aq, ad, as, as16, u, qh, rope, xo, ph, nw, cwb, red, flag, prof, total;
  int kmax, uf;
};
constexpr int DK_XO = 256;   // owned rows of x kept in shared memory
constexpr int CONS_T = DK_THREADS - 32;  // consumer threads
constexpr int DK_CWW = 64;   // words of chain-warp bits (chunks per CTA < 32 * DK_CWW - 31)

__host__ __device__ inline size_t up16(size_t x) { return (x + 15) & ~(size_t)15; }

__host__ __device__ inline Layout dk_layout(int n_embd, int n_ff, int qdim, int n_ctx, int n_layer) {
  Layout L;
  int km = n_embd > n_ff ? n_embd : n_ff;
  km = km > qdim ? km : qdim;
  L.kmax = (km + 15) / 16 * 16;
  int uf = DK_NB * DK_TS;
  uf = uf > km ? uf : km;
  uf = uf > n_ctx + 4 + CONS_T ? uf : n_ctx + 4 + CONS_T;  // scores, then the fast order's value partials
  L.uf = (uf + 3) / 4 * 4;
  size_t o = 0;
  L.ring = o; o += (size_t)DK_NS * DK_SLOT;
  L.full = o; o += DK_NS * 8;
  L.empty = o; o += DK_NS * 8;
  o = up16(o);
  L.desc = o; o += DK_NS * sizeof(DChunk);
  L.aq = o; o += up16(L.kmax);
  L.ad = o; o += up16((size_t)L.kmax / 32 * 4);
  L.as = o; o += up16((size_t)L.kmax / 32 * 4);
  L.as16 = o; o += up16((size_t)L.kmax / 16 * 4);
  L.u = o; o += (size_t)L.uf * 4;
  L.qh = o; o += 3 * 256 * 4;  // q, current k, current v of one head
  L.rope = o; o += 2 * 128 * 4;  // cos, sin of this step's position
  L.xo = o; o += DK_XO * 4;
  L.ph = o; o += up16((size_t)(4 * n_layer + 2) * 4);
  L.nw = o; o += up16((size_t)n_embd * 4);  // the next RMSNorm's weights
  L.cwb = o; o += DK_CWW * 4;               // chain-warp bit per chunk of this CTA
  L.red = o; o += 64 * 4;
  L.flag = o; o += 16;  // [0] abort
  L.prof = o; o += 8 * 8;  // profile cycle accumulators
  L.total = o;
  return L;
}

struct Smem {
  uint8_t *ring;
  uint64_t *full, *empty;
  DChunk *desc;
  float *rope, *xo, *nw;
  int *ph;
  uint32_t *cwb;
  int8_t *aq;
  float *ad;
  float *as;     // per 32-block sum of q, as a float (exact)
  int32_t *as16;  // per 16-element sum of q
  float *u, *qh, *red;
  volatile int *flag;  // [0] abort
  unsigned long long *prof;
};

__device__ __forceinline__ Smem carve(uint8_t *base, const Layout &L) {
  Smem s;
  s.ring = base + L.ring;
  s.full = (uint64_t *)(base + L.full);
  s.empty = (uint64_t *)(base + L.empty);
  s.desc = (DChunk *)(base + L.desc);
  s.rope = (float *)(base + L.rope);
  s.xo = (float *)(base + L.xo);
  s.nw = (float *)(base + L.nw);
  s.ph = (int *)(base + L.ph);
  s.cwb = (uint32_t *)(base + L.cwb);
  s.aq = (int8_t *)(base + L.aq);
  s.ad = (float *)(base + L.ad);
  s.as = (float *)(base + L.as);
  s.as16 = (int32_t *)(base + L.as16);
  s.u = (float *)(base + L.u);
  s.qh = (float *)(base + L.qh);
  s.red = (float *)(base + L.red);
  s.flag = (volatile int *)(base + L.flag);
  s.prof = (unsigned long long *)(base + L.prof);
  return s;
}

__host__ __device__ inline int dk_gpb(int t) { return (t == T_Q4_K || t == T_Q6_K) ? 4 : 1; }
__host__ __device__ inline int dk_tpg(int t) { return t == T_Q4_K ? 2 : (t == T_Q6_K ? 4 : 1); }

__device__ __forceinline__ void sst_v4(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ void sst_v2(uint32_t a, uint32_t x, uint32_t y) {
  asm volatile("st.shared.v2.u32 [%0], {%1,%2};" ::"r"(a), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void sst_i(uint32_t a, int v) { asm volatile("st.shared.s32 [%0], %1;" ::"r"(a), "r"(v) : "memory"); }

// The Q8 activation in shared memory, by shared address: q [k] i8, d [k/32]
// f32, s [k/32] f32 block sums, s16 [k/16] i32 half-block sums.
struct DAct {
  uint32_t q, d, s, s16;
};

// Q8Act::prepare (quant_int.rs:36-53) of one 32-block held E = 32 / L
// elements per lane in an aligned group of L lanes: amax of |x| ignoring NaN,
// d = amax/127, inv = 1/d (0 if d == 0), q = clamp(round_half_away(x*inv),
// +-127), NaN -> 0.  Besides q and d it stores the sum of q as a float
// (exact: |sum| <= 4064) and the sums of q over each 16-element half.  With
// L > 1 all 32 lanes of the warp must call it (the group reductions
// shuffle).  q_sa: this lane's E bytes; b: the block.
template <int L>
__device__ __forceinline__ void q8_lanes(const float (&v)[32 / L], bool store, int l, uint32_t q_sa, const DAct &A,
                                         int b) {
  constexpr int E = 32 / L;
  float amax = 0.0f;  // every |x| below is >= 0, so starting at 0 leaves the maximum unchanged
#pragma unroll
  for (int i = 0; i < E; i++) {
    const float a = fabsf(v[i]);
    const float t = a > 0.0f ? a : 0.0f;  // NaN -> 0
    amax = t > amax ? t : amax;
  }
#pragma unroll
  for (int o = 1; o < L; o <<= 1) {
    const float t = __shfl_xor_sync(0xffffffffu, amax, o);
    amax = t > amax ? t : amax;
  }
  const float dd = fdiv(amax, 127.0f);
  const float inv = dd > 0.0f ? fdiv(1.0f, dd) : 0.0f;
  uint32_t w[E / 4];
  int sh[2] = {0, 0};  // sums over this lane's elements of each 16-element half
#pragma unroll
  for (int j = 0; j < E / 4; j++) {
    uint32_t word = 0;
#pragma unroll
    for (int u = 0; u < 4; u++) {
      float r = roundf(fmul(v[4 * j + u], inv));
      r = r < -127.0f ? -127.0f : r;
      r = r > 127.0f ? 127.0f : r;
      const int qi = isnan(r) ? 0 : (int)r;
      sh[j * 4 >= 16 ? 1 : 0] += qi;
      word |= (uint32_t)(qi & 0xFF) << (8 * u);
    }
    w[j] = word;
  }
  static_assert(L == 1 || L == 2 || L == 4, "4, 2 or 1 lanes per block");
  int h0 = sh[0], h1 = sh[1];
  if (L == 4) {  // lanes 0-1 hold the first half, lanes 2-3 the second
    const int pair = sh[0] + __shfl_xor_sync(0xffffffffu, sh[0], 1);
    const int other = __shfl_xor_sync(0xffffffffu, pair, 2);
    h0 = (l & 2) ? other : pair;
    h1 = (l & 2) ? pair : other;
  } else if (L == 2) {  // lane 0 holds the first half, lane 1 the second
    const int other = __shfl_xor_sync(0xffffffffu, sh[0], 1);
    h0 = (l & 1) ? other : sh[0];
    h1 = (l & 1) ? sh[0] : other;
  }
  if (store) {
    if constexpr (E == 32) {
      sst_v4(q_sa, w[0], w[1], w[2], w[3]);
      sst_v4(q_sa + 16, w[4], w[5], w[6], w[7]);
    } else if constexpr (E == 16) {
      sst_v4(q_sa, w[0], w[1], w[2], w[3]);
    } else {
      sst_v2(q_sa, w[0], w[1]);
    }
    if (l == 0) {
      sst_f(A.d + 4u * (uint32_t)b, dd);
      sst_f(A.s + 4u * (uint32_t)b, (float)(h0 + h1));
      sst_v2(A.s16 + 8u * (uint32_t)b, (uint32_t)h0, (uint32_t)h1);
    }
  }
}

// Sequential float chains over shared memory (shared addresses, byte
// strides).  The reference adds terms one at a time, so only the add itself
// may sit on the dependency path: operands are loaded a batch of eight ahead
// of the adds that consume them.
//   acc + p[0] + p[s] + ... + p[(n-1)s], in that order.
__device__ __forceinline__ float chain_add(float acc, uint32_t p, uint32_t s, int n) {
  int j = 0;
  if (n >= 8) {
    float cur[8];
#pragma unroll
    for (int u = 0; u < 8; u++) cur[u] = sld_f(p + u * s);
    for (j = 8; j + 8 <= n; j += 8) {
      float nxt[8];
      const uint32_t q = p + (uint32_t)j * s;
#pragma unroll
      for (int u = 0; u < 8; u++) nxt[u] = sld_f(q + u * s);
#pragma unroll
      for (int u = 0; u < 8; u++) acc = fadd(acc, cur[u]);
#pragma unroll
      for (int u = 0; u < 8; u++) cur[u] = nxt[u];
    }
#pragma unroll
    for (int u = 0; u < 8; u++) acc = fadd(acc, cur[u]);
  }
  for (; j < n; j++) acc = fadd(acc, sld_f(p + (uint32_t)j * s));
  return acc;
}

__device__ __forceinline__ float add8(float acc, const float4 a, const float4 b) {
  acc = fadd(acc, a.x); acc = fadd(acc, a.y); acc = fadd(acc, a.z); acc = fadd(acc, a.w);
  acc = fadd(acc, b.x); acc = fadd(acc, b.y); acc = fadd(acc, b.z); acc = fadd(acc, b.w);
  return acc;
}

//   acc + p[0] + p[1] + ... + p[n-1] over contiguous floats (p 16-byte
// aligned, readable up to the next multiple of eight): 128-bit loads a batch
// of eight ahead of the adds, no scalar tail.  The last batch's slots past n
// add +0.0, an exact identity here: the sum starts at +0.0 and, rounding to
// nearest, never becomes -0.0.
__device__ __forceinline__ float chain_add_v(float acc, uint32_t p, int n) {
  const int nb = (n + 7) >> 3;
  if (nb == 0) return acc;
  // two batches of eight in flight ahead of the adds
  float4 a = sld_v4f(p), b = sld_v4f(p + 16);
  float4 a2 = nb > 1 ? sld_v4f(p + 32) : make_float4(0.f, 0.f, 0.f, 0.f), b2 = nb > 1 ? sld_v4f(p + 48) : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = 2; i < nb; i++) {
    const float4 na = sld_v4f(p + 32u * i), nb8 = sld_v4f(p + 32u * i + 16u);
    acc = add8(acc, a, b);
    a = a2;
    b = b2;
    a2 = na;
    b2 = nb8;
  }
  if (nb > 1) {
    acc = add8(acc, a, b);
    a = a2;
    b = b2;
  }
  const int r = n - 8 * (nb - 1);  // live slots of the last batch, 1..8
  const float4 za = make_float4(a.x, r > 1 ? a.y : 0.0f, r > 2 ? a.z : 0.0f, r > 3 ? a.w : 0.0f);
  const float4 zb = make_float4(r > 4 ? b.x : 0.0f, r > 5 ? b.y : 0.0f, r > 6 ? b.z : 0.0f, r > 7 ? b.w : 0.0f);
  return add8(acc, za, zb);
}

// fma(p[(n-1)s], p[(n-1)s], ... fma(p[0], p[0], acc)): one f32_sum_sq lane.
__device__ __forceinline__ float chain_sq(float acc, uint32_t p, uint32_t s, int n) {
  int j = 0;
  if (n >= 8) {
    float cur[8];
#pragma unroll
    for (int u = 0; u < 8; u++) cur[u] = sld_f(p + u * s);
    for (j = 8; j + 8 <= n; j += 8) {
      float nxt[8];
      const uint32_t q = p + (uint32_t)j * s;
#pragma unroll
      for (int u = 0; u < 8; u++) nxt[u] = sld_f(q + u * s);
#pragma unroll
      for (int u = 0; u < 8; u++) acc = __fmaf_rn(cur[u], cur[u], acc);
#pragma unroll
      for (int u = 0; u < 8; u++) cur[u] = nxt[u];
    }
#pragma unroll
    for (int u = 0; u < 8; u++) acc = __fmaf_rn(cur[u], cur[u], acc);
  }
  for (; j < n; j++) {
    const float x = sld_f(p + (uint32_t)j * s);
    acc = __fmaf_rn(x, x, acc);
  }
  return acc;
}

// acc + e_0*v_0 + e_1*v_1 + ... with the terms of zero weights skipped
// (model.rs:1076-1085).  A skipped term adds -0.0, which leaves every float
// (signed zeros and NaN included) unchanged, so the product and the choice
// stay off the dependency path.  e: 4-byte stride, v: byte stride vs.
__device__ __forceinline__ float chain_wv(float acc, uint32_t e, uint32_t v, uint32_t vs, int n) {
  // e is 16-byte aligned: the weights of eight positions come in two vector loads
  auto term = [](float ew, float vv) { return ew != 0.0f ? fmul(ew, vv) : -0.0f; };
  int j = 0;
  if (n >= 8) {
    float4 ca = sld_v4f(e), cb = sld_v4f(e + 16);
    float cv[8];
#pragma unroll
    for (int u = 0; u < 8; u++) cv[u] = sld_f(v + u * vs);
    for (j = 8; j + 8 <= n; j += 8) {
      const float4 na = sld_v4f(e + 4 * j), nb = sld_v4f(e + 4 * j + 16);
      float nv[8];
#pragma unroll
      for (int u = 0; u < 8; u++) nv[u] = sld_f(v + (uint32_t)(j + u) * vs);
      const float ce[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
#pragma unroll
      for (int u = 0; u < 8; u++) acc = fadd(acc, term(ce[u], cv[u]));
      ca = na;
      cb = nb;
#pragma unroll
      for (int u = 0; u < 8; u++) cv[u] = nv[u];
    }
    const float ce[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
#pragma unroll
    for (int u = 0; u < 8; u++) acc = fadd(acc, term(ce[u], cv[u]));
  }
  for (; j < n; j++) acc = fadd(acc, term(sld_f(e + 4 * j), sld_f(v + (uint32_t)j * vs)));
  return acc;
}

// ---------------------------------------------------------------- term items
// The reference's row dots (quant_int.rs:282-419, lanes::*) add one float
// term per (sub-)block to the row's accumulator.  An item computes the terms
// of one staged block (Q8_0, Q4_0) or superblock (Q4_K: 8 terms, Q6_K: 16) of
// one row and stores them contiguously at t_a (term i at t_a + 4i; 16-byte
// aligned for the 8-term items).  Integer dots are exact
// in any order; every float expression keeps the reference's operand order.

__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {  // unsigned bytes of a times signed bytes of b
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Shared-memory loads and stores are volatile asm, which keeps them in
// program order: every item issues all its loads first, computes, and stores
// its terms last, so the loads' latencies overlap instead of adding up.

// lanes::q4_k (quant_int.rs:354-365): term_j = (d*da_j)*sc_j*dot_j - (da_j*dmin)*m_j*sa_j.
__device__ __forceinline__ void sst_v4f(uint32_t a, float x, float y, float z, float w) {
  asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(a), "f"(x), "f"(y), "f"(z), "f"(w) : "memory");
}

__device__ __forceinline__ void item_q4k(uint32_t w_a, int blk, const DAct &A, uint32_t t_a) {
  const uint32_t xq = A.q + (uint32_t)blk * 256u, xf = (uint32_t)blk * 32u;
  const uint4 hdr = sld_v4(w_a);
  uint4 w[8];
  int4 x[16];
  float da[8], sa[8];
#pragma unroll
  for (int i = 0; i < 8; i++) w[i] = sld_v4(w_a + 16 + 16 * i);  // pair p: w[2p] (lo16), w[2p+1]
#pragma unroll
  for (int i = 0; i < 16; i++) x[i] = sld_v4i(xq + 16u * i);  // sub-block j: x[2j], x[2j+1]
  {  // the superblock's eight activation scales and block sums: two 16-byte loads each
    const float4 d0 = sld_v4f(A.d + xf), d1 = sld_v4f(A.d + xf + 16), s0 = sld_v4f(A.s + xf), s1 = sld_v4f(A.s + xf + 16);
    da[0] = d0.x; da[1] = d0.y; da[2] = d0.z; da[3] = d0.w; da[4] = d1.x; da[5] = d1.y; da[6] = d1.z; da[7] = d1.w;
    sa[0] = s0.x; sa[1] = s0.y; sa[2] = s0.z; sa[3] = s0.w; sa[4] = s1.x; sa[5] = s1.y; sa[6] = s1.z; sa[7] = s1.w;
  }
  const float d = f16f((uint16_t)(hdr.x & 0xFFFFu)), dmin = f16f((uint16_t)(hdr.x >> 16));
  // get_scale_min_k4 (quant.rs:80-86) for all eight sub-blocks, a byte each:
  // the 12 scale bytes are hdr.y | hdr.z | hdr.w.
  const uint32_t sc_lo = hdr.y & 0x3F3F3F3Fu, m_lo = hdr.z & 0x3F3F3F3Fu;
  const uint32_t sc_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
  const uint32_t m_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
  const uint32_t M = 0x0F0F0F0Fu, H = 0xF0F0F0F0u;
  float t[8];
#pragma unroll
  for (int p = 0; p < 4; p++) {  // sub-blocks 2p (low nibbles) and 2p + 1 (high nibbles, dotted in place: 16x)
    const uint4 w0 = w[2 * p], w1 = w[2 * p + 1];
    const int4 x0 = x[4 * p], x1 = x[4 * p + 1], x2 = x[4 * p + 2], x3 = x[4 * p + 3];
    int d0a = 0, d0b = 0, d1a = 0, d1b = 0;
    d0a = __dp4a((int)(w0.x & M), x0.x, d0a); d0b = __dp4a((int)(w0.y & M), x0.y, d0b);
    d0a = __dp4a((int)(w0.z & M), x0.z, d0a); d0b = __dp4a((int)(w0.w & M), x0.w, d0b);
    d0a = __dp4a((int)(w1.x & M), x1.x, d0a); d0b = __dp4a((int)(w1.y & M), x1.y, d0b);
    d0a = __dp4a((int)(w1.z & M), x1.z, d0a); d0b = __dp4a((int)(w1.w & M), x1.w, d0b);
    d1a = dp4a_us(w0.x & H, x2.x, d1a); d1b = dp4a_us(w0.y & H, x2.y, d1b);
    d1a = dp4a_us(w0.z & H, x2.z, d1a); d1b = dp4a_us(w0.w & H, x2.w, d1b);
    d1a = dp4a_us(w1.x & H, x3.x, d1a); d1b = dp4a_us(w1.y & H, x3.y, d1b);
    d1a = dp4a_us(w1.z & H, x3.z, d1a); d1b = dp4a_us(w1.w & H, x3.w, d1b);
    const int dot0 = d0a + d0b, dot1 = (d1a + d1b) >> 4;
    const uint32_t scw = p < 2 ? sc_lo : sc_hi, mw = p < 2 ? m_lo : m_hi;
    const int sh = (2 * p & 3) * 8;
    const float sc0 = (float)((scw >> sh) & 0xFFu), m0 = (float)((mw >> sh) & 0xFFu);
    const float sc1 = (float)((scw >> (sh + 8)) & 0xFFu), m1 = (float)((mw >> (sh + 8)) & 0xFFu);
    t[2 * p] = fsub(fmul(fmul(fmul(d, da[2 * p]), sc0), (float)dot0), fmul(fmul(fmul(da[2 * p], dmin), m0), sa[2 * p]));
    t[2 * p + 1] =
        fsub(fmul(fmul(fmul(d, da[2 * p + 1]), sc1), (float)dot1), fmul(fmul(fmul(da[2 * p + 1], dmin), m1), sa[2 * p + 1]));
  }
  sst_v4f(t_a, t[0], t[1], t[2], t[3]);
  sst_v4f(t_a + 16, t[4], t[5], t[6], t[7]);
}

// lanes::q6_k (quant_int.rs:386-413) for half h of a superblock: per
// 16-element piece, order (g, s), term = ((d*scale)*da)*dot with
// dot = sum((q - 32) a), computed as sum(q a) - 32 sum(a).  Term i of the
// half is the superblock's term 8h + i.
__device__ __forceinline__ void item_q6k(uint32_t w_a, uint32_t d_a, int blk, int h, const DAct &A, uint32_t t_a) {
  const uint2 scw = sld_v2(w_a + 192 + 8 * h);  // this half's eight scales
  const uint16_t dbits = sld_u16(d_a);
  uint4 qa[2], qb[2], qh[2];
  int4 x[8];
  float da[4];
  int s16[8];
#pragma unroll
  for (int g = 0; g < 2; g++) {
    qa[g] = sld_v4(w_a + h * 64 + g * 16);
    qb[g] = sld_v4(w_a + h * 64 + 32 + g * 16);
    qh[g] = sld_v4(w_a + 128 + h * 32 + g * 16);
  }
#pragma unroll
  for (int s = 0; s < 4; s++) {
    const uint32_t ab = (uint32_t)(blk * 8 + 4 * h + s);  // activation block
    x[2 * s] = sld_v4i(A.q + ab * 32u);
    x[2 * s + 1] = sld_v4i(A.q + ab * 32u + 16u);
  }
  {  // the half's four activation scales and eight 16-element sums (16-byte loads)
    const uint32_t ab0 = (uint32_t)(blk * 8 + 4 * h);
    const float4 dv = sld_v4f(A.d + ab0 * 4u);
    const int4 h0 = sld_v4i(A.s16 + ab0 * 8u), h1 = sld_v4i(A.s16 + ab0 * 8u + 16u);
    da[0] = dv.x; da[1] = dv.y; da[2] = dv.z; da[3] = dv.w;
    s16[0] = h0.x; s16[1] = h0.y; s16[2] = h0.z; s16[3] = h0.w;
    s16[4] = h1.x; s16[5] = h1.y; s16[6] = h1.z; s16[7] = h1.w;
  }
  const float d = f16f(dbits);
  const unsigned long long sw = (unsigned long long)scw.y << 32 | scw.x;
  float t[8];
#pragma unroll
  for (int g = 0; g < 2; g++) {
#pragma unroll
    for (int s = 0; s < 4; s++) {
      const int4 xs = x[2 * s + g];
      int pa = 0, pb = 0;
#pragma unroll
      for (int w = 0; w < 4; w++) {  // quant_int.rs:386-394 unpacking, four bytes at a time (0..63)
        const uint32_t lo = word_of(s & 1 ? qb[g] : qa[g], w), hh = word_of(qh[g], w);
        const uint32_t q = ((s & 2 ? lo >> 4 : lo) & 0x0F0F0F0Fu) | ((s == 0 ? hh << 4 : s == 1 ? hh << 2 : s == 2 ? hh : hh >> 2) & 0x30303030u);
        const int xw = w == 0 ? xs.x : w == 1 ? xs.y : w == 2 ? xs.z : xs.w;
        if (w & 1) pb = __dp4a((int)q, xw, pb);
        else pa = __dp4a((int)q, xw, pa);
      }
      const int dot = pa + pb - 32 * s16[2 * s + g];
      const float scale = (float)(int8_t)(uint8_t)(sw >> (8 * (g + 2 * s)));
      t[g * 4 + s] = fmul(fmul(fmul(d, scale), da[s]), (float)dot);
    }
  }
  sst_v4f(t_a, t[0], t[1], t[2], t[3]);
  sst_v4f(t_a + 16, t[4], t[5], t[6], t[7]);
}

// lanes::q8_0 (quant_int.rs:291-296): term = (d*da)*dot.
__device__ __forceinline__ void item_q80(uint32_t w_a, uint32_t d_a, int blk, const DAct &A, uint32_t t_a) {
  const uint4 w0 = sld_v4(w_a), w1 = sld_v4(w_a + 16);
  const uint32_t xa = A.q + (uint32_t)blk * 32u;
  const int4 x0 = sld_v4i(xa), x1 = sld_v4i(xa + 16);
  const float d = f16f(sld_u16(d_a)), da = sld_f(A.d + (uint32_t)blk * 4u);
  int pa = 0, pb = 0;
  pa = __dp4a((int)w0.x, x0.x, pa); pb = __dp4a((int)w0.y, x0.y, pb);
  pa = __dp4a((int)w0.z, x0.z, pa); pb = __dp4a((int)w0.w, x0.w, pb);
  pa = __dp4a((int)w1.x, x1.x, pa); pb = __dp4a((int)w1.y, x1.y, pb);
  pa = __dp4a((int)w1.z, x1.z, pa); pb = __dp4a((int)w1.w, x1.w, pb);
  sst_f(t_a, fmul(fmul(d, da), (float)(pa + pb)));
}

// lanes::q4_0 (quant_int.rs:316-323): term = (d*da)*(dot - 8*sa).
__device__ __forceinline__ void item_q40(uint32_t w_a, uint32_t d_a, int blk, const DAct &A, uint32_t t_a) {
  const uint4 w = sld_v4(w_a);
  const uint32_t xa = A.q + (uint32_t)blk * 32u;
  const int4 x0 = sld_v4i(xa), x1 = sld_v4i(xa + 16);
  const float d = f16f(sld_u16(d_a)), da = sld_f(A.d + (uint32_t)blk * 4u), sa = sld_f(A.s + (uint32_t)blk * 4u);
  int pa = 0, pb = 0;
  pa = __dp4a(lo4(w.x), x0.x, pa); pb = __dp4a(lo4(w.y), x0.y, pb);
  pa = __dp4a(lo4(w.z), x0.z, pa); pb = __dp4a(lo4(w.w), x0.w, pb);
  pa = __dp4a(hi4(w.x), x1.x, pa); pb = __dp4a(hi4(w.y), x1.y, pb);
  pa = __dp4a(hi4(w.z), x1.z, pa); pb = __dp4a(hi4(w.w), x1.w, pb);
  sst_f(t_a, fmul(fmul(d, da), fsub((float)(pa + pb), fmul(8.0f, sa))));
}

// ---------------------------------------------------------- fast-order items
// The fast order keeps every integer dot and the Q8 activation bit-exact and
// regroups only the float arithmetic of a row: each item returns one partial
// sum (its terms regrouped algebraically, with fused multiply-adds), and the
// chain adds a row's partials in k order.  Products of exact integers below
// 2^24 (scale x dot, min x block sum) are formed in integer or exact float
// arithmetic first.  The result differs from the reference's sequential
// float chain by rounding only (well inside 1e-3 relative per matvec).

// Q4_K superblock: d * sum_j da_j (sc_j dot_j) - dmin * sum_j da_j (m_j sa_j).
__device__ __forceinline__ void item_q4k_f(uint32_t w_a, int blk, const DAct &A, uint32_t t_a) {
  const uint32_t xq = A.q + (uint32_t)blk * 256u, xf = (uint32_t)blk * 32u;
  const uint4 hdr = sld_v4(w_a);
  uint4 w[8];
  int4 x[16];
  float da[8], sa[8];
#pragma unroll
  for (int i = 0; i < 8; i++) w[i] = sld_v4(w_a + 16 + 16 * i);
#pragma unroll
  for (int i = 0; i < 16; i++) x[i] = sld_v4i(xq + 16u * i);
  {
    const float4 d0 = sld_v4f(A.d + xf), d1 = sld_v4f(A.d + xf + 16), s0 = sld_v4f(A.s + xf), s1 = sld_v4f(A.s + xf + 16);
    da[0] = d0.x; da[1] = d0.y; da[2] = d0.z; da[3] = d0.w; da[4] = d1.x; da[5] = d1.y; da[6] = d1.z; da[7] = d1.w;
    sa[0] = s0.x; sa[1] = s0.y; sa[2] = s0.z; sa[3] = s0.w; sa[4] = s1.x; sa[5] = s1.y; sa[6] = s1.z; sa[7] = s1.w;
  }
  const float d = f16f((uint16_t)(hdr.x & 0xFFFFu)), dmin = f16f((uint16_t)(hdr.x >> 16));
  const uint32_t sc_lo = hdr.y & 0x3F3F3F3Fu, m_lo = hdr.z & 0x3F3F3F3Fu;
  const uint32_t sc_hi = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
  const uint32_t m_hi = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
  const uint32_t M = 0x0F0F0F0Fu, H = 0xF0F0F0F0u;
  float a1 = 0.0f, a2 = 0.0f;
#pragma unroll
  for (int p = 0; p < 4; p++) {
    const uint4 w0 = w[2 * p], w1 = w[2 * p + 1];
    const int4 x0 = x[4 * p], x1 = x[4 * p + 1], x2 = x[4 * p + 2], x3 = x[4 * p + 3];
    int d0a = 0, d0b = 0, d1a = 0, d1b = 0;
    d0a = __dp4a((int)(w0.x & M), x0.x, d0a); d0b = __dp4a((int)(w0.y & M), x0.y, d0b);
    d0a = __dp4a((int)(w0.z & M), x0.z, d0a); d0b = __dp4a((int)(w0.w & M), x0.w, d0b);
    d0a = __dp4a((int)(w1.x & M), x1.x, d0a); d0b = __dp4a((int)(w1.y & M), x1.y, d0b);
    d0a = __dp4a((int)(w1.z & M), x1.z, d0a); d0b = __dp4a((int)(w1.w & M), x1.w, d0b);
    d1a = dp4a_us(w0.x & H, x2.x, d1a); d1b = dp4a_us(w0.y & H, x2.y, d1b);
    d1a = dp4a_us(w0.z & H, x2.z, d1a); d1b = dp4a_us(w0.w & H, x2.w, d1b);
    d1a = dp4a_us(w1.x & H, x3.x, d1a); d1b = dp4a_us(w1.y & H, x3.y, d1b);
    d1a = dp4a_us(w1.z & H, x3.z, d1a); d1b = dp4a_us(w1.w & H, x3.w, d1b);
    const int dot0 = d0a + d0b, dot1 = (d1a + d1b) >> 4;
    const uint32_t scw = p < 2 ? sc_lo : sc_hi, mw = p < 2 ? m_lo : m_hi;
    const int sh = (2 * p & 3) * 8;
    const int sc0 = (int)((scw >> sh) & 0xFFu), sc1 = (int)((scw >> (sh + 8)) & 0xFFu);
    const float m0 = (float)((mw >> sh) & 0xFFu), m1 = (float)((mw >> (sh + 8)) & 0xFFu);
    a1 = __fmaf_rn(da[2 * p], (float)(sc0 * dot0), a1);  // |sc dot| <= 63 * 60960 < 2^24: exact
    a2 = __fmaf_rn(da[2 * p], m0 * sa[2 * p], a2);      // |m sa| <= 63 * 4064: exact
    a1 = __fmaf_rn(da[2 * p + 1], (float)(sc1 * dot1), a1);
    a2 = __fmaf_rn(da[2 * p + 1], m1 * sa[2 * p + 1], a2);
  }
  sst_f(t_a, __fmaf_rn(d, a1, -(dmin * a2)));
}

// Q6_K half superblock: d * sum_s da_s (sum_g scale_gs dot_gs).
__device__ __forceinline__ void item_q6k_f(uint32_t w_a, uint32_t d_a, int blk, int h, const DAct &A, uint32_t t_a) {
  const uint2 scw = sld_v2(w_a + 192 + 8 * h);
  const uint16_t dbits = sld_u16(d_a);
  uint4 qa[2], qb[2], qh[2];
  int4 x[8];
  float da[4];
  int s16[8];
#pragma unroll
  for (int g = 0; g < 2; g++) {
    qa[g] = sld_v4(w_a + h * 64 + g * 16);
    qb[g] = sld_v4(w_a + h * 64 + 32 + g * 16);
    qh[g] = sld_v4(w_a + 128 + h * 32 + g * 16);
  }
#pragma unroll
  for (int s = 0; s < 4; s++) {
    const uint32_t ab = (uint32_t)(blk * 8 + 4 * h + s);
    x[2 * s] = sld_v4i(A.q + ab * 32u);
    x[2 * s + 1] = sld_v4i(A.q + ab * 32u + 16u);
  }
  {
    const uint32_t ab0 = (uint32_t)(blk * 8 + 4 * h);
    const float4 dv = sld_v4f(A.d + ab0 * 4u);
    const int4 h0 = sld_v4i(A.s16 + ab0 * 8u), h1 = sld_v4i(A.s16 + ab0 * 8u + 16u);
    da[0] = dv.x; da[1] = dv.y; da[2] = dv.z; da[3] = dv.w;
    s16[0] = h0.x; s16[1] = h0.y; s16[2] = h0.z; s16[3] = h0.w;
    s16[4] = h1.x; s16[5] = h1.y; s16[6] = h1.z; s16[7] = h1.w;
  }
  const unsigned long long sw = (unsigned long long)scw.y << 32 | scw.x;
  float acc = 0.0f;
#pragma unroll
  for (int s = 0; s < 4; s++) {
    int is = 0;  // |sum over g of scale * dot| <= 2 * 128 * 65024 < 2^24: exact as a float
#pragma unroll
    for (int g = 0; g < 2; g++) {
      const int4 xs = x[2 * s + g];
      int pa = 0, pb = 0;
#pragma unroll
      for (int w = 0; w < 4; w++) {
        const uint32_t lo = word_of(s & 1 ? qb[g] : qa[g], w), hh = word_of(qh[g], w);
        const uint32_t q = ((s & 2 ? lo >> 4 : lo) & 0x0F0F0F0Fu) | ((s == 0 ? hh << 4 : s == 1 ? hh << 2 : s == 2 ? hh : hh >> 2) & 0x30303030u);
        const int xw = w == 0 ? xs.x : w == 1 ? xs.y : w == 2 ? xs.z : xs.w;
        if (w & 1) pb = __dp4a((int)q, xw, pb);
        else pa = __dp4a((int)q, xw, pa);
      }
      is += (int)(int8_t)(uint8_t)(sw >> (8 * (g + 2 * s))) * (pa + pb - 32 * s16[2 * s + g]);
    }
    acc = __fmaf_rn(da[s], (float)is, acc);
  }
  sst_f(t_a, f16f(dbits) * acc);
}

// Q8_0 / Q4_0: FQ consecutive blocks (n <= FQ of them live) of one row.
constexpr int FQ = 4;
__device__ __forceinline__ void item_q80_f(uint32_t w_a, uint32_t d_a, int blk, int n, const DAct &A, uint32_t t_a) {
  uint4 w[2 * FQ];
  int4 x[2 * FQ];
  float da[FQ];
  uint16_t db[FQ];
#pragma unroll
  for (int b = 0; b < FQ; b++) {
    const int bb = b < n ? b : 0;  // dead slots re-read block 0 (in range) and add nothing
    w[2 * b] = sld_v4(w_a + 32u * bb);
    w[2 * b + 1] = sld_v4(w_a + 32u * bb + 16u);
    const uint32_t xa = A.q + (uint32_t)(blk + bb) * 32u;
    x[2 * b] = sld_v4i(xa);
    x[2 * b + 1] = sld_v4i(xa + 16);
    db[b] = sld_u16(d_a + 2u * bb);
    da[b] = sld_f(A.d + (uint32_t)(blk + bb) * 4u);
  }
  float acc = 0.0f;
#pragma unroll
  for (int b = 0; b < FQ; b++) {
    const uint4 w0 = w[2 * b], w1 = w[2 * b + 1];
    const int4 x0 = x[2 * b], x1 = x[2 * b + 1];
    int pa = 0, pb = 0;
    pa = __dp4a((int)w0.x, x0.x, pa); pb = __dp4a((int)w0.y, x0.y, pb);
    pa = __dp4a((int)w0.z, x0.z, pa); pb = __dp4a((int)w0.w, x0.w, pb);
    pa = __dp4a((int)w1.x, x1.x, pa); pb = __dp4a((int)w1.y, x1.y, pb);
    pa = __dp4a((int)w1.z, x1.z, pa); pb = __dp4a((int)w1.w, x1.w, pb);
    if (b < n) acc = __fmaf_rn(f16f(db[b]) * da[b], (float)(pa + pb), acc);
  }
  sst_f(t_a, acc);
}
__device__ __forceinline__ void item_q40_f(uint32_t w_a, uint32_t d_a, int blk, int n, const DAct &A, uint32_t t_a) {
  uint4 w[FQ];
  int4 x[2 * FQ];
  float da[FQ], sa[FQ];
  uint16_t db[FQ];
#pragma unroll
  for (int b = 0; b < FQ; b++) {
    const int bb = b < n ? b : 0;
    w[b] = sld_v4(w_a + 16u * bb);
    const uint32_t xa = A.q + (uint32_t)(blk + bb) * 32u;
    x[2 * b] = sld_v4i(xa);
    x[2 * b + 1] = sld_v4i(xa + 16);
    db[b] = sld_u16(d_a + 2u * bb);
    da[b] = sld_f(A.d + (uint32_t)(blk + bb) * 4u);
    sa[b] = sld_f(A.s + (uint32_t)(blk + bb) * 4u);
  }
  float acc = 0.0f;
#pragma unroll
  for (int b = 0; b < FQ; b++) {
    const uint4 wv = w[b];
    const int4 x0 = x[2 * b], x1 = x[2 * b + 1];
    int pa = 0, pb = 0;
    pa = __dp4a(lo4(wv.x), x0.x, pa); pb = __dp4a(lo4(wv.y), x0.y, pb);
    pa = __dp4a(lo4(wv.z), x0.z, pa); pb = __dp4a(lo4(wv.w), x0.w, pb);
    pa = __dp4a(hi4(wv.x), x1.x, pa); pb = __dp4a(hi4(wv.y), x1.y, pb);
    pa = __dp4a(hi4(wv.z), x1.z, pa); pb = __dp4a(hi4(wv.w), x1.w, pb);
    // dot - 8 sa is an exact integer (sa is an exact float)
    if (b < n) acc = __fmaf_rn(f16f(db[b]) * da[b], (float)(pa + pb - 8 * (int)sa[b]), acc);
  }
  sst_f(t_a, acc);
}

// Partial sums per row of a chunk in the fast order: one per item.
__host__ __device__ inline int dk_items_fast(int type, int nblk) {
  return type == T_Q4_K ? nblk : type == T_Q6_K ? 2 * nblk : (nblk + FQ - 1) / FQ;
}
// Term-buffer floats between rows for n partials (as term_pitch: a multiple
// of 8 rounded up, then an odd multiple of 4).
__host__ __device__ inline int dk_pitch(int n) { return 4 * (((n + 7) / 8) * 2 + 1); }

// History positions [r0, r1) of 0..pos-1 that attention unit j of J scores:
// near-equal contiguous shares starting on multiples of 4 (the K copies move
// whole groups of 4 positions).
__host__ __device__ inline void att_range(int pos, int j, int J, int &r0, int &r1) {
  r0 = j == 0 ? 0 : (int)(((long)pos * j / J) & ~3L);
  r1 = j == J - 1 ? pos : (int)(((long)pos * (j + 1) / J) & ~3L);
}

// A chunk descriptor copied from shared memory into registers.
__device__ __forceinline__ DChunk load_desc(uint32_t a) {
  DChunk c;
  uint4 *w = reinterpret_cast<uint4 *>(&c);
  w[0] = sld_v4(a);
  w[1] = sld_v4(a + 16);
  w[2] = sld_v4(a + 32);
  w[3] = sld_v4(a + 48);
  return c;
}

// Ring position shared by the producer and every consumer thread: both walk
// the same sequence of transfers.
struct Ring {
  uint32_t slot = 0, par = 0;
  // slot and phase parity of the transfer j places ahead
  __device__ uint32_t slot_at(int j) const { return (slot + j) % DK_NS; }
  __device__ uint32_t par_at(int j) const { return par ^ (((slot + j) / DK_NS) & 1u); }
  __device__ void next() {
    if (++slot == DK_NS) {
      slot = 0;
      par ^= 1u;
    }
  }
};

// ------------------------------------------------------------------ producer
// The whole of warp 0: lane 0 claims each slot (bounded wait on its empty
// barrier), writes the descriptor and arms the full barrier with the byte
// count; then the lanes share out the copies (one per row of a split chunk,
// one per dimension of a K chunk).
template <bool TRACE>
__device__ void producer(const DecodeArgs &a, const Smem &S, int pos, const DChunk *ch, const int *ph) {
  const int lane = threadIdx.x & 31;
  Ring rg;
  uint32_t armed[DK_NS];
  bool used[DK_NS];
  for (int i = 0; i < DK_NS; i++) used[i] = false;
  bool ok = true;
  unsigned long long pst = 0;  // SM cycles spent waiting for a free slot (profile trace)
  auto note = [&](int layer) {
    if ((TRACE && a.trace) && lane == 0) {
      const int i = 1 + DK_TRW * (5 * a.n_layer + 1) + layer;
      if (i < a.n_trace) a.trace[(size_t)blockIdx.x * a.n_trace + i] = pst;
      pst = 0;
    }
  };
  // Claim the next slot for tx bytes (desc: the chunk descriptor, or null);
  // false on abort / timeout, on every lane.
  auto claim = [&](uint32_t tx, const DChunk *desc) -> bool {
    int got = 1;
    if (lane == 0) {
      const long long t0 = (TRACE && a.trace) ? clock64() : 0;
      got = mbar_wait(&S.empty[rg.slot], rg.par ^ 1u, S.flag, 20000u) ? 1 : 0;
      if ((TRACE && a.trace)) pst += (unsigned long long)(clock64() - t0);
      if (!got) {
        if (!*S.flag) atomicCAS(a.err, 0, PK_ERR_TIMEOUT);
        S.flag[0] = 1;
      } else {
        used[rg.slot] = true;
        armed[rg.slot] = rg.par;
        if (desc) S.desc[rg.slot] = *desc;  // visible to the consumers once the full barrier completes
        mbar_expect(&S.full[rg.slot], tx);
      }
    }
    got = __shfl_sync(0xffffffffu, got, 0);
    ok = got != 0;
    return ok;
  };
  const int group = a.n_head / a.n_kv;
  const int ppc = DK_SLOT / (a.dh * 4);
  for (int p = 0; p < a.n_phase && ok; p++) {
    if (p > 0 && (p & 3) == 0) note(p / 4 - 1);
    for (int ci = ph[p]; ci < ph[p + 1] && ok; ci++) {
      const DChunk c = ch[ci];
      const uint32_t dl = c.d ? c.d_len : 0u;
      const uint32_t tx = c.full ? c.q_len + dl : (uint32_t)c.rows * (c.q_len + dl);
      if (!claim(tx, &c)) break;
      uint8_t *dst = S.ring + (size_t)rg.slot * DK_SLOT;
      uint64_t *fb = &S.full[rg.slot];
      if (lane == 0 && ci + 1 < ph[p + 1]) prefetch_l1(ch + ci + 1);
      if (c.full) {
        if (lane == 0) {
          bulk_g2s(dst, c.q, c.q_len, fb);
          if (c.d) bulk_g2s(dst + c.d_off, align16_down(c.d), c.d_len, fb);
        }
      } else {
        const uint32_t pitch = c.q_len + 16u * c.qpad;
        for (int r = lane; r < c.rows; r += 32) {
          bulk_g2s(dst + (size_t)r * pitch, c.q + (size_t)r * c.q_stride, c.q_len, fb);
          if (c.d) bulk_g2s(dst + c.d_off + (size_t)r * c.d_len, align16_down(c.d + (size_t)r * c.d_stride), c.d_len, fb);
        }
      }
      rg.next();
    }
    if ((p & 3) == 0 && p < 4 * a.n_layer && ok) {  // attention of layer p/4: K then V history of each owned unit
      const int L = p >> 2;
      for (int u = blockIdx.x; u < a.n_head * a.att_j && ok; u += gridDim.x) {
        const int h = u / a.att_j, j = u - h * a.att_j;
        const size_t base = ((size_t)L * a.n_kv + h / group) * a.n_ctx * a.dh;
        int r0, r1;
        att_range(pos, j, a.att_j, r0, r1);
        // K (d-major) of the unit's share [r0, r1): one run of positions per
        // dimension, rounded up to a multiple of 4 positions (the slot's extra
        // entries are not read; r0 is a multiple of 4 and n_ctx too).
        for (int p0 = r0; p0 < r1 && ok; p0 += ppc) {
          const int n4 = (min(ppc, r1 - p0) + 3) & ~3;
          if (!claim((uint32_t)(a.dh * n4 * 4), nullptr)) break;
          uint8_t *dst = S.ring + (size_t)rg.slot * DK_SLOT;
          for (int d = lane; d < a.dh; d += 32)
            bulk_g2s(dst + (size_t)d * ppc * 4, a.kcache + base + (size_t)d * a.n_ctx + p0, (uint32_t)n4 * 4,
                     &S.full[rg.slot]);
          rg.next();
        }
        // V (position-major): this unit's att_ds dimensions of every
        // position, tensor-map boxes of DK_VB positions laid end to end, so
        // the slot holds [position][att_ds].  A box that runs past the cache
        // is zero-filled and still counts its full size.
        const int ds = a.att_ds, ppv = DK_SLOT / (ds * 4), row0 = (L * a.n_kv + h / group) * a.n_ctx;
        const uint32_t box = (uint32_t)(DK_VB * ds * 4);
        for (int p0 = 0; p0 < pos && ok; p0 += ppv) {
          const int nb = (min(ppv, pos - p0) + DK_VB - 1) / DK_VB;
          if (!claim((uint32_t)nb * box, nullptr)) break;
          uint8_t *dst = S.ring + (size_t)rg.slot * DK_SLOT;
          for (int b = lane; b < nb; b += 32)
            tma_2d(dst + (size_t)b * box, &a.vmap, j * ds, row0 + p0 + b * DK_VB, &S.full[rg.slot]);
          rg.next();
        }
      }
    }
  }
  note(a.n_layer);
  // Every copy this CTA issued lands before the CTA may exit.
  if (lane == 0)
    for (int i = 0; i < DK_NS; i++)
      if (used[i]) mbar_wait(&S.full[i], armed[i], nullptr);
  __syncwarp();
}

// ------------------------------------------------------------------ consumers
// FAST: the fast float order (see the fast-order items); otherwise every
// float operation follows the reference's order.
template <bool TRACE, bool FAST>
struct Cons {
  const DecodeArgs &a;
  const Smem &S;
  const DChunk *ch;
  const int *ph;
  int pos, tid, ctid, cwarp, lane, own0, cw_base;
  uint32_t ring_a, u_a, desc_a, nw_a;
  DAct act_a;
  Ring rg;
  int mv = 0, mv_total = 0;
  unsigned gen = 0;
  uint32_t epoch = 0;  // this launch's tag epoch
  // chain-warp state
  float acc = 0.0f, gval = 0.0f, best_v = -INFINITY;
  int best_i = INT_MAX;

  __device__ Cons(const DecodeArgs &a_, const Smem &S_, const DChunk *ch_, const int *ph_, int pos_)
      : a(a_), S(S_), ch(ch_), ph(ph_), pos(pos_) {
    tid = threadIdx.x;
    ctid = tid - 32;
    cwarp = ctid >> 5;
    lane = tid & 31;
    mv_total = ph[a.n_phase];  // ph is the shared-memory copy
    epoch = *(volatile const unsigned *)(a.sync + 2);
    own0 = a.own[2 * blockIdx.x];
    cw_base = a.cta_chunk0[blockIdx.x] & 31;  // S.cwb[0] holds the word with this CTA's first chunk
    ring_a = shaddr(S.ring);
    u_a = shaddr(S.u);
    desc_a = shaddr(S.desc);
    nw_a = shaddr(S.nw);
    act_a = DAct{shaddr(S.aq), shaddr(S.ad), shaddr(S.as), shaddr(S.as16)};
  }

  // Ring-data stalls are timed for consumer thread 0 (attention) and the
  // first term thread (matvec phases).
  static constexpr int TT0 = 32 * DK_CHAINS;
  __device__ __forceinline__ void wait_full_at(int j) {  // the transfer j places ahead
    const bool timed = (TRACE && a.trace) && (ctid == 0 || ctid == TT0);
    const long long t0 = timed ? clock64() : 0;
    const bool ok = mbar_wait(&S.full[rg.slot_at(j)], rg.par_at(j), S.flag, DATA_SLEEP_NS);
    if (timed) pacc(ctid == 0 ? 0 : 1, clock64() - t0);
    if (!ok && !*S.flag) {
      atomicCAS(a.err, 0, PK_ERR_TIMEOUT);
      S.flag[0] = 1;
    }
  }
  __device__ __forceinline__ void wait_full() {
    const bool timed = (TRACE && a.trace) && (ctid == 0 || ctid == TT0);
    const long long t0 = timed ? clock64() : 0;
    const bool ok = mbar_wait(&S.full[rg.slot], rg.par, S.flag, DATA_SLEEP_NS);
    if (timed) pacc(ctid == 0 ? 0 : 1, clock64() - t0);
    if (!ok && !*S.flag) {
      atomicCAS(a.err, 0, PK_ERR_TIMEOUT);
      S.flag[0] = 1;
    }
  }

  // Profile trace (only when (TRACE && a.trace) is set), per CTA:
  //   [0] start (ns); phase q = 5L + {qkv, attn, o, gate/up, down} (q = 5n:
  //   the head), base 1 + DK_TRW q: [+0] prologue end, [+1] compute end,
  //   [+2] barrier exit (ns); SM cycles: [+3] waiting for ring data, [+4]
  //   term warps waiting for a term buffer, [+5] term computation, [+6]
  //   chain warp 0 waiting for terms, [+7] chain warp 0 sums + epilogue;
  //   [+8 .. +15] fine stamps (ns) inside the phase;
  //   [1 + DK_TRW (5n + 1) + layer] SM cycles the producer waited for a slot.
  // Accumulators live in shared memory: S.prof[0] data wait of consumer
  // thread 0, [1] of the first term thread, [2..5] the term / chain figures.
  __device__ __forceinline__ void pacc(int i, long long c) {
    if ((TRACE && a.trace)) S.prof[i] += (unsigned long long)c;
  }
  __device__ __forceinline__ void stamp(int i, unsigned long long v) {
    if ((TRACE && a.trace) && i < a.n_trace) a.trace[(size_t)blockIdx.x * a.n_trace + i] = v;
  }
  __device__ __forceinline__ void mark(int q, int j) {
    if ((TRACE && a.trace) && ctid == 0) stamp(1 + DK_TRW * q + j, gtime());
  }
  // fine-grained stamp i (< 8) inside the current phase
  __device__ __forceinline__ void fine(int i) {
    if ((TRACE && a.trace) && ctid == 0) stamp(1 + DK_TRW * (int)gen + 8 + i, gtime());
  }

  __device__ __forceinline__ uint32_t tag_of(int q) const { return (epoch << 10) | (uint32_t)q; }

  // Bounded poll: false (with the error recorded) once the wait has run out
  // or another CTA has failed.  `it` counts the caller's polls.
  __device__ __forceinline__ bool poll_ok(unsigned long long t0, unsigned it) {
    if ((it & 63u) == 63u && *(volatile int *)a.err) {
      S.flag[0] = 1;
      return false;
    }
    if (gtime() - t0 > WAIT_NS) {
      atomicCAS(a.err, 0, PK_ERR_TIMEOUT);
      S.flag[0] = 1;
      return false;
    }
    return true;
  }

  // The end of a phase for this CTA (no grid-wide wait: the next phase's
  // readers poll the tagged words).  True when the kernel is being abandoned.
  __device__ bool phase_end() {
    const int q = (int)gen;
    mark(q, 1);
    if ((TRACE && a.trace)) bar_sync(NB_CONS, CONS);  // every accumulator of this phase is final
    if ((TRACE && a.trace) && ctid == 0) {
      stamp(1 + DK_TRW * q + 3, S.prof[q % 5 == 1 ? 0 : 1]);
      for (int i = 2; i < 6; i++) stamp(1 + DK_TRW * q + 2 + i, S.prof[i]);
      if (q % 5 != 1) {  // matvec phases: chain-add cycles and terms chained (fine slots 6, 7 unused there)
        stamp(1 + DK_TRW * q + 14, S.prof[6]);
        stamp(1 + DK_TRW * q + 15, S.prof[7]);
      }
      for (int i = 0; i < 8; i++) S.prof[i] = 0ull;
    }
    // every consumer is done with this phase's shared buffers; stop together
    const bool stop = bar_or(NB_CONS, CONS, S.flag[0] != 0);
    gen++;
    mark(q, 2);
    return stop;
  }

  // x = dequant_row(token_embd, ids[0]) (model.rs:857-869): kept in the
  // staging buffer for layer 0 and, for the owned rows, in the residual rows.
  __device__ void embed() {
    const uint32_t id = *a.ids;
    const uint8_t *row = a.embd + (size_t)id * a.embd_row_bytes;
    const int o0 = a.own[2 * blockIdx.x], o1 = a.own[2 * blockIdx.x + 1];
    for (int j = ctid; j < a.n_embd; j += CONS) {
      const float v = dequant_elem(a.embd_type, row, j);
      S.u[j] = v;
      if (j >= o0 && j < o1) S.xo[j - o0] = v;
    }
    bar_sync(NB_CONS, CONS);
  }

  // The previous phase's k-vector (tagged words) -> staging buffer.  Each
  // consumer thread reads its words coalesced, re-reads the ones whose tag is
  // not yet `tag` (their writer has not finished), then stores the values.
  // True (on every consumer) when a wait ran out and the kernel stops.
  __device__ bool stage_ll(const unsigned long long *src, int k, uint32_t tag) {
    constexpr int NP = 8;  // word pairs (16-byte loads) in flight per thread
    const unsigned long long t0 = gtime();
    unsigned it = 0;
    const int np = k >> 1;  // k is even; src is 16-byte aligned
    for (int base = 0; base < np; base += NP * CONS) {  // the same trip count on every consumer thread
      unsigned long long w[2 * NP];
#pragma unroll
      for (int j = 0; j < NP; j++) {
        const int i = base + ctid + j * CONS;
        if (i < np) {
          ld_ll2(src + 2 * i, w[2 * j], w[2 * j + 1]);
        } else {
          w[2 * j] = w[2 * j + 1] = (unsigned long long)tag << 32;
        }
      }
      for (;;) {
        bool all = true;
#pragma unroll
        for (int j = 0; j < 2 * NP; j++) all = all && ll_ok(w[j], tag);
        if (all || !poll_ok(t0, ++it)) break;
        __nanosleep(POLL_SLEEP_NS);  // the words come from other SMs through L2: do not spin on issue slots
#pragma unroll
        for (int j = 0; j < NP; j++) {
          const int i = base + ctid + j * CONS;
          if (!ll_ok(w[2 * j], tag) || !ll_ok(w[2 * j + 1], tag)) ld_ll2(src + 2 * i, w[2 * j], w[2 * j + 1]);
        }
      }
#pragma unroll
      for (int j = 0; j < NP; j++) {
        const int i = base + ctid + j * CONS;
        if (i < np) {
          S.u[2 * i] = ll_val(w[2 * j]);
          S.u[2 * i + 1] = ll_val(w[2 * j + 1]);
        }
      }
    }
    const bool stop = bar_or(NB_CONS, CONS, S.flag[0] != 0);
    fine(0);
    return stop;
  }

  // The next RMSNorm's weights go to shared memory with asynchronous copies
  // issued one phase ahead; norm_q8 waits for them.
  __device__ void prefetch_norm(const float *nw, int k) {
    for (int i = ctid; i < k / 4; i += CONS)
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(S.nw + 4 * i)), "l"(nw + 4 * i) : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
  }

  // Q8 of a k-vector, L lanes per 32-block.  FROM_G: read it from global
  // memory (this launch's data, through L2); otherwise from the staging
  // buffer, optionally as v = (x * scale) * w with w in the norm buffer.
  template <int L, bool FROM_G>
  __device__ void quant_l(const float *src, int k, bool norm, float scale) {
    constexpr int E = 32 / L;
    const int nb = k >> 5, per = CONS / L, l = ctid % L;
    for (int base = 0; base < nb; base += per) {  // the same trip count on every consumer thread
      const int b = base + ctid / L;
      const bool ok = b < nb;
      const int e0 = b * 32 + l * E;  // first element of this lane
      float v[E];
#pragma unroll
      for (int j = 0; j < E / 4; j++) {
        float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (ok) {
          if (FROM_G) {
            x = __ldcg(reinterpret_cast<const float4 *>(src + e0) + j);
          } else {
            x = sld_v4f(u_a + 4u * (uint32_t)(e0 + 4 * j));
            if (norm) {
              const float4 w = sld_v4f(nw_a + 4u * (uint32_t)(e0 + 4 * j));
              x = make_float4(fmul(fmul(x.x, scale), w.x), fmul(fmul(x.y, scale), w.y), fmul(fmul(x.z, scale), w.z),
                              fmul(fmul(x.w, scale), w.w));
            }
          }
        }
        v[4 * j] = x.x;
        v[4 * j + 1] = x.y;
        v[4 * j + 2] = x.z;
        v[4 * j + 3] = x.w;
      }
      q8_lanes<L>(v, ok, l, act_a.q + (uint32_t)e0, act_a, b);
    }
    bar_sync(NB_CONS, CONS);
  }
  // One round where the consumers allow: four lanes per block when every
  // block fits, else two, else one.
  __device__ void quant(const float *src, int k, bool norm, float scale, bool from_g) {
    if ((k >> 5) * 4 <= CONS) {
      if (from_g) quant_l<4, true>(src, k, norm, scale);
      else quant_l<4, false>(src, k, norm, scale);
    } else if ((k >> 5) * 2 <= CONS && !from_g) {
      quant_l<2, false>(src, k, norm, scale);
    } else {
      if (from_g) quant_l<1, true>(src, k, norm, scale);
      else quant_l<1, false>(src, k, norm, scale);
    }
  }

  // RMSNorm (b == 1 order, simd.rs:47-64) + Q8 of the staged vector; the
  // weights were requested with prefetch_norm.
  __device__ void norm_q8(int k) {
    asm volatile("cp.async.wait_all;" ::: "memory");
    float *xv = S.u;
    if (FAST) {  // sum of squares: per-thread partials, warp trees, then the warps' sums in order
      float sq = 0.0f;
      for (int i = ctid; i < k; i += CONS) sq = __fmaf_rn(xv[i], xv[i], sq);
      sq = warp_sum_f(sq);
      if (lane == 0) S.red[cwarp] = sq;
      bar_sync(NB_CONS, CONS);
      if (ctid == 0) {
        float s = 0.0f;
        for (int w = 0; w < CONS / 32; w++) s += S.red[w];
        S.red[32] = 1.0f / sqrtf(s / (float)k + a.eps);
      }
      bar_sync(NB_CONS, CONS);
      fine(1);
      quant(nullptr, k, true, S.red[32], false);
      return;
    }
    const int n8 = k / 8 * 8;
    if (ctid < 8) S.red[ctid] = chain_sq(0.0f, u_a + 4 * ctid, 32u, n8 / 8);
    bar_sync(NB_CONS, CONS);
    if (ctid == 0) {
      const float c0 = fadd(S.red[0], S.red[4]), c1 = fadd(S.red[1], S.red[5]), c2 = fadd(S.red[2], S.red[6]),
                  c3 = fadd(S.red[3], S.red[7]);
      float s = fadd(fadd(c0, c1), fadd(c2, c3));
      for (int i = n8; i < k; i++) s = fadd(s, fmul(xv[i], xv[i]));
      S.red[32] = fdiv(1.0f, __fsqrt_rn(fadd(fdiv(s, (float)k), a.eps)));
    }
    bar_sync(NB_CONS, CONS);
    fine(1);
    quant(nullptr, k, true, S.red[32], false);
  }

  // The terms of one staged chunk: one item per (row, block or superblock),
  // rows fastest, so the lanes of a warp share activation blocks and read
  // the weights of different rows (staged row pitches are odd multiples of
  // 16 bytes: conflict-free 16-byte loads).
  template <int T>
  __device__ void terms(const DChunk &c, uint32_t sl, uint32_t Tb, int gt, int ng) {  // thread gt of a group of ng
    // items per row: exact order, one per block or superblock (Q6_K: half
    // superblocks, j = 2 superblock + half), TPI terms each; fast order, one
    // partial per superblock (Q6_K: half), or per FQ blocks (Q8_0, Q4_0)
    constexpr int TPI = FAST ? 1 : (T == T_Q4_K ? 8 : (T == T_Q6_K ? 8 : 1));
    constexpr int IPB = T == T_Q6_K ? 2 : 1;
    constexpr int BPI = (FAST && (T == T_Q8_0 || T == T_Q4_0)) ? FQ : 1;  // blocks per item
    constexpr int QB = T == T_Q4_K ? 144 : (T == T_Q6_K ? 208 : (T == T_Q8_0 ? 32 : 16));
    const int R = c.rows, nblk = c.b1 - c.b0, ipr = FAST ? dk_items_fast(T, nblk) : nblk * IPB, items = R * ipr;
    const int rs = FAST ? dk_pitch(ipr) : c.rs;
    const uint32_t pitch = c.full ? c.q_stride : c.q_len + 16u * c.qpad;
    const uintptr_t d0 = (uintptr_t)c.d;
    const int dr = ng % R, dj = ng / R;
    int t = gt, r = t % R, j = t / R;
    for (; t < items; t += ng) {
      const int jb = BPI > 1 ? j * BPI : j / IPB;  // first block or superblock of the item within the staged row
      const uint32_t w_a = sl + (uint32_t)r * pitch + (uint32_t)(jb * QB);
      const uint32_t t_a = Tb + 4u * (uint32_t)(r * rs + j * TPI);  // [row][term], rs: the row pitch
      uint32_t d_a = 0u;
      if (T != T_Q4_K)
        d_a = sl + c.d_off + 2u * (uint32_t)jb +
              (uint32_t)(c.full ? (d0 & 15) + (size_t)r * c.d_stride
                                : (size_t)r * c.d_len + ((d0 + (size_t)r * c.d_stride) & 15));
      const int blk = c.b0 + jb;
      if (FAST) {
        if (T == T_Q4_K) item_q4k_f(w_a, blk, act_a, t_a);
        else if (T == T_Q6_K) item_q6k_f(w_a, d_a, blk, j & 1, act_a, t_a);
        else if (T == T_Q8_0) item_q80_f(w_a, d_a, blk, min(BPI, nblk - jb), act_a, t_a);
        else item_q40_f(w_a, d_a, blk, min(BPI, nblk - jb), act_a, t_a);
      } else {
        if (T == T_Q4_K) item_q4k(w_a, blk, act_a, t_a);
        else if (T == T_Q6_K) item_q6k(w_a, d_a, blk, j & 1, act_a, t_a);
        else if (T == T_Q8_0) item_q80(w_a, d_a, blk, act_a, t_a);
        else item_q40(w_a, d_a, blk, act_a, t_a);
      }
      r += dr;
      j += dj;
      if (r >= R) {
        r -= R;
        j++;
      }
    }
  }

  struct ChainInfo {
    int row0, rows, role, layer, flags, nt, rs;
  };

  __device__ void epilogue(const ChainInfo &c) {
    const float val = fadd(0.0f, acc);  // Pool::matmul: out zero-filled, then out += acc
    const int r = c.row0 + lane;
    const bool live = lane < c.rows;
    switch (c.role) {
      case DR_Q:
      case DR_K: {  // model.rs:953-979
        const float partner = __shfl_xor_sync(0xffffffffu, val, 1);
        const int hd = r / a.dh, d = r - hd * a.dh;
        float o = val;
        if (d < 2 * a.half) {
          const int i = d >> 1;
          const float cs = S.rope[i], sn = S.rope[128 + i];
          o = (d & 1) == 0 ? fsub(fmul(val, cs), fmul(partner, sn)) : fadd(fmul(partner, sn), fmul(val, cs));
        }
        if (live) {
          if (c.role == DR_Q) {
            st_ll(a.q_ll + r, o, tag_of(5 * c.layer));
          } else {
            a.kcache[(((size_t)c.layer * a.n_kv + hd) * a.dh + d) * a.n_ctx + pos] = o;  // K is d-major
            st_ll(a.kv_ll + r, o, tag_of(5 * c.layer));
          }
        }
        break;
      }
      case DR_V:
        if (live) {
          const int hd = r / a.dh, d = r - hd * a.dh;
          a.vcache[(((size_t)c.layer * a.n_kv + hd) * a.n_ctx + pos) * a.dh + d] = val;
          st_ll(a.kv_ll + (size_t)a.n_kv * a.dh + r, val, tag_of(5 * c.layer));
        }
        break;
      case DR_O:
      case DR_DOWN:
        if (live) {
          float *xr = S.xo + (r - own0);
          const float nx = fadd(*xr, val);
          *xr = nx;
          if (c.role == DR_O) st_ll(a.x_ll + r, nx, tag_of(5 * c.layer + 2));
          else st_ll(a.x_ll + a.n_embd + r, nx, tag_of(5 * c.layer + 4));
        }
        break;
      case DR_GATE:
        gval = val;
        break;
      case DR_UP:  // model.rs:1111-1115
        if (live) st_ll(a.h_ll + r, fmul(fdiv(gval, fadd(1.0f, expf_lib(-gval))), val), tag_of(5 * c.layer + 3));
        break;
      case DR_HEAD: {
        if (live) a.logits[r] = val;
        float v = (live && !isnan(val)) ? val : -INFINITY;
        int i = live ? r : INT_MAX;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, v, o);
          const int oi = __shfl_xor_sync(0xffffffffu, i, o);
          if (ov > v || (ov == v && oi < i)) {
            v = ov;
            i = oi;
          }
        }
        if (v > best_v) {  // row groups ascend: a strict > keeps the first maximum
          best_v = v;
          best_i = i;
        }
        break;
      }
    }
  }

  // The matvec chunks of phase p.
  // Chain warp that sums chunk ci of this CTA (plan bit list in shared memory).
  __device__ __forceinline__ int owner(int ci) const {
    const int bi = cw_base + ci;
    return (int)((S.cwb[bi >> 5] >> (bi & 31)) & 1u);
  }

  // Barrier protocol per term buffer b and chain warp w: FULLT(b, w) and
  // EMPTYT(b, w) are used by one chunk at a time (chunk mv uses buffer
  // mv % DK_NB, and its group waits for the release of chunk mv - DK_NB before
  // it writes), and each use has exactly the chunk's group and its chain warp,
  // nb_pair(mv) threads.
  __device__ void run_mv(int p) {
    const int wid = tid >> 5, cw = chain_of_warp(wid);
    const bool chain = cw >= 0, term = term_warp(wid);
    const int ti = term ? 32 * term_rank(wid) + lane : 0;  // term thread index
    const int grp = ti < TG0 ? 0 : 1, gt = grp ? ti - TG0 : ti;
    for (int ci = ph[p]; ci < ph[p + 1]; ci++) {
      const int buf = mv % DK_NB;
      const uint32_t Tb = u_a + 4u * (uint32_t)(buf * DK_TS);
      if (term && (mv & 1) == grp) {
        const bool tp = (TRACE && a.trace) && ctid == 32 * DK_CHAINS;
        long long c0 = tp ? clock64() : 0;
        if (mv >= DK_NB) bar_sync(NB_EMPTYT + buf * DK_CHAINS + owner(ci - DK_NB), nb_pair(mv));
        if (tp) pacc(2, clock64() - c0);
        wait_full();
        if (tp) c0 = clock64();
        const DChunk c = load_desc(desc_a + rg.slot * (uint32_t)sizeof(DChunk));
        const uint32_t sl = ring_a + rg.slot * (uint32_t)DK_SLOT;
        const int ng = grp ? TG1 : TG0;
        switch (c.type) {
          case T_Q4_K: terms<T_Q4_K>(c, sl, Tb, gt, ng); break;
          case T_Q6_K: terms<T_Q6_K>(c, sl, Tb, gt, ng); break;
          case T_Q8_0: terms<T_Q8_0>(c, sl, Tb, gt, ng); break;
          default: terms<T_Q4_0>(c, sl, Tb, gt, ng); break;
        }
        if (tp) pacc(3, clock64() - c0);
        bar_arrive(NB_FULLT + buf * DK_CHAINS + owner(ci), nb_pair(mv));
      } else if (chain) {
        // Ownership comes from the plan's bit list (the descriptor may only be
        // read by the owner, before it hands the slot back).
        const bool tp = (TRACE && a.trace) && ctid == 0;
        if (owner(ci) == cw) {
          long long c0 = tp ? clock64() : 0;
          bar_sync(NB_FULLT + buf * DK_CHAINS + cw, nb_pair(mv));
          if (ci == ph[p]) fine(3);  // first chunk's terms are in
          if (tp) {
            const long long c1 = clock64();
            pacc(4, c1 - c0);
            c0 = c1;
          }
          const DChunk d0 = load_desc(desc_a + rg.slot * (uint32_t)sizeof(DChunk));
          ChainInfo c;
          c.row0 = d0.row0;
          c.rows = d0.rows;
          c.role = d0.role;
          c.layer = d0.layer;
          c.flags = d0.flags;
          if (FAST) {
            c.nt = dk_items_fast(d0.type, d0.b1 - d0.b0);
            c.rs = dk_pitch(c.nt);
          } else {
            c.nt = (d0.b1 - d0.b0) * dk_gpb(d0.type) * dk_tpg(d0.type);
            c.rs = d0.rs;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&S.empty[rg.slot]);  // every term warp is done with the slot
          if (c.flags & DF_FIRST) acc = 0.0f;
          const long long ca = tp ? clock64() : 0;
          if (lane < c.rows) acc = chain_add_v(acc, Tb + 16u * (uint32_t)(lane * (c.rs >> 2)), c.nt);
          if (tp) {  // profile (lane 0): its chain adds alone, and how many terms they covered
            pacc(6, clock64() - ca);
            pacc(7, c.nt);
          }
          __syncwarp();
          // the term buffer is free again, for chunk mv + DK_NB and its group
          if (mv + DK_NB < mv_total) bar_arrive(NB_EMPTYT + buf * DK_CHAINS + cw, nb_pair(mv + DK_NB));
          if (c.flags & DF_LAST) epilogue(c);
          if (tp) pacc(5, clock64() - c0);
          if (ci == ph[p]) fine(4);  // first chunk chained
        }
      }
      rg.next();
      mv++;
    }
  }

  // The fast order's softmax sum and weighted values for unit (h, d0): the
  // weights e_p = exp(s_p - M) are in sc[0..pos]; consumer thread (g, d) adds
  // positions p = g (mod G) of dimension d, and the G partials of each
  // dimension and the sum's warp partials are added in a fixed order.
  __device__ void attention_fast(int u, int h, int d0, int pos, int L) {
    const int ds = a.att_ds, ppv = DK_SLOT / (ds * 4), G = CONS / ds;
    const int g = ctid / ds, d = ctid - g * ds;
    const float *sc = S.u;
    float es = 0.0f;
    for (int p = ctid; p <= pos; p += CONS) es += sc[p];
    es = warp_sum_f(es);
    if (lane == 0) S.red[cwarp] = es;
    float vacc = 0.0f;
    for (int p0 = 0; p0 < pos; p0 += ppv) {
      const int n = min(ppv, pos - p0);
      wait_full();
      const float *vc = reinterpret_cast<const float *>(S.ring + (size_t)rg.slot * DK_SLOT);
      if (g < G)
        for (int p = g; p < n; p += G) vacc = __fmaf_rn(sc[p0 + p], vc[p * ds + d], vacc);
      bar_sync(NB_CONS, CONS);
      if (ctid == 0) mbar_arrive(&S.empty[rg.slot]);
      rg.next();
    }
    if (g == 0) vacc = __fmaf_rn(sc[pos], S.qh[512 + d0 + d], vacc);  // this position's v
    float *part = S.u + ((pos + 4) & ~3);  // past the weights
    if (g < G) part[g * ds + d] = vacc;
    bar_sync(NB_CONS, CONS);
    if (ctid < ds) {
      float v = 0.0f;
      for (int i = 0; i < G; i++) v += part[i * ds + ctid];
      float sum = 0.0f;
      for (int w = 0; w < CONS / 32; w++) sum += S.red[w];
      st_ll(a.att_ll + (size_t)h * a.dh + d0 + ctid, sum > 0.0f ? v / sum : 0.0f, tag_of(5 * L + 1));
    }
    bar_sync(NB_CONS, CONS);
  }

  // Exact single-token attention (model.rs:993-1087) for the units this CTA
  // owns: unit (h, j) scores every position of head h (the same values on
  // each of the head's att_j units) and runs the value chains of dimensions
  // [j ds, (j + 1) ds).
  __device__ void attention(int L) {
    const int dh = a.dh, group = a.n_head / a.n_kv, ppc = DK_SLOT / (dh * 4), ds = a.att_ds, ppv = DK_SLOT / (ds * 4);
    const int J = a.att_j;
    float *sc = S.u;
    for (int u = blockIdx.x; u < a.n_head * J; u += gridDim.x) {
      const int h = u / J, j = u - h * J, d0 = j * ds;
      const int kh = h / group;
      int r0, r1;  // the history positions this unit scores
      att_range(pos, j, J, r0, r1);
      float *kcur = S.qh + 256, *vcur = S.qh + 512;
      const uint32_t tag = tag_of(5 * L + 1);
      unsigned long long *scg = a.sc_ll + (size_t)h * a.n_ctx;
      {  // q and this position's k, v: tagged words of the qkv phase
        const uint32_t tq = tag_of(5 * L);
        const unsigned long long t0 = gtime();
        unsigned it = 0;
        for (int d = ctid; d < dh; d += CONS) {
          const unsigned long long *pq = a.q_ll + (size_t)h * dh + d, *pk = a.kv_ll + (size_t)kh * dh + d,
                                   *pv = a.kv_ll + (size_t)(a.n_kv + kh) * dh + d;
          unsigned long long wq = ld_ll(pq), wk = ld_ll(pk), wv = ld_ll(pv);
          while (!(ll_ok(wq, tq) && ll_ok(wk, tq) && ll_ok(wv, tq)) && poll_ok(t0, ++it)) {
            __nanosleep(POLL_SLEEP_NS);
            if (!ll_ok(wq, tq)) wq = ld_ll(pq);
            if (!ll_ok(wk, tq)) wk = ld_ll(pk);
            if (!ll_ok(wv, tq)) wv = ld_ll(pv);
          }
          S.qh[d] = ll_val(wq);
          kcur[d] = ll_val(wk);
          vcur[d] = ll_val(wv);
        }
      }
      bar_sync(NB_CONS, CONS);
      if (u == (int)blockIdx.x) fine(0);
      float mx = -INFINITY;
      // s_p = f32_dot(q, k_p) * scale: eight unfused chains over d = 8t + l,
      // combined ((c0+c1)+(c2+c3)) + ((c4+c5)+(c6+c7)), then the tail.  One
      // thread per position; k_p[d] sits at kp + d * ks (bytes).
      const uint32_t qh_a = shaddr(S.qh);
      auto score = [&](uint32_t kp, uint32_t ks) -> float {
        const int n8 = dh - (dh & 7);
        float c[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        for (int t = 0; t < n8; t += 8) {
#pragma unroll
          for (int u = 0; u < 8; u++) c[u] = fadd(c[u], fmul(sld_f(qh_a + 4u * (t + u)), sld_f(kp + (uint32_t)(t + u) * ks)));
        }
        float r = fadd(fadd(fadd(c[0], c[1]), fadd(c[2], c[3])), fadd(fadd(c[4], c[5]), fadd(c[6], c[7])));
        for (int t = n8; t < dh; t++) r = fadd(r, fmul(sld_f(qh_a + 4u * t), sld_f(kp + (uint32_t)t * ks)));
        return fmul(r, a.scale);
      };
      // This unit's share of the history: K chunks of [r0, r1), up to KG at a
      // time (one position per consumer thread); each score also goes to the
      // head's score row in global memory for the head's other units.
      constexpr int KG = 3;
      const int nk = (r1 - r0 + ppc - 1) / ppc;
      for (int k0 = 0; k0 < nk; k0 += KG) {
        const int g = min(KG, nk - k0), np = min(g * ppc, r1 - r0 - k0 * ppc);
        for (int jj = 0; jj < g; jj++) wait_full_at(jj);
        for (int pi = ctid; pi < np; pi += CONS) {
          const int jj = pi / ppc, pj = pi - jj * ppc;
          const uint32_t kc = ring_a + rg.slot_at(jj) * (uint32_t)DK_SLOT;  // [dh][ppc] floats
          const float sv = score(kc + 4u * pj, 4u * ppc);
          const int p = r0 + k0 * ppc + pi;
          sc[p] = sv;
          if (J > 1) st_ll(scg + p, sv, tag);
          mx = sv > mx ? sv : mx;
        }
        bar_sync(NB_CONS, CONS);
        if (ctid == 0)
          for (int jj = 0; jj < g; jj++) mbar_arrive(&S.empty[rg.slot_at(jj)]);
        for (int jj = 0; jj < g; jj++) rg.next();
        if (u == (int)blockIdx.x && k0 == 0) fine(1);
      }
      if (ctid == 0) {  // the position written by this step's qkv phase
        const float sv = score(shaddr(kcur), 4u);
        sc[pos] = sv;
        mx = sv > mx ? sv : mx;
      }
      if (J > 1) {  // the head's other units' scores (their tagged words)
        const unsigned long long t0 = gtime();
        unsigned it = 0;
        for (int p = ctid; p < pos; p += CONS) {
          if (p >= r0 && p < r1) continue;
          unsigned long long w = ld_ll(scg + p);
          while (!ll_ok(w, tag) && poll_ok(t0, ++it)) {
            __nanosleep(POLL_SLEEP_NS);
            w = ld_ll(scg + p);
          }
          const float sv = ll_val(w);
          sc[p] = sv;
          mx = sv > mx ? sv : mx;
        }
      }
      if (u == (int)blockIdx.x) {
        fine(2);
        mark(5 * L + 1, 0);
      }
      const bool tp = TRACE && a.trace && u == (int)blockIdx.x;
      long long c0 = (tp && ctid == 0) ? clock64() : 0;
      mx = warp_max(mx);
      if (lane == 0) S.red[cwarp] = mx;
      bar_sync(NB_CONS, CONS);
      if (ctid == 0) {
        float m = -INFINITY;
        for (int w = 0; w < CONS / 32; w++) m = S.red[w] > m ? S.red[w] : m;
        S.red[32] = m;
      }
      bar_sync(NB_CONS, CONS);
      if (u == (int)blockIdx.x) fine(3);
      const float M = S.red[32];
      for (int p = ctid; p <= pos; p += CONS) sc[p] = expf_lib(fsub(sc[p], M));
      bar_sync(NB_CONS, CONS);
      if (u == (int)blockIdx.x) fine(4);
      if (tp && ctid == 0) {  // profile: max + exp
        const long long c1 = clock64();
        pacc(2, c1 - c0);
        c0 = c1;
      }
      if (FAST) {
        attention_fast(u, h, d0, pos, L);
        continue;
      }
      // The softmax sum: one chain over e_0 .. e_pos on the last consumer
      // warp, while the others form each V slot's products in place
      // (e_p != 0 ? e_p * v_p[d] : -0.0, the reference's skipped term being
      // an exact -0.0) and run one value chain per dimension over them.
      constexpr int VT = CONS - 32;  // threads of the value work
      float vacc = 0.0f;
      if (ctid >= VT) {
        if (ctid == VT) {
          const long long s0 = tp ? clock64() : 0;
          const float sum = chain_add(0.0f, u_a, 4u, pos + 1);
          S.red[33] = sum > 0.0f ? fdiv(1.0f, sum) : 0.0f;
          if (tp) pacc(4, clock64() - s0);  // profile: softmax sum chain
        }
        for (int p0 = 0; p0 < pos; p0 += ppv) rg.next();
      } else {
        const int sh = __ffs(ds) - 1;  // ds is a power of two
        for (int p0 = 0; p0 < pos; p0 += ppv) {  // slots of [position][ds] (the unit's dimensions)
          const int n = min(ppv, pos - p0);
          wait_full();
          float *vc = reinterpret_cast<float *>(S.ring + (size_t)rg.slot * DK_SLOT);
          for (int i = ctid; i < (n << sh); i += VT) {
            const float e = sc[p0 + (i >> sh)];
            vc[i] = e != 0.0f ? fmul(e, vc[i]) : -0.0f;
          }
          bar_sync(NB_V, VT);
          if (u == (int)blockIdx.x && p0 == 0) fine(6);
          if (ctid < ds) vacc = chain_add(vacc, shaddr(vc) + 4u * ctid, 4u * ds, n);
          bar_sync(NB_V, VT);
          if (ctid == 0) mbar_arrive(&S.empty[rg.slot]);
          rg.next();
        }
        if (ctid < ds) {
          const float e = sc[pos];
          if (e != 0.0f) vacc = fadd(vacc, fmul(e, vcur[d0 + ctid]));
        }
      }
      if (u == (int)blockIdx.x) fine(5);
      if (tp && ctid == 0) {  // profile: value chains
        const long long c1 = clock64();
        pacc(3, c1 - c0);
        c0 = c1;
      }
      bar_sync(NB_CONS, CONS);
      if (ctid < ds) st_ll(a.att_ll + (size_t)h * dh + d0 + ctid, fmul(vacc, S.red[33]), tag_of(5 * L + 1));
      bar_sync(NB_CONS, CONS);
      if (tp && ctid == 0) pacc(5, clock64() - c0);  // profile: output
    }
  }

  __device__ void finish() {
    const int cw = chain_of_warp(tid >> 5);
    if (cw >= 0 && lane == 0) {  // each chain warp's first maximum over its row groups
      S.red[40 + cw] = best_v;
      reinterpret_cast<volatile int *>(S.red)[48 + cw] = best_i;
    }
    bar_sync(NB_CONS, CONS);
    if (ctid == 0) {  // larger value wins; equal values: the lower row index (first maximum)
      float bv = S.red[40];
      int bi = reinterpret_cast<volatile int *>(S.red)[48];
      for (int w = 1; w < DK_CHAINS; w++) {
        const float v = S.red[40 + w];
        const int i = reinterpret_cast<volatile int *>(S.red)[48 + w];
        if (v > bv || (v == bv && i < bi)) {
          bv = v;
          bi = i;
        }
      }
      a.cand_v[blockIdx.x] = bv;
      a.cand_i[blockIdx.x] = bi;
    }
    bar_sync(NB_CONS, CONS);
    if (ctid == 0) {
      mark(5 * a.n_layer, 1);
      __threadfence();
      const unsigned prev = atomicAdd(a.sync + 1, 1u);
      if (prev == gridDim.x - 1) {  // the last CTA: greedy pick over the per-CTA candidates
        __threadfence();
        float bv = -INFINITY;
        int bi = INT_MAX;
        for (int c = 0; c < (int)gridDim.x; c++) {  // CTA row ranges ascend: strict > keeps the first maximum
          const float v = __ldcg(a.cand_v + c);
          if (v > bv) {
            bv = v;
            bi = __ldcg(a.cand_i + c);
          }
        }
        const uint32_t t = bi == INT_MAX ? 0u : (uint32_t)bi;  // nothing above -inf: index 0
        *a.tok = t;
        if (a.mode == 1) {  // feed the token back: the next launch decodes it at pos + 1
          a.ids[0] = t;
          a.hist[*a.step] = t;
          *a.step += 1;
          *a.pos += 1;
        }
        a.sync[1] = 0u;
        a.sync[2] = epoch + 1u > (1u << 22) - 1u ? 1u : epoch + 1u;  // every CTA read the epoch at its start
        __threadfence();
      }
    }
  }

  // One loop over the phases so that every large step has a single call site
  // (the kernel's code stays small enough for the instruction caches).
  //   q = 5L + 0 qkv | 1 attention | 2 o | 3 gate+up | 4 down;  q = 5n: head
  __device__ void run() {
    if ((TRACE && a.trace) && ctid == 0) stamp(0, gtime());
    prefetch_norm(a.layers[0].attn_norm, a.n_embd);
    embed();
    const int qdim = a.n_head * a.dh, nq = 5 * a.n_layer;
    for (int q = 0; q <= nq; q++) {
      const int L = q / 5, kind = q == nq ? 5 : q % 5;
      if (kind == 1) {
        attention(L);
      } else {
        // prologue: stage the input vector, then RMSNorm + Q8 or Q8 alone
        if (kind == 2) prefetch_norm(a.layers[L].ffn_norm, a.n_embd);  // the qkv norm is done with the buffer
        if (kind == 4) prefetch_norm(L + 1 < a.n_layer ? a.layers[L + 1].attn_norm : a.out_norm, a.n_embd);
        const bool norm = kind == 0 || kind == 3 || kind == 5;
        // the previous phase's output: residual after down (qkv, head), attention
        // output (o), residual after o (gate+up), SwiGLU output (down)
        const unsigned long long *src = kind == 2 ? a.att_ll : kind == 4 ? a.h_ll : kind == 3 ? a.x_ll : a.x_ll + a.n_embd;
        const int k = kind == 2 ? qdim : kind == 4 ? a.n_ff : a.n_embd;
        // the test hook's phase waits for a tag no launch writes (epoch 0)
        const uint32_t want = a.poison == q ? 0x3FFu : tag_of(q - 1);
        if (q > 0 && stage_ll(src, k, want)) return;  // layer 0's input was staged by embed()
        if (norm) norm_q8(k);
        else quant(nullptr, k, false, 1.0f, false);
        mark(q, 0);
        run_mv(kind == 5 ? 4 * a.n_layer : 4 * L + (kind == 0 ? 0 : kind - 1));
      }
      if (kind == 5) break;
      if (phase_end()) return;
    }
    finish();
  }
};

template <bool TRACE, bool FAST>
__global__ void __launch_bounds__(DK_THREADS, 1) k_decode(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const Layout L = dk_layout(a.n_embd, a.n_ff, a.n_head * a.dh, a.n_ctx, a.n_layer);
  const Smem S = carve(smem_raw, L);
  if (threadIdx.x == 0) {
    for (int i = 0; i < DK_NS; i++) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.empty[i], 1);
    }
    for (int i = 0; i < 4; i++) S.flag[i] = 0;
    for (int i = 0; i < 8; i++) S.prof[i] = 0ull;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int pos = *a.pos;
  const DChunk *ch = a.chunks + a.cta_chunk0[blockIdx.x];
  const int *ph_g = a.phase0 + (size_t)blockIdx.x * (a.n_phase + 1);
  for (int i = threadIdx.x; i <= a.n_phase; i += DK_THREADS) S.ph[i] = ph_g[i];
  {
    const int c0 = a.cta_chunk0[blockIdx.x], c1 = a.cta_chunk0[blockIdx.x + 1];
    const int w0 = c0 >> 5, nw = ((c1 + 31) >> 5) - w0;
    for (int i = threadIdx.x; i < nw && i < DK_CWW; i += DK_THREADS) S.cwb[i] = a.cwbits[w0 + i];
  }
  for (int i = threadIdx.x; i < a.half; i += DK_THREADS) {
    S.rope[i] = a.rope_cos[(size_t)pos * a.half + i];
    S.rope[128 + i] = a.rope_sin[(size_t)pos * a.half + i];
  }
  __syncthreads();
  const int *ph = S.ph;
  if (TRACE && a.trace && threadIdx.x == 32) {  // SM cycles and ns at the start (clock check)
    a.trace[(size_t)blockIdx.x * a.n_trace + a.n_trace - 4] = (unsigned long long)clock64();
    a.trace[(size_t)blockIdx.x * a.n_trace + a.n_trace - 3] = gtime();
  }
  if (threadIdx.x < 32) {
    producer<TRACE>(a, S, pos, ch, ph);
    return;
  }
  Cons<TRACE, FAST> c(a, S, ch, ph, pos);
  c.run();
  if (TRACE && a.trace && threadIdx.x == 32) {  // and at the end
    a.trace[(size_t)blockIdx.x * a.n_trace + a.n_trace - 2] = (unsigned long long)clock64();
    a.trace[(size_t)blockIdx.x * a.n_trace + a.n_trace - 1] = gtime();
  }
}

}  // namespace

size_t decode_smem_bytes(int n_embd, int n_ff, int qdim, int n_ctx, int dh, int n_layer) {
  if (dh <= 0 || dh > 256 || dh % 4 != 0 || DK_SLOT / (dh * 4) < 1) return 0;
  const Layout L = dk_layout(n_embd, n_ff, qdim, n_ctx, n_layer);
  return L.total <= 227 * 1024 ? L.total : 0;
}

int decode_grid_for(const std::vector<DecLayer> &layers, const DevTensor &out, int sms) {
  long units = sms;
  auto lim = [&](int rows) { units = std::min<long>(units, rows / 2); };  // whole row pairs per CTA
  for (const DecLayer &L : layers) {
    lim(L.q.rows); lim(L.k.rows); lim(L.v.rows); lim(L.o.rows); lim(L.gate.rows); lim(L.down.rows);
  }
  lim(out.rows);
  return (int)std::max<long>(1, units);
}

int decode_grid() {
  int dev = 0, v = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
  return v > 0 ? v : 148;
}

cudaError_t prepare_decode(size_t smem, int grid) {
  cudaError_t e = cudaFuncSetAttribute(k_decode<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_decode<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_decode<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_decode<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode<false, false>, DK_THREADS, smem);
  if (e != cudaSuccess) return e;
  return per_sm >= 1 && grid <= per_sm * decode_grid() ? cudaSuccess : cudaErrorCooperativeLaunchTooLarge;
}

// The V cache [n_layer * n_kv * n_ctx][dh] f32 as a 2-D tensor map with boxes
// of DK_VB positions x ds dimensions.  The encoder is the driver's, reached
// through the runtime (the library does not link libcuda).
int make_vcache_map(CUtensorMap *map, const float *vcache, int n_layer, int n_kv, int n_ctx, int dh, int ds,
                    std::string &why) {
  using Encode = decltype(&cuTensorMapEncodeTiled);
  static Encode encode = nullptr;
  if (!encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      cudaGetLastError();
      why = "cuTensorMapEncodeTiled is not available";
      return -1;
    }
    encode = reinterpret_cast<Encode>(fn);
  }
  if (((uintptr_t)vcache & 15) || ds <= 0 || ds > 256 || (ds * 4) % 16 || dh % ds || (dh * 4) % 16) {
    why = "V cache does not suit a tensor map";
    return -1;
  }
  const cuuint64_t dims[2] = {(cuuint64_t)dh, (cuuint64_t)n_layer * n_kv * n_ctx};
  const cuuint64_t strides[1] = {(cuuint64_t)dh * 4};
  const cuuint32_t box[2] = {(cuuint32_t)ds, (cuuint32_t)DK_VB};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(vcache), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    why = "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")";
    return -1;
  }
  return 0;
}

cudaError_t launch_decode(const DecodeArgs &a, int grid, size_t smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(DK_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident at once, or the launch fails
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (a.fast) return a.trace ? cudaLaunchKernelEx(&cfg, k_decode<true, true>, a) : cudaLaunchKernelEx(&cfg, k_decode<false, true>, a);
  return a.trace ? cudaLaunchKernelEx(&cfg, k_decode<true, false>, a) : cudaLaunchKernelEx(&cfg, k_decode<false, false>, a);
}


// ------------------------------------------------------------------ host plan
namespace {

struct TypeGeo {
  int be, qb, gpb, tpg;
  bool has_d;
};

TypeGeo type_geo(int t) {
  switch (t) {
    case T_Q4_K: return {256, 144, 4, 2, false};
    case T_Q6_K: return {256, 208, 4, 4, true};
    case T_Q8_0: return {32, 32, 1, 1, true};
    default: return {32, 16, 1, 1, true};
  }
}

size_t up16h(size_t x) { return (x + 15) & ~(size_t)15; }
// Floats between rows of a term buffer: at least nt rounded up to a multiple
// of 8 (the row chains read whole batches of eight), and an odd multiple of 4
// (rows start on distinct 16-byte bank groups: conflict-free 128-bit accesses).
int term_pitch(int nt) {
  const int q = ((nt + 7) / 8) * 2;
  return 4 * (q + 1);
}

// [a, b) of n items split into `parts` near-equal pieces on multiples of 2.
void split2(int n, int parts, int i, int &a, int &b) {
  const long units = (n + 1) / 2;
  a = (int)std::min<long>(n, 2 * (units * i / parts));
  b = (int)std::min<long>(n, 2 * (units * (i + 1) / parts));
}

struct Builder {
  std::vector<DChunk> &out;
  std::string &why;
  long load[DK_CHAINS] = {};  // chain terms given to each chain warp in this phase
  void new_phase() {
    for (long &l : load) l = 0;
  }

  DChunk base(const DevTensor &W, uint8_t role, int layer, int r, int rows, int b0, int b1, bool full) {
    const TypeGeo g = type_geo(W.type);
    const int nblk = W.k / g.be;
    const size_t row_q = (size_t)nblk * g.qb, row_d = g.has_d ? (size_t)nblk * 2 : 0;
    DChunk c{};
    c.type = (uint8_t)W.type;
    c.role = role;
    c.layer = layer;
    c.row0 = r;
    c.rows = (uint16_t)rows;
    c.rs = (uint16_t)term_pitch((b1 - b0) * g.gpb * g.tpg);
    c.b0 = b0;
    c.b1 = b1;
    c.full = full ? 1 : 0;
    c.q = W.q + (size_t)r * row_q + (size_t)b0 * g.qb;
    c.q_stride = (uint32_t)row_q;
    c.d_stride = (uint32_t)row_d;
    if (full) {
      c.q_len = (uint32_t)(rows * row_q);
      c.d_off = c.q_len;
    } else {
      c.q_len = (uint32_t)((size_t)(b1 - b0) * g.qb);
      c.qpad = (uint8_t)(((c.q_len >> 4) & 1u) ? 0 : 1);  // odd pitch / 16: rows land on distinct banks
      c.d_off = (uint32_t)((size_t)rows * (c.q_len + 16u * c.qpad));
    }
    if (g.has_d) {
      c.d = reinterpret_cast<const uint8_t *>(W.d) + (size_t)r * row_d + (size_t)b0 * 2;
      c.d_len = full ? (uint32_t)up16h(((uintptr_t)c.d & 15) + rows * row_d) : (uint32_t)up16h((size_t)(b1 - b0) * 2 + 15);
    }
    return c;
  }

  // Rows [r0, r1) of W (and, when W2 is given, the same rows of W2 right
  // after each row group of W: gate then up).  Rows too long for a slot are
  // split along k; the row chain carries across those chunks.
  struct Mode {
    TypeGeo g;
    int nblk;
    size_t row_q, row_d, terms_row;
    bool full;
    int rg;
  };
  Mode mode(const DevTensor &M, int own) {
    Mode m;
    m.g = type_geo(M.type);
    m.nblk = M.k / m.g.be;
    m.row_q = (size_t)m.nblk * m.g.qb;
    m.row_d = m.g.has_d ? (size_t)m.nblk * 2 : 0;
    m.terms_row = (size_t)m.nblk * m.g.gpb * m.g.tpg;
    int rgf = 0;
    for (int rg = std::min(DK_MAX_RG, own); rg >= 2; rg--)
      if (full_fits(m, rg)) {
        rgf = rg & ~1;
        break;
      }
    m.full = rgf >= 2 && rgf >= std::min(8, own);
    m.rg = m.full ? rgf : std::min(DK_MAX_RG, std::max(2, own)) & ~1;
    return m;
  }
  static bool full_fits(const Mode &m, int rg) {
    const size_t bytes = rg * m.row_q + (m.g.has_d ? up16h(15 + rg * m.row_d) : 0);
    return bytes <= (size_t)DK_SLOT && (size_t)rg * term_pitch((int)m.terms_row) <= (size_t)DK_TS;
  }

  bool rows(const DevTensor &W, const DevTensor *W2, int r0, int r1, uint8_t role, uint8_t role2, int layer) {
    if (r1 <= r0) return true;
    if (!type_is_matvec(W.type) || (W2 && (!type_is_matvec(W2->type) || W2->k != W.k || W2->rows != W.rows))) {
      why = "unsupported matrix pairing";
      return false;
    }
    const int own = r1 - r0;
    Mode md[2] = {mode(W, own), W2 ? mode(*W2, own) : mode(W, own)};
    const int rg_max = std::max(2, std::min(md[0].rg, md[1].rg));
    const int units = (own + 1) / 2, ng = (units + rg_max / 2 - 1) / (rg_max / 2);
    for (int gi = 0; gi < ng; gi++) {
      int a, b;
      split2(own, ng, gi, a, b);
      const int R = b - a;
      if (R <= 0) continue;
      // the chain warp with the least work so far sums this group (and its pair)
      int cw = 0;
      for (int w = 1; w < DK_CHAINS; w++)
        if (load[w] < load[cw]) cw = w;
      load[cw] += (long)md[0].terms_row + (W2 ? (long)md[1].terms_row : 0L);
      for (int w = 0; w < (W2 ? 2 : 1); w++) {
        const DevTensor &M = w ? *W2 : W;
        const Mode &m = md[w];
        const bool full = m.full && full_fits(m, R);
        int nkc = 1;
        if (!full) {
          int nbmax = 0;
          for (int nb = m.nblk; nb >= 1; nb--) {
            const size_t bytes = (size_t)R * (nb * (size_t)m.g.qb + 16 + (m.g.has_d ? up16h((size_t)nb * 2 + 15) : 0));
            if (bytes <= (size_t)DK_SLOT && (size_t)R * term_pitch(nb * m.g.gpb * m.g.tpg) <= (size_t)DK_TS) {
              nbmax = nb;
              break;
            }
          }
          if (nbmax == 0) {
            why = "a block of these rows does not fit a ring slot";
            return false;
          }
          nkc = (m.nblk + nbmax - 1) / nbmax;
        }
        for (int j = 0; j < nkc; j++) {
          const int b0 = full ? 0 : (int)((long)m.nblk * j / nkc), b1 = full ? m.nblk : (int)((long)m.nblk * (j + 1) / nkc);
          DChunk c = base(M, w ? role2 : role, layer, r0 + a, R, b0, b1, full);
          c.flags = (uint8_t)((j == 0 ? DF_FIRST : 0) | (j == nkc - 1 ? DF_LAST : 0));
          c.cw = (uint8_t)cw;
          out.push_back(c);
        }
      }
    }
    return true;
  }
};

}  // namespace

bool build_decode_plan(const std::vector<DecLayer> &layers, const DevTensor &out, int n_embd, int n_ff, int n_head,
                       int n_kv, int dh, int n_ctx, int grid, DecodePlan &plan, std::string &why) {
  plan = DecodePlan{};
  plan.grid = grid;
  plan.smem = decode_smem_bytes(n_embd, n_ff, n_head * dh, n_ctx, dh, (int)layers.size());
  if (!plan.smem) {
    why = "model does not fit the persistent kernel's shared memory";
    return false;
  }
  if (n_embd % 32 || n_ff % 32 || (n_head * dh) % 32 || n_head % n_kv || 2 * ((n_embd / 2 + grid - 1) / grid) > DK_XO ||
      n_ctx % 4 || dh % 16) {  // K chunks copy whole groups of 4 positions; V boxes are 16-dimension multiples
    why = "unsupported dimensions";
    return false;
  }
  // Attention units: the most value-dimension slices (of 16 or more) whose
  // units all have a CTA of their own.
  plan.att_j = 1;
  while (2 * plan.att_j * n_head <= grid && dh % (2 * plan.att_j * 16) == 0) plan.att_j *= 2;
  if (decode_grid_for(layers, out, grid) < grid) {  // the tagged hand-off needs rows of every matrix on every CTA
    why = "more CTAs than row pairs of some matrix";
    return false;
  }
  const int nl = (int)layers.size();
  plan.n_phase = 4 * nl + 1;
  plan.cta_chunk0.assign(grid + 1, 0);
  plan.phase0.assign((size_t)grid * (plan.n_phase + 1), 0);
  plan.own.assign((size_t)grid * 2, 0);
  for (int c = 0; c < grid; c++) {
    plan.cta_chunk0[c] = (int)plan.chunks.size();
    std::vector<DChunk> v;
    Builder B{v, why};
    int *ph = &plan.phase0[(size_t)c * (plan.n_phase + 1)];
    int oa, ob;
    split2(n_embd, grid, c, oa, ob);  // o / down rows, and the rows of x this CTA writes
    plan.own[2 * c] = oa;
    plan.own[2 * c + 1] = ob;
    for (int L = 0; L < nl; L++) {
      const DecLayer &Y = layers[L];
      int a, b;
      ph[4 * L] = (int)v.size();
      B.new_phase();  // v first: its Q6_K rows have the longest chains
      split2(Y.v.rows, grid, c, a, b);
      if (!B.rows(Y.v, nullptr, a, b, DR_V, 0, L)) return false;
      split2(Y.q.rows, grid, c, a, b);
      if (!B.rows(Y.q, nullptr, a, b, DR_Q, 0, L)) return false;
      split2(Y.k.rows, grid, c, a, b);
      if (!B.rows(Y.k, nullptr, a, b, DR_K, 0, L)) return false;
      ph[4 * L + 1] = (int)v.size();
      B.new_phase();
      if (!B.rows(Y.o, nullptr, oa, ob, DR_O, 0, L)) return false;
      ph[4 * L + 2] = (int)v.size();
      B.new_phase();
      split2(Y.gate.rows, grid, c, a, b);
      if (!B.rows(Y.gate, &Y.up, a, b, DR_GATE, DR_UP, L)) return false;
      ph[4 * L + 3] = (int)v.size();
      B.new_phase();
      if (!B.rows(Y.down, nullptr, oa, ob, DR_DOWN, 0, L)) return false;
    }
    ph[4 * nl] = (int)v.size();
    B.new_phase();
    int a, b;
    split2(out.rows, grid, c, a, b);
    if (!B.rows(out, nullptr, a, b, DR_HEAD, 0, nl)) return false;
    ph[4 * nl + 1] = (int)v.size();
    plan.chunks.insert(plan.chunks.end(), v.begin(), v.end());
  }
  plan.cta_chunk0[grid] = (int)plan.chunks.size();
  plan.cwbits.assign((plan.chunks.size() + 31) / 32 + 1, 0u);
  for (size_t i = 0; i < plan.chunks.size(); i++)
    if (plan.chunks[i].cw) plan.cwbits[i / 32] |= 1u << (i % 32);
  for (int c = 0; c < grid; c++)
    if (plan.cta_chunk0[c + 1] - plan.cta_chunk0[c] > 32 * DK_CWW - 31) {
      why = "too many chunks per CTA for the chain-warp bit list";
      return false;
    }
  return true;
}

}  // namespace pk
