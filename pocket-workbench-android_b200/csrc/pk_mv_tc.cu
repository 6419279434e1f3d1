// pk_mv_tc.cu -- multi-lane k-quant x Q8 matvec on the fifth-generation
// tensor cores (tcgen05, sm_100a): the b > 8 case of Pool::matmul, i.e. the
// 32-token prefill chunk (model.rs:242-321 over lanes::*, quant_int.rs:282-419).
//
// The reference adds one float term per (row, lane, sub-block) to the row's
// running sum, sub-block after sub-block.  Each sub-block's integer dot
// therefore has to come out of the tensor core on its own: every
// 32-element block (Q4_K sub-block, Q8_0 / Q4_0 block; for Q6_K each
// 16-element piece) is one tcgen05.mma kind::i8 of M = 128 rows x N = 8
// lanes x K = 32, written (not accumulated) into its own 8 TMEM columns.
// The epilogue threads read the int32 dots back with tcgen05.ld and form the
// reference's terms, operand for operand, adding them in the reference's
// order.  Integer dots are exact in any order, so the results are the
// reference's bits.
//
// Work item = 128 rows x 8 lanes.  One persistent CTA per SM takes items
// blockIdx.x, blockIdx.x + grid, ...; 288 threads:
//   warps 0-7  compute: thread = row 32 (w & 3) + lane (TMEM lane quarter
//              w & 3) and lanes 4 (w >> 2) .. + 3 of the item.  They unpack
//              the staged weight bytes into int8 operand tiles (canonical
//              K-major, no swizzle), write the activation operands, issue
//              the MMAs (thread 0), and run the float epilogue of the
//              previous stage while the tensor core works on the current
//              one (TMEM holds two stages);
//   warp 8     producer: bulk copies (cp.async.bulk, mbarrier complete_tx)
//              of each stage's weight rows into a ring of up to eight slots,
//              running ahead across the CTA's items.
// A stage is 256 elements of k: a Q4_K / Q6_K superblock, or eight Q8_0 /
// Q4_0 blocks (fewer in a row's last stage).  Q6_K pieces use the whole
// 32-element weight block with an activation operand whose other 16-byte
// half is a zero core matrix (the B descriptor's leading offset points at
// it), so a piece's dot is exact without splitting the weights.
//
// Every wait is bounded; one that runs out records PK_ERR_TIMEOUT in the
// kernel's error word, and every path frees the CTA's TMEM and waits for its
// own copies in flight before it returns.  No load uses cluster multicast.
#include <cuda.h>  // CUtensorMap (the encoder is reached through cudaGetDriverEntryPoint)
#include <stdint.h>

#include <algorithm>

#include "pk.h"
#include "pk_device.cuh"
#include "pk_kernels.h"

namespace pk {
namespace {

constexpr int TC_ROWS = 128;                 // MMA M
constexpr int TC_NT = 8;                     // lanes per work item (MMA N)
constexpr int TC_CW = 8;                     // compute warps: two per TMEM lane quarter
constexpr int TC_CT = 32 * TC_CW;            // compute threads
constexpr int TC_THREADS = TC_CT + 32;       // + the producer warp
constexpr int TC_SMAX = 8;                   // weight ring slots, at most
constexpr int TC_MPS = 16;                   // MMAs per stage, at most (Q6_K: 8 blocks x 2 pieces)
constexpr int TC_TMEM_COLS = 2 * TC_MPS * TC_NT;  // two stages of D: 256 columns
constexpr int TC_ATILE = TC_ROWS * 32;       // bytes of one A operand (128 rows x 32 int8)
constexpr int TC_BTILE = TC_NT * 32;         // bytes of one B operand (8 lanes x 32 int8)
constexpr unsigned long long TC_WAIT_NS = 2000000000ull;
constexpr uint32_t TC_SMEM = 227 * 1024;     // one CTA an SM

// Instruction descriptor (kind::i8): D s32, A s8, B s8, both K-major,
// N = 8, M = 128.
constexpr uint32_t TC_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_NT >> 3) << 17) |
                              ((uint32_t)(TC_ROWS >> 4) << 24);

// Weight geometry of one type: bytes of a block, and 16-byte chunks of a
// row in one stage (a Q4_K / Q6_K superblock, eight Q8_0 / Q4_0 blocks).
// A stage lands in shared memory as [chunk][128 rows][16 bytes]: the rows
// of one chunk are contiguous, so a warp's 32 rows read 512 contiguous
// bytes, and for Q8_0 chunks 2j, 2j + 1 are already block j's A operand in
// the canonical K-major layout.
template <int T> struct TcGeo;
template <> struct TcGeo<T_Q4_K> { static constexpr int QB = 144, NCH = 9; };
template <> struct TcGeo<T_Q6_K> { static constexpr int QB = 208, NCH = 13; };
template <> struct TcGeo<T_Q8_0> { static constexpr int QB = 32, NCH = 16; };
template <> struct TcGeo<T_Q4_0> { static constexpr int QB = 16, NCH = 8; };
__host__ __device__ constexpr int tc_nch(int t) {
  return t == T_Q4_K ? TcGeo<T_Q4_K>::NCH : t == T_Q6_K ? TcGeo<T_Q6_K>::NCH : t == T_Q8_0 ? TcGeo<T_Q8_0>::NCH
                                                                                         : TcGeo<T_Q4_0>::NCH;
}
constexpr int TC_CHUNK = TC_ROWS * 16;  // bytes of one chunk of a stage

// Shared memory: [zero core matrix Z0][B operands x 2][zero core matrix Z1]
// [A operands][epilogue data x 3][weight ring: nst slots][barriers].
struct TcLayout {
  uint32_t z0, b[2], z1, a, epi[3], ring, bar, total;
  int nst, nch;
};
// Epilogue data of a stage: per row 16 bytes of scales / header and 8 f16
// row scales (d); per lane and block the activation scale and block sum.
constexpr uint32_t TC_EPI_ROW = 32;
constexpr uint32_t TC_EPI = TC_ROWS * TC_EPI_ROW + 2 * 8 * TC_NT * 4;

// nch: the most chunks a stage of the launch's matrices has; the ring gets
// as many slots as the shared memory holds (at most TC_SMAX).
__host__ __device__ inline TcLayout tc_layout(int nch) {
  TcLayout L{};
  uint32_t o = 0;
  L.z0 = o; o += 128;
  L.b[0] = o; o += 8 * TC_BTILE;
  L.b[1] = o; o += 8 * TC_BTILE;
  L.z1 = o; o += 128;
  L.a = o; o += 8 * TC_ATILE;
  for (int e = 0; e < 3; e++) {  // written by a stage's unpack, read by its epilogue one stage later
    L.epi[e] = o; o += TC_EPI;
  }
  const uint32_t bar_bytes = 8 * (2 * TC_SMAX + 2) + 16;  // full, empty, MMA done x 2, TMEM address, abort
  const uint32_t slot = (uint32_t)(nch * TC_CHUNK);
  o = (o + 1023u) & ~1023u;  // tensor-copy destinations: 1024-byte aligned slots
  int n = (int)((TC_SMEM - o - bar_bytes) / slot);
  L.nst = n < TC_SMAX ? n : TC_SMAX;
  L.nch = nch;
  L.ring = o; o += (uint32_t)L.nst * slot;
  L.bar = o; o += bar_bytes;
  L.total = o;
  return L;
}

__device__ int g_tc_err;  // 0 or PK_ERR_TIMEOUT (a bounded wait ran out in some CTA)

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ unsigned long long gtime_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(b) : "memory");
}
__device__ __forceinline__ void mbar_expect(uint32_t b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(b), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint32_t b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(b), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for phase `parity` of mbarrier b; false on timeout or when
// another thread of the CTA (*abort) or another CTA (the error word) has
// given up.
__device__ __forceinline__ bool mbar_wait(uint32_t b, uint32_t parity, const volatile int *abort) {
  if (mbar_test(b, parity)) return true;
  const unsigned long long t0 = gtime_ns();
  for (;;) {
    if (mbar_test(b, parity)) return true;
    if (abort && (*abort || *(volatile int *)&g_tc_err)) return false;
    if (gtime_ns() - t0 > TC_WAIT_NS) return false;
  }
}
// Tiled 3-D tensor copy global -> this CTA's own shared memory (no
// multicast): the box of `map` at (x, y, z), completion counted on mbarrier
// bar.  x * element size is 0 at every call site.
__device__ __forceinline__ void tma_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ void sts32(uint32_t a, uint32_t x) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(x) : "memory");
}
__device__ __forceinline__ void bar_compute() { asm volatile("bar.sync 1, %0;" ::"n"(TC_CT) : "memory"); }
// Barrier of the compute threads that also ORs a predicate over them: every
// compute thread gets the same answer.
__device__ __forceinline__ bool bar_or_compute(bool v) {
  uint32_t r;
  asm volatile("{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}"
               : "=r"(r)
               : "r"((uint32_t)v), "n"(TC_CT)
               : "memory");
  return r != 0;
}

// tcgen05 ------------------------------------------------------------------
// Shared-memory matrix descriptor, K-major without swizzle: core matrices of
// 8 rows x 16 bytes (128 contiguous bytes); lbo = bytes between the two
// 16-byte halves of K, sbo = bytes between groups of 8 rows.
__device__ __forceinline__ uint64_t tc_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);  // version 1 (sm_100), no swizzle
}
// Issued by the whole of one warp with converged lanes: the descriptors are
// warp-uniform, and the lane that elect.sync picks (lane 0, the same one each
// time) issues the MMA and, later, its commit.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a, uint64_t b) {
  asm volatile(
      "{\n .reg .pred p, e;\n elect.sync _|e, 0xffffffff;\n setp.ne.b32 p, %4, 0;\n"
      " @e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(TC_IDESC), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile(
      "{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n"
      " @e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 4 consecutive 32-bit TMEM columns of this thread's lane.
__device__ __forceinline__ void tc_ld4(uint32_t taddr, int (&v)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(taddr)
               : "memory");
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Exact int -> float for |x| < 2^22 on the integer and FP32 pipes.
__device__ __forceinline__ float dotf(int x) { return fsub(__int_as_float(x + 0x4B400000), 12582912.0f); }

// A segment of rows: one matrix of a launch (q/k/v or gate/up share one).
struct TcSeg {
  DevTensor W;
  float *out;
  long os_row, os_lane;
  int add;
  int item0;  // first work item of this segment
};
constexpr int TC_MAX_SEGS = 3;
struct TcSegs {
  // Segment s's weights as a 3-D byte tensor (16-byte chunk offset, row,
  // chunk) with strides (1, row bytes, 16): a box of (16, 128, chunks of a
  // stage) lands as [chunk][row][16 bytes].
  CUtensorMap map[TC_MAX_SEGS];
  TcSeg s[TC_MAX_SEGS];
  int n, items, groups;  // segments, work items, lane groups of 8
  int nch;               // the shared-memory layout's chunks per stage
};

// Canonical K-major position of (row r, 16-byte half h) in an A operand.
__device__ __forceinline__ uint32_t a_off(int r, int h) { return (uint32_t)(h * (TC_ATILE / 2) + (r >> 3) * 128 + (r & 7) * 16); }

// A work item: rows [r0, r0 + 128) of segment s x lanes [l0, l0 + 8).
// Items of one row tile are consecutive (lane groups fastest), so the CTAs
// that work on a tile at the same time share its weights through L2.
struct TcItem {
  const TcSeg *S;
  const CUtensorMap *map;
  int r0, nr, l0, nl;
};
__device__ __forceinline__ TcItem tc_item(const TcSegs &ss, const Q8Dev &act, int it) {
  const int si = (ss.n > 2 && it >= ss.s[2].item0) ? 2 : (ss.n > 1 && it >= ss.s[1].item0) ? 1 : 0;
  TcItem m;
  m.S = &ss.s[si];
  m.map = &ss.map[si];
  const int local = it - ss.s[si].item0, tile = local / ss.groups, grp = local - tile * ss.groups;
  m.r0 = tile * TC_ROWS;
  m.nr = min(TC_ROWS, m.S->W.rows - m.r0);
  m.l0 = grp * TC_NT;
  m.nl = min(TC_NT, act.b - m.l0);
  return m;
}

// Shared state of one CTA.
struct TcCta {
  uint32_t sb, tmem;
  TcLayout L;
  volatile int *abort;
  __device__ uint32_t full(int slot) const { return sb + L.bar + 8u * slot; }
  __device__ uint32_t empty(int slot) const { return sb + L.bar + 8u * (TC_SMAX + slot); }
  __device__ uint32_t mma(int h) const { return sb + L.bar + 8u * (2 * TC_SMAX + h); }
  __device__ uint32_t slot_addr(int slot) const { return sb + L.ring + (uint32_t)(slot * L.nch * TC_CHUNK); }
};
__device__ __forceinline__ void tc_fail(const TcCta &C) {
  if (!*C.abort) atomicCAS(&g_tc_err, 0, PK_ERR_TIMEOUT);
  *C.abort = 1;
}

template <int T>
__device__ __forceinline__ int tc_nstage(int k) {
  return (T == T_Q4_K || T == T_Q6_K) ? k / 256 : ((k >> 5) + 7) / 8;
}

// Producer (one warp): the weight rows of every stage of item m into the
// ring, stages numbered from g0 across the CTA's items; *armed counts the
// stages whose copies were issued.  False when a wait ran out (the warp then
// stops issuing).
template <int T>
__device__ __forceinline__ bool tc_produce(const TcCta C, const TcItem m, uint32_t g0, uint32_t &armed) {
  using G = TcGeo<T>;
  const int lane = threadIdx.x & 31;
  const int ns = tc_nstage<T>(m.S->W.k);
  for (int i = 0; i < ns; i++) {
    const uint32_t g = g0 + (uint32_t)i;
    const int slot = (int)(g % (uint32_t)C.L.nst);
    if (g >= (uint32_t)C.L.nst) {  // the slot's previous stage has been consumed
      int ok = 1;
      if (lane == 0) ok = mbar_wait(C.empty(slot), ((g / C.L.nst) - 1) & 1, C.abort) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, ok, 0)) {
        if (lane == 0) tc_fail(C);
        return false;
      }
    }
    // one tensor copy: the stage's chunks of the item's 128 rows (rows and
    // chunks past the matrix are filled with zeros and still counted)
    if (lane == 0) {
      mbar_expect(C.full(slot), (uint32_t)(G::NCH * TC_CHUNK));
      tma_3d(C.slot_addr(slot), m.map, 0, m.r0, i * G::NCH, C.full(slot));
    }
    __syncwarp();
    armed = g + 1;
  }
  return true;
}

// Compute warps: every stage of item m (stages g0 .. g0 + ns - 1).  Thread
// = row 32 q + lane (q = warp & 3, the TMEM lane quarter) and lane half th =
// warp >> 2 (lanes 4 th .. 4 th + 3 of the item).  Per stage: wait for the
// weights; unpack them into the A operands (th 0: A operands 0-3, th 1:
// 4-7), the B operands and the epilogue data; thread 0 issues the MMAs;
// then the previous stage's float terms are added while the tensor core
// runs.  False when a wait ran out (every compute thread returns false).
template <int T>
__device__ __forceinline__ bool tc_compute(const TcCta C, const Q8Dev &act, const TcItem m, uint32_t g0) {
  using G = TcGeo<T>;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, q = warp & 3, th = warp >> 2;
  const int r = 32 * q + lane, gr = m.r0 + min(r, m.nr - 1);
  const DevTensor &W = m.S->W;
  const int k = W.k, nb32 = k >> 5, ns = tc_nstage<T>(k);
  const uint32_t sb = C.sb, a_base = sb + C.L.a, z0 = sb + C.L.z0, z1 = sb + C.L.z1;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  auto blocks_of = [&](int i) { return min(8, nb32 - i * 8); };
  // Inputs of the next stage's unpack, loaded one stage ahead: this row's
  // f16 scales (Q6_K: 1, Q8_0 / Q4_0: up to 8), one lane scale or block sum
  // (th 0 threads) or 16 bytes of a lane's activation (th 1 threads).
  uint16_t dpre[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  float spre = 0.0f;
  uint4 bpre = make_uint4(0u, 0u, 0u, 0u);
  auto prefetch = [&](int i) {
    const int nb = blocks_of(i);
    if (th == 0) {
      if (T == T_Q6_K) dpre[0] = __ldg(W.d + (size_t)gr * (k / 256) + i);
      if (T == T_Q8_0 || T == T_Q4_0)
#pragma unroll
        for (int j = 0; j < 8; j++) dpre[j] = j < nb ? __ldg(W.d + (size_t)gr * nb32 + i * 8 + j) : (uint16_t)0;
      // thread t < 128: lane t % 8, block (t / 8) % 8; t < 64 the scale, else the block sum
      const int n = tid & 7, j = (tid >> 3) & 7, gl = m.l0 + min(n, m.nl - 1), bj = i * 8 + min(j, nb - 1);
      spre = tid < 64 ? __ldg(act.d + (size_t)gl * nb32 + bj) : (float)__ldg(act.s + (size_t)gl * nb32 + bj);
    } else {
      // thread 128 + c: piece c = (block j, lane n, half h) of the B operands
      const int c = tid - 128, j = c >> 4, n = (c >> 1) & 7, h = c & 1;
      const int gl = m.l0 + min(n, m.nl - 1), bj = i * 8 + min(j, nb - 1);
      bpre = __ldg(reinterpret_cast<const uint4 *>(act.q + (size_t)gl * k + (size_t)bj * 32 + h * 16));
    }
  };
  // float terms of stage i (global g), added in the reference's order
  auto epilogue = [&](int i, uint32_t g) {
    const int nb = blocks_of(i);
    const uint32_t ep = sb + C.L.epi[g % 3];
    const uint32_t lsc = ep + TC_ROWS * TC_EPI_ROW;  // [da | sa][block][lane] floats
    const uint32_t tbase = C.tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)((g & 1) * TC_MPS * TC_NT + 4 * th);
    const uint4 hdr = sld_v4(ep + (uint32_t)r * TC_EPI_ROW);       // Q4_K header / Q6_K scales
    const uint4 dw = sld_v4(ep + (uint32_t)r * TC_EPI_ROW + 16u);  // f16 row scales
    const uint32_t lo = 16u * th;                                   // this thread's lanes in a block's 32 bytes
    if (T == T_Q4_K) {  // lanes::q4_k (quant_int.rs:354-365): term = (d*da)*sc*dot - (da*dmin)*m*sa
      const float d = f16f((uint16_t)(hdr.x & 0xFFFFu)), dmin = f16f((uint16_t)(hdr.x >> 16));
      int dot[8][4];
#pragma unroll
      for (int j = 0; j < 8; j++) tc_ld4(tbase + (uint32_t)(j * TC_NT), dot[j]);
      tc_wait_ld();
#pragma unroll
      for (int j = 0; j < 8; j++) {
        int sc, mn;
        scale_min_k4(hdr, j, sc, mn);
        const float scf = (float)sc, mf = (float)mn;
        const float4 da = sld_v4f(lsc + 32u * j + lo), sa = sld_v4f(lsc + 256u + 32u * j + lo);
        const float dv[4] = {da.x, da.y, da.z, da.w}, sv[4] = {sa.x, sa.y, sa.z, sa.w};
#pragma unroll
        for (int n = 0; n < 4; n++)
          acc[n] = fadd(acc[n], fsub(fmul(fmul(fmul(d, dv[n]), scf), dotf(dot[j][n])), fmul(fmul(fmul(dv[n], dmin), mf), sv[n])));
      }
    } else if (T == T_Q6_K) {  // lanes::q6_k (quant_int.rs:386-413): ((d*scale)*da)*dot, order (half, piece, block)
      const float d = f16f((uint16_t)(dw.x & 0xFFFFu));
      const uint32_t scw[4] = {hdr.x, hdr.y, hdr.z, hdr.w};
#pragma unroll
      for (int hh = 0; hh < 2; hh++) {
        int dot[8][4];
#pragma unroll
        for (int e = 0; e < 8; e++) tc_ld4(tbase + (uint32_t)((8 * hh + e) * TC_NT), dot[e]);
        tc_wait_ld();
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const int mm = 8 * hh + e, g2 = (mm >> 2) & 1, s4 = mm & 3, blk = 4 * hh + s4, si = 8 * hh + g2 + 2 * s4;
          const float scale = dotf((int)(int8_t)(uint8_t)(scw[si >> 2] >> (8 * (si & 3))));
          const float4 da = sld_v4f(lsc + 32u * blk + lo);
          const float dv[4] = {da.x, da.y, da.z, da.w};
          const float ds = fmul(d, scale);
#pragma unroll
          for (int n = 0; n < 4; n++) acc[n] = fadd(acc[n], fmul(fmul(ds, dv[n]), dotf(dot[e][n])));
        }
      }
    } else {  // Q8_0: (d*da)*dot (quant_int.rs:291-296); Q4_0: (d*da)*(dot - 8*sa) (:316-323)
      const uint32_t dws[4] = {dw.x, dw.y, dw.z, dw.w};
      int dot[8][4];
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (j < nb) tc_ld4(tbase + (uint32_t)(j * TC_NT), dot[j]);
      tc_wait_ld();
#pragma unroll
      for (int j = 0; j < 8; j++) {
        if (j >= nb) break;
        const float d = f16f((uint16_t)(dws[j >> 1] >> (16 * (j & 1))));
        const float4 da = sld_v4f(lsc + 32u * j + lo);
        const float dv[4] = {da.x, da.y, da.z, da.w};
        if (T == T_Q8_0) {
#pragma unroll
          for (int n = 0; n < 4; n++) acc[n] = fadd(acc[n], fmul(fmul(d, dv[n]), dotf(dot[j][n])));
        } else {
          const float4 sa = sld_v4f(lsc + 256u + 32u * j + lo);
          const float sv[4] = {sa.x, sa.y, sa.z, sa.w};
#pragma unroll
          for (int n = 0; n < 4; n++) acc[n] = fadd(acc[n], fmul(fmul(d, dv[n]), fsub(dotf(dot[j][n]), fmul(8.0f, sv[n]))));
        }
      }
    }
    tc_fence_before();  // these TMEM reads are ordered before the next barrier (and the MMAs after it)
  };

  prefetch(0);
  bool stop = false;
  for (int i = 0; i < ns; i++) {
    const uint32_t g = g0 + (uint32_t)i;
    const int slot = (int)(g % (uint32_t)C.L.nst);
    // stage g - 1's MMAs are done (A operands, B buffer and its ring slot
    // free, its dots in TMEM); stage g's weights have landed
    bool ok = true;
    if (i > 0) {
      ok = mbar_wait(C.mma((g - 1) & 1), ((g - 1) >> 1) & 1, C.abort);
      tc_fence_after();
      if (ok && tid == 0) mbar_arrive(C.empty((int)((g - 1) % (uint32_t)C.L.nst)));
    }
    if (ok) ok = mbar_wait(C.full(slot), (g / C.L.nst) & 1, C.abort);
    if (!ok) tc_fail(C);
    if (bar_or_compute(!ok)) {
      stop = true;
      break;
    }
    const int nb = blocks_of(i);
    const uint32_t src = C.slot_addr(slot) + (uint32_t)(r * 16);  // chunk c of this row: src + c * TC_CHUNK
    const uint32_t ep = sb + C.L.epi[g % 3] + (uint32_t)r * TC_EPI_ROW;
    // this row's part of the A operands (int8, canonical K-major)
    if (T == T_Q4_K) {  // sub-block 2p: low nibbles of qs[32p .. 32p+32); 2p+1: high nibbles
      if (th == 0) {
        const uint4 hdr = sld_v4(src);
        sts128(ep, hdr.x, hdr.y, hdr.z, hdr.w);
      }
#pragma unroll
      for (int pp = 0; pp < 2; pp++)
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int p = 2 * th + pp;
          const uint4 w = sld_v4(src + (uint32_t)((1 + 2 * p + h) * TC_CHUNK));  // qs[32p + 16h, +16)
          const uint32_t M = 0x0F0F0F0Fu;
          sts128(a_base + (uint32_t)((2 * p) * TC_ATILE) + a_off(r, h), w.x & M, w.y & M, w.z & M, w.w & M);
          sts128(a_base + (uint32_t)((2 * p + 1) * TC_ATILE) + a_off(r, h), (w.x >> 4) & M, (w.y >> 4) & M,
                 (w.z >> 4) & M, (w.w >> 4) & M);
        }
    } else if (T == T_Q6_K) {  // block 4h + s, 16-byte piece g: quant_int.rs:386-394 unpacking, minus 32
      const int h = th;
      if (th == 0) {
        const uint4 scv = sld_v4(src + 12u * TC_CHUNK);  // the 16 scales (bytes 192..207)
        sts128(ep, scv.x, scv.y, scv.z, scv.w);
        sts32(ep + 16u, (uint32_t)dpre[0]);
      }
#pragma unroll
      for (int gg = 0; gg < 2; gg++) {
        // ql bytes 64h + 16g and 64h + 32 + 16g, qh bytes 128 + 32h + 16g
        const uint4 la = sld_v4(src + (uint32_t)((4 * h + gg) * TC_CHUNK)), lb = sld_v4(src + (uint32_t)((4 * h + 2 + gg) * TC_CHUNK));
        const uint4 qh = sld_v4(src + (uint32_t)((8 + 2 * h + gg) * TC_CHUNK));
#pragma unroll
        for (int s4 = 0; s4 < 4; s4++) {
          uint32_t o[4];
#pragma unroll
          for (int wi = 0; wi < 4; wi++) {
            const uint32_t lw = word_of(s4 & 1 ? lb : la, wi), hw = word_of(qh, wi);
            const uint32_t qv = ((s4 & 2 ? lw >> 4 : lw) & 0x0F0F0F0Fu) |
                                ((s4 == 0 ? hw << 4 : s4 == 1 ? hw << 2 : s4 == 2 ? hw : hw >> 2) & 0x30303030u);
            o[wi] = __vsub4(qv, 0x20202020u);
          }
          sts128(a_base + (uint32_t)((4 * h + s4) * TC_ATILE) + a_off(r, gg), o[0], o[1], o[2], o[3]);
        }
      }
    } else {
      // Q8_0: the staged chunks are already the A operands (no unpack)
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
        const int j = 4 * th + jj;
        if (T == T_Q8_0 || j >= nb) break;
        {  // Q4_0: low nibbles = elements 0-15, high = 16-31
          const uint4 w = sld_v4(src + (uint32_t)(j * TC_CHUNK));
          const uint32_t M = 0x0F0F0F0Fu;
          sts128(a_base + (uint32_t)(j * TC_ATILE) + a_off(r, 0), w.x & M, w.y & M, w.z & M, w.w & M);
          sts128(a_base + (uint32_t)(j * TC_ATILE) + a_off(r, 1), (w.x >> 4) & M, (w.y >> 4) & M, (w.z >> 4) & M,
                 (w.w >> 4) & M);
        }
      }
      if (th == 0)
        sts128(ep + 16u, (uint32_t)dpre[0] | (uint32_t)dpre[1] << 16, (uint32_t)dpre[2] | (uint32_t)dpre[3] << 16,
               (uint32_t)dpre[4] | (uint32_t)dpre[5] << 16, (uint32_t)dpre[6] | (uint32_t)dpre[7] << 16);
    }
    if (th == 0) {  // lane scales and block sums of this stage, [da | sa][block][lane]
      const int n = tid & 7, j = (tid >> 3) & 7;
      sts32(sb + C.L.epi[g % 3] + TC_ROWS * TC_EPI_ROW + (uint32_t)((tid >> 6) * 256 + j * 32 + n * 4),
            __float_as_uint(spre));
    } else {  // B operands: block j, lane n, half h at b + 256 j + 128 h + 16 n
      const int c = tid - 128, j = c >> 4, n = (c >> 1) & 7, h = c & 1;
      sts128(sb + C.L.b[g & 1] + (uint32_t)(j * TC_BTILE + h * 128 + n * 16), bpre.x, bpre.y, bpre.z, bpre.w);
    }
    if (i + 1 < ns) prefetch(i + 1);
    fence_async_smem();  // the operands written above are visible to the tensor core
    bar_compute();
    if (warp == 0) {  // warp-uniform descriptors; one elected lane issues
      tc_fence_after();
      const uint32_t d0 = C.tmem + (uint32_t)((g & 1) * TC_MPS * TC_NT);
      const uint32_t bb = sb + C.L.b[g & 1];
      if (T == T_Q6_K) {
        // piece 0 of block b: B half 0 = the block's first 16 bytes, half 1 = Z1;
        // piece 1: half 0 = Z0, half 1 = the block's last 16 bytes
#pragma unroll
        for (int mm = 0; mm < 16; mm++) {
          const int h = mm >> 3, g2 = (mm >> 2) & 1, s4 = mm & 3, blk = 4 * h + s4;
          const uint64_t ad = tc_desc(a_base + (uint32_t)(blk * TC_ATILE), TC_ATILE / 2, 128);
          const uint32_t bk = bb + (uint32_t)(blk * TC_BTILE);
          const uint64_t bd = g2 == 0 ? tc_desc(bk, z1 - bk, 128) : tc_desc(z0, bk + 128 - z0, 128);
          tc_mma(d0 + (uint32_t)(mm * TC_NT), ad, bd);
        }
      } else {
        for (int j = 0; j < nb; j++) {
          // Q8_0: block j's A operand is chunks 2j, 2j + 1 of the ring slot
          const uint64_t ad = T == T_Q8_0 ? tc_desc(C.slot_addr(slot) + (uint32_t)(2 * j * TC_CHUNK), TC_CHUNK, 128)
                                          : tc_desc(a_base + (uint32_t)(j * TC_ATILE), TC_ATILE / 2, 128);
          const uint64_t bd = tc_desc(bb + (uint32_t)(j * TC_BTILE), 128, 128);
          tc_mma(d0 + (uint32_t)(j * TC_NT), ad, bd);
        }
      }
      tc_commit(C.mma(g & 1));
    }
    if (i > 0) epilogue(i - 1, g - 1);  // the previous stage's float terms, while the tensor core runs this one
  }
  if (!stop) {  // the item's last stage
    const uint32_t g = g0 + (uint32_t)(ns - 1);
    const bool ok = mbar_wait(C.mma(g & 1), (g >> 1) & 1, C.abort);
    tc_fence_after();
    if (ok && tid == 0) mbar_arrive(C.empty((int)(g % (uint32_t)C.L.nst)));
    if (!ok) tc_fail(C);
    stop = bar_or_compute(!ok);
    if (!stop) epilogue(ns - 1, g);
  }
  if (stop) return false;
  // out = 0.0 + acc (Pool::matmul zero-fills, then adds), or x += that
  if (r < m.nr)
#pragma unroll
    for (int n = 0; n < 4; n++)
      if (4 * th + n < m.nl) {
        float *o = m.S->out + (long)(m.r0 + r) * m.S->os_row + (long)(m.l0 + 4 * th + n) * m.S->os_lane;
        const float v = fadd(0.0f, acc[n]);
        *o = m.S->add ? fadd(*o, v) : v;
      }
  return true;
}

// Persistent CTAs (one per SM): CTA c takes work items c, c + grid, ...;
// the producer runs ahead through the same items' stages, the ring's depth
// ahead of the compute warps.
__global__ void __launch_bounds__(TC_THREADS, 1) k_mv_tc(const __grid_constant__ TcSegs ss, Q8Dev act) {
  extern __shared__ __align__(128) uint8_t tc_smem[];
  TcCta C;
  C.sb = smem_u32(tc_smem);
  C.L = tc_layout(ss.nch);
  C.abort = reinterpret_cast<volatile int *>(tc_smem + C.L.bar + 8 * (2 * TC_SMAX + 2) + 4);
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    for (int i = 0; i < C.L.nst; i++) {
      mbar_init(C.full(i), 1);   // the producer's expect_tx
      mbar_init(C.empty(i), 1);  // compute thread 0, once the stage's MMAs are done
    }
    mbar_init(C.mma(0), 1);  // tcgen05.commit
    mbar_init(C.mma(1), 1);
    *C.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // zero core matrices (the Q6_K pieces' other halves)
  if (tid < 16) sts128(C.sb + (tid < 8 ? C.L.z0 : C.L.z1) + 16u * (tid & 7), 0u, 0u, 0u, 0u);
  // the previous kernel's outputs are complete before any read; no TMEM is
  // held while waiting
  pdl_wait();
  const uint32_t taddr_smem = C.sb + C.L.bar + 8 * (2 * TC_SMAX + 2);
  if (warp == 0) {  // TMEM for two stages of D
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(taddr_smem),
                 "r"(TC_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  C.tmem = *reinterpret_cast<volatile uint32_t *>(tc_smem + C.L.bar + 8 * (2 * TC_SMAX + 2));
  pdl_trigger();
  uint32_t g = 0;  // stages this CTA has started (the ring and TMEM positions)
  if (warp == TC_CW) {  // ------------------------------------------ producer
    bool ok = true;
    uint32_t armed = 0;
    for (int it = blockIdx.x; it < ss.items && ok; it += gridDim.x) {
      const TcItem m = tc_item(ss, act, it);
      switch (m.S->W.type) {
        case T_Q4_K: ok = tc_produce<T_Q4_K>(C, m, g, armed); g += (uint32_t)tc_nstage<T_Q4_K>(m.S->W.k); break;
        case T_Q6_K: ok = tc_produce<T_Q6_K>(C, m, g, armed); g += (uint32_t)tc_nstage<T_Q6_K>(m.S->W.k); break;
        case T_Q8_0: ok = tc_produce<T_Q8_0>(C, m, g, armed); g += (uint32_t)tc_nstage<T_Q8_0>(m.S->W.k); break;
        default: ok = tc_produce<T_Q4_0>(C, m, g, armed); g += (uint32_t)tc_nstage<T_Q4_0>(m.S->W.k); break;
      }
    }
    // every copy this warp issued lands before the CTA may exit: the stages
    // armed last (at most one ring's worth can still be in flight)
    if ((tid & 31) == 0) {
      const uint32_t n = armed < (uint32_t)C.L.nst ? armed : (uint32_t)C.L.nst;
      for (uint32_t j = armed - n; j < armed; j++) mbar_wait(C.full((int)(j % (uint32_t)C.L.nst)), (j / C.L.nst) & 1, nullptr);
    }
    __syncwarp();
  } else {  // ------------------------------------------------------ compute
    for (int it = blockIdx.x; it < ss.items; it += gridDim.x) {
      const TcItem m = tc_item(ss, act, it);
      bool ok;
      switch (m.S->W.type) {
        case T_Q4_K: ok = tc_compute<T_Q4_K>(C, act, m, g); g += (uint32_t)tc_nstage<T_Q4_K>(m.S->W.k); break;
        case T_Q6_K: ok = tc_compute<T_Q6_K>(C, act, m, g); g += (uint32_t)tc_nstage<T_Q6_K>(m.S->W.k); break;
        case T_Q8_0: ok = tc_compute<T_Q8_0>(C, act, m, g); g += (uint32_t)tc_nstage<T_Q8_0>(m.S->W.k); break;
        default: ok = tc_compute<T_Q4_0>(C, act, m, g); g += (uint32_t)tc_nstage<T_Q4_0>(m.S->W.k); break;
      }
      if (!ok) break;  // every compute thread stops together (bar_or_compute)
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(C.tmem), "r"(TC_TMEM_COLS) : "memory");
  }
}

}  // namespace

bool mv_tc_supports(const DevTensor &w, const Q8Dev &act) {
  if (!type_is_matvec(w.type) || act.b < 1 || w.k != act.k || w.rows < 1) return false;
  if (w.k % 32) return false;
  if ((w.type == T_Q4_K || w.type == T_Q6_K) && w.k % 256) return false;
  // bulk copies: 16-byte aligned sources (row starts, the lanes' activation rows)
  // tensor map: 16-byte aligned base and row stride; lanes' activation rows 16-byte aligned
  const size_t row_bytes = (size_t)(w.k / ((w.type == T_Q4_K || w.type == T_Q6_K) ? 256 : 32)) *
                           (w.type == T_Q4_K ? 144 : w.type == T_Q6_K ? 208 : w.type == T_Q8_0 ? 32 : 16);
  return ((uintptr_t)w.q & 15) == 0 && row_bytes % 16 == 0 && ((uintptr_t)act.q & 15) == 0;
}

// Segment weights as the kernel's 3-D tensor map (see TcSegs).
static cudaError_t tc_weight_map(CUtensorMap *map, const DevTensor &w) {
  using Encode = decltype(&cuTensorMapEncodeTiled);
  static Encode encode = nullptr;
  if (!encode) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      cudaGetLastError();
      return cudaErrorNotSupported;
    }
    encode = reinterpret_cast<Encode>(fn);
  }
  const int be = (w.type == T_Q4_K || w.type == T_Q6_K) ? 256 : 32;
  const size_t row_bytes = (size_t)(w.k / be) * (w.type == T_Q4_K ? 144 : w.type == T_Q6_K ? 208 : w.type == T_Q8_0 ? 32 : 16);
  const cuuint64_t dims[3] = {16, (cuuint64_t)w.rows, (cuuint64_t)(row_bytes / 16)};
  const cuuint64_t strides[2] = {(cuuint64_t)row_bytes, 16};
  const cuuint32_t box[3] = {16, (cuuint32_t)TC_ROWS, (cuuint32_t)tc_nch(w.type)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(w.q), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_mv_tc(int n, const MvOut *outs, const Q8Dev &act, cudaStream_t st) {
  if (n < 1 || n > TC_MAX_SEGS) return cudaErrorInvalidValue;
  TcSegs ss{};
  ss.n = n;
  ss.groups = (act.b + TC_NT - 1) / TC_NT;
  int items = 0, nch = 0;
  cudaError_t e;
  for (int i = 0; i < n; i++) {
    const MvOut &o = outs[i];
    if (!mv_tc_supports(o.w, act)) return cudaErrorInvalidValue;
    if ((e = tc_weight_map(&ss.map[i], o.w)) != cudaSuccess) return e;
    ss.s[i] = TcSeg{o.w, o.out, o.os_row, o.os_lane, o.add ? 1 : 0, items};
    items += (o.w.rows + TC_ROWS - 1) / TC_ROWS * ss.groups;
    nch = std::max(nch, tc_nch(o.w.type));
  }
  ss.items = items;
  ss.nch = nch;
  const TcLayout L = tc_layout(nch);
  if (L.nst < 2) return cudaErrorInvalidValue;
  static bool attr = false;
  if (!attr) {
    if ((e = cudaFuncSetAttribute(k_mv_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TC_SMEM)) != cudaSuccess)
      return e;
    attr = true;
  }
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(items, sms));
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_mv_tc, ss, act);
}

int mv_tc_error(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tc_err, sizeof(int)) != cudaSuccess) return PK_ERR_CUDA;
  if (clear && v) {
    const int z = 0;
    cudaMemcpyToSymbol(g_tc_err, &z, sizeof(int));
  }
  return v;
}

}  // namespace pk
