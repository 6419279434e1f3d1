// pk_quant.cuh -- per-block arithmetic of the GGUF k-quant formats, shared by
// the op-level kernels (pk_kernels.cu) and the persistent decode kernel
// (pk_decode.cu).
//
// Reference semantics (Aleinto97/pocket-workbench-android, rust/pocketinfer/src):
//   dequant_row                   quant.rs:102-359
//   int8 k-quant row dots         quant_int.rs:282-419 (lanes::*)
#pragma once
#include "pk_device.cuh"
#include "pk_kernels.h"

namespace pk {

__device__ __forceinline__ uint16_t ld16u(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

// One element of quant.rs:102-359 dequant_row, same expression per element.
__device__ __forceinline__ float dequant_elem(int t, const uint8_t *row, int j) {
  switch (t) {
    case T_F32: {
      uint32_t b = (uint32_t)row[4 * j] | ((uint32_t)row[4 * j + 1] << 8) | ((uint32_t)row[4 * j + 2] << 16) |
                   ((uint32_t)row[4 * j + 3] << 24);
      return __uint_as_float(b);
    }
    case T_F16: return f16f(ld16u(row + 2 * j));
    case T_BF16: return __uint_as_float((uint32_t)ld16u(row + 2 * j) << 16);
    case T_Q4_0: {
      const uint8_t *b = row + (j / 32) * 18;
      int jj = j % 32;
      uint8_t v = b[2 + (jj & 15)];
      int nib = jj < 16 ? (v & 0xF) : (v >> 4);
      return fmul(fsub((float)nib, 8.0f), f16f(ld16u(b)));
    }
    case T_Q4_1: {
      const uint8_t *b = row + (j / 32) * 20;
      int jj = j % 32;
      uint8_t v = b[4 + (jj & 15)];
      int nib = jj < 16 ? (v & 0xF) : (v >> 4);
      return fadd(fmul((float)nib, f16f(ld16u(b))), f16f(ld16u(b + 2)));
    }
    case T_Q5_0: case T_Q5_1: {
      const int bb = t == T_Q5_0 ? 22 : 24, qo = t == T_Q5_0 ? 2 : 4;
      const uint8_t *b = row + (j / 32) * bb;
      int jj = j % 32;
      uint32_t qh = (uint32_t)b[qo] | ((uint32_t)b[qo + 1] << 8) | ((uint32_t)b[qo + 2] << 16) |
                    ((uint32_t)b[qo + 3] << 24);
      uint32_t q;
      if (jj < 16) q = (uint32_t)(b[qo + 4 + jj] & 0xF) | (((qh >> jj) << 4) & 0x10u);
      else q = (uint32_t)(b[qo + 4 + jj - 16] >> 4) | ((qh >> (jj - 16 + 12)) & 0x10u);
      float d = f16f(ld16u(b));
      if (t == T_Q5_0) return fmul(fsub((float)q, 16.0f), d);
      return fadd(fmul((float)q, d), f16f(ld16u(b + 2)));
    }
    case T_Q8_0: {
      const uint8_t *b = row + (j / 32) * 34;
      return fmul((float)(int8_t)b[2 + (j % 32)], f16f(ld16u(b)));
    }
    case T_Q4_K: case T_Q5_K: {
      const int bb = t == T_Q4_K ? 144 : 176;
      const uint8_t *b = row + (j / 256) * bb;
      int jj = j % 256, n64 = jj / 64, w = jj % 64, l = w % 32;
      int is = 2 * n64 + (w >= 32 ? 1 : 0);
      const uint8_t *scales = b + 4;
      int sc, m;
      if (is < 4) { sc = scales[is] & 63; m = scales[is + 4] & 63; }
      else { sc = (scales[is + 4] & 0xF) | ((scales[is - 4] >> 6) << 4); m = (scales[is + 4] >> 4) | ((scales[is] >> 6) << 4); }
      float d = f16f(ld16u(b)), dmin = f16f(ld16u(b + 2));
      int q;
      if (t == T_Q4_K) {
        uint8_t v = b[16 + n64 * 32 + l];
        q = w < 32 ? (v & 0xF) : (v >> 4);
      } else {
        const uint8_t *qh = b + 16, *ql = b + 48;
        uint8_t v = ql[n64 * 32 + l];
        uint8_t u = (uint8_t)((w < 32 ? 1 : 2) << (2 * n64));
        q = (w < 32 ? (v & 0xF) : (v >> 4)) + ((qh[n64 * 32 + l] & u) ? 16 : 0);
      }
      return fsub(fmul(fmul(d, (float)sc), (float)q), fmul(dmin, (float)m));
    }
    case T_Q6_K: {
      const uint8_t *b = row + (j / 256) * 210;
      int jj = j % 256, half = jj / 128, w = jj % 128, quarter = w / 32, l = w % 32, is = l / 16;
      const uint8_t *ql = b + half * 64, *qh = b + 128 + half * 32, *sc = b + 192 + half * 8;
      int lo = (quarter & 1) ? ql[l + 32] : ql[l];
      lo = (quarter & 2) ? (lo >> 4) : (lo & 0xF);
      int q = (lo | (((qh[l] >> (2 * quarter)) & 3) << 4)) - 32;
      float d = f16f(ld16u(b + 208));
      return fmul(fmul(d, (float)(int8_t)sc[is + 2 * quarter]), (float)q);
    }
    case T_Q8_K: {
      const uint8_t *b = row + (j / 256) * 292;
      uint32_t db = (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16) | ((uint32_t)b[3] << 24);
      return fmul((float)(int8_t)b[4 + (j % 256)], __uint_as_float(db));
    }
  }
  return 0.0f;
}


template <int T> struct Geo;
template <> struct Geo<T_Q4_K> { static constexpr int GE = 64, TPG = 2; };
template <> struct Geo<T_Q6_K> { static constexpr int GE = 64, TPG = 4; };
template <> struct Geo<T_Q8_0> { static constexpr int GE = 32, TPG = 1; };
template <> struct Geo<T_Q4_0> { static constexpr int GE = 32, TPG = 1; };

struct ActRef {  // one lane's Q8 activation: q [k], d/s [k/32]
  const int8_t *q;
  const float *d;
  const int32_t *s;
};

__device__ __forceinline__ int lo4(uint32_t w) { return (int)(w & 0x0F0F0F0Fu); }
__device__ __forceinline__ int hi4(uint32_t w) { return (int)((w >> 4) & 0x0F0F0F0Fu); }

// A group of one row's blocks, read from the device layout in global memory
// (load), combined with a Q8 activation (terms -> finish).  gi is the
// group's index within the row.
template <int T> struct GroupW;

template <> struct GroupW<T_Q4_K> {
  uint4 hdr, w0, w1;
  int blk, sb0;
  __device__ __forceinline__ void load(const DevTensor &W, int row, int gi) {
    const int nblk = W.k >> 8;
    blk = gi >> 2;
    const int g = gi & 3;
    sb0 = 2 * g;
    const uint8_t *base = W.q + ((size_t)row * nblk + blk) * 144;
    hdr = ldw16(base);
    w0 = ldw16(base + 16 + g * 32);
    w1 = ldw16(base + 32 + g * 32);
  }
  __device__ __forceinline__ void terms(const ActRef &A, float *t) const {
    const int4 *ap = reinterpret_cast<const int4 *>(A.q + blk * 256 + sb0 * 32);
    const int ai = blk * 8 + sb0;
    finish(ap[0], ap[1], ap[2], ap[3], A.d[ai], A.d[ai + 1], A.s[ai], A.s[ai + 1], t);
  }
  // quant_int.rs:354-365: acc += d*da*s*dot - da*dmin*m*sa per sub-block.
  __device__ __forceinline__ void finish(const int4 a00, const int4 a01, const int4 a10, const int4 a11, float da0,
                                         float da1, int sa0, int sa1, float *t) const {
    // integer sums are exact in any order: two partial chains each
    int d0a = 0, d0b = 0, d1a = 0, d1b = 0;
    d0a = __dp4a(lo4(w0.x), a00.x, d0a); d0b = __dp4a(lo4(w0.y), a00.y, d0b);
    d0a = __dp4a(lo4(w0.z), a00.z, d0a); d0b = __dp4a(lo4(w0.w), a00.w, d0b);
    d0a = __dp4a(lo4(w1.x), a01.x, d0a); d0b = __dp4a(lo4(w1.y), a01.y, d0b);
    d0a = __dp4a(lo4(w1.z), a01.z, d0a); d0b = __dp4a(lo4(w1.w), a01.w, d0b);
    d1a = __dp4a(hi4(w0.x), a10.x, d1a); d1b = __dp4a(hi4(w0.y), a10.y, d1b);
    d1a = __dp4a(hi4(w0.z), a10.z, d1a); d1b = __dp4a(hi4(w0.w), a10.w, d1b);
    d1a = __dp4a(hi4(w1.x), a11.x, d1a); d1b = __dp4a(hi4(w1.y), a11.y, d1b);
    d1a = __dp4a(hi4(w1.z), a11.z, d1a); d1b = __dp4a(hi4(w1.w), a11.w, d1b);
    const int d0 = d0a + d0b, d1 = d1a + d1b;
    const float d = f16f((uint16_t)(hdr.x & 0xFFFFu)), dmin = f16f((uint16_t)(hdr.x >> 16));
    // get_scale_min_k4 (quant.rs:80-86) for sub-blocks sb0 and sb0 + 1; the
    // 12 scale bytes are hdr.y | hdr.z | hdr.w.
    const int sh = (sb0 & 3) * 8;
    int sc0, m0, sc1, m1;
    if (sb0 < 4) {
      sc0 = (int)((hdr.y >> sh) & 63u);
      m0 = (int)((hdr.z >> sh) & 63u);
      sc1 = (int)((hdr.y >> (sh + 8)) & 63u);
      m1 = (int)((hdr.z >> (sh + 8)) & 63u);
    } else {
      sc0 = (int)(((hdr.w >> sh) & 0xFu) | ((hdr.y >> (sh + 2)) & 0x30u));
      m0 = (int)(((hdr.w >> (sh + 4)) & 0xFu) | ((hdr.z >> (sh + 2)) & 0x30u));
      sc1 = (int)(((hdr.w >> (sh + 8)) & 0xFu) | ((hdr.y >> (sh + 10)) & 0x30u));
      m1 = (int)(((hdr.w >> (sh + 12)) & 0xFu) | ((hdr.z >> (sh + 10)) & 0x30u));
    }
    t[0] = fsub(fmul(fmul(fmul(d, da0), (float)sc0), (float)d0), fmul(fmul(fmul(da0, dmin), (float)m0), (float)sa0));
    t[1] = fsub(fmul(fmul(fmul(d, da1), (float)sc1), (float)d1), fmul(fmul(fmul(da1, dmin), (float)m1), (float)sa1));
  }
};

template <> struct GroupW<T_Q6_K> {
  int q[4][4];  // [s][word]: signed 6-bit weights minus 32, 16 per s
  uint4 scv;
  float d;
  int blk, h, g;
  __device__ __forceinline__ void load(const DevTensor &W, int row, int gi) {
    const int nblk = W.k >> 8;
    blk = gi >> 2;
    h = (gi >> 1) & 1;
    g = gi & 1;
    const size_t bidx = (size_t)row * nblk + blk;
    const uint8_t *base = W.q + bidx * 208;
    scv = ldw16(base + 192);
    d = f16f(__ldg(W.d + bidx));
    unpack(ldw16(base + h * 64 + g * 16), ldw16(base + h * 64 + 32 + g * 16), ldw16(base + 128 + h * 32 + g * 16));
  }
  __device__ __forceinline__ void unpack(const uint4 &qa, const uint4 &qb, const uint4 &qh) {
#pragma unroll
    for (int w = 0; w < 4; w++) {  // quant_int.rs:386-394 unpacking, four bytes at a time
      const uint32_t a = word_of(qa, w), b = word_of(qb, w), hh = word_of(qh, w);
      q[0][w] = (int)__vsub4((a & 0x0F0F0F0Fu) | ((hh << 4) & 0x30303030u), 0x20202020u);
      q[1][w] = (int)__vsub4((b & 0x0F0F0F0Fu) | ((hh << 2) & 0x30303030u), 0x20202020u);
      q[2][w] = (int)__vsub4(((a >> 4) & 0x0F0F0F0Fu) | (hh & 0x30303030u), 0x20202020u);
      q[3][w] = (int)__vsub4(((b >> 4) & 0x0F0F0F0Fu) | ((hh >> 2) & 0x30303030u), 0x20202020u);
    }
  }
  __device__ __forceinline__ void terms(const ActRef &A, float *t) const {
    int4 a[4];
    float da[4];
#pragma unroll
    for (int s = 0; s < 4; s++) {
      a[s] = *reinterpret_cast<const int4 *>(A.q + blk * 256 + (4 * h + s) * 32 + g * 16);
      da[s] = A.d[blk * 8 + 4 * h + s];
    }
    finish(a, da, t);
  }
  // quant_int.rs:397-413: acc += d*scale*da*dot per 16-element piece, order (half, g, s).
  __device__ __forceinline__ void finish(const int4 *a, const float *da, float *t) const {
    // scales of this half: bytes h*8 .. h*8+7 of the 16 scale bytes
    const unsigned long long sw = h ? ((unsigned long long)scv.w << 32 | scv.z) : ((unsigned long long)scv.y << 32 | scv.x);
#pragma unroll
    for (int s = 0; s < 4; s++) {
      int pa = 0, pb = 0;
      pa = __dp4a(q[s][0], a[s].x, pa);
      pb = __dp4a(q[s][1], a[s].y, pb);
      pa = __dp4a(q[s][2], a[s].z, pa);
      pb = __dp4a(q[s][3], a[s].w, pb);
      const int dot = pa + pb;
      const float scale = (float)(int8_t)(uint8_t)(sw >> (8 * (g + 2 * s)));
      t[s] = fmul(fmul(fmul(d, scale), da[s]), (float)dot);
    }
  }
};

template <> struct GroupW<T_Q8_0> {
  uint4 w0, w1;
  float d;
  int blk;
  __device__ __forceinline__ void load(const DevTensor &W, int row, int gi) {
    blk = gi;
    const uint8_t *qs = W.q + (size_t)row * W.k + (size_t)gi * 32;
    w0 = ldw16(qs);
    w1 = ldw16(qs + 16);
    d = f16f(__ldg(W.d + (size_t)row * (W.k >> 5) + gi));
  }
  __device__ __forceinline__ void terms(const ActRef &A, float *t) const {
    const int4 *ap = reinterpret_cast<const int4 *>(A.q + blk * 32);
    finish(ap[0], ap[1], A.d[blk], t);
  }
  // quant_int.rs:291-296: acc += d*da*dot.
  __device__ __forceinline__ void finish(const int4 a0, const int4 a1, float da_, float *t) const {
    int da = 0, db = 0;
    da = __dp4a((int)w0.x, a0.x, da); db = __dp4a((int)w0.y, a0.y, db);
    da = __dp4a((int)w0.z, a0.z, da); db = __dp4a((int)w0.w, a0.w, db);
    da = __dp4a((int)w1.x, a1.x, da); db = __dp4a((int)w1.y, a1.y, db);
    da = __dp4a((int)w1.z, a1.z, da); db = __dp4a((int)w1.w, a1.w, db);
    const int dot = da + db;
    t[0] = fmul(fmul(d, da_), (float)dot);
  }
};

template <> struct GroupW<T_Q4_0> {
  uint4 w;
  float d;
  int blk;
  __device__ __forceinline__ void load(const DevTensor &W, int row, int gi) {
    blk = gi;
    w = ldw16(W.q + (size_t)row * (W.k >> 1) + (size_t)gi * 16);
    d = f16f(__ldg(W.d + (size_t)row * (W.k >> 5) + gi));
  }
  __device__ __forceinline__ void terms(const ActRef &A, float *t) const {
    const int4 *ap = reinterpret_cast<const int4 *>(A.q + blk * 32);
    finish(ap[0], ap[1], A.d[blk], A.s[blk], t);
  }
  // quant_int.rs:316-323: acc += d*dq*(dot - 8*sq).
  __device__ __forceinline__ void finish(const int4 a0, const int4 a1, float da_, int sa, float *t) const {
    int da = 0, db = 0;
    da = __dp4a(lo4(w.x), a0.x, da); db = __dp4a(lo4(w.y), a0.y, db);
    da = __dp4a(lo4(w.z), a0.z, da); db = __dp4a(lo4(w.w), a0.w, db);
    da = __dp4a(hi4(w.x), a1.x, da); db = __dp4a(hi4(w.y), a1.y, db);
    da = __dp4a(hi4(w.z), a1.z, da); db = __dp4a(hi4(w.w), a1.w, db);
    const int dot = da + db;
    t[0] = fmul(fmul(d, da_), fsub((float)dot, fmul(8.0f, (float)sa)));
  }
};

}  // namespace pk
