// pk_capi.cpp -- extern "C" entry points declared in include/pk.h.
#include <cuda_runtime.h>

#include <cmath>
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <new>
#include <string>
#include <utility>

#include "pk.h"
#include "pk_engine.h"
#include "pk_gguf.h"
#include "pk_text.h"
#include "pk_tp.h"

namespace pk {

static thread_local std::string t_err;

int set_error(int code, const std::string &msg) {
  t_err = msg;
  return code;
}

int cuda_error(cudaError_t e, const char *what) {
  t_err = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  return e == cudaErrorMemoryAllocation ? PK_ERR_OOM : PK_ERR_CUDA;
}

}  // namespace pk

using namespace pk;

#define CK(expr)                                          \
  do {                                                    \
    cudaError_t _e = (expr);                              \
    if (_e != cudaSuccess) return cuda_error(_e, #expr);  \
  } while (0)

namespace {

bool q8_ok(const pk_q8act *a, int k) {
  return a && a->q && a->d && a->sum && a->k == k && a->b >= 1 && a->b <= 64;
}

Q8Dev to_dev(const pk_q8act *a) {
  Q8Dev d;
  d.q = a->q;
  d.d = a->d;
  d.s = a->sum;
  d.k = a->k;
  d.b = a->b;
  return d;
}

int check_matvec_shape(uint32_t ttype, int k, int n_rows) {
  if (!type_is_matvec((int)ttype))
    return set_error(PK_ERR_UNSUPPORTED, "type " + std::to_string(ttype) + " not supported on the device");
  int be = 0, bb = 0;
  type_block((int)ttype, &be, &bb);
  if (k <= 0 || n_rows <= 0 || k % be != 0 || k % 32 != 0)
    return set_error(PK_ERR_INVALID, "k must be a positive multiple of the block size and of 32");
  return PK_OK;
}

int matmul_packed(uint32_t ttype, const void *packed, int k, int n_rows, const pk_q8act *act, float *out,
                  cudaStream_t st) {
  const DevTensor w = packed_view((int)ttype, k, n_rows, packed);
  const Q8Dev a = to_dev(act);
  if (a.b == 1) {
    B1Src src;
    src.act = a;
    CK(launch_mv_b1(w, src, out, false, st));
  } else {
    CK(launch_mv_lanes(w, a, out, a.b, 1, false, st));
  }
  return PK_OK;
}

// ---- host f32 dot for the backend self-test (quant.rs:260-287, 323-347, 377-441)
float h_f16(uint16_t h) {
  const uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
  float v;
  if (exp == 0) v = std::ldexp((float)mant, -24);
  else if (exp == 31) v = mant ? NAN : INFINITY;
  else v = std::ldexp((float)(mant | 0x400u), (int)exp - 25);
  return sign ? -v : v;
}

float host_dot_f32(uint32_t t, const uint8_t *w, int k, const float *x) {
  float sum = 0.0f;
  for (int blk = 0; blk < k / 256; blk++) {
    if (t == PK_TYPE_Q4_K) {
      const uint8_t *b = w + blk * 144;
      const float d = h_f16((uint16_t)(b[0] | (b[1] << 8))), dmin = h_f16((uint16_t)(b[2] | (b[3] << 8)));
      const uint8_t *sc = b + 4, *qs = b + 16;
      for (int j = 0; j < 256; j++) {
        const int n64 = j / 64, wi = j % 64, l = wi % 32, is = 2 * n64 + (wi >= 32);
        int s, m;
        if (is < 4) { s = sc[is] & 63; m = sc[is + 4] & 63; }
        else { s = (sc[is + 4] & 0xF) | ((sc[is - 4] >> 6) << 4); m = (sc[is + 4] >> 4) | ((sc[is] >> 6) << 4); }
        const int q = wi < 32 ? (qs[n64 * 32 + l] & 0xF) : (qs[n64 * 32 + l] >> 4);
        sum += (d * (float)s * (float)q - dmin * (float)m) * x[blk * 256 + j];
      }
    } else {
      const uint8_t *b = w + blk * 210;
      const float d = h_f16((uint16_t)(b[208] | (b[209] << 8)));
      for (int j = 0; j < 256; j++) {
        const int half = j / 128, wi = j % 128, quarter = wi / 32, l = wi % 32, is = l / 16;
        int lo = (quarter & 1) ? b[half * 64 + l + 32] : b[half * 64 + l];
        lo = (quarter & 2) ? (lo >> 4) : (lo & 0xF);
        const int q = (lo | (((b[128 + half * 32 + l] >> (2 * quarter)) & 3) << 4)) - 32;
        sum += d * (float)(int8_t)b[192 + half * 8 + is + 2 * quarter] * (float)q * x[blk * 256 + j];
      }
    }
  }
  return sum;
}

}  // namespace

// The OpenClBackend analogue (backend/opencl.rs:79-516).
struct pk_backend {
  int device = 0;
  cudaStream_t st = nullptr;
  std::map<std::pair<const void *, size_t>, void *> weights;  // (host ptr, len) -> packed device copy
  float *d_x = nullptr, *d_out = nullptr;
  size_t x_cap = 0, out_cap = 0;
  Q8Dev act;
  int act_k = 0;
  ~pk_backend() {
    if (st) cudaStreamSynchronize(st);
    for (auto &kv : weights) cudaFree(kv.second);
    cudaFree(d_x);
    cudaFree(d_out);
    cudaFree(act.q);
    cudaFree(act.d);
    cudaFree(act.s);
    if (st) cudaStreamDestroy(st);
  }
};

struct pk_engine {
  Engine eng;
};

extern "C" {

const char *pk_last_error(void) { return t_err.c_str(); }
int pk_version(void) { return 100; }
int pk_device_binary_version(int *out) {
  if (!out) return set_error(PK_ERR_INVALID, "null out");
  CK(kernels_binary_version(out));
  return PK_OK;
}
int pk_supports(uint32_t ttype) { return type_is_matvec((int)ttype) ? 1 : 0; }

int pk_q8_quantize(const float *x, int k, int b, pk_q8act *act, void *stream) {
  if (!x || k <= 0 || k % 32 != 0 || b < 1 || b > 64)
    return set_error(PK_ERR_INVALID, "pk_q8_quantize: k must be a positive multiple of 32 and b in 1..64");
  if (!q8_ok(act, k) || act->b != b) return set_error(PK_ERR_INVALID, "pk_q8_quantize: activation buffer does not match k/b");
  CK(launch_q8(x, b, 1, k, b, to_dev(act), (cudaStream_t)stream));
  return PK_OK;
}

int pk_expf(const float *x, float *out, int n, void *stream) {
  if (!x || !out || n < 0) return set_error(PK_ERR_INVALID, "pk_expf: bad arguments");
  if (n == 0) return PK_OK;
  CK(launch_expf(x, out, n, (cudaStream_t)stream));
  return PK_OK;
}

size_t pk_packed_bytes(uint32_t ttype, int k, int n_rows) {
  if (!type_is_matvec((int)ttype) || k <= 0 || n_rows <= 0) return 0;
  return packed_bytes((int)ttype, k, n_rows);
}

int pk_pack_weights(uint32_t ttype, const void *raw, size_t row_bytes, int k, int n_rows, void *packed, void *stream) {
  int rc = check_matvec_shape(ttype, k, n_rows);
  if (rc) return rc;
  int be, bb;
  type_block((int)ttype, &be, &bb);
  if (row_bytes != (size_t)(k / be) * bb) return set_error(PK_ERR_INVALID, "row_bytes does not match k for this type");
  if (!raw || !packed || ((uintptr_t)packed & 15)) return set_error(PK_ERR_INVALID, "packed buffer must be 16-byte aligned");
  CK(launch_pack((int)ttype, raw, row_bytes, k, n_rows, packed, (cudaStream_t)stream));
  return PK_OK;
}

int pk_matmul_packed(uint32_t ttype, const void *packed, int k, int n_rows, const pk_q8act *act, float *out,
                     void *stream) {
  int rc = check_matvec_shape(ttype, k, n_rows);
  if (rc) return rc;
  if (!q8_ok(act, k)) return set_error(PK_ERR_INVALID, "activation does not match k");
  if (!packed || !out || ((uintptr_t)packed & 15)) return set_error(PK_ERR_INVALID, "packed weights must be 16-byte aligned");
  return matmul_packed(ttype, packed, k, n_rows, act, out, (cudaStream_t)stream);
}

int pk_matmul(uint32_t ttype, const void *w, size_t row_bytes, int k, int n_rows, const pk_q8act *act, float *out,
              void *stream) {
  int rc = check_matvec_shape(ttype, k, n_rows);
  if (rc) return rc;
  if (!q8_ok(act, k)) return set_error(PK_ERR_INVALID, "activation does not match k");
  int be, bb;
  type_block((int)ttype, &be, &bb);
  if (row_bytes != (size_t)(k / be) * bb) return set_error(PK_ERR_INVALID, "row_bytes does not match k for this type");
  if (!w || !out) return set_error(PK_ERR_INVALID, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (ttype == PK_TYPE_Q4_K && ((uintptr_t)w & 15) == 0)  // the device layout of Q4_K is the GGUF layout
    return matmul_packed(ttype, w, k, n_rows, act, out, st);
  void *tmp = nullptr;
  CK(cudaMallocAsync(&tmp, packed_bytes((int)ttype, k, n_rows), st));
  cudaError_t e = launch_pack((int)ttype, w, row_bytes, k, n_rows, tmp, st);
  if (e != cudaSuccess) {
    cudaFreeAsync(tmp, st);
    return cuda_error(e, "pack");
  }
  rc = matmul_packed(ttype, tmp, k, n_rows, act, out, st);
  cudaFreeAsync(tmp, st);
  return rc;
}

int pk_matmul_noalloc(uint32_t ttype, const void *w, size_t row_bytes, int k, int n_rows, const pk_q8act *act,
                      float *out, void *stream) {
  int rc = check_matvec_shape(ttype, k, n_rows);
  if (rc) return rc;
  if (!q8_ok(act, k)) return set_error(PK_ERR_INVALID, "activation does not match k");
  int be, bb;
  type_block((int)ttype, &be, &bb);
  if (row_bytes != (size_t)(k / be) * bb) return set_error(PK_ERR_INVALID, "row_bytes does not match k for this type");
  if (!w || !out) return set_error(PK_ERR_INVALID, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (ttype == PK_TYPE_Q4_K && ((uintptr_t)w & 15) == 0)  // used in place: no scratch
    return matmul_packed(ttype, w, k, n_rows, act, out, st);
  const size_t need = packed_bytes((int)ttype, k, n_rows);
  if (need > PK_NOALLOC_SCRATCH_BYTES)
    return set_error(PK_ERR_INVALID, "pk_matmul_noalloc: these rows need " + std::to_string(need) +
                                         " bytes of scratch, the fixed scratch holds " +
                                         std::to_string((size_t)PK_NOALLOC_SCRATCH_BYTES));
  void *scratch = nullptr;
  CK(noalloc_scratch(&scratch));
  CK(launch_pack((int)ttype, w, row_bytes, k, n_rows, scratch, st));
  return matmul_packed(ttype, scratch, k, n_rows, act, out, st);
}

int pk_backend_new(int device, pk_backend **out) {
  if (!out) return set_error(PK_ERR_INVALID, "null out");
  int n = 0;
  CK(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return set_error(PK_ERR_INVALID, "no CUDA device " + std::to_string(device));
  auto *be = new (std::nothrow) pk_backend();
  if (!be) return set_error(PK_ERR_OOM, "out of host memory");
  be->device = device;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&be->st, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete be;
    return cuda_error(e, "pk_backend_new");
  }
  void *scratch = nullptr;  // reserve pk_matmul_noalloc's scratch on this device now (see pk.h)
  if (noalloc_scratch(&scratch) != cudaSuccess) cudaGetLastError();
  *out = be;
  return PK_OK;
}

void pk_backend_free(pk_backend *be) { delete be; }

int pk_backend_supports(pk_backend *, uint32_t ttype) { return pk_supports(ttype); }

int pk_backend_matvec(pk_backend *be, uint32_t ttype, const void *w, size_t w_len, int k, const float *x, float *out,
                      int n_rows) {
  if (!be || !w || !x || !out) return set_error(PK_ERR_INVALID, "null argument");
  int rc = check_matvec_shape(ttype, k, n_rows);
  if (rc) return rc;
  int bsz, bb;
  type_block((int)ttype, &bsz, &bb);
  const size_t row_bytes = (size_t)(k / bsz) * bb;
  if (w_len != row_bytes * (size_t)n_rows) return set_error(PK_ERR_INVALID, "weight slice length does not match k x n_rows");
  CK(cudaSetDevice(be->device));
  auto key = std::make_pair(w, w_len);
  auto it = be->weights.find(key);
  void *packed = nullptr;
  if (it == be->weights.end()) {
    void *raw = nullptr;
    CK(cudaMalloc(&packed, packed_bytes((int)ttype, k, n_rows)));
    cudaError_t e = cudaMalloc(&raw, w_len);
    if (e == cudaSuccess) e = cudaMemcpyAsync(raw, w, w_len, cudaMemcpyHostToDevice, be->st);
    if (e == cudaSuccess) e = launch_pack((int)ttype, raw, row_bytes, k, n_rows, packed, be->st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(be->st);
    cudaFree(raw);
    if (e != cudaSuccess) {
      cudaFree(packed);
      return cuda_error(e, "weight upload");
    }
    be->weights[key] = packed;
  } else {
    packed = it->second;
  }
  if ((size_t)k * 4 > be->x_cap) {
    cudaFree(be->d_x);
    be->d_x = nullptr;
    be->x_cap = 0;
    CK(cudaMalloc((void **)&be->d_x, (size_t)k * 4));
    be->x_cap = (size_t)k * 4;
  }
  if ((size_t)n_rows * 4 > be->out_cap) {
    cudaFree(be->d_out);
    be->d_out = nullptr;
    be->out_cap = 0;
    CK(cudaMalloc((void **)&be->d_out, (size_t)n_rows * 4));
    be->out_cap = (size_t)n_rows * 4;
  }
  if (k > be->act_k) {
    cudaFree(be->act.q);
    cudaFree(be->act.d);
    cudaFree(be->act.s);
    be->act = Q8Dev();
    be->act_k = 0;
    CK(cudaMalloc((void **)&be->act.q, (size_t)k));
    CK(cudaMalloc((void **)&be->act.d, (size_t)k / 32 * 4));
    CK(cudaMalloc((void **)&be->act.s, (size_t)k / 32 * 4));
    be->act_k = k;
  }
  Q8Dev a = be->act;
  a.k = k;
  a.b = 1;
  CK(cudaMemcpyAsync(be->d_x, x, (size_t)k * 4, cudaMemcpyHostToDevice, be->st));
  CK(launch_q8(be->d_x, 1, 1, k, 1, a, be->st));
  B1Src src;
  src.act = a;
  CK(launch_mv_b1(packed_view((int)ttype, k, n_rows, packed), src, be->d_out, false, be->st));
  CK(cudaMemcpyAsync(out, be->d_out, (size_t)n_rows * 4, cudaMemcpyDeviceToHost, be->st));
  CK(cudaStreamSynchronize(be->st));
  return PK_OK;
}

// backend/opencl.rs:391-430
int pk_backend_selftest(pk_backend *be) {
  if (!be) return set_error(PK_ERR_INVALID, "null backend");
  const int k = 256;
  float x[256];
  for (int j = 0; j < k; j++) x[j] = (float)(j % 7) * 0.1f - 0.3f;
  uint8_t w4[144], w6[210];
  std::memset(w4, 0, sizeof(w4));
  w4[0] = 0x00; w4[1] = 0x3C;
  w4[4] = 1;
  for (int i = 0; i < 128; i++) w4[16 + i] = 0x21;
  for (int i = 0; i < 128; i++) w6[i] = 0x95;
  for (int i = 0; i < 64; i++) w6[128 + i] = 0x1B;
  for (int i = 0; i < 16; i++) w6[192 + i] = 2;
  w6[208] = 0x00; w6[209] = 0x3C;
  struct Case { uint32_t t; const uint8_t *w; size_t len; const char *name; } cases[2] = {
      {PK_TYPE_Q4_K, w4, sizeof(w4), "q4_K"}, {PK_TYPE_Q6_K, w6, sizeof(w6), "q6_K"}};
  int result = PK_OK;
  for (auto &c : cases) {
    float got = 0.0f;
    int rc = pk_backend_matvec(be, c.t, c.w, c.len, k, x, &got, 1);
    if (rc) { result = rc; break; }
    const float want = host_dot_f32(c.t, c.w, k, x);
    if (std::fabs(got - want) > std::fabs(want) * 0.02f + 0.01f) {
      result = set_error(PK_ERR_INVALID, std::string(c.name) + " self-test failed: gpu=" + std::to_string(got) +
                                             " cpu=" + std::to_string(want));
      break;
    }
  }
  for (auto &kv : be->weights) cudaFree(kv.second);  // clear_weight_cache (the buffers were stack-local)
  be->weights.clear();
  return result;
}

int pk_create(int device, int n_ctx, int max_batch, pk_engine **out) {
  if (!out) return set_error(PK_ERR_INVALID, "null out");
  auto *e = new (std::nothrow) pk_engine();
  if (!e) return set_error(PK_ERR_OOM, "out of host memory");
  int rc = e->eng.create(device, n_ctx, max_batch);
  if (rc) {
    delete e;
    return rc;
  }
  *out = e;
  return PK_OK;
}

int pk_load_gguf(pk_engine *e, const char *path) {
  if (!e || !path) return set_error(PK_ERR_INVALID, "null argument");
  return e->eng.load(path);
}

void pk_destroy(pk_engine *e) { delete e; }

int pk_model_info_get(pk_engine *e, pk_model_info *info) {
  if (!e || !info) return set_error(PK_ERR_INVALID, "null argument");
  return e->eng.info(info);
}

int pk_forward(pk_engine *e, const uint32_t *ids, const int *positions, int n, int want_logits) {
  if (!e || !ids || !positions) return set_error(PK_ERR_INVALID, "null argument");
  return e->eng.forward(ids, positions, n, want_logits != 0);
}

int pk_logits(pk_engine *e, float *out, int n) {
  if (!e || !out) return set_error(PK_ERR_INVALID, "null argument");
  return e->eng.logits(out, n);
}

int pk_argmax(pk_engine *e, uint32_t *token) {
  if (!e || !token) return set_error(PK_ERR_INVALID, "null argument");
  return e->eng.argmax(token);
}

int pk_generate(pk_engine *e, const uint32_t *prompt, int n, const pk_gen_opts *opts, pk_token_cb cb, void *user,
                uint32_t *out_ids, int out_cap, int *n_out, pk_gen_stats *stats) {
  if (!e || !prompt || !opts) return set_error(PK_ERR_INVALID, "null argument");
  return e->eng.generate(prompt, n, *opts, cb, user, out_ids, out_cap, n_out, stats);
}

int pk_decode_steps_device(pk_engine *e, int n_steps, uint32_t *out_ids, float *device_ms) {
  if (!e) return set_error(PK_ERR_INVALID, "null engine");
  return e->eng.decode_steps_device(n_steps, out_ids, device_ms);
}

int pk_set_matmul_path(int path) {
  if (path != PK_MATMUL_MMA_SYNC && path != PK_MATMUL_TCGEN05) return set_error(PK_ERR_INVALID, "unknown matmul path");
  set_mv_path(path);
  return PK_OK;
}

int pk_set_kv_type(pk_engine *e, int type) {
  if (!e) return set_error(PK_ERR_INVALID, "null engine");
  return e->eng.set_kv_type(type);
}

int pk_set_order(pk_engine *e, int order) {
  if (!e) return set_error(PK_ERR_INVALID, "null engine");
  return e->eng.set_order(order);
}

int pk_set_position(pk_engine *e, int pos) {
  if (!e) return set_error(PK_ERR_INVALID, "null engine");
  return e->eng.set_position(pos);
}

int pk_streams_begin(pk_engine *e, int n_streams) {
  if (!e) return set_error(PK_ERR_INVALID, "null engine");
  return e->eng.streams_begin(n_streams);
}

int pk_stream_prefill(pk_engine *e, int s, const uint32_t *prompt, int n) {
  if (!e || !prompt) return set_error(PK_ERR_INVALID, "null argument");
  return e->eng.stream_prefill(s, prompt, n);
}

int pk_streams_decode(pk_engine *e, int n_steps, uint32_t *out_ids, float *device_ms) {
  if (!e) return set_error(PK_ERR_INVALID, "null engine");
  return e->eng.streams_decode(n_steps, out_ids, device_ms);
}

int pk_streams_set_position(pk_engine *e, int pos) {
  if (!e) return set_error(PK_ERR_INVALID, "null engine");
  return e->eng.streams_set_position(pos);
}

int pk_decode_profile(pk_engine *e, pk_kernel_stat *out, int cap, int *n_out) {
  if (!e || (!out && cap > 0)) return set_error(PK_ERR_INVALID, "null argument");
  return e->eng.decode_profile(out, cap, n_out);
}

int pk_selftest_bounded_wait(pk_engine *e, int *status) {
  if (!e || !status) return set_error(PK_ERR_INVALID, "null argument");
  return e->eng.selftest_bounded_wait(status);
}

int pk_set_debug(pk_engine *e, int on) {
  if (!e) return set_error(PK_ERR_INVALID, "null engine");
  return e->eng.set_debug(on != 0);
}

int pk_get_dump(pk_engine *e, const char *name, float *out, int cap, int *n_out) {
  if (!e || !name) return set_error(PK_ERR_INVALID, "null argument");
  return e->eng.get_dump(name, out, cap, n_out);
}

void pk_request_stop(void) { g_stop.store(true); }
void pk_clear_stop(void) { g_stop.store(false); }

size_t pk_sample_scratch_bytes(int n) { return n > 0 ? sample_scratch_bytes(n) : 0; }

int pk_sample(const float *logits, int n, float temp, float top_p, uint64_t *rng_state, void *scratch,
              uint32_t *tok, void *stream) {
  if (!logits || !rng_state || !scratch || !tok || n < 1 || !(temp > 0.0f))
    return set_error(PK_ERR_INVALID, "pk_sample: null pointer, n < 1 or temp <= 0");
  if (((uintptr_t)scratch) & 255) return set_error(PK_ERR_INVALID, "pk_sample: scratch must be 256-byte aligned");
  CK(launch_sample(logits, n, temp, top_p, (unsigned long long *)rng_state, scratch, tok, (cudaStream_t)stream));
  return PK_OK;
}

// ---- tensor-parallel decode
struct pk_tp {
  pk::TpEngine eng;
};

int pk_tp_create(int device, int n_ctx, int rank, int world, pk_tp **out) {
  if (!out) return set_error(PK_ERR_INVALID, "null argument");
  *out = nullptr;
  pk_tp *t = new (std::nothrow) pk_tp;
  if (!t) return set_error(PK_ERR_OOM, "out of host memory");
  const int rc = t->eng.create(device, n_ctx, rank, world);
  if (rc) {
    delete t;
    return rc;
  }
  *out = t;
  return PK_OK;
}

void pk_tp_destroy(pk_tp *t) { delete t; }

int pk_tp_load_gguf(pk_tp *t, const char *path) {
  if (!t || !path) return set_error(PK_ERR_INVALID, "null argument");
  return t->eng.load(path);
}

int pk_tp_load_synthetic(pk_tp *t, const pk_tp_model *m, uint64_t seed) {
  if (!t || !m) return set_error(PK_ERR_INVALID, "null argument");
  pk::Config c;
  c.arch = "llama";
  c.n_layer = m->n_layer;
  c.n_embd = m->n_embd;
  c.n_head = m->n_head;
  c.n_head_kv = m->n_head_kv;
  c.head_dim = m->head_dim;
  c.n_ff = m->n_ff;
  c.n_vocab = m->n_vocab;
  c.n_rot = m->n_rot;
  c.rope_theta = m->rope_theta;
  c.rms_eps = m->rms_eps;
  return t->eng.load_synthetic(c, m->n_vocab, seed);
}

int pk_tp_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int pk_tp_ipc_handle(pk_tp *t, void *out) {
  if (!t || !out) return set_error(PK_ERR_INVALID, "null argument");
  return t->eng.ipc_handle(out);
}

int pk_tp_open_peers(pk_tp *t, const void *handles) {
  if (!t || !handles) return set_error(PK_ERR_INVALID, "null argument");
  return t->eng.open_peers(handles);
}

int pk_tp_nccl_id_bytes(void) { return tp_nccl_id_bytes(); }

int pk_tp_nccl_id(void *out) { return tp_nccl_id(out); }

int pk_tp_use_nccl(pk_tp *t, const void *id) {
  if (!t || !id) return set_error(PK_ERR_INVALID, "null argument");
  return t->eng.use_nccl(id);
}

int pk_tp_prefill(pk_tp *t, const uint32_t *prompt, int n) {
  if (!t || !prompt) return set_error(PK_ERR_INVALID, "null argument");
  return t->eng.prefill(prompt, n);
}

int pk_tp_decode(pk_tp *t, int n_steps, uint32_t *out_ids, float *device_ms) {
  if (!t) return set_error(PK_ERR_INVALID, "null argument");
  return t->eng.decode(n_steps, out_ids, device_ms);
}

int pk_tp_logits(pk_tp *t, float *out, int n, int *n_local, int *vocab0) {
  if (!t || (!out && n > 0)) return set_error(PK_ERR_INVALID, "null argument");
  return t->eng.logits(out, n, n_local, vocab0);
}

int pk_tp_info_get(pk_tp *t, pk_tp_info *info) {
  if (!t || !info) return set_error(PK_ERR_INVALID, "null argument");
  return t->eng.info(info);
}

int pk_tp_split(int n_head, int n_head_kv, int head_dim, int n_ff, int n_vocab, int rank, int world, int o_block,
                int down_block, int out[5]) {
  if (!out) return set_error(PK_ERR_INVALID, "null argument");
  pk::Config c;
  c.n_head = n_head;
  c.n_head_kv = n_head_kv;
  c.head_dim = head_dim;
  c.n_ff = n_ff;
  pk::TpSplit s;
  std::string why;
  if (!pk::tp_split(c, n_vocab, rank, world, o_block, down_block, s, why)) return set_error(PK_ERR_UNSUPPORTED, why);
  out[0] = s.nh;
  out[1] = s.nkv;
  out[2] = s.ff;
  out[3] = s.vocab0;
  out[4] = s.nvocab;
  return PK_OK;
}

uint32_t pk_tp_pick(const float *vals, const int *idx, int world) {
  if (!vals || !idx || world < 1 || world > pk::TP_MAX) return 0;
  return pk::tp_pick(vals, idx, world);
}

}  // extern "C"

// ---------------------------------------------------------------- prompt text
struct pk_tokenizer {
  pk::text::Tokenizer tok;
};

namespace {

// Roles and contents of chat messages: present and valid UTF-8 (the
// reference receives them as Rust strings, which always are).
int read_messages(const pk_chat_message *msgs, int n_msgs, std::vector<pk::text::Message> &m) {
  m.assign((size_t)n_msgs, pk::text::Message{});
  std::u32string check;
  for (int i = 0; i < n_msgs; i++) {
    if (!msgs[i].role || !msgs[i].content) return set_error(PK_ERR_INVALID, "message with a null role or content");
    m[i].role = msgs[i].role;
    m[i].content = msgs[i].content;
    if (!pk::text::utf8_decode(m[i].role.data(), m[i].role.size(), &check) ||
        !pk::text::utf8_decode(m[i].content.data(), m[i].content.size(), &check))
      return set_error(PK_ERR_INVALID, "message " + std::to_string(i) + " is not valid UTF-8");
  }
  return PK_OK;
}

template <class T>
int copy_out(const T *src, size_t n, T *out, size_t cap, size_t *n_out, const char *what) {
  if (n_out) *n_out = n;
  if (out && cap) std::memcpy(out, src, std::min(n, cap) * sizeof(T));
  if (n > cap) return set_error(PK_ERR_INVALID, std::string(what) + ": output needs " + std::to_string(n) + " entries");
  return PK_OK;
}

}  // namespace

extern "C" {

int pk_tokenizer_load(const char *path, pk_tokenizer **out) {
  if (!path || !out) return set_error(PK_ERR_INVALID, "null argument");
  *out = nullptr;
  pk::Gguf g;
  std::string err;
  if (!g.open(path, err)) return set_error(PK_ERR_IO, err);
  pk_tokenizer *t = new (std::nothrow) pk_tokenizer;
  if (!t) return set_error(PK_ERR_OOM, "tokenizer allocation");
  if (!t->tok.load(g, err)) {
    delete t;
    return set_error(PK_ERR_IO, err);
  }
  *out = t;
  return PK_OK;
}

void pk_tokenizer_free(pk_tokenizer *t) { delete t; }

int pk_tokenizer_info_get(const pk_tokenizer *t, pk_tokenizer_info *o) {
  if (!t || !o) return set_error(PK_ERR_INVALID, "null argument");
  std::memset(o, 0, sizeof(*o));
  o->n_vocab = (int32_t)t->tok.n_vocab();
  o->bos_id = t->tok.bos_id();
  const auto &e = t->tok.eos_ids();
  o->n_eos = (int32_t)e.size();
  for (size_t i = 0; i < e.size() && i < 16; i++) o->eos_ids[i] = e[i];
  o->ignore_merges = t->tok.ignore_merges() ? 1 : 0;
  std::snprintf(o->pre, sizeof(o->pre), "%s", t->tok.pre().c_str());
  return PK_OK;
}

int pk_tokenize(const pk_tokenizer *t, const char *text, size_t len, int parse_special, uint32_t *out, size_t cap,
                size_t *n_out) {
  if (!t || (!text && len) || (!out && cap)) return set_error(PK_ERR_INVALID, "null argument");
  std::u32string check;
  if (!pk::text::utf8_decode(text, len, &check)) return set_error(PK_ERR_INVALID, "text is not valid UTF-8");
  const std::vector<uint32_t> ids = t->tok.encode(std::string(text ? text : "", len), parse_special != 0);
  return copy_out(ids.data(), ids.size(), out, cap, n_out, "pk_tokenize");
}

int pk_token_bytes(const pk_tokenizer *t, uint32_t id, uint8_t *out, size_t cap, size_t *n_out) {
  if (!t || (!out && cap)) return set_error(PK_ERR_INVALID, "null argument");
  const std::string b = t->tok.token_bytes(id);
  return copy_out(reinterpret_cast<const uint8_t *>(b.data()), b.size(), out, cap, n_out, "pk_token_bytes");
}

int pk_token_is_eog(const pk_tokenizer *t, uint32_t id) { return t && t->tok.is_eog(id) ? 1 : 0; }

int pk_utf8_flush(uint8_t *pending, size_t *n_pending, uint8_t *out, size_t cap, size_t *n_out) {
  if (!n_pending || (!pending && *n_pending) || (!out && cap)) return set_error(PK_ERR_INVALID, "null argument");
  std::string text;
  const size_t used = pk::text::utf8_flush(pending, *n_pending, text);
  const int rc = copy_out(reinterpret_cast<const uint8_t *>(text.data()), text.size(), out, cap, n_out,
                          "pk_utf8_flush");
  if (rc) return rc;
  std::memmove(pending, pending + used, *n_pending - used);
  *n_pending -= used;
  return PK_OK;
}

int pk_text_find(const char *pattern, size_t plen, const char *text, size_t tlen, uint32_t *bounds, size_t cap,
                 size_t *n_out) {
  if ((!pattern && plen) || (!text && tlen) || (!bounds && cap)) return set_error(PK_ERR_INVALID, "null argument");
  std::u32string p, t;
  if (!pk::text::utf8_decode(pattern, plen, &p) || !pk::text::utf8_decode(text, tlen, &t))
    return set_error(PK_ERR_INVALID, "pattern or text is not valid UTF-8");
  const pk::text::Pattern pat(p);
  std::vector<uint32_t> b;
  for (const auto &m : pat.find(t)) {
    b.push_back((uint32_t)m.first);
    b.push_back((uint32_t)m.second);
  }
  return copy_out(b.data(), b.size(), bounds, cap, n_out, "pk_text_find");
}

int pk_chat_apply(const pk_chat_message *msgs, int n_msgs, int minicpm5, int add_generation_prompt, char *out,
                  size_t cap, size_t *n_out) {
  if ((!msgs && n_msgs) || n_msgs < 0 || (!out && cap)) return set_error(PK_ERR_INVALID, "null argument");
  std::vector<pk::text::Message> m;
  if (const int rc = read_messages(msgs, n_msgs, m)) return rc;
  const std::string s = minicpm5 ? pk::text::apply_minicpm5(m, add_generation_prompt != 0)
                                 : pk::text::apply_generic(m, add_generation_prompt != 0);
  return copy_out(s.data(), s.size(), out, cap, n_out, "pk_chat_apply");
}

int pk_chat_prompt(const pk_tokenizer *t, const pk_chat_message *msgs, int n_msgs, int minicpm5, int direct_answer,
                   size_t n_ctx, uint32_t *ids, size_t cap, size_t *n_ids, int *n_dropped, int *direct_applied) {
  if (!t || (!msgs && n_msgs) || n_msgs < 0 || (!ids && cap)) return set_error(PK_ERR_INVALID, "null argument");
  std::vector<pk::text::Message> all;
  if (const int rc = read_messages(msgs, n_msgs, all)) return rc;
  // n_ctx - 1024 as the bridge's unsigned arithmetic has it: below 1024 the
  // difference wraps and nothing is dropped
  const size_t limit = n_ctx >= 1024 ? n_ctx - 1024 : SIZE_MAX;
  std::vector<size_t> kept((size_t)n_msgs);
  for (size_t i = 0; i < kept.size(); i++) kept[i] = i;
  std::vector<uint32_t> toks;
  bool direct = false;
  for (;;) {
    std::vector<pk::text::Message> view;
    for (size_t i : kept) view.push_back(all[i]);
    std::string prompt = minicpm5 ? pk::text::apply_minicpm5(view, true) : pk::text::apply_generic(view, true);
    const std::string head = "<|im_start|>assistant\n";
    direct = direct_answer && minicpm5 && prompt.size() >= head.size() &&
             prompt.compare(prompt.size() - head.size(), head.size(), head) == 0;
    if (direct) prompt += pk::text::direct_suffix();
    toks = t->tok.encode(prompt, true);
    if (toks.size() <= limit) break;
    const size_t oldest = (!kept.empty() && all[kept[0]].role == "system") ? 2 : 1;
    if (kept.size() <= oldest + 1)
      return set_error(PK_ERR_CONTEXT_FULL,
                       "Latest request exceeds the context window. Select a larger window or shorten the message.");
    kept.erase(kept.begin() + (long)oldest);
  }
  if (n_dropped) *n_dropped = n_msgs - (int)kept.size();
  if (direct_applied) *direct_applied = direct ? 1 : 0;
  return copy_out(toks.data(), toks.size(), ids, cap, n_ids, "pk_chat_prompt");
}

int pk_chat_is_minicpm5(const char *pre, const char *name) {
  return pk::text::is_minicpm5(pre ? pre : "", name ? name : "") ? 1 : 0;
}

const char *pk_chat_direct_suffix(void) { return pk::text::direct_suffix(); }
const char *pk_chat_thinking_suffix(void) { return pk::text::thinking_on_suffix(); }

}  // extern "C"
