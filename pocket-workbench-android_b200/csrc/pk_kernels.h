// pk_kernels.h -- host-side view of the sm_100a kernels (launchers).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace pk {

// A weight matrix in the device layout (n_rows rows of k elements).
//   Q4_K : q = raw GGUF blocks (144 B, already 16-byte aligned), d = nullptr
//   Q6_K : q = [rows][nblk][208 B] (ql | qh | scales), d = [rows][nblk] f16
//   Q8_0 : q = [rows][k] int8,                         d = [rows][k/32] f16
//   Q4_0 : q = [rows][k/2] nibbles (GGUF order),      d = [rows][k/32] f16
// The split keeps every per-thread load 16-byte aligned; the bytes are the
// GGUF block bytes rearranged, so the arithmetic is unchanged.
struct DevTensor {
  int type = -1, k = 0, rows = 0;
  const uint8_t *q = nullptr;
  const uint16_t *d = nullptr;
};

// Q8Act in device memory: q [b][k], d/s [b][k/32].
struct Q8Dev {
  int8_t *q = nullptr;
  float *d = nullptr;
  int32_t *s = nullptr;
  int k = 0, b = 0;
};

bool type_is_matvec(int type);
bool type_block(int type, int *be, int *bb);
size_t packed_q_bytes(int type, int k, int rows);
size_t packed_bytes(int type, int k, int rows);
DevTensor packed_view(int type, int k, int rows, const void *packed);

// Raw GGUF rows (device) -> device layout.
cudaError_t launch_pack(int type, const void *raw, size_t row_bytes, int k, int rows, void *packed,
                        cudaStream_t st);
// Dequantise rows of a raw GGUF tensor: out[i][k] = row ids[i] (ids on device, or
// ids == nullptr for rows 0..n-1).  Used for the embedding and norm weights.
cudaError_t launch_dequant_rows(int type, const void *raw, size_t row_bytes, int k, const uint32_t *ids,
                                int n, float *out, cudaStream_t st);

// Q8Act::prepare on x[i * xs_elem + bi * xs_lane].
cudaError_t launch_q8(const float *x, long xs_elem, long xs_lane, int k, int b, Q8Dev act, cudaStream_t st);
// binaryVersion of this library's device code as loaded on the current device.
cudaError_t kernels_binary_version(int *v);
// RMSNorm (model.rs:812-822) + Q8 of token-major x [b][k]; xn (optional) gets the normed floats.
// neon: the sum of squares in the reference's b == 1 order (simd.rs:47-64)
// for every row, instead of the b > 1 sequential chain.
cudaError_t launch_rmsnorm_q8(const float *x, const float *nw, float eps, int k, int b, Q8Dev act, float *xn,
                              cudaStream_t st, bool neon = false);

// SwiGLU + Q8 of token-major g, u [b][k]; h (optional) gets the floats.
cudaError_t launch_swiglu_q8(const float *g, const float *u, int k, int b, Q8Dev act, float *h, cudaStream_t st);

// Multi-lane matvec: out[r * os_row + lane * os_lane] (+)= row r . lane.
cudaError_t launch_mv_lanes(const DevTensor &w, const Q8Dev &act, float *out, long os_row, long os_lane,
                            bool add, cudaStream_t st);
// Several matrices (at most three) against the same activation in one launch.
struct MvOut {
  DevTensor w;
  float *out;
  long os_row, os_lane;
  bool add;
};
// b > 8 runs on the tcgen05 tensor cores (pk_mv_tc.cu) when that path is
// selected (set_mv_path(1), or PK_PREFILL_MMA=tc) and every matrix suits
// it; otherwise, and for every b <= 8, on the mma.sync tiles.
cudaError_t launch_mv_multi(int n, const MvOut *outs, const Q8Dev &act, cudaStream_t st);
// The tcgen05 matvec (pk_mv_tc.cu): whether it takes this matrix and
// activation, the launch, and its error word (0, or PK_ERR_TIMEOUT after a
// bounded wait ran out; clear resets it).
bool mv_tc_supports(const DevTensor &w, const Q8Dev &act);
cudaError_t launch_mv_tc(int n, const MvOut *outs, const Q8Dev &act, cudaStream_t st);
int mv_tc_error(bool clear);
// Selects the b > 8 matvec kernel: 0 mma.sync tiles, 1 tcgen05.
void set_mv_path(int path);

// Single-lane matvec with the activation quantised inside each CTA:
// src = x (k floats, optionally RMS-normalised by nw) or a precomputed Q8 act.
struct B1Src {
  const float *x = nullptr;
  const float *nw = nullptr;
  float eps = 0.0f;
  Q8Dev act;  // used when x == nullptr
};
cudaError_t launch_mv_b1(const DevTensor &w, const B1Src &src, float *out, bool add, cudaStream_t st);

// Fused q/k/v matvecs + RoPE + KV write for one decode token.
struct QkvArgs {
  DevTensor wq, wk, wv;
  B1Src src;
  const int *pos = nullptr;          // device scalar: position of the token
  const float *rope_cos = nullptr;   // [n_ctx][half]
  const float *rope_sin = nullptr;
  int half = 0, dh = 0, n_ctx = 0;
  float *qout = nullptr;   // [n_head * dh]
  float *kcache = nullptr; // this layer: K d-major [n_kv][dh][n_ctx]
  float *vcache = nullptr;
  int kv16 = 0;            // 1: the caches hold f16 entries (same element offsets)
};
cudaError_t launch_qkv_b1(const QkvArgs &a, cudaStream_t st);
// Fused gate/up matvecs + SwiGLU (model.rs:1105-1115) for one token.
cudaError_t launch_gateup_b1(const DevTensor &wg, const DevTensor &wu, const B1Src &src, float *h,
                             cudaStream_t st);

// RoPE + KV write for b tokens (token-major q [b][qdim], k/v [b][kdim]).
// kv16: the caches hold f16 entries (each value rounded to nearest even).
cudaError_t launch_rope_kv(float *q, const float *k, const float *v, int b, const int *pos, const float *rope_cos,
                           const float *rope_sin, int half, int dh, int n_head, int n_kv, int n_ctx, float *kcache,
                           float *vcache, cudaStream_t st, size_t lane_stride = 0, bool kv16 = false);
// out[i] = expf_lib(x[i]) (the C library's expf, bit for bit).
cudaError_t launch_expf(const float *x, float *out, long n, cudaStream_t st);

// Causal GQA attention (model.rs:993-1087) for b tokens at positions pos[b].
struct AttnArgs {
  const float *q;      // [b][n_head * dh]
  const float *kcache; // layer base, K d-major [n_kv][dh][n_ctx]
  const float *vcache;
  const int *pos;      // [b] device
  float *out;          // [b][n_head * dh]
  int b, n_head, n_kv, dh, n_ctx;
  float scale;
  float *scores;       // scratch [b][n_head][n_ctx]
  Q8Dev q8{};          // optional (q8.q != nullptr): Q8 of out, k = n_head * dh
  size_t lane_stride = 0;  // elements from token i's K/V cache to token i + 1's (0: one shared cache)
  int b1_order = 0;        // 1: every token scored in the b == 1 order (simd.rs:19-43), one CTA each
  int kv16 = 0;            // 1: the caches hold f16 entries (k_attn, one CTA per token and head)
  // b == 1 order over long histories: pchunk positions per scoring CTA (a
  // multiple of 128) and pmax scratch [b][n_head][ceil(n_ctx / pchunk)] for
  // their maxima; then the value pass runs one CTA per (token, head, 32 d).
  float *pmax = nullptr;
  int pchunk = 0;
};
cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st);

// sampler.rs:21-92 for temp > 0 (temperature + top-p) on the device: the
// token into *tok, rng (the splitmix64 state, device memory) advanced when
// a draw happens.  scratch: sample_scratch_bytes(n) bytes, 256-aligned.
size_t sample_scratch_bytes(int n);
cudaError_t launch_sample(const float *logits, int n, float temp, float top_p, unsigned long long *rng, void *scratch,
                          uint32_t *tok, cudaStream_t st);

// First index of the maximum (sampler.rs:26-36); NaNs never win.
// rows > 1: one index per row of x [rows][n] into out_idx[row].
cudaError_t launch_argmax(const float *x, int n, uint32_t *out_idx, cudaStream_t st, int rows = 1);
// Decode feedback on the device, per row r < rows: ids[r] = tok[r]; pos[r] += 1;
// hist[r * hist_stride + step[r]] = tok[r]; step[r] += 1.
cudaError_t launch_advance(const uint32_t *tok, uint32_t *ids, int *pos, uint32_t *hist, int *step, cudaStream_t st,
                           int rows = 1, size_t hist_stride = 0);

// Device address of pk_matmul_noalloc's fixed scratch on the current device
// (pk_noalloc.cu); looked up once per device.
cudaError_t noalloc_scratch(void **ptr);

}  // namespace pk
