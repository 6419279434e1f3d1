// pk_engine.cu -- device engine: GGUF -> HBM, forward pass, decode graphs,
// and Engine::generate with the reference's prefix-KV reuse rules.
//
// Reference: rust/pocketinfer/src/model.rs (Aleinto97/pocket-workbench-android)
//   Config::from_gguf        :32-97      Model::load / finish :487-601
//   KvCache                  :352-387    Scratch (RoPE tables) :408-461
//   forward_inner / layers   :833-1172   generate            :1235-1352
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "pk_engine.h"

namespace pk {

std::atomic<bool> g_stop{false};  // util.rs:274-282 STOP_REQUESTED

#define PK_CK(expr)                                          \
  do {                                                       \
    cudaError_t _e = (expr);                                 \
    if (_e != cudaSuccess) return cuda_error(_e, #expr);     \
  } while (0)

static size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

Engine::~Engine() {
  if (st_) cudaStreamSynchronize(st_);
  release_graphs();
  if (g_streams_) cudaGraphExecDestroy(g_streams_);
  cudaFree(d_weights_);
  cudaFree(d_kcache_);
  cudaFree(d_vcache_);
  cudaFree(d_rope_cos_);
  cudaFree(d_rope_sin_);
  cudaFree(d_act_arena_);
  cudaFree(d_decode_);
  cudaFree(d_rng_);
  cudaFree(d_sample_scratch_);
  cudaFree(d_sk_);
  cudaFree(d_sv_);
  cudaFree(d_slogits_);
  cudaFreeHost(h_ids_);
  cudaFreeHost(h_pos_);
  cudaFreeHost(h_tok_);
  for (int i = 1; i < NLANES; i++) {
    if (lane_[i].st) cudaStreamSynchronize(lane_[i].st);
    cudaFree(d_lane_arena_[i]);
  }
  cudaFreeHost(h_pids_);
  cudaFreeHost(h_ppos_);
  for (auto &v : kv_ev_)
    for (cudaEvent_t e : v) cudaEventDestroy(e);
  if (fork_ev_) cudaEventDestroy(fork_ev_);
  for (cudaEvent_t e : join_ev_)
    if (e) cudaEventDestroy(e);
  for (int i = 1; i < NLANES; i++)
    if (lane_[i].st) cudaStreamDestroy(lane_[i].st);
  if (st_) cudaStreamDestroy(st_);
}

void Engine::release_graphs() {
  if (g_fwd1_) cudaGraphExecDestroy(g_fwd1_);
  if (g_step_) cudaGraphExecDestroy(g_step_);
  g_fwd1_ = g_step_ = nullptr;
}

int Engine::create(int device, int n_ctx, int max_batch) {
  if (n_ctx <= 0 || max_batch <= 0 || max_batch > 64)
    return set_error(PK_ERR_INVALID, "n_ctx must be > 0 and max_batch in 1..64");
  int ndev = 0;
  PK_CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return set_error(PK_ERR_INVALID, "no CUDA device " + std::to_string(device));
  device_ = device;
  n_ctx_ = n_ctx;
  max_batch_ = max_batch;
  if (const char *o = std::getenv("PK_ORDER")) order_ = std::strcmp(o, "fast") == 0 ? PK_ORDER_FAST : PK_ORDER_EXACT;
  PK_CK(cudaSetDevice(device_));
  PK_CK(cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking));
  PK_CK(cudaHostAlloc((void **)&h_ids_, 64 * sizeof(uint32_t), cudaHostAllocDefault));
  PK_CK(cudaHostAlloc((void **)&h_pos_, 64 * sizeof(int), cudaHostAllocDefault));
  PK_CK(cudaHostAlloc((void **)&h_tok_, 4 * sizeof(uint32_t), cudaHostAllocDefault));
  void *scratch = nullptr;  // reserve pk_matmul_noalloc's scratch on this device now (see pk.h)
  if (noalloc_scratch(&scratch) != cudaSuccess) cudaGetLastError();
  return PK_OK;
}

// Config::from_gguf (model.rs:32-97)
int config_from_gguf(const Gguf &g, Config &c) {
  const std::string arch = g.get_str("general.architecture");
  const std::string p = arch.empty() ? "llama" : arch;
  uint64_t v;
  auto need = [&](const char *key, int *out) -> bool {
    if (!g.get_u64(p + "." + key, &v)) return false;
    *out = (int)v;
    return true;
  };
  if (!need("block_count", &c.n_layer)) return set_error(PK_ERR_INVALID, "missing metadata " + p + ".block_count");
  if (!need("embedding_length", &c.n_embd)) return set_error(PK_ERR_INVALID, "missing metadata " + p + ".embedding_length");
  if (!need("feed_forward_length", &c.n_ff)) return set_error(PK_ERR_INVALID, "missing metadata " + p + ".feed_forward_length");
  if (!need("attention.head_count", &c.n_head)) return set_error(PK_ERR_INVALID, "missing metadata " + p + ".attention.head_count");
  if (c.n_layer == 0 || c.n_embd == 0 || c.n_ff == 0 || c.n_head == 0)
    return set_error(PK_ERR_INVALID, "invalid model configuration: zero layer, hidden, FFN or head count");
  c.n_head_kv = g.get_u64(p + ".attention.head_count_kv", &v) ? (int)v : c.n_head;
  c.head_dim = g.get_u64(p + ".attention.key_length", &v) ? (int)v : c.n_embd / c.n_head;
  if (c.head_dim == 0 || c.n_head_kv == 0 || c.n_head % c.n_head_kv != 0)
    return set_error(PK_ERR_INVALID, "invalid GQA configuration");
  if (g.get_u64(p + ".attention.value_length", &v) && (int)v != c.head_dim)
    return set_error(PK_ERR_INVALID, "value head dimension differs from key dimension");
  c.n_rot = g.get_u64(p + ".rope.dimension_count", &v) ? (int)v : c.head_dim;
  float f;
  c.rope_theta = g.get_f32(p + ".rope.freq_base", &f) ? f : 10000.0f;
  c.rms_eps = g.get_f32(p + ".attention.layer_norm_rms_epsilon", &f) ? f : 1e-5f;
  c.n_vocab = g.get_u64(p + ".vocab_size", &v) ? (int)v : 0;
  if (c.n_rot == 0 || c.n_rot > c.head_dim || c.n_rot % 2 != 0 || !std::isfinite(c.rope_theta) || c.rope_theta <= 0.0f ||
      !std::isfinite(c.rms_eps) || c.rms_eps <= 0.0f)
    return set_error(PK_ERR_INVALID, "invalid RoPE / RMSNorm configuration");
  if (c.head_dim > 256 || c.head_dim % 4 != 0)
    return set_error(PK_ERR_UNSUPPORTED, "head_dim must be a multiple of 4 and <= 256 on the device");
  if (c.n_embd % 32 != 0 || c.n_ff % 32 != 0)
    return set_error(PK_ERR_UNSUPPORTED, "hidden and FFN sizes must be multiples of 32 for Q8 activations");
  c.arch = p;
  return PK_OK;
}

// Model::load find (model.rs:494-523)
int find_tensor(const Gguf &g, const std::string &name, TRef &out) {
  const GgufTensor *t = g.tensor(name);
  if (!t) return set_error(PK_ERR_INVALID, "missing tensor " + name);
  int be, bb;
  if (!type_block((int)t->type, &be, &bb)) return set_error(PK_ERR_UNSUPPORTED, "tensor " + name + ": unsupported type");
  if (t->type == 10 || t->type == 11)  // Q2_K / Q3_K
    return set_error(PK_ERR_UNSUPPORTED, "tensor " + name + ": Q2_K/Q3_K are not handled");
  if (t->ne.empty() || t->ne.size() > 2) return set_error(PK_ERR_INVALID, "tensor " + name + ": expected one or two nonzero dimensions");
  for (auto n : t->ne)
    if (n == 0) return set_error(PK_ERR_INVALID, "tensor " + name + ": expected one or two nonzero dimensions");
  if (t->ne[0] % (uint64_t)be != 0) return set_error(PK_ERR_INVALID, "tensor " + name + ": dim0 not divisible by block");
  out.name = name;
  out.type = (int)t->type;
  out.ne0 = (size_t)t->ne[0];
  out.ne1 = t->ne.size() == 2 ? (size_t)t->ne[1] : 1;
  out.row_bytes = out.ne0 / be * bb;
  out.off = g.data_offset() + (size_t)t->offset;
  if (out.off + out.row_bytes * out.ne1 > g.size() || out.off < g.data_offset())
    return set_error(PK_ERR_INVALID, "tensor " + name + ": out of range");
  return PK_OK;
}

int check_shape(const TRef &t, size_t cols, size_t rows) {  // model.rs:650-655
  if (t.ne0 != cols || t.ne1 != rows)
    return set_error(PK_ERR_INVALID, "tensor " + t.name + " has shape " + std::to_string(t.ne0) + "x" +
                                         std::to_string(t.ne1) + ", expected " + std::to_string(cols) + "x" +
                                         std::to_string(rows));
  return PK_OK;
}

int Engine::load(const char *path) {
  if (!st_) return set_error(PK_ERR_INVALID, "engine not created");
  if (loaded_) return set_error(PK_ERR_INVALID, "engine already holds a model");
  PK_CK(cudaSetDevice(device_));
  Gguf g;
  std::string err;
  if (!g.open(path, err)) return set_error(PK_ERR_IO, err);
  int rc = config_from_gguf(g, cfg_);
  if (rc) return rc;
  const Config &c = cfg_;
  TRef embd, output, onorm;
  if ((rc = find_tensor(g, "token_embd.weight", embd))) return rc;
  if (g.tensor("output.weight")) {
    if ((rc = find_tensor(g, "output.weight", output))) return rc;
  } else {
    output = embd;
  }
  if ((rc = find_tensor(g, "output_norm.weight", onorm))) return rc;
  struct LRef { TRef q, k, v, o, an, gate, up, down, fn; };
  std::vector<LRef> L(c.n_layer);
  for (int i = 0; i < c.n_layer; i++) {
    const std::string p = "blk." + std::to_string(i) + ".";
    if ((rc = find_tensor(g, p + "attn_q.weight", L[i].q)) || (rc = find_tensor(g, p + "attn_k.weight", L[i].k)) ||
        (rc = find_tensor(g, p + "attn_v.weight", L[i].v)) || (rc = find_tensor(g, p + "attn_output.weight", L[i].o)) ||
        (rc = find_tensor(g, p + "attn_norm.weight", L[i].an)) || (rc = find_tensor(g, p + "ffn_gate.weight", L[i].gate)) ||
        (rc = find_tensor(g, p + "ffn_up.weight", L[i].up)) || (rc = find_tensor(g, p + "ffn_down.weight", L[i].down)) ||
        (rc = find_tensor(g, p + "ffn_norm.weight", L[i].fn)))
      return rc;
  }
  // Model::finish (model.rs:571-601); without a tokenizer the vocabulary is
  // the embedding's row count.
  vocab_ = (int)embd.ne1;
  if (embd.ne0 != (size_t)c.n_embd || (c.n_vocab != 0 && c.n_vocab != vocab_))
    return set_error(PK_ERR_INVALID, "embedding / metadata / tokenizer vocab dimensions disagree");
  const size_t qdim = (size_t)c.n_head * c.head_dim, kdim = (size_t)c.n_head_kv * c.head_dim;
  if ((rc = check_shape(output, c.n_embd, vocab_)) || (rc = check_shape(onorm, c.n_embd, 1))) return rc;
  for (auto &l : L) {
    if ((rc = check_shape(l.an, c.n_embd, 1)) || (rc = check_shape(l.fn, c.n_embd, 1)) ||
        (rc = check_shape(l.q, c.n_embd, qdim)) || (rc = check_shape(l.k, c.n_embd, kdim)) ||
        (rc = check_shape(l.v, c.n_embd, kdim)) || (rc = check_shape(l.o, qdim, c.n_embd)) ||
        (rc = check_shape(l.gate, c.n_embd, c.n_ff)) || (rc = check_shape(l.up, c.n_embd, c.n_ff)) ||
        (rc = check_shape(l.down, c.n_ff, c.n_embd)))
      return rc;
    for (const TRef *t : {&l.q, &l.k, &l.v, &l.o, &l.gate, &l.up, &l.down})
      if (!type_is_matvec(t->type))
        return set_error(PK_ERR_UNSUPPORTED, "tensor " + t->name + ": the device matvec handles Q4_K/Q6_K/Q4_0/Q8_0");
  }
  if (!type_is_matvec(output.type))
    return set_error(PK_ERR_UNSUPPORTED, "tensor " + output.name + ": the device matvec handles Q4_K/Q6_K/Q4_0/Q8_0");
  if (qdim % 32 != 0) return set_error(PK_ERR_UNSUPPORTED, "n_head * head_dim must be a multiple of 32");

  // ---- device weight arena: packed matrices | f32 norms | raw embedding
  size_t total = 0, max_raw = 0;
  auto mat_bytes = [&](const TRef &t) { return a256(packed_bytes(t.type, (int)t.ne0, (int)t.ne1)); };
  stream_bytes_ = 0;
  for (auto &l : L) {
    for (const TRef *t : {&l.q, &l.k, &l.v, &l.o, &l.gate, &l.up, &l.down}) {
      total += mat_bytes(*t);
      max_raw = std::max(max_raw, t->row_bytes * t->ne1);
      stream_bytes_ += t->row_bytes * t->ne1;
    }
    total += 2 * a256((size_t)c.n_embd * 4);
    max_raw = std::max(max_raw, l.an.row_bytes);
    stream_bytes_ += 2 * (size_t)c.n_embd * 4;
  }
  total += mat_bytes(output) + a256(embd.row_bytes * embd.ne1) + a256((size_t)c.n_embd * 4);
  max_raw = std::max(max_raw, output.row_bytes * output.ne1);
  stream_bytes_ += output.row_bytes * output.ne1 + (size_t)c.n_embd * 4 + embd.row_bytes;
  total += 256;  // the decode kernel's scale copies may read up to 30 bytes past a matrix
  PK_CK(cudaMalloc((void **)&d_weights_, total));
  weight_bytes_ = total;
  uint8_t *staging = nullptr;
  PK_CK(cudaMalloc((void **)&staging, a256(max_raw)));
  size_t off = 0;
  const uint8_t *file = g.data();
  auto upload_mat = [&](const TRef &t, DevTensor &dst) -> int {
    uint8_t *slot = d_weights_ + off;
    off += mat_bytes(t);
    PK_CK(cudaMemcpyAsync(staging, file + t.off, t.row_bytes * t.ne1, cudaMemcpyHostToDevice, st_));
    PK_CK(launch_pack(t.type, staging, t.row_bytes, (int)t.ne0, (int)t.ne1, slot, st_));
    PK_CK(cudaStreamSynchronize(st_));
    dst = packed_view(t.type, (int)t.ne0, (int)t.ne1, slot);
    return PK_OK;
  };
  auto upload_norm = [&](const TRef &t, float **dst) -> int {
    float *slot = (float *)(d_weights_ + off);
    off += a256((size_t)c.n_embd * 4);
    PK_CK(cudaMemcpyAsync(staging, file + t.off, t.row_bytes, cudaMemcpyHostToDevice, st_));
    PK_CK(launch_dequant_rows(t.type, staging, t.row_bytes, (int)t.ne0, nullptr, 1, slot, st_));
    PK_CK(cudaStreamSynchronize(st_));
    *dst = slot;
    return PK_OK;
  };
  layers_.resize(c.n_layer);
  for (int i = 0; i < c.n_layer && !rc; i++) {
    LayerDev &d = layers_[i];
    if ((rc = upload_mat(L[i].q, d.q)) || (rc = upload_mat(L[i].k, d.k)) || (rc = upload_mat(L[i].v, d.v)) ||
        (rc = upload_mat(L[i].o, d.o)) || (rc = upload_mat(L[i].gate, d.gate)) || (rc = upload_mat(L[i].up, d.up)) ||
        (rc = upload_mat(L[i].down, d.down)) || (rc = upload_norm(L[i].an, &d.attn_norm)) ||
        (rc = upload_norm(L[i].fn, &d.ffn_norm)))
      break;
  }
  if (!rc) {
    if (!(rc = upload_mat(output, output_))) rc = upload_norm(onorm, &output_norm_);
  }
  cudaFree(staging);
  if (rc) return rc;
  embd_raw_ = d_weights_ + off;
  PK_CK(cudaMemcpyAsync((void *)embd_raw_, file + embd.off, embd.row_bytes * embd.ne1, cudaMemcpyHostToDevice, st_));
  off += a256(embd.row_bytes * embd.ne1);
  embd_type_ = embd.type;
  embd_row_bytes_ = embd.row_bytes;

  // ---- KV cache (model.rs:352-387), f32: V as the reference lays it out,
  // [layer][kv_head][n_ctx][dh]; K d-major, [layer][kv_head][dh][n_ctx], so a
  // run of positions of one dimension is contiguous for the score pass.
  kv_bytes_ = 2 * (size_t)c.n_layer * c.n_head_kv * n_ctx_ * c.head_dim * (kv_f16_ ? 2 : 4);
  PK_CK(cudaMalloc((void **)&d_kcache_, kv_bytes_ / 2));
  PK_CK(cudaMalloc((void **)&d_vcache_, kv_bytes_ / 2));
  PK_CK(cudaMemsetAsync(d_kcache_, 0, kv_bytes_ / 2, st_));
  PK_CK(cudaMemsetAsync(d_vcache_, 0, kv_bytes_ / 2, st_));

  // ---- RoPE tables, computed exactly like Scratch::new / ensure_rope
  // (model.rs:414-417, 452-457) with the C library's powf/cosf/sinf.
  const int half = c.n_rot / 2;
  std::vector<float> inv(std::max(half, 1)), tc((size_t)n_ctx_ * half), ts((size_t)n_ctx_ * half);
  for (int i = 0; i < half; i++) inv[i] = 1.0f / powf(c.rope_theta, 2.0f * (float)i / (float)c.n_rot);
  for (int p = 0; p < n_ctx_; p++)
    for (int i = 0; i < half; i++) {
      const float a = (float)p * inv[i];
      tc[(size_t)p * half + i] = cosf(a);
      ts[(size_t)p * half + i] = sinf(a);
    }
  PK_CK(cudaMalloc((void **)&d_rope_cos_, std::max<size_t>(tc.size(), 1) * 4));
  PK_CK(cudaMalloc((void **)&d_rope_sin_, std::max<size_t>(ts.size(), 1) * 4));
  PK_CK(cudaMemcpyAsync(d_rope_cos_, tc.data(), tc.size() * 4, cudaMemcpyHostToDevice, st_));
  PK_CK(cudaMemcpyAsync(d_rope_sin_, ts.data(), ts.size() * 4, cudaMemcpyHostToDevice, st_));

  // ---- activations and scratch (one arena)
  const size_t B = max_batch_, ne = c.n_embd, ff = c.n_ff;
  const size_t kmax = std::max(std::max(ne, ff), qdim);
  const size_t H = c.n_head, dh = c.head_dim;
  const std::vector<size_t> sizes = {
      B * ne * 4, B * qdim * 4, B * kdim * 4, B * kdim * 4, B * qdim * 4,  // x q k v attn
      B * ff * 4, B * ff * 4, B * ff * 4, (size_t)vocab_ * 4,            // gate up h logits
      B * kmax, B * (kmax / 32) * 4, B * (kmax / 32) * 4,                  // act q d s
      B * H * n_ctx_ * 4,                                                  // attention scores
      64 * 4, 64 * 4, 16, (size_t)n_ctx_ * 4 + 16, 16};                 // ids pos tok hist step
  size_t arena = 0;
  for (size_t s : sizes) arena += a256(s);
  PK_CK(cudaMalloc((void **)&d_act_arena_, arena));
  PK_CK(cudaMemsetAsync(d_act_arena_, 0, arena, st_));
  uint8_t *pa = d_act_arena_;
  size_t si = 0;
  auto take = [&]() {
    uint8_t *r = pa;
    pa += a256(sizes[si++]);
    return r;
  };
  x_ = (float *)take(); q_ = (float *)take(); k_ = (float *)take(); v_ = (float *)take(); attn_ = (float *)take();
  gate_ = (float *)take(); up_ = (float *)take(); h_ = (float *)take(); logits_ = (float *)take();
  act_.q = (int8_t *)take(); act_.d = (float *)take(); act_.s = (int32_t *)take();
  att_scores_ = (float *)take();
  d_ids_ = (uint32_t *)take(); d_pos_ = (int *)take(); d_tok_ = (uint32_t *)take(); d_hist_ = (uint32_t *)take();
  d_step_ = (int *)take();

  // prefill lanes (lanes 1.. : their own per-chunk scratch and stream)
  lane_[0].st = st_;
  lane_[0].x = x_; lane_[0].q = q_; lane_[0].k = k_; lane_[0].v = v_; lane_[0].attn = attn_;
  lane_[0].gate = gate_; lane_[0].up = up_; lane_[0].h = h_; lane_[0].scores = att_scores_;
  lane_[0].act = act_; lane_[0].ids = d_ids_; lane_[0].pos = d_pos_;
  {
    const std::vector<size_t> s1 = {B * ne * 4, B * qdim * 4, B * kdim * 4, B * kdim * 4, B * qdim * 4,
                                    B * ff * 4, B * ff * 4, B * ff * 4, B * kmax, B * (kmax / 32) * 4,
                                    B * (kmax / 32) * 4, B * H * n_ctx_ * 4, 64 * 4, 64 * 4};
    size_t a1 = 0;
    for (size_t v : s1) a1 += a256(v);
    for (int li = 1; li < NLANES; li++) {
      PK_CK(cudaMalloc((void **)&d_lane_arena_[li], a1));
      PK_CK(cudaMemsetAsync(d_lane_arena_[li], 0, a1, st_));
      uint8_t *p1 = d_lane_arena_[li];
      size_t i1 = 0;
      auto take1 = [&]() {
        uint8_t *r = p1;
        p1 += a256(s1[i1++]);
        return r;
      };
      Lane &L = lane_[li];
      L.x = (float *)take1(); L.q = (float *)take1(); L.k = (float *)take1(); L.v = (float *)take1();
      L.attn = (float *)take1(); L.gate = (float *)take1(); L.up = (float *)take1(); L.h = (float *)take1();
      L.act = act_;
      L.act.q = (int8_t *)take1(); L.act.d = (float *)take1(); L.act.s = (int32_t *)take1();
      L.scores = (float *)take1(); L.ids = (uint32_t *)take1(); L.pos = (int *)take1();
      PK_CK(cudaStreamCreateWithFlags(&L.st, cudaStreamNonBlocking));
    }
    for (auto &v : kv_ev_) {
      v.resize(c.n_layer);
      for (auto &e : v) PK_CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    PK_CK(cudaEventCreateWithFlags(&fork_ev_, cudaEventDisableTiming));
    for (auto &e : join_ev_) PK_CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    PK_CK(cudaHostAlloc((void **)&h_pids_, (size_t)n_ctx_ * sizeof(uint32_t), cudaHostAllocDefault));
    PK_CK(cudaHostAlloc((void **)&h_ppos_, (size_t)n_ctx_ * sizeof(int), cudaHostAllocDefault));
  }

  // Tokenizer::from_gguf end-of-generation ids (tokenizer.rs:82-92)
  uint64_t eos;
  if (g.get_u64("tokenizer.ggml.eos_token_id", &eos)) eos_ids_.push_back((uint32_t)eos);
  if (const GgufValue *tv = g.get("tokenizer.ggml.tokens"))
    for (size_t i = 0; i < tv->arr_str.size(); i++) {
      const std::string &s = tv->arr_str[i];
      if (s == "<|im_end|>" || s == "<|eot|>" || s == "<|endoftext|>") eos_ids_.push_back((uint32_t)i);
    }
  std::sort(eos_ids_.begin(), eos_ids_.end());
  eos_ids_.erase(std::unique(eos_ids_.begin(), eos_ids_.end()), eos_ids_.end());
  PK_CK(cudaStreamSynchronize(st_));
  loaded_ = true;
  return setup_decode();
}

// Plan and device tables of the persistent decode kernel.  A model it cannot
// run (shared memory, shapes) keeps the per-op kernel sequence; the
// environment variable PK_DECODE=ops selects that sequence as well.
int Engine::setup_decode() {
  use_decode_ = false;
  const char *env = std::getenv("PK_DECODE");
  if (env && std::strcmp(env, "ops") == 0) {
    decode_why_ = "PK_DECODE=ops";
    return PK_OK;
  }
  if (kv_f16_) {
    decode_why_ = "f16 KV cache: decode runs the per-op kernels";
    return PK_OK;
  }
  const Config &c = cfg_;
  std::vector<DecLayer> dl(c.n_layer);
  for (int i = 0; i < c.n_layer; i++) {
    const LayerDev &L = layers_[i];
    dl[i] = DecLayer{L.q, L.k, L.v, L.o, L.gate, L.up, L.down, L.attn_norm, L.ffn_norm};
  }
  const int grid = decode_grid_for(dl, output_, decode_grid());
  if (!build_decode_plan(dl, output_, c.n_embd, c.n_ff, c.n_head, c.n_head_kv, c.head_dim, n_ctx_, grid, plan_,
                         decode_why_))
    return PK_OK;
  // Every bulk copy must stay inside the weight arena.
  const uintptr_t lo = (uintptr_t)d_weights_, hi = lo + weight_bytes_;
  for (const DChunk &k : plan_.chunks) {
    const size_t nq = k.full ? 1 : k.rows, qlen = k.q_len;
    const uintptr_t q0 = (uintptr_t)k.q, q1 = q0 + (nq - 1) * (size_t)k.q_stride + qlen;
    bool ok = (q0 & 15) == 0 && (qlen & 15) == 0 && q0 >= lo && q1 <= hi && (k.d_off & 15) == 0;
    size_t tx = k.full ? qlen : (size_t)k.rows * qlen;
    if (k.d) {
      const uintptr_t d0 = (uintptr_t)k.d & ~(uintptr_t)15;
      const uintptr_t d1 = k.full ? d0 + k.d_len : (((uintptr_t)k.d + (k.rows - 1) * (size_t)k.d_stride) & ~(uintptr_t)15) + k.d_len;
      ok = ok && d0 >= lo && d1 <= hi && (k.d_len & 15) == 0;
      tx += k.full ? k.d_len : (size_t)k.rows * k.d_len;
    }
    ok = ok && tx <= (size_t)DK_SLOT && k.rows >= 1 && k.rows <= DK_MAX_RG;
    if (!ok) {
      decode_why_ = "decode plan failed its bounds check";
      return PK_OK;
    }
  }
  if (prepare_decode(plan_.smem, plan_.grid) != cudaSuccess) {
    cudaGetLastError();
    decode_why_ = "the persistent kernel's grid does not fit the device at once";
    return PK_OK;
  }
  const int n_trace = 1 + DK_TRW * (5 * c.n_layer + 1) + c.n_layer + 1 + 4;  // + SM cycles / ns at start and end
  const size_t n_ch = plan_.chunks.size() * sizeof(DChunk), n_c0 = plan_.cta_chunk0.size() * 4,
               n_ph = plan_.phase0.size() * 4, n_own = plan_.own.size() * 4, n_ly = dl.size() * sizeof(DecLayer),
               n_cw = plan_.cwbits.size() * 4,
               n_tr = (size_t)grid * n_trace * 8;
  const size_t qdim = (size_t)c.n_head * c.head_dim, kdim = (size_t)c.n_head_kv * c.head_dim;
  const std::vector<size_t> sizes = {n_ch, n_c0, n_ph, n_own, n_ly, 16, 16, (size_t)grid * 4, (size_t)grid * 4, n_tr, n_cw,
                                     2 * (size_t)c.n_embd * 8, qdim * 8, (size_t)c.n_ff * 8, qdim * 8, 2 * kdim * 8,
                                     (size_t)c.n_head * n_ctx_ * 8};
  size_t total = 0;
  for (size_t z : sizes) total += a256(z);
  PK_CK(cudaMalloc((void **)&d_decode_, total));
  PK_CK(cudaMemsetAsync(d_decode_, 0, total, st_));
  uint8_t *p = d_decode_;
  size_t si = 0;
  auto take = [&]() {
    uint8_t *r = p;
    p += a256(sizes[si++]);
    return r;
  };
  DChunk *chunks = (DChunk *)take();
  int *c0 = (int *)take(), *ph = (int *)take(), *own = (int *)take();
  DecLayer *layers = (DecLayer *)take();
  d_sync_ = (unsigned *)take();
  d_err_ = (int *)take();
  float *cv = (float *)take();
  int *ci = (int *)take();
  d_trace_ = (unsigned long long *)take();
  uint32_t *cwb = (uint32_t *)take();
  unsigned long long *x_ll = (unsigned long long *)take(), *att_ll = (unsigned long long *)take(),
                     *h_ll = (unsigned long long *)take(), *q_ll = (unsigned long long *)take(),
                     *kv_ll = (unsigned long long *)take(), *sc_ll = (unsigned long long *)take();
  PK_CK(cudaMemcpyAsync(chunks, plan_.chunks.data(), n_ch, cudaMemcpyHostToDevice, st_));
  PK_CK(cudaMemcpyAsync(c0, plan_.cta_chunk0.data(), n_c0, cudaMemcpyHostToDevice, st_));
  PK_CK(cudaMemcpyAsync(ph, plan_.phase0.data(), n_ph, cudaMemcpyHostToDevice, st_));
  PK_CK(cudaMemcpyAsync(own, plan_.own.data(), n_own, cudaMemcpyHostToDevice, st_));
  PK_CK(cudaMemcpyAsync(layers, dl.data(), n_ly, cudaMemcpyHostToDevice, st_));
  PK_CK(cudaMemcpyAsync(cwb, plan_.cwbits.data(), n_cw, cudaMemcpyHostToDevice, st_));
  const unsigned epoch0 = 1;  // tags of zeroed words (epoch 0) never match
  PK_CK(cudaMemcpyAsync(d_sync_ + 2, &epoch0, 4, cudaMemcpyHostToDevice, st_));
  PK_CK(cudaStreamSynchronize(st_));
  DecodeArgs &a = dargs_;
  a = DecodeArgs{};
  a.layers = layers;
  a.out = output_;
  a.out_norm = output_norm_;
  a.embd = embd_raw_;
  a.embd_row_bytes = (uint32_t)embd_row_bytes_;
  a.embd_type = embd_type_;
  a.n_layer = c.n_layer; a.n_embd = c.n_embd; a.n_ff = c.n_ff; a.n_head = c.n_head; a.n_kv = c.n_head_kv;
  a.dh = c.head_dim; a.half = c.n_rot / 2; a.n_ctx = n_ctx_; a.n_vocab = vocab_;
  a.eps = c.rms_eps;
  a.scale = 1.0f / sqrtf((float)c.head_dim);
  a.rope_cos = d_rope_cos_; a.rope_sin = d_rope_sin_;
  a.kcache = d_kcache_; a.vcache = d_vcache_;
  a.att_j = plan_.att_j;
  a.att_ds = c.head_dim / plan_.att_j;
  if (make_vcache_map(&a.vmap, d_vcache_, c.n_layer, c.n_head_kv, n_ctx_, c.head_dim, a.att_ds, decode_why_)) return PK_OK;
  a.logits = logits_;
  a.x_ll = x_ll; a.att_ll = att_ll; a.h_ll = h_ll; a.q_ll = q_ll; a.kv_ll = kv_ll; a.sc_ll = sc_ll;
  a.ids = d_ids_; a.tok = d_tok_; a.hist = d_hist_; a.pos = d_pos_; a.step = d_step_;
  a.chunks = chunks; a.cta_chunk0 = c0; a.phase0 = ph; a.n_phase = plan_.n_phase; a.own = own; a.cwbits = cwb;
  a.sync = d_sync_; a.err = d_err_; a.cand_v = cv; a.cand_i = ci;
  a.mode = 0;
  a.fast = order_ == PK_ORDER_FAST ? 1 : 0;
  a.trace = nullptr;
  a.n_trace = n_trace;
  use_decode_ = true;
  return PK_OK;
}

// After a persistent-kernel launch: a bounded wait that ran out leaves an
// error code.  The finish counter is reset and the tag epoch advanced (the
// stopped launch did not advance it), so words that launch left behind can
// never match the next launch's tags.
// After b > 1 work: the tensor-core matvec's error word (a bounded wait in
// one of its CTAs ran out), read and cleared.
int Engine::check_tc_error() {
  const int t = mv_tc_error(true);
  if (t == PK_ERR_TIMEOUT) return set_error(PK_ERR_TIMEOUT, "a tensor-core matvec's bounded wait ran out");
  if (t) return set_error(t, "reading the tensor-core matvec's error word");
  return PK_OK;
}

int Engine::check_decode_error() {
  if (!use_decode_) return PK_OK;
  int err = 0;
  PK_CK(cudaMemcpyAsync(&err, d_err_, 4, cudaMemcpyDeviceToHost, st_));
  PK_CK(cudaStreamSynchronize(st_));
  if (err == 0) return PK_OK;
  unsigned sync[4] = {0, 0, 0, 0};
  PK_CK(cudaMemcpyAsync(sync, d_sync_, 16, cudaMemcpyDeviceToHost, st_));
  PK_CK(cudaStreamSynchronize(st_));
  sync[0] = 0;
  sync[1] = 0;
  sync[2] = sync[2] + 1 > (1u << 22) - 1 ? 1 : sync[2] + 1;
  PK_CK(cudaMemsetAsync(d_err_, 0, 4, st_));
  PK_CK(cudaMemcpyAsync(d_sync_, sync, 16, cudaMemcpyHostToDevice, st_));
  PK_CK(cudaStreamSynchronize(st_));
  return set_error(err, "decode kernel: a bounded wait ran out (a phase input or a copy did not arrive)");
}

int Engine::info(pk_model_info *o) const {
  if (!loaded_) return set_error(PK_ERR_INVALID, "no model loaded");
  o->n_layer = cfg_.n_layer; o->n_embd = cfg_.n_embd; o->n_ff = cfg_.n_ff; o->n_head = cfg_.n_head;
  o->n_head_kv = cfg_.n_head_kv; o->head_dim = cfg_.head_dim; o->n_rot = cfg_.n_rot; o->n_vocab = vocab_;
  o->n_ctx = n_ctx_; o->rope_theta = cfg_.rope_theta; o->rms_eps = cfg_.rms_eps;
  o->weight_bytes = weight_bytes_; o->kv_bytes = kv_bytes_; o->stream_bytes = stream_bytes_;
  o->decode_kernels = use_decode_ ? 1 : 3 + 5 * cfg_.n_layer + 1;
  return PK_OK;
}

void Engine::dump(const char *name, const float *dev, size_t n) {
  if (!dbg_on_) return;
  std::vector<float> h(n);
  cudaStreamSynchronize(st_);
  cudaMemcpyAsync(h.data(), dev, n * 4, cudaMemcpyDeviceToHost, st_);
  dbg_.emplace_back(name, std::move(h));
}

int Engine::prof_begin(const char *name, double bytes) {
  if (!prof_) return PK_OK;
  ProfMark m{name, bytes, nullptr, nullptr};
  PK_CK(cudaEventCreate(&m.start));
  PK_CK(cudaEventCreate(&m.stop));
  PK_CK(cudaEventRecord(m.start, st_));
  prof_->push_back(m);
  return PK_OK;
}

int Engine::prof_end() {
  if (!prof_) return PK_OK;
  PK_CK(cudaEventRecord(prof_->back().stop, st_));
  return PK_OK;
}

// Bytes of a matrix in the GGUF block layout (the algorithmic weight stream).
static double mat_stream_bytes(const DevTensor &w) {
  int be = 1, bb = 1;
  type_block(w.type, &be, &bb);
  return (double)w.rows * (double)(w.k / be) * (double)bb;
}

#define PROF(name, bytes, launch)                 \
  do {                                            \
    int _rc = prof_begin(name, (double)(bytes));  \
    if (_rc) return _rc;                          \
    PK_CK(launch);                                \
    if ((_rc = prof_end())) return _rc;           \
  } while (0)

// The per-token kernel sequence (model.rs:857-1170) on prefill lane li.
// Reads ids/positions from the lane's device buffers, so a b == 1 pass
// (lane 0) can be captured once as a CUDA graph.  kv & KV_RECORD: record
// kv_ev_[li][l] once layer l's K/V are written; kv & KV_WAIT: layer l's
// attention first waits for the previous lane's kv_ev_ of layer l.
int Engine::enqueue_forward(int b, bool want_logits, bool cancellable, int li, int kv) {
  const Lane &S = lane_[li];
  const Config &c = cfg_;
  const int ne = c.n_embd, dh = c.head_dim, qdim = c.n_head * dh, kdim = c.n_head_kv * dh, ff = c.n_ff;
  const size_t layer_kv = (size_t)c.n_head_kv * n_ctx_ * dh;
  const double f4 = 4.0, kv_pos = (double)next_pos_ + 1.0;  // positions attended in a profiled decode step
  PROF("k_dequant_rows", embd_row_bytes_ + ne * f4,
       launch_dequant_rows(embd_type_, embd_raw_, embd_row_bytes_, ne, S.ids, b, S.x, S.st));
  dump("embd", S.x, (size_t)b * ne);
  AttnArgs at{};
  at.q = S.q; at.pos = S.pos; at.out = S.attn; at.b = b; at.n_head = c.n_head; at.n_kv = c.n_head_kv; at.dh = dh;
  at.n_ctx = n_ctx_; at.scale = 1.0f / sqrtf((float)dh);
  at.scores = S.scores;
  for (int l = 0; l < c.n_layer; l++) {
    if (cancellable && g_stop.load()) return set_error(PK_ERR_STOPPED, "generation stopped");
    const LayerDev &L = layers_[l];
    float *kc = kv_at(d_kcache_, l * layer_kv), *vc = kv_at(d_vcache_, l * layer_kv);
    at.kcache = kc; at.vcache = vc; at.kv16 = kv_f16_ ? 1 : 0;
    if (b == 1) {
      QkvArgs qa;
      qa.wq = L.q; qa.wk = L.k; qa.wv = L.v;
      qa.src.x = S.x; qa.src.nw = L.attn_norm; qa.src.eps = c.rms_eps;
      qa.pos = S.pos; qa.rope_cos = d_rope_cos_; qa.rope_sin = d_rope_sin_;
      qa.half = c.n_rot / 2; qa.dh = dh; qa.n_ctx = n_ctx_;
      qa.qout = S.q; qa.kcache = kc; qa.vcache = vc; qa.kv16 = kv_f16_ ? 1 : 0;
      PROF("k_qkv_b1", mat_stream_bytes(L.q) + mat_stream_bytes(L.k) + mat_stream_bytes(L.v) + 2 * ne * f4 +
                           (qdim + 2 * kdim) * f4,
           launch_qkv_b1(qa, S.st));
      if (l == 0) dump("Qrope-0", S.q, (size_t)qdim);
      if (kv & KV_RECORD) PK_CK(cudaEventRecord(kv_ev_[li][l], S.st));
      if (kv & KV_WAIT) PK_CK(cudaStreamWaitEvent(S.st, kv_ev_[(li + NLANES - 1) % NLANES][l], 0));
      PROF("k_attn", 2.0 * c.n_head_kv * kv_pos * dh * f4 + 2 * qdim * f4, launch_attention(at, S.st));
      B1Src so;
      so.x = S.attn;
      PROF("k_mv_b1", mat_stream_bytes(L.o) + qdim * f4 + 2 * ne * f4, launch_mv_b1(L.o, so, S.x, true, S.st));
      if (l == 0) dump("ffn_inp-0", S.x, (size_t)ne);
      B1Src sf;
      sf.x = S.x; sf.nw = L.ffn_norm; sf.eps = c.rms_eps;
      PROF("k_gateup_b1", mat_stream_bytes(L.gate) + mat_stream_bytes(L.up) + 2 * ne * f4 + ff * f4,
           launch_gateup_b1(L.gate, L.up, sf, S.h, S.st));
      B1Src sd;
      sd.x = S.h;
      PROF("k_mv_b1", mat_stream_bytes(L.down) + ff * f4 + 2 * ne * f4, launch_mv_b1(L.down, sd, S.x, true, S.st));
    } else {
      const cudaStream_t st = S.st;
      Q8Dev a = S.act;
      a.k = ne; a.b = b;
      PK_CK(launch_rmsnorm_q8(S.x, L.attn_norm, c.rms_eps, ne, b, a, nullptr, st));
      const MvOut qkv[3] = {{L.q, S.q, 1, qdim, false}, {L.k, S.k, 1, kdim, false}, {L.v, S.v, 1, kdim, false}};
      PK_CK(launch_mv_multi(3, qkv, a, st));
      if (l == 0) { dump("Qcur-0", S.q, (size_t)b * qdim); dump("Kcur-0", S.k, (size_t)b * kdim); dump("Vcur-0", S.v, (size_t)b * kdim); }
      PK_CK(launch_rope_kv(S.q, S.k, S.v, b, S.pos, d_rope_cos_, d_rope_sin_, c.n_rot / 2, dh, c.n_head, c.n_head_kv,
                           n_ctx_, kc, vc, st, 0, kv_f16_));
      if (kv & KV_RECORD) PK_CK(cudaEventRecord(kv_ev_[li][l], st));
      if (l == 0) dump("Qrope-0", S.q, (size_t)b * qdim);
      if (kv & KV_WAIT) PK_CK(cudaStreamWaitEvent(st, kv_ev_[(li + NLANES - 1) % NLANES][l], 0));
      a.k = qdim;
      AttnArgs atq = at;
      atq.q8 = a;  // the attention kernel also writes Q8 of its output
      PK_CK(launch_attention(atq, st));
      PK_CK(launch_mv_lanes(L.o, a, S.x, 1, ne, true, st));
      if (l == 0) dump("ffn_inp-0", S.x, (size_t)b * ne);
      a.k = ne;
      PK_CK(launch_rmsnorm_q8(S.x, L.ffn_norm, c.rms_eps, ne, b, a, nullptr, st));
      const MvOut gu[2] = {{L.gate, S.gate, 1, ff, false}, {L.up, S.up, 1, ff, false}};
      PK_CK(launch_mv_multi(2, gu, a, st));
      a.k = ff;
      PK_CK(launch_swiglu_q8(S.gate, S.up, ff, b, a, S.h, st));
      PK_CK(launch_mv_lanes(L.down, a, S.x, 1, ne, true, st));
    }
    if (l == 0) {
      dump("kqv_out-0", S.attn, (size_t)b * qdim);
      dump("ffn_swiglu-0", S.h, (size_t)b * ff);
      dump("l_out-0", S.x, (size_t)b * ne);
    }
  }
  if (want_logits) {
    if (cancellable && g_stop.load()) return set_error(PK_ERR_STOPPED, "generation stopped");
    B1Src sh;
    sh.x = S.x + (size_t)(b - 1) * ne; sh.nw = output_norm_; sh.eps = c.rms_eps;
    PROF("k_mv_b1", mat_stream_bytes(output_) + 2 * ne * f4 + (double)vocab_ * f4,
         launch_mv_b1(output_, sh, logits_, false, S.st));
    dump("result_output", logits_, (size_t)vocab_);
  }
  return PK_OK;
}

int Engine::ensure_graphs() {
  if (g_fwd1_ && g_step_) return PK_OK;
  release_graphs();
  for (int which = 0; which < 2; which++) {
    cudaGraph_t graph = nullptr;
    PK_CK(cudaStreamBeginCapture(st_, cudaStreamCaptureModeThreadLocal));
    int rc = PK_OK;
    cudaError_t e = cudaSuccess;
    if (use_decode_) {
      DecodeArgs a = dargs_;
      a.mode = which;  // the step graph also picks the next token and feeds it back
      e = launch_decode(a, plan_.grid, plan_.smem, st_);
    } else {
      if (which == 1) {
        e = launch_argmax(logits_, vocab_, d_tok_, st_);
        if (e == cudaSuccess) e = launch_advance(d_tok_, d_ids_, d_pos_, d_hist_, d_step_, st_);
      }
      if (e == cudaSuccess) rc = enqueue_forward(1, true, false);
    }
    cudaError_t ee = cudaStreamEndCapture(st_, &graph);
    if (e != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      return cuda_error(e, "decode graph capture");
    }
    if (rc) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    if (ee != cudaSuccess) return cuda_error(ee, "cudaStreamEndCapture");
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_error(e, "cudaGraphInstantiate");
    (which == 0 ? g_fwd1_ : g_step_) = exec;
  }
  return PK_OK;
}

// forward_inner (model.rs:833-902)
int Engine::forward_inner(const uint32_t *ids, const int *pos, int b, bool want_logits, bool cancellable) {
  if (!loaded_) return set_error(PK_ERR_INVALID, "no model loaded");
  if (b <= 0 || b > max_batch_) return set_error(PK_ERR_INVALID, "invalid batch " + std::to_string(b));
  for (int i = 0; i < b; i++) {
    if (pos[i] < 0 || pos[i] >= n_ctx_) return set_error(PK_ERR_CONTEXT_FULL, "context full");
    if (ids[i] >= (uint32_t)vocab_) return set_error(PK_ERR_INVALID, "token " + std::to_string(ids[i]) + " out of vocab");
  }
  PK_CK(cudaSetDevice(device_));
  std::memcpy(h_ids_, ids, b * sizeof(uint32_t));
  std::memcpy(h_pos_, pos, b * sizeof(int));
  PK_CK(cudaMemcpyAsync(d_ids_, h_ids_, b * sizeof(uint32_t), cudaMemcpyHostToDevice, st_));
  PK_CK(cudaMemcpyAsync(d_pos_, h_pos_, b * sizeof(int), cudaMemcpyHostToDevice, st_));
  have_logits_ = false;
  if (b == 1 && want_logits && !dbg_on_) {
    int rc = ensure_graphs();
    if (rc) return rc;
    PK_CK(cudaGraphLaunch(g_fwd1_, st_));
  } else {
    int rc = enqueue_forward(b, want_logits, cancellable);
    if (rc) {
      cudaStreamSynchronize(st_);
      return rc;
    }
  }
  PK_CK(cudaStreamSynchronize(st_));
  PK_CK(cudaGetLastError());
  if (b == 1 && want_logits && !dbg_on_) {
    const int rc = check_decode_error();
    if (rc) return rc;
  }
  if (b > 1) {
    const int rc = check_tc_error();
    if (rc) return rc;
  }
  next_pos_ = pos[b - 1] + 1;
  have_logits_ = want_logits;
  return PK_OK;
}

int Engine::forward(const uint32_t *ids, const int *pos, int n, bool want_logits) {  // model.rs:825-831
  kv_tokens_.clear();
  cached_prefill_len_ = 0;
  dbg_.clear();
  return forward_inner(ids, pos, n, want_logits, false);
}

int Engine::logits(float *out, int n) {
  if (!loaded_) return set_error(PK_ERR_INVALID, "no model loaded");
  const int m = std::min(n, vocab_);
  PK_CK(cudaMemcpyAsync(out, logits_, (size_t)m * 4, cudaMemcpyDeviceToHost, st_));
  PK_CK(cudaStreamSynchronize(st_));
  return PK_OK;
}

int Engine::argmax(uint32_t *tok) {
  if (!loaded_) return set_error(PK_ERR_INVALID, "no model loaded");
  PK_CK(launch_argmax(logits_, vocab_, d_tok_, st_));
  PK_CK(cudaMemcpyAsync(h_tok_, d_tok_, 4, cudaMemcpyDeviceToHost, st_));
  PK_CK(cudaStreamSynchronize(st_));
  *tok = h_tok_[0];
  return PK_OK;
}

// sampler.rs:21-92 with temp > 0 on the current logits (the device Rng
// state advances when a draw happens).
int Engine::sample(float temp, float top_p, uint32_t *tok) {
  if (!loaded_ || !d_rng_) return set_error(PK_ERR_INVALID, "no model loaded or no sampler state");
  PK_CK(launch_sample(logits_, vocab_, temp, top_p, d_rng_, d_sample_scratch_, d_tok_, st_));
  PK_CK(cudaMemcpyAsync(h_tok_, d_tok_, 4, cudaMemcpyDeviceToHost, st_));
  PK_CK(cudaStreamSynchronize(st_));
  *tok = h_tok_[0];
  return PK_OK;
}

// The prompt's chunks [off, n) (chunk tokens each) on the prefill lanes in
// turn: chunk c + 1 runs its layer l while chunk c is still in later layers,
// waiting only for chunk c's K/V of layer l before its attention.
// Every kernel sees the same inputs as in chunk order, so the results are
// the same bits.  Returns with both lanes idle.
int Engine::prefill_lanes(const uint32_t *prompt, int n, int off, int chunk, bool *stopped) {
  if (n > n_ctx_) return set_error(PK_ERR_CONTEXT_FULL, "context full");
  for (int i = off; i < n; i++)
    if (prompt[i] >= (uint32_t)vocab_) return set_error(PK_ERR_INVALID, "token " + std::to_string(prompt[i]) + " out of vocab");
  PK_CK(cudaSetDevice(device_));
  for (int i = off; i < n; i++) {
    h_pids_[i] = prompt[i];
    h_ppos_[i] = i;
  }
  have_logits_ = false;
  PK_CK(cudaEventRecord(fork_ev_, st_));
  for (int i = 1; i < NLANES; i++) PK_CK(cudaStreamWaitEvent(lane_[i].st, fork_ev_, 0));
  int rc = PK_OK;
  cudaError_t e = cudaSuccess;
  for (int o = off, c = 0; o < n; o += chunk, c++) {
    if (g_stop.load()) {
      *stopped = true;
      break;
    }
    const int m = std::min(chunk, n - o), li = c % NLANES;
    const Lane &L = lane_[li];
    e = cudaMemcpyAsync(L.ids, h_pids_ + o, m * sizeof(uint32_t), cudaMemcpyHostToDevice, L.st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(L.pos, h_ppos_ + o, m * sizeof(int), cudaMemcpyHostToDevice, L.st);
    if (e != cudaSuccess) break;
    if ((rc = enqueue_forward(m, o + m >= n, true, li, KV_RECORD | (c > 0 ? KV_WAIT : 0)))) break;
  }
  // the other lanes join lane 0, then all are drained
  cudaError_t ej = cudaSuccess;
  for (int i = 1; i < NLANES; i++) {
    if (ej == cudaSuccess) ej = cudaEventRecord(join_ev_[i], lane_[i].st);
    if (ej == cudaSuccess) ej = cudaStreamWaitEvent(st_, join_ev_[i], 0);
  }
  const cudaError_t es = cudaStreamSynchronize(st_);
  for (int i = 1; i < NLANES; i++) cudaStreamSynchronize(lane_[i].st);
  if (rc) return rc;
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyAsync (prefill ids)");
  if (ej != cudaSuccess) return cuda_error(ej, "prefill lane join");
  if (es != cudaSuccess) return cuda_error(es, "prefill");
  PK_CK(cudaGetLastError());
  if ((rc = check_tc_error())) return rc;
  if (*stopped) return PK_OK;
  next_pos_ = n;
  have_logits_ = true;
  return PK_OK;
}

// Engine::generate (model.rs:1235-1352).  The device engine is this
// process's only engine, so prefix reuse follows the reference's CPU rules
// (cpu_only == true): full 32-token prefill chunks of an exactly matching
// prefix are reused, decode tokens never are.
int Engine::generate(const uint32_t *prompt, int n, const pk_gen_opts &opts, pk_token_cb cb, void *user,
                     uint32_t *out_ids, int out_cap, int *n_out, pk_gen_stats *stats) {
  pk_gen_stats s;
  std::memset(&s, 0, sizeof(s));
  std::snprintf(s.stop, sizeof(s.stop), "max_tokens");
  int nout = 0;
  auto finish = [&](int rc) {
    if (stats) *stats = s;
    if (n_out) *n_out = nout;
    return rc;
  };
  if (!loaded_) return finish(set_error(PK_ERR_INVALID, "no model loaded"));
  if (n <= 0) return finish(set_error(PK_ERR_INVALID, "empty prompt"));
  const bool sampling = opts.temp > 0.0f;
  if (sampling) {  // Rng::new(seed) (sampler.rs:6-8) for this call, on the device
    if (!d_rng_) {
      PK_CK(cudaMalloc((void **)&d_rng_, 256));
      PK_CK(cudaMalloc((void **)&d_sample_scratch_, sample_scratch_bytes(vocab_)));
    }
    h_rng_ = opts.seed + 0x9E3779B97F4A7C15ULL;
    PK_CK(cudaMemcpyAsync(d_rng_, &h_rng_, 8, cudaMemcpyHostToDevice, st_));
  }
  const auto t0 = std::chrono::steady_clock::now();
  const int chunk = std::min(max_batch_, 32);
  size_t common = 0;
  while (common < kv_tokens_.size() && common < (size_t)n && kv_tokens_[common] == prompt[common]) common++;
  const size_t reused = std::min(std::min(common, cached_prefill_len_), (size_t)n - 1) / chunk * chunk;
  if (kv_tokens_.size() > reused) kv_tokens_.resize(reused);
  cached_prefill_len_ = 0;
  s.prefill_cached_tokens = (int)reused;
  int off = (int)reused;
  bool user_stop = false;
  std::vector<int> positions(chunk);
  if (!dbg_on_ && n - off > chunk) {  // two or more chunks: lanes in turn
    bool stopped = false;
    const int rc = prefill_lanes(prompt, n, off, chunk, &stopped);
    if (rc && !g_stop.load()) {
      kv_tokens_.clear();
      return finish(rc);
    }
    if (rc || stopped) {
      user_stop = true;
    } else {
      kv_tokens_.insert(kv_tokens_.end(), prompt + off, prompt + n);
      off = n;
    }
  }
  while (off < n && !user_stop) {
    if (g_stop.load()) { user_stop = true; break; }
    const int m = std::min(chunk, n - off);
    for (int i = 0; i < m; i++) positions[i] = off + i;
    const bool last = off + m >= n;
    const int rc = forward_inner(prompt + off, positions.data(), m, last, true);
    if (rc) {
      kv_tokens_.clear();
      if (g_stop.load()) { user_stop = true; break; }
      return finish(rc);
    }
    kv_tokens_.insert(kv_tokens_.end(), prompt + off, prompt + off + m);
    off += m;
  }
  s.prefill_tokens = off - (int)reused;
  s.prefill_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  if (user_stop) {
    std::snprintf(s.stop, sizeof(s.stop), "user_stop");
    kv_tokens_.clear();
    return finish(PK_OK);
  }
  cached_prefill_len_ = n;
  int pos = n;
  const auto g0 = std::chrono::steady_clock::now();
  for (int i = 0; i < opts.max_tokens; i++) {
    if (g_stop.load()) { std::snprintf(s.stop, sizeof(s.stop), "user_stop"); break; }
    uint32_t tok = 0;
    int rc = sampling ? sample(opts.temp, opts.top_p, &tok) : argmax(&tok);
    if (rc) return finish(rc);
    if (opts.stop_at_eog && std::binary_search(eos_ids_.begin(), eos_ids_.end(), tok)) {
      std::snprintf(s.stop, sizeof(s.stop), "eog");
      break;
    }
    s.gen_tokens++;
    if (nout < out_cap && out_ids) out_ids[nout] = tok;
    nout++;
    if (cb && !cb(tok, user)) {
      std::snprintf(s.stop, sizeof(s.stop), "callback_error");
      kv_tokens_.clear();
      cached_prefill_len_ = 0;
      break;
    }
    if (i + 1 == opts.max_tokens) break;
    if (pos >= n_ctx_) { std::snprintf(s.stop, sizeof(s.stop), "context_full"); break; }
    rc = forward_inner(&tok, &pos, 1, true, true);
    if (rc) {
      kv_tokens_.clear();
      cached_prefill_len_ = 0;
      if (g_stop.load()) { std::snprintf(s.stop, sizeof(s.stop), "user_stop"); break; }
      return finish(rc);
    }
    kv_tokens_.push_back(tok);
    pos++;
  }
  if (std::strcmp(s.stop, "user_stop") == 0) {
    kv_tokens_.clear();
    cached_prefill_len_ = 0;
  }
  s.gen_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - g0).count();
  return finish(PK_OK);
}

// n_steps greedy steps with the token fed back on the device: per step one
// graph launch (argmax -> advance -> b=1 forward), no host round trip.
int Engine::decode_steps_device(int n_steps, uint32_t *out_ids, float *device_ms) {
  if (!loaded_) return set_error(PK_ERR_INVALID, "no model loaded");
  if (!have_logits_) return set_error(PK_ERR_INVALID, "no logits: run a forward pass with want_logits first");
  if (device_ms) *device_ms = 0.0f;
  if (n_steps <= 0) return PK_OK;
  if (next_pos_ + n_steps > n_ctx_) return set_error(PK_ERR_CONTEXT_FULL, "context full");
  int rc = ensure_graphs();
  if (rc) return rc;
  h_pos_[0] = next_pos_ - 1;
  PK_CK(cudaMemcpyAsync(d_pos_, h_pos_, sizeof(int), cudaMemcpyHostToDevice, st_));
  PK_CK(cudaMemsetAsync(d_step_, 0, sizeof(int), st_));
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  PK_CK(cudaEventCreate(&e0));
  PK_CK(cudaEventCreate(&e1));
  cudaError_t e = cudaEventRecord(e0, st_);
  if (use_decode_ && e == cudaSuccess) {  // the first token comes from the logits already there
    e = launch_argmax(logits_, vocab_, d_tok_, st_);
    if (e == cudaSuccess) e = launch_advance(d_tok_, d_ids_, d_pos_, d_hist_, d_step_, st_);
  }
  for (int i = 0; i < n_steps && e == cudaSuccess; i++) e = cudaGraphLaunch(g_step_, st_);
  if (e == cudaSuccess) e = cudaEventRecord(e1, st_);
  std::vector<uint32_t> hist(n_steps);
  if (e == cudaSuccess) e = cudaMemcpyAsync(hist.data(), d_hist_, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, st_);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st_);
  float ms = 0.0f;
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (e != cudaSuccess) return cuda_error(e, "decode_steps_device");
  rc = check_decode_error();
  if (rc) return rc;
  if (device_ms) *device_ms = ms;
  if (out_ids) std::memcpy(out_ids, hist.data(), (size_t)n_steps * 4);
  kv_tokens_.insert(kv_tokens_.end(), hist.begin(), hist.end());
  next_pos_ += n_steps;
  return PK_OK;
}

// The K/V cache's entry type, before the model loads (the caches are sized
// then).  f16 entries are each value rounded to nearest even; attention then
// runs on the per-(token, head) kernel and decode on the per-op kernels.
int Engine::set_kv_type(int type) {
  if (type != PK_KV_F32 && type != PK_KV_F16) return set_error(PK_ERR_INVALID, "unknown KV cache type");
  if (loaded_) return set_error(PK_ERR_INVALID, "the KV cache type is set before the model loads");
  kv_f16_ = type == PK_KV_F16;
  return PK_OK;
}

int Engine::set_order(int order) {
  if (order != PK_ORDER_EXACT && order != PK_ORDER_FAST) return set_error(PK_ERR_INVALID, "unknown decode order");
  if (order != order_) {
    order_ = order;
    dargs_.fast = order == PK_ORDER_FAST ? 1 : 0;
    release_graphs();  // the captured step holds the other order's kernel
  }
  return PK_OK;
}

int Engine::set_position(int pos) {
  if (!loaded_) return set_error(PK_ERR_INVALID, "no model loaded");
  if (pos <= 0 || pos > next_pos_) return set_error(PK_ERR_INVALID, "position must be in 1..current length");
  next_pos_ = pos;
  if (kv_tokens_.size() > (size_t)pos) kv_tokens_.resize(pos);
  cached_prefill_len_ = std::min(cached_prefill_len_, (size_t)pos);
  return PK_OK;
}

// ---- independent streams (no reference counterpart: the reference keeps one
// sequence per engine).  Each stream has its own KV cache; a step decodes one
// token of every stream in one batch, the weights read once for all.  The
// step uses the b == 1 arithmetic for every stream (the sum of squares in
// the f32_sum_sq order, scores in the f32_dot order, one attention CTA per
// stream and head), and the lanes matvec equals the single-lane one bit for
// bit, so each stream's tokens are those it gets decoded alone.
int Engine::streams_begin(int n) {
  if (!loaded_) return set_error(PK_ERR_INVALID, "no model loaded");
  if (n < 1 || n > max_batch_ || n > 64) return set_error(PK_ERR_INVALID, "streams: 1..max_batch streams");
  if (n_streams_) return set_error(PK_ERR_INVALID, "streams already begun");
  PK_CK(cudaSetDevice(device_));
  const size_t half = kv_bytes_ / 2;
  PK_CK(cudaMalloc((void **)&d_sk_, half * n));
  PK_CK(cudaMalloc((void **)&d_sv_, half * n));
  PK_CK(cudaMemsetAsync(d_sk_, 0, half * n, st_));
  PK_CK(cudaMemsetAsync(d_sv_, 0, half * n, st_));
  // histories above 1024 positions: the attention's scores are split over
  // chunks of 512 (1024 above 8192) positions, whose maxima need scratch
  spchunk_ = n_ctx_ > 1024 ? (n_ctx_ > 8192 ? 1024 : 512) : 0;
  const size_t nch = spchunk_ ? (size_t)(n_ctx_ + spchunk_ - 1) / spchunk_ : 0;
  const size_t aux = (size_t)n * vocab_ * 4 + 256 + (size_t)n * 4 * 4 + (size_t)n * n_ctx_ * 4 +
                     (size_t)n * cfg_.n_head * nch * 4;
  PK_CK(cudaMalloc((void **)&d_slogits_, aux));
  uint8_t *p = (uint8_t *)d_slogits_ + (size_t)n * vocab_ * 4 + 256 - (((size_t)n * vocab_ * 4) & 255);
  d_sids_ = (uint32_t *)p;
  d_stok_ = d_sids_ + n;
  d_spos_ = (int *)(d_stok_ + n);
  d_sstep_ = d_spos_ + n;
  d_shist_ = (uint32_t *)(d_sstep_ + n);
  d_spmax_ = spchunk_ ? (float *)(d_shist_ + (size_t)n * n_ctx_) : nullptr;
  PK_CK(cudaStreamSynchronize(st_));
  n_streams_ = n;
  spos_.assign(n, 0);
  stok_.assign(n, 0);
  sready_.assign(n, 0);
  return PK_OK;
}

// The prompt into stream s's cache: the engine's prefill (32-token chunks,
// lanes for two or more) with stream s's cache in place of the engine's; the
// greedy pick of its last logits is the stream's next token.
int Engine::stream_prefill(int s, const uint32_t *prompt, int n) {
  if (s < 0 || s >= n_streams_) return set_error(PK_ERR_INVALID, "no such stream");
  if (n <= 0 || n > n_ctx_) return set_error(PK_ERR_CONTEXT_FULL, "prompt empty or longer than n_ctx");
  for (int i = 0; i < n; i++)
    if (prompt[i] >= (uint32_t)vocab_) return set_error(PK_ERR_INVALID, "token out of vocab");
  PK_CK(cudaSetDevice(device_));
  const size_t per = (size_t)cfg_.n_layer * cfg_.n_head_kv * n_ctx_ * cfg_.head_dim;  // entries of one cache
  float *k0 = d_kcache_, *v0 = d_vcache_;
  d_kcache_ = kv_at(d_sk_, (size_t)s * per);
  d_vcache_ = kv_at(d_sv_, (size_t)s * per);
  kv_tokens_.clear();
  cached_prefill_len_ = 0;
  int rc = PK_OK;
  const int chunk = std::min(max_batch_, 32);
  if (n > chunk) {
    bool stopped = false;
    rc = prefill_lanes(prompt, n, 0, chunk, &stopped);
    if (!rc && stopped) rc = set_error(PK_ERR_STOPPED, "generation stopped");
  } else {
    for (int i = 0; i < n; i++) {
      h_ids_[i] = prompt[i];
      h_pos_[i] = i;
    }
    cudaError_t e = cudaMemcpyAsync(d_ids_, h_ids_, n * sizeof(uint32_t), cudaMemcpyHostToDevice, st_);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_pos_, h_pos_, n * sizeof(int), cudaMemcpyHostToDevice, st_);
    rc = e != cudaSuccess ? cuda_error(e, "stream prefill ids") : enqueue_forward(n, true, false);
    const cudaError_t es = cudaStreamSynchronize(st_);
    if (!rc && es != cudaSuccess) rc = cuda_error(es, "stream prefill");
  }
  uint32_t tok = 0;
  if (!rc) rc = argmax(&tok);
  d_kcache_ = k0;
  d_vcache_ = v0;
  have_logits_ = false;  // the engine's own sequence is not what the logits belong to
  next_pos_ = 0;
  if (rc) return rc;
  spos_[s] = n;
  stok_[s] = tok;
  sready_[s] = 1;
  return PK_OK;
}

int Engine::enqueue_streams_step() {
  const Config &c = cfg_;
  const int S = n_streams_, ne = c.n_embd, dh = c.head_dim, qdim = c.n_head * dh, kdim = c.n_head_kv * dh, ff = c.n_ff;
  const size_t layer_kv = (size_t)c.n_head_kv * n_ctx_ * dh, stride = (size_t)c.n_layer * layer_kv;
  PK_CK(launch_dequant_rows(embd_type_, embd_raw_, embd_row_bytes_, ne, d_sids_, S, x_, st_));
  for (int l = 0; l < c.n_layer; l++) {
    const LayerDev &L = layers_[l];
    float *kc = kv_at(d_sk_, l * layer_kv), *vc = kv_at(d_sv_, l * layer_kv);
    Q8Dev a = act_;
    a.k = ne; a.b = S;
    PK_CK(launch_rmsnorm_q8(x_, L.attn_norm, c.rms_eps, ne, S, a, nullptr, st_, true));
    const MvOut qkv[3] = {{L.q, q_, 1, qdim, false}, {L.k, k_, 1, kdim, false}, {L.v, v_, 1, kdim, false}};
    PK_CK(launch_mv_multi(3, qkv, a, st_));
    PK_CK(launch_rope_kv(q_, k_, v_, S, d_spos_, d_rope_cos_, d_rope_sin_, c.n_rot / 2, dh, c.n_head, c.n_head_kv,
                         n_ctx_, kc, vc, st_, stride, kv_f16_));
    AttnArgs at{};
    at.q = q_; at.kcache = kc; at.vcache = vc; at.pos = d_spos_; at.out = attn_; at.b = S;
    at.n_head = c.n_head; at.n_kv = c.n_head_kv; at.dh = dh; at.n_ctx = n_ctx_;
    at.scale = 1.0f / sqrtf((float)dh); at.scores = att_scores_;
    at.lane_stride = stride; at.b1_order = 1; at.kv16 = kv_f16_ ? 1 : 0;
    at.pmax = d_spmax_; at.pchunk = spchunk_;
    a.k = qdim;
    at.q8 = a;
    PK_CK(launch_attention(at, st_));
    PK_CK(launch_mv_lanes(L.o, a, x_, 1, ne, true, st_));
    a.k = ne;
    PK_CK(launch_rmsnorm_q8(x_, L.ffn_norm, c.rms_eps, ne, S, a, nullptr, st_, true));
    const MvOut gu[2] = {{L.gate, gate_, 1, ff, false}, {L.up, up_, 1, ff, false}};
    PK_CK(launch_mv_multi(2, gu, a, st_));
    a.k = ff;
    PK_CK(launch_swiglu_q8(gate_, up_, ff, S, a, h_, st_));
    PK_CK(launch_mv_lanes(L.down, a, x_, 1, ne, true, st_));
  }
  Q8Dev a = act_;
  a.k = ne; a.b = S;
  PK_CK(launch_rmsnorm_q8(x_, output_norm_, c.rms_eps, ne, S, a, nullptr, st_, true));
  PK_CK(launch_mv_lanes(output_, a, d_slogits_, 1, vocab_, false, st_));
  PK_CK(launch_argmax(d_slogits_, vocab_, d_stok_, st_, S));
  PK_CK(launch_advance(d_stok_, d_sids_, d_spos_, d_shist_, d_sstep_, st_, S, (size_t)n_ctx_));
  return PK_OK;
}

// n_steps tokens of every stream, as decode_steps_device: the token picked
// last, then the next n_steps - 1 (the n_steps steps also pick the token the
// next call starts with).  out_ids: [n_steps][n_streams].
int Engine::streams_decode(int n_steps, uint32_t *out_ids, float *device_ms) {
  if (!n_streams_) return set_error(PK_ERR_INVALID, "no streams");
  if (n_steps < 1) return set_error(PK_ERR_INVALID, "n_steps must be >= 1");
  const int S = n_streams_;
  for (int s = 0; s < S; s++) {
    if (!sready_[s]) return set_error(PK_ERR_INVALID, "stream " + std::to_string(s) + " has no prefill");
    if (spos_[s] + n_steps > n_ctx_) return set_error(PK_ERR_CONTEXT_FULL, "context full");
  }
  PK_CK(cudaSetDevice(device_));
  if (!g_streams_) {  // every pointer of the step is fixed once the streams exist: one graph, replayed
    cudaGraph_t graph = nullptr;
    PK_CK(cudaStreamBeginCapture(st_, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue_streams_step();
    const cudaError_t ee = cudaStreamEndCapture(st_, &graph);
    if (rc || ee != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      return rc ? rc : cuda_error(ee, "streams graph capture");
    }
    const cudaError_t ei = cudaGraphInstantiate(&g_streams_, graph, 0);
    cudaGraphDestroy(graph);
    if (ei != cudaSuccess) {
      g_streams_ = nullptr;
      return cuda_error(ei, "streams graph instantiate");
    }
  }
  std::vector<int> zero(S, 0);
  PK_CK(cudaMemcpyAsync(d_sids_, stok_.data(), S * 4, cudaMemcpyHostToDevice, st_));
  PK_CK(cudaMemcpyAsync(d_spos_, spos_.data(), S * 4, cudaMemcpyHostToDevice, st_));
  PK_CK(cudaMemcpyAsync(d_sstep_, zero.data(), S * 4, cudaMemcpyHostToDevice, st_));
  cudaEvent_t e0, e1;
  PK_CK(cudaEventCreate(&e0));
  PK_CK(cudaEventCreate(&e1));
  cudaError_t e = cudaEventRecord(e0, st_);
  for (int i = 0; i < n_steps && e == cudaSuccess; i++) e = cudaGraphLaunch(g_streams_, st_);
  if (e == cudaSuccess) e = cudaEventRecord(e1, st_);
  std::vector<uint32_t> hist((size_t)S * n_ctx_);
  if (e == cudaSuccess) e = cudaMemcpyAsync(hist.data(), d_shist_, hist.size() * 4, cudaMemcpyDeviceToHost, st_);
  const cudaError_t es = cudaStreamSynchronize(st_);
  float ms = 0.0f;
  if (e == cudaSuccess && es == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (e != cudaSuccess) return cuda_error(e, "streams decode");
  if (es != cudaSuccess) return cuda_error(es, "streams decode");
  for (int s = 0; s < S; s++) {
    const uint32_t *hs = hist.data() + (size_t)s * n_ctx_;
    if (out_ids) {
      out_ids[s] = stok_[s];
      for (int i = 1; i < n_steps; i++) out_ids[(size_t)i * S + s] = hs[i - 1];
    }
    stok_[s] = hs[n_steps - 1];
    spos_[s] += n_steps;
  }
  if (device_ms) *device_ms = ms;
  return PK_OK;
}

// Every stream's position set to pos: the next step decodes at pos over the
// cache entries 0..pos - 1 as they are.  Entries past a stream's own tokens
// hold zeros (or an earlier run's values), so a pos beyond a stream's length
// is for timing long-context steps only; the tokens then are not a sequence.
int Engine::streams_set_position(int pos) {
  if (!n_streams_) return set_error(PK_ERR_INVALID, "no streams");
  if (pos < 1 || pos >= n_ctx_) return set_error(PK_ERR_INVALID, "position must be in 1..n_ctx-1");
  for (int s = 0; s < n_streams_; s++) {
    if (!sready_[s]) return set_error(PK_ERR_INVALID, "stream " + std::to_string(s) + " has no prefill");
    spos_[s] = pos;
  }
  return PK_OK;
}

// One persistent-kernel launch whose o-phase readers (layer 0) wait for a tag
// that no phase writes: every CTA's bounded wait runs out, the launch stops
// with PK_ERR_TIMEOUT in the error word and returns, and the engine recovers
// (the error path resets the counters and advances the tag epoch).  The
// launch does not feed a token back, so the sequence is unchanged.
int Engine::selftest_bounded_wait(int *status) {
  if (!loaded_) return set_error(PK_ERR_INVALID, "no model loaded");
  if (!use_decode_) return set_error(PK_ERR_UNSUPPORTED, "the persistent decode kernel is not in use");
  if (next_pos_ + 1 > n_ctx_) return set_error(PK_ERR_CONTEXT_FULL, "context full");
  h_pos_[0] = next_pos_;
  PK_CK(cudaMemcpyAsync(d_pos_, h_pos_, sizeof(int), cudaMemcpyHostToDevice, st_));
  DecodeArgs a = dargs_;
  a.mode = 0;
  a.poison = 2;  // phase 2: layer 0's o phase reads the attention output
  PK_CK(launch_decode(a, plan_.grid, plan_.smem, st_));
  PK_CK(cudaStreamSynchronize(st_));
  *status = check_decode_error();  // its message stays in pk_last_error()
  return PK_OK;
}

int Engine::decode_profile(pk_kernel_stat *out, int cap, int *n_out) {
  if (!loaded_) return set_error(PK_ERR_INVALID, "no model loaded");
  if (!have_logits_) return set_error(PK_ERR_INVALID, "no logits: run a forward pass with want_logits first");
  if (next_pos_ + 1 > n_ctx_) return set_error(PK_ERR_CONTEXT_FULL, "context full");
  std::vector<ProfMark> marks;
  prof_ = &marks;
  h_pos_[0] = next_pos_ - 1;
  int rc = PK_OK;
  cudaError_t e = cudaMemcpyAsync(d_pos_, h_pos_, sizeof(int), cudaMemcpyHostToDevice, st_);
  if (e == cudaSuccess) e = cudaMemsetAsync(d_step_, 0, sizeof(int), st_);
  if (e == cudaSuccess) {
    rc = prof_begin("k_argmax", (double)vocab_ * 4.0);
    if (!rc) e = launch_argmax(logits_, vocab_, d_tok_, st_);
    if (!rc && e == cudaSuccess) rc = prof_end();
    if (!rc && e == cudaSuccess) e = launch_advance(d_tok_, d_ids_, d_pos_, d_hist_, d_step_, st_);
    if (use_decode_) {
      DecodeArgs a = dargs_;
      a.mode = 1;
      a.trace = d_trace_;
      const Config &c = cfg_;
      const double kv = 2.0 * c.n_layer * c.n_head_kv * c.head_dim * 4.0 * ((double)next_pos_ + 1.0);
      if (!rc && e == cudaSuccess) rc = prof_begin("k_decode", (double)stream_bytes_ + kv);
      if (!rc && e == cudaSuccess) e = launch_decode(a, plan_.grid, plan_.smem, st_);
      if (!rc && e == cudaSuccess) rc = prof_end();
    } else if (!rc && e == cudaSuccess) {
      rc = enqueue_forward(1, true, false);
    }
  }
  prof_ = nullptr;
  if (e == cudaSuccess) e = cudaStreamSynchronize(st_);
  std::vector<pk_kernel_stat> agg;
  for (auto &m : marks) {
    float ms = 0.0f;
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, m.start, m.stop);
    cudaEventDestroy(m.start);
    cudaEventDestroy(m.stop);
    pk_kernel_stat *s = nullptr;
    for (auto &a : agg)
      if (m.name == a.name) s = &a;
    if (!s) {
      agg.push_back(pk_kernel_stat{});
      s = &agg.back();
      std::snprintf(s->name, sizeof(s->name), "%s", m.name.c_str());
    }
    s->launches++;
    s->ms += ms;
    s->bytes += m.bytes;
  }
  if (rc) return rc;
  if (e != cudaSuccess) return cuda_error(e, "decode_profile");
  if (use_decode_) {
    if ((rc = check_decode_error())) return rc;
    // Phase times inside the persistent kernel from its per-CTA trace (layout
    // in pk_decode.cu): wall time per phase from the barrier exits, and per
    // CTA averages of prologue, compute, barrier wait and ring-data stall.
    const Config &c = cfg_;
    const int nt = dargs_.n_trace, grid = plan_.grid, nl = c.n_layer;
    std::vector<unsigned long long> tr((size_t)grid * nt);
    PK_CK(cudaMemcpyAsync(tr.data(), d_trace_, tr.size() * 8, cudaMemcpyDeviceToHost, st_));
    PK_CK(cudaStreamSynchronize(st_));
    if (const char *dump = std::getenv("PK_TRACE_DUMP")) {  // raw per-CTA trace: grid x n_trace u64 words
      if (FILE *f = std::fopen(dump, "wb")) {
        std::fwrite(tr.data(), 8, tr.size(), f);
        std::fclose(f);
      }
    }
    auto at = [&](int g, int i) { return (double)tr[(size_t)g * nt + i]; };
    int khz = 0;
    PK_CK(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, device_));
    const double cyc_ms = 1.0 / std::max(1.0, (double)khz);  // SM cycles -> ms at the rated clock
    auto exit_of = [&](int g, int q) { return q < 0 ? at(g, 0) : at(g, 1 + DK_TRW * q + 2); };
    auto max_exit = [&](int q) {
      double v = 0;
      for (int g = 0; g < grid; g++) v = std::max(v, exit_of(g, q));
      return v;
    };
    const char *names[6] = {"dk_qkv", "dk_attn", "dk_o", "dk_gateup", "dk_down", "dk_head"};
    const char *subs[7] = {"prologue", "compute", "barrier", "data_wait", "term_bufwait", "term_work", "chain_wait"};
    double wall[6] = {0}, sub[6][8] = {{0}}, bytes[6] = {0};
    const double f4 = 4.0, kvp = (double)next_pos_ + 1.0;
    for (int q = 0; q < 5 * nl; q++) {
      const int j = q % 5;
      wall[j] += (max_exit(q) - max_exit(q - 1)) * 1e-6;
      // attention sub-phases: only the CTAs that own a head stamp them
      const int ng = j == 1 ? std::min(grid, c.n_head * plan_.att_j) : grid;
      for (int g = 0; g < ng; g++) {
        const int b0 = 1 + DK_TRW * q;
        sub[j][0] += (at(g, b0) - exit_of(g, q - 1)) * 1e-6 / ng;
        sub[j][1] += (at(g, b0 + 1) - at(g, b0)) * 1e-6 / ng;
        sub[j][2] += (at(g, b0 + 2) - at(g, b0 + 1)) * 1e-6 / ng;
        for (int i = 3; i < 8; i++) sub[j][i] += at(g, b0 + i) * cyc_ms / ng;
      }
    }
    // fine stamps: average offset from the phase start, summed over layers
    double fine_ms[5][8] = {{0}};
    double chain_cyc[5] = {0}, chain_terms[5] = {0};
    for (int q = 0; q < 5 * nl; q++) {
      const int j = q % 5;
      if (j != 1)
        for (int g = 0; g < grid; g++) {
          chain_cyc[j] += at(g, 1 + DK_TRW * q + 14);
          chain_terms[j] += at(g, 1 + DK_TRW * q + 15);
        }
      for (int i = 0; i < (j == 1 ? 8 : 6); i++) {
        double sum = 0;
        int cnt = 0;
        for (int g = 0; g < grid; g++) {
          const double v = at(g, 1 + DK_TRW * q + 8 + i);
          if (v > 0) {
            sum += (v - exit_of(g, q - 1)) * 1e-6;
            cnt++;
          }
        }
        if (cnt) fine_ms[j][i] += sum / cnt;
      }
    }
    double head_end = 0, prod = 0;
    for (int g = 0; g < grid; g++) {
      head_end = std::max(head_end, at(g, 1 + DK_TRW * 5 * nl + 1));
      sub[5][0] += (at(g, 1 + DK_TRW * 5 * nl) - exit_of(g, 5 * nl - 1)) * 1e-6 / grid;
      sub[5][1] += (at(g, 1 + DK_TRW * 5 * nl + 1) - at(g, 1 + DK_TRW * 5 * nl)) * 1e-6 / grid;
      for (int L = 0; L <= nl; L++) prod += at(g, 1 + DK_TRW * (5 * nl + 1) + L) * cyc_ms / grid;
    }
    wall[5] = (head_end - max_exit(5 * nl - 1)) * 1e-6;
    for (int L = 0; L < nl; L++) {
      const LayerDev &Y = layers_[L];
      bytes[0] += mat_stream_bytes(Y.q) + mat_stream_bytes(Y.k) + mat_stream_bytes(Y.v) + c.n_embd * f4;
      bytes[1] += 2.0 * c.n_head_kv * kvp * c.head_dim * f4;
      bytes[2] += mat_stream_bytes(Y.o);
      bytes[3] += mat_stream_bytes(Y.gate) + mat_stream_bytes(Y.up) + c.n_embd * f4;
      bytes[4] += mat_stream_bytes(Y.down);
    }
    bytes[5] = mat_stream_bytes(output_) + c.n_embd * f4 + embd_row_bytes_;
    auto add = [&](const std::string &n, int launches, double ms, double by) {
      pk_kernel_stat st{};
      std::snprintf(st.name, sizeof(st.name), "%s", n.c_str());
      st.launches = launches;
      st.ms = ms;
      st.bytes = by;
      agg.push_back(st);
    };
    for (int j = 0; j < 6; j++) add(names[j], j == 5 ? 1 : nl, wall[j], bytes[j]);
    // Sub-phase averages over CTAs (bytes 0: not kernels of their own).
    for (int j = 0; j < 6; j++)
      for (int i = 0; i < (j == 5 ? 2 : 8); i++)
        add(std::string(names[j]) + "/" + (i < 7 ? subs[i] : "chain_work"), j == 5 ? 1 : nl, sub[j][i], 0.0);
    add("dk_producer/slot_wait", 1, prod, 0.0);
    for (int j = 0; j < 5; j++)  // chain warp 0: SM cycles per term of its row chains (in the ms field)
      if (j != 1 && chain_terms[j] > 0)
        add(std::string(names[j]) + "/chain_cycles_per_term", nl, chain_cyc[j] / chain_terms[j] * nl, 0.0);
    {  // the SM clock the launch ran at: SM cycles over globaltimer ns, averaged over CTAs
      double mhz = 0.0;
      for (int g = 0; g < grid; g++) {
        const double dc = at(g, nt - 2) - at(g, nt - 4), dn = at(g, nt - 1) - at(g, nt - 3);
        mhz += dn > 0 ? dc / dn * 1e3 / grid : 0.0;
      }
      add("k_decode/clock_mhz", 1, mhz, 0.0);  // in the ms field: MHz
    }
    for (int j = 0; j < 5; j++)
      for (int i = 0; i < 8; i++)
        if (fine_ms[j][i] > 0) add(std::string(names[j]) + "/at" + std::to_string(i), nl, fine_ms[j][i], 0.0);
  }
  uint32_t tok = 0;
  PK_CK(cudaMemcpyAsync(&tok, d_tok_, 4, cudaMemcpyDeviceToHost, st_));
  kv_tokens_.push_back(tok);
  next_pos_ += 1;
  for (int i = 0; i < (int)agg.size() && i < cap; i++) out[i] = agg[i];
  if (n_out) *n_out = (int)agg.size();
  return PK_OK;
}

int Engine::set_debug(bool on) {
  dbg_on_ = on;
  dbg_.clear();
  return PK_OK;
}

int Engine::get_dump(const char *name, float *out, int cap, int *n_out) {
  if (std::strncmp(name, "decode.", 7) == 0 && use_decode_) {
    // The persistent kernel's phase outputs of its last launch (last layer),
    // read from the tagged words (value in the low half).
    const DecodeArgs &a = dargs_;
    const size_t qd = (size_t)a.n_head * a.dh, kd = (size_t)a.n_kv * a.dh;
    const std::string n = name + 7;
    const unsigned long long *src = nullptr;
    size_t cnt = 0;
    if (n == "q") src = a.q_ll, cnt = qd;
    else if (n == "k") src = a.kv_ll, cnt = kd;
    else if (n == "v") src = a.kv_ll + kd, cnt = kd;
    else if (n == "att") src = a.att_ll, cnt = qd;
    else if (n == "x_o") src = a.x_ll, cnt = (size_t)a.n_embd;
    else if (n == "x") src = a.x_ll + a.n_embd, cnt = (size_t)a.n_embd;
    else if (n == "h") src = a.h_ll, cnt = (size_t)a.n_ff;
    if (src) {
      std::vector<unsigned long long> w(cnt);
      PK_CK(cudaMemcpyAsync(w.data(), src, cnt * 8, cudaMemcpyDeviceToHost, st_));
      PK_CK(cudaStreamSynchronize(st_));
      if (out)
        for (size_t i = 0; i < std::min(cnt, (size_t)std::max(cap, 0)); i++) {
          const uint32_t lo = (uint32_t)w[i];
          std::memcpy(out + i, &lo, 4);
        }
      if (n_out) *n_out = (int)cnt;
      return PK_OK;
    }
  }
  for (auto &d : dbg_)
    if (d.first == name) {
      const int n = (int)d.second.size();
      if (out) std::memcpy(out, d.second.data(), (size_t)std::min(cap, n) * 4);
      if (n_out) *n_out = n;
      return PK_OK;
    }
  if (n_out) *n_out = 0;
  return set_error(PK_ERR_INVALID, std::string("no dump named ") + name);
}

}  // namespace pk
