// pk_engine.h -- the device engine behind pk_create / pk_load_gguf / pk_generate.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <string>
#include <vector>

#include "pk.h"
#include "pk_gguf.h"
#include "pk_decode.h"
#include "pk_kernels.h"

namespace pk {

int set_error(int code, const std::string &msg);
int cuda_error(cudaError_t e, const char *what);
extern std::atomic<bool> g_stop;

// model.rs:14-97 Config.
struct Config {
  std::string arch;
  int n_layer = 0, n_embd = 0, n_ff = 0, n_head = 0, n_head_kv = 0, head_dim = 0, n_rot = 0, n_vocab = 0;
  float rope_theta = 10000.0f, rms_eps = 1e-5f;
};

// A GGUF tensor: type, shape (ne0 = row length) and file offset.
struct TRef {
  std::string name;
  int type = 0;
  size_t ne0 = 0, ne1 = 0, row_bytes = 0, off = 0;
};
int config_from_gguf(const Gguf &g, Config &c);
int find_tensor(const Gguf &g, const std::string &name, TRef &out);
int check_shape(const TRef &t, size_t cols, size_t rows);

struct LayerDev {
  DevTensor q, k, v, o, gate, up, down;
  float *attn_norm = nullptr, *ffn_norm = nullptr;
};

class Engine {
 public:
  ~Engine();
  int create(int device, int n_ctx, int max_batch);
  int load(const char *path);
  int info(pk_model_info *out) const;

  int forward(const uint32_t *ids, const int *pos, int n, bool want_logits);
  int logits(float *out, int n);
  int argmax(uint32_t *tok);
  int sample(float temp, float top_p, uint32_t *tok);
  int generate(const uint32_t *prompt, int n, const pk_gen_opts &opts, pk_token_cb cb, void *user,
               uint32_t *out_ids, int out_cap, int *n_out, pk_gen_stats *stats);
  int decode_steps_device(int n_steps, uint32_t *out_ids, float *device_ms);
  int set_position(int pos);
  int set_order(int order);
  int set_kv_type(int type);
  // Independent streams, each with its own KV cache, decoded together.
  int streams_begin(int n_streams);
  int stream_prefill(int s, const uint32_t *prompt, int n);
  int streams_decode(int n_steps, uint32_t *out_ids, float *device_ms);
  int streams_set_position(int pos);
  int decode_profile(pk_kernel_stat *out, int cap, int *n_out);
  int selftest_bounded_wait(int *status);
  int set_debug(bool on);
  int get_dump(const char *name, float *out, int cap, int *n_out);

 private:
  int forward_inner(const uint32_t *ids, const int *pos, int b, bool want_logits, bool cancellable);
  enum { KV_RECORD = 1, KV_WAIT = 2 };
  int enqueue_forward(int b, bool want_logits, bool cancellable, int li = 0, int kv = 0);
  int prefill_lanes(const uint32_t *prompt, int n, int off, int chunk, bool *stopped);
  int enqueue_streams_step();
  int setup_decode();
  int check_tc_error();
  int check_decode_error();
  int ensure_graphs();
  void release_graphs();
  void dump(const char *name, const float *dev, size_t n);

  int device_ = 0, n_ctx_ = 0, max_batch_ = 0;
  bool loaded_ = false;
  cudaStream_t st_ = nullptr;
  Config cfg_;
  std::vector<LayerDev> layers_;
  DevTensor output_;
  float *output_norm_ = nullptr;
  const uint8_t *embd_raw_ = nullptr;
  int embd_type_ = 0;
  size_t embd_row_bytes_ = 0;
  int vocab_ = 0;
  std::vector<uint32_t> eos_ids_;
  size_t weight_bytes_ = 0, stream_bytes_ = 0, kv_bytes_ = 0;

  // device allocations
  uint8_t *d_weights_ = nullptr;
  float *d_kcache_ = nullptr, *d_vcache_ = nullptr;
  float *d_rope_cos_ = nullptr, *d_rope_sin_ = nullptr;
  uint8_t *d_act_arena_ = nullptr;
  float *x_ = nullptr, *q_ = nullptr, *k_ = nullptr, *v_ = nullptr, *attn_ = nullptr;
  float *gate_ = nullptr, *up_ = nullptr, *h_ = nullptr, *logits_ = nullptr;
  Q8Dev act_;
  float *att_scores_ = nullptr;
  uint32_t *d_ids_ = nullptr, *d_tok_ = nullptr, *d_hist_ = nullptr;
  int *d_pos_ = nullptr, *d_step_ = nullptr;
  // pinned host staging
  uint32_t *h_ids_ = nullptr, *h_tok_ = nullptr;
  int *h_pos_ = nullptr;
  // streams: one KV cache each ([stream][layer][...] as the engine's own), the
  // batch's token ids / positions / picks on the device, each stream's
  // history of picks, and the host view of every stream
  int n_streams_ = 0;
  float *d_sk_ = nullptr, *d_sv_ = nullptr, *d_slogits_ = nullptr;
  uint32_t *d_sids_ = nullptr, *d_stok_ = nullptr, *d_shist_ = nullptr;
  int *d_spos_ = nullptr, *d_sstep_ = nullptr;
  float *d_spmax_ = nullptr;  // long histories: per-chunk score maxima of the split attention
  int spchunk_ = 0;
  std::vector<int> spos_;
  std::vector<uint32_t> stok_;
  std::vector<char> sready_;
  // temperature / top-p sampling: the Rng state and the sampler's scratch
  unsigned long long *d_rng_ = nullptr, h_rng_ = 0;
  uint8_t *d_sample_scratch_ = nullptr;

  // Prefill lanes: the scratch of one chunk's forward pass and the stream it
  // runs on.  Lane 0 is the buffers above and st_; the others have their
  // own, so consecutive chunks of a prompt run on lanes in turn, chunk c + 1's
  // layer l waiting only for chunk c's K/V of layer l (kv_ev_).
  struct Lane {
    cudaStream_t st = nullptr;
    float *x = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr;
    float *gate = nullptr, *up = nullptr, *h = nullptr, *scores = nullptr;
    Q8Dev act;
    uint32_t *ids = nullptr;
    int *pos = nullptr;
  };
  static constexpr int NLANES = 6;
  Lane lane_[NLANES];
  uint8_t *d_lane_arena_[NLANES] = {};
  std::vector<cudaEvent_t> kv_ev_[NLANES];
  cudaEvent_t fork_ev_ = nullptr, join_ev_[NLANES] = {};
  uint32_t *h_pids_ = nullptr;  // pinned prompt ids / positions, n_ctx each
  int *h_ppos_ = nullptr;

  // persistent decode kernel (pk_decode.cu): plan, device tables and args
  bool use_decode_ = false;
  int order_ = PK_ORDER_EXACT;  // float order of the b = 1 decode step (pk_set_order)
  bool kv_f16_ = false;         // f16 K/V cache entries (pk_set_kv_type, before the model loads)
  // base + elems cache entries (f32 or f16), as the caches' float pointer type
  float *kv_at(float *base, size_t elems) const {
    return reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(base) + elems * (kv_f16_ ? 2 : 4));
  }
  std::string decode_why_;
  DecodePlan plan_;
  DecodeArgs dargs_{};
  uint8_t *d_decode_ = nullptr;
  int *d_err_ = nullptr;
  unsigned *d_sync_ = nullptr;
  unsigned long long *d_trace_ = nullptr;

  // decode graphs: fwd1 = one b=1 forward with logits; step = argmax + advance + fwd1
  cudaGraphExec_t g_fwd1_ = nullptr, g_step_ = nullptr;
  cudaGraphExec_t g_streams_ = nullptr;  // one batched streams step (its state lives on the device)

  // Engine::generate prefix-reuse state (model.rs:689-694)
  std::vector<uint32_t> kv_tokens_;
  size_t cached_prefill_len_ = 0;
  int next_pos_ = 0;
  bool have_logits_ = false;

  bool dbg_on_ = false;
  std::vector<std::pair<std::string, std::vector<float>>> dbg_;

  // decode_profile: events around each launch of an eager b == 1 step
  struct ProfMark {
    std::string name;
    double bytes;
    cudaEvent_t start, stop;
  };
  std::vector<ProfMark> *prof_ = nullptr;
  int prof_begin(const char *name, double bytes);
  int prof_end();
};

}  // namespace pk
