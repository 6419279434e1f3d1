// pk_tp.h -- tensor-parallel decode: one process per GPU, rank r of T holding
// a shard of every matrix, partial sums exchanged through peer memory.
//
// Split (a llama-style stack, b = 1 decode):
//   q / k / v  rows of whole heads      (q heads n_head / T, kv heads n_kv / T)
//   o          k range of whole heads   (the rank's attention output is its k slice)
//   gate / up  rows n_ff / T
//   down       k range n_ff / T          (the rank's SwiGLU output is its k slice)
//   output     vocabulary rows ceil(V / T); the token is the first maximum over
//              all shards (sampler.rs:26-36 semantics, as k_argmax)
// The residual x (n_embd) is replicated.  After o and after down every rank
// holds a partial row sum; each rank stores its partial into slot `rank` of
// every rank's exchange buffer (peer stores over NVLink), raises its flag
// there, and then adds the T slots in rank order to x, so every rank ends
// with the same bits.  With T = 1 the step is the single-GPU b = 1 op
// sequence bit for bit (x += 0.0 + acc).
#pragma once
#include <cuda_runtime.h>

#include <string>
#include <vector>

#include "pk.h"
#include "pk_engine.h"
#include "pk_kernels.h"

namespace pk {

constexpr int TP_MAX = 8;

// Row / k ranges of rank r of T, and whether a model splits (error text if not).
struct TpSplit {
  int nh = 0, nkv = 0, ff = 0;    // local q heads, kv heads, FFN rows
  int vocab0 = 0, nvocab = 0;     // local vocabulary rows [vocab0, vocab0 + nvocab)
};
bool tp_split(const Config &c, int vocab, int rank, int world, int o_block, int down_block, TpSplit &s,
              std::string &why);

// The first maximum over shards given each shard's (value, global index)
// in rank order: strict '>' in rank order; no value above -inf gives 0.
__host__ __device__ inline uint32_t tp_pick(const float *vals, const int *idx, int world) {
  float bv = -INFINITY;
  int bi = -1;
  for (int r = 0; r < world; r++)
    if (idx[r] >= 0 && vals[r] > bv) {
      bv = vals[r];
      bi = idx[r];
    }
  return bi < 0 ? 0u : (uint32_t)bi;
}

// Device pointers into every rank's exchange buffer (the own one included).
struct TpPeers {
  float *slots[TP_MAX];                 // [2][T][n_embd]
  float2 *amax[TP_MAX];                 // [2][T] {value, index bits}
  unsigned long long *flags[TP_MAX];    // [T]: the last sequence number rank s published here
};

// Bytes of an NCCL unique id, and a new one (rank 0 makes it, every rank
// passes it to TpEngine::use_nccl).  NCCL is loaded on first use.
int tp_nccl_id_bytes();
int tp_nccl_id(void *out);

class TpEngine {
 public:
  ~TpEngine();
  int create(int device, int n_ctx, int rank, int world);
  size_t exchange_bytes() const;
  int ipc_handle(void *out);  // cudaIpcMemHandle_t of this rank's exchange buffer
  int open_peers(const void *handles);  // T handles in rank order
  // The o / down exchange through an NCCL all-reduce (every rank, after
  // open_peers, with the same unique id) instead of the peer-memory push.
  int use_nccl(const void *id);
  int load(const char *path);
  int load_synthetic(const Config &c, int vocab, uint64_t seed);
  int prefill(const uint32_t *prompt, int n);  // b = 1 steps; ends with the first generated token on the device
  int decode(int n_steps, uint32_t *out_ids, float *device_ms);
  int logits(float *out, int n, int *n_local, int *vocab0);
  int info(pk_tp_info *out) const;

 private:
  int finish_load(const Config &c, int vocab);
  int step(bool feedback);  // one token: layers, head, first maximum over shards
  int allreduce_add(float *part, float *x);
  int check_error();

  int device_ = 0, n_ctx_ = 0, rank_ = 0, world_ = 1;
  bool loaded_ = false, peers_open_ = false;
  cudaStream_t st_ = nullptr;
  Config cfg_;
  TpSplit sp_;
  int vocab_ = 0;
  std::vector<LayerDev> layers_;
  DevTensor output_;
  float *output_norm_ = nullptr;
  uint8_t *d_weights_ = nullptr, *embd_raw_ = nullptr;
  int embd_type_ = 0;
  size_t embd_row_bytes_ = 0, weight_bytes_ = 0, stream_bytes_ = 0;
  float *d_kcache_ = nullptr, *d_vcache_ = nullptr, *d_rope_cos_ = nullptr, *d_rope_sin_ = nullptr;
  float *x_ = nullptr, *q_ = nullptr, *attn_ = nullptr, *h_ = nullptr, *part_ = nullptr, *logits_ = nullptr;
  float *scores_ = nullptr;
  uint32_t *d_ids_ = nullptr, *d_hist_ = nullptr;
  int *d_pos_ = nullptr, *d_step_ = nullptr, *d_err_ = nullptr;
  unsigned *d_count_ = nullptr;
  uint32_t *h_ids_ = nullptr;
  int *h_pos_ = nullptr;
  uint8_t *d_arena_ = nullptr;      // scratch
  uint8_t *d_x_ = nullptr;          // exchange buffer (IPC-exported)
  void *peer_base_[TP_MAX] = {};    // opened peer buffers (nullptr for the own rank)
  TpPeers peers_{};
  unsigned long long seq_ = 0;
  void *nccl_comm_ = nullptr;  // ncclComm_t once use_nccl succeeded
  int next_pos_ = 0;
  uint32_t last_tok_ = 0;
  bool have_tok_ = false;
};

}  // namespace pk
