// pk_tp.cu -- tensor-parallel decode engine (see pk_tp.h for the split).
//
// Each rank runs the single-GPU b = 1 kernels (k_qkv_b1, k_attn, k_mv_b1,
// k_gateup_b1) on its shard.  The collectives are two kernels of our own over
// peer memory:
//   k_tp_push: store the rank's partial into slot `rank` of every rank's
//              exchange buffer (plain stores to NVLink-mapped peer memory),
//              then the last CTA publishes the sequence number in every
//              rank's flag word for this rank (st.release.sys);
//   k_tp_sum:  wait (bounded) until every rank's flag here reaches the
//              sequence number (ld.acquire.sys), then x += slot 0 + slot 1 +
//              ... in rank order.
// Slots alternate by the parity of the sequence number: a rank can only
// publish sequence s + 1 after every rank published s, which each does only
// after it finished reading s - 1 from the slots s + 1 reuses.
// Alternatively (use_nccl) the o / down partials go through an NCCL
// all-reduce on the engine's stream, and k_tp_add adds the sum to x.
#include "pk_tp.h"

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstring>

#include "pk_device.cuh"
#include "pk_gguf.h"

namespace pk {

#define PK_CK(expr)                                          \
  do {                                                       \
    cudaError_t _e = (expr);                                 \
    if (_e != cudaSuccess) return cuda_error(_e, #expr);     \
  } while (0)

namespace {

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

template <typename... KArgs, typename... Args>
cudaError_t tp_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
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

constexpr long TP_SPIN = 20L * 1000 * 1000;  // ~2 s of 100 ns sleeps, then PK_ERR_TIMEOUT
constexpr int TP_PUSH_CTAS = 16;

__device__ __forceinline__ void st_release_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait for every rank's flag to reach seq; thread 0 waits, the CTA
// learns the outcome.  On expiry err gets 1 + the first missing rank, and
// later waits return at once until the host has read and cleared err.
__device__ bool wait_flags(const unsigned long long *flags, int world, unsigned long long seq, int *err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    int good = *(volatile int *)err == 0;  // after one expired wait the rest of the step does not wait again
    for (int s = 0; s < world && good; s++) {
      long it = 0;
      while (ld_acquire_sys(flags + s) < seq) {
        if (++it > TP_SPIN) {
          good = 0;
          atomicCAS(err, 0, 1 + s);
          break;
        }
        __nanosleep(100);
      }
    }
    ok = good;
  }
  __syncthreads();
  return ok != 0;
}

__global__ void __launch_bounds__(256) k_tp_push(const float *__restrict__ src, int n, TpPeers P, int rank, int world,
                                                 unsigned long long seq, unsigned *count) {
  pdl_trigger();
  pdl_wait();
  const int par = (int)(seq & 1ULL), n4 = n / 4;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4 * world; i += gridDim.x * blockDim.x) {
    const int dst = i / n4, j = i - dst * n4;
    const float4 v = __ldcg(reinterpret_cast<const float4 *>(src) + j);
    reinterpret_cast<float4 *>(P.slots[dst] + ((size_t)par * world + rank) * n)[j] = v;
  }
  // The CTA's stores, ordered by the barrier, then one system-scope fence by
  // the thread that counts the CTA in (the grid barrier's pattern): the fence
  // is cumulative over what the barrier made visible to that thread.
  __syncthreads();
  if (threadIdx.x == 0) __threadfence_system();
  if (threadIdx.x == 0 && atomicAdd(count, 1u) == gridDim.x - 1) {  // every CTA's stores are out
    *count = 0;
    __threadfence_system();
    for (int dst = 0; dst < world; dst++) st_release_sys(P.flags[dst] + rank, seq);
  }
}

// x += part after an NCCL all-reduce of the partials (at T = 2 the sum of
// the two partials is the same in either order, so x gets the peer
// exchange's bits).
__global__ void __launch_bounds__(256) k_tp_add(float *x, int n, const float *part) {
  pdl_trigger();
  pdl_wait();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) x[i] = fadd(x[i], part[i]);
}

// NCCL, loaded on first use so that the library does not depend on it: the
// process's copy when one is loaded already (a PyTorch process has one),
// else the system's libnccl.so.2.
struct NcclApi {
  bool ok = false;
  std::string why;
  ncclResult_t (*get_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*destroy)(ncclComm_t) = nullptr;
  const char *(*err)(ncclResult_t) = nullptr;
};

const NcclApi &nccl_api() {
  static const NcclApi api = [] {
    NcclApi a;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char *e = dlerror();
      a.why = e ? e : "dlopen(libnccl.so.2) failed";
      return a;
    }
    a.get_id = reinterpret_cast<decltype(a.get_id)>(dlsym(h, "ncclGetUniqueId"));
    a.init_rank = reinterpret_cast<decltype(a.init_rank)>(dlsym(h, "ncclCommInitRank"));
    a.all_reduce = reinterpret_cast<decltype(a.all_reduce)>(dlsym(h, "ncclAllReduce"));
    a.destroy = reinterpret_cast<decltype(a.destroy)>(dlsym(h, "ncclCommDestroy"));
    a.err = reinterpret_cast<decltype(a.err)>(dlsym(h, "ncclGetErrorString"));
    a.ok = a.get_id && a.init_rank && a.all_reduce && a.destroy && a.err;
    if (!a.ok) a.why = "libnccl.so.2 lacks an entry point";
    return a;
  }();
  return api;
}

__global__ void __launch_bounds__(256) k_tp_sum(float *x, int n, const float *slots, const unsigned long long *flags,
                                                int world, unsigned long long seq, int *err) {
  pdl_trigger();
  pdl_wait();
  if (!wait_flags(flags, world, seq, err)) return;
  const float *base = slots + (size_t)(seq & 1ULL) * world * n;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float s = __ldcg(base + i);
    for (int r = 1; r < world; r++) s = fadd(s, __ldcg(base + (size_t)r * n + i));
    x[i] = fadd(x[i], s);
  }
}

// The local shard's first maximum (as k_argmax: strict '>', NaN never wins,
// lowest index on ties), published to every rank as {value, global index}.
__global__ void __launch_bounds__(1024) k_tp_argmax_push(const float *__restrict__ x, int n, int vocab0, TpPeers P,
                                                         int rank, int world, unsigned long long seq) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_trigger();
  pdl_wait();
  float bv = -INFINITY;
  int bi = INT_MAX;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = x[i];
    if (v > bv) { bv = v; bi = i; }
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
    const int gi = bi == INT_MAX ? -1 : vocab0 + bi;
    const int par = (int)(seq & 1ULL);
    for (int dst = 0; dst < world; dst++) {
      float2 *slot = P.amax[dst] + par * world + rank;
      __stcg(slot, make_float2(bv, __int_as_float(gi)));
    }
    __threadfence_system();
    for (int dst = 0; dst < world; dst++) st_release_sys(P.flags[dst] + rank, seq);
  }
}

// The token: the first maximum over the shards, fed back for the next step
// (ids[0] = tok, pos += 1, hist[step++] = tok).
__global__ void k_tp_pick(const float2 *amax, const unsigned long long *flags, int world, unsigned long long seq,
                          uint32_t *ids, int *pos, uint32_t *hist, int *step, int *err) {
  pdl_trigger();
  pdl_wait();
  if (!wait_flags(flags, world, seq, err)) return;
  if (threadIdx.x != 0) return;
  float v[TP_MAX];
  int ix[TP_MAX];
  const int par = (int)(seq & 1ULL);
  for (int r = 0; r < world; r++) {
    const float2 a = __ldcg(amax + par * world + r);
    v[r] = a.x;
    ix[r] = __float_as_int(a.y);
  }
  const uint32_t tok = tp_pick(v, ix, world);
  ids[0] = tok;
  pos[0] += 1;
  hist[*step] = tok;
  *step += 1;
}

// Synthetic weights, generated on the device from (seed, tensor, global row,
// global block), so every split of the same model holds the same values.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
__device__ __forceinline__ float unit_u(uint64_t h) { return (float)(h >> 40) * (1.0f / 16777216.0f); }

__global__ void k_tp_synth(int type, uint8_t *out, int rows, int nkb, long row0, int kb0, int bb, uint64_t tseed) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < (long)rows * nkb; i += (long)gridDim.x * blockDim.x) {
    const long r = i / nkb;
    const int b = (int)(i - r * nkb);
    const uint64_t h = mix64(tseed ^ mix64((uint64_t)(row0 + r) * 0x100000001B3ULL + (uint64_t)(kb0 + b)));
    uint8_t *blk = out + i * bb;
    for (int w = 0; w < bb; w++) blk[w] = (uint8_t)(mix64(h + (uint64_t)(w >> 3)) >> (8 * (w & 7)));
    const float u = unit_u(h);
    if (type == T_Q4_K) {  // dequantised std about 0.02, mean about 0 (dmin = 7.5 d)
      const float d = 7.75e-5f * (0.75f + 0.5f * u);
      const __half hd = __float2half_rn(d), hm = __float2half_rn(7.5f * d);
      memcpy(blk, &hd, 2);
      memcpy(blk + 2, &hm, 2);
    } else if (type == T_Q6_K) {
      for (int w = 192; w < 208; w++) blk[w] = (uint8_t)((int)(blk[w] & 63) - 32);
      const __half hd = __float2half_rn(5.8e-5f * (0.75f + 0.5f * u));
      memcpy(blk + 208, &hd, 2);
    } else if (type == T_Q8_0) {
      const __half hd = __float2half_rn(2.7e-4f * (0.75f + 0.5f * u));
      memcpy(blk, &hd, 2);
    } else {  // Q4_0
      const __half hd = __float2half_rn(4.3e-3f * (0.75f + 0.5f * u));
      memcpy(blk, &hd, 2);
    }
  }
}

__global__ void k_tp_norm(float *w, int n, uint64_t tseed) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    w[i] = 1.0f + 0.04f * (unit_u(mix64(tseed + (uint64_t)i)) - 0.5f);
}

uint64_t host_mix(uint64_t z) {
  z += 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

}  // namespace

bool tp_split(const Config &c, int vocab, int rank, int world, int o_block, int down_block, TpSplit &s,
              std::string &why) {
  if (world < 1 || world > TP_MAX || rank < 0 || rank >= world) {
    why = "rank / world out of range (world 1..8)";
    return false;
  }
  if (c.n_head % world || c.n_head_kv % world || c.n_ff % world) {
    why = "heads, kv heads and FFN rows must divide by the world size";
    return false;
  }
  s.nh = c.n_head / world;
  s.nkv = c.n_head_kv / world;
  s.ff = c.n_ff / world;
  if ((s.nh * c.head_dim) % o_block || (s.nh * c.head_dim) % 32) {
    why = "the o matrix's k slice (local heads x head_dim) must be a multiple of its block size";
    return false;
  }
  if (s.ff % down_block || s.ff % 32) {
    why = "the down matrix's k slice (n_ff / world) must be a multiple of its block size";
    return false;
  }
  const int per = (vocab + world - 1) / world;
  s.vocab0 = std::min(vocab, rank * per);
  s.nvocab = std::min(vocab, s.vocab0 + per) - s.vocab0;
  if (s.nvocab < 1) {
    why = "vocabulary smaller than the world size";
    return false;
  }
  return true;
}

TpEngine::~TpEngine() {
  if (st_) cudaStreamSynchronize(st_);
  if (nccl_comm_) nccl_api().destroy(static_cast<ncclComm_t>(nccl_comm_));
  for (void *p : peer_base_)
    if (p) cudaIpcCloseMemHandle(p);
  cudaFree(d_weights_);
  cudaFree(d_kcache_);
  cudaFree(d_vcache_);
  cudaFree(d_rope_cos_);
  cudaFree(d_rope_sin_);
  cudaFree(d_arena_);
  cudaFree(d_x_);
  cudaFreeHost(h_ids_);
  cudaFreeHost(h_pos_);
  if (st_) cudaStreamDestroy(st_);
}

int TpEngine::create(int device, int n_ctx, int rank, int world) {
  if (n_ctx <= 0 || world < 1 || world > TP_MAX || rank < 0 || rank >= world)
    return set_error(PK_ERR_INVALID, "n_ctx must be > 0, world in 1..8 and rank in 0..world-1");
  int ndev = 0;
  PK_CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return set_error(PK_ERR_INVALID, "no CUDA device " + std::to_string(device));
  device_ = device;
  n_ctx_ = n_ctx;
  rank_ = rank;
  world_ = world;
  PK_CK(cudaSetDevice(device_));
  PK_CK(cudaStreamCreateWithFlags(&st_, cudaStreamNonBlocking));
  PK_CK(cudaHostAlloc((void **)&h_ids_, (size_t)n_ctx_ * sizeof(uint32_t), cudaHostAllocDefault));
  PK_CK(cudaHostAlloc((void **)&h_pos_, (size_t)n_ctx_ * sizeof(int), cudaHostAllocDefault));
  return PK_OK;
}

size_t TpEngine::exchange_bytes() const {
  return a256((size_t)2 * world_ * cfg_.n_embd * 4) + 256 + a256((size_t)world_ * 8);
}

int TpEngine::ipc_handle(void *out) {
  if (!loaded_) return set_error(PK_ERR_INVALID, "load a model before exchanging handles");
  cudaIpcMemHandle_t h;
  PK_CK(cudaSetDevice(device_));
  PK_CK(cudaIpcGetMemHandle(&h, d_x_));
  std::memcpy(out, &h, sizeof(h));
  return PK_OK;
}

int TpEngine::open_peers(const void *handles) {
  if (!loaded_) return set_error(PK_ERR_INVALID, "load a model before opening peers");
  if (peers_open_) return world_ == 1 ? PK_OK : set_error(PK_ERR_INVALID, "peers already open");
  PK_CK(cudaSetDevice(device_));
  const size_t sl = a256((size_t)2 * world_ * cfg_.n_embd * 4);
  for (int r = 0; r < world_; r++) {
    uint8_t *base = d_x_;
    if (r != rank_) {
      cudaIpcMemHandle_t h;
      std::memcpy(&h, (const uint8_t *)handles + r * sizeof(cudaIpcMemHandle_t), sizeof(h));
      void *p = nullptr;
      PK_CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
      peer_base_[r] = p;
      base = (uint8_t *)p;
    }
    peers_.slots[r] = (float *)base;
    peers_.amax[r] = (float2 *)(base + sl);
    peers_.flags[r] = (unsigned long long *)(base + sl + 256);
  }
  peers_open_ = true;
  return PK_OK;
}

// The rank's shard of every matrix, from a GGUF file (same checks as Engine::load).
int TpEngine::load(const char *path) {
  if (!st_) return set_error(PK_ERR_INVALID, "engine not created");
  if (loaded_) return set_error(PK_ERR_INVALID, "engine already holds a model");
  PK_CK(cudaSetDevice(device_));
  Gguf g;
  std::string err;
  if (!g.open(path, err)) return set_error(PK_ERR_IO, err);
  Config c;
  int rc = config_from_gguf(g, c);
  if (rc) return rc;
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
  const int vocab = (int)embd.ne1;
  const size_t qdim = (size_t)c.n_head * c.head_dim, kdim = (size_t)c.n_head_kv * c.head_dim;
  if ((rc = check_shape(output, c.n_embd, vocab)) || (rc = check_shape(onorm, c.n_embd, 1))) return rc;
  int o_block = 32, down_block = 32;
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
    int be, bb;
    type_block(l.o.type, &be, &bb);
    o_block = std::max(o_block, be);
    type_block(l.down.type, &be, &bb);
    down_block = std::max(down_block, be);
  }
  if (!type_is_matvec(output.type)) return set_error(PK_ERR_UNSUPPORTED, "output: unsupported type");
  std::string why;
  if (!tp_split(c, vocab, rank_, world_, o_block, down_block, sp_, why)) return set_error(PK_ERR_UNSUPPORTED, why);

  // shard sizes
  auto row_shard = [&](const TRef &t, size_t r0, size_t nr) { return a256(packed_bytes(t.type, (int)t.ne0, (int)nr)); };
  auto k_shard = [&](const TRef &t, size_t k) { return a256(packed_bytes(t.type, (int)k, (int)t.ne1)); };
  const size_t qd = (size_t)sp_.nh * c.head_dim, kd = (size_t)sp_.nkv * c.head_dim;
  size_t total = 256, max_raw = 0;
  stream_bytes_ = 0;
  auto raw_rows = [&](const TRef &t, size_t nr) { return t.row_bytes * nr; };
  for (auto &l : L) {
    total += row_shard(l.q, 0, qd) + row_shard(l.k, 0, kd) + row_shard(l.v, 0, kd) + k_shard(l.o, qd) +
             row_shard(l.gate, 0, sp_.ff) + row_shard(l.up, 0, sp_.ff) + k_shard(l.down, sp_.ff) +
             2 * a256((size_t)c.n_embd * 4);
    max_raw = std::max({max_raw, raw_rows(l.q, qd), raw_rows(l.gate, sp_.ff), l.o.row_bytes * l.o.ne1,
                        l.down.row_bytes * l.down.ne1});
    stream_bytes_ += raw_rows(l.q, qd) + raw_rows(l.k, kd) + raw_rows(l.v, kd) + raw_rows(l.gate, sp_.ff) +
                     raw_rows(l.up, sp_.ff) + l.o.row_bytes * l.o.ne1 * qd / qdim +
                     l.down.row_bytes * l.down.ne1 * sp_.ff / c.n_ff + 2 * (size_t)c.n_embd * 4;
  }
  total += row_shard(output, 0, sp_.nvocab) + a256(embd.row_bytes * embd.ne1) + a256((size_t)c.n_embd * 4);
  max_raw = std::max(max_raw, output.row_bytes * (size_t)sp_.nvocab);
  stream_bytes_ += output.row_bytes * (size_t)sp_.nvocab + embd.row_bytes + (size_t)c.n_embd * 4;
  PK_CK(cudaMalloc((void **)&d_weights_, total));
  weight_bytes_ = total;
  uint8_t *staging = nullptr;
  PK_CK(cudaMalloc((void **)&staging, a256(max_raw)));
  size_t off = 0;
  const uint8_t *file = g.data();
  // rows [r0, r0 + nr) of t
  auto up_rows = [&](const TRef &t, size_t r0, size_t nr, DevTensor &dst) -> int {
    uint8_t *slot = d_weights_ + off;
    off += row_shard(t, r0, nr);
    PK_CK(cudaMemcpyAsync(staging, file + t.off + r0 * t.row_bytes, t.row_bytes * nr, cudaMemcpyHostToDevice, st_));
    PK_CK(launch_pack(t.type, staging, t.row_bytes, (int)t.ne0, (int)nr, slot, st_));
    PK_CK(cudaStreamSynchronize(st_));
    dst = packed_view(t.type, (int)t.ne0, (int)nr, slot);
    return PK_OK;
  };
  // columns [k0, k0 + k) of every row of t
  auto up_cols = [&](const TRef &t, size_t k0, size_t k, DevTensor &dst) -> int {
    int be, bb;
    type_block(t.type, &be, &bb);
    const size_t b0 = k0 / be * bb, w = k / be * bb;
    uint8_t *slot = d_weights_ + off;
    off += k_shard(t, k);
    PK_CK(cudaMemcpy2DAsync(staging, w, file + t.off + b0, t.row_bytes, w, t.ne1, cudaMemcpyHostToDevice, st_));
    PK_CK(launch_pack(t.type, staging, w, (int)k, (int)t.ne1, slot, st_));
    PK_CK(cudaStreamSynchronize(st_));
    dst = packed_view(t.type, (int)k, (int)t.ne1, slot);
    return PK_OK;
  };
  auto up_norm = [&](const TRef &t, float **dst) -> int {
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
    const LRef &l = L[i];
    if ((rc = up_rows(l.q, rank_ * qd, qd, d.q)) || (rc = up_rows(l.k, rank_ * kd, kd, d.k)) ||
        (rc = up_rows(l.v, rank_ * kd, kd, d.v)) || (rc = up_cols(l.o, rank_ * qd, qd, d.o)) ||
        (rc = up_rows(l.gate, (size_t)rank_ * sp_.ff, sp_.ff, d.gate)) ||
        (rc = up_rows(l.up, (size_t)rank_ * sp_.ff, sp_.ff, d.up)) ||
        (rc = up_cols(l.down, (size_t)rank_ * sp_.ff, sp_.ff, d.down)) || (rc = up_norm(l.an, &d.attn_norm)) ||
        (rc = up_norm(l.fn, &d.ffn_norm)))
      break;
  }
  if (!rc && !(rc = up_rows(output, sp_.vocab0, sp_.nvocab, output_))) rc = up_norm(onorm, &output_norm_);
  cudaFree(staging);
  if (rc) return rc;
  embd_raw_ = d_weights_ + off;
  PK_CK(cudaMemcpyAsync(embd_raw_, file + embd.off, embd.row_bytes * embd.ne1, cudaMemcpyHostToDevice, st_));
  embd_type_ = embd.type;
  embd_row_bytes_ = embd.row_bytes;
  return finish_load(c, vocab);
}

// An M70-shaped (or any) llama stack with synthetic blocks generated on the
// device: Q4_K q/k/o/gate/up/down, Q6_K v and output, Q4_K embedding, f32
// norms 1 +- 0.02.  Only this rank's shard is generated.
int TpEngine::load_synthetic(const Config &cin, int vocab, uint64_t seed) {
  if (!st_) return set_error(PK_ERR_INVALID, "engine not created");
  if (loaded_) return set_error(PK_ERR_INVALID, "engine already holds a model");
  PK_CK(cudaSetDevice(device_));
  Config c = cin;
  if (c.n_layer < 1 || c.n_embd % 256 || c.n_ff % 256 || c.head_dim % 4 || c.head_dim > 256 || c.n_head_kv < 1 ||
      c.n_head % c.n_head_kv || vocab < 1 || c.n_rot < 2 || c.n_rot > c.head_dim || c.n_rot % 2)
    return set_error(PK_ERR_INVALID, "synthetic model: unsupported dimensions");
  std::string why;
  if (!tp_split(c, vocab, rank_, world_, 256, 256, sp_, why)) return set_error(PK_ERR_UNSUPPORTED, why);
  const size_t qd = (size_t)sp_.nh * c.head_dim, kd = (size_t)sp_.nkv * c.head_dim;
  auto pk_bytes = [&](int t, size_t k, size_t rows) { return a256(packed_bytes(t, (int)k, (int)rows)); };
  auto rb = [&](int t, size_t k) {
    int be, bb;
    type_block(t, &be, &bb);
    return k / be * bb;
  };
  const size_t ne = c.n_embd;
  size_t total = 256, max_raw = 0;
  const size_t per_layer = pk_bytes(T_Q4_K, ne, qd) + pk_bytes(T_Q4_K, ne, kd) + pk_bytes(T_Q6_K, ne, kd) +
                           pk_bytes(T_Q4_K, qd, ne) + 2 * pk_bytes(T_Q4_K, ne, sp_.ff) + pk_bytes(T_Q4_K, sp_.ff, ne) +
                           2 * a256(ne * 4);
  total += per_layer * c.n_layer + pk_bytes(T_Q6_K, ne, sp_.nvocab) + a256(rb(T_Q4_K, ne) * vocab) + a256(ne * 4);
  max_raw = std::max({rb(T_Q4_K, ne) * std::max(qd, (size_t)sp_.ff), rb(T_Q4_K, qd) * ne, rb(T_Q4_K, sp_.ff) * ne,
                      rb(T_Q6_K, ne) * (size_t)sp_.nvocab});
  stream_bytes_ = (size_t)c.n_layer * (rb(T_Q4_K, ne) * (qd + kd + 2 * sp_.ff) + rb(T_Q6_K, ne) * kd +
                                       rb(T_Q4_K, qd) * ne + rb(T_Q4_K, sp_.ff) * ne + 2 * ne * 4) +
                  rb(T_Q6_K, ne) * sp_.nvocab + rb(T_Q4_K, ne) + ne * 4;
  PK_CK(cudaMalloc((void **)&d_weights_, total));
  weight_bytes_ = total;
  uint8_t *staging = nullptr;
  PK_CK(cudaMalloc((void **)&staging, a256(max_raw)));
  size_t off = 0;
  uint64_t tid = 0;
  const int grid = 148 * 8;
  // rows [r0, r0 + nr) x blocks [kb0, kb0 + nkb) of a (tensor id) matrix of row length k_full
  auto gen = [&](int t, size_t k, size_t r0, size_t nr, size_t k0, DevTensor &dst) -> int {
    int be, bb;
    type_block(t, &be, &bb);
    const uint64_t ts = host_mix(seed * 0x9E3779B97F4A7C15ULL + (++tid));
    uint8_t *slot = d_weights_ + off;
    off += pk_bytes(t, k, nr);
    PK_CK(tp_launch(k_tp_synth, dim3(grid), dim3(256), 0, st_, t, staging, (int)nr, (int)(k / be), (long)r0,
                    (int)(k0 / be), bb, ts));
    PK_CK(launch_pack(t, staging, k / be * bb, (int)k, (int)nr, slot, st_));
    PK_CK(cudaStreamSynchronize(st_));
    dst = packed_view(t, (int)k, (int)nr, slot);
    return PK_OK;
  };
  auto norm = [&](float **dst) -> int {
    float *slot = (float *)(d_weights_ + off);
    off += a256(ne * 4);
    PK_CK(tp_launch(k_tp_norm, dim3(16), dim3(256), 0, st_, slot, (int)ne, host_mix(seed + 0x51ED * (++tid))));
    *dst = slot;
    return PK_OK;
  };
  int rc = PK_OK;
  layers_.resize(c.n_layer);
  for (int i = 0; i < c.n_layer && !rc; i++) {
    LayerDev &d = layers_[i];
    if ((rc = gen(T_Q4_K, ne, rank_ * qd, qd, 0, d.q)) || (rc = gen(T_Q4_K, ne, rank_ * kd, kd, 0, d.k)) ||
        (rc = gen(T_Q6_K, ne, rank_ * kd, kd, 0, d.v)) || (rc = gen(T_Q4_K, qd, 0, ne, rank_ * qd, d.o)) ||
        (rc = gen(T_Q4_K, ne, (size_t)rank_ * sp_.ff, sp_.ff, 0, d.gate)) ||
        (rc = gen(T_Q4_K, ne, (size_t)rank_ * sp_.ff, sp_.ff, 0, d.up)) ||
        (rc = gen(T_Q4_K, sp_.ff, 0, ne, (size_t)rank_ * sp_.ff, d.down)) || (rc = norm(&d.attn_norm)) ||
        (rc = norm(&d.ffn_norm)))
      break;
  }
  if (!rc && !(rc = gen(T_Q6_K, ne, sp_.vocab0, sp_.nvocab, 0, output_))) rc = norm(&output_norm_);
  cudaFree(staging);
  if (rc) return rc;
  // the embedding: raw Q4_K rows, every rank the whole table
  embd_raw_ = d_weights_ + off;
  embd_type_ = T_Q4_K;
  embd_row_bytes_ = rb(T_Q4_K, ne);
  PK_CK(tp_launch(k_tp_synth, dim3(grid), dim3(256), 0, st_, (int)T_Q4_K, embd_raw_, vocab, (int)(ne / 256), 0L, 0,
                  144, host_mix(seed ^ 0xE3BDULL)));
  PK_CK(cudaStreamSynchronize(st_));
  return finish_load(c, vocab);
}

// KV cache, RoPE tables, scratch and the exchange buffer.
int TpEngine::finish_load(const Config &c, int vocab) {
  cfg_ = c;
  vocab_ = vocab;
  const int dh = c.head_dim, ne = c.n_embd;
  const size_t kvb = (size_t)c.n_layer * sp_.nkv * n_ctx_ * dh * 4;
  PK_CK(cudaMalloc((void **)&d_kcache_, kvb));
  PK_CK(cudaMalloc((void **)&d_vcache_, kvb));
  PK_CK(cudaMemsetAsync(d_kcache_, 0, kvb, st_));
  PK_CK(cudaMemsetAsync(d_vcache_, 0, kvb, st_));
  // RoPE tables as Engine::load (model.rs:414-417, 452-457)
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
  PK_CK(cudaMemcpy(d_rope_cos_, tc.data(), tc.size() * 4, cudaMemcpyHostToDevice));
  PK_CK(cudaMemcpy(d_rope_sin_, ts.data(), ts.size() * 4, cudaMemcpyHostToDevice));
  // scratch
  const size_t qd = (size_t)sp_.nh * dh;
  const std::vector<size_t> sizes = {(size_t)ne * 4, qd * 4, qd * 4, (size_t)sp_.ff * 4, (size_t)ne * 4,
                                     (size_t)sp_.nvocab * 4, (size_t)sp_.nh * n_ctx_ * 4, 16, (size_t)n_ctx_ * 4 + 16,
                                     16, 16, 16, 16};
  size_t arena = 0;
  for (size_t s : sizes) arena += a256(s);
  PK_CK(cudaMalloc((void **)&d_arena_, arena));
  PK_CK(cudaMemsetAsync(d_arena_, 0, arena, st_));
  uint8_t *pa = d_arena_;
  size_t si = 0;
  auto take = [&]() {
    uint8_t *r = pa;
    pa += a256(sizes[si++]);
    return r;
  };
  x_ = (float *)take(); q_ = (float *)take(); attn_ = (float *)take(); h_ = (float *)take(); part_ = (float *)take();
  logits_ = (float *)take(); scores_ = (float *)take(); d_ids_ = (uint32_t *)take(); d_hist_ = (uint32_t *)take();
  d_pos_ = (int *)take(); d_step_ = (int *)take(); d_err_ = (int *)take(); d_count_ = (unsigned *)take();
  // exchange buffer: slots [2][T][n_embd] | amax [2][T] | flags [T]
  PK_CK(cudaMalloc((void **)&d_x_, exchange_bytes()));
  PK_CK(cudaMemsetAsync(d_x_, 0, exchange_bytes(), st_));
  PK_CK(cudaStreamSynchronize(st_));
  loaded_ = true;
  if (world_ == 1) return open_peers(nullptr);
  return PK_OK;
}

int TpEngine::allreduce_add(float *part, float *x) {
  ++seq_;
  const int ne = cfg_.n_embd;
  if (nccl_comm_) {
    const NcclApi &n = nccl_api();
    const ncclResult_t r =
        n.all_reduce(part, part, (size_t)ne, ncclFloat32, ncclSum, static_cast<ncclComm_t>(nccl_comm_), st_);
    if (r != ncclSuccess) return set_error(PK_ERR_CUDA, std::string("ncclAllReduce: ") + n.err(r));
    PK_CK(tp_launch(k_tp_add, dim3(8), dim3(256), 0, st_, x, ne, (const float *)part));
    return PK_OK;
  }
  PK_CK(tp_launch(k_tp_push, dim3(TP_PUSH_CTAS), dim3(256), 0, st_, part, ne, peers_, rank_, world_, seq_, d_count_));
  PK_CK(tp_launch(k_tp_sum, dim3(8), dim3(256), 0, st_, x, ne, (const float *)peers_.slots[rank_],
                  (const unsigned long long *)peers_.flags[rank_], world_, seq_, d_err_));
  return PK_OK;
}

int tp_nccl_id_bytes() { return (int)sizeof(ncclUniqueId); }

int tp_nccl_id(void *out) {
  if (!out) return set_error(PK_ERR_INVALID, "null id buffer");
  const NcclApi &n = nccl_api();
  if (!n.ok) return set_error(PK_ERR_UNSUPPORTED, "NCCL is not available: " + n.why);
  ncclUniqueId id;
  const ncclResult_t r = n.get_id(&id);
  if (r != ncclSuccess) return set_error(PK_ERR_CUDA, std::string("ncclGetUniqueId: ") + n.err(r));
  std::memcpy(out, &id, sizeof id);
  return PK_OK;
}

// Collective over the T ranks: every rank calls it with rank 0's id and
// blocks until all have joined.
int TpEngine::use_nccl(const void *id) {
  if (!peers_open_) return set_error(PK_ERR_INVALID, "open the peers first");
  if (!id) return set_error(PK_ERR_INVALID, "null NCCL id");
  if (nccl_comm_) return set_error(PK_ERR_INVALID, "the NCCL exchange is already in use");
  const NcclApi &n = nccl_api();
  if (!n.ok) return set_error(PK_ERR_UNSUPPORTED, "NCCL is not available: " + n.why);
  PK_CK(cudaSetDevice(device_));
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof uid);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = n.init_rank(&comm, world_, uid, rank_);
  if (r != ncclSuccess) return set_error(PK_ERR_CUDA, std::string("ncclCommInitRank: ") + n.err(r));
  nccl_comm_ = comm;
  return PK_OK;
}

// One token at d_pos_ with id d_ids_: the b = 1 op sequence (model.rs:857-1170)
// on this rank's shard, with the two collectives per layer; with the head
// (feedback) the first maximum over all shards becomes the next token.
int TpEngine::step(bool feedback) {
  const Config &c = cfg_;
  const int ne = c.n_embd, dh = c.head_dim;
  const size_t layer_kv = (size_t)sp_.nkv * n_ctx_ * dh;
  PK_CK(launch_dequant_rows(embd_type_, embd_raw_, embd_row_bytes_, ne, d_ids_, 1, x_, st_));
  AttnArgs at{};
  at.q = q_; at.pos = d_pos_; at.out = attn_; at.b = 1; at.n_head = sp_.nh; at.n_kv = sp_.nkv; at.dh = dh;
  at.n_ctx = n_ctx_; at.scale = 1.0f / sqrtf((float)dh); at.scores = scores_;
  for (int l = 0; l < c.n_layer; l++) {
    if (g_stop.load()) return set_error(PK_ERR_STOPPED, "generation stopped");
    const LayerDev &L = layers_[l];
    float *kc = d_kcache_ + l * layer_kv, *vc = d_vcache_ + l * layer_kv;
    QkvArgs qa;
    qa.wq = L.q; qa.wk = L.k; qa.wv = L.v;
    qa.src.x = x_; qa.src.nw = L.attn_norm; qa.src.eps = c.rms_eps;
    qa.pos = d_pos_; qa.rope_cos = d_rope_cos_; qa.rope_sin = d_rope_sin_;
    qa.half = c.n_rot / 2; qa.dh = dh; qa.n_ctx = n_ctx_;
    qa.qout = q_; qa.kcache = kc; qa.vcache = vc;
    PK_CK(launch_qkv_b1(qa, st_));
    at.kcache = kc; at.vcache = vc;
    PK_CK(launch_attention(at, st_));
    B1Src so;
    so.x = attn_;
    PK_CK(launch_mv_b1(L.o, so, part_, false, st_));
    int rc = allreduce_add(part_, x_);
    if (rc) return rc;
    B1Src sf;
    sf.x = x_; sf.nw = L.ffn_norm; sf.eps = c.rms_eps;
    PK_CK(launch_gateup_b1(L.gate, L.up, sf, h_, st_));
    B1Src sd;
    sd.x = h_;
    PK_CK(launch_mv_b1(L.down, sd, part_, false, st_));
    if ((rc = allreduce_add(part_, x_))) return rc;
  }
  if (!feedback) return PK_OK;
  B1Src sh;
  sh.x = x_; sh.nw = output_norm_; sh.eps = c.rms_eps;
  PK_CK(launch_mv_b1(output_, sh, logits_, false, st_));
  ++seq_;
  PK_CK(tp_launch(k_tp_argmax_push, dim3(1), dim3(1024), 0, st_, (const float *)logits_, sp_.nvocab, sp_.vocab0,
                  peers_, rank_, world_, seq_));
  PK_CK(tp_launch(k_tp_pick, dim3(1), dim3(32), 0, st_, (const float2 *)peers_.amax[rank_],
                  (const unsigned long long *)peers_.flags[rank_], world_, seq_, d_ids_, d_pos_, d_hist_, d_step_,
                  d_err_));
  return PK_OK;
}

int TpEngine::check_error() {
  int err = 0;
  PK_CK(cudaMemcpy(&err, d_err_, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) {
    PK_CK(cudaMemset(d_err_, 0, sizeof(int)));
    return set_error(PK_ERR_TIMEOUT, "tensor-parallel exchange: rank " + std::to_string(err - 1) +
                                         " did not publish within the wait bound");
  }
  return PK_OK;
}

int TpEngine::prefill(const uint32_t *prompt, int n) {
  if (!loaded_ || !peers_open_) return set_error(PK_ERR_INVALID, "load a model and open the peers first");
  if (n <= 0 || n > n_ctx_) return set_error(PK_ERR_CONTEXT_FULL, "prompt empty or longer than n_ctx");
  for (int i = 0; i < n; i++)
    if (prompt[i] >= (uint32_t)vocab_) return set_error(PK_ERR_INVALID, "token out of vocab");
  PK_CK(cudaSetDevice(device_));
  for (int i = 0; i < n; i++) {
    h_ids_[i] = prompt[i];
    h_pos_[i] = i;
  }
  PK_CK(cudaMemsetAsync(d_step_, 0, sizeof(int), st_));
  for (int i = 0; i < n; i++) {
    PK_CK(cudaMemcpyAsync(d_ids_, h_ids_ + i, sizeof(uint32_t), cudaMemcpyHostToDevice, st_));
    PK_CK(cudaMemcpyAsync(d_pos_, h_pos_ + i, sizeof(int), cudaMemcpyHostToDevice, st_));
    const int rc = step(i == n - 1);
    if (rc) {
      cudaStreamSynchronize(st_);
      return rc;
    }
  }
  PK_CK(cudaStreamSynchronize(st_));
  PK_CK(cudaGetLastError());
  const int rc = check_error();
  if (rc) return rc;
  PK_CK(cudaMemcpy(&last_tok_, d_hist_, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  next_pos_ = n;
  have_tok_ = true;
  return PK_OK;
}

// n_steps tokens, as Engine::decode_steps_device: the token picked last (by
// the prefill or the previous call) and the next n_steps - 1; each of the
// n_steps steps runs that token through the model and picks the next, so
// the token after them is ready for the next call.
int TpEngine::decode(int n_steps, uint32_t *out_ids, float *device_ms) {
  if (!have_tok_) return set_error(PK_ERR_INVALID, "run a prefill first");
  if (n_steps < 1) return set_error(PK_ERR_INVALID, "n_steps must be >= 1");
  if (next_pos_ + n_steps > n_ctx_) return set_error(PK_ERR_CONTEXT_FULL, "context full");
  PK_CK(cudaSetDevice(device_));
  PK_CK(cudaMemsetAsync(d_step_, 0, sizeof(int), st_));
  cudaEvent_t e0, e1;
  PK_CK(cudaEventCreate(&e0));
  PK_CK(cudaEventCreate(&e1));
  cudaError_t e = cudaEventRecord(e0, st_);
  int rc = PK_OK;
  for (int i = 0; i < n_steps && e == cudaSuccess && !rc; i++) rc = step(true);
  if (e == cudaSuccess) e = cudaEventRecord(e1, st_);
  std::vector<uint32_t> hist(n_steps + 1);
  if (e == cudaSuccess) e = cudaMemcpyAsync(hist.data() + 1, d_hist_, (size_t)n_steps * 4, cudaMemcpyDeviceToHost, st_);
  const cudaError_t es = cudaStreamSynchronize(st_);
  float ms = 0.0f;
  if (e == cudaSuccess && es == cudaSuccess) e = cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc) return rc;
  if (e != cudaSuccess) return cuda_error(e, "tp decode");
  if (es != cudaSuccess) return cuda_error(es, "tp decode");
  if ((rc = check_error())) return rc;
  hist[0] = last_tok_;
  last_tok_ = hist[n_steps];
  if (out_ids) std::memcpy(out_ids, hist.data(), (size_t)n_steps * 4);
  if (device_ms) *device_ms = ms;
  next_pos_ += n_steps;
  return PK_OK;
}

int TpEngine::logits(float *out, int n, int *n_local, int *vocab0) {
  if (!loaded_) return set_error(PK_ERR_INVALID, "no model loaded");
  const int m = std::min(n, sp_.nvocab);
  PK_CK(cudaMemcpy(out, logits_, (size_t)m * 4, cudaMemcpyDeviceToHost));
  if (n_local) *n_local = sp_.nvocab;
  if (vocab0) *vocab0 = sp_.vocab0;
  return PK_OK;
}

int TpEngine::info(pk_tp_info *o) const {
  if (!loaded_) return set_error(PK_ERR_INVALID, "no model loaded");
  std::memset(o, 0, sizeof(*o));
  o->rank = rank_;
  o->world = world_;
  o->n_layer = cfg_.n_layer;
  o->n_embd = cfg_.n_embd;
  o->n_head = cfg_.n_head;
  o->n_head_kv = cfg_.n_head_kv;
  o->head_dim = cfg_.head_dim;
  o->n_ff = cfg_.n_ff;
  o->n_vocab = vocab_;
  o->local_heads = sp_.nh;
  o->local_kv_heads = sp_.nkv;
  o->local_ff = sp_.ff;
  o->vocab0 = sp_.vocab0;
  o->local_vocab = sp_.nvocab;
  o->weight_bytes = weight_bytes_;
  o->stream_bytes = stream_bytes_;
  o->collectives_per_token = 2 * cfg_.n_layer + 1;
  return PK_OK;
}

}  // namespace pk
