/*
 * pk.h -- C ABI of libpocketinfer_b200.so, the B200 (sm_100a) implementation
 * of pocketinfer's decode token loop and its 32-token prefill.
 *
 * Every entry point is extern "C", takes plain pointers and sizes, returns an
 * int status (PK_OK == 0) and leaves a message for pk_last_error() on failure.
 * Nothing falls back to the CPU: a failure is an error status.
 *
 * Reference interfaces replaced (Aleinto97/pocket-workbench-android,
 * paths relative to rust/pocketinfer/src/):
 *   pk_supports            quant_int.rs:75-80 supported(), backend/opencl.rs:432-434 supports()
 *   pk_q8_quantize         quant_int.rs:17-56 Q8Act::prepare
 *   pk_matmul              model.rs:242-321 Pool::matmul (int8 act path, raw GGUF blocks)
 *   pk_pack_weights /
 *   pk_matmul_packed       the same contraction on the device weight layout
 *   pk_backend_*           backend/opencl.rs:261-500 OpenClBackend::{new,selftest,supports,matvec}
 *   pk_create/pk_load_gguf model.rs:698-723 Engine::load (+ gguf.rs, util.rs MappedFile)
 *   pk_forward             model.rs:825-831 Engine::forward
 *   pk_logits              model.rs:1231-1233 Engine::logits
 *   pk_argmax              sampler.rs:26-36 sample() with temp <= 0
 *   pk_generate            model.rs:1235-1352 Engine::generate (prefix-KV reuse included)
 *   pk_request_stop        util.rs:274-282 request_stop / STOP_REQUESTED
 *   pk_set_debug/get_dump  model.rs:870-872,942-1168 Engine.dbg intermediates
 *   pk_tokenizer_load, pk_tokenize, pk_token_bytes, pk_token_is_eog
 *                          tokenizer.rs:38-110 from_gguf, :187-224 encode, :226-250 decode_token,
 *                          :252-254 is_eog (pre-tokenizer patterns: regexlite.rs)
 *   pk_chat_apply etc.     chat.rs:16-18 is_minicpm5, :20-97 apply_minicpm5 / apply_generic,
 *                          :99-109 the thinking / direct suffixes
 *
 * Threading: one engine per host thread; calls on one engine are serialised
 * by the caller (the reference serialises with a global Mutex, jni.rs:211).
 * Op-level calls are ordered on the CUDA stream passed in (NULL = default).
 */
#ifndef PK_H
#define PK_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PK_OK 0
#define PK_ERR_INVALID 1      /* bad argument, shape or layout */
#define PK_ERR_UNSUPPORTED 2  /* tensor type not handled on the device */
#define PK_ERR_CUDA 3         /* CUDA runtime / launch failure */
#define PK_ERR_OOM 4          /* device or host allocation failed */
#define PK_ERR_IO 5           /* file or GGUF parse error */
#define PK_ERR_CONTEXT_FULL 6 /* position >= n_ctx */
#define PK_ERR_STOPPED 7      /* pk_request_stop() observed */
#define PK_ERR_TIMEOUT 8      /* a bounded device wait expired */

/* GGML tensor type ids (quant.rs:3-17). */
#define PK_TYPE_F32 0
#define PK_TYPE_F16 1
#define PK_TYPE_Q4_0 2
#define PK_TYPE_Q8_0 8
#define PK_TYPE_Q4_K 12
#define PK_TYPE_Q6_K 14
#define PK_TYPE_BF16 30

/* Last error message of the calling thread ("" if none). */
const char *pk_last_error(void);
/* ABI version: major * 100 + minor. */
int pk_version(void);
/* Architecture of the device code this library runs on the current device,
 * as CUDA reports it for a loaded kernel (cudaFuncAttributes::binaryVersion,
 * major * 10 + minor: 100 for sm_100a).  No reference counterpart. */
int pk_device_binary_version(int *out);

/* 1 if the device matvec handles ttype (Q4_K, Q6_K, Q4_0, Q8_0), else 0.
 * Replaces quant_int.rs:75-80 supported() and opencl.rs:432-434 supports(). */
int pk_supports(uint32_t ttype);

/* ---------------------------------------------------------------- op level */

/* The device exp used by softmax and SwiGLU: bit-identical to the C library's
 * expf, which the reference's f32::exp calls (model.rs:1042, 1113). Exported
 * so it can be verified.  x and out are device arrays of n floats. */
int pk_expf(const float *x, float *out, int n, void *stream);

/* Quantised activations, Q8Act layout (quant_int.rs:3-10), device memory:
 *   q   int8  [b][k]        (lane-major)
 *   d   float [b][k / 32]
 *   sum int32 [b][k / 32]
 * k must be a multiple of 32. */
typedef struct {
  int8_t *q;
  float *d;
  int32_t *sum;
  int k;
  int b;
} pk_q8act;

/* Q8Act::prepare (quant_int.rs:17-56).  x is feature-major [k][b] (x[i*b+bi]),
 * the reference's activation layout.  Bit-exact with the reference. */
int pk_q8_quantize(const float *x, int k, int b, pk_q8act *act, void *stream);

/* Pool::matmul with the int8 act path (model.rs:242-321, quant_int.rs:282-419).
 * w: device pointer to raw GGUF blocks, n_rows rows of row_bytes each.
 * out: [n_rows][b] (out[r*b + lane]), overwritten ("zero-filled then +=").
 * Q6_K/Q4_0/Q8_0 rows are first packed into a stream-ordered temporary
 * (cudaMallocAsync); callers that reuse a tensor should pack once with
 * pk_pack_weights and call pk_matmul_packed. */
int pk_matmul(uint32_t ttype, const void *w, size_t row_bytes, int k, int n_rows,
              const pk_q8act *act, float *out, void *stream);

/* pk_matmul that allocates no device memory.  No counterpart in the
 * reference, which has no device allocator to avoid.  Same arguments and
 * result as pk_matmul; the rows that pk_matmul packs into a temporary are
 * packed into one fixed scratch array inside this library's device image
 * instead, so a call needing more than PK_NOALLOC_SCRATCH_BYTES of packed
 * rows (pk_packed_bytes) fails with PK_ERR_INVALID before anything runs.
 * 16-byte aligned Q4_K rows are used in place and have no size limit.
 * The scratch's device memory is reserved on a device when CUDA loads the
 * library module that holds it, which it does lazily: at the first
 * pk_create, pk_backend_new or pk_matmul_noalloc on that device (each looks
 * up the scratch's address with that device current, cudaGetSymbolAddress).
 * A host that gives the device's free memory to its own pool must make one
 * of those calls on the device before it does, and the first
 * pk_matmul_noalloc call must come before any stream capture.  The address
 * is kept for the life of the process: a cudaDeviceReset after the first
 * call is not supported.  There is one scratch per device: calls that
 * overlap in time (other streams, other host threads) race on it and must be
 * serialised by the caller.  Nothing in the scratch needs to start at zero:
 * the pack kernel writes every byte the matvec then reads. */
#define PK_NOALLOC_SCRATCH_BYTES (16u << 20)
int pk_matmul_noalloc(uint32_t ttype, const void *w, size_t row_bytes, int k, int n_rows,
                      const pk_q8act *act, float *out, void *stream);

/* Which tensor-core kernel runs the multi-lane (b > 8) matvecs of this
 * process: every pk_matmul* call and every engine's prefill chunks.  No
 * counterpart in the reference (its lanes path is CPU code,
 * quant_int.rs:282-419).  PK_MATMUL_MMA_SYNC (the default): warp-level
 * int8 mma.sync tiles.  PK_MATMUL_TCGEN05: one tcgen05.mma per 32-element
 * block into TMEM, weights staged by tensor copies.  Both give the
 * reference's bits; b <= 8 always uses the mma.sync tiles.  The environment
 * variable PK_PREFILL_MMA=tc sets the tcgen05 path at load.  Calls in flight
 * keep the kernel they were launched with. */
#define PK_MATMUL_MMA_SYNC 0
#define PK_MATMUL_TCGEN05 1
int pk_set_matmul_path(int path);

/* Device weight layout: bytes needed for n_rows x k of ttype (>= raw size). */
size_t pk_packed_bytes(uint32_t ttype, int k, int n_rows);
/* Raw GGUF blocks (device) -> device layout (device, 16-byte aligned). */
int pk_pack_weights(uint32_t ttype, const void *raw, size_t row_bytes, int k, int n_rows,
                    void *packed, void *stream);
/* Same contraction as pk_matmul on packed weights; out [n_rows][b]. */
int pk_matmul_packed(uint32_t ttype, const void *packed, int k, int n_rows,
                     const pk_q8act *act, float *out, void *stream);

/* ------------------------------------------------- accelerator-backend level */

/* Mirrors OpenClBackend (backend/opencl.rs:261-500): weights are host
 * buffers (the GGUF mmap), copied to the device once and cached by
 * (pointer, length); x and out are host buffers; the call is synchronous.
 * x is quantised with Q8Act::prepare on the device, so results equal the
 * reference's int8 path (not the f32 OpenCL kernels). */
typedef struct pk_backend pk_backend;
int pk_backend_new(int device, pk_backend **out);
void pk_backend_free(pk_backend *be);
/* opencl.rs:391-430: one Q4_K and one Q6_K block against the f32 dot,
 * tolerance 2% + 0.01. */
int pk_backend_selftest(pk_backend *be);
int pk_backend_supports(pk_backend *be, uint32_t ttype);
int pk_backend_matvec(pk_backend *be, uint32_t ttype, const void *w, size_t w_len, int k,
                      const float *x, float *out, int n_rows);

/* ------------------------------------------------------------- engine level */

typedef struct pk_engine pk_engine;

typedef struct {
  int n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_rot, n_vocab, n_ctx;
  float rope_theta, rms_eps;
  size_t weight_bytes;      /* device weight bytes (packed layout) */
  size_t kv_bytes;          /* device KV cache bytes */
  size_t stream_bytes;      /* weight + norm + embedding-row bytes one decode token reads */
  int decode_kernels;       /* kernel launches per b == 1 decode step: 1 when the persistent
                               decode kernel runs this model, else the per-op sequence */
} pk_model_info;

typedef struct {
  float temp;     /* <= 0: greedy argmax */
  float top_p;
  uint64_t seed;  /* splitmix64 (sampler.rs:1-19) */
  int max_tokens;
  int stop_at_eog; /* 1: stop on an end-of-generation id (tokenizer.rs:252) */
} pk_gen_opts;

typedef struct {
  int prefill_tokens;
  int prefill_cached_tokens;
  double prefill_ms;
  int gen_tokens;
  double gen_ms;
  char stop[32]; /* "max_tokens" | "eog" | "user_stop" | "context_full" | "callback_error" */
} pk_gen_stats;

/* Token callback: return 0 to abort ("callback_error"). */
typedef int (*pk_token_cb)(uint32_t token, void *user);

/* Engine::load split in two: create the device context, then load a GGUF.
 * max_batch bounds the prefill chunk (<= 64, MAX_BATCH of model.rs:12). */
int pk_create(int device, int n_ctx, int max_batch, pk_engine **out);
int pk_load_gguf(pk_engine *eng, const char *path);
void pk_destroy(pk_engine *eng);
int pk_model_info_get(pk_engine *eng, pk_model_info *info);

/* Float order of the b = 1 decode step (no reference counterpart: the
 * reference has one order).  PK_ORDER_EXACT: every float operation in the
 * reference's order (model.rs:777-1170, quant_int.rs:282-419), so logits and
 * tokens are bit-identical to its CPU path.  PK_ORDER_FAST: the Q8
 * activations and every per-block integer dot stay bit-exact, and the float
 * combines of each matvec row, RMSNorm's sum of squares and the softmax and
 * value sums are regrouped into partial sums (within 1e-3 relative per
 * matvec).  Applies to pk_forward(n = 1), pk_generate's decode steps and
 * pk_decode_steps_device; prefill chunks always take the exact order.  The
 * default is PK_ORDER_EXACT, or PK_ORDER_FAST when the environment variable
 * PK_ORDER=fast is set at pk_create. */
#define PK_ORDER_EXACT 0
#define PK_ORDER_FAST 1
int pk_set_order(pk_engine *eng, int order);

/* No counterpart in the reference (its KvCache, model.rs:352-387, is f32; its
 * README:10,23 dropped an f16 cache): the entry type of the engine's K/V
 * caches, set after pk_create and before pk_load_gguf.  PK_KV_F16 stores
 * each K and V value rounded to nearest even, halving the cache (M26: 368,640
 * instead of 737,280 bytes a position); every later read converts it back
 * exactly, and all other arithmetic is unchanged.  With f16 entries decode
 * runs the per-op kernels and attention the per-(token, head) kernel. */
#define PK_KV_F32 0
#define PK_KV_F16 1
int pk_set_kv_type(pk_engine *eng, int type);

/* Engine::forward: invalidates prefix reuse.  ids/positions are host arrays. */
int pk_forward(pk_engine *eng, const uint32_t *ids, const int *positions, int n, int want_logits);
/* Copies the last logits (n_vocab floats) to host memory. */
int pk_logits(pk_engine *eng, float *out, int n);
/* Greedy sample of the current logits on the device (first maximum wins). */
int pk_argmax(pk_engine *eng, uint32_t *token);
/* sampler.rs:21-92 with temp > 0 (temperature, then top-p when 0 < top_p < 1) on device
 * logits[n]: the token into *tok (device), *rng_state (device, the splitmix64 state
 * Rng::new(seed) holds: seed + 0x9E3779B97F4A7C15) advanced when a draw happens.  Same
 * arithmetic and order as the reference; equal probabilities in the top-p sort are ordered by
 * index.  scratch: pk_sample_scratch_bytes(n) bytes of device memory, 256-byte aligned.
 * pk_generate uses it when pk_gen_opts.temp > 0. */
size_t pk_sample_scratch_bytes(int n);
int pk_sample(const float *logits, int n, float temp, float top_p, uint64_t *rng_state, void *scratch,
              uint32_t *tok, void *stream);
/* Engine::generate.  out_ids receives up to out_cap generated ids. */
int pk_generate(pk_engine *eng, const uint32_t *prompt, int n, const pk_gen_opts *opts,
                pk_token_cb cb, void *user, uint32_t *out_ids, int out_cap, int *n_out,
                pk_gen_stats *stats);

/* Greedy decode loop kept on the device: n_steps steps of (argmax of the
 * current logits -> feed the token back -> one b=1 forward), one CUDA-graph
 * launch per step and no host synchronisation between steps.  Writes the
 * produced ids; device_ms (nullable) receives the CUDA-event time of the
 * steps measured on the engine's stream. */
int pk_decode_steps_device(pk_engine *eng, int n_steps, uint32_t *out_ids, float *device_ms);
/* Rewinds the sequence to pos tokens (0 < pos <= current length), keeping the
 * current logits as the next step's input.  Positions >= pos are rewritten
 * before they are read again.  Invalidates prefix reuse beyond pos. */
int pk_set_position(pk_engine *eng, int pos);

/* Independent greedy streams on one engine, decoded together (no reference
 * counterpart: the reference's engine holds one sequence, engine.rs; these
 * serve many sequences per GPU).  Each stream has its own KV cache of n_ctx
 * positions; one step decodes one token of every stream with the weights read
 * once.  Every stream's tokens equal those pk_generate gives it alone.
 * pk_streams_begin allocates n_streams caches (1 <= n_streams <= max_batch,
 * at most 64, once per engine); pk_stream_prefill runs a prompt into stream
 * s's cache and picks its next token (the engine's own sequence and prefix
 * reuse are reset); pk_streams_decode writes [n_steps][n_streams] ids, as
 * pk_decode_steps_device per stream; pk_streams_set_position moves every
 * stream to pos (a pos past a stream's tokens attends zero-filled cache
 * entries: for timing long contexts only). */
int pk_streams_begin(pk_engine *eng, int n_streams);
int pk_stream_prefill(pk_engine *eng, int s, const uint32_t *prompt, int n);
int pk_streams_decode(pk_engine *eng, int n_steps, uint32_t *out_ids, float *device_ms);
int pk_streams_set_position(pk_engine *eng, int pos);

/* One decode step run eagerly with CUDA events around every kernel: per
 * kernel name the launch count, device time and algorithmic bytes. */
typedef struct {
  char name[32];
  int launches;
  double ms;
  double bytes;
} pk_kernel_stat;
int pk_decode_profile(pk_engine *eng, pk_kernel_stat *out, int cap, int *n_out);

/* Test hook (no reference counterpart): one persistent decode launch in which
 * the readers of one phase wait for a tag nothing writes, so every bounded
 * wait in the kernel runs out.  *status receives the launch's status
 * (PK_ERR_TIMEOUT expected); the engine stays usable and the sequence is
 * unchanged.  PK_ERR_UNSUPPORTED when the persistent kernel is not in use. */
int pk_selftest_bounded_wait(pk_engine *eng, int *status);

/* Records layer-0 intermediates for parity bisection (Engine.dbg). */
int pk_set_debug(pk_engine *eng, int on);
/* Copies the named layer-0 dump (token-major [b][dim]); returns elements via n_out.
 * Names "decode.q", "decode.k", "decode.v", "decode.att", "decode.x_o" (the
 * residual after o), "decode.h" (the SwiGLU output) and "decode.x" (after
 * down) give the persistent decode kernel's last layer of its latest launch
 * instead (no set_debug needed; parity bisection of the decode step). */
int pk_get_dump(pk_engine *eng, const char *name, float *out, int cap, int *n_out);

void pk_request_stop(void);
void pk_clear_stop(void);

/* ------------------------------------------------- tensor-parallel decode
 * No reference counterpart: the reference runs one engine per process on the
 * CPU.  This splits a llama stack over T GPUs, one process per GPU (the
 * 70B-shaped configuration), for b = 1 decode:
 *   q/k/v rows of whole heads, o and down k ranges, gate/up rows, output
 *   vocabulary rows; after o and after down the ranks' partial row sums are
 *   added in rank order through peer memory (cudaIpc handles exchanged by
 *   the caller); the token is the first maximum over the vocabulary shards.
 * Every rank makes the same calls in the same order.  With T = 1 a step is
 * the single-GPU b = 1 op sequence bit for bit. */
typedef struct pk_tp pk_tp;

typedef struct {
  int rank, world, n_layer, n_embd, n_head, n_head_kv, head_dim, n_ff, n_vocab;
  int local_heads, local_kv_heads, local_ff, vocab0, local_vocab;
  size_t weight_bytes;       /* this rank's device weight bytes */
  size_t stream_bytes;       /* bytes this rank's weights stream per token */
  int collectives_per_token; /* 2 per layer + the token pick */
} pk_tp_info;

/* A synthetic llama stack (Q4_K q/k/o/gate/up/down, Q6_K v/output, Q4_K
 * embedding) generated on the device, each rank its own shard. */
typedef struct {
  int n_layer, n_embd, n_head, n_head_kv, head_dim, n_ff, n_vocab, n_rot;
  float rope_theta, rms_eps;
} pk_tp_model;

int pk_tp_create(int device, int n_ctx, int rank, int world, pk_tp **out);
void pk_tp_destroy(pk_tp *tp);
int pk_tp_load_gguf(pk_tp *tp, const char *path);
int pk_tp_load_synthetic(pk_tp *tp, const pk_tp_model *model, uint64_t seed);
/* Bytes of one peer-memory handle (a cudaIpcMemHandle_t). */
int pk_tp_handle_bytes(void);
/* This rank's handle (after a load); then every rank passes all T handles in rank order. */
int pk_tp_ipc_handle(pk_tp *tp, void *out);
int pk_tp_open_peers(pk_tp *tp, const void *handles);
/* The o / down exchange through an NCCL all-reduce instead of the peer-memory
 * push (no counterpart in the reference, which runs on one device).  Rank 0
 * makes an id with pk_tp_nccl_id (pk_tp_nccl_id_bytes bytes); every rank
 * passes that id to pk_tp_use_nccl after pk_tp_open_peers, and the call
 * returns once all T ranks have joined.  NCCL is loaded at the first call
 * (the process's libnccl.so.2); PK_ERR_UNSUPPORTED when none can be loaded. */
int pk_tp_nccl_id_bytes(void);
int pk_tp_nccl_id(void *out);
int pk_tp_use_nccl(pk_tp *tp, const void *id);
/* The prompt as b = 1 steps; the last step picks the first generated token. */
int pk_tp_prefill(pk_tp *tp, const uint32_t *prompt, int n);
/* n_steps tokens as pk_decode_steps_device: the token picked last, then the next n_steps - 1; the
 * n_steps steps also pick the token the next call starts with (device time in *device_ms). */
int pk_tp_decode(pk_tp *tp, int n_steps, uint32_t *out_ids, float *device_ms);
/* This rank's logits of the last step with the head: rows [vocab0, vocab0 + n_local). */
int pk_tp_logits(pk_tp *tp, float *out, int n, int *n_local, int *vocab0);
int pk_tp_info_get(pk_tp *tp, pk_tp_info *info);
/* Host restatements for tests: the shard of rank r of T (out = {local heads,
 * local kv heads, local ffn rows, vocab0, local vocab}), and the pick over
 * the shards' {value, global index or -1}. */
int pk_tp_split(int n_head, int n_head_kv, int head_dim, int n_ff, int n_vocab, int rank, int world, int o_block,
                int down_block, int out[5]);
uint32_t pk_tp_pick(const float *vals, const int *idx, int world);

/* ---- Prompt text (host code): the GGUF's byte-level BPE tokenizer and the chat template. */
typedef struct pk_tokenizer pk_tokenizer;
typedef struct {
  int32_t n_vocab;
  int32_t n_eos;         /* end-of-generation ids (eos_token_id and the <|im_end|>-like specials) */
  int64_t bos_id;        /* -1: the GGUF names none */
  uint32_t eos_ids[16];  /* the first min(n_eos, 16), ascending */
  int32_t ignore_merges; /* 1 when tokenizer.ggml.pre is "minicpm5" */
  char pre[64];          /* tokenizer.ggml.pre (truncated, NUL-terminated) */
} pk_tokenizer_info;

/* Reads tokenizer.ggml.{tokens, token_type, merges, pre, bos_token_id, eos_token_id};
 * PK_ERR_IO when the file does not parse or has no token list. */
int pk_tokenizer_load(const char *gguf_path, pk_tokenizer **out);
void pk_tokenizer_free(pk_tokenizer *tok);
int pk_tokenizer_info_get(const pk_tokenizer *tok, pk_tokenizer_info *out);
/* UTF-8 text of len bytes -> token ids (parse_special: special-token texts become their ids).
 * Writes min(cap, n) ids and *n_out = n; PK_ERR_INVALID for malformed UTF-8 or n > cap. */
int pk_tokenize(const pk_tokenizer *tok, const char *text, size_t len, int parse_special, uint32_t *out,
                size_t cap, size_t *n_out);
/* The bytes one token stands for (special tokens: their text).  Unknown ids give 0 bytes.
 * Writes min(cap, n) bytes and *n_out = n; PK_ERR_INVALID for n > cap. */
int pk_token_bytes(const pk_tokenizer *tok, uint32_t id, uint8_t *out, size_t cap, size_t *n_out);
/* 1 when id ends generation, else 0. */
int pk_token_is_eog(const pk_tokenizer *tok, uint32_t id);
/* model.rs:1355-1388 flush_utf8, for streaming the text of generated tokens (pk_token_bytes appended
 * to a pending buffer after every token): the text ready in pending[0 .. *n_pending) -- the longest
 * valid UTF-8 prefix, each invalid sequence (its maximal valid-so-far part) replaced by U+FFFD,
 * repeated until only an incomplete trailing sequence or nothing is left.  That tail moves to the
 * front of pending and *n_pending becomes its length.  Writes min(cap, n) text bytes to out and
 * *n_out = n (at most 3 * *n_pending); PK_ERR_INVALID for n > cap, pending unchanged then. */
int pk_utf8_flush(uint8_t *pending, size_t *n_pending, uint8_t *out, size_t cap, size_t *n_out);
/* Host restatement for tests: the matches of a pre-tokenizer pattern (UTF-8, plen bytes) over a
 * UTF-8 text, as (start, end) code-point offsets, two entries per match.  Writes min(cap, n)
 * entries and *n_out = n; PK_ERR_INVALID for malformed UTF-8 or n > cap. */
int pk_text_find(const char *pattern, size_t plen, const char *text, size_t tlen, uint32_t *bounds, size_t cap,
                 size_t *n_out);

typedef struct {
  const char *role;    /* "system", "user", "assistant", "tool" (other roles are dropped) */
  const char *content; /* UTF-8, NUL-terminated */
} pk_chat_message;
/* The prompt text of a conversation: minicpm5 != 0 the MiniCPM5 template, else generic
 * <|im_start|>role turns; add_generation_prompt appends the assistant header.  Writes min(cap, n)
 * bytes (no terminator) and *n_out = n; PK_ERR_INVALID for n > cap or a message that is not UTF-8. */
int pk_chat_apply(const pk_chat_message *msgs, int n_msgs, int minicpm5, int add_generation_prompt, char *out,
                  size_t cap, size_t *n_out);
/* The prompt ids of a chat request as the reference's Android bridge builds them (jni.rs:416-456):
 * the template over the kept turns, the direct-answer suffix when direct_answer is set, the template
 * is MiniCPM5 and the text ends with the assistant header (*direct_applied = 1), then pk_tokenize with
 * special tokens.  While the ids exceed n_ctx - 1024 (no limit when n_ctx < 1024), one old turn is
 * dropped: the second kept turn, or the third when the first is a system turn; *n_dropped counts
 * them.  PK_ERR_CONTEXT_FULL when only that many turns are left and the ids still do not fit.
 * Writes min(cap, n) ids and *n_ids = n; PK_ERR_INVALID for n > cap or a message that is not UTF-8. */
int pk_chat_prompt(const pk_tokenizer *tok, const pk_chat_message *msgs, int n_msgs, int minicpm5,
                   int direct_answer, size_t n_ctx, uint32_t *ids, size_t cap, size_t *n_ids, int *n_dropped,
                   int *direct_applied);
/* 1 when the tokenizer's pre name or the model name selects the MiniCPM5 template. */
int pk_chat_is_minicpm5(const char *pre, const char *name);
/* Suffixes a host appends after the generation prompt: a direct answer (empty reasoning block)
 * or an open reasoning block. */
const char *pk_chat_direct_suffix(void);
const char *pk_chat_thinking_suffix(void);

#ifdef __cplusplus
}
#endif
#endif /* PK_H */
