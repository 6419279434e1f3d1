/*
 * pk_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of pocketinfer's CPU kernels and decode loop
 * (Aleinto97/pocket-workbench-android, rust/pocketinfer/src), used as the
 * parity checker for the B200 path.  Only tests/, __graft_entry__.smoke() and
 * bench.py (cpu_baseline leg and --impl reference arm) may load this library.
 * The product library (libpocketinfer_b200.so) never links or calls it.
 *
 * Restated paths (file:line refer to rust/pocketinfer/src/ in the reference):
 *   - f16 <-> f32:                 util.rs:76-138
 *   - type table, tensor_nbytes:   quant.rs:3-72
 *   - dequant_row:                 quant.rs:102-359
 *   - dot_row_scalar:              quant.rs:377-441   (the x86 f32 path)
 *   - row_dot_multi (scalar):      quant.rs:443-476
 *   - Q8Act::prepare (scalar):     quant_int.rs:17-56 (bit-identical to the
 *                                  NEON b==1 path by simd_q8.rs:57-80)
 *   - int8 dots dp::* / lanes::*:  quant_int.rs:103-229, 282-419
 *   - Pool::matmul:                model.rs:242-321
 *   - rmsnorm / RoPE / attention / SwiGLU / residual (portable branches):
 *                                  model.rs:777-823, 408-461, 905-1172
 *   - sample (greedy + top-p):     sampler.rs:1-92
 *   - Engine::generate incl. prefix-KV reuse: model.rs:1235-1352
 *
 * Parity pin: the reference cannot be built here (no Rust toolchain, and its
 * int8 kernels exist only on aarch64).  The restatement is pinned against the
 * reference's own known-answer tests (tests/quant_layout.rs, simd_q8.rs:57-80,
 * backend/opencl.rs:391-430) which tests/test_oracle_kats.py re-runs.
 */
#ifndef PK_ORACLE_H
#define PK_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float pko_f16_to_f32(uint16_t h);
uint16_t pko_f32_to_f16(float v);

/* (block elements, block bytes); returns 0 for unknown types. */
int pko_type_block(uint32_t ttype, size_t *be, size_t *bb);
/* -1 on error (dim0 not block-divisible, overflow). */
int64_t pko_tensor_nbytes(uint32_t ttype, uint64_t ne0, uint64_t ne1);

void pko_dequant_row(uint32_t ttype, const uint8_t *data, size_t k, float *out);
float pko_dot_row_scalar(uint32_t ttype, const uint8_t *data, size_t k, const float *x);
void pko_row_dot_multi(uint32_t ttype, const uint8_t *row, size_t k, const float *xt, size_t b,
                       float *out);

/* Q8Act::prepare: x feature-major [k][b]; q [b][k], d/sum [b][k/32]. */
void pko_q8_prepare(const float *x, size_t k, size_t b, int8_t *q, float *d, int32_t *sum);

/* Single-lane int8 dot (dp::*): act arrays are the full [b][...] buffers. */
float pko_dot_row_q8(uint32_t ttype, const uint8_t *row, size_t k, const int8_t *q,
                     const float *d, const int32_t *sum, size_t lane);
/* Multi-lane int8 dot (lanes::*): out[lane] += acc[lane]. */
void pko_dot_row_q8_lanes(uint32_t ttype, const uint8_t *row, size_t k, const int8_t *q,
                          const float *d, const int32_t *sum, size_t b, float *out);
/* Integer dot of every term of one row for one lane, in the reference's
 * accumulation order (Q4_K: 8 per super-block; Q6_K: 16 per super-block;
 * Q4_0/Q8_0: 1 per block).  Returns the number of terms written. */
size_t pko_row_int_dots(uint32_t ttype, const uint8_t *row, size_t k, const int8_t *q,
                        size_t lane, int32_t *dots);

/* Pool::matmul.  use_act != 0 selects the int8 lanes path with (q,d,sum). */
void pko_matmul(uint32_t ttype, const uint8_t *w, size_t row_bytes, size_t k, const float *xt,
                size_t b, float *out, size_t n_rows, int use_act, const int8_t *q,
                const float *d, const int32_t *sum, size_t threads);

/* Persistent Pool (model.rs:151-235) for repeated matmul calls. */
typedef struct pko_pool pko_pool;
pko_pool *pko_pool_new(size_t threads);
void pko_pool_free(pko_pool *p);
void pko_pool_matmul(pko_pool *p, uint32_t ttype, const uint8_t *w, size_t row_bytes, size_t k,
                     const float *xt, size_t b, float *out, size_t n_rows, int use_act,
                     const int8_t *q, const float *d, const int32_t *sum);

/* Model-level engine (Engine::load / forward / generate). */
typedef struct pko_engine pko_engine;
typedef struct {
  size_t prefill_tokens;
  size_t prefill_cached_tokens;
  double prefill_ms;
  size_t gen_tokens;
  double gen_ms;
  char stop[32];
} pko_stats;

pko_engine *pko_engine_load(const char *path, size_t n_ctx, size_t threads, char *err,
                            size_t errlen);
void pko_engine_free(pko_engine *e);
void pko_engine_set_int8(pko_engine *e, int enabled);
void pko_engine_set_eog(pko_engine *e, int enabled);
/* K / V cache entries rounded to f16 at store (round to nearest even): the
 * checker of the B200 library's f16 cache.  The reference keeps f32. */
void pko_engine_set_kv_f16(pko_engine *e, int on);
size_t pko_engine_vocab(pko_engine *e);
/* Engine::forward (public: invalidates prefix reuse).  0 = ok. */
int pko_forward(pko_engine *e, const uint32_t *ids, const size_t *pos, size_t b, int want_logits,
                char *err, size_t errlen);
/* Copy the logits buffer (vocab floats). */
size_t pko_logits(pko_engine *e, float *out, size_t n);
int pko_generate(pko_engine *e, const uint32_t *prompt, size_t n, size_t max_tokens, float temp,
                 float top_p, uint64_t seed, uint32_t *out_ids, size_t out_cap, size_t *n_out,
                 pko_stats *stats, char *err, size_t errlen);
/* Dumps of layer-0 intermediates (Engine.dbg). */
void pko_engine_set_debug(pko_engine *e, int on);
/* Copies the named dump (b lanes x dim, feature-major) into out; returns elements or 0. */
size_t pko_engine_dump(pko_engine *e, const char *name, float *out, size_t cap);

void pko_request_stop(void);
void pko_clear_stop(void);

/* The C library's expf over an array (f32::exp in the reference). */
void pko_expf_batch(const float *x, float *out, size_t n);

/* sampler.rs */
uint32_t pko_sample(float *logits, size_t n, float temp, float top_p, uint64_t *rng_state);
uint64_t pko_rng_new(uint64_t seed);
uint64_t pko_rng_next_u64(uint64_t *state);
float pko_rng_next_f32(uint64_t *state);

#ifdef __cplusplus
}
#endif
#endif
