// pk_decode.h -- the persistent single-token decode kernel (pk_decode.cu).
//
// One launch runs a whole b == 1 forward pass (model.rs:833-1170): the
// embedding row, every layer, the final norm and the output head, and
// optionally the greedy pick and the device-side token feedback.  One CTA
// runs on each SM.  In each CTA one producer thread streams that CTA's share
// of the weights (and, for the CTAs that own an attention head, the head's
// K/V history) through a ring of shared-memory slots with bulk copies; the
// consumer warps compute.  Weights never depend on activations, so the
// producer runs ahead across the grid-wide dependency points.
#pragma once
#include <cuda.h>  // CUtensorMap (the type only; the encoder is reached through cudaGetDriverEntryPoint)
#include <stdint.h>

#include <string>
#include <vector>

#include "pk_kernels.h"

namespace pk {

constexpr int DK_THREADS = 512;     // warp 0 producer, warps 1-2 row chains, warps 3..15 terms
constexpr int DK_CHAINS = 2;        // chain warps
constexpr int DK_NB = 3;            // term buffers
constexpr int DK_NS = 5;            // ring slots
constexpr int DK_SLOT = 32768;      // bytes per slot
constexpr int DK_TS = 2560;         // floats per term buffer
constexpr int DK_MAX_RG = 32;       // rows per row group (one chain lane each)
constexpr int DK_TRW = 16;          // profile-trace words per phase
constexpr int DK_VB = 32;           // V-history positions per tensor-map box

enum : uint8_t { DR_Q = 0, DR_K, DR_V, DR_O, DR_GATE, DR_UP, DR_DOWN, DR_HEAD };
enum : uint8_t { DF_FIRST = 1, DF_LAST = 2 };

// One ring transfer: rows [row0, row0 + rows) x blocks [b0, b1) of one matrix.
// full: the rows are whole and contiguous, one copy for q and one for d.
// Otherwise one q copy and one d copy per row, the staged rows q_len +
// 16 qpad bytes apart.  d copies start at the 16-byte boundary at or below
// the row's first scale; the consumer recovers the skew from the source
// address.
struct DChunk {
  const uint8_t *q;   // row 0's q bytes at block b0
  const uint8_t *d;   // row 0's first f16 scale at block b0 (nullptr: scales inline)
  uint32_t q_stride;  // bytes between rows' q parts in global memory
  uint32_t d_stride;  // bytes between rows' scale arrays in global memory
  uint32_t q_len;     // bytes per q copy
  uint32_t d_len;     // bytes per d copy
  uint32_t d_off;     // slot offset of the scale area
  uint16_t rows, rs;  // rows; term-buffer row pitch in floats (terms of a row contiguous; an odd multiple of 4)
  uint8_t type, role, full, flags;
  int row0, b0, b1, layer;
  uint8_t cw;          // chain warp that sums these rows
  uint8_t qpad;        // not full: extra 16-byte units after each staged row (odd row pitch / 16)
  uint8_t pad_[2];
};
static_assert(sizeof(DChunk) == 64, "DChunk is one 64-byte record");

struct DecLayer {
  DevTensor q, k, v, o, gate, up, down;
  const float *attn_norm, *ffn_norm;
};

struct DecodeArgs {
  // V cache [L * n_kv * n_ctx][dh] as a 2-D tensor map: boxes of DK_VB
  // positions x att_ds dimensions (one attention unit's slice).
  alignas(64) CUtensorMap vmap;
  const DecLayer *layers;
  DevTensor out;
  const float *out_norm;
  const uint8_t *embd;
  uint32_t embd_row_bytes;
  int embd_type;
  int n_layer, n_embd, n_ff, n_head, n_kv, dh, half, n_ctx, n_vocab;
  // Attention units: head h's value dimensions are split into att_j slices
  // of att_ds, unit u = h * att_j + j on CTA u % grid.
  int att_j, att_ds;
  float eps, scale;
  const float *rope_cos, *rope_sin;
  float *kcache, *vcache;             // K [L][n_kv][dh][n_ctx] (d-major), V [L][n_kv][n_ctx][dh]
  float *logits;
  // Vectors passed between CTAs, one 8-byte word per element: the f32 value
  // in the low half, in the high half the tag (epoch << 10 | phase) of the
  // phase that wrote it.  A reader polls until every word it needs carries
  // the previous phase's tag, so no grid barrier separates the phases.
  unsigned long long *x_ll;           // [2][n_embd] residual after o (0) and after down (1)
  unsigned long long *att_ll;         // [n_head * dh] attention output
  unsigned long long *h_ll;           // [n_ff] SwiGLU output
  unsigned long long *q_ll;           // [n_head * dh] roped q
  unsigned long long *kv_ll;          // [2][n_kv * dh] this position's roped k (0) and v (1)
  unsigned long long *sc_ll;          // [n_head][n_ctx] attention scores shared by a head's units
  uint32_t *ids, *tok, *hist;
  int *pos, *step;
  const DChunk *chunks;
  const int *cta_chunk0;              // [grid + 1]
  const int *phase0;                  // [grid][n_phase + 1], relative to the CTA's first chunk
  int n_phase;                        // 4 * n_layer + 1
  const int *own;                     // [grid][2] rows of x written by this CTA
  const uint32_t *cwbits;             // bit per chunk: which chain warp sums it
  unsigned *sync;                     // [1] finished CTAs, [2] launch epoch (>= 1; the last CTA advances it)
  int *err;                           // 0 or a PK_ERR_* code
  float *cand_v;
  int *cand_i;                        // [grid]
  int mode;                           // 1: greedy pick + token feedback after the head
  int fast;                           // 1: the fast float order (integer dots and Q8 still exact)
  int poison;                         // > 0 (test hook): phase `poison` waits for a tag no phase writes
  unsigned long long *trace;          // optional [grid][n_trace] globaltimer stamps
  int n_trace;
};

// Host-built work split: every CTA's chunk list in consumption order.
struct DecodePlan {
  std::vector<DChunk> chunks;
  std::vector<int> cta_chunk0, phase0, own;
  std::vector<uint32_t> cwbits;  // bit i: chain warp of chunk i
  int grid = 0, n_phase = 0;
  int att_j = 1;  // value-dimension slices per attention head
  size_t smem = 0;
};
// false (with the reason) when this model cannot use the persistent kernel.
bool build_decode_plan(const std::vector<DecLayer> &layers, const DevTensor &out, int n_embd, int n_ff, int n_head,
                       int n_kv, int dh, int n_ctx, int grid, DecodePlan &plan, std::string &why);

// Largest grid for which every CTA owns rows of every matrix (the tagged
// phase hand-off relies on it), at most `sms`.
int decode_grid_for(const std::vector<DecLayer> &layers, const DevTensor &out, int sms);

// Shared memory the kernel needs for this model (0 if it does not fit).
size_t decode_smem_bytes(int n_embd, int n_ff, int qdim, int n_ctx, int dh, int n_layer);
// Sets the kernel's shared-memory limit and checks that `grid` CTAs fit at once.
cudaError_t prepare_decode(size_t smem, int grid);
cudaError_t launch_decode(const DecodeArgs &a, int grid, size_t smem, cudaStream_t st);
// DecodeArgs::vmap for a V cache (0, or -1 with the reason).
int make_vcache_map(CUtensorMap *map, const float *vcache, int n_layer, int n_kv, int n_ctx, int dh, int ds,
                    std::string &why);
int decode_grid();

}  // namespace pk
