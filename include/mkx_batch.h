/* C ABI of the episode-batch path of the action expert (Euler steps 2..N for B episodes at once).
 *
 * The reference megakernel runs one episode per launch (`assert x_t.shape[0] == 1`,
 * src/mk_expert.py:488); its benchmark configuration asks for 1, 8, 32 and 128 independent episodes
 * per GPU. Here the B episodes' 10-row action blocks are stacked into M = B * T token rows and every
 * weight byte is streamed once per Euler step for all of them: each dense stage is one tcgen05 GEMM
 * (swap-AB: a 128-row weight tile is the M = 128 operand, up to 256 token rows the N operand, fp32
 * accumulator in TMEM, operands by TMA / bulk copy), followed by the same fused epilogues as the
 * batch-1 kernel (bf16 rounding, gated residual, SiLU-mul); attention runs per (episode, head); the
 * step tail per episode. The math and rounding points are those of src/mk_expert.py:106-299 per
 * episode. No counterpart in the reference (which has no batch path); the per-episode inputs are the
 * reference's `run` inputs stacked over episodes.
 *
 * All pointers are device pointers of the handle's device; bf16 arrays are uint16_t bit patterns.
 * Entry points that select the handle's device make it current for the call and restore the caller's
 * device before they return; mkx_batch_run launches on `stream`, which must belong to that device.
 */
#ifndef MKX_BATCH_H
#define MKX_BATCH_H

#include <stdint.h>
#include <cuda_runtime_api.h>
#include "mkx.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mkx_batch_handle mkx_batch_handle;

/* Inputs of Euler steps 2..N for B episodes, each array stacked over episodes (episode e first). */
typedef struct {
  const float* x_in;        /* [B, T, A] fp32: action state after Euler step 1 */
  float* x_out;             /* [B, T, A] fp32: state after step N (padded dims: 0 + dt * v) */
  const uint16_t* mods;     /* [B, N, MODW] bf16 per-step modulations (row 0, step 1, unused) */
  const float* dt;          /* [B] fp32 */
  const uint16_t* memk;     /* [B, L, PM, NH, HD] bf16 register memory K (rows >= kv_start[e] valid) */
  const uint16_t* memv;
  const int* kv_start;      /* [B] int32 */
  int mem_rows;             /* PM <= 256 */
  const uint16_t* kca;      /* [B, L, SP, NH, HD] bf16 cross-attention K (rows < src_rows[e] valid) */
  const uint16_t* vca;
  const int* src_rows;      /* [B] int32, 1 <= S <= SP */
  int ca_rows;              /* SP <= 4096 */
  const float* sa_cos;      /* [B, T, HD] fp32 RoPE tables (self-attention positions) */
  const float* sa_sin;
  const float* ca_cos;      /* [B, T, HD] fp32 (cross-attention positions) */
  const float* ca_sin;
  int B;                    /* episodes, 1 <= B <= max_episodes */
  int T;                    /* action rows per episode, 1..16 */
  int n_steps;              /* Euler steps to run (= N - 1), >= 1 */
  int action_dim;           /* 1..8 */
} mkx_batch_inputs;

/* Packs the weights (reference stacked layout, mkx_weights of mkx.h) into tcgen05 tiles owned by the
 * handle and allocates activations for max_episodes * 16 token rows. Synchronous. dims->max_rows and
 * dims->grid are ignored. */
mkx_status mkx_batch_create(const mkx_dims* dims, const mkx_weights* w, int max_episodes, int device,
                            mkx_batch_handle** out);

/* Enqueues the whole loop (11 launches per layer and Euler step, see mkx_batch_launches) on
 * `stream`, each launch a programmatic dependent of the one before; no host
 * synchronisation, capturable in a CUDA graph. One run in flight per handle. */
mkx_status mkx_batch_run(mkx_batch_handle* h, const mkx_batch_inputs* in, cudaStream_t stream);

/* Inputs of the register pass: the R register rows of the current frame through every layer of the
 * expert with plain norms (no modulation: AdaRMS scale and shift 0, residual gates 1), each layer
 * first writing the rows' own K (per-head RMSNorm with 1 + k_norm, RoPE) and V into the memory rows
 * [mem_rows - R, mem_rows), then attending over the memory rows [kv_start, mem_rows) -- the older
 * frames and the current one -- and over the cross-attention source. Restates the register half of
 * Kyutai's Euler step 1 (`_expert_first_step`, bound at src/mk_expert.py:527-533, described in the
 * reference README: register rows with plain norms, attention over the register buffer, the register
 * K/V as output); that function is absent from the reference checkout, so the restatement is not
 * pinned to it. One memory and one source for all R rows (one episode). */
typedef struct {
  const uint16_t* reg_in;   /* [R, H] bf16 register rows entering layer 0 */
  uint16_t* memk;           /* [L, PM, NH, HD] bf16 register memory K: rows [PM - R, PM) written */
  uint16_t* memv;
  const int* kv_start;      /* [1] int32 first valid memory row (<= PM - R) */
  int mem_rows;             /* PM, R <= PM <= 256 */
  const uint16_t* kca;      /* [L, SP, NH, HD] bf16 cross-attention K (rows < src_rows valid) */
  const uint16_t* vca;
  const int* src_rows;      /* [1] int32, 1 <= S <= SP */
  int ca_rows;              /* SP <= 4096 */
  const float* sa_cos;      /* [R, HD] fp32 RoPE tables of the register rows (self-attention) */
  const float* sa_sin;
  const float* ca_cos;      /* [R, HD] fp32 (cross-attention) */
  const float* ca_sin;
  int R;                    /* register rows: a multiple of 16, <= 16 * max_episodes */
} mkx_register_inputs;

/* Enqueues the register pass on `stream` (11 launches per layer, programmatic dependents, no
 * host synchronisation, capturable). Uses the handle's activation buffers: not concurrent with
 * mkx_batch_run on the same handle. */
mkx_status mkx_batch_register_pass(mkx_batch_handle* h, const mkx_register_inputs* in, cudaStream_t stream);

/* Reads the device error word (synchronous): 0 when every bounded wait completed. */
mkx_status mkx_batch_last_error(mkx_batch_handle* h, int* code);

/* Number of kernel launches one mkx_batch_run of n_steps Euler steps enqueues for B episodes of T
 * action rows (-1 for arguments out of range). */
int mkx_batch_launches(const mkx_batch_handle* h, int B, int T, int n_steps);

/* Inspection (synchronous): copies the first `bytes` of one of the handle's activation buffers to
 * device memory `dst`: 0 h [Mp][H] bf16 (layer output), 1 AdaRMS rows, 2 qkv [Mp][3H] (the last CA
 * query as rows of H at its start), 3 attention output [Mp][H], 4 gate/up product [Mp][I], 5 action
 * state [B][T][A] fp32. Rows are the episodes' action rows, e * T + t. */
mkx_status mkx_batch_copy_state(mkx_batch_handle* h, int which, void* dst, size_t bytes);

/* Last CUDA error string seen by the batch entry points (thread-local, static storage). */
const char* mkx_batch_last_cuda_error(void);

void mkx_batch_destroy(mkx_batch_handle* h);

#ifdef __cplusplus
}
#endif
#endif
