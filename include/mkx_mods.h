/* C ABI of the per-step modulation vectors ("_step_modulations") on sm_100a.
 *
 * REKI's expert takes, for every Euler step s of a predict, one AdaRMS modulation row of
 * MODW = 3L*3H + 2H values ([scale, shift, gate] of the self-attention, cross-attention and MLP
 * blocks of each layer, then [scale, shift] of the final norm; layout read by the megakernel,
 * src/mk_expert.py:336-340,423). The reference obtains them from Kyutai's
 * `RekiFlowModel._step_modulations(num_steps, state_cond) -> (mods, dt)` (called by `install`,
 * src/mk_expert.py:527-535); that code is not part of the reference checkout, so this library
 * restates it (parity unpinned) as a DiT-style conditioning network:
 *
 *   t_s     = 1 - s / N                                              s = 0 .. N-1
 *   temb_s  = [cos(1000 t_s f_i), sin(1000 t_s f_i)]_i,  f_i = 10000^(-i / (tdim/2))
 *   e_s     = 8 (W_t temb_s + W_s state)      [H], temb in double, the products summed in fp32
 *   a_s     = bf16(silu(e_s))                                        the projection's bf16 input
 *   mods_s  = bf16(W_m a_s + b_m)                                    [MODW], fp32 accumulation
 *   dt      = 1 / N
 *
 * W_m is MODW x H bf16 (54 M weights at REKI's sizes, 108.5 MB); the projection streams it from
 * HBM once per call for all N steps (tensor-core mma.sync tiles of 16 rows x 16 steps).
 *
 * All pointers are device pointers of the handle's device unless marked otherwise; bf16 arrays
 * are uint16_t bit patterns. Status codes are those of mkx.h. *
 * Entry points that select the handle's device make it current for the call and restore the
 * caller's current device before they return.
 */
#ifndef MKX_MODS_H
#define MKX_MODS_H

#include <stdint.h>
#include <cuda_runtime_api.h>
#include "mkx.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mkx_mods_handle mkx_mods_handle;

typedef struct {
  int H;     /* width, must be 768 */
  int L;     /* layers: MODW = 3 L 3 H + 2 H */
  int tdim;  /* timestep-embedding width, even, <= 1024 (256 for REKI) */
  int sdim;  /* proprio-state width, 1 .. 64 */
} mkx_mods_dims;

/* w_t: [H][tdim] fp32; w_s: [H][sdim] fp32; w_m: [MODW][H] bf16; b_m: [MODW] fp32. All are copied
 * into the handle (W_m repacked into MMA-fragment order); the caller may free them once this
 * returns. Synchronises the device. */
mkx_status mkx_mods_create(const mkx_mods_dims* dims, const float* w_t, const float* w_s, const uint16_t* w_m,
                           const float* b_m, int device, mkx_mods_handle** out);

/* Modulation rows of an N-step predict: state [sdim] fp32 (device); mods_out [N][MODW] bf16, rows
 * contiguous (row stride MODW); dt_out: one fp32 (device), receives 1 / N. 1 <= N <= 16.
 * Asynchronous on `stream` (two kernel launches, the second a programmatic dependent of the first;
 * no spin waits); graph-capturable. */
mkx_status mkx_mods_run(mkx_mods_handle* h, int N, const float* state, uint16_t* mods_out, float* dt_out,
                        cudaStream_t stream);

/* Reads the device error word (synchronises the handle's last stream first): 0 = no error. The
 * kernels have no waits that can run out of time; the word stays 0 unless a future kernel sets it. */
mkx_status mkx_mods_last_error(mkx_mods_handle* h, int* code);

/* MODW of a handle. */
int mkx_mods_width(const mkx_mods_handle* h);

/* Copies the projection input of the handle's last run, a [16][H] bf16 (rows >= N zero), to dst
 * (device, 16-byte aligned), asynchronously on `stream`. For verification of the two stages. */
mkx_status mkx_mods_input(mkx_mods_handle* h, uint16_t* dst, cudaStream_t stream);

void mkx_mods_destroy(mkx_mods_handle* h);

#ifdef __cplusplus
}
#endif
#endif
