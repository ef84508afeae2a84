/* C ABI of the cross-attention K/V preparation ("register_prepare") on sm_100a.
 *
 * The reference expert megakernel consumes per-layer cross-attention K and V that were projected
 * once per predict from the VLM source rows (`past.cross_attn_kv`, src/mk_expert.py:486-495; the
 * producer, Kyutai's `register_prepare`, is not part of the reference checkout: README.md:279-281
 * describes it as the "31 M weights" projection of the 2048-wide source). This library restates it
 * (parity unpinned):
 *
 *   K[l, n, h, :] = bf16( RoPE_n( RMSNorm_HD(src[n] . Wk[l]^T restricted to head h) * (1 + kn[l]) ) )
 *   V[l, n, h, :] = bf16( src[n] . Wv[l]^T restricted to head h )
 *
 * with bf16 src and weights, fp32 accumulation, fp32 norm and rotate-half RoPE, one rounding at the
 * end. It runs as one tcgen05 (tensor-core, TMEM accumulator) GEMM over all layers, fed by TMA.
 * This entry point has no counterpart in the reference megakernel itself.
 *
 * All pointers are device pointers of the handle's device unless marked otherwise; bf16 arrays
 * are uint16_t bit patterns. Status codes are those of mkx.h. *
 * Entry points that select the handle's device make it current for the call and restore the
 * caller's current device before they return.
 */
#ifndef MKX_PREPARE_H
#define MKX_PREPARE_H

#include <stdint.h>
#include <cuda_runtime_api.h>
#include "mkx.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mkx_prep_handle mkx_prep_handle;

typedef struct {
  int L;        /* layers */
  int H;        /* width: NH * HD, must be 768 */
  int NH;       /* heads, must be 12 */
  int HD;       /* head dim, must be 64 */
  int src_dim;  /* source width, a multiple of 64 (2048 for REKI) */
  float eps;    /* RMSNorm epsilon of the K norm */
} mkx_prep_dims;

/* wkv: [L][2][H][src_dim] bf16 (K projection then V projection of each layer, row-major [out, in]);
 * kn: [L][HD] fp32 (K norm weight, scale = 1 + kn). Both are copied into the handle (W repacked into
 * tile-contiguous, pre-swizzled blocks, L * 3 MB at src_dim = 2048); the caller may free them once
 * this returns. Synchronises the device. */
mkx_status mkx_prep_create(const mkx_prep_dims* dims, const uint16_t* wkv, const float* kn, int device,
                           mkx_prep_handle** out);

/* src: [S][src_dim] bf16, 16-byte aligned rows; cos, sin: [S][HD] fp32 RoPE tables of the source
 * positions, 16-byte aligned (MKX_ERR_INVALID_ARG otherwise, as for src, k_out and v_out); k_out, v_out: [L][SP][NH][HD] bf16 with SP >= S (rows S..SP-1 are not written).
 * 1 <= S <= 4096. Asynchronous on `stream`; graph-capturable. A device-side wait that runs out of
 * time sets the error word (mkx_prep_last_error) and the launch returns without hanging. */
mkx_status mkx_prep_run(mkx_prep_handle* h, const uint16_t* src, int S, const float* cos, const float* sin,
                        uint16_t* k_out, uint16_t* v_out, int SP, cudaStream_t stream);

/* Reads the device error word (synchronises the handle's stream first): 0 = no error. */
mkx_status mkx_prep_last_error(mkx_prep_handle* h, int* code);

void mkx_prep_destroy(mkx_prep_handle* h);

#ifdef __cplusplus
}
#endif
#endif
