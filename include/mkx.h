/*
 * mkx.h -- C ABI of the B200 action-expert megakernel (REKI expert, Euler steps 2..N).
 *
 * Plain C: device pointers, sizes and a cudaStream_t; no torch types. Every entry point returns an
 * mkx_status (0 = success). All pointers marked "device" must point to memory of the device the
 * handle was created on. Entry points that need the handle's device (create, error read-back,
 * clear, destroy) make it current for the call and restore the caller's current device before
 * they return; mkx_run and mkx_run_static launch on the device of the stream they are given, which
 * must be the calling thread's current device.
 *
 * Reference interface each entry point replaces (project muninn-huginn/reki-megakernel):
 *   mkx_create      <- ExpertMegakernel.__init__(model)            src/mk_expert.py:436-481
 *   mkx_run         <- ExpertMegakernel.run(x_t, mods, dt, past, action_dim)
 *                                                                  src/mk_expert.py:483-515
 *   mkx_sync_points <- ExpertMegakernel.barriers(n_steps)          src/mk_expert.py:517-518
 *   mkx_last_error  <- (stage counter) test_mk.py's read-back of the barrier counter, compared
 *                      with nprog * barriers(n_steps)                    src/test_mk.py:43-45
 *                      (error word) the reference has none: a broken grid barrier deadlocks
 *                      (README.md:262-263); here every device-side wait is bounded and reports
 *   mkx_destroy     <- Python object lifetime of ExpertMegakernel
 *   mkx_set_timeout_ns, mkx_clear_error, mkx_set_fault_injection, mkx_set_launch_sequence,
 *   mkx_launch_shape, mkx_last_cuda_error <- no counterpart (bounded waits, test hooks, introspection)
 */
#ifndef MKX_H_
#define MKX_H_

#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MKX_MAX_LAYERS 16

typedef int mkx_status;
enum {
  MKX_OK = 0,
  MKX_ERR_INVALID_ARG = 1,   /* null pointer, bad shape, misaligned pointer */
  MKX_ERR_UNSUPPORTED = 2,   /* geometry the kernel is not built for */
  MKX_ERR_CUDA = 3,          /* a CUDA runtime call failed (see mkx_last_cuda_error) */
  MKX_ERR_DEVICE = 4,        /* the kernel reported an error (timeout); see mkx_last_error */
  MKX_ERR_RESOURCES = 5      /* not enough SMs / shared memory for a co-resident grid */
};

typedef struct mkx_handle mkx_handle;

/* Expert geometry (REKI: L=10, H=768, NH=12, HD=64, I=3072, A=32). H, NH, HD are fixed by the
 * kernel (768 / 12 / 64); L <= MKX_MAX_LAYERS; I a multiple of 128; 8 <= A <= 32. */
typedef struct {
  int L, H, NH, HD, I, A;
  float eps;          /* AdaRMS epsilon (input_layernorm.eps == action_expert.norm.eps) */
  float qk_eps;       /* per-head q/k RMSNorm epsilon */
  int max_rows;       /* largest T (action rows) a run may use; <= 16 */
  int grid;           /* CTAs of the persistent launch; 0 = one per SM */
} mkx_dims;

/* Expert weights in the reference's stacked layout (src/mk_expert.py:445-460); device pointers,
 * row-major, read once by mkx_create (the handle keeps its own packed copy). */
typedef struct {
  const uint16_t* wqkv;   /* bf16 [L, 3H, H]  cat(q_proj, k_proj, v_proj) */
  const uint16_t* wo;     /* bf16 [L, H, H]   self_attn.o_proj */
  const uint16_t* wqca;   /* bf16 [L, H, H]   cross_attn.q_proj */
  const uint16_t* woca;   /* bf16 [L, H, H]   cross_attn.o_proj */
  const uint16_t* wg;     /* bf16 [L, I, H]   mlp.gate_proj */
  const uint16_t* wu;     /* bf16 [L, I, H]   mlp.up_proj */
  const uint16_t* wd;     /* bf16 [L, H, I]   mlp.down_proj */
  const uint16_t* qn;     /* bf16 [L, HD]     self_attn.q_norm.weight (scale = 1 + w) */
  const uint16_t* kn;     /* bf16 [L, HD]     self_attn.k_norm.weight */
  const uint16_t* qcan;   /* bf16 [L, HD]     cross_attn.q_norm.weight */
  const float* win;       /* fp32 [A, H]      action_in_proj.weight TRANSPOSED */
  const float* bin;       /* fp32 [H]         action_in_proj.bias */
  const float* wout;      /* fp32 [A, H]      action_out_proj.weight */
  const float* bout;      /* fp32 [A]         action_out_proj.bias */
} mkx_weights;

/* Inputs of one call of Euler steps 2..N (batch 1). Device pointers unless noted. */
typedef struct {
  const float* x_in;      /* [T, A] fp32: action state after Euler step 1 */
  float* x_out;           /* [T, A] fp32: action state after step N (padded dims: 0 + dt * v) */
  const void* mods;       /* [N, MODW] per-step modulations, row 0 (step 1) unused; MODW = 9LH + 2H */
  int mods_fp32;          /* 0: bf16 mods, 1: fp32 mods */
  const float* dt;        /* [1] fp32 Euler step */
  /* register memory K/V per layer: [PM, NH, HD] bf16 rows, valid rows [cu_kv[0], PM), already
   * normed and rotated (past.register_step['mem_kv'][l]) */
  const uint16_t* memk[MKX_MAX_LAYERS];
  const uint16_t* memv[MKX_MAX_LAYERS];
  int mem_rows;           /* PM */
  int mem_row_stride;     /* elements between consecutive rows (NH*HD when contiguous) */
  const int* cu_kv;       /* device int32; cu_kv[0] = first valid memory row */
  /* cross-attention source K/V per layer: [SP, NH, HD] bf16, valid rows [0, cu_src[1]) */
  const uint16_t* kca[MKX_MAX_LAYERS];
  const uint16_t* vca[MKX_MAX_LAYERS];
  int ca_rows;            /* SP: rows allocated per layer (the kernel reads min(cu_src[1], SP) rows) */
  int ca_row_stride;      /* elements between consecutive rows */
  const int* cu_src;      /* device int32; cu_src[1] = S valid source rows */
  const float* sa_cos;    /* [T, HD] fp32 RoPE tables of the action rows (self-attention) */
  const float* sa_sin;
  const float* ca_cos;    /* [T, HD] fp32 RoPE tables of the action rows (cross-attention) */
  const float* ca_sin;
  int T;                  /* action rows, 1..max_rows */
  int n_steps;            /* Euler steps to run (= N - 1), >= 1 */
  int action_dim;         /* real action dims, 1..8 */
  uint16_t* trace_h;      /* optional [n_steps, L, T, H] bf16: every layer's output h; may be NULL */
  unsigned long long* prof; /* optional [grid, 1 + mkx_sync_points(n_steps)] %globaltimer stamps (ns):
                             * per CTA, the launch start then the end of every stage; may be NULL */
  /* optional (no counterpart in the reference, whose K/V are always on the device): readiness words
   * for K/V that are still being copied in while the launch runs. When kv_ready is non-NULL
   * (device int32 [L], 4-byte aligned), the launch reads layer l's memory and cross-attention K/V
   * only once kv_ready[l] == kv_ready_value; the caller writes that value after the layer's copies,
   * in the same copy stream (a 4-byte host-to-device copy: a kernel there would wait for the SMs
   * this launch holds). A word that never arrives ends the launch with a timeout error
   * (mkx_last_error) instead of a hang. NULL: every input is in place at launch. Read by mkx_run;
 * mkx_run_static ignores these two fields. */
  const int* kv_ready;
  int kv_ready_value;
} mkx_step_inputs;

/* Packs the weights into the handle's own device memory (one-off, synchronous on `stream`'s
 * device) and allocates the launch's scratch. */
mkx_status mkx_create(const mkx_dims* dims, const mkx_weights* w, int device, mkx_handle** out);

/* Enqueues one persistent launch for steps 2..N on `stream`. No host synchronisation, no host
 * reads of device data: capturable in a CUDA graph. One launch in flight per handle. */
mkx_status mkx_run(mkx_handle* h, const mkx_step_inputs* in, cudaStream_t stream);

/* Number of dependent exchange points (the dataflow counterpart of grid barriers) per launch. */
int mkx_sync_points(const mkx_handle* h, int n_steps);

/* Reads (synchronously) the device status words: *code = 0 when every wait completed; otherwise
 * an encoded (cta << 16 | kind << 8 | stage) of the first failed wait. *stages = sum over CTAs of
 * the stages each CTA completed, accumulated over the launches since mkx_create or the last
 * mkx_clear_error (one launch of n steps: grid * mkx_sync_points(n)). Either pointer may be NULL. */
mkx_status mkx_last_error(mkx_handle* h, int* code, long long* stages);

/* Clears the device error word and the stage counter (synchronous). */
mkx_status mkx_clear_error(mkx_handle* h);

/* Device-side wait limit in nanoseconds (default 2e9). */
mkx_status mkx_set_timeout_ns(mkx_handle* h, unsigned long long ns);

/* Test hook for the failure path (no GPU fault involved): with stage == 1, CTA 0 withholds its
 * layer-0 QKV words in later launches, so the bounded waits on them run out and the launch reports
 * MKX_ERR_DEVICE through mkx_last_error. 0 disables it. */
mkx_status mkx_set_fault_injection(mkx_handle* h, int stage);

/* Test hook: sets the handle's launch sequence number (synchronous). Exchange-word tags are
 * sequence * 4096 + instance + 1 in 32 bits, so they repeat every 2^20 launches; every launch sets
 * the words it will not rewrite (rows >= T, action-state words >= action_dim, an unused parity) to
 * tag 0, so a launch exactly 2^20 launches later never finds a stale word with its own tag. The hook
 * lets a test jump the sequence by 2^20 instead of running a million launches. */
mkx_status mkx_set_launch_sequence(mkx_handle* h, unsigned int seq);

/* Grid size actually used and dynamic shared memory bytes per CTA. */
mkx_status mkx_launch_shape(const mkx_handle* h, int* grid, int* smem_bytes);

/* Weights already in the kernel's packed layout, in device memory the caller owns. The layout
 * depends on the grid size; reki_megakernel_b200/packing.py writes it from the stacked weights:
 *   w[0..5]  bf16 QKV, O, CA-Q, CA-O, gate+up, down: each CTA's rows as [K/16][rows][16]
 *   nrm      fp32 [3, L, HD]: 1 + q_norm, 1 + k_norm, 1 + ca q_norm
 *   tailw    fp32 [8 * H + H + 32]: action_in_proj rows 0..7 (transposed), its bias, the out bias
 *   wout     fp32 [A, H]: action_out_proj.weight */
typedef struct {
  const uint16_t* w[6];
  const float* nrm;
  const float* tailw;
  const float* wout;
} mkx_packed_weights;

/* No counterpart in the reference: an extra entry point for callers that cannot allocate device
 * memory themselves -- a runtime that hands every buffer out of one arena reserved at start-up, or
 * a control loop that may not call cudaMalloc/cudaFree once it is running, because an allocation
 * can block on the device and break the loop's timing. It runs one launch of the same kernel as
 * mkx_run without a handle: the caller passes packed weights (mkx_packed_weights, packed for
 * dims->grid; 0 = one CTA per SM), the step inputs and x_out, all in memory it owns, plus an
 * optional device int err_out (4-byte aligned, else MKX_ERR_INVALID_ARG) that receives the launch's
 * error word (0 when every wait finished).
 * The kernel's scratch -- the exchange buffers and status words -- is a file-scope static device
 * array of 2,072,608 bytes, which every GPU that loads this library keeps until the process exits;
 * it holds I <= 3072 and T <= 16, and larger sizes return MKX_ERR_UNSUPPORTED with a message in
 * mkx_last_cuda_error(). Nothing in this call allocates. The first call on a device looks up the
 * array's device address and raises the kernel's shared-memory limit, so make that first call
 * before any stream capture. That set-up is kept for the life of the process: after a
 * cudaDeviceReset (or any reset of the device's primary context) the address and the limit are
 * stale, so do not call this entry point on that device again in the same process. All calls share the one array and it keeps the last call's contents
 * (the error word and stage counter are cleared on the stream before each launch): two calls
 * whose launches overlap on the GPU race and corrupt each other. */
mkx_status mkx_run_static(const mkx_dims* dims, const mkx_packed_weights* w, const mkx_step_inputs* in,
                          int* err_out, cudaStream_t stream);

/* Enqueues n host-to-device copies on `stream`, one cudaMemcpyAsync each, in order: dst[i] (device)
 * <- src[i] (pinned host), bytes[i] bytes. The copies of a streamed launch (the small inputs ahead of
 * it, then per layer its K/V followed by its 4-byte readiness word, see kv_ready) are issued with
 * one call each instead of one host call per tensor. No counterpart in the reference. */
mkx_status mkx_h2d_copies(int n, void* const* dst, const void* const* src, const size_t* bytes, cudaStream_t stream);

/* Enqueues n pitched host-to-device copies on `stream`, one cudaMemcpy2DAsync each, in order: height[i]
 * rows of width[i] bytes from src[i] (pinned host, rows spitch[i] bytes apart) to dst[i] (device, rows
 * dpitch[i] bytes apart); width[i] <= both pitches, height[i] >= 1 (MKX_ERR_INVALID_ARG otherwise,
 * before anything is enqueued). Streamed launches use it to copy only the K/V rows the kernel reads
 * (memory rows from kv_start, source rows below S) of a run of layers with one command. No
 * counterpart in the reference. */
mkx_status mkx_h2d_copies_2d(int n, void* const* dst, const size_t* dpitch, const void* const* src,
                             const size_t* spitch, const size_t* width, const size_t* height, cudaStream_t stream);

/* Last CUDA error string seen by the library (thread-local, static storage). */
const char* mkx_last_cuda_error(void);

void mkx_destroy(mkx_handle* h);

#ifdef __cplusplus
}
#endif
#endif /* MKX_H_ */
