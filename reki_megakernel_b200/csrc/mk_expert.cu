// B200 (sm_100a) persistent megakernel for REKI's action-expert Euler loop, steps 2..N, batch 1.
//
// Replaces the reference's Triton `expert_megakernel` (src/mk_expert.py:302-426) and its launcher
// `ExpertMegakernel` (src/mk_expert.py:433-518). Same math and rounding points; different machine:
//
// * One CTA per SM, cooperative launch (co-residency is guaranteed or the launch fails).
// * Weights: every weight stage's output rows are split in column pairs over all CTAs; each CTA's
//   rows are packed once (mkx_create) into one contiguous chunk laid out in mma.sync A-fragment
//   order ([K/16][rows][16 permuted]), streamed HBM -> shared memory by one 1D bulk copy (TMA)
//   per stage, a whole layer ahead, completion on an mbarrier. Six single-buffered slots (QKV, O,
//   CA-Q, CA-O, gate+up, down) hold one layer; a slot is refilled for the next layer as soon as
//   its MMA has read it.
// * Modulation vectors ([scale, shift, gate] per sub-block, [scale, shift] of the final norm) are
//   streamed by TMA into a two-slot shared-memory ring two blocks ahead of their use.
// * Stage-to-stage exchange: activations go through small L2-resident buffers of 8-byte words
//   {bf16 x2 payload, 32-bit tag}. A consumer polls the words it needs until every tag equals the
//   producing stage's epoch: the poll is the data load, so no separate grid barrier or flag
//   round trip exists. Buffers are double-buffered by layer parity; tags never repeat between
//   consecutive launches (a per-handle launch sequence number is part of the tag).
// * Skinny GEMMs (10 action rows): swap-AB tensor-core MMA, weights as the 16-row A operand from
//   shared memory, the activations as the 8-column B operand, fp32 accumulate; K split across
//   warps, partials reduced through shared memory; fused epilogues (bf16 rounding, gated residual,
//   SiLU-mul).
// * Attention: one CTA per (head, action row) unit; K/V rows loaded into registers before the
//   query is available; fp32 softmax; bf16(P) V.
// * Euler step tail: CTA n < T computes the fp32 velocity of action row n and publishes the new
//   action state (one small exchange); every CTA then recomputes the fp32 in-projection locally,
//   so the next step's first GEMM reads its input from shared memory.
// * Every spin-wait is bounded (%globaltimer); a timeout records an error word that all CTAs
//   watch, in-flight bulk copies are drained, and the kernel returns.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <new>

#include "mkx.h"
#include "mkx_device.cuh"

namespace mkx {

constexpr int H = 768, NH = 12, HD = 64;
constexpr int NT = 256, NW = 8;          // threads / warps per CTA
constexpr int ISSUER = NT - 1;           // thread that refills weight / modulation slots
constexpr int TP = 16;                   // padded action rows
constexpr int AO = 8;                    // carried action dims (src/mk_expert.py:478)
constexpr int XS = H + 16;               // shared X row stride (bf16 elements): conflict-free 8-byte B loads
constexpr int HWORDS = H / 2;            // exchange words per H-wide row
constexpr int QKVWORDS = 3 * H / 2;
constexpr int XWORDS = 32;               // exchange words per action-state row (fp32 payloads)
constexpr int NG = NT / 8;               // attention: 8-lane key groups per CTA
constexpr int MAXK = 5;                  // keys per group per attention chunk (NG * MAXK = 160 keys); more
                                         // key registers would spill in the attention unit
constexpr int MAX_MEM_ROWS = 256;        // memory rows per layer (any number of chunks)
constexpr int PSTR = 20;                 // partials: floats per token row of a 16-row m-tile block
constexpr int PM = TP * PSTR;            // partials: floats per (m-tile, K-split) block
constexpr int RESW = 8;                  // residual columns kept per CTA (o / ca-o / down rows)
constexpr int SROW = NT / TP;            // staging threads per action row
constexpr int SPAIRS = HWORDS / 2 / SROW; // 16-byte word pairs per staging thread
constexpr int NCOL = (H + NT - 1) / NT;   // in-projection columns per thread
constexpr int TAIL_FLOATS = AO * H + H + 32;   // win rows 0..7 | bin | bout (padded)
constexpr int MAX_STEP_TAGS = 4096;      // tag = seq * 4096 + instance + 1

enum Buf { B_QKV = 0, B_Y, B_H2, B_QCA, B_YCA, B_H3, B_G, B_HOUT, B_X, B_DP, NBUF };
// The down projection runs in two levels: the CTAs form NGRP groups; group j multiplies the g columns
// [j I / NGRP, (j + 1) I / NGRP) by the matching K-slice of Wd for all H outputs (each CTA a run of
// output columns) and publishes fp32 partial sums (B_DP: per token row, NGRP x H words of one fp32
// each); the owner of an output column then adds the NGRP partials in group order.
constexpr int NGRP = 4;
constexpr int DPWORDS = NGRP * H;         // B_DP words per token row
enum Slot { S_QKV = 0, S_O, S_QCA, S_OCA, S_GU, S_D, NSLOT };
constexpr int BAR_MODS = NSLOT;          // mbarriers NSLOT, NSLOT + 1: modulation ring slots
constexpr int NBAR = NSLOT + 2;
enum Stage { ST_INIT = 0, ST_QKV, ST_SA, ST_O, ST_CAQ, ST_CA, ST_OCA, ST_GU, ST_DOWN, ST_TAIL, ST_MBAR };
enum Kind { K_TIMEOUT = 1, K_MBAR = 3 };

struct Params {
  const uint16_t* w[NSLOT];       // packed weight chunks
  const float* nrm;               // [3][L][HD] fp32: 1 + q_norm, 1 + k_norm, 1 + ca q_norm
  const float* tailw;             // TAIL_FLOATS fp32
  const float* wout;              // [A][H] fp32
  u64* xb[NBUF];                  // exchange buffers [2][TP][row words]
  int* status;                    // [0] error word, [1] launch sequence, [2..3] stage counter (u64)
  const float* x_in;
  float* x_out;
  const void* mods;
  const float* dt;
  const uint16_t* memk[MKX_MAX_LAYERS];
  const uint16_t* memv[MKX_MAX_LAYERS];
  const uint16_t* kca[MKX_MAX_LAYERS];
  const uint16_t* vca[MKX_MAX_LAYERS];
  const int* cu_kv;
  const int* cu_src;
  const float* sa_cos;
  const float* sa_sin;
  const float* ca_cos;
  const float* ca_sin;
  uint16_t* trace_h;
  unsigned long long* prof;
  const int* kv_ready;            // optional per-layer readiness words of streamed-in K/V
  int kv_ready_value;
  unsigned long long timeout_ns;
  int drop_stage;                 // test hook: CTA 0 withholds its layer-0 words of this stage
  int mem_rows, mem_row_stride, ca_rows, ca_row_stride;
  int L, I, T, A, adim, n_steps;
  float eps, qk_eps, sm_scale;
  int s_slot[NSLOT];              // shared-memory byte offsets
  int s_x, s_p, s_mods, s_xs, s_res, s_red, s_bar, s_cnt;
};

__host__ __device__ __forceinline__ int part_lo(int i, int P, int G) {
  return (int)(((long long)i * P) / G);
}

// ---------------------------------------------------------------------------------------------
// Modulation values held in shared memory as bf16 or fp32.
template <typename ModT> __device__ __forceinline__ float2 mod2(const ModT* m, int col);
template <> __device__ __forceinline__ float2 mod2<uint16_t>(const uint16_t* m, int col) {
  const uint32_t v = *reinterpret_cast<const uint32_t*>(m + col);
  return make_float2(bf_lo(v), bf_hi(v));
}
template <> __device__ __forceinline__ float2 mod2<float>(const float* m, int col) {
  return *reinterpret_cast<const float2*>(m + col);
}

// ---------------------------------------------------------------------------------------------
// Dynamic shared memory of the persistent kernel; regions at the Params s_* offsets. Named at
// namespace scope so every access compiles to 32-bit shared-window addressing.
extern __shared__ __align__(1024) char g_smem[];

struct Cta {
  int r0_qkv, R_qkv, c0, R_h, u0, R_gu;
  int dgrp, d0, R_dp;  // down partials: group, first output column, output columns
  uint32_t tag0;
  int tid, warp, lane, cta, G;
  int stages;
};
// Shared-memory regions (offsets live in the kernel parameters, so nothing stays in registers).
__device__ __forceinline__ char* cSlot(const Params& p, const Cta& c, int s) { return g_smem + p.s_slot[s]; }
// X: [TP][XS] bf16, each 16-column block stored as columns 0,1,8,9, 2,3,10,11, ..., 6,7,14,15 (the
// mma.sync B-fragment order): the four columns of exchange word pair q sit at bytes [8q, 8q + 8) of
// a row, and a lane's B fragment of a k-block is one 8-byte load.
__device__ __forceinline__ char* cX(const Params& p, const Cta& c) { return g_smem + p.s_x; }
__device__ __forceinline__ float* cP(const Params& p, const Cta& c) {                          // partials / attention
  return reinterpret_cast<float*>(g_smem + p.s_p);
}
__device__ __forceinline__ char* cMods(const Params& p, const Cta& c) { return g_smem + p.s_mods; }  // 2 x 3H ModT
__device__ __forceinline__ float* cXs(const Params& p, const Cta& c) {                         // action state [TP][32]
  return reinterpret_cast<float*>(g_smem + p.s_xs);
}
__device__ __forceinline__ float* cRes(const Params& p, const Cta& c) {                        // residual [TP][RESW]
  return reinterpret_cast<float*>(g_smem + p.s_res);
}
__device__ __forceinline__ float* cRed(const Params& p, const Cta& c) {                        // small reductions
  return reinterpret_cast<float*>(g_smem + p.s_red);
}
__device__ __forceinline__ uint64_t* cBar(const Params& p, const Cta& c) {                     // NBAR mbarriers
  return reinterpret_cast<uint64_t*>(g_smem + p.s_bar);
}
__device__ __forceinline__ int* cCnt(const Params& p, const Cta& c) {                          // issued, consumed
  return reinterpret_cast<int*>(g_smem + p.s_cnt);
}

__device__ __forceinline__ void record_error(const Params& p, const Cta& c, int kind, int stage) {
  atomicCAS(p.status, 0, (c.cta << 16) | (kind << 8) | stage);
}

// Sub-stage tracing, compiled only with -DMKX_SUBSTAGE_TRACE (a separate profiling build): thread 0
// of CTAs 0 and 100 stamps %globaltimer at numbered points inside each stage, after the per-CTA
// stage-end stamps of the prof buffer: [2][1 + stages][8].
#ifdef MKX_SUBSTAGE_TRACE
__device__ __forceinline__ void trace_point(const Params& p, const Cta& c, int pt) {
  if (p.prof != nullptr && c.tid == 0 && (c.cta == 0 || c.cta == 100)) {
    const size_t per_cta = 2 + (size_t)p.n_steps * (8 * p.L + 1);
    p.prof[(size_t)c.G * per_cta + (c.cta == 0 ? 0 : per_cta * 8) + (size_t)c.stages * 8 + pt] = globaltimer();
  }
}
// The stamp taken only once `dep` is computed (a plain stamp may be scheduled ahead of the work it
// follows in the source).
__device__ __forceinline__ void trace_point_after(const Params& p, const Cta& c, int pt, uint32_t dep) {
  if (p.prof != nullptr && c.tid == 0 && (c.cta == 0 || c.cta == 100)) {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t) : "r"(dep) : "memory");
    const size_t per_cta = 2 + (size_t)p.n_steps * (8 * p.L + 1);
    p.prof[(size_t)c.G * per_cta + (c.cta == 0 ? 0 : per_cta * 8) + (size_t)c.stages * 8 + pt] = t;
  }
}
#define MKX_TRACE(pt) trace_point(p, c, pt)
#define MKX_TRACE_AFTER(pt, dep) trace_point_after(p, c, pt, dep)
#else
#define MKX_TRACE(pt) ((void)0)
#define MKX_TRACE_AFTER(pt, dep) ((void)0)
#endif

// Optional timeline: thread 0 of every CTA stamps %globaltimer at the launch start (index 0) and at
// the end of every stage (index 1 + stage).
__device__ __forceinline__ void stage_done(const Params& p, Cta& c) {
  MKX_TRACE(7);
  c.stages++;
  if (p.prof != nullptr && c.tid == 0)
    p.prof[(size_t)c.cta * (2 + p.n_steps * (8 * p.L + 1)) + c.stages] = globaltimer();
}

__device__ __forceinline__ const uint16_t* slot_src(const Params& p, const Cta& c, int slot, int l) {
  const size_t HH = (size_t)H * H;
  switch (slot) {
    case S_QKV: return p.w[S_QKV] + (size_t)l * 3 * HH + (size_t)c.r0_qkv * H;
    case S_O: return p.w[S_O] + (size_t)l * HH + (size_t)c.c0 * H;
    case S_QCA: return p.w[S_QCA] + (size_t)l * HH + (size_t)c.c0 * H;
    case S_OCA: return p.w[S_OCA] + (size_t)l * HH + (size_t)c.c0 * H;
    case S_GU: return p.w[S_GU] + (size_t)l * 2 * p.I * H + (size_t)2 * c.u0 * H;
    default: {
      const int KS = p.I / NGRP;
      return p.w[S_D] + (size_t)l * H * p.I + (size_t)c.dgrp * H * KS + (size_t)c.d0 * KS;
    }
  }
}

// ISSUER thread only.
__device__ __forceinline__ uint32_t slot_bytes(const Params& p, const Cta& c, int slot) {
  switch (slot) {
    case S_QKV: return (uint32_t)c.R_qkv * H * 2;
    case S_GU: return (uint32_t)c.R_gu * H * 4;
    case S_D: return (uint32_t)c.R_dp * (p.I / NGRP) * 2;
    default: return (uint32_t)c.R_h * H * 2;
  }
}
__device__ __forceinline__ void issue_slot(const Params& p, Cta& c, int slot, int l) {
  const uint32_t bytes = slot_bytes(p, c, slot);
  fence_proxy_async();
  mbar_expect_tx(&cBar(p, c)[slot], bytes);
  bulk_g2s_hint(cSlot(p, c, slot), slot_src(p, c, slot, l), bytes, &cBar(p, c)[slot], l2_evict_first());
  cCnt(p, c)[slot] += 1;
}

// Modulation blocks: per Euler step s, 3L + 1 blocks in use order: for each layer l the SA, CA and
// MLP blocks [scale, shift, gate] (3H values at 9Hl + 3Hb of the step's row, src/mk_expert.py:336-340),
// then the final-norm block [scale, shift] (2H values at 9HL, src/mk_expert.py:423). Block q goes to
// ring slot q & 1. ISSUER thread only.
template <typename ModT>
__device__ __forceinline__ void issue_mods(const Params& p, Cta& c, int q) {
  const int per = 3 * p.L + 1;
  if (q >= p.n_steps * per) return;
  const int s = q / per, r = q % per;
  const size_t MODW = (size_t)9 * p.L * H + 2 * H;
  const size_t off = (size_t)(1 + s) * MODW + (r < 3 * p.L ? (size_t)9 * H * (r / 3) + (size_t)3 * H * (r % 3)
                                                           : (size_t)9 * H * p.L);
  const uint32_t bytes = (uint32_t)((r < 3 * p.L ? 3 : 2) * H * sizeof(ModT));
  const int b = BAR_MODS + (q & 1);
  fence_proxy_async();
  mbar_expect_tx(&cBar(p, c)[b], bytes);
  bulk_g2s_hint(cMods(p, c) + (size_t)(q & 1) * 3 * H * sizeof(ModT), reinterpret_cast<const ModT*>(p.mods) + off, bytes,
           &cBar(p, c)[b], l2_evict_first());
  cCnt(p, c)[b] += 1;
}
template <typename ModT>
__device__ __forceinline__ const ModT* mods_slot(const Params& p, const Cta& c, int q) {
  return reinterpret_cast<const ModT*>(cMods(p, c) + (size_t)(q & 1) * 3 * H * sizeof(ModT));
}

// All threads. Returns false on timeout (error recorded).
__device__ bool wait_bar(const Params& p, Cta& c, int b) {
  const uint32_t parity = (uint32_t)(cCnt(p, c)[NBAR + b] & 1);
  uint32_t spins = 0;
  uint64_t t0 = 0;
  while (!mbar_try_wait(&cBar(p, c)[b], parity)) {
    if ((++spins & 255u) == 0u) {
      const uint64_t now = globaltimer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > p.timeout_ns) {
        record_error(p, c, K_MBAR, ST_MBAR);
        return false;
      }
    }
  }
  return true;
}
// After every thread passed wait_bar(b) and a __syncthreads: thread 0 bumps the consumed count.
__device__ __forceinline__ void consumed(const Params& p, Cta& c, int b) {
  if (c.tid == 0) cCnt(p, c)[NBAR + b] += 1;
}

// Exchange polls. issue_pairs loads N 16-byte pairs of words at addr(i) (entries outside `valid`
// count as fresh); complete_pairs re-polls the stale ones until both tags of every pair equal `tag`.
// Each round checks every pair first and then reissues all stale ones together (reissuing each
// stale pair as soon as it was checked was 1 % slower per predict); no pause between rounds (a
// 128 ns __nanosleep made the predict 50 % slower). Addresses are recomputed rather than held, to
// keep registers for the data.
// Returns 0, or the Waiter code (1 timeout, 2 abort seen).
template <int N, typename Addr>
__device__ __forceinline__ void issue_pairs(Addr addr, u64 (&w0)[N], u64 (&w1)[N], uint32_t valid, uint32_t tag) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    if ((valid >> i) & 1u) {
      ld_volatile_v2(addr(i), w0[i], w1[i]);
    } else {
      w0[i] = make_word(tag, 0u);
      w1[i] = w0[i];
    }
  }
}
template <int N, typename Addr>
__device__ __forceinline__ int complete_pairs(Addr addr, u64 (&w0)[N], u64 (&w1)[N], uint32_t tag, Waiter& wt) {
  while (true) {
    uint32_t bad = 0;
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (tag_of(w0[i]) != tag || tag_of(w1[i]) != tag) bad |= 1u << i;
    if (bad == 0u) return 0;
    const int r = wt.tick();
    if (r) return r;
#pragma unroll
    for (int i = 0; i < N; ++i)
      if ((bad >> i) & 1u) ld_volatile_v2(addr(i), w0[i], w1[i]);
  }
}
__device__ __forceinline__ int poll_word(const u64* ptr, u64& w, uint32_t tag, Waiter& wt) {
  w = ld_volatile(ptr);
  while (tag_of(w) != tag) {
    const int r = wt.tick();
    if (r) return r;
    w = ld_volatile(ptr);
  }
  return 0;
}

__device__ __forceinline__ int fail_code(const Params& p, const Cta& c, int r, int stage) {
  if (r == 1) record_error(p, c, K_TIMEOUT, stage);
  return r != 0;
}

// ---------------------------------------------------------------------------------------------
// AdaRMS staging: thread (n = tid / SROW, part = tid % SROW) owns SPAIRS word pairs of action row n,
// q = part + SROW j, i.e. columns {16kb + 2cc, +1} and {16kb + 2cc + 8, +9} with kb = q / 4, cc = q % 4.
__device__ __forceinline__ int col_a_of(int q) { return 16 * (q >> 2) + 2 * (q & 3); }

// AdaRMS of action rows into X (src/mk_expert.py:93-122): a = bf16(h * rstd * (1 + scale) + shift),
// rows >= T zero, and h kept at the CTA's residual columns. Thread (n = tid / SROW, part) owns the
// 4 SPAIRS columns of word pairs part + SROW j of row n, held in registers from load to store: h
// comes polled from an exchange buffer (`rows`), or, with rows == nullptr, from X itself (layer 0,
// where the step tail left h0). The SROW threads of a row are one half-warp, so the row's sum of
// squares is a shuffle reduction. msc: [scale H | shift H] in shared memory, already waited for.
// Returns nonzero on a failed wait (not CTA-uniform).
template <typename ModT>
__device__ int stage_rows_adarms(const Params& p, Cta& c, const u64* rows, uint32_t tag, int stage,
                                 const ModT* msc) {
  const int n = c.tid / SROW, part = c.tid % SROW;
  char* xrow = cX(p, c) + (size_t)n * XS * 2;
  const bool live = n < p.T;
  u64 w0[SPAIRS], w1[SPAIRS];
  int r = 0;
  // bf16 modulation pairs of this thread's columns, read before the polls go out: once they are in
  // flight, a shared-memory load waits behind the CTA's outstanding exchange loads (1.4 % per
  // predict). fp32 rows would need twice the registers and are read in the loop below.
  uint32_t msr[2 * SPAIRS], mhr[2 * SPAIRS];
  if constexpr (sizeof(ModT) == 2) {
#pragma unroll
    for (int j = 0; j < 2 * SPAIRS; ++j) {
      const int col = col_a_of(part + SROW * (j >> 1)) + 8 * (j & 1);
      msr[j] = *reinterpret_cast<const uint32_t*>(msc + col);
      mhr[j] = *reinterpret_cast<const uint32_t*>(msc + H + col);
    }
  }
  if (rows != nullptr) {
    const u64* base = rows + (size_t)n * HWORDS + 2 * part;
    auto addr = [base](int j) { return base + 2 * SROW * j; };
    Waiter wt(p.status, p.timeout_ns);
    issue_pairs<SPAIRS>(addr, w0, w1, live ? (1u << SPAIRS) - 1u : 0u, tag);
    r = complete_pairs<SPAIRS>(addr, w0, w1, tag, wt);
    MKX_TRACE_AFTER(6, (uint32_t)w0[SPAIRS - 1] ^ (uint32_t)w1[SPAIRS - 1]);
  } else {
#pragma unroll
    for (int j = 0; j < SPAIRS; ++j) {
      const uint2 v = *reinterpret_cast<const uint2*>(xrow + (size_t)(part + SROW * j) * 8);
      w0[j] = v.x;
      w1[j] = v.y;
    }
  }
  // Sum of squares in four independent chains (12 FMAs deep instead of 48), then across the row's
  // SROW lanes.
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < SPAIRS; ++j) {
    const uint32_t u = payload_of(w0[j]), v = payload_of(w1[j]);
    const float a = bf_lo(u), b = bf_hi(u), d = bf_lo(v), e = bf_hi(v);
    s4[0] = fmaf(a, a, s4[0]);
    s4[1] = fmaf(b, b, s4[1]);
    s4[2] = fmaf(d, d, s4[2]);
    s4[3] = fmaf(e, e, s4[3]);
  }
  float ss = (s4[0] + s4[1]) + (s4[2] + s4[3]);
#pragma unroll
  for (int o = SROW / 2; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (rows != nullptr) MKX_TRACE_AFTER(4, __float_as_uint(ss));
  const float rstd = rsqrtf(ss / (float)H + p.eps);
  const ModT* msh = msc + H;
  float* res = cRes(p, c) + n * RESW;
  // All modulation loads and arithmetic first, then all stores: a store to X could alias a later
  // modulation load (both shared memory), so interleaved they serialise load -> store -> load.
  uint32_t outv[2 * SPAIRS];
#pragma unroll
  for (int j = 0; j < 2 * SPAIRS; ++j) {  // column pairs (ca, ca+1) then (ca+8, ca+9) of word pair j / 2
    const int col = col_a_of(part + SROW * (j >> 1)) + 8 * (j & 1);
    const uint32_t u = payload_of((j & 1) ? w1[j >> 1] : w0[j >> 1]);
    const float h0 = bf_lo(u), h1 = bf_hi(u);
    float2 sc, sh;
    if constexpr (sizeof(ModT) == 2) {
      sc = make_float2(bf_lo(msr[j]), bf_hi(msr[j]));
      sh = make_float2(bf_lo(mhr[j]), bf_hi(mhr[j]));
    } else {
      sc = mod2<ModT>(msc, col);
      sh = mod2<ModT>(msh, col);
    }
    const float a0 = fmaf(h0 * rstd, 1.f + sc.x, sh.x);
    const float a1 = fmaf(h1 * rstd, 1.f + sc.y, sh.y);
    outv[j] = live ? pack_bf2(a0, a1) : 0u;
  }
  if (rows != nullptr) MKX_TRACE_AFTER(1, outv[2 * SPAIRS - 1] ^ outv[0]);
#pragma unroll
  for (int i = 0; i < SPAIRS; ++i)  // word pair q of the row = X bytes [8q, 8q + 8)
    *reinterpret_cast<uint2*>(xrow + (size_t)(part + SROW * i) * 8) = make_uint2(outv[2 * i], outv[2 * i + 1]);
#pragma unroll
  for (int j = 0; j < 2 * SPAIRS; ++j) {
    const int col = col_a_of(part + SROW * (j >> 1)) + 8 * (j & 1);
    // c0 and R_h are even: a column pair is entirely inside or outside the residual columns
    if (live && (unsigned)(col - c.c0) < (unsigned)c.R_h) {
      const uint32_t u = payload_of((j & 1) ? w1[j >> 1] : w0[j >> 1]);
      *reinterpret_cast<float2*>(res + (col - c.c0)) = make_float2(bf_lo(u), bf_hi(u));
    }
  }
  return fail_code(p, c, r, stage);
}

// ---------------------------------------------------------------------------------------------
// Split of a shared-memory GEMM over the NW warps: `nmat` matrices (<= 2) of R rows (<= 32), i.e. mt
// m-tiles of 16 rows in total (1, 2 or 4: a power of two), each K-split ks = NW / mt ways. Shifts and
// masks only: these sit on the critical path of every stage.
struct Split {
  int lmtpm, lmt, lks;  // log2 of m-tiles per matrix, of m-tiles, of K-splits
};
__device__ __forceinline__ Split gemm_split(int nmat, int R) {
  Split q;
  q.lmtpm = R > 16 ? 1 : 0;
  q.lmt = q.lmtpm + (nmat > 1 ? 1 : 0);
  q.lks = 3 - q.lmt;  // NW = 8
  return q;
}
static_assert(NW == 8, "gemm_split assumes 8 warps");

// ---------------------------------------------------------------------------------------------
// K-split partials, token-major: P[block][token n][PSTR] holds the 16 output rows of a (m-tile, K-split)
// block for token n. The epilogue reads a lane's two rows (2pp, 2pp + 1) as one aligned float2 and
// consecutive lanes read consecutive float2s; the MMA lanes' stores fall in distinct banks (8 cc + g).
__device__ __forceinline__ void store_partials(const Params& p, const Cta& c, const float (&d0)[4], const float (&d1)[4]) {
  const int g = c.lane >> 2, cc = c.lane & 3;
  float* P = cP(p, c) + c.warp * PM;
  P[(2 * cc) * PSTR + g] = d0[0];
  P[(2 * cc + 1) * PSTR + g] = d0[1];
  P[(2 * cc) * PSTR + g + 8] = d0[2];
  P[(2 * cc + 1) * PSTR + g + 8] = d0[3];
  P[(8 + 2 * cc) * PSTR + g] = d1[0];
  P[(8 + 2 * cc + 1) * PSTR + g] = d1[1];
  P[(8 + 2 * cc) * PSTR + g + 8] = d1[2];
  P[(8 + 2 * cc + 1) * PSTR + g + 8] = d1[3];
}

// GEMM with the B operand (activations) from shared X: `nmat` matrices of R rows each (K = H).
__device__ void mma_from_x(const Params& p, Cta& c, const char* wslot, int nmat, int R) {
  const Split q = gemm_split(nmat, R);
  const int g = c.lane >> 2, cc = c.lane & 3;
  const bool two = p.T > 8;
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
  {  // mt * ks == NW: every warp has a (m-tile, K-range)
    const int m = c.warp & ((1 << q.lmt) - 1), ksl = c.warp >> q.lmt;
    const int j = m >> q.lmtpm, mm = m & ((1 << q.lmtpm) - 1);
    const char* A = wslot + (size_t)j * R * H * 2 + cc * 8;
    constexpr int KB = H / 16;
    const int kb0 = (ksl * KB) >> q.lks, kb1 = ((ksl + 1) * KB) >> q.lks;
    const int ra = mm * 16 + g, rb = ra + 8;
    const bool va = ra < R, vb = rb < R;
    const char* x0 = cX(p, c) + (size_t)g * XS * 2 + cc * 8;
    const char* x1 = cX(p, c) + (size_t)(8 + g) * XS * 2 + cc * 8;
#pragma unroll 4
    for (int kb = kb0; kb < kb1; ++kb) {
      const char* blk = A + (size_t)kb * R * 32;
      const uint2 a = va ? lds64(blk + ra * 32) : make_uint2(0u, 0u);
      const uint2 b = vb ? lds64(blk + rb * 32) : make_uint2(0u, 0u);
      const uint2 bx = lds64(x0 + kb * 32);
      mma_bf16(d0, a.x, b.x, a.y, b.y, bx.x, bx.y);
      if (two) {
        const uint2 ex = lds64(x1 + kb * 32);
        mma_bf16(d1, a.x, b.x, a.y, b.y, ex.x, ex.y);
      }
    }
  }
  store_partials(p, c, d0, d1);
}

// GEMM with the B operand polled straight from an exchange buffer (rows of K/2 words); one matrix
// of R <= 16 rows, K split over the 8 warps, in chunks of CH k-blocks with the next chunk's loads
// in flight while the current chunk is checked and multiplied. Returns nonzero on a failed wait.
template <int CH>
struct WordChunk {
  u64 w0[2 * CH], w1[2 * CH];
};

__device__ int mma_from_words(const Params& p, Cta& c, const char* wslot, int R, int K, const u64* rows,
                              uint32_t tag, int stage) {
  constexpr int CH = 4;
  const int g = c.lane >> 2, cc = c.lane & 3;
  const int RW = K >> 1, KB = K >> 4;
  const int kb0 = c.warp * KB / NW, kb1 = (c.warp + 1) * KB / NW;
  const bool v0 = g < p.T, v1 = (8 + g) < p.T, two = p.T > 8;
  const u64* row0 = rows + (size_t)g * RW + 2 * cc;
  const size_t d1off = (size_t)8 * RW;  // row 8 + g
  const char* A = wslot + cc * 8;
  const bool va = g < R, vb = g + 8 < R;
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
  Waiter wt(p.status, p.timeout_ns);
  const int nch = (kb1 - kb0 + CH - 1) / CH;
  WordChunk<CH> buf0, buf1;
  auto issue = [&](WordChunk<CH>& b, int ch) {
    const int kbase = kb0 + ch * CH;
    uint32_t valid = 0;
#pragma unroll
    for (int i = 0; i < CH; ++i)
      if (kbase + i < kb1) valid |= ((v0 ? 1u : 0u) | (v1 ? 2u : 0u)) << (2 * i);
    const u64* base = row0 + kbase * 8;
    issue_pairs<2 * CH>([base, d1off](int i) { return base + (i >> 1) * 8 + ((i & 1) ? d1off : 0); }, b.w0, b.w1,
                        valid, tag);
  };
  // Weight fragments of two chunks, read before their polls go out (a shared-memory load issued
  // behind outstanding exchange loads waits for them).
  uint2 ap0[CH], bp0[CH], ap1[CH], bp1[CH];
  auto prefetch = [&](uint2 (&ap)[CH], uint2 (&bp)[CH], int ch) {
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int kb = kb0 + ch * CH + i;
      const char* blk = A + (size_t)kb * R * 32;
      ap[i] = (kb < kb1 && va) ? lds64(blk + g * 32) : make_uint2(0u, 0u);
      bp[i] = (kb < kb1 && vb) ? lds64(blk + (g + 8) * 32) : make_uint2(0u, 0u);
    }
  };
  auto consume = [&](WordChunk<CH>& b, int ch, const uint2 (&ap)[CH], const uint2 (&bp)[CH]) -> int {
    const int kbase = kb0 + ch * CH;
    const u64* base = row0 + kbase * 8;
    int rc = complete_pairs<2 * CH>([base, d1off](int i) { return base + (i >> 1) * 8 + ((i & 1) ? d1off : 0); },
                                    b.w0, b.w1, tag, wt);
    if (__any_sync(0xffffffffu, rc != 0)) return rc ? rc : 2;  // keep the warp converged for mma.sync
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int kb = kbase + i;
      if (kb < kb1) {
        const uint2 a = ap[i], bb = bp[i];
        mma_bf16(d0, a.x, bb.x, a.y, bb.y, payload_of(b.w0[2 * i]), payload_of(b.w1[2 * i]));
        if (two) mma_bf16(d1, a.x, bb.x, a.y, bb.y, payload_of(b.w0[2 * i + 1]), payload_of(b.w1[2 * i + 1]));
      }
    }
    return 0;
  };
  int rc = 0;
  prefetch(ap0, bp0, 0);
  prefetch(ap1, bp1, 1);
  if (nch > 0) issue(buf0, 0);
  for (int ch = 0; ch < nch; ch += 2) {
    if (ch + 1 < nch) issue(buf1, ch + 1);
    rc = consume(buf0, ch, ap0, bp0);
    if (rc || ch + 1 >= nch) break;
    if (ch + 2 < nch) {
      prefetch(ap0, bp0, ch + 2);
      issue(buf0, ch + 2);
    }
    rc = consume(buf1, ch + 1, ap1, bp1);
    if (rc) break;
    if (ch + 3 < nch) prefetch(ap1, bp1, ch + 3);
  }
  store_partials(p, c, d0, d1);
  return fail_code(p, c, rc, stage);
}

// Sum of the K-split partials for output rows 2pp, 2pp + 1 (of matrix j), token n.
__device__ __forceinline__ float2 part_sum2(const Params& p, const Cta& c, const Split& q, int j, int pp, int n) {
  const int r = 2 * pp;
  const int m = (j << q.lmtpm) + (r >> 4);
  const float* P = cP(p, c) + m * PM + n * PSTR + (r & 15);
  const int ks = NW >> q.lmt, mt = 1 << q.lmt;
  float2 s[NW];  // independent loads, summed as a tree (the K-split order is fixed per geometry)
#pragma unroll
  for (int k = 0; k < NW; ++k) s[k] = k < ks ? *reinterpret_cast<const float2*>(P + mt * k * PM) : make_float2(0.f, 0.f);
#pragma unroll
  for (int w = NW / 2; w >= 1; w >>= 1)
#pragma unroll
    for (int k = 0; k < w; ++k) {
      s[k].x += s[k + w].x;
      s[k].y += s[k + w].y;
    }
  return s[0];
}

// Epilogues ----------------------------------------------------------------------------------
// Linear output rounded to bf16 (QKV, CA query): words of columns [col0, col0 + R).
// Epilogue threads: e -> (column pair pp = e % npairs, action row n = e / npairs): consecutive lanes
// publish consecutive words of a row (coalesced exchange stores).
__device__ void epi_plain(const Params& p, const Cta& c, int R, int col0, u64* out_rows, int row_words,
                          uint32_t tag) {
  const int npairs = R >> 1, pp = c.tid % npairs, n = c.tid / npairs;
  if (c.tid < npairs * p.T) {
    const Split q = gemm_split(1, R);
    const float2 v = part_sum2(p, c, q, 0, pp, n);
    const float v0 = v.x, v1 = v.y;
    st_volatile(out_rows + (size_t)n * row_words + word_pos((col0 >> 1) + pp), make_word(tag, pack_bf2(v0, v1)));
  }
}

// Gated residual out = bf16(res + bf16(acc) * gate) (src/mk_expert.py:162-172) of the column pair
// c0 + 2 pp, token n; gate in shared memory.
template <typename ModT>
__device__ __forceinline__ void gated_pair_store(const Params& p, const Cta& c, const ModT* gate, u64* out_rows,
                                                 uint32_t tag, uint16_t* trace, int pp, int n, float2 v) {
  const float2 gv = mod2<ModT>(gate, c.c0 + 2 * pp);
  const float a0 = round_bf(v.x), a1 = round_bf(v.y);
  const float o0 = fmaf(a0, gv.x, cRes(p, c)[n * RESW + 2 * pp]);
  const float o1 = fmaf(a1, gv.y, cRes(p, c)[n * RESW + 2 * pp + 1]);
  const uint32_t pl = pack_bf2(o0, o1);
  st_volatile(out_rows + (size_t)n * HWORDS + word_pos((c.c0 >> 1) + pp), make_word(tag, pl));
  if (trace) *reinterpret_cast<uint32_t*>(trace + (size_t)n * H + c.c0 + 2 * pp) = pl;
}
template <typename ModT>
__device__ void epi_gated(const Params& p, const Cta& c, const ModT* gate, u64* out_rows, uint32_t tag) {
  const int npairs = c.R_h >> 1, pp = c.tid % npairs, n = c.tid / npairs;
  if (c.tid < npairs * p.T)
    gated_pair_store<ModT>(p, c, gate, out_rows, tag, nullptr, pp, n, part_sum2(p, c, gemm_split(1, c.R_h), 0, pp, n));
}

// g = bf16(silu(bf16(gate)) * bf16(up)) (src/mk_expert.py:403-413).
__device__ void epi_gu(const Params& p, const Cta& c, u64* out_rows, uint32_t tag) {
  const int R = c.R_gu, row_words = p.I >> 1;
  const int npairs = R >> 1, pp = c.tid % npairs, n = c.tid / npairs;
  if (c.tid < npairs * p.T) {
    const Split q = gemm_split(2, R);
    const float2 gv = part_sum2(p, c, q, 0, pp, n), uv = part_sum2(p, c, q, 1, pp, n);
    float o[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float gf = round_bf(k ? gv.y : gv.x);
      const float uf = round_bf(k ? uv.y : uv.x);
      o[k] = __fdividef(gf, 1.f + __expf(-gf)) * uf;
    }
    st_volatile(out_rows + (size_t)n * row_words + word_pos((c.u0 >> 1) + pp), make_word(tag, pack_bf2(o[0], o[1])));
  }
}

// ---------------------------------------------------------------------------------------------
// Attention for one (head h, action row t) unit. Thread = (key group kg = tid / 8, l8 = tid % 8);
// each 8-lane group owns keys kg, kg + 32, ...; lane l8 owns 8 of the 64 head dims, namely the
// columns of words 4*l8 .. 4*l8 + 3 of the head's 32-word segment, in "lane order"
// [d0, d0+1, d0+8, d0+9, d0+2, d0+3, d0+10, d0+11] with d0 = 16 (l8 / 2) + 4 (l8 % 2).
struct Lane8 {
  float v[8];
};
__device__ __forceinline__ void bf_words_to_lane(Lane8& x, uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
  x.v[0] = bf_lo(w0); x.v[1] = bf_hi(w0);
  x.v[2] = bf_lo(w1); x.v[3] = bf_hi(w1);
  x.v[4] = bf_lo(w2); x.v[5] = bf_hi(w2);
  x.v[6] = bf_lo(w3); x.v[7] = bf_hi(w3);
}
// Natural-order bf16 row chunk (dims d0..d0+3 in A, d0+8..d0+11 in B) to lane order.
__device__ __forceinline__ void bf_nat_to_lane(Lane8& x, uint2 A, uint2 B) { bf_words_to_lane(x, A.x, B.x, A.y, B.y); }
__device__ __forceinline__ void f32_nat_to_lane(Lane8& x, float4 A, float4 B) {
  x.v[0] = A.x; x.v[1] = A.y; x.v[2] = B.x; x.v[3] = B.y;
  x.v[4] = A.z; x.v[5] = A.w; x.v[6] = B.z; x.v[7] = B.w;
}
__device__ __forceinline__ void f32_lane_pin(Lane8& x, const float* row, int d0) {
  f32_nat_to_lane(x, ldg_f4_pin(row + d0), ldg_f4_pin(row + d0 + 8));
}
__device__ __forceinline__ float group8_sum(float s) {
  s += __shfl_xor_sync(0xffffffffu, s, 1);
  s += __shfl_xor_sync(0xffffffffu, s, 2);
  s += __shfl_xor_sync(0xffffffffu, s, 4);
  return s;
}
// Per-head RMSNorm (weight 1 + w) then rotate-half RoPE, bf16 rounded after each
// (src/mk_expert.py:175-193). Partner dim d + 32 lives in lane l8 ^ 4 at the same slot.
__device__ __forceinline__ void norm_rope(Lane8& x, const Lane8& wn, const Lane8& cs, const Lane8& sn, float eps,
                                          int l8) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) ss = fmaf(x.v[i], x.v[i], ss);
  ss = group8_sum(ss);
  const float r = rsqrtf(ss / (float)HD + eps);
  const float sign = l8 < 4 ? -1.f : 1.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float xn = round_bf(x.v[i] * r * wn.v[i]);
    const float xp = __shfl_xor_sync(0xffffffffu, xn, 4);
    x.v[i] = round_bf(fmaf(xn, cs.v[i], sign * xp * sn.v[i]));
  }
}
__device__ __forceinline__ float dot8(const Lane8& a, const Lane8& b) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s = fmaf(a.v[i], b.v[i], s);
  return group8_sum(s);
}
// Block-wide max of a value that is uniform within each 8-lane group, with an OR of `fail` over
// the block taken at the same barrier. The per-warp slots alternate with `buf` (the chunk parity):
// a thread writing slot set b has passed the previous chunk's barrier, after which nobody reads
// set b any more.
__device__ __forceinline__ float block_max(const Params& p, const Cta& c, float v, int buf, int fail, int& any_fail) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
  float* red = cRed(p, c) + buf * NW;
  if (c.lane == 0) red[c.warp] = v;
  any_fail = __syncthreads_or(fail);
  float m[NW];
#pragma unroll
  for (int w = 0; w < NW; ++w) m[w] = red[w];
#pragma unroll
  for (int w = NW / 2; w >= 1; w >>= 1)
#pragma unroll
    for (int k = 0; k < w; ++k) m[k] = fmaxf(m[k], m[k + w]);
  return m[0];
}

// SA = true: self-attention (queries of row t over memory rows [cu_kv[0], PM) and the T action
// rows, src/mk_expert.py:196-222). SA = false: cross-attention over the S valid source rows
// (src/mk_expert.py:225-251). Returns nonzero on a failed wait.
__device__ __forceinline__ int attention_unit(const Params& p, Cta& c, const bool SA, int l, int h, int t,
                                              const u64* src_rows, u64* y_rows, uint32_t tag) {
  const int kg = c.tid >> 3, l8 = c.tid & 7;
  const int d0 = 16 * (l8 >> 1) + 4 * (l8 & 1);
  const int nkeys = SA ? p.mem_rows : min(__ldg(p.cu_src + 1), p.ca_rows);
  const int kbeg = SA ? __ldg(p.cu_kv) : 0;
  const uint16_t* Kb = SA ? p.memk[l] : p.kca[l];
  const uint16_t* Vb = SA ? p.memv[l] : p.vca[l];
  const int stride = SA ? p.mem_row_stride : p.ca_row_stride;
  const float* nrm = p.nrm + (size_t)((SA ? 0 : 2) * p.L + l) * HD;
  const float* cosr = (SA ? p.sa_cos : p.ca_cos);
  const float* sinr = (SA ? p.sa_sin : p.ca_sin);

  // Load chunk 0 of K/V and the per-row tables; none of it depends on the exchange, and the pinned
  // loads are in flight while the query is polled.
  uint2 kA[MAXK], kB[MAXK], vA[MAXK], vB[MAXK];
  const uint64_t keep = l2_evict_last();  // K/V are re-read every Euler step: keep them in L2
  auto load_chunk = [&](int base) {
#pragma unroll
    for (int i = 0; i < MAXK; ++i) {
      const int j = base + kg + NG * i;
      kA[i] = kB[i] = vA[i] = vB[i] = make_uint2(0u, 0u);
      if (j < nkeys) {
        const uint16_t* kr = Kb + (size_t)j * stride + h * HD + d0;
        const uint16_t* vr = Vb + (size_t)j * stride + h * HD + d0;
        kA[i] = ldg_u2_pin_hint(kr, keep);
        kB[i] = ldg_u2_pin_hint(kr + 8, keep);
        vA[i] = ldg_u2_pin_hint(vr, keep);
        vB[i] = ldg_u2_pin_hint(vr + 8, keep);
      }
    }
  };
  load_chunk(kbeg);
  Lane8 wq, cq, sq;
  f32_lane_pin(wq, nrm, d0);
  f32_lane_pin(cq, cosr + (size_t)t * HD, d0);
  f32_lane_pin(sq, sinr + (size_t)t * HD, d0);
  const bool own = SA && kg < p.T;
  Lane8 wk, ck, sk;
  if (SA) {
    const int krow = kg < p.T ? kg : p.T - 1;  // groups without an own row compute a discarded key
    f32_lane_pin(wk, nrm + (size_t)p.L * HD, d0);
    f32_lane_pin(ck, cosr + (size_t)krow * HD, d0);
    f32_lane_pin(sk, sinr + (size_t)krow * HD, d0);
  }

  // Poll the query (and, for SA, this group's own action row's k and v).
  const int qoff = h * 32 + 4 * l8;
  const int row_words = SA ? QKVWORDS : HWORDS;
  u64 w0[6], w1[6];
  const u64* qrow = src_rows + (size_t)t * row_words + qoff;
  const u64* krow = src_rows + (size_t)kg * row_words + HWORDS + qoff;  // k at +HWORDS, v at +2 HWORDS
  auto addr = [qrow, krow](int i) { return (i < 2 ? qrow : krow + (i >> 2) * HWORDS) + 2 * (i & 1); };
  Waiter wt(p.status, p.timeout_ns);
  issue_pairs<6>(addr, w0, w1, own ? 0x3fu : 0x3u, tag);
  // A failed wait is OR-ed over the block at the first chunk's block_max barrier; until then the
  // lanes compute on whatever they hold (registers only).
  const int rc = complete_pairs<6>(addr, w0, w1, tag, wt);
  const int fail = fail_code(p, c, rc, SA ? ST_SA : ST_CA);
  MKX_TRACE(1);

  Lane8 q;
  bf_words_to_lane(q, payload_of(w0[0]), payload_of(w1[0]), payload_of(w0[1]), payload_of(w1[1]));
  norm_rope(q, wq, cq, sq, p.qk_eps, l8);
  Lane8 ko, vo;
  float s_own = -INFINITY;
  if (SA) {
    bf_words_to_lane(ko, payload_of(w0[2]), payload_of(w1[2]), payload_of(w0[3]), payload_of(w1[3]));
    bf_words_to_lane(vo, payload_of(w0[4]), payload_of(w1[4]), payload_of(w0[5]), payload_of(w1[5]));
    norm_rope(ko, wk, ck, sk, p.qk_eps, l8);  // all lanes: the shuffles need the full warp
  }

  float m_run = -INFINITY, den = 0.f;
  float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  int chunk = 0;
  bool checked = false;  // the poll's failure flag went through a block_max barrier
  for (int base = kbeg; base < nkeys || (SA && base == kbeg); base += NG * MAXK, ++chunk) {
    if (base != kbeg) load_chunk(base);
    // Scores of the MAXK key slots (and, on SA's first chunk, of the own row): every slot's 8-term
    // lane sum first, then each group-of-8 shuffle level across all slots at once (the same
    // reduction order as dot8, without a shuffle chain per slot). Slots without a key hold zero K
    // and are masked below; all lanes run every shuffle.
    const bool with_own = SA && base == kbeg;  // uniform
    float s[MAXK + 1];
#pragma unroll
    for (int i = 0; i <= MAXK; ++i) {
      s[i] = 0.f;
      if (i < MAXK || with_own) {
        Lane8 k;
        if (i < MAXK) bf_nat_to_lane(k, kA[i], kB[i]);
        else k = ko;
#pragma unroll
        for (int e = 0; e < 8; ++e) s[i] = fmaf(q.v[e], k.v[e], s[i]);
      }
    }
#pragma unroll
    for (int lv = 1; lv <= 4; lv <<= 1)
#pragma unroll
      for (int i = 0; i <= MAXK; ++i)
        if (i < MAXK || with_own) s[i] += __shfl_xor_sync(0xffffffffu, s[i], lv);
    if (with_own && own) s_own = s[MAXK] * p.sm_scale;
    float mloc = with_own ? s_own : -INFINITY;
#pragma unroll
    for (int i = 0; i < MAXK; ++i) {
      const int j = base + kg + NG * i;
      s[i] = j < nkeys ? s[i] * p.sm_scale : -INFINITY;
      mloc = fmaxf(mloc, s[i]);
    }
    int any_fail;
    const float m_new = fmaxf(m_run, block_max(p, c, mloc, chunk & 1, fail, any_fail));
    if (any_fail) return 1;
    checked = true;
    MKX_TRACE(3);
    const float alpha = __expf(m_run - m_new);  // 0 on the first chunk
    den *= alpha;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] *= alpha;
    if (SA && base == kbeg && own) {
      const float pe = __expf(s_own - m_new);
      den += pe;
      const float pb = round_bf(pe);
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = fmaf(pb, vo.v[e], o[e]);
    }
#pragma unroll
    for (int i = 0; i < MAXK; ++i) {
      const int j = base + kg + NG * i;
      if (j < nkeys) {
        const float pe = __expf(s[i] - m_new);
        den += pe;
        const float pb = round_bf(pe);
        Lane8 v;
        bf_nat_to_lane(v, vA[i], vB[i]);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = fmaf(pb, v.v[e], o[e]);
      }
    }
    m_run = m_new;
    if (base + NG * MAXK >= nkeys) break;
  }
  if (!checked && __syncthreads_or(fail)) return 1;  // no key at all (uniform)
  // Reduce the NG key groups: the 4 groups of a warp by shuffles (lanes l8, l8 + 8, l8 + 16, l8 + 24
  // hold the same dims), then the NW warps' partials through shared memory. o is in lane order; den
  // is uniform within a group. The previous reader of P finished before the stage's last barrier.
  MKX_TRACE(2);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    o[e] += __shfl_xor_sync(0xffffffffu, o[e], 8);
    o[e] += __shfl_xor_sync(0xffffffffu, o[e], 16);
  }
  den += __shfl_xor_sync(0xffffffffu, den, 8);
  den += __shfl_xor_sync(0xffffffffu, den, 16);
  float* ro = cP(p, c);          // [NW][64]
  float* rd = ro + NW * 64;      // [NW]
  if (c.lane < 8) {
#pragma unroll
    for (int e = 0; e < 8; ++e) ro[c.warp * 64 + l8 * 8 + e] = o[e];
    if (l8 == 0) rd[c.warp] = den;
  }
  MKX_TRACE(4);
  __syncthreads();
  MKX_TRACE(5);
  if (c.tid < 64) {
    float acc[NW], dsum[NW];
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      acc[w] = ro[w * 64 + c.tid];
      dsum[w] = rd[w];
    }
#pragma unroll
    for (int w = NW / 2; w >= 1; w >>= 1)
#pragma unroll
      for (int k = 0; k < w; ++k) {
        acc[k] += acc[k + w];
        dsum[k] += dsum[k + w];
      }
    const float val = acc[0] / dsum[0];
    const float nxt = __shfl_down_sync(0xffffffffu, val, 1);
    if ((c.tid & 1) == 0)
      st_volatile(y_rows + (size_t)t * HWORDS + h * 32 + (c.tid >> 1), make_word(tag, pack_bf2(val, nxt)));
  }
  return 0;
}

// ---------------------------------------------------------------------------------------------
// Step tail (src/mk_expert.py:254-299), split in two:
//
// velocity_row: CTA n < T, action row n. o = bf16(AdaRMS_final(h[n])) (final-norm scale/shift from
// the modulation ring), v_a = o . Wout[a] + bout[a] in fp32, x_a <- xpad_a + dt v_a. Thread t < 192
// owns the 4 columns of word pair t of row n. Intermediate steps publish x_a (a < action_dim) as
// tagged fp32 words; the last step writes x_out[n][0..A) (dims >= action_dim: 0 + dt v_a).
template <typename ModT>
__device__ int velocity_row(const Params& p, Cta& c, int n, bool last, const ModT* mfin, const u64* hrows,
                            uint32_t htag, u64* xrows, uint32_t xtag) {
  const int t = c.tid;
  const bool act = t < HWORDS / 2;
  const int ca = col_a_of(act ? t : 0);
  const float dt = __ldg(p.dt);
  float2 wa[AO], wb[AO];
  const int ndim = last ? p.A : p.adim;
  if (!last) {
#pragma unroll
    for (int a = 0; a < AO; ++a) {
      const bool ok = act && a < ndim;
      wa[a] = ok ? ldg_f2_pin(p.wout + (size_t)a * H + ca) : make_float2(0.f, 0.f);
      wb[a] = ok ? ldg_f2_pin(p.wout + (size_t)a * H + ca + 8) : make_float2(0.f, 0.f);
    }
  }
  u64 w0 = make_word(htag, 0u), w1 = w0;
  Waiter wt(p.status, p.timeout_ns);
  int rc = 0;
  if (act) {
    const u64* ptr = hrows + (size_t)n * HWORDS + 2 * t;
    ld_volatile_v2(ptr, w0, w1);
    while (rc == 0 && (tag_of(w0) != htag || tag_of(w1) != htag)) {
      rc = wt.tick();
      ld_volatile_v2(ptr, w0, w1);
    }
  }
  fail_code(p, c, rc, ST_TAIL);
  if (__syncthreads_or(rc != 0)) return 1;
  const float h0 = bf_lo(payload_of(w0)), h1 = bf_hi(payload_of(w0));
  const float h2 = bf_lo(payload_of(w1)), h3 = bf_hi(payload_of(w1));
  float ss = h0 * h0 + h1 * h1 + h2 * h2 + h3 * h3;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (c.lane == 0) cRed(p, c)[c.warp] = ss;
  __syncthreads();
  ss = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) ss += cRed(p, c)[w];
  const float rstd = rsqrtf(ss / (float)H + p.eps);
  const float2 sa = mod2<ModT>(mfin, ca), sb = mod2<ModT>(mfin, ca + 8);
  const float2 ha = mod2<ModT>(mfin + H, ca), hb = mod2<ModT>(mfin + H, ca + 8);
  const float o0 = act ? round_bf(fmaf(h0 * rstd, 1.f + sa.x, ha.x)) : 0.f;
  const float o1 = act ? round_bf(fmaf(h1 * rstd, 1.f + sa.y, ha.y)) : 0.f;
  const float o2 = act ? round_bf(fmaf(h2 * rstd, 1.f + sb.x, hb.x)) : 0.f;
  const float o3 = act ? round_bf(fmaf(h3 * rstd, 1.f + sb.y, hb.y)) : 0.f;
  float* vred = cRed(p, c) + 16;  // [NW][AO]
  for (int a0 = 0; a0 < ndim; a0 += AO) {
    if (last) {
#pragma unroll
      for (int a = 0; a < AO; ++a) {
        const bool ok = act && a0 + a < ndim;
        wa[a] = ok ? ldg_f2_pin(p.wout + (size_t)(a0 + a) * H + ca) : make_float2(0.f, 0.f);
        wb[a] = ok ? ldg_f2_pin(p.wout + (size_t)(a0 + a) * H + ca + 8) : make_float2(0.f, 0.f);
      }
    }
#pragma unroll
    for (int a = 0; a < AO; ++a) {
      float acc = o0 * wa[a].x;
      acc = fmaf(o1, wa[a].y, acc);
      acc = fmaf(o2, wb[a].x, acc);
      acc = fmaf(o3, wb[a].y, acc);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (c.lane == 0) vred[c.warp * AO + a] = acc;
    }
    __syncthreads();
    if (t < AO && a0 + t < ndim) {
      const int a = a0 + t;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) v += vred[w * AO + t];
      v += __ldg(p.tailw + AO * H + H + a);
      const float xp = a < p.adim ? cXs(p, c)[n * 32 + a] : 0.f;
      const float xn = fmaf(dt, v, xp);
      if (last)
        p.x_out[(size_t)n * p.A + a] = xn;
      else
        st_volatile(xrows + (size_t)n * XWORDS + a, make_word(xtag, __float_as_uint(xn)));
    }
    __syncthreads();
  }
  return 0;
}

// Every CTA: the new action state from the exchange (intermediate steps). Returns nonzero (CTA-
// uniform) on a failed wait.
__device__ int take_new_x(const Params& p, Cta& c, const u64* xrows, uint32_t xtag) {
  const int t = c.tid;
  const int n = t >> 3, a = t & 7;
  int rc = 0;
  if (n < p.T && a < p.adim) {
    Waiter wt(p.status, p.timeout_ns);
    u64 w;
    rc = poll_word(xrows + (size_t)n * XWORDS + a, w, xtag, wt);
    if (rc == 0) cXs(p, c)[n * 32 + a] = __uint_as_float(payload_of(w));
  }
  fail_code(p, c, rc, ST_TAIL);
  return __syncthreads_or(rc != 0);
}

// In-projection h0 = bf16(xpad[:AO] @ Win[:AO] + bin) in fp32 (src/mk_expert.py:280-293) into X
// (in X's permuted column order); thread t owns columns t, t + NT, ... below H, whose Win / bin
// values it loads up front.
__device__ __forceinline__ void load_inproj(const Params& p, const Cta& c, float (&win)[NCOL][AO], float (&bin)[NCOL]) {
#pragma unroll
  for (int k = 0; k < NCOL; ++k) {
    const int col = min(c.tid + NT * k, H - 1);  // threads past H load a valid column and skip it
#pragma unroll
    for (int a = 0; a < AO; ++a) win[k][a] = ldg_f1_pin(p.tailw + (size_t)a * H + col);
    bin[k] = ldg_f1_pin(p.tailw + AO * H + col);
  }
}

__device__ void in_proj_to_x(const Params& p, Cta& c, const float (&win)[NCOL][AO], const float (&bin)[NCOL]) {
#pragma unroll 1
  for (int n = 0; n < TP; ++n) {
    float xp[AO];
#pragma unroll
    for (int a = 0; a < AO; ++a) xp[a] = (a < p.adim && n < p.T) ? cXs(p, c)[n * 32 + a] : 0.f;
#pragma unroll
    for (int k = 0; k < NCOL; ++k) {
      if (c.tid + NT * k >= H) break;
      float acc = bin[k];
#pragma unroll
      for (int a = 0; a < AO; ++a) acc = fmaf(xp[a], win[k][a], acc);
      const int col = c.tid + NT * k;  // X holds each 16-column block as 0,1,8,9, 2,3,10,11, ...
      const int pos = (col & ~15) + ((col & 7) >> 1) * 4 + ((col >> 3) & 1) * 2 + (col & 1);
      reinterpret_cast<__nv_bfloat16*>(cX(p, c))[(size_t)n * XS + pos] =
          __float2bfloat16_rn(n < p.T ? acc : 0.f);
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Stage routines. The per-layer loop below calls each routine from exactly one place, so each
// distinct stage exists once in the binary: the loop's code stays resident in the SM instruction
// cache instead of being re-fetched from L2 every layer. Each returns nonzero (CTA-uniform) after a
// failed wait.

// AdaRMS + GEMM stages. which = 0: QKV of AdaRMS(h; sa) (h from the previous layer, or from X for
// layer 0, where the step tail left h0); 1: CA query of AdaRMS(h2; ca); 2: gate/up of
// AdaRMS(h3; mlp) with g = bf16(silu(bf16(gate)) * bf16(up)).
template <typename ModT>
__device__ __forceinline__ int stage_norm_gemm(const Params& p, Cta& c, int which, int gi, int l, int q) {
  const int par = gi & 1;
  const uint32_t tag = c.tag0 + (uint32_t)gi;
  u64* const* xb = p.xb;
  // Every thread waits on the modulation and weight mbarriers itself (completion makes the bulk
  // copies visible to it), so one barrier after the staging covers all three waits.
  int fail = !wait_bar(p, c, BAR_MODS + (q & 1));
  const u64* rows = nullptr;  // layer 0's h0 is already in X (step tail)
  if (!(which == 0 && l == 0))
    rows = which == 0 ? xb[B_HOUT] + (size_t)((gi - 1) & 1) * TP * HWORDS
                      : xb[which == 1 ? B_H2 : B_H3] + (size_t)par * TP * HWORDS;
  fail |= stage_rows_adarms<ModT>(p, c, rows, which == 0 ? tag - 1u : tag, ST_QKV + 3 * which,
                                  mods_slot<ModT>(p, c, q));
  MKX_TRACE_AFTER(0, (uint32_t)fail);
  const int slot = which == 0 ? S_QKV : (which == 1 ? S_QCA : S_GU);
  fail |= !wait_bar(p, c, slot);
  if (__syncthreads_or(fail)) return 1;
  MKX_TRACE(2);
  consumed(p, c, BAR_MODS + (q & 1));
  consumed(p, c, slot);
  const int R = which == 0 ? c.R_qkv : (which == 1 ? c.R_h : c.R_gu);
  mma_from_x(p, c, cSlot(p, c, slot), which == 2 ? 2 : 1, R);
  __syncthreads();
  MKX_TRACE(3);
  if (c.tid == ISSUER && gi + 1 < p.n_steps * p.L) issue_slot(p, c, slot, (gi + 1) % p.L);
  if (which == 2) {
    epi_gu(p, c, xb[B_G] + (size_t)par * TP * (p.I >> 1), tag);
  } else if (which == 1) {
    epi_plain(p, c, c.R_h, c.c0, xb[B_QCA] + (size_t)par * TP * HWORDS, HWORDS, tag);
  } else if (!(p.drop_stage == ST_QKV && c.cta == 0 && gi == 0)) {
    epi_plain(p, c, c.R_qkv, c.r0_qkv, xb[B_QKV] + (size_t)par * TP * QKVWORDS, QKVWORDS, tag);
  }
  MKX_TRACE(5);
  return 0;
}

// GEMM stages fed straight from an exchange buffer, with a gated-residual epilogue.
// which = 0: h2 = bf16(h + bf16(y @ Wo^T) * gate_sa); 1: h3 = bf16(h2 + bf16(y_ca @ Woca^T) * gate_ca).
// q: the modulation block holding the gate.
template <typename ModT>
__device__ __forceinline__ int stage_words_gemm(const Params& p, Cta& c, int which, int gi, int q) {
  const int par = gi & 1;
  const uint32_t tag = c.tag0 + (uint32_t)gi;
  u64* const* xb = p.xb;
  const int slot = which == 0 ? S_O : S_OCA;
  const u64* rows = xb[which == 0 ? B_Y : B_YCA] + (size_t)par * TP * HWORDS;
  __syncthreads();
  int fail = !wait_bar(p, c, slot);
  if (__syncthreads_or(fail)) return 1;
  consumed(p, c, slot);
  MKX_TRACE(0);
  fail = mma_from_words(p, c, cSlot(p, c, slot), c.R_h, H, rows, tag, ST_O + 3 * which);
  if (__syncthreads_or(fail)) return 1;
  MKX_TRACE(1);
  if (c.tid == ISSUER && gi + 1 < p.n_steps * p.L) issue_slot(p, c, slot, (gi + 1) % p.L);
  u64* out = xb[which == 0 ? B_H2 : B_H3] + (size_t)par * TP * HWORDS;
  epi_gated<ModT>(p, c, mods_slot<ModT>(p, c, q) + 2 * H, out, tag);
  MKX_TRACE(5);
  __syncthreads();
  MKX_TRACE(6);
  if (c.tid == ISSUER) issue_mods<ModT>(p, c, q + 2);  // this block's last use
  return 0;
}

// Down projection, level 1 (src/mk_expert.py:416-419 with K split over the NGRP groups): this CTA's
// R_dp output columns from d0 over its group's K-slice of g, polled straight from B_G (a warp's
// whole K range in flight at once), up to two m-tiles, K split over the 8 warps. Partials to P as
// [m-tile][warp] blocks. Returns nonzero on a failed wait.
__device__ int down_partial(const Params& p, Cta& c, int par, uint32_t tag) {
  constexpr int CH = 6;
  const int RW = p.I >> 1, KB = (p.I / NGRP) >> 4, R = c.R_dp;
  const int g = c.lane >> 2, cc = c.lane & 3;
  const int kb0 = c.warp * KB / NW, kb1 = (c.warp + 1) * KB / NW;
  const bool v0 = g < p.T, v1 = (8 + g) < p.T, two = p.T > 8, m1 = R > 16;
  const u64* row0 = p.xb[B_G] + (size_t)par * TP * RW + (size_t)g * RW + 2 * cc + (size_t)c.dgrp * KB * 8;
  const size_t d1off = (size_t)8 * RW;  // token row 8 + g
  const char* A = cSlot(p, c, S_D) + cc * 8;
  const bool va0 = g < R, vb0 = g + 8 < R, va1 = g + 16 < R, vb1 = g + 24 < R;
  float d[2][2][4] = {};  // [m-tile][token rows 0-7 / 8-15][fragment]
  Waiter wt(p.status, p.timeout_ns);
  int rc = 0;
  for (int kc = kb0; kc < kb1; kc += CH) {
    u64 w0[2 * CH], w1[2 * CH];
    uint32_t valid = 0;
#pragma unroll
    for (int i = 0; i < CH; ++i)
      if (kc + i < kb1) valid |= ((v0 ? 1u : 0u) | (v1 ? 2u : 0u)) << (2 * i);
    const u64* base = row0 + (size_t)kc * 8;
    auto addr = [base, d1off](int i) { return base + (i >> 1) * 8 + ((i & 1) ? d1off : 0); };
    issue_pairs<2 * CH>(addr, w0, w1, valid, tag);
    const int r = complete_pairs<2 * CH>(addr, w0, w1, tag, wt);
    if (__any_sync(0xffffffffu, r != 0)) {  // keep the warp converged for mma.sync
      rc = r ? r : 2;
      break;
    }
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      if (kc + i < kb1) {
        const char* blk = A + (size_t)(kc + i) * R * 32;
        const uint32_t b0 = payload_of(w0[2 * i]), b1 = payload_of(w1[2 * i]);
        const uint32_t e0 = payload_of(w0[2 * i + 1]), e1 = payload_of(w1[2 * i + 1]);
        {
          const uint2 a = va0 ? lds64(blk + g * 32) : make_uint2(0u, 0u);
          const uint2 b = vb0 ? lds64(blk + (g + 8) * 32) : make_uint2(0u, 0u);
          mma_bf16(d[0][0], a.x, b.x, a.y, b.y, b0, b1);
          if (two) mma_bf16(d[0][1], a.x, b.x, a.y, b.y, e0, e1);
        }
        if (m1) {
          const uint2 a = va1 ? lds64(blk + (g + 16) * 32) : make_uint2(0u, 0u);
          const uint2 b = vb1 ? lds64(blk + (g + 24) * 32) : make_uint2(0u, 0u);
          mma_bf16(d[1][0], a.x, b.x, a.y, b.y, b0, b1);
          if (two) mma_bf16(d[1][1], a.x, b.x, a.y, b.y, e0, e1);
        }
      }
    }
  }
#pragma unroll
  for (int mt = 0; mt < 2; ++mt) {
    float* P = cP(p, c) + (mt * NW + c.warp) * PM;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      P[(8 * h + 2 * cc) * PSTR + g] = d[mt][h][0];
      P[(8 * h + 2 * cc + 1) * PSTR + g] = d[mt][h][1];
      P[(8 * h + 2 * cc) * PSTR + g + 8] = d[mt][h][2];
      P[(8 * h + 2 * cc + 1) * PSTR + g + 8] = d[mt][h][3];
    }
  }
  return fail_code(p, c, rc, ST_DOWN);
}

// Down projection stage: level 1 (partials of the group's K-slice to B_DP), then level 2: the
// NGRP partials of this CTA's columns [c0, c0 + R_h) added in group order, and the gated residual
// h = bf16(h3 + bf16(g @ Wd^T) * gate_mlp) to B_HOUT. q: the MLP modulation block.
template <typename ModT>
__device__ __forceinline__ int stage_down(const Params& p, Cta& c, int gi, int q) {
  const int par = gi & 1;
  const uint32_t tag = c.tag0 + (uint32_t)gi;
  __syncthreads();
  int fail = !wait_bar(p, c, S_D);
  if (__syncthreads_or(fail)) return 1;
  consumed(p, c, S_D);
  MKX_TRACE(0);
  fail = down_partial(p, c, par, tag);
  if (__syncthreads_or(fail)) return 1;
  MKX_TRACE(1);
  if (c.tid == ISSUER && gi + 1 < p.n_steps * p.L) issue_slot(p, c, S_D, (gi + 1) % p.L);
  {  // partial sums (token n, column r): columns fastest, consecutive lanes store consecutive words
    u64* dp = p.xb[B_DP] + (size_t)par * TP * DPWORDS + (size_t)c.dgrp * H + c.d0;
    for (int e = c.tid; e < p.T * c.R_dp; e += NT) {
      const int n = e / c.R_dp, r = e - n * c.R_dp;
      const float* P = cP(p, c) + (r >> 4) * NW * PM + n * PSTR + (r & 15);
      float v[NW];
#pragma unroll
      for (int k = 0; k < NW; ++k) v[k] = P[k * PM];
#pragma unroll
      for (int w = NW / 2; w >= 1; w >>= 1)
#pragma unroll
        for (int k = 0; k < w; ++k) v[k] += v[k + w];
      st_volatile(dp + (size_t)n * DPWORDS + r, make_word(tag, __float_as_uint(v[0])));
    }
  }
  MKX_TRACE(2);
  __syncthreads();  // P is reused below
  float* S = cP(p, c);  // [NGRP][TP][RESW] partials of this CTA's columns
  {
    const u64* src = p.xb[B_DP] + (size_t)par * TP * DPWORDS + c.c0;
    const int per = p.T * c.R_h;
    Waiter wt(p.status, p.timeout_ns);
    int r = 0;
    for (int e = c.tid; e < NGRP * per && r == 0; e += NT) {
      const int j = e / per, rem = e - j * per, n = rem / c.R_h, col = rem - n * c.R_h;
      u64 w = 0;
      r = poll_word(src + (size_t)n * DPWORDS + (size_t)j * H + col, w, tag, wt);
      S[(j * TP + n) * RESW + col] = __uint_as_float(payload_of(w));
    }
    fail = fail_code(p, c, r, ST_DOWN);
  }
  if (__syncthreads_or(fail)) return 1;
  MKX_TRACE(3);
  {
    const int npairs = c.R_h >> 1, pp = c.tid % npairs, n = c.tid / npairs;
    if (c.tid < npairs * p.T) {
      float2 v = make_float2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < NGRP; ++j) {
        const float2 t = *reinterpret_cast<const float2*>(S + (j * TP + n) * RESW + 2 * pp);
        v.x += t.x;
        v.y += t.y;
      }
      gated_pair_store<ModT>(p, c, mods_slot<ModT>(p, c, q) + 2 * H, p.xb[B_HOUT] + (size_t)par * TP * HWORDS, tag,
                             p.trace_h ? p.trace_h + (size_t)gi * p.T * H : nullptr, pp, n, v);
    }
  }
  MKX_TRACE(5);
  __syncthreads();
  MKX_TRACE(6);
  if (c.tid == ISSUER) issue_mods<ModT>(p, c, q + 2);  // this block's last use
  return 0;
}

// Self-attention (sa) or cross-attention, one (head, row) unit per CTA; one routine for both.
// Streamed inputs: before the first Euler step's self-attention of layer l reads any K/V, thread 0
// waits (bounded) until kv_ready[l] holds this launch's value. The copies of layer l's memory and
// cross-attention K/V precede that word in their stream, so both attention stages of the layer see
// them; later Euler steps find them in place.
__device__ __forceinline__ int wait_kv_ready(const Params& p, Cta& c, int l) {
  int r = 0;
  if (c.tid == 0) {
    Waiter wt(p.status, p.timeout_ns);
    while (r == 0 && ld_acquire_i32(p.kv_ready + l) != p.kv_ready_value) r = wt.tick();
    r = fail_code(p, c, r, ST_SA);
  }
  return __syncthreads_or(r);
}

__device__ __forceinline__ int stage_attention(const Params& p, Cta& c, const bool sa, int gi, int l) {
  if (sa && p.kv_ready != nullptr && gi < p.L && c.cta < NH * p.T && wait_kv_ready(p, c, l)) return 1;
  const int par = gi & 1;
  const uint32_t tag = c.tag0 + (uint32_t)gi;
  const u64* src = sa ? p.xb[B_QKV] + (size_t)par * TP * QKVWORDS : p.xb[B_QCA] + (size_t)par * TP * HWORDS;
  u64* y = p.xb[sa ? B_Y : B_YCA] + (size_t)par * TP * HWORDS;
  for (int u = c.cta; u < NH * p.T; u += c.G) {
    const int fail = attention_unit(p, c, sa, l, u % NH, u / NH, src, y, tag);
    if (__syncthreads_or(fail)) return 1;
  }
  return 0;
}

// Exchange words this launch will not rewrite, set to tag 0 (never a valid tag: instance + 1 is
// in 1..4095). A tag repeats after 2^20 launches (the sequence number has 20 bits left above the
// instance); a word last written that long ago -- a row >= T of a launch with more action rows, an
// action-state word >= action_dim, a parity that a short launch never uses -- would otherwise pass
// for fresh in a later launch whose geometry reads it. Each CTA clears only words it alone produces
// (the same ownership as its epilogues) and that no stage of this launch writes or reads, so the
// stores race with nothing; they run at the launch's exit (also after a failed wait), and the next
// launch on the stream sees them. After every launch each word holds 0 or a tag of that launch or
// of an earlier one that a later launch has not overwritten.
__device__ void clear_stale_words(const Params& p, const Cta& c) {
  const bool par1 = p.n_steps * p.L >= 2;  // parity 1 is used by instances 1, 3, ...
  int xpar = 0;                             // bit mask: parities of the action-state words of steps 0..n-2
  for (int s = 0; s + 1 < p.n_steps && s < 2; ++s) xpar |= 1 << ((s * p.L + p.L - 1) & 1);
  auto clear_owned = [&](int b, int w0, int nw, int rw, bool perm) {  // nw <= NT words per row
    if (c.tid >= nw) return;
    const int pos = perm ? word_pos(w0 + c.tid) : w0 + c.tid;
#pragma unroll 1
    for (int par = 0; par < 2; ++par) {
      u64* col = p.xb[b] + (size_t)par * TP * rw + pos;
#pragma unroll 1
      for (int n = (par == 0 || par1) ? p.T : 0; n < TP; ++n) st_volatile(col + (size_t)n * rw, 0ull);
    }
  };
  clear_owned(B_QKV, c.r0_qkv >> 1, c.R_qkv >> 1, QKVWORDS, true);
  clear_owned(B_H2, c.c0 >> 1, c.R_h >> 1, HWORDS, true);
  clear_owned(B_QCA, c.c0 >> 1, c.R_h >> 1, HWORDS, true);
  clear_owned(B_H3, c.c0 >> 1, c.R_h >> 1, HWORDS, true);
  clear_owned(B_HOUT, c.c0 >> 1, c.R_h >> 1, HWORDS, true);
  clear_owned(B_G, c.u0 >> 1, c.R_gu >> 1, p.I >> 1, true);
  clear_owned(B_DP, c.dgrp * H + c.d0, c.R_dp, DPWORDS, false);
  // attention outputs: unit u = (head u % NH, row u / NH), produced by CTA u % G
  for (int u = c.cta; u < NH * TP; u += c.G) {
    const int n = u / NH, h = u % NH;
    for (int par = 0; par < 2; ++par) {
      if (n < p.T && (par == 0 || par1)) continue;
      if (c.tid < 64)
        st_volatile(p.xb[c.tid < 32 ? B_Y : B_YCA] + (size_t)par * TP * HWORDS + (size_t)n * HWORDS + h * 32 + (c.tid & 31),
                    0ull);
    }
  }
  // action state: row n produced by CTA n (words a < action_dim, intermediate steps only)
  if (c.cta < TP && c.tid < 2 * XWORDS) {
    const int n = c.cta, par = c.tid / XWORDS, a = c.tid % XWORDS;
    if (!(((xpar >> par) & 1) && n < p.T && a < p.adim)) st_volatile(p.xb[B_X] + (size_t)par * TP * XWORDS + (size_t)n * XWORDS + a, 0ull);
  }
}

// Euler step tail of step s: velocity rows (CTAs n < T), action-state exchange, and every CTA's
// in-projection of the next step's h0 into X.
template <typename ModT>
__device__ __forceinline__ int stage_tail(const Params& p, Cta& c, int s) {
  const int L = p.L;
  const int gl = s * L + L - 1;
  const int q_fin = s * (3 * L + 1) + 3 * L;
  const bool last = s + 1 == p.n_steps;
  const uint32_t tl = c.tag0 + (uint32_t)gl;
  u64* xrows = p.xb[B_X] + (size_t)(gl & 1) * TP * XWORDS;
  int fail = !wait_bar(p, c, BAR_MODS + (q_fin & 1));
  if (__syncthreads_or(fail)) return 1;
  consumed(p, c, BAR_MODS + (q_fin & 1));
  if (c.cta < p.T) {
    fail = velocity_row<ModT>(p, c, c.cta, last, mods_slot<ModT>(p, c, q_fin),
                              p.xb[B_HOUT] + (size_t)(gl & 1) * TP * HWORDS, tl, xrows, tl) != 0;
    if (__syncthreads_or(fail)) return 1;
  }
  __syncthreads();
  if (c.tid == ISSUER) issue_mods<ModT>(p, c, q_fin + 2);
  if (!last) {
    float win[NCOL][AO], bin[NCOL];
    load_inproj(p, c, win, bin);  // in flight while the new action state is polled
    if (take_new_x(p, c, xrows, tl)) return 1;
    in_proj_to_x(p, c, win, bin);
    __syncthreads();
  }
  return 0;
}

template <typename ModT>
__global__ void __launch_bounds__(NT, 1) expert_kernel(const __grid_constant__ Params p) {
  Cta c;
  c.tid = threadIdx.x;
  c.warp = c.tid >> 5;
  c.lane = c.tid & 31;
  c.cta = blockIdx.x;
  c.G = gridDim.x;
  c.stages = 0;
  {
    const int G = c.G, i = c.cta;
    int lo = part_lo(i, 3 * H / 2, G), hi = part_lo(i + 1, 3 * H / 2, G);
    c.r0_qkv = 2 * lo; c.R_qkv = 2 * (hi - lo);
    lo = part_lo(i, H / 2, G); hi = part_lo(i + 1, H / 2, G);
    c.c0 = 2 * lo; c.R_h = 2 * (hi - lo);
    lo = part_lo(i, p.I / 2, G); hi = part_lo(i + 1, p.I / 2, G);
    c.u0 = 2 * lo; c.R_gu = 2 * (hi - lo);
    int j = 0;
    while (j + 1 < NGRP && i >= part_lo(j + 1, G, NGRP)) ++j;
    const int g0 = part_lo(j, G, NGRP), gn = part_lo(j + 1, G, NGRP) - g0;
    lo = part_lo(i - g0, H / 2, gn); hi = part_lo(i - g0 + 1, H / 2, gn);
    c.dgrp = j; c.d0 = 2 * lo; c.R_dp = 2 * (hi - lo);
  }
  if (p.prof != nullptr && c.tid == 0) p.prof[(size_t)c.cta * (2 + p.n_steps * (8 * p.L + 1))] = globaltimer();
  const uint32_t seq = (uint32_t)ld_volatile_i32(p.status + 1);
  c.tag0 = seq * (uint32_t)MAX_STEP_TAGS + 1u;
  const int L = p.L;
  const int per = 3 * L + 1;  // modulation blocks per Euler step

  if (c.tid == 0) {
    for (int b = 0; b < NBAR; ++b) {
      mbar_init(&cBar(p, c)[b], 1);
      cCnt(p, c)[b] = 0;
      cCnt(p, c)[NBAR + b] = 0;
    }
    fence_mbar_init();
  }
  if (c.tid < TP * 32) cXs(p, c)[c.tid] = 0.f;
  __syncthreads();
  if (c.tid == ISSUER) {
    for (int s = 0; s < NSLOT; ++s) issue_slot(p, c, s, 0);
    issue_mods<ModT>(p, c, 0);
    issue_mods<ModT>(p, c, 1);
  }
  {
    // FIRST tail: h0 from the action state after step 1, into X.
    float win[NCOL][AO], bin[NCOL];
    load_inproj(p, c, win, bin);
    for (int e = c.tid; e < p.T * p.A; e += NT) cXs(p, c)[(e / p.A) * 32 + (e % p.A)] = __ldg(p.x_in + e);
    __syncthreads();
    in_proj_to_x(p, c, win, bin);
    __syncthreads();
  }
  stage_done(p, c);

  // Stage sequence of one layer (src/mk_expert.py:342-421): 0 QKV, 1 SA, 2 SA out, 3 CA query,
  // 4 CA, 5 CA out, 6 gate/up, 7 down; then, after the last layer, the step tail (8).
  for (int s = 0; s < p.n_steps; ++s) {
    for (int l = 0; l < L; ++l) {
      const int gi = s * L + l;
      const int q_sa = s * per + 3 * l;
      for (int st = 0; st < 9; ++st) {
        int rc = 0;
        if (st == 8) {
          if (l + 1 < L) break;
          rc = stage_tail<ModT>(p, c, s);
        } else if (st == 0 || st == 3 || st == 6) {
          rc = stage_norm_gemm<ModT>(p, c, st / 3, gi, l, q_sa + st / 3);
        } else if (st == 1 || st == 4) {
          rc = stage_attention(p, c, st == 1, gi, l);
        } else if (st == 7) {
          rc = stage_down<ModT>(p, c, gi, q_sa + 2);
        } else {  // st 2, 5
          const int which = st == 2 ? 0 : 1;
          rc = stage_words_gemm<ModT>(p, c, which, gi, q_sa + which);
        }
        if (rc) goto drain;
        stage_done(p, c);
      }
    }
  }

drain:
  clear_stale_words(p, c);
  // Normal exit: nothing is in flight. After a failed wait: drain every issued bulk copy (bounded).
  __syncthreads();
  if (c.tid == 0) {
    int* cnt = cCnt(p, c);
    for (int b = 0; b < NBAR; ++b) {
      while (cnt[NBAR + b] < cnt[b]) {
        const uint32_t parity = (uint32_t)(cnt[NBAR + b] & 1);
        const uint64_t t0 = globaltimer();
        bool ok = false;
        while (!(ok = mbar_try_wait(&cBar(p, c)[b], parity))) {
          if (globaltimer() - t0 > p.timeout_ns) break;
        }
        cnt[NBAR + b] += 1;
        if (!ok) break;
      }
    }
    atomicAdd(reinterpret_cast<unsigned long long*>(p.status + 2), (unsigned long long)c.stages);
    if (c.cta == 0) {  // also after a failure: the next launch must not match this one's tags
      __threadfence();
      atomicExch(p.status + 1, (int)(seq + 1u));
    }
  }
}

// ---------------------------------------------------------------------------------------------
// Packing: rows of a row-major [L][N][K] bf16 weight, split in column pairs over G CTAs, each
// CTA's rows stored as [K/16][R][16] with the 16 k of a block permuted so that lane (g, c) of an
// mma.sync A fragment reads {a0, a2} (or {a1, a3}) as one 8-byte word.
__host__ __device__ __forceinline__ int perm16(int kk) { return ((kk & 7) >> 1) * 4 + (kk >> 3) * 2 + (kk & 1); }

__device__ __forceinline__ int owner_of_pair(int pp, int P, int G) {
  int i = (int)((((long long)pp + 1) * G - 1) / P);
  if (i >= G) i = G - 1;
  while (i > 0 && part_lo(i, P, G) > pp) --i;
  while (i + 1 < G && part_lo(i + 1, P, G) <= pp) ++i;
  return i;
}

// nmat = 1: dst[l] region of N*K; nmat = 2 (gate/up): dst[l] region of 2*N*K, each CTA's gate chunk
// then its up chunk.
__global__ void pack_kernel(const uint16_t* __restrict__ src0, const uint16_t* __restrict__ src1, uint16_t* dst,
                            int L, int N, int K, int G, int nmat) {
  const long long total = (long long)L * nmat * N * K;
  const int P = N / 2;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
    const int k = (int)(e % K);
    long long rest = e / K;
    const int n = (int)(rest % N);
    rest /= N;
    const int mat = (int)(rest % nmat);
    const int l = (int)(rest / nmat);
    const int i = owner_of_pair(n >> 1, P, G);
    const int r0 = 2 * part_lo(i, P, G);
    const int R = 2 * part_lo(i + 1, P, G) - r0;
    const uint16_t* src = mat ? src1 : src0;
    const long long so = ((long long)l * N + n) * K + k;
    const long long base = (long long)l * nmat * N * K + (long long)nmat * r0 * K + (long long)mat * R * K;
    const long long d = base + (long long)(k >> 4) * R * 16 + (long long)(n - r0) * 16 + perm16(k & 15);
    dst[d] = src[so];
  }
}

// Packs Wd [L, H, I] for the two-level down projection: layer block l, then group j's block of
// all H rows over K-slice j (I / NGRP columns), inside which CTA t of the group (Gj CTAs) stores its
// R output rows from r0 (pairs split like every other matrix, over Gj) as [KS / 16][R][16] with the
// A-fragment order of each 16-column block.
__global__ void pack_down_kernel(const uint16_t* __restrict__ src, uint16_t* dst, int L, int I, int G) {
  const long long total = (long long)L * H * I;
  const int KS = I / NGRP;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
    const int k = (int)(e % I);
    const long long rest = e / I;
    const int n = (int)(rest % H);
    const int l = (int)(rest / H);
    const int j = k / KS, kl = k - j * KS;
    const int gn = part_lo(j + 1, G, NGRP) - part_lo(j, G, NGRP);
    const int t = owner_of_pair(n >> 1, H / 2, gn);
    const int r0 = 2 * part_lo(t, H / 2, gn);
    const int R = 2 * part_lo(t + 1, H / 2, gn) - r0;
    const long long d = (long long)l * H * I + (long long)j * H * KS + (long long)r0 * KS + (long long)(kl >> 4) * R * 16 +
                        (long long)(n - r0) * 16 + perm16(kl & 15);
    dst[d] = src[e];
  }
}

__global__ void norm_kernel(const uint16_t* qn, const uint16_t* kn, const uint16_t* qcan, float* out, int L) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= 3 * L * HD) return;
  const int which = e / (L * HD), r = e % (L * HD);
  const uint16_t* s = which == 0 ? qn : (which == 1 ? kn : qcan);
  out[e] = 1.0f + __uint_as_float(((uint32_t)s[r]) << 16);
}

}  // namespace mkx

// =============================================================================================
// Host side: the C ABI.
using namespace mkx;

struct mkx_handle {
  mkx_dims dims;
  int device;
  int G;
  int smem;
  Params base;     // weight / scratch pointers and smem layout; per-call fields filled in mkx_run
  void* alloc[24];
  int nalloc;
  unsigned long long timeout_ns;
  int drop_stage;
};

static thread_local char g_cuda_err[256] = "";

static mkx_status cuda_fail(cudaError_t e, const char* what) {
  snprintf(g_cuda_err, sizeof(g_cuda_err), "%s: %s", what, cudaGetErrorString(e));
  return MKX_ERR_CUDA;
}
#define MKX_CUDA(call)                                 \
  do {                                                 \
    cudaError_t e_ = (call);                           \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
  } while (0)

extern "C" const char* mkx_last_cuda_error(void) { return g_cuda_err; }

extern "C" mkx_status mkx_h2d_copies(int n, void* const* dst, const void* const* src, const size_t* bytes,
                                     cudaStream_t stream) {
  if (n < 0 || (n > 0 && (!dst || !src || !bytes))) return MKX_ERR_INVALID_ARG;
  for (int i = 0; i < n; ++i) {
    if (!dst[i] || !src[i]) return MKX_ERR_INVALID_ARG;
    MKX_CUDA(cudaMemcpyAsync(dst[i], src[i], bytes[i], cudaMemcpyHostToDevice, stream));
  }
  return MKX_OK;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

static void* halloc(mkx_handle* h, size_t bytes, cudaError_t* err) {
  void* p = nullptr;
  *err = cudaMalloc(&p, bytes);
  if (*err == cudaSuccess) h->alloc[h->nalloc++] = p;
  return p;
}

struct Layout {
  int s_slot[NSLOT];
  int s_x, s_p, s_mods, s_xs, s_res, s_red, s_bar, s_cnt, total;
  int max_rows_qkv, max_rows_h, max_rows_gu, max_rows_dp;
};

static int max_part(int P, int G) {
  int m = 0;
  for (int i = 0; i < G; ++i) {
    const int r = part_lo(i + 1, P, G) - part_lo(i, P, G);
    if (r > m) m = r;
  }
  return m;
}
static int min_part(int P, int G) {
  int m = 1 << 30;
  for (int i = 0; i < G; ++i) {
    const int r = part_lo(i + 1, P, G) - part_lo(i, P, G);
    if (r < m) m = r;
  }
  return m;
}

static Layout make_layout(int I, int G) {
  Layout ly;
  ly.max_rows_qkv = 2 * max_part(3 * H / 2, G);
  ly.max_rows_h = 2 * max_part(H / 2, G);
  ly.max_rows_gu = 2 * max_part(I / 2, G);
  ly.max_rows_dp = 0;
  for (int j = 0; j < NGRP; ++j) {
    const int r = 2 * max_part(H / 2, part_lo(j + 1, G, NGRP) - part_lo(j, G, NGRP));
    if (r > ly.max_rows_dp) ly.max_rows_dp = r;
  }
  int off = 0;
  auto take = [&](int bytes) {
    const int o = off;
    off += (bytes + 127) & ~127;
    return o;
  };
  ly.s_slot[S_QKV] = take(ly.max_rows_qkv * H * 2);
  ly.s_slot[S_O] = take(ly.max_rows_h * H * 2);
  ly.s_slot[S_QCA] = take(ly.max_rows_h * H * 2);
  ly.s_slot[S_OCA] = take(ly.max_rows_h * H * 2);
  ly.s_slot[S_GU] = take(ly.max_rows_gu * H * 4);
  ly.s_slot[S_D] = take(ly.max_rows_dp * (I / NGRP) * 2);
  ly.s_x = take(TP * XS * 2);
  constexpr int attn_floats = NW * 64 + NW;  // attention output reduction: per-warp o and den
  ly.s_p = take((attn_floats > 2 * NW * PM ? attn_floats : 2 * NW * PM) * 4);  // down: two m-tiles of partials
  ly.s_mods = take(2 * 3 * H * 4);  // sized for fp32 modulations
  ly.s_xs = take(TP * 32 * 4);
  ly.s_res = take(TP * RESW * 4);
  ly.s_red = take((16 + NW * AO) * 4);
  ly.s_bar = take(NBAR * 8);
  ly.s_cnt = take(2 * NBAR * 4);
  ly.total = off;
  return ly;
}

template <typename ModT>
static cudaError_t set_smem_attr(int bytes) {
  return cudaFuncSetAttribute(expert_kernel<ModT>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

extern "C" mkx_status mkx_create(const mkx_dims* dims, const mkx_weights* w, int device, mkx_handle** out) {
  if (!dims || !w || !out) return MKX_ERR_INVALID_ARG;
  *out = nullptr;
  const mkx_dims d = *dims;
  if (d.H != H || d.NH != NH || d.HD != HD) return MKX_ERR_UNSUPPORTED;
  if (d.L < 1 || d.L > MKX_MAX_LAYERS || d.I < 128 || d.I % 128 != 0 || d.A < AO || d.A > 32) return MKX_ERR_UNSUPPORTED;
  if (d.max_rows < 1 || d.max_rows > TP) return MKX_ERR_UNSUPPORTED;
  const void* ptrs[] = {w->wqkv, w->wo, w->wqca, w->woca, w->wg, w->wu, w->wd, w->qn, w->kn, w->qcan,
                        w->win, w->bin, w->wout, w->bout};
  for (const void* q : ptrs)
    if (!q) return MKX_ERR_INVALID_ARG;
  DeviceScope dev_scope(device);
  MKX_CUDA(dev_scope.err);
  int sms = 0, smem_optin = 0;
  MKX_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  MKX_CUDA(cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  const int G = d.grid > 0 ? d.grid : sms;
  if (G < d.A || G < TP || G > H / 2 || G > sms) return MKX_ERR_RESOURCES;
  if (min_part(d.I / 2, G) < 1) return MKX_ERR_RESOURCES;
  const Layout ly = make_layout(d.I, G);
  // one epilogue element (column pair, action row) per thread; this also keeps every matrix at <= 32
  // rows per CTA, the bound gemm_split assumes
  // and the down partials at <= two m-tiles per CTA
  if (ly.max_rows_qkv / 2 * TP > NT || ly.max_rows_h > RESW || ly.max_rows_gu / 2 * TP > NT || ly.max_rows_dp > 32)
    return MKX_ERR_RESOURCES;
  if (ly.total > smem_optin) return MKX_ERR_RESOURCES;

  mkx_handle* h = new (std::nothrow) mkx_handle();
  if (!h) return MKX_ERR_RESOURCES;
  memset(h, 0, sizeof(*h));
  h->dims = d;
  h->device = device;
  h->G = G;
  h->smem = ly.total;
  h->timeout_ns = 2000000000ull;
  const int L = d.L, I = d.I, A = d.A;
  const size_t HH = (size_t)H * H;
  cudaError_t err = cudaSuccess;
  uint16_t* wp[NSLOT];
  const size_t welems[NSLOT] = {(size_t)L * 3 * HH, (size_t)L * HH, (size_t)L * HH, (size_t)L * HH,
                                (size_t)L * 2 * I * H, (size_t)L * H * I};
  for (int s = 0; s < NSLOT; ++s) {
    wp[s] = (uint16_t*)halloc(h, welems[s] * 2, &err);
    if (err != cudaSuccess) { mkx_destroy(h); return cuda_fail(err, "cudaMalloc(weights)"); }
  }
  float* nrm = (float*)halloc(h, (size_t)3 * L * HD * 4, &err);
  float* tailw = err == cudaSuccess ? (float*)halloc(h, TAIL_FLOATS * 4, &err) : nullptr;
  float* wout = err == cudaSuccess ? (float*)halloc(h, (size_t)A * H * 4, &err) : nullptr;
  const int rw[NBUF] = {QKVWORDS, HWORDS, HWORDS, HWORDS, HWORDS, HWORDS, I / 2, HWORDS, XWORDS, DPWORDS};
  size_t xwords = 0;
  for (int b = 0; b < NBUF; ++b) xwords += (size_t)2 * TP * rw[b];
  u64* xbase = err == cudaSuccess ? (u64*)halloc(h, xwords * 8, &err) : nullptr;
  int* status = err == cudaSuccess ? (int*)halloc(h, 64, &err) : nullptr;
  if (err != cudaSuccess) { mkx_destroy(h); return cuda_fail(err, "cudaMalloc(scratch)"); }

  cudaStream_t st;
  if ((err = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking)) != cudaSuccess) { mkx_destroy(h); return cuda_fail(err, "stream"); }
  const int blocks = sms * 8;
  pack_kernel<<<blocks, 256, 0, st>>>(w->wqkv, nullptr, wp[S_QKV], L, 3 * H, H, G, 1);
  pack_kernel<<<blocks, 256, 0, st>>>(w->wo, nullptr, wp[S_O], L, H, H, G, 1);
  pack_kernel<<<blocks, 256, 0, st>>>(w->wqca, nullptr, wp[S_QCA], L, H, H, G, 1);
  pack_kernel<<<blocks, 256, 0, st>>>(w->woca, nullptr, wp[S_OCA], L, H, H, G, 1);
  pack_kernel<<<blocks, 256, 0, st>>>(w->wg, w->wu, wp[S_GU], L, I, H, G, 2);
  pack_down_kernel<<<blocks, 256, 0, st>>>(w->wd, wp[S_D], L, I, G);
  norm_kernel<<<(3 * L * HD + 255) / 256, 256, 0, st>>>(w->qn, w->kn, w->qcan, nrm, L);
  // tail weights: win rows 0..7 | bin | bout (padded to 32); wout keeps all A rows
  cudaMemsetAsync(tailw, 0, TAIL_FLOATS * 4, st);
  cudaMemcpyAsync(tailw, w->win, (size_t)AO * H * 4, cudaMemcpyDeviceToDevice, st);
  cudaMemcpyAsync(tailw + AO * H, w->bin, (size_t)H * 4, cudaMemcpyDeviceToDevice, st);
  cudaMemcpyAsync(tailw + AO * H + H, w->bout, (size_t)A * 4, cudaMemcpyDeviceToDevice, st);
  cudaMemcpyAsync(wout, w->wout, (size_t)A * H * 4, cudaMemcpyDeviceToDevice, st);
  cudaMemsetAsync(xbase, 0, xwords * 8, st);
  cudaMemsetAsync(status, 0, 64, st);
  const int one = 1;
  cudaMemcpyAsync(status + 1, &one, 4, cudaMemcpyHostToDevice, st);
  err = cudaStreamSynchronize(st);
  cudaError_t e2 = cudaGetLastError();
  cudaStreamDestroy(st);
  if (err != cudaSuccess || e2 != cudaSuccess) {
    mkx_destroy(h);
    return cuda_fail(err != cudaSuccess ? err : e2, "pack");
  }
  // The attribute belongs to the kernel function, shared by every handle in the process: always
  // allow the device maximum so a smaller handle never lowers what a larger one needs.
  if ((err = set_smem_attr<uint16_t>(smem_optin)) != cudaSuccess || (err = set_smem_attr<float>(smem_optin)) != cudaSuccess) {
    mkx_destroy(h);
    return cuda_fail(err, "cudaFuncSetAttribute");
  }
  int occ = 0;
  if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, expert_kernel<uint16_t>, NT, ly.total)) != cudaSuccess || occ < 1) {
    mkx_destroy(h);
    return err != cudaSuccess ? cuda_fail(err, "occupancy") : MKX_ERR_RESOURCES;
  }

  Params& p = h->base;
  for (int s = 0; s < NSLOT; ++s) p.w[s] = wp[s];
  p.nrm = nrm;
  p.tailw = tailw;
  p.wout = wout;
  u64* xp = xbase;
  for (int b = 0; b < NBUF; ++b) {
    p.xb[b] = xp;
    xp += (size_t)2 * TP * rw[b];
  }
  p.status = status;
  p.L = L;
  p.I = I;
  p.A = A;
  p.eps = d.eps;
  p.qk_eps = d.qk_eps;
  p.sm_scale = 1.0f / sqrtf((float)HD);
  for (int s = 0; s < NSLOT; ++s) p.s_slot[s] = ly.s_slot[s];
  p.s_x = ly.s_x; p.s_p = ly.s_p; p.s_mods = ly.s_mods; p.s_xs = ly.s_xs; p.s_res = ly.s_res;
  p.s_red = ly.s_red; p.s_bar = ly.s_bar; p.s_cnt = ly.s_cnt;
  *out = h;
  return MKX_OK;
}

extern "C" mkx_status mkx_run(mkx_handle* h, const mkx_step_inputs* in, cudaStream_t stream) {
  if (!h || !in) return MKX_ERR_INVALID_ARG;
  const mkx_dims& d = h->dims;
  if (in->T < 1 || in->T > d.max_rows || in->n_steps < 1 || in->n_steps * d.L >= MAX_STEP_TAGS - 1)
    return MKX_ERR_INVALID_ARG;
  if (in->action_dim < 1 || in->action_dim > AO) return MKX_ERR_INVALID_ARG;
  if (!in->x_in || !in->x_out || !in->mods || !in->dt || !in->cu_kv || !in->cu_src || !in->sa_cos || !in->sa_sin ||
      !in->ca_cos || !in->ca_sin)
    return MKX_ERR_INVALID_ARG;
  if (in->kv_ready && (reinterpret_cast<uintptr_t>(in->kv_ready) & 3u)) return MKX_ERR_INVALID_ARG;
  if (in->mem_rows < 1 || in->mem_rows > MAX_MEM_ROWS || in->ca_rows < 1) return MKX_ERR_UNSUPPORTED;
  if (in->mem_row_stride < H || in->mem_row_stride % 8 || in->ca_row_stride < H || in->ca_row_stride % 8)
    return MKX_ERR_INVALID_ARG;
  if (!aligned16(in->sa_cos) || !aligned16(in->sa_sin) || !aligned16(in->ca_cos) || !aligned16(in->ca_sin) ||
      !aligned16(in->mods))
    return MKX_ERR_INVALID_ARG;
  for (int l = 0; l < d.L; ++l) {
    if (!in->memk[l] || !in->memv[l] || !in->kca[l] || !in->vca[l]) return MKX_ERR_INVALID_ARG;
    if (((uintptr_t)in->memk[l] | (uintptr_t)in->memv[l] | (uintptr_t)in->kca[l] | (uintptr_t)in->vca[l]) & 7u)
      return MKX_ERR_INVALID_ARG;
  }
  Params p = h->base;
  p.x_in = in->x_in;
  p.x_out = in->x_out;
  p.mods = in->mods;
  p.dt = in->dt;
  for (int l = 0; l < MKX_MAX_LAYERS; ++l) {
    p.memk[l] = l < d.L ? in->memk[l] : nullptr;
    p.memv[l] = l < d.L ? in->memv[l] : nullptr;
    p.kca[l] = l < d.L ? in->kca[l] : nullptr;
    p.vca[l] = l < d.L ? in->vca[l] : nullptr;
  }
  p.mem_rows = in->mem_rows;
  p.mem_row_stride = in->mem_row_stride;
  p.ca_row_stride = in->ca_row_stride;
  p.ca_rows = in->ca_rows;
  p.cu_kv = in->cu_kv;
  p.cu_src = in->cu_src;
  p.sa_cos = in->sa_cos;
  p.sa_sin = in->sa_sin;
  p.ca_cos = in->ca_cos;
  p.ca_sin = in->ca_sin;
  p.trace_h = in->trace_h;
  p.prof = in->prof;
  p.kv_ready = in->kv_ready;
  p.kv_ready_value = in->kv_ready_value;
  p.timeout_ns = h->timeout_ns;
  p.drop_stage = h->drop_stage;
  p.T = in->T;
  p.adim = in->action_dim;
  p.n_steps = in->n_steps;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(h->G);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = h->smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = in->mods_fp32 ? cudaLaunchKernelEx(&cfg, expert_kernel<float>, p)
                                : cudaLaunchKernelEx(&cfg, expert_kernel<uint16_t>, p);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(expert_kernel)");
  return MKX_OK;
}

extern "C" int mkx_sync_points(const mkx_handle* h, int n_steps) {
  if (!h) return -1;
  return 1 + n_steps * (8 * h->dims.L + 1);
}

extern "C" mkx_status mkx_last_error(mkx_handle* h, int* code, long long* stages) {
  if (!h) return MKX_ERR_INVALID_ARG;
  int st[4] = {0, 0, 0, 0};
  DeviceScope dev_scope(h->device);
  MKX_CUDA(dev_scope.err);
  MKX_CUDA(cudaMemcpy(st, h->base.status, sizeof(st), cudaMemcpyDeviceToHost));
  if (code) *code = st[0];
  if (stages) {
    unsigned long long v;
    memcpy(&v, st + 2, 8);
    *stages = (long long)v;
  }
  return st[0] ? MKX_ERR_DEVICE : MKX_OK;
}

extern "C" mkx_status mkx_clear_error(mkx_handle* h) {
  if (!h) return MKX_ERR_INVALID_ARG;
  DeviceScope dev_scope(h->device);
  MKX_CUDA(dev_scope.err);
  int st[4] = {0, 0, 0, 0};
  MKX_CUDA(cudaMemcpy(st, h->base.status, sizeof(st), cudaMemcpyDeviceToHost));
  st[0] = 0;
  st[1] += 1;  // a new tag generation: words a failed launch left behind can never match
  st[2] = st[3] = 0;
  MKX_CUDA(cudaMemcpy(h->base.status, st, sizeof(st), cudaMemcpyHostToDevice));
  return MKX_OK;
}

extern "C" mkx_status mkx_set_timeout_ns(mkx_handle* h, unsigned long long ns) {
  if (!h || ns == 0) return MKX_ERR_INVALID_ARG;
  h->timeout_ns = ns;
  return MKX_OK;
}

extern "C" mkx_status mkx_set_fault_injection(mkx_handle* h, int stage) {
  if (!h || (stage != 0 && stage != ST_QKV)) return MKX_ERR_INVALID_ARG;
  h->drop_stage = stage;
  return MKX_OK;
}

extern "C" mkx_status mkx_set_launch_sequence(mkx_handle* h, unsigned int seq) {
  if (!h) return MKX_ERR_INVALID_ARG;
  DeviceScope dev_scope(h->device);
  MKX_CUDA(dev_scope.err);
  MKX_CUDA(cudaMemcpy(h->base.status + 1, &seq, sizeof(seq), cudaMemcpyHostToDevice));
  return MKX_OK;
}

extern "C" mkx_status mkx_launch_shape(const mkx_handle* h, int* grid, int* smem_bytes) {
  if (!h) return MKX_ERR_INVALID_ARG;
  if (grid) *grid = h->G;
  if (smem_bytes) *smem_bytes = h->smem;
  return MKX_OK;
}

extern "C" void mkx_destroy(mkx_handle* h) {
  if (!h) return;
  DeviceScope dev_scope(h->device);
  for (int i = 0; i < h->nalloc; ++i) cudaFree(h->alloc[i]);
  delete h;
}

// =============================================================================================
// mkx_run_static: the same kernel for callers that cannot allocate. Its scratch lives in a
// file-scope device array instead of handle memory; nothing below allocates.
#include <mutex>

namespace mkx {
constexpr int STATIC_MAX_I = 3072;
// exchange words of every buffer, both parities, TP rows, at the largest I; then 8 status ints
constexpr size_t STATIC_XWORDS = (size_t)2 * TP * (QKVWORDS + 6 * HWORDS + STATIC_MAX_I / 2 + XWORDS + DPWORDS);
constexpr size_t STATIC_WORDS = STATIC_XWORDS + 4;  // 2,072,608 bytes
static __device__ __align__(256) u64 g_static_scratch[STATIC_WORDS];
}  // namespace mkx

namespace {
struct StaticDevice {
  bool ready = false;
  u64* scratch = nullptr;  // device address of g_static_scratch on this device
  int sms = 0, smem_optin = 0;
};
StaticDevice g_static_dev[64];
std::mutex g_static_mu;

mkx_status static_fail(const char* msg, mkx_status st) {
  snprintf(g_cuda_err, sizeof(g_cuda_err), "mkx_run_static: %s", msg);
  return st;
}

// Once per device, with that device current: the scratch array's device address (the host-side
// name g_static_scratch is only a stand-in) and the kernel's shared-memory limit.
mkx_status static_setup(int dev, StaticDevice** out) {
  std::lock_guard<std::mutex> lock(g_static_mu);
  StaticDevice& sd = g_static_dev[dev];
  if (!sd.ready) {
    void* ptr = nullptr;
    MKX_CUDA(cudaGetSymbolAddress(&ptr, g_static_scratch));
    MKX_CUDA(cudaDeviceGetAttribute(&sd.sms, cudaDevAttrMultiProcessorCount, dev));
    MKX_CUDA(cudaDeviceGetAttribute(&sd.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    MKX_CUDA(set_smem_attr<uint16_t>(sd.smem_optin));
    MKX_CUDA(set_smem_attr<float>(sd.smem_optin));
    sd.scratch = static_cast<u64*>(ptr);
    sd.ready = true;
  }
  *out = &sd;
  return MKX_OK;
}
}  // namespace

extern "C" mkx_status mkx_run_static(const mkx_dims* dims, const mkx_packed_weights* w, const mkx_step_inputs* in,
                                     int* err_out, cudaStream_t stream) {
  if (!dims || !w || !in) return MKX_ERR_INVALID_ARG;
  if (err_out && (reinterpret_cast<uintptr_t>(err_out) & 3u)) return static_fail("err_out must be 4-byte aligned", MKX_ERR_INVALID_ARG);
  const mkx_dims d = *dims;
  if (d.H != H || d.NH != NH || d.HD != HD || d.L < 1 || d.L > MKX_MAX_LAYERS || d.I < 128 || d.I % 128 != 0 ||
      d.A < AO || d.A > 32)
    return static_fail("unsupported expert geometry", MKX_ERR_UNSUPPORTED);
  if (d.I > STATIC_MAX_I) return static_fail("I exceeds the static scratch maximum of 3072", MKX_ERR_UNSUPPORTED);
  if (in->T < 1 || in->T > TP) return static_fail("T exceeds the static scratch maximum of 16 rows", MKX_ERR_UNSUPPORTED);
  if (in->n_steps < 1 || in->n_steps * d.L >= MAX_STEP_TAGS - 1 || in->action_dim < 1 || in->action_dim > AO)
    return MKX_ERR_INVALID_ARG;
  for (int s = 0; s < NSLOT; ++s)
    if (!w->w[s] || !aligned16(w->w[s])) return MKX_ERR_INVALID_ARG;
  if (!w->nrm || !w->tailw || !w->wout || !aligned16(w->tailw) || !aligned16(w->wout)) return MKX_ERR_INVALID_ARG;
  if (!in->x_in || !in->x_out || !in->mods || !in->dt || !in->cu_kv || !in->cu_src || !in->sa_cos || !in->sa_sin ||
      !in->ca_cos || !in->ca_sin)
    return MKX_ERR_INVALID_ARG;
  if (in->mem_rows < 1 || in->mem_rows > MAX_MEM_ROWS || in->ca_rows < 1) return MKX_ERR_UNSUPPORTED;
  if (in->mem_row_stride < H || in->mem_row_stride % 8 || in->ca_row_stride < H || in->ca_row_stride % 8)
    return MKX_ERR_INVALID_ARG;
  if (!aligned16(in->sa_cos) || !aligned16(in->sa_sin) || !aligned16(in->ca_cos) || !aligned16(in->ca_sin) ||
      !aligned16(in->mods))
    return MKX_ERR_INVALID_ARG;
  for (int l = 0; l < d.L; ++l) {
    if (!in->memk[l] || !in->memv[l] || !in->kca[l] || !in->vca[l]) return MKX_ERR_INVALID_ARG;
    if (((uintptr_t)in->memk[l] | (uintptr_t)in->memv[l] | (uintptr_t)in->kca[l] | (uintptr_t)in->vca[l]) & 7u)
      return MKX_ERR_INVALID_ARG;
  }
  int dev = 0;
  MKX_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return MKX_ERR_UNSUPPORTED;
  StaticDevice* sd = nullptr;
  const mkx_status st = static_setup(dev, &sd);
  if (st != MKX_OK) return st;
  const int G = d.grid > 0 ? d.grid : sd->sms;
  if (G < d.A || G < TP || G > H / 2 || G > sd->sms || min_part(d.I / 2, G) < 1) return MKX_ERR_RESOURCES;
  const Layout ly = make_layout(d.I, G);
  if (ly.max_rows_qkv / 2 * TP > NT || ly.max_rows_h > RESW || ly.max_rows_gu / 2 * TP > NT || ly.max_rows_dp > 32 ||
      ly.total > sd->smem_optin)
    return MKX_ERR_RESOURCES;

  Params p;
  memset(&p, 0, sizeof(p));
  for (int s = 0; s < NSLOT; ++s) p.w[s] = w->w[s];
  p.nrm = w->nrm;
  p.tailw = w->tailw;
  p.wout = w->wout;
  const int rw[NBUF] = {QKVWORDS, HWORDS, HWORDS, HWORDS, HWORDS, HWORDS, d.I / 2, HWORDS, XWORDS, DPWORDS};
  u64* xp = sd->scratch;
  for (int b = 0; b < NBUF; ++b) {
    p.xb[b] = xp;
    xp += (size_t)2 * TP * rw[b];
  }
  p.status = reinterpret_cast<int*>(sd->scratch + STATIC_XWORDS);  // [0] error, [1] sequence, [2..3] stages
  p.L = d.L;
  p.I = d.I;
  p.A = d.A;
  p.eps = d.eps;
  p.qk_eps = d.qk_eps;
  p.sm_scale = 1.0f / sqrtf((float)HD);
  for (int s = 0; s < NSLOT; ++s) p.s_slot[s] = ly.s_slot[s];
  p.s_x = ly.s_x; p.s_p = ly.s_p; p.s_mods = ly.s_mods; p.s_xs = ly.s_xs; p.s_res = ly.s_res;
  p.s_red = ly.s_red; p.s_bar = ly.s_bar; p.s_cnt = ly.s_cnt;
  p.x_in = in->x_in;
  p.x_out = in->x_out;
  p.mods = in->mods;
  p.dt = in->dt;
  for (int l = 0; l < d.L; ++l) {
    p.memk[l] = in->memk[l];
    p.memv[l] = in->memv[l];
    p.kca[l] = in->kca[l];
    p.vca[l] = in->vca[l];
  }
  p.mem_rows = in->mem_rows;
  p.mem_row_stride = in->mem_row_stride;
  p.ca_row_stride = in->ca_row_stride;
  p.ca_rows = in->ca_rows;
  p.cu_kv = in->cu_kv;
  p.cu_src = in->cu_src;
  p.sa_cos = in->sa_cos;
  p.sa_sin = in->sa_sin;
  p.ca_cos = in->ca_cos;
  p.ca_sin = in->ca_sin;
  p.trace_h = in->trace_h;
  p.prof = in->prof;
  p.timeout_ns = 2000000000ull;
  p.drop_stage = 0;
  p.T = in->T;
  p.adim = in->action_dim;
  p.n_steps = in->n_steps;

  // The array keeps the previous call's contents: the error word and the stage counter must start
  // at zero (the launch sequence number in between must not: it keeps tags from matching old words).
  MKX_CUDA(cudaMemsetAsync(p.status, 0, sizeof(int), stream));
  MKX_CUDA(cudaMemsetAsync(p.status + 2, 0, 2 * sizeof(int), stream));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = ly.total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = in->mods_fp32 ? cudaLaunchKernelEx(&cfg, expert_kernel<float>, p)
                                : cudaLaunchKernelEx(&cfg, expert_kernel<uint16_t>, p);
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(expert_kernel, static scratch)");
  if (err_out) MKX_CUDA(cudaMemcpyAsync(err_out, p.status, sizeof(int), cudaMemcpyDeviceToDevice, stream));
  return MKX_OK;
}
