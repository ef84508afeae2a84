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
// * Stage-to-stage exchange: activations go through small L2-resident buffers of 8-byte words
//   {bf16 x2 payload, 32-bit tag}. A consumer polls the words it needs until every tag equals the
//   producing stage's epoch: the poll is the data load, so no separate grid barrier or flag
//   round trip exists. Buffers are double-buffered by layer parity; tags never repeat between
//   consecutive launches (a per-handle launch sequence number is part of the tag).
// * Skinny GEMMs (10 action rows): swap-AB tensor-core MMA, weights as the 16-row A operand from
//   shared memory, the activations as the 8-column B operand, fp32 accumulate; K split across
//   warps, partials reduced through shared memory; fused epilogues (bf16 rounding, gated residual,
//   SiLU-mul).
// * Attention: one CTA per (head, action row) unit; K/V rows prefetched into registers before the
//   query is available; fp32 softmax; bf16(P) V.
// * Euler step tail: every CTA recomputes it (final AdaRMS, fp32 velocity of the real action dims,
//   Euler update, fp32 in-projection) so the next step's first GEMM needs no extra exchange.
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
constexpr int TP = 16;                   // padded action rows
constexpr int AO = 8;                    // carried action dims (src/mk_expert.py:478)
constexpr int XS = H + 8;                // shared X row stride (bf16 elements): conflict-free B loads
constexpr int HWORDS = H / 2;            // exchange words per H-wide row
constexpr int QKVWORDS = 3 * H / 2;
constexpr int MAXK = 8;                  // keys per 8-lane group per attention chunk (x32 groups)
constexpr int RESW = 8;                  // residual columns kept per CTA (o / ca-o / down rows)
constexpr int TAIL_FLOATS = 2 * AO * H + H + 32;   // wout rows 0..7 | win rows 0..7 | bin | bout
constexpr int TAIL_BYTES = TAIL_FLOATS * 4;
constexpr int MAX_STEP_TAGS = 4096;      // tag = seq * 4096 + instance + 1

enum Buf { B_QKV = 0, B_Y, B_H2, B_QCA, B_YCA, B_H3, B_G, B_HOUT, NBUF };
enum Slot { S_QKV = 0, S_O, S_QCA, S_OCA, S_GU, S_D, NSLOT };
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
  unsigned long long timeout_ns;
  int drop_stage;                 // test hook: CTA 0 withholds its layer-0 words of this stage
  int mem_rows, mem_row_stride, ca_rows, ca_row_stride;
  int L, I, T, A, adim, n_steps;
  float eps, qk_eps, sm_scale;
  int s_slot[NSLOT];              // shared-memory byte offsets
  int s_u, s_p, s_x, s_res, s_red, s_bar, s_cnt;
};

__host__ __device__ __forceinline__ int part_lo(int i, int P, int G) {
  return (int)(((long long)i * P) / G);
}

// ---------------------------------------------------------------------------------------------
// mods: bf16 or fp32 rows; a "pair" is two consecutive columns.
template <typename ModT> struct ModPair;
template <> struct ModPair<uint16_t> {
  uint32_t v;
  __device__ __forceinline__ void load(const uint16_t* m, int col) {
    v = __ldg(reinterpret_cast<const unsigned int*>(m + col));
  }
  __device__ __forceinline__ float lo() const { return bf_lo(v); }
  __device__ __forceinline__ float hi() const { return bf_hi(v); }
};
template <> struct ModPair<float> {
  float2 v;
  __device__ __forceinline__ void load(const float* m, int col) {
    v = __ldg(reinterpret_cast<const float2*>(m + col));
  }
  __device__ __forceinline__ float lo() const { return v.x; }
  __device__ __forceinline__ float hi() const { return v.y; }
};
template <typename ModT> __device__ __forceinline__ float mod_at(const ModT* m, int col);
template <> __device__ __forceinline__ float mod_at<uint16_t>(const uint16_t* m, int col) {
  return bf_at(__ldg(reinterpret_cast<const unsigned short*>(m + col)));
}
template <> __device__ __forceinline__ float mod_at<float>(const float* m, int col) { return __ldg(m + col); }

// ---------------------------------------------------------------------------------------------
struct Cta {
  char* slot[NSLOT];
  char* U;         // union: X [TP][XS] bf16 during GEMM stages, tail weights during the step tail
  float* P;        // partials [NW][16][16] / attention reductions [32][64]
  float* xs;       // action state [TP][32]
  float* res;      // residual columns [TP][RESW]
  float* red;      // small reductions
  uint64_t* bar;   // NSLOT weight slots + 1 tail region
  int* cnt;        // issued[NSLOT + 1], consumed[NSLOT + 1]
  int r0_qkv, R_qkv, c0, R_h, u0, R_gu;
  uint32_t slot_bytes[NSLOT];
  uint32_t tag0;
  int tid, warp, lane, cta, G;
  int stages;
};

__device__ __forceinline__ void record_error(const Params& p, const Cta& c, int kind, int stage) {
  atomicCAS(p.status, 0, (c.cta << 16) | (kind << 8) | stage);
}

__device__ __forceinline__ const uint16_t* slot_src(const Params& p, const Cta& c, int slot, int l) {
  const size_t HH = (size_t)H * H;
  switch (slot) {
    case S_QKV: return p.w[S_QKV] + (size_t)l * 3 * HH + (size_t)c.r0_qkv * H;
    case S_O: return p.w[S_O] + (size_t)l * HH + (size_t)c.c0 * H;
    case S_QCA: return p.w[S_QCA] + (size_t)l * HH + (size_t)c.c0 * H;
    case S_OCA: return p.w[S_OCA] + (size_t)l * HH + (size_t)c.c0 * H;
    case S_GU: return p.w[S_GU] + (size_t)l * 2 * p.I * H + (size_t)2 * c.u0 * H;
    default: return p.w[S_D] + (size_t)l * H * p.I + (size_t)c.c0 * p.I;
  }
}

// Thread 0 only.
__device__ __forceinline__ void issue_slot(const Params& p, Cta& c, int slot, int l) {
  fence_proxy_async();
  mbar_expect_tx(&c.bar[slot], c.slot_bytes[slot]);
  bulk_g2s(c.slot[slot], slot_src(p, c, slot, l), c.slot_bytes[slot], &c.bar[slot]);
  c.cnt[slot] += 1;
}
__device__ __forceinline__ void issue_tail(const Params& p, Cta& c) {
  fence_proxy_async();
  mbar_expect_tx(&c.bar[NSLOT], TAIL_BYTES);
  bulk_g2s(c.U, p.tailw, TAIL_BYTES, &c.bar[NSLOT]);
  c.cnt[NSLOT] += 1;
}

// All threads. Returns false on timeout (error recorded).
__device__ bool wait_bar(const Params& p, Cta& c, int b) {
  const uint32_t parity = (uint32_t)(c.cnt[NSLOT + 1 + b] & 1);
  uint32_t spins = 0;
  uint64_t t0 = 0;
  while (!mbar_try_wait(&c.bar[b], parity)) {
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
__device__ __forceinline__ void consumed(Cta& c, int b) {
  if (c.tid == 0) c.cnt[NSLOT + 1 + b] += 1;
}

// Poll N 16-byte pairs of exchange words until both tags of every valid pair equal `tag`.
// Returns 0, or the Waiter code (1 timeout, 2 abort seen).
template <int N>
__device__ __forceinline__ int poll_pairs(const u64* (&ptr)[N], u64 (&w0)[N], u64 (&w1)[N], uint32_t valid,
                                          uint32_t tag, Waiter& wt) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    if ((valid >> i) & 1u) {
      ld_volatile_v2(ptr[i], w0[i], w1[i]);
    } else {
      w0[i] = make_word(tag, 0u);
      w1[i] = w0[i];
    }
  }
  while (true) {
    uint32_t bad = 0;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      if (tag_of(w0[i]) != tag || tag_of(w1[i]) != tag) {
        bad |= 1u << i;
        ld_volatile_v2(ptr[i], w0[i], w1[i]);
      }
    }
    if (bad == 0u) return 0;
    const int r = wt.tick();
    if (r) return r;
  }
}

__device__ __forceinline__ int fail_code(const Params& p, const Cta& c, int r, int stage) {
  if (r == 1) record_error(p, c, K_TIMEOUT, stage);
  return r != 0;
}

// ---------------------------------------------------------------------------------------------
// AdaRMS staging: thread (n = tid / 16, part = tid % 16) owns 12 word pairs of action row n,
// q = part + 16 j, i.e. columns {16kb + 2cc, +1} and {16kb + 2cc + 8, +9} with kb = q / 4, cc = q % 4.
// hv[2j], hv[2j+1]: the two bf16-pair payloads. Writes a = bf16(h * rstd * (1 + scale) + shift)
// into X (rows >= T zero) and keeps h at the CTA's residual columns (src/mk_expert.py:93-122).
__device__ __forceinline__ int col_a_of(int q) { return 16 * (q >> 2) + 2 * (q & 3); }

template <typename ModT>
__device__ int load_rows_poll(const Params& p, const Cta& c, const u64* rows, uint32_t tag, uint32_t (&hv)[24],
                              int stage) {
  const int n = c.tid >> 4, part = c.tid & 15;
  const u64* ptr[12];
  u64 w0[12], w1[12];
#pragma unroll
  for (int j = 0; j < 12; ++j) ptr[j] = rows + (size_t)n * HWORDS + 2 * (part + 16 * j);
  Waiter wt(p.status, p.timeout_ns);
  const int r = poll_pairs<12>(ptr, w0, w1, n < p.T ? 0xfffu : 0u, tag, wt);
#pragma unroll
  for (int j = 0; j < 12; ++j) {
    hv[2 * j] = payload_of(w0[j]);
    hv[2 * j + 1] = payload_of(w1[j]);
  }
  return fail_code(p, c, r, stage);
}

template <typename ModT>
__device__ void stage_adarms(const Params& p, Cta& c, const uint32_t (&hv)[24], const ModT* msc) {
  const int n = c.tid >> 4, part = c.tid & 15;
  const ModT* msh = msc + H;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 24; ++j) {
    const float a = bf_lo(hv[j]), b = bf_hi(hv[j]);
    ss = fmaf(a, a, ss);
    ss = fmaf(b, b, ss);
  }
  ss += __shfl_xor_sync(0xffffffffu, ss, 8);
  ss += __shfl_xor_sync(0xffffffffu, ss, 4);
  ss += __shfl_xor_sync(0xffffffffu, ss, 2);
  ss += __shfl_xor_sync(0xffffffffu, ss, 1);
  const float rstd = rsqrtf(ss / (float)H + p.eps);
  const bool live = n < p.T;
  char* xrow = c.U + (size_t)n * XS * 2;
#pragma unroll
  for (int j = 0; j < 12; ++j) {
    const int q = part + 16 * j;
    const int ca = col_a_of(q), cb = ca + 8;
    ModPair<ModT> sa, sb, ha, hb;
    sa.load(msc, ca);
    sb.load(msc, cb);
    ha.load(msh, ca);
    hb.load(msh, cb);
    const float h0 = bf_lo(hv[2 * j]), h1 = bf_hi(hv[2 * j]);
    const float h2 = bf_lo(hv[2 * j + 1]), h3 = bf_hi(hv[2 * j + 1]);
    const float a0 = fmaf(h0 * rstd, 1.f + sa.lo(), ha.lo());
    const float a1 = fmaf(h1 * rstd, 1.f + sa.hi(), ha.hi());
    const float a2 = fmaf(h2 * rstd, 1.f + sb.lo(), hb.lo());
    const float a3 = fmaf(h3 * rstd, 1.f + sb.hi(), hb.hi());
    *reinterpret_cast<uint32_t*>(xrow + ca * 2) = live ? pack_bf2(a0, a1) : 0u;
    *reinterpret_cast<uint32_t*>(xrow + cb * 2) = live ? pack_bf2(a2, a3) : 0u;
    if (live) {
      int o = ca - c.c0;
      if (o >= 0 && o < c.R_h) c.res[n * RESW + o] = h0;
      if (o + 1 >= 0 && o + 1 < c.R_h) c.res[n * RESW + o + 1] = h1;
      o = cb - c.c0;
      if (o >= 0 && o < c.R_h) c.res[n * RESW + o] = h2;
      if (o + 1 >= 0 && o + 1 < c.R_h) c.res[n * RESW + o + 1] = h3;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// GEMM with the B operand (activations) from shared X: `nmat` matrices of R rows each (K = H).
__device__ void mma_from_x(const Params& p, Cta& c, const char* wslot, int nmat, int R) {
  const int mtpm = (R + 15) >> 4, mt = nmat * mtpm, ks = NW / mt;
  const int g = c.lane >> 2, cc = c.lane & 3;
  const bool two = p.T > 8;
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
  if (c.warp < mt * ks) {
    const int m = c.warp % mt, ksl = c.warp / mt;
    const int j = m / mtpm, mm = m % mtpm;
    const char* A = wslot + (size_t)j * R * H * 2 + cc * 8;
    constexpr int KB = H / 16;
    const int kb0 = ksl * KB / ks, kb1 = (ksl + 1) * KB / ks;
    const int ra = mm * 16 + g, rb = ra + 8;
    const bool va = ra < R, vb = rb < R;
    const char* x0 = c.U + (size_t)g * XS * 2 + cc * 4;
    const char* x1 = c.U + (size_t)(8 + g) * XS * 2 + cc * 4;
#pragma unroll 4
    for (int kb = kb0; kb < kb1; ++kb) {
      const char* blk = A + (size_t)kb * R * 32;
      const uint2 a = va ? lds64(blk + ra * 32) : make_uint2(0u, 0u);
      const uint2 b = vb ? lds64(blk + rb * 32) : make_uint2(0u, 0u);
      const uint32_t b0 = lds32(x0 + kb * 32), b1 = lds32(x0 + kb * 32 + 16);
      mma_bf16(d0, a.x, b.x, a.y, b.y, b0, b1);
      if (two) {
        const uint32_t e0 = lds32(x1 + kb * 32), e1 = lds32(x1 + kb * 32 + 16);
        mma_bf16(d1, a.x, b.x, a.y, b.y, e0, e1);
      }
    }
  }
  float* P = c.P + c.warp * 256;
  P[g * 16 + 2 * cc] = d0[0];
  P[g * 16 + 2 * cc + 1] = d0[1];
  P[(g + 8) * 16 + 2 * cc] = d0[2];
  P[(g + 8) * 16 + 2 * cc + 1] = d0[3];
  P[g * 16 + 8 + 2 * cc] = d1[0];
  P[g * 16 + 8 + 2 * cc + 1] = d1[1];
  P[(g + 8) * 16 + 8 + 2 * cc] = d1[2];
  P[(g + 8) * 16 + 8 + 2 * cc + 1] = d1[3];
}

// GEMM with the B operand polled straight from an exchange buffer (rows of K/2 words); one
// matrix of R <= 16 rows, K split over the 8 warps. Returns nonzero on a failed wait.
__device__ int mma_from_words(const Params& p, Cta& c, const char* wslot, int R, int K, const u64* rows,
                              uint32_t tag, int stage) {
  const int g = c.lane >> 2, cc = c.lane & 3;
  const int RW = K >> 1, KB = K >> 4;
  const int kb0 = c.warp * KB / NW, kb1 = (c.warp + 1) * KB / NW;
  const bool v0 = g < p.T, v1 = (8 + g) < p.T, two = p.T > 8;
  const u64* row0 = rows + (size_t)g * RW + 2 * cc;
  const u64* row1 = rows + (size_t)(8 + g) * RW + 2 * cc;
  const char* A = wslot + cc * 8;
  const bool va = g < R, vb = g + 8 < R;
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
  Waiter wt(p.status, p.timeout_ns);
  int rc = 0;
  constexpr int CH = 6;
  for (int kbc = kb0; kbc < kb1; kbc += CH) {
    const u64* ptr[2 * CH];
    u64 w0[2 * CH], w1[2 * CH];
    uint32_t valid = 0;
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int kb = kbc + i;
      ptr[2 * i] = row0 + kb * 8;
      ptr[2 * i + 1] = row1 + kb * 8;
      if (kb < kb1) valid |= ((v0 ? 1u : 0u) | (v1 ? 2u : 0u)) << (2 * i);
    }
    rc = poll_pairs<2 * CH>(ptr, w0, w1, valid, tag, wt);
    if (__any_sync(0xffffffffu, rc != 0)) {  // keep the warp converged for mma.sync
      if (rc == 0) rc = 2;
      break;
    }
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int kb = kbc + i;
      if (kb < kb1) {
        const char* blk = A + (size_t)kb * R * 32;
        const uint2 a = va ? lds64(blk + g * 32) : make_uint2(0u, 0u);
        const uint2 b = vb ? lds64(blk + (g + 8) * 32) : make_uint2(0u, 0u);
        mma_bf16(d0, a.x, b.x, a.y, b.y, payload_of(w0[2 * i]), payload_of(w1[2 * i]));
        if (two) mma_bf16(d1, a.x, b.x, a.y, b.y, payload_of(w0[2 * i + 1]), payload_of(w1[2 * i + 1]));
      }
    }
  }
  float* P = c.P + c.warp * 256;
  P[g * 16 + 2 * cc] = d0[0];
  P[g * 16 + 2 * cc + 1] = d0[1];
  P[(g + 8) * 16 + 2 * cc] = d0[2];
  P[(g + 8) * 16 + 2 * cc + 1] = d0[3];
  P[g * 16 + 8 + 2 * cc] = d1[0];
  P[g * 16 + 8 + 2 * cc + 1] = d1[1];
  P[(g + 8) * 16 + 8 + 2 * cc] = d1[2];
  P[(g + 8) * 16 + 8 + 2 * cc + 1] = d1[3];
  return fail_code(p, c, rc, stage);
}

// Sum of the K-split partials for output row r (of matrix j), token n.
__device__ __forceinline__ float part_sum(const Cta& c, int j, int R, int nmat, int r, int n) {
  const int mtpm = (R + 15) >> 4, mt = nmat * mtpm, ks = NW / mt;
  const int m = j * mtpm + (r >> 4);
  const int idx = (r & 15) * 16 + n;
  float s = 0.f;
  for (int k = 0; k < ks; ++k) s += c.P[(m + mt * k) * 256 + idx];
  return s;
}

// Epilogues ----------------------------------------------------------------------------------
// Linear output rounded to bf16 (QKV, CA query): words of columns [col0, col0 + R).
__device__ void epi_plain(const Params& p, const Cta& c, int R, int col0, u64* out_rows, int row_words,
                          uint32_t tag) {
  const int npairs = R >> 1;
  for (int e = c.tid; e < npairs * p.T; e += NT) {
    const int pp = e % npairs, n = e / npairs;
    const float v0 = part_sum(c, 0, R, 1, 2 * pp, n), v1 = part_sum(c, 0, R, 1, 2 * pp + 1, n);
    st_volatile(out_rows + (size_t)n * row_words + word_pos((col0 >> 1) + pp), make_word(tag, pack_bf2(v0, v1)));
  }
}

// Gated residual out = bf16(res + bf16(acc) * gate) (src/mk_expert.py:162-172).
template <typename ModT>
__device__ void epi_gated(const Params& p, const Cta& c, const ModT* gate, u64* out_rows, uint32_t tag,
                          uint16_t* trace) {
  const int npairs = c.R_h >> 1;
  for (int e = c.tid; e < npairs * p.T; e += NT) {
    const int pp = e % npairs, n = e / npairs;
    float o[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int r = 2 * pp + k;
      const float acc = round_bf(part_sum(c, 0, c.R_h, 1, r, n));
      o[k] = fmaf(acc, mod_at<ModT>(gate, c.c0 + r), c.res[n * RESW + r]);
    }
    const uint32_t pl = pack_bf2(o[0], o[1]);
    st_volatile(out_rows + (size_t)n * HWORDS + word_pos((c.c0 >> 1) + pp), make_word(tag, pl));
    if (trace) *reinterpret_cast<uint32_t*>(trace + (size_t)n * H + c.c0 + 2 * pp) = pl;
  }
}

// g = bf16(silu(bf16(gate)) * bf16(up)) (src/mk_expert.py:403-413).
__device__ void epi_gu(const Params& p, const Cta& c, u64* out_rows, uint32_t tag) {
  const int R = c.R_gu, npairs = R >> 1, row_words = p.I >> 1;
  for (int e = c.tid; e < npairs * p.T; e += NT) {
    const int pp = e % npairs, n = e / npairs;
    float o[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int r = 2 * pp + k;
      const float gf = round_bf(part_sum(c, 0, R, 2, r, n));
      const float uf = round_bf(part_sum(c, 1, R, 2, r, n));
      o[k] = gf / (1.f + __expf(-gf)) * uf;
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
__device__ __forceinline__ void f32_nat_to_lane(Lane8& x, const float* row, int d0) {
  const float4 A = __ldg(reinterpret_cast<const float4*>(row + d0));
  const float4 B = __ldg(reinterpret_cast<const float4*>(row + d0 + 8));
  x.v[0] = A.x; x.v[1] = A.y; x.v[2] = B.x; x.v[3] = B.y;
  x.v[4] = A.z; x.v[5] = A.w; x.v[6] = B.z; x.v[7] = B.w;
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
// Block-wide max of a value that is uniform within each 8-lane group.
__device__ __forceinline__ float block_max(const Cta& c, float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
  __syncthreads();
  if (c.lane == 0) c.red[c.warp] = v;
  __syncthreads();
  float m = c.red[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) m = fmaxf(m, c.red[w]);
  return m;
}

// SA = true: self-attention (queries of row t over memory rows [cu_kv[0], PM) and the T action
// rows, src/mk_expert.py:196-222). SA = false: cross-attention over the S valid source rows
// (src/mk_expert.py:225-251). Returns nonzero on a failed wait.
template <bool SA>
__device__ int attention_unit(const Params& p, Cta& c, int l, int h, int t, const u64* src_rows, u64* y_rows,
                              uint32_t tag) {
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

  // Prefetch chunk 0 of K/V and the per-row tables; none of it depends on the exchange.
  uint2 kA[MAXK], kB[MAXK], vA[MAXK], vB[MAXK];
  auto load_chunk = [&](int base) {
#pragma unroll
    for (int i = 0; i < MAXK; ++i) {
      const int j = base + kg + 32 * i;
      kA[i] = kB[i] = vA[i] = vB[i] = make_uint2(0u, 0u);
      if (j < nkeys) {
        const uint16_t* kr = Kb + (size_t)j * stride + h * HD + d0;
        const uint16_t* vr = Vb + (size_t)j * stride + h * HD + d0;
        kA[i] = __ldg(reinterpret_cast<const uint2*>(kr));
        kB[i] = __ldg(reinterpret_cast<const uint2*>(kr + 8));
        vA[i] = __ldg(reinterpret_cast<const uint2*>(vr));
        vB[i] = __ldg(reinterpret_cast<const uint2*>(vr + 8));
      }
    }
  };
  load_chunk(kbeg);
  Lane8 wq, cq, sq;
  f32_nat_to_lane(wq, nrm, d0);
  f32_nat_to_lane(cq, cosr + (size_t)t * HD, d0);
  f32_nat_to_lane(sq, sinr + (size_t)t * HD, d0);
  const bool own = SA && kg < p.T;
  Lane8 wk, ck, sk;
  if (SA) {
    f32_nat_to_lane(wk, nrm + (size_t)p.L * HD, d0);
    const int krow = kg < p.T ? kg : p.T - 1;  // groups without an own row compute a discarded key
    f32_nat_to_lane(ck, cosr + (size_t)krow * HD, d0);
    f32_nat_to_lane(sk, sinr + (size_t)krow * HD, d0);
  }

  // Poll the query (and, for SA, this group's own action row's k and v).
  const int qoff = h * 32 + 4 * l8;
  const int row_words = SA ? QKVWORDS : HWORDS;
  const u64* ptr[6];
  u64 w0[6], w1[6];
  ptr[0] = src_rows + (size_t)t * row_words + qoff;
  ptr[1] = ptr[0] + 2;
  ptr[2] = src_rows + (size_t)kg * row_words + HWORDS + qoff;
  ptr[3] = ptr[2] + 2;
  ptr[4] = src_rows + (size_t)kg * row_words + 2 * HWORDS + qoff;
  ptr[5] = ptr[4] + 2;
  Waiter wt(p.status, p.timeout_ns);
  const int rc = poll_pairs<6>(ptr, w0, w1, own ? 0x3fu : 0x3u, tag, wt);
  fail_code(p, c, rc, SA ? ST_SA : ST_CA);
  if (__syncthreads_or(rc != 0)) return 1;

  Lane8 q;
  bf_words_to_lane(q, payload_of(w0[0]), payload_of(w1[0]), payload_of(w0[1]), payload_of(w1[1]));
  norm_rope(q, wq, cq, sq, p.qk_eps, l8);
  Lane8 ko, vo;
  float s_own = -INFINITY;
  if (SA) {
    bf_words_to_lane(ko, payload_of(w0[2]), payload_of(w1[2]), payload_of(w0[3]), payload_of(w1[3]));
    bf_words_to_lane(vo, payload_of(w0[4]), payload_of(w1[4]), payload_of(w0[5]), payload_of(w1[5]));
    norm_rope(ko, wk, ck, sk, p.qk_eps, l8);  // all lanes: the shuffles need the full warp
    const float so = dot8(q, ko) * p.sm_scale;
    if (own) s_own = so;
  }

  float m_run = -INFINITY, den = 0.f;
  float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int base = kbeg; base < nkeys || (SA && base == kbeg); base += 32 * MAXK) {
    if (base != kbeg) load_chunk(base);
    float s[MAXK];
    float mloc = (SA && base == kbeg) ? s_own : -INFINITY;
#pragma unroll
    for (int i = 0; i < MAXK; ++i) {
      // Key slot i holds a valid key for some groups only when nkeys - base is not a multiple of
      // 32: the group-of-8 shuffles in dot8 must still run on every lane of the warp.
      if (base + 32 * i >= nkeys) {  // uniform: no group has a key in this slot
        s[i] = -INFINITY;
        continue;
      }
      const int j = base + kg + 32 * i;
      Lane8 k;
      bf_nat_to_lane(k, kA[i], kB[i]);
      const float dv = dot8(q, k) * p.sm_scale;
      s[i] = j < nkeys ? dv : -INFINITY;
      mloc = fmaxf(mloc, s[i]);
    }
    const float m_new = fmaxf(m_run, block_max(c, mloc));
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
      const int j = base + kg + 32 * i;
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
    if (base + 32 * MAXK >= nkeys) break;
  }
  // Reduce the 32 groups: o in lane order per lane, den per group.
  __syncthreads();
  float* ro = c.P;            // [32][64]
  float* rd = c.P + 32 * 64;  // [32]
#pragma unroll
  for (int e = 0; e < 8; ++e) ro[kg * 64 + l8 * 8 + e] = o[e];
  if (l8 == 0) rd[kg] = den;
  __syncthreads();
  if (c.tid < 64) {
    float acc = 0.f, dsum = 0.f;
    for (int gi = 0; gi < 32; ++gi) {
      acc += ro[gi * 64 + c.tid];
      dsum += rd[gi];
    }
    const float val = acc / dsum;
    const float nxt = __shfl_down_sync(0xffffffffu, val, 1);
    if ((c.tid & 1) == 0)
      st_volatile(y_rows + (size_t)t * HWORDS + h * 32 + (c.tid >> 1), make_word(tag, pack_bf2(val, nxt)));
  }
  return 0;
}

// ---------------------------------------------------------------------------------------------
// Step tail (src/mk_expert.py:254-299). Thread (n, part) owns the 48 columns of its word pairs.
// mode 0: FIRST (h0 from x_in), 1: intermediate step (velocity, Euler update, h0), 2: last step
// (CTA a < A writes output dim a). Produces hv (h0 payloads) for modes 0 and 1.
template <typename ModT>
__device__ int step_tail(const Params& p, Cta& c, int mode, const ModT* modf, const u64* hrows, uint32_t htag,
                         uint32_t (&hv)[24]) {
  const int n = c.tid >> 4, part = c.tid & 15;
  const float* tw = reinterpret_cast<const float*>(c.U);
  const float* s_wout = tw;
  const float* s_win = tw + AO * H;
  const float* s_bin = tw + 2 * AO * H;
  const float* s_bout = s_bin + H;
  const float dt = __ldg(p.dt);
  const int adim = p.adim;
  const int a_out = c.cta;  // output dim of this CTA in mode 2
  if (mode == 2 && a_out >= p.A) return 0;  // uniform per CTA: only CTAs 0..A-1 write the output
  float wrow[48];
  if (mode == 2) {
#pragma unroll
    for (int j = 0; j < 12; ++j) {
      const int ca = col_a_of(part + 16 * j);
      const float2 A = __ldg(reinterpret_cast<const float2*>(p.wout + (size_t)a_out * H + ca));
      const float2 B = __ldg(reinterpret_cast<const float2*>(p.wout + (size_t)a_out * H + ca + 8));
      wrow[4 * j] = A.x; wrow[4 * j + 1] = A.y; wrow[4 * j + 2] = B.x; wrow[4 * j + 3] = B.y;
    }
  }
  float xo[AO];
  if (mode != 0) {
    // o = bf16(AdaRMS_final(h)), v_a = o . Wout[a] + bout[a]
    ModPair<ModT> sa[12], sb[12], ha[12], hb[12];
#pragma unroll
    for (int j = 0; j < 12; ++j) {
      const int ca = col_a_of(part + 16 * j);
      sa[j].load(modf, ca); sb[j].load(modf, ca + 8);
      ha[j].load(modf + H, ca); hb[j].load(modf + H, ca + 8);
    }
    const int rc = load_rows_poll<ModT>(p, c, hrows, htag, hv, ST_TAIL);
    if (__syncthreads_or(rc)) return 1;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 24; ++j) {
      const float a = bf_lo(hv[j]), b = bf_hi(hv[j]);
      ss = fmaf(a, a, ss);
      ss = fmaf(b, b, ss);
    }
    ss += __shfl_xor_sync(0xffffffffu, ss, 8);
    ss += __shfl_xor_sync(0xffffffffu, ss, 4);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    const float rstd = rsqrtf(ss / (float)H + p.eps);
    float ov[48];
#pragma unroll
    for (int j = 0; j < 12; ++j) {
      ov[4 * j] = round_bf(fmaf(bf_lo(hv[2 * j]) * rstd, 1.f + sa[j].lo(), ha[j].lo()));
      ov[4 * j + 1] = round_bf(fmaf(bf_hi(hv[2 * j]) * rstd, 1.f + sa[j].hi(), ha[j].hi()));
      ov[4 * j + 2] = round_bf(fmaf(bf_lo(hv[2 * j + 1]) * rstd, 1.f + sb[j].lo(), hb[j].lo()));
      ov[4 * j + 3] = round_bf(fmaf(bf_hi(hv[2 * j + 1]) * rstd, 1.f + sb[j].hi(), hb[j].hi()));
    }
    if (mode == 2) {
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 48; ++e) acc = fmaf(ov[e], wrow[e], acc);
      acc += __shfl_xor_sync(0xffffffffu, acc, 8);
      acc += __shfl_xor_sync(0xffffffffu, acc, 4);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      const float v = acc + __ldg(p.tailw + 2 * AO * H + H + a_out);
      if (part == 0 && n < p.T) {
        const float xp = a_out < adim ? c.xs[n * 32 + a_out] : 0.f;
        p.x_out[(size_t)n * p.A + a_out] = fmaf(dt, v, xp);
      }
      return 0;
    }
#pragma unroll
    for (int a = 0; a < AO; ++a) {
      float acc = 0.f;
      if (a < adim) {
        const float* wr = s_wout + a * H;
#pragma unroll
        for (int j = 0; j < 12; ++j) {
          const int ca = col_a_of(part + 16 * j);
          acc = fmaf(ov[4 * j], wr[ca], acc);
          acc = fmaf(ov[4 * j + 1], wr[ca + 1], acc);
          acc = fmaf(ov[4 * j + 2], wr[ca + 8], acc);
          acc = fmaf(ov[4 * j + 3], wr[ca + 9], acc);
        }
      }
      acc += __shfl_xor_sync(0xffffffffu, acc, 8);
      acc += __shfl_xor_sync(0xffffffffu, acc, 4);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      const float v = acc + s_bout[a];
      xo[a] = a < adim ? fmaf(dt, v, c.xs[n * 32 + a]) : 0.f;
    }
    __syncwarp();
    if (part == 0 && n < p.T) {
#pragma unroll
      for (int a = 0; a < AO; ++a)
        if (a < adim) c.xs[n * 32 + a] = xo[a];
    }
  } else {
#pragma unroll
    for (int a = 0; a < AO; ++a) xo[a] = (a < adim && n < p.T) ? c.xs[n * 32 + a] : 0.f;
  }
  // h0 = bf16(xpad[:AO] @ Win[:AO] + bin) in fp32.
#pragma unroll
  for (int j = 0; j < 12; ++j) {
    const int ca = col_a_of(part + 16 * j);
    float hq[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = ca + (e & 1) + (e >> 1) * 8;
      float acc = s_bin[col];
#pragma unroll
      for (int a = 0; a < AO; ++a) acc = fmaf(xo[a], s_win[a * H + col], acc);
      hq[e] = acc;
    }
    hv[2 * j] = n < p.T ? pack_bf2(hq[0], hq[1]) : 0u;
    hv[2 * j + 1] = n < p.T ? pack_bf2(hq[2], hq[3]) : 0u;
  }
  return 0;
}

// ---------------------------------------------------------------------------------------------
template <typename ModT>
__global__ void __launch_bounds__(NT, 1) expert_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) char smem[];
  Cta c;
  c.tid = threadIdx.x;
  c.warp = c.tid >> 5;
  c.lane = c.tid & 31;
  c.cta = blockIdx.x;
  c.G = gridDim.x;
  c.stages = 0;
#pragma unroll
  for (int s = 0; s < NSLOT; ++s) c.slot[s] = smem + p.s_slot[s];
  c.U = smem + p.s_u;
  c.P = reinterpret_cast<float*>(smem + p.s_p);
  c.xs = reinterpret_cast<float*>(smem + p.s_x);
  c.res = reinterpret_cast<float*>(smem + p.s_res);
  c.red = reinterpret_cast<float*>(smem + p.s_red);
  c.bar = reinterpret_cast<uint64_t*>(smem + p.s_bar);
  c.cnt = reinterpret_cast<int*>(smem + p.s_cnt);
  {
    const int G = c.G, i = c.cta;
    int lo = part_lo(i, 3 * H / 2, G), hi = part_lo(i + 1, 3 * H / 2, G);
    c.r0_qkv = 2 * lo; c.R_qkv = 2 * (hi - lo);
    lo = part_lo(i, H / 2, G); hi = part_lo(i + 1, H / 2, G);
    c.c0 = 2 * lo; c.R_h = 2 * (hi - lo);
    lo = part_lo(i, p.I / 2, G); hi = part_lo(i + 1, p.I / 2, G);
    c.u0 = 2 * lo; c.R_gu = 2 * (hi - lo);
    c.slot_bytes[S_QKV] = (uint32_t)c.R_qkv * H * 2;
    c.slot_bytes[S_O] = c.slot_bytes[S_QCA] = c.slot_bytes[S_OCA] = (uint32_t)c.R_h * H * 2;
    c.slot_bytes[S_GU] = (uint32_t)c.R_gu * H * 4;
    c.slot_bytes[S_D] = (uint32_t)c.R_h * p.I * 2;
  }
  const uint32_t seq = (uint32_t)ld_volatile_i32(p.status + 1);
  c.tag0 = seq * (uint32_t)MAX_STEP_TAGS + 1u;
  const int L = p.L;
  const int total = p.n_steps * L;
  const size_t MODW = (size_t)9 * L * H + 2 * H;
  const ModT* mods = reinterpret_cast<const ModT*>(p.mods);
  bool fail = false;

  if (c.tid == 0) {
    for (int b = 0; b < NSLOT + 1; ++b) {
      mbar_init(&c.bar[b], 1);
      c.cnt[b] = 0;
      c.cnt[NSLOT + 1 + b] = 0;
    }
    fence_mbar_init();
  }
  if (c.tid < TP * 32) c.xs[c.tid] = 0.f;
  __syncthreads();
  if (c.tid == 0) {
    issue_tail(p, c);
    for (int s = 0; s < NSLOT; ++s) issue_slot(p, c, s, 0);
  }
  for (int e = c.tid; e < p.T * p.A; e += NT) c.xs[(e / p.A) * 32 + (e % p.A)] = __ldg(p.x_in + e);
  __syncthreads();

  uint32_t hv[24];
  // FIRST tail: h0 from x after step 1.
  fail = !wait_bar(p, c, NSLOT);
  if (__syncthreads_or(fail)) goto drain;
  consumed(c, NSLOT);
  step_tail<ModT>(p, c, 0, nullptr, nullptr, 0u, hv);
  c.stages++;
  __syncthreads();  // the tail weights in U are dead from here; X takes U over

  for (int s = 0; s < p.n_steps; ++s) {
    const ModT* mrow = mods + (size_t)(1 + s) * MODW;
    for (int l = 0; l < L; ++l) {
      const int gi = s * L + l;
      const int par = gi & 1;
      const uint32_t tag = c.tag0 + (uint32_t)gi;
      const ModT* m_sa = mrow + (size_t)9 * l * H;
      const ModT* m_ca = m_sa + 3 * H;
      const ModT* m_mlp = m_ca + 3 * H;
      u64* const* xb = p.xb;

      // 1. QKV = bf16(AdaRMS(h; sa) @ Wqkv^T)
      if (l > 0) {
        const u64* hin = xb[B_HOUT] + (size_t)((gi - 1) & 1) * TP * HWORDS;
        fail = load_rows_poll<ModT>(p, c, hin, tag - 1u, hv, ST_QKV) != 0;
        if (__syncthreads_or(fail)) goto drain;
      }
      stage_adarms<ModT>(p, c, hv, m_sa);
      fail = !wait_bar(p, c, S_QKV);
      if (__syncthreads_or(fail)) goto drain;
      consumed(c, S_QKV);
      mma_from_x(p, c, c.slot[S_QKV], 1, c.R_qkv);
      __syncthreads();
      if (c.tid == 0 && gi + 1 < total) issue_slot(p, c, S_QKV, (gi + 1) % L);
      if (!(p.drop_stage == ST_QKV && c.cta == 0 && gi == 0))
        epi_plain(p, c, c.R_qkv, c.r0_qkv, xb[B_QKV] + (size_t)par * TP * QKVWORDS, QKVWORDS, tag);
      c.stages++;

      // 2. self-attention, one (head, row) unit per CTA
      for (int u = c.cta; u < NH * p.T; u += c.G) {
        fail = attention_unit<true>(p, c, l, u % NH, u / NH, xb[B_QKV] + (size_t)par * TP * QKVWORDS,
                                    xb[B_Y] + (size_t)par * TP * HWORDS, tag) != 0;
        if (__syncthreads_or(fail)) goto drain;
      }
      c.stages++;

      // 3. h2 = bf16(h + bf16(y @ Wo^T) * gate_sa)
      __syncthreads();
      fail = !wait_bar(p, c, S_O);
      if (__syncthreads_or(fail)) goto drain;
      consumed(c, S_O);
      fail = mma_from_words(p, c, c.slot[S_O], c.R_h, H, xb[B_Y] + (size_t)par * TP * HWORDS, tag, ST_O) != 0;
      if (__syncthreads_or(fail)) goto drain;
      if (c.tid == 0 && gi + 1 < total) issue_slot(p, c, S_O, (gi + 1) % L);
      epi_gated<ModT>(p, c, m_sa + 2 * H, xb[B_H2] + (size_t)par * TP * HWORDS, tag, nullptr);
      c.stages++;
      __syncthreads();

      // 4. CA query = bf16(AdaRMS(h2; ca) @ Wqca^T)
      fail = load_rows_poll<ModT>(p, c, xb[B_H2] + (size_t)par * TP * HWORDS, tag, hv, ST_CAQ) != 0;
      if (__syncthreads_or(fail)) goto drain;
      stage_adarms<ModT>(p, c, hv, m_ca);
      fail = !wait_bar(p, c, S_QCA);
      if (__syncthreads_or(fail)) goto drain;
      consumed(c, S_QCA);
      mma_from_x(p, c, c.slot[S_QCA], 1, c.R_h);
      __syncthreads();
      if (c.tid == 0 && gi + 1 < total) issue_slot(p, c, S_QCA, (gi + 1) % L);
      epi_plain(p, c, c.R_h, c.c0, xb[B_QCA] + (size_t)par * TP * HWORDS, HWORDS, tag);
      c.stages++;

      // 5. cross-attention
      for (int u = c.cta; u < NH * p.T; u += c.G) {
        fail = attention_unit<false>(p, c, l, u % NH, u / NH, xb[B_QCA] + (size_t)par * TP * HWORDS,
                                     xb[B_YCA] + (size_t)par * TP * HWORDS, tag) != 0;
        if (__syncthreads_or(fail)) goto drain;
      }
      c.stages++;

      // 6. h3 = bf16(h2 + bf16(y_ca @ Woca^T) * gate_ca)
      __syncthreads();
      fail = !wait_bar(p, c, S_OCA);
      if (__syncthreads_or(fail)) goto drain;
      consumed(c, S_OCA);
      fail = mma_from_words(p, c, c.slot[S_OCA], c.R_h, H, xb[B_YCA] + (size_t)par * TP * HWORDS, tag, ST_OCA) != 0;
      if (__syncthreads_or(fail)) goto drain;
      if (c.tid == 0 && gi + 1 < total) issue_slot(p, c, S_OCA, (gi + 1) % L);
      epi_gated<ModT>(p, c, m_ca + 2 * H, xb[B_H3] + (size_t)par * TP * HWORDS, tag, nullptr);
      c.stages++;
      __syncthreads();

      // 7. g = bf16(silu(gate) * up) of AdaRMS(h3; mlp)
      fail = load_rows_poll<ModT>(p, c, xb[B_H3] + (size_t)par * TP * HWORDS, tag, hv, ST_GU) != 0;
      if (__syncthreads_or(fail)) goto drain;
      stage_adarms<ModT>(p, c, hv, m_mlp);
      fail = !wait_bar(p, c, S_GU);
      if (__syncthreads_or(fail)) goto drain;
      consumed(c, S_GU);
      mma_from_x(p, c, c.slot[S_GU], 2, c.R_gu);
      __syncthreads();
      if (c.tid == 0) {
        if (gi + 1 < total) issue_slot(p, c, S_GU, (gi + 1) % L);
        if (l == L - 1 && s + 1 < p.n_steps) issue_tail(p, c);  // X is dead until the tail
      }
      epi_gu(p, c, xb[B_G] + (size_t)par * TP * (p.I >> 1), tag);
      c.stages++;

      // 8. h = bf16(h3 + bf16(g @ Wd^T) * gate_mlp)
      __syncthreads();
      fail = !wait_bar(p, c, S_D);
      if (__syncthreads_or(fail)) goto drain;
      consumed(c, S_D);
      fail = mma_from_words(p, c, c.slot[S_D], c.R_h, p.I, xb[B_G] + (size_t)par * TP * (p.I >> 1), tag, ST_DOWN) != 0;
      if (__syncthreads_or(fail)) goto drain;
      if (c.tid == 0 && gi + 1 < total) issue_slot(p, c, S_D, (gi + 1) % L);
      epi_gated<ModT>(p, c, m_mlp + 2 * H, xb[B_HOUT] + (size_t)par * TP * HWORDS, tag,
                      p.trace_h ? p.trace_h + (size_t)gi * p.T * H : nullptr);
      c.stages++;
      __syncthreads();
    }
    // Euler step tail: final AdaRMS, velocity, x update, next step's h0.
    {
      const int gl = s * L + L - 1;
      const u64* hrows = p.xb[B_HOUT] + (size_t)(gl & 1) * TP * HWORDS;
      const ModT* modf = mrow + (size_t)9 * L * H;
      const bool last = s + 1 == p.n_steps;
      if (!last) {
        fail = !wait_bar(p, c, NSLOT);
        if (__syncthreads_or(fail)) goto drain;
        consumed(c, NSLOT);
      }
      fail = step_tail<ModT>(p, c, last ? 2 : 1, modf, hrows, c.tag0 + (uint32_t)gl, hv) != 0;
      if (__syncthreads_or(fail)) goto drain;
      c.stages++;
    }
  }

drain:
  // Normal exit: nothing is in flight. After a failed wait: drain every issued bulk copy (bounded).
  if (c.tid == 0) {
    for (int b = 0; b < NSLOT + 1; ++b) {
      while (c.cnt[NSLOT + 1 + b] < c.cnt[b]) {
        const uint32_t parity = (uint32_t)(c.cnt[NSLOT + 1 + b] & 1);
        uint64_t t0 = globaltimer();
        bool ok = false;
        while (!(ok = mbar_try_wait(&c.bar[b], parity))) {
          if (globaltimer() - t0 > p.timeout_ns) break;
        }
        c.cnt[NSLOT + 1 + b] += 1;
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
  void* alloc[16];
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

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

static void* halloc(mkx_handle* h, size_t bytes, cudaError_t* err) {
  void* p = nullptr;
  *err = cudaMalloc(&p, bytes);
  if (*err == cudaSuccess) h->alloc[h->nalloc++] = p;
  return p;
}

struct Layout {
  int s_slot[NSLOT];
  int s_u, s_p, s_x, s_res, s_red, s_bar, s_cnt, total;
  int max_rows_qkv, max_rows_h, max_rows_gu;
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
  ly.s_slot[S_D] = take(ly.max_rows_h * I * 2);
  const int xbytes = TP * XS * 2;
  ly.s_u = take(xbytes > TAIL_BYTES ? xbytes : TAIL_BYTES);
  ly.s_p = take(NW * 256 * 4 > (32 * 64 + 32) * 4 ? NW * 256 * 4 : (32 * 64 + 32) * 4);
  ly.s_x = take(TP * 32 * 4);
  ly.s_res = take(TP * RESW * 4);
  ly.s_red = take(64 * 4);
  ly.s_bar = take((NSLOT + 1) * 8);
  ly.s_cnt = take(2 * (NSLOT + 1) * 4);
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
  MKX_CUDA(cudaSetDevice(device));
  int sms = 0, smem_optin = 0;
  MKX_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  MKX_CUDA(cudaDeviceGetAttribute(&smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  const int G = d.grid > 0 ? d.grid : sms;
  if (G < d.A || G > H / 2 || G > sms) return MKX_ERR_RESOURCES;
  if (min_part(d.I / 2, G) < 1) return MKX_ERR_RESOURCES;
  const Layout ly = make_layout(d.I, G);
  if (ly.max_rows_qkv > 128 || ly.max_rows_h > RESW || ly.max_rows_gu > 64) return MKX_ERR_RESOURCES;
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
  float* tailw = err == cudaSuccess ? (float*)halloc(h, TAIL_BYTES, &err) : nullptr;
  float* wout = err == cudaSuccess ? (float*)halloc(h, (size_t)A * H * 4, &err) : nullptr;
  const int rw[NBUF] = {QKVWORDS, HWORDS, HWORDS, HWORDS, HWORDS, HWORDS, I / 2, HWORDS};
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
  pack_kernel<<<blocks, 256, 0, st>>>(w->wd, nullptr, wp[S_D], L, H, I, G, 1);
  norm_kernel<<<(3 * L * HD + 255) / 256, 256, 0, st>>>(w->qn, w->kn, w->qcan, nrm, L);
  // tail weights: wout rows 0..7 | win rows 0..7 | bin | bout (padded to 32)
  cudaMemsetAsync(tailw, 0, TAIL_BYTES, st);
  cudaMemcpyAsync(tailw, w->wout, (size_t)AO * H * 4, cudaMemcpyDeviceToDevice, st);
  cudaMemcpyAsync(tailw + AO * H, w->win, (size_t)AO * H * 4, cudaMemcpyDeviceToDevice, st);
  cudaMemcpyAsync(tailw + 2 * AO * H, w->bin, (size_t)H * 4, cudaMemcpyDeviceToDevice, st);
  cudaMemcpyAsync(tailw + 2 * AO * H + H, w->bout, (size_t)A * 4, cudaMemcpyDeviceToDevice, st);
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
  if ((err = set_smem_attr<uint16_t>(ly.total)) != cudaSuccess || (err = set_smem_attr<float>(ly.total)) != cudaSuccess) {
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
  p.s_u = ly.s_u; p.s_p = ly.s_p; p.s_x = ly.s_x; p.s_res = ly.s_res;
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
  if (in->mem_rows < 1 || in->mem_rows > 32 * MAXK || in->ca_rows < 1) return MKX_ERR_UNSUPPORTED;
  if (in->mem_row_stride < H || in->mem_row_stride % 8 || in->ca_row_stride < H || in->ca_row_stride % 8)
    return MKX_ERR_INVALID_ARG;
  if (!aligned16(in->sa_cos) || !aligned16(in->sa_sin) || !aligned16(in->ca_cos) || !aligned16(in->ca_sin) ||
      ((uintptr_t)in->mods & 7u))
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
  MKX_CUDA(cudaSetDevice(h->device));
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
  MKX_CUDA(cudaSetDevice(h->device));
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

extern "C" mkx_status mkx_launch_shape(const mkx_handle* h, int* grid, int* smem_bytes) {
  if (!h) return MKX_ERR_INVALID_ARG;
  if (grid) *grid = h->G;
  if (smem_bytes) *smem_bytes = h->smem;
  return MKX_OK;
}

extern "C" void mkx_destroy(mkx_handle* h) {
  if (!h) return;
  cudaSetDevice(h->device);
  for (int i = 0; i < h->nalloc; ++i) cudaFree(h->alloc[i]);
  delete h;
}
