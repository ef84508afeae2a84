// Episode-batch path of REKI's action expert on sm_100a (include/mkx_batch.h): B episodes' action
// rows stacked into M = B * T token rows, every weight byte streamed once per Euler step for all.
//
// Per layer and Euler step (src/mk_expert.py:342-421 per episode):
//   adarms(SA) -> gemm QKV -> attention SA -> gemm O (+ gated residual, in place on h)
//   adarms(CA) -> gemm CA query -> attention CA -> gemm CA out (+ gated residual)
//   adarms(MLP) -> gemm gate/up (+ SiLU-mul) -> gemm down (+ gated residual)
// then the step tail per episode (src/mk_expert.py:254-299).
//
// GEMM (swap-AB, tcgen05): D[128 features x ntok tokens] = W_tile[128 x K] . X[ntok x K]^T, one CTA per
// (feature tile, token tile, K split). Warp 0 streams the W tile (packed at create time into
// 128-byte-swizzled, tile-contiguous 16 KB blocks: one bulk copy each) and the token rows (TMA with
// the same swizzle) into an mbarrier ring; warp 1 issues tcgen05.mma kind::f16 (M 128, N ntok, K 16)
// into a TMEM accumulator; warps 2-5 read it back (tcgen05.ld) into a transposed fp32 tile in the
// drained ring; then all six warps run the epilogue with 4-byte coalesced stores. A GEMM with too few
// tiles to cover the SMs splits K over a thread-block cluster of up to 8 CTAs: each keeps its fp32
// partial tile in shared memory, and after a cluster barrier every CTA adds one slice of token rows
// over the cluster (distributed shared memory, split order) and runs the epilogue on it. Up to 128
// token rows the split depends only on the GEMM's shape, so a row's result does not depend on the
// other rows of the launch. The W stream
// does not depend on the previous kernel, so each GEMM is launched as a programmatic dependent: its
// producer starts the W copies before griddepcontrol.wait and only the token-row loads wait for the
// previous kernel. Every wait on an mbarrier is bounded by %globaltimer; after a timeout the CTA
// records the error, drains its copies and MMAs, frees TMEM and returns.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <new>

#include "mkx.h"
#include "mkx_batch.h"
#include "mkx_device.cuh"
#include "mkx_tma.cuh"

namespace mkxb {
using namespace mkx;

constexpr int H = 768, NH = 12, HD = 64, AO = 8, TPMAX = 16;
constexpr int BM = 128, BK = 64, MAXN = 256, MAX_STAGES = 8, GEMM_THREADS = 192;
constexpr int A_BYTES = BM * BK * 2;
constexpr int SMEM_BUDGET = 227 * 1024;
constexpr int TS = BM + 4;  // transposed accumulator tile: floats per token row
constexpr int MAX_SPLITS = 8;  // K splits of one GEMM tile: the last CTA of a tile reads them all back
constexpr int SMALL_M = 128;   // token rows up to which a GEMM is one token tile with a shape-fixed K split
enum Epi { E_STORE = 0, E_GATED = 1, E_GU = 2 };
enum Gemm { G_QKV = 0, G_O, G_CAQ, G_OCA, G_GU, G_D, NGEMM };

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// thread-block clusters: rank, barrier (release / acquire: shared-memory writes before it are visible
// to the cluster after it), and loads from another CTA's shared memory
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_cluster(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr)
               : "memory");
  return v;
}

struct GemmParams {
  const uint16_t* wpk;      // this layer's W tiles: [ntiles][ktiles] blocks of A_BYTES
  int ktiles, kps, splits;  // k tiles in all, per split, splits
  int ntok, M, T, stages, epi, ttiles, tmem_cols;
  uint16_t* out;            // bf16 [M][ldo]
  int ldo;
  const uint16_t* gate;     // E_GATED: gate of episode e, feature f at gate[e * gate_stride + f]
  long long gate_stride;
  int* status;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity, unsigned long long limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > limit) return false;
  return true;
}

extern __shared__ __align__(1024) char bsmem[];

__global__ void __launch_bounds__(GEMM_THREADS, 1) bt_gemm(const __grid_constant__ CUtensorMap tb,
                                                           const __grid_constant__ GemmParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, ttile = blockIdx.y, split = blockIdx.z, tok0 = ttile * p.ntok;
  const int kt0 = split * p.kps, kt1 = min(p.ktiles, kt0 + p.kps), nk = kt1 - kt0;
  const int stage_bytes = A_BYTES + p.ntok * BK * 2;  // a multiple of 1024
  char* ring = bsmem + ((1024u - (smem_u32(bsmem) & 1023u)) & 1023u);
  const int STAGES = p.stages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + STAGES * stage_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + MAX_STAGES;
  uint64_t* done = bars + 2 * MAX_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * MAX_STAGES + 1);
  int* consumed_slot = reinterpret_cast<int*>(tmem_slot + 1);
  // E_GATED: the tile's residual rows [ntok][BM] bf16, prefetched by the epilogue warps during the
  // mainloop (the ring is reused for the accumulator tile, so they live past it)
  uint16_t* res_s = reinterpret_cast<uint16_t*>(reinterpret_cast<char*>(bars) + 256);
  const bool pre_res = p.epi == E_GATED;

  int issued = 0;  // producer (thread 0)
  const uint16_t* wsrc = p.wpk + (size_t)tile * p.ktiles * (A_BYTES / 2);
  const int pre = nk < STAGES ? nk : STAGES;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *consumed_slot = 0;
    fence_mbar_init();
    // the W tiles of the first stages need nothing from the previous kernel: they go out before the
    // TMEM allocation and the block barrier
    const uint64_t pol = l2_evict_first();
    for (int i = 0; i < pre; ++i) {
      mbar_expect_tx(&full[i], (uint32_t)stage_bytes);
      bulk_g2s_hint(ring + i * stage_bytes, wsrc + (size_t)(kt0 + i) * (A_BYTES / 2), (uint32_t)A_BYTES, &full[i], pol);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, (uint32_t)p.tmem_cols);
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) grid_dep_launch();  // the next kernel's CTAs may take free SMs and start their W

  if (warp == 0 && lane == 0) {
    // producer
    const uint64_t pol = l2_evict_first();
    grid_dep_wait();  // the token rows are the previous kernel's output
    for (int i = 0; i < nk; ++i) {
      const int s = i % STAGES, kb = kt0 + i;
      char* a = ring + s * stage_bytes;
      if (i >= STAGES) {
        if (!wait_bounded(&empty[s], ((i / STAGES) & 1) ^ 1, p.timeout_ns)) {
          atomicCAS(p.status, 0, 0x200 | 1);
          break;
        }
        mbar_expect_tx(&full[s], (uint32_t)stage_bytes);
        bulk_g2s_hint(a, wsrc + (size_t)kb * (A_BYTES / 2), (uint32_t)A_BYTES, &full[s], pol);
      }
      tma_load_2d(a + A_BYTES, &tb, kb * BK, tok0, &full[s]);
      issued = i + 1;
    }
    if (issued < pre) issued = pre;  // the W copies of the first stages were issued in any case
  } else if (warp == 1 && lane == 0) {
    const uint32_t idesc = umma_idesc(BM, p.ntok);
    int i = 0;
    for (; i < nk; ++i) {
      const int s = i % STAGES;
      if (!wait_bounded(&full[s], (i / STAGES) & 1, p.timeout_ns)) {
        atomicCAS(p.status, 0, 0x200 | 2);
        break;
      }
      tmem_fence_after();
      const uint32_t a = smem_u32(ring + s * stage_bytes), b = a + A_BYTES;
#pragma unroll
      for (int k = 0; k < BK / 16; ++k)
        umma_bf16(tmem, sw128_desc(a + 32 * k), sw128_desc(b + 32 * k), idesc, (i | k) != 0 ? 1u : 0u);
      umma_commit(&empty[s]);
    }
    *consumed_slot = i;
    umma_commit(done);
  }
  // accumulator -> transposed fp32 tile [token][feature] in the drained ring (warps 2-5)
  float* tsm = reinterpret_cast<float*>(ring);
  bool ok = true;
  if (warp >= 2) {
    if (pre_res) {
      grid_dep_wait();  // the residual is an earlier kernel's output
      const int nvr = min(p.ntok, p.M - tok0);
      for (int c = threadIdx.x - 64; c < nvr * (BM / 8); c += GEMM_THREADS - 64) {
        const int tl = c / (BM / 8), q = c % (BM / 8);
        cp_async16(res_s + tl * BM + 8 * q, p.out + (size_t)(tok0 + tl) * p.ldo + tile * BM + 8 * q);
      }
      cp_async_commit();
    }
    ok = __all_sync(0xffffffffu, wait_bounded(done, 0, p.timeout_ns));
    if (!ok && lane == 0) atomicCAS(p.status, 0, 0x200 | 3);
    tmem_fence_after();
    const int q = warp & 3, r = 32 * q + lane;
    if (ok) {
      for (int c0 = 0; c0 < p.ntok; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) tsm[(c0 + j) * TS + r] = __uint_as_float(v[j]);
      }
    }
    if (pre_res) cp_async_wait<0>();
    tmem_fence_before();
  }
  ok = __syncthreads_and(ok);
  const int nv = min(p.ntok, p.M - tok0);   // valid token rows of this tile
  // split K: the splits of one tile form a thread-block cluster; each holds its fp32 partial tile in
  // its own shared memory. After a cluster barrier CTA r sums rows [r0, r1) of every partial, in split
  // order (the same order in every CTA: deterministic), into its own tile -- no other CTA reads those
  // rows from it -- and runs the epilogue on them; a second barrier before exit keeps every tile
  // readable until the whole cluster is done with it.
  int r0 = 0, r1 = nv;
  if (p.splits > 1) {
    const int per = (nv + p.splits - 1) / p.splits;
    r0 = min(nv, (int)cluster_ctarank() * per);
    r1 = min(nv, r0 + per);
    cluster_sync();
    const uint32_t base = smem_u32(tsm);
    for (int i = threadIdx.x; i < (r1 - r0) * (BM / 4); i += GEMM_THREADS) {
      const int tl = r0 + i / (BM / 4), c = i % (BM / 4);
      const uint32_t off = (uint32_t)(tl * TS + 4 * c) * 4u;
      float4 acc = ld_cluster_f4(map_cluster(base + off, 0));
      for (int z = 1; z < p.splits; ++z) {
        const float4 t = ld_cluster_f4(map_cluster(base + off, (uint32_t)z));
        acc.x += t.x;
        acc.y += t.y;
        acc.z += t.z;
        acc.w += t.w;
      }
      *reinterpret_cast<float4*>(tsm + tl * TS + 4 * c) = acc;
    }
    __syncthreads();
  }
  if (ok) {
    if (p.epi == E_GU) {
      // rows 0..63 of the tile are gate rows, 64..127 the up rows of the same 64 columns:
      // g = bf16(silu(bf16(gate)) * bf16(up)) (src/mk_expert.py:403-413)
      for (int i = threadIdx.x; i < (r1 - r0) * 32; i += GEMM_THREADS) {
        const int tl = r0 + (i >> 5), cp = i & 31;
        const float2 gt = *reinterpret_cast<const float2*>(tsm + tl * TS + 2 * cp);
        const float2 up = *reinterpret_cast<const float2*>(tsm + tl * TS + 64 + 2 * cp);
        const float g0 = round_bf(gt.x), g1 = round_bf(gt.y);
        const float o0 = __fdividef(g0, 1.f + __expf(-g0)) * round_bf(up.x);
        const float o1 = __fdividef(g1, 1.f + __expf(-g1)) * round_bf(up.y);
        *reinterpret_cast<uint32_t*>(p.out + (size_t)(tok0 + tl) * p.ldo + tile * 64 + 2 * cp) = pack_bf2(o0, o1);
      }
    } else {
      // items (token tl, feature pair fp), 8 per thread per round: every load of a round is issued
      // before its stores, so the round costs one memory latency, not eight
      constexpr int U = 8;
      const int n = (r1 - r0) * (BM / 2);
      for (int base = threadIdx.x; base < n; base += GEMM_THREADS * U) {
        float2 v[U];
        uint32_t rv[U], gv[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
          const int i = base + GEMM_THREADS * k;
          rv[k] = gv[k] = 0u;
          v[k] = make_float2(0.f, 0.f);
          if (i < n) {
            const int tl = r0 + i / (BM / 2), fp = i % (BM / 2);
            const int m = tok0 + tl, f = tile * BM + 2 * fp;
            v[k] = *reinterpret_cast<const float2*>(tsm + tl * TS + 2 * fp);
            if (p.epi == E_GATED) {
              rv[k] = *reinterpret_cast<const uint32_t*>(res_s + tl * BM + 2 * fp);
              gv[k] = __ldg(reinterpret_cast<const unsigned int*>(p.gate + (size_t)(m / p.T) * p.gate_stride + f));
            }
          }
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
          const int i = base + GEMM_THREADS * k;
          if (i >= n) break;
          const int tl = r0 + i / (BM / 2), fp = i % (BM / 2);
          const int m = tok0 + tl, f = tile * BM + 2 * fp;
          uint32_t* dst = reinterpret_cast<uint32_t*>(p.out + (size_t)m * p.ldo + f);
          if (p.epi == E_STORE)
            *dst = pack_bf2(v[k].x, v[k].y);
          else  // gated residual bf16(res + bf16(acc) * gate) (src/mk_expert.py:162-172), in place
            *dst = pack_bf2(fmaf(round_bf(v[k].x), bf_lo(gv[k]), bf_lo(rv[k])),
                            fmaf(round_bf(v[k].y), bf_hi(gv[k]), bf_hi(rv[k])));
        }
      }
    }
  }
  if (p.splits > 1) cluster_sync();  // no CTA leaves while another may still read its partial tile
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = *consumed_slot; i < issued; ++i)
      if (!wait_bounded(&full[i % STAGES], (i / STAGES) & 1, p.timeout_ns)) break;
  }
  if (warp == 1) {
    wait_bounded(done, 0, p.timeout_ns);
    tmem_fence_after();
    tmem_free(tmem, (uint32_t)p.tmem_cols);
  }
}

// ---------------------------------------------------------------------------------------------
// AdaRMS (src/mk_expert.py:93-122): a[m] = bf16(h[m] * rstd_m * (1 + scale_e) + shift_e), one warp per
// token row (lane: columns 8 (lane + 32 i) .. + 7); rows >= M are zero. mods_blk: [scale H | shift H]
// of the block for episode 0, episodes ep_stride apart.
__global__ void __launch_bounds__(256) bt_adarms(const uint16_t* __restrict__ h, uint16_t* __restrict__ a, int M, int Mp,
                                                 int T, const uint16_t* __restrict__ mods_blk, long long ep_stride,
                                                 float eps) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + warp;
  uint4 v[3], s4[3], h4[3];
  if (row < M) {  // the modulation rows are inputs of the launch sequence: read before the wait
    const uint16_t* sc = mods_blk + (size_t)(row / T) * ep_stride;
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      s4[i] = __ldg(reinterpret_cast<const uint4*>(sc) + lane + 32 * i);
      h4[i] = __ldg(reinterpret_cast<const uint4*>(sc + H) + lane + 32 * i);
    }
  }
  grid_dep_wait();
  if (threadIdx.x == 0) grid_dep_launch();
  if (row >= Mp) return;
  uint4* dst = reinterpret_cast<uint4*>(a + (size_t)row * H);
  if (row >= M) {
#pragma unroll
    for (int i = 0; i < 3; ++i) dst[lane + 32 * i] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(h + (size_t)row * H);
#pragma unroll
  for (int i = 0; i < 3; ++i) v[i] = src[lane + 32 * i];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) ss = fmaf(bf_lo(w[k]), bf_lo(w[k]), fmaf(bf_hi(w[k]), bf_hi(w[k]), ss));
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = rsqrtf(ss / (float)H + eps);
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
    const uint32_t s[4] = {s4[i].x, s4[i].y, s4[i].z, s4[i].w};
    const uint32_t t[4] = {h4[i].x, h4[i].y, h4[i].z, h4[i].w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      o[k] = pack_bf2(fmaf(bf_lo(w[k]) * rstd, 1.f + bf_lo(s[k]), bf_lo(t[k])),
                      fmaf(bf_hi(w[k]) * rstd, 1.f + bf_hi(s[k]), bf_hi(t[k])));
    dst[lane + 32 * i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------------------------------------
constexpr int SA_MAXK = 320;          // memory rows + own rows (<= 256 + 16), whole 64-key blocks
constexpr int CA_BLK = 64;
constexpr int CA_ALL_ROWS = 3 * CA_BLK;  // padded source rows up to which CA stages all of them at once
constexpr int CA_ALL_UNITS_PER_SM = 4;     // ... while there are at most this many (episode, head) units per SM
constexpr int KS = 72;                // shared row stride (bf16) of the Q / K / V tiles: ldmatrix rows of
                                      // 144 bytes fall in distinct bank quadruples

// Warp-wide: norm + RoPE of one head row held as dims (2 lane, 2 lane + 1) in x0, x1; returns the
// rotated bf16-rounded values (partner dims d +- 32 live in lane ^ 16).
__device__ __forceinline__ float2 norm_rope_row(float x0, float x1, float2 w, float2 cs, float2 sn, float eps, int lane) {
  float ss = fmaf(x0, x0, x1 * x1);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)HD + eps);
  const float n0 = round_bf(x0 * r * w.x), n1 = round_bf(x1 * r * w.y);
  const float p0 = __shfl_xor_sync(0xffffffffu, n0, 16), p1 = __shfl_xor_sync(0xffffffffu, n1, 16);
  const float sg = lane < 16 ? -1.f : 1.f;
  return make_float2(round_bf(fmaf(n0, cs.x, sg * p0 * sn.x)), round_bf(fmaf(n1, cs.y, sg * p1 * sn.y)));
}

__device__ __forceinline__ void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
// Scores of the 16 query rows against the 16 keys at shared rows [k0, k0 + 16) of Ks: two n8 tiles (c[nt]:
// keys 8 nt + 2 cc, +1 of rows g and g + 8, unscaled). The B operand K^T comes from K rows by ldmatrix.
__device__ __forceinline__ void scores16(const uint32_t (&qa)[4][4], const uint16_t* Ks, int k0, int lane,
                                         float (&c)[2][4]) {
  const int mat = lane >> 3, r = lane & 7;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) c[nt][0] = c[nt][1] = c[nt][2] = c[nt][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
    uint32_t b0, b1, b2, b3;
    ldsm_x4(Ks + (size_t)(k0 + 8 * (mat >> 1) + r) * KS + 16 * ks + 8 * (mat & 1), b0, b1, b2, b3);
    mma_bf16(c[0], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b0, b1);
    mma_bf16(c[1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], b2, b3);
  }
}

// o += P V over the 16 keys [k0, k0 + 16): P (bf16 values in fp32) as the A operand, V by ldmatrix.trans.
__device__ __forceinline__ void pv16(const float (&pc)[2][4], const uint16_t* Vs, int k0, int lane, float (&o)[8][4]) {
  const int mat = lane >> 3, r = lane & 7;
  const uint32_t a0 = pack_bf2(pc[0][0], pc[0][1]), a1 = pack_bf2(pc[0][2], pc[0][3]);
  const uint32_t a2 = pack_bf2(pc[1][0], pc[1][1]), a3 = pack_bf2(pc[1][2], pc[1][3]);
#pragma unroll
  for (int dp = 0; dp < 4; ++dp) {
    uint32_t b0, b1, b2, b3;
    ldsm_x4_t(Vs + (size_t)(k0 + 8 * (mat & 1) + r) * KS + 16 * dp + 8 * (mat >> 1), b0, b1, b2, b3);
    mma_bf16(o[2 * dp], a0, a1, a2, a3, b0, b1);
    mma_bf16(o[2 * dp + 1], a0, a1, a2, a3, b2, b3);
  }
}

// Attention of one (episode, head), one warp. Per-head RMSNorm (weight 1 + w) then rotate-half RoPE with
// a bf16 rounding after each (src/mk_expert.py:175-193) on the queries (and, SA, the action rows' own
// keys); scores and P V on tensor cores (mma.sync m16n8k16, bf16 in, fp32 accumulate: the products of
// bf16 values are exact, as in the reference's fp32 dot products). SA (src/mk_expert.py:196-222): one
// softmax over the memory rows [kv_start, PM) and the T own rows, P rounded to bf16 against the max over
// all keys (two passes over the keys). CA (src/mk_expert.py:225-251): online softmax over the S source
// rows in 64-row blocks (the next block's copy in flight during the current one). y = bf16(o / den).
struct AttnParams {
  const uint16_t* src;   // SA: qkv [Mp][3H]; CA: q [Mp][H]
  int src_ld;
  uint16_t* y;           // [Mp][H]
  const uint16_t* kb;    // this layer's K rows of episode 0: [rows][NH][HD], episodes kv_ep apart
  const uint16_t* vb;
  long long kv_ep;
  int kv_rows;           // PM (SA) or SP (CA)
  const int* lim;        // SA: kv_start[B]; CA: S[B]
  const float* cos;      // [B][T][HD]
  const float* sin;
  const float* wq;       // [HD] 1 + q norm weight (SA q / CA q)
  const float* wk;       // [HD] 1 + k norm weight (SA own keys)
  int T;
  int kcap;              // key rows of the shared K / V tiles: SA PM + T rounded up to 64; CA 2 blocks, or
                         // the whole padded source (ca_all) when it has at most CA_ALL_ROWS rows
  int own;               // SA: 1 the query rows' own keys follow the memory rows; 0 memory rows only
  int kv_input;          // 1: K / V and lim were in memory before the launch sequence (staged early)
  int ca_all;            // CA: 1 = the whole padded source (kcap rows) staged at once
  int lim_stride;        // episode stride of lim (0: one value for all episodes)
  // SA, register pass: the memory rows [frame_row0, kv_rows) are this layer's frame, the K (per-head
  // norm + RoPE) and V of the frame_rows rows of src, computed here: placed after the older rows in
  // shared memory, and written to the memory (mk_out / mv_out, episode e writes its own T rows).
  // frame_row0 < 0: none.
  int frame_row0, frame_rows;
  uint16_t* mk_out;
  uint16_t* mv_out;
  float qk_eps, scale;
};

constexpr int ATT_WARPS = 4;
constexpr int OPS = HD + 4;  // floats per row of a warp's partial attention output

template <bool SA>
__global__ void __launch_bounds__(32 * ATT_WARPS) bt_attention(const __grid_constant__ AttnParams p) {
  // K / V (and the row limits) that were in memory before the launch sequence began are staged before
  // waiting for the previous kernel; K / V a kernel of the sequence writes, after
  if (!p.kv_input) grid_dep_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, cc = lane & 3, T = p.T;
  extern __shared__ __align__(16) char asmem[];
  __shared__ float st_s[ATT_WARPS][16][2];  // per warp and query row: softmax max, sum
  const int e = blockIdx.x / NH, h = blockIdx.x % NH;
  uint16_t* Qs = reinterpret_cast<uint16_t*>(asmem);             // [16][KS]
  uint16_t* Ks = Qs + 16 * KS;                                    // SA: [SA_MAXK][KS]; CA: [2][64][KS]
  // CA with kcap > 2 blocks: every source row staged at once (no double buffering)
  const bool ca_all = !SA && p.ca_all;
  uint16_t* Vs = Ks + ((SA || ca_all) ? p.kcap : 2 * CA_BLK) * KS;
  const uint16_t* kb = p.kb + (size_t)e * p.kv_ep + h * HD;
  const uint16_t* vb = p.vb + (size_t)e * p.kv_ep + h * HD;
  const uint32_t zero = 0u;
  // key rows [k0, k0 + nrows) of K and V into shared rows [dst, dst + nrows) (asynchronous copies)
  auto stage = [&](int k0, int nrows, int dst, int t0, int nt) {
    for (int c = t0; c < nrows * 8; c += nt) {
      const int j = c >> 3, q = c & 7;
      cp_async16(Ks + (size_t)(dst + j) * KS + 8 * q, kb + (size_t)(k0 + j) * H + 8 * q);
      cp_async16(Vs + (size_t)(dst + j) * KS + 8 * q, vb + (size_t)(k0 + j) * H + 8 * q);
    }
  };
  auto zero_rows = [&](int r0, int r1, int t0, int nt) {  // padding keys: finite zeros (0 x V must stay 0)
    for (int c = t0; c < (r1 - r0) * 32; c += nt) {
      const int j = r0 + (c >> 5), q = c & 31;
      reinterpret_cast<uint32_t*>(Ks + (size_t)j * KS)[q] = zero;
      reinterpret_cast<uint32_t*>(Vs + (size_t)j * KS)[q] = zero;
    }
  };
  int nm = 0, nk = 0, S = 0, k0 = 0;
  const bool frame = SA && p.frame_row0 >= 0;
  if (SA) {
    k0 = min(max(p.lim[e * p.lim_stride], 0), p.kv_rows);
    nm = p.kv_rows - k0;
    nk = nm + (p.own ? T : 0);
    stage(k0, frame ? max(p.frame_row0 - k0, 0) : nm, 0, tid, 32 * ATT_WARPS);  // rows written before the sequence
    zero_rows(nk, (nk + CA_BLK - 1) / CA_BLK * CA_BLK, tid, 32 * ATT_WARPS);
  } else {
    S = min(max(p.lim[e * p.lim_stride], 1), p.kv_rows);
    const int nb = ca_all ? S : min(CA_BLK, S);
    stage(0, nb, 0, tid, 32 * ATT_WARPS);
    zero_rows(nb, ca_all ? (S + CA_BLK - 1) / CA_BLK * CA_BLK : CA_BLK, tid, 32 * ATT_WARPS);
  }
  cp_async_commit();
  if (p.kv_input) grid_dep_wait();  // the queries are the previous kernel's output
  if (tid == 0) grid_dep_launch();
  // queries (and SA own keys / values), bf16, rows >= T zero: warp w takes rows w, w + 4, ...; every
  // global load of the warp's rows goes out before the first row's arithmetic (one L2 round trip)
  constexpr int QR = 16 / ATT_WARPS;
  {
    uint32_t qu[QR], ku[QR], vu[QR];
    float2 cs[QR], sn[QR];
#pragma unroll
    for (int j = 0; j < QR; ++j) {
      const int t = warp + ATT_WARPS * j;
      if (t < T) {
        const size_t m = (size_t)e * T + t;
        cs[j] = *reinterpret_cast<const float2*>(p.cos + m * HD + 2 * lane);
        sn[j] = *reinterpret_cast<const float2*>(p.sin + m * HD + 2 * lane);
        const uint16_t* row = p.src + m * p.src_ld + h * HD;
        qu[j] = *reinterpret_cast<const uint32_t*>(row + 2 * lane);
        if (SA && p.own) {
          ku[j] = *reinterpret_cast<const uint32_t*>(row + H + 2 * lane);
          vu[j] = *reinterpret_cast<const uint32_t*>(row + 2 * H + 2 * lane);
        }
      }
    }
    const float2 wq = *reinterpret_cast<const float2*>(p.wq + 2 * lane);
#pragma unroll
    for (int j = 0; j < QR; ++j) {
      const int t = warp + ATT_WARPS * j;
      uint32_t qv = 0u;
      if (t < T) {  // warp-uniform: the norm's shuffles need all lanes
        const float2 q = norm_rope_row(bf_lo(qu[j]), bf_hi(qu[j]), wq, cs[j], sn[j], p.qk_eps, lane);
        qv = pack_bf2(q.x, q.y);
        if (SA && p.own) {
          const float2 k = norm_rope_row(bf_lo(ku[j]), bf_hi(ku[j]), *reinterpret_cast<const float2*>(p.wk + 2 * lane),
                                         cs[j], sn[j], p.qk_eps, lane);
          reinterpret_cast<uint32_t*>(Ks + (size_t)(nm + t) * KS)[lane] = pack_bf2(k.x, k.y);
          reinterpret_cast<uint32_t*>(Vs + (size_t)(nm + t) * KS)[lane] = vu[j];
        }
      }
      reinterpret_cast<uint32_t*>(Qs + (size_t)t * KS)[lane] = qv;
    }
  }
  if (frame) {  // the frame's K / V from the QKV output (same rounding as the action rows' own keys)
    constexpr int FU = 8;  // rows per warp and round, loaded before any is processed
    const float2 wk = *reinterpret_cast<const float2*>(p.wk + 2 * lane);
    for (int m0 = warp; m0 < p.frame_rows; m0 += ATT_WARPS * FU) {
      uint32_t ku[FU], vu[FU];
      float2 cs[FU], sn[FU];
#pragma unroll
      for (int j = 0; j < FU; ++j) {
        const int m = m0 + ATT_WARPS * j;
        if (m < p.frame_rows) {
          const uint16_t* row = p.src + (size_t)m * p.src_ld + h * HD;
          ku[j] = *reinterpret_cast<const uint32_t*>(row + H + 2 * lane);
          vu[j] = *reinterpret_cast<const uint32_t*>(row + 2 * H + 2 * lane);
          cs[j] = *reinterpret_cast<const float2*>(p.cos + (size_t)m * HD + 2 * lane);
          sn[j] = *reinterpret_cast<const float2*>(p.sin + (size_t)m * HD + 2 * lane);
        }
      }
#pragma unroll
      for (int j = 0; j < FU; ++j) {
        const int m = m0 + ATT_WARPS * j;
        if (m < p.frame_rows) {  // warp-uniform
          const float2 k = norm_rope_row(bf_lo(ku[j]), bf_hi(ku[j]), wk, cs[j], sn[j], p.qk_eps, lane);
          const uint32_t kv = pack_bf2(k.x, k.y);
          const int r = p.frame_row0 + m;
          if (r >= k0) {
            reinterpret_cast<uint32_t*>(Ks + (size_t)(r - k0) * KS)[lane] = kv;
            reinterpret_cast<uint32_t*>(Vs + (size_t)(r - k0) * KS)[lane] = vu[j];
          }
          if (m / T == e) {
            *reinterpret_cast<uint32_t*>(p.mk_out + (size_t)r * H + h * HD + 2 * lane) = kv;
            *reinterpret_cast<uint32_t*>(p.mv_out + (size_t)r * H + h * HD + 2 * lane) = vu[j];
          }
        }
      }
    }
  }
  // Every warp takes the 16-key slice [64 b + 16 warp, + 16) of each 64-key block b, with its own
  // softmax statistics (rows g and g + 8 of the quad's lanes); the warps' partial results are merged
  // at the end. SA: the max over all keys first, then P = bf16(exp(s - max)) against it (the
  // reference's two passes); CA: an online softmax over the warp's slices, the blocks double-buffered
  // in shared memory with the next block's copy in flight.
  uint32_t qa[4][4];
  float o[8][4];
#pragma unroll
  for (int dn = 0; dn < 8; ++dn) o[dn][0] = o[dn][1] = o[dn][2] = o[dn][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  float c[2][4];
  auto load_q = [&]() {
    const int mat = lane >> 3, r = lane & 7;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
      ldsm_x4(Qs + (size_t)(r + 8 * (mat & 1)) * KS + 16 * ks + 8 * (mat >> 1), qa[ks][0], qa[ks][1], qa[ks][2],
              qa[ks][3]);
  };
  auto quad_max = [&](float& a, float& b) {
#pragma unroll
    for (int x = 1; x <= 2; x <<= 1) {
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, x));
      b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, x));
    }
  };
  if (SA) {
    cp_async_wait<0>();
    __syncthreads();
    load_q();
    const int nblk = (nk + CA_BLK - 1) / CA_BLK;
    for (int b = 0; b < nblk; ++b) {  // pass 1: the max of the warp's slices
      const int k0 = b * CA_BLK + 16 * warp;
      if (k0 >= nk) break;
      scores16(qa, Ks, k0, lane, c);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const bool ok = k0 + 8 * nt + 2 * cc + i < nk;
          m0 = fmaxf(m0, ok ? c[nt][i] * p.scale : -INFINITY);
          m1 = fmaxf(m1, ok ? c[nt][2 + i] * p.scale : -INFINITY);
        }
    }
    quad_max(m0, m1);
    if (cc == 0) {
      st_s[warp][g][0] = m0;
      st_s[warp][g + 8][0] = m1;
    }
    __syncthreads();
#pragma unroll
    for (int w = 0; w < ATT_WARPS; ++w) {  // the max over all keys
      m0 = fmaxf(m0, st_s[w][g][0]);
      m1 = fmaxf(m1, st_s[w][g + 8][0]);
    }
    for (int b = 0; b < nblk; ++b) {  // pass 2: P = bf16(exp(s - max)), P V and the sums
      const int k0 = b * CA_BLK + 16 * warp;
      if (k0 >= nk) break;
      scores16(qa, Ks, k0, lane, c);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const bool ok = k0 + 8 * nt + 2 * cc + i < nk;
          const float p0 = ok ? __expf(c[nt][i] * p.scale - m0) : 0.f;
          const float p1 = ok ? __expf(c[nt][2 + i] * p.scale - m1) : 0.f;
          l0 += p0;
          l1 += p1;
          c[nt][i] = round_bf(p0);
          c[nt][2 + i] = round_bf(p1);
        }
      pv16(c, Vs, k0, lane, o);
    }
  } else {
    const int nblk = (S + CA_BLK - 1) / CA_BLK;
    for (int b = 0; b < nblk; ++b) {
      const int buf = ca_all ? b : b & 1;  // shared block of block b
      cp_async_wait<0>();
      __syncthreads();  // block b is in shared memory; every warp is done with block b - 1
      if (b == 0) load_q();
      if (!ca_all && b + 1 < nblk) {  // the next block into the other buffer (last read in block b - 1)
        const int nb = min(CA_BLK, S - (b + 1) * CA_BLK);
        stage((b + 1) * CA_BLK, nb, (buf ^ 1) * CA_BLK, tid, 32 * ATT_WARPS);
        zero_rows((buf ^ 1) * CA_BLK + nb, (buf ^ 1) * CA_BLK + CA_BLK, tid, 32 * ATT_WARPS);
        cp_async_commit();
      }
      const int kg = b * CA_BLK + 16 * warp;  // global key index of the slice
      if (kg >= S) continue;                   // warp-uniform
      scores16(qa, Ks, buf * CA_BLK + 16 * warp, lane, c);
      float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const bool ok = kg + 8 * nt + 2 * cc + i < S;
          c[nt][i] = ok ? c[nt][i] * p.scale : -INFINITY;
          c[nt][2 + i] = ok ? c[nt][2 + i] * p.scale : -INFINITY;
          bm0 = fmaxf(bm0, c[nt][i]);
          bm1 = fmaxf(bm1, c[nt][2 + i]);
        }
      quad_max(bm0, bm1);
      const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
      const float al0 = __expf(m0 - mn0), al1 = __expf(m1 - mn1);  // 0 on the warp's first slice
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float p0 = __expf(c[nt][i] - mn0), p1 = __expf(c[nt][2 + i] - mn1);
          s0 += p0;
          s1 += p1;
          c[nt][i] = round_bf(p0);
          c[nt][2 + i] = round_bf(p1);
        }
      l0 = l0 * al0 + s0;
      l1 = l1 * al1 + s1;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int dn = 0; dn < 8; ++dn) {
        o[dn][0] *= al0;
        o[dn][1] *= al0;
        o[dn][2] *= al1;
        o[dn][3] *= al1;
      }
      pv16(c, Vs, buf * CA_BLK + 16 * warp, lane, o);
    }
  }
  // merge: each warp's (max, sum) and partial output, then y = sum_w o_w e^(m_w - M) / sum_w l_w e^(m_w - M)
#pragma unroll
  for (int x = 1; x <= 2; x <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, x);
    l1 += __shfl_xor_sync(0xffffffffu, l1, x);
  }
  __syncthreads();  // every warp is done with K / V: the partial outputs go over them
  float* Op = reinterpret_cast<float*>(Ks);  // [ATT_WARPS][16][OPS]
  if (cc == 0) {
    st_s[warp][g][0] = m0;
    st_s[warp][g][1] = l0;
    st_s[warp][g + 8][0] = m1;
    st_s[warp][g + 8][1] = l1;
  }
#pragma unroll
  for (int dn = 0; dn < 8; ++dn) {
    const int d = 8 * dn + 2 * cc;
    *reinterpret_cast<float2*>(Op + (warp * 16 + g) * OPS + d) = make_float2(o[dn][0], o[dn][1]);
    *reinterpret_cast<float2*>(Op + (warp * 16 + g + 8) * OPS + d) = make_float2(o[dn][2], o[dn][3]);
  }
  __syncthreads();
  for (int i = tid; i < T * (HD / 2); i += 32 * ATT_WARPS) {  // (row, column pair)
    const int t = i / (HD / 2), d = 2 * (i % (HD / 2));
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < ATT_WARPS; ++w) M = fmaxf(M, st_s[w][t][0]);
    float L = 0.f, y0 = 0.f, y1 = 0.f;
#pragma unroll
    for (int w = 0; w < ATT_WARPS; ++w) {
      const float f = __expf(st_s[w][t][0] - M);  // 0 for a warp without keys (max -inf)
      const float2 v = *reinterpret_cast<const float2*>(Op + (w * 16 + t) * OPS + d);
      L = fmaf(st_s[w][t][1], f, L);
      y0 = fmaf(v.x, f, y0);
      y1 = fmaf(v.y, f, y1);
    }
    *reinterpret_cast<uint32_t*>(p.y + ((size_t)e * T + t) * H + h * HD + d) = pack_bf2(y0 / L, y1 / L);
  }
}

// ---------------------------------------------------------------------------------------------
// Step tail (src/mk_expert.py:254-299), one CTA of 256 threads per action row (episode e, row t):
// o = bf16(AdaRMS_final(h)), v_a = o . Wout[a] + bout[a] (fp32, a < A), x_a <- (a < action_dim ? x_a
// : 0) + dt v_a; the last step writes x_out, the others the next step's h0 = bf16(xpad[:AO] . Win[:AO]
// + bin). first = 1: only the in-projection of x_in (the loop's first h0).
struct TailParams {
  const float* x_in;
  float* xs;           // [B][T][A] running state
  float* x_out;
  uint16_t* h;         // [Mp][H]
  const uint16_t* mfin;  // final-norm [scale | shift] of episode 0 at this step, episodes ep_stride apart
  long long ep_stride;
  const float* dt;
  const float* win;    // [A][H] (rows 0..AO-1 used)
  const float* bin;    // [H]
  const float* wout;   // [A][H]
  const float* bout;   // [A]
  int T, A, adim, first, last;
  float eps;
};

__global__ void __launch_bounds__(256) bt_tail(const __grid_constant__ TailParams p) {
  __shared__ float red[8][32];
  __shared__ float xnew[32];
  __shared__ float ssum[8];
  const int e = blockIdx.x / p.T, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const size_t m = blockIdx.x;  // = e * T + t
  // the final norm's modulation columns are inputs of the launch sequence: read before the wait
  float ms[3], mh[3];
  if (!p.first) {
    const uint16_t* mf = p.mfin + (size_t)e * p.ep_stride;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      ms[k] = bf_at(mf[tid + 256 * k]);
      mh[k] = bf_at(mf[H + tid + 256 * k]);
    }
  }
  grid_dep_wait();
  if (threadIdx.x == 0) grid_dep_launch();
  float* xr = p.xs + m * p.A;
  if (p.first) {
    if (tid < p.A) {
      xnew[tid] = p.x_in[m * p.A + tid];
      xr[tid] = xnew[tid];
    }
  } else {
    // final AdaRMS of row m: thread owns columns tid, tid + 256, tid + 512
    float hv[3], ss = 0.f;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      hv[k] = bf_at(p.h[m * H + tid + 256 * k]);
      ss = fmaf(hv[k], hv[k], ss);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) ssum[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += ssum[w];
    const float rstd = rsqrtf(tot / (float)H + p.eps);
    float o[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) o[k] = round_bf(fmaf(hv[k] * rstd, 1.f + ms[k], mh[k]));
    // v_a for every a < A: per-thread partials over its 3 columns, then warp and block sums; the
    // weights of 8 outputs are loaded before any of them is summed (one L2 round trip per 8)
    for (int a0 = 0; a0 < p.A; a0 += 8) {
      float w[8][3];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (a0 + j < p.A)
#pragma unroll
          for (int k = 0; k < 3; ++k) w[j][k] = p.wout[(a0 + j) * H + tid + 256 * k];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (a0 + j >= p.A) break;  // block-uniform
        float v = o[0] * w[j][0];
        v = fmaf(o[1], w[j][1], v);
        v = fmaf(o[2], w[j][2], v);
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
        if (lane == 0) red[warp][a0 + j] = v;
      }
    }
    __syncthreads();
    if (tid < p.A) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) v += red[w][tid];
      v += p.bout[tid];
      const float xp = tid < p.adim ? xr[tid] : 0.f;
      const float xn = fmaf(p.dt[e], v, xp);
      xnew[tid] = xn;
      xr[tid] = xn;
      if (p.last) p.x_out[m * p.A + tid] = xn;
    }
  }
  if (p.last) return;
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const int col = tid + 256 * k;
    float acc = p.bin[col];
#pragma unroll
    for (int a = 0; a < AO; ++a) acc = fmaf(a < p.adim ? xnew[a] : 0.f, p.win[a * H + col], acc);
    p.h[m * H + col] = __bfloat16_as_ushort(__float2bfloat16_rn(acc));
  }
}

// ---------------------------------------------------------------------------------------------
// Weight packing: rows of a GEMM's [N][K] bf16 weight (gate/up: tile t = 64 gate rows then the 64 up
// rows of columns 64 t ..) into [tile][kb][128 rows x 64] blocks in the 128-byte-swizzled K-major
// order (16-byte chunk c of row r at r * 128 + (c ^ (r % 8)) * 16) the MMA reads.
__global__ void bt_pack_kernel(const uint16_t* __restrict__ w0, const uint16_t* __restrict__ w1, uint16_t* __restrict__ out,
                               int tiles, int ktiles, int K, int gu) {
  const long long total = (long long)tiles * ktiles * BM * 8;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(e & 7), r = (int)((e >> 3) % BM);
    const long long blk = e / (8 * BM);
    const int kb = (int)(blk % ktiles), tile = (int)(blk / ktiles);
    const uint16_t* src = gu ? (r < 64 ? w0 + (size_t)(tile * 64 + r) * K : w1 + (size_t)(tile * 64 + r - 64) * K)
                             : w0 + (size_t)(tile * BM + r) * K;
    const uint4 v = *reinterpret_cast<const uint4*>(src + kb * BK + c * 8);
    *reinterpret_cast<uint4*>(reinterpret_cast<char*>(out) + blk * A_BYTES + r * 128 + ((c ^ (r & 7)) << 4)) = v;
  }
}

__global__ void bt_norm_kernel(const uint16_t* qn, const uint16_t* kn, const uint16_t* qcan, float* out, int L) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= 3 * L * HD) return;
  const int which = e / (L * HD), r = e % (L * HD);
  const uint16_t* s = which == 0 ? qn : (which == 1 ? kn : qcan);
  out[e] = 1.0f + __uint_as_float(((uint32_t)s[r]) << 16);
}

}  // namespace mkxb

// =============================================================================================
using namespace mkxb;

namespace {
struct GemmShape {
  int N, K, ntiles, ktiles, epi;
};

GemmShape gemm_shape(int g, int I) {
  switch (g) {
    case G_QKV: return {3 * H, H, 3 * H / BM, H / BK, E_STORE};
    case G_O: return {H, H, H / BM, H / BK, E_GATED};
    case G_CAQ: return {H, H, H / BM, H / BK, E_STORE};
    case G_OCA: return {H, H, H / BM, H / BK, E_GATED};
    case G_GU: return {2 * I, H, I / 64, H / BK, E_GU};
    default: return {H, I, H / BM, I / BK, E_GATED};
  }
}

thread_local char g_batch_err[256] = "";
}  // namespace

struct mkx_batch_handle {
  mkx_dims d;
  int device, max_ep, Mp_max, sms;
  uint16_t* wpk[NGEMM];  // per GEMM: [L][tiles][ktiles] blocks
  float* nrm;            // [3][L][HD] 1 + norm weights
  uint16_t* plain;       // one modulation row [MODW] bf16: scale = shift = 0, gates 1 (register rows)
  float *win, *bin, *wout, *bout;
  uint16_t *h, *a, *qkv, *y, *g;
  float* xs;
  int* status;
  unsigned long long timeout_ns;
  // tensor maps of the GEMM B operands (AdaRMS rows, attention output, gate/up product) per token
  // tile size ntok = 16 (k + 1), encoded on first use
  bool map_ok[3][MAXN / 16];
  CUtensorMap maps[3][MAXN / 16];
};

static mkx_status batch_fail(cudaError_t e, const char* what) {
  snprintf(g_batch_err, sizeof(g_batch_err), "%s: %s", what, cudaGetErrorString(e));
  return MKX_ERR_CUDA;
}

extern "C" mkx_status mkx_batch_create(const mkx_dims* dims, const mkx_weights* w, int max_episodes, int device,
                                       mkx_batch_handle** out) {
  if (!dims || !w || !out || max_episodes < 1 || max_episodes > 4096) return MKX_ERR_INVALID_ARG;
  *out = nullptr;
  const mkx_dims d = *dims;
  if (d.H != H || d.NH != NH || d.HD != HD || d.L < 1 || d.L > MKX_MAX_LAYERS || d.I < 128 || d.I % 128 != 0 ||
      d.A < AO || d.A > 32)
    return MKX_ERR_UNSUPPORTED;
  const void* ptrs[] = {w->wqkv, w->wo, w->wqca, w->woca, w->wg, w->wu, w->wd, w->qn, w->kn, w->qcan,
                        w->win, w->bin, w->wout, w->bout};
  for (const void* q : ptrs)
    if (!q) return MKX_ERR_INVALID_ARG;
  DeviceScope dev_scope(device);
  if (dev_scope.err != cudaSuccess) return batch_fail(dev_scope.err, "cudaSetDevice");
  mkx_batch_handle* h = new (std::nothrow) mkx_batch_handle();
  if (!h) return MKX_ERR_RESOURCES;
  memset(h, 0, sizeof(*h));
  h->d = d;
  h->device = device;
  h->max_ep = max_episodes;
  h->timeout_ns = 2000000000ull;
  cudaDeviceGetAttribute(&h->sms, cudaDevAttrMultiProcessorCount, device);
  const int L = d.L, I = d.I, A = d.A;
  const int Mp = ((max_episodes * TPMAX + 15) / 16) * 16;
  h->Mp_max = Mp;
  bool ok = true;
  auto alloc = [&](void** pp, size_t bytes) {
    if (ok && cudaMalloc(pp, bytes) != cudaSuccess) ok = false;
  };
  for (int g = 0; g < NGEMM; ++g) {
    const GemmShape s = gemm_shape(g, I);
    alloc((void**)&h->wpk[g], (size_t)L * s.ntiles * s.ktiles * A_BYTES);
  }
  alloc((void**)&h->nrm, (size_t)3 * L * HD * 4);
  alloc((void**)&h->plain, (size_t)(9 * L * H + 2 * H) * 2);
  alloc((void**)&h->win, (size_t)A * H * 4);
  alloc((void**)&h->bin, (size_t)H * 4);
  alloc((void**)&h->wout, (size_t)A * H * 4);
  alloc((void**)&h->bout, (size_t)A * 4);
  alloc((void**)&h->h, (size_t)Mp * H * 2);
  alloc((void**)&h->a, (size_t)Mp * H * 2);
  alloc((void**)&h->qkv, (size_t)Mp * 3 * H * 2);
  alloc((void**)&h->y, (size_t)Mp * H * 2);
  alloc((void**)&h->g, (size_t)Mp * I * 2);
  alloc((void**)&h->xs, (size_t)max_episodes * TPMAX * A * 4);
  alloc((void**)&h->status, 64);
  if (!ok) {
    mkx_batch_destroy(h);
    return batch_fail(cudaErrorMemoryAllocation, "cudaMalloc(batch)");
  }
  const size_t HH = (size_t)H * H;
  for (int l = 0; l < L && ok; ++l) {
    const uint16_t* src0[NGEMM] = {w->wqkv + (size_t)l * 3 * HH, w->wo + (size_t)l * HH, w->wqca + (size_t)l * HH,
                                   w->woca + (size_t)l * HH, w->wg + (size_t)l * I * H, w->wd + (size_t)l * H * I};
    for (int g = 0; g < NGEMM; ++g) {
      const GemmShape s = gemm_shape(g, I);
      const size_t per = (size_t)s.ntiles * s.ktiles * (A_BYTES / 2);
      bt_pack_kernel<<<h->sms * 4, 256>>>(src0[g], g == G_GU ? w->wu + (size_t)l * I * H : nullptr, h->wpk[g] + l * per,
                                          s.ntiles, s.ktiles, s.K, g == G_GU ? 1 : 0);
    }
  }
  bt_norm_kernel<<<(3 * L * HD + 255) / 256, 256>>>(w->qn, w->kn, w->qcan, h->nrm, L);
  {
    const int MODW = 9 * L * H + 2 * H;
    uint16_t* pl = new (std::nothrow) uint16_t[MODW];
    if (!pl) ok = false;
    if (ok) {
      for (int i = 0; i < MODW; ++i) {
        const int within = i < 9 * L * H ? (i % (3 * H)) / H : 0;  // 0 scale, 1 shift, 2 gate
        pl[i] = within == 2 ? (uint16_t)0x3F80 : (uint16_t)0;       // bf16 1.0 / 0.0
      }
      cudaMemcpy(h->plain, pl, (size_t)MODW * 2, cudaMemcpyHostToDevice);
    }
    delete[] pl;
  }
  cudaMemcpy(h->win, w->win, (size_t)A * H * 4, cudaMemcpyDeviceToDevice);
  cudaMemcpy(h->bin, w->bin, (size_t)H * 4, cudaMemcpyDeviceToDevice);
  cudaMemcpy(h->wout, w->wout, (size_t)A * H * 4, cudaMemcpyDeviceToDevice);
  cudaMemcpy(h->bout, w->bout, (size_t)A * 4, cudaMemcpyDeviceToDevice);
  cudaMemset(h->h, 0, (size_t)Mp * H * 2);
  cudaMemset(h->a, 0, (size_t)Mp * H * 2);
  cudaMemset(h->qkv, 0, (size_t)Mp * 3 * H * 2);
  cudaMemset(h->y, 0, (size_t)Mp * H * 2);
  cudaMemset(h->g, 0, (size_t)Mp * I * 2);
  cudaMemset(h->status, 0, 64);
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaFuncSetAttribute(bt_gemm, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BUDGET);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(bt_attention<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (16 + 2 * SA_MAXK) * KS * 2);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(bt_attention<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 100 * 1024);
  if (e != cudaSuccess) {
    mkx_batch_destroy(h);
    return batch_fail(e, "mkx_batch_create");
  }
  *out = h;
  return MKX_OK;
}

namespace {
// Launch with the programmatic-dependent attribute (the kernel waits for its predecessor itself).
// cluster_z > 1: thread-block clusters of (1, 1, cluster_z) CTAs.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, int cluster_z,
                               Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster_z > 1) {
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = 1;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = (unsigned)cluster_z;
    n = 2;
  }
  cfg.attrs = at;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  return launch_pdl_cluster(k, grid, block, smem, st, 1, args...);
}

// Token tile of a GEMM with `ntiles` feature tiles: about one CTA per SM (each token tile re-reads the
// weight tile from L2, not HBM), a multiple of 16 rows, at most 256.
int gemm_token_tile(int M, int ntiles, int sms) {
  int tt = (sms + ntiles - 1) / ntiles;
  if (tt < 1) tt = 1;
  int per = (M + tt - 1) / tt;
  if (per > MAXN) per = MAXN;
  per = ((per + 15) / 16) * 16;
  const int nt = (M + per - 1) / per;  // balance the tiles
  return (((M + nt - 1) / nt) + 15) / 16 * 16;
}

struct GemmLaunch {
  int stages, smem, tmem_cols;
};
// Ring stages for a token tile of a CTA with nk k tiles: no more than its k tiles (a short K range
// leaves room for more CTAs per SM, so the next kernel's CTAs can start their weight streams while
// this one finishes) and no more than fit next to the barriers (and, gated epilogues, the residual
// tile); the transposed accumulator tile reuses the ring. TMEM: ntok columns rounded up to a power
// of two >= 32; the shared-memory size is raised so that no more CTAs fit on an SM than their TMEM
// columns allow (512 per SM), so a TMEM allocation never waits. false if the accumulator tile does not
// fit.
bool gemm_launch_shape(int ntok, bool residual, int nk, GemmLaunch* out) {
  const int stage_bytes = A_BYTES + ntok * BK * 2, slack = 1024 + 256, extra = residual ? ntok * BM * 2 : 0;
  int fit = (SMEM_BUDGET - slack - extra) / stage_bytes;
  if (fit > MAX_STAGES) fit = MAX_STAGES;
  const int tile_bytes = ((ntok + 31) / 32) * 32 * TS * 4;
  int st = nk < fit ? nk : fit;
  if (st < 1) st = 1;
  while (st < fit && st * stage_bytes < tile_bytes) ++st;
  if (st * stage_bytes < tile_bytes) return false;
  int cols = 32;
  while (cols < ntok) cols *= 2;
  out->stages = st;
  out->tmem_cols = cols;
  out->smem = st * stage_bytes + slack + extra;
  const int per_sm = 512 / cols, floor_bytes = 228 * 1024 / (per_sm + 1) + 1024;
  if (out->smem < floor_bytes) out->smem = floor_bytes;
  return out->smem <= SMEM_BUDGET;
}

// K splits of a GEMM (one thread-block cluster per tile): as many as keep the launch within one wave
// of CTAs (floor of SMs / tiles), at least 2 k tiles (128 K) each, at most MAX_SPLITS (the portable
// cluster size).
int gemm_splits(const GemmShape& s, int ttiles, int sms) {
  int z = sms / (s.ntiles * ttiles);
  if (z > s.ktiles / 2) z = s.ktiles / 2;
  if (z > MAX_SPLITS) z = MAX_SPLITS;
  if (z < 1) z = 1;
  const int kps = (s.ktiles + z - 1) / z;
  return (s.ktiles + kps - 1) / kps;
}
}  // namespace

extern "C" int mkx_batch_launches(const mkx_batch_handle* h, int B, int T, int n_steps) {
  if (!h || B < 1 || B > h->max_ep || T < 1 || T > TPMAX || n_steps < 1) return -1;
  return 1 + n_steps * (11 * h->d.L + 1);
}

namespace {
// The tensor map of B-operand buffer `buf` (0 AdaRMS rows, 1 attention output, 2 gate/up product) for a
// token tile of ntok rows (box 64 columns x ntok rows, 128-byte swizzle); nullptr if encoding fails.
const CUtensorMap* token_map(mkx_batch_handle* h, int buf, int ntok) {
  const int k = ntok / 16 - 1;
  if (!h->map_ok[buf][k]) {
    void* base = buf == 0 ? (void*)h->a : (buf == 1 ? (void*)h->y : (void*)h->g);
    const uint64_t cols = buf == 2 ? (uint64_t)h->d.I : (uint64_t)H;
    if (!encode_bf16_sw128(&h->maps[buf][k], base, (uint64_t)h->Mp_max, cols, (uint32_t)ntok)) return nullptr;
    h->map_ok[buf][k] = true;
  }
  return &h->maps[buf][k];
}
}  // namespace

namespace {
// One enqueue sequence: the launches of a run share these.
struct Seq {
  mkx_batch_handle* h;
  cudaStream_t stream;
  int B, T, M, Mp;
  long long ep_stride;  // episode stride of the modulation rows (0: one row for every episode)
  cudaError_t err;
  mkx_status st;
};

void seq_gemm(Seq& q, int g, int l, int buf, uint16_t* out, int ldo, const uint16_t* gate) {
  if (q.err != cudaSuccess || q.st != MKX_OK) return;
  mkx_batch_handle* h = q.h;
  const GemmShape s = gemm_shape(g, h->d.I);
  // up to SMALL_M token rows: one token tile and a K split fixed by the GEMM's shape, so a row's
  // result does not depend on how many other rows share the launch; beyond, token tiles for about
  // one CTA per SM and K splits only while the launch stays within one wave
  const bool small = q.M <= SMALL_M;
  const int ntok = small ? (q.M + 15) / 16 * 16 : gemm_token_tile(q.M, s.ntiles, h->sms);
  const int ttiles = (q.M + ntok - 1) / ntok;
  const CUtensorMap* map = token_map(h, buf, ntok);
  GemmParams p;
  memset(&p, 0, sizeof(p));
  p.splits = gemm_splits(s, ttiles, h->sms);
  p.kps = (s.ktiles + p.splits - 1) / p.splits;
  p.epi = s.epi;
  p.ttiles = ttiles;
  GemmLaunch gl;
  if (!map || !gemm_launch_shape(ntok, p.epi == E_GATED, p.kps, &gl)) {
    q.st = map ? MKX_ERR_UNSUPPORTED : MKX_ERR_CUDA;
    return;
  }
  p.wpk = h->wpk[g] + (size_t)l * s.ntiles * s.ktiles * (A_BYTES / 2);
  p.ktiles = s.ktiles;
  p.ntok = ntok;
  p.M = q.M;
  p.T = q.T;
  p.stages = gl.stages;
  p.tmem_cols = gl.tmem_cols;
  p.out = out;
  p.ldo = ldo;
  p.gate = gate;
  p.gate_stride = q.ep_stride;
  p.status = h->status;
  p.timeout_ns = h->timeout_ns;
  q.err = launch_pdl_cluster(bt_gemm, dim3(s.ntiles, ttiles, p.splits), dim3(GEMM_THREADS), (size_t)gl.smem, q.stream,
                             p.splits, *map, p);
}

void seq_adarms(Seq& q, const uint16_t* blk) {
  if (q.err != cudaSuccess) return;
  q.err = launch_pdl(bt_adarms, dim3((q.Mp + 7) / 8), dim3(256), 0, q.stream, (const uint16_t*)q.h->h, q.h->a, q.M, q.Mp,
                     q.T, blk, q.ep_stride, q.h->d.eps);
}

// What one layer reads besides the handle's buffers: the episodes' register memory and
// cross-attention K/V of this layer (episode strides kvm_ep / kvc_ep; 0 = shared by all), their row
// limits (lim_stride 0 = one value for all), the RoPE tables of the query rows, and -- register pass
// only -- the memory rows [frame_row0, frame_row0 + M) where the self-attention launch writes the
// rows' own K / V (and reads them as the memory's newest rows; own = 0: no own-row keys besides).
struct LayerIO {
  const uint16_t* memk;
  const uint16_t* memv;
  long long kvm_ep;
  int mem_rows;
  const int* kv_start;
  const uint16_t* kca;
  const uint16_t* vca;
  long long kvc_ep;
  int ca_rows;
  const int* src_rows;
  int lim_stride, own;
  int sa_input, ca_input;  // memory / cross-attention K/V written before the sequence (bt_attention kv_input)
  const float *sa_cos, *sa_sin, *ca_cos, *ca_sin;
  int frame_row0;  // < 0: no frame to write
};

// The 11 launches of one layer (src/mk_expert.py:342-421); blk: this layer's modulation blocks
// [SA | CA | MLP] x [scale, shift, gate] of episode 0.
void seq_layer(Seq& q, int l, const uint16_t* blk, const LayerIO& io) {
  mkx_batch_handle* h = q.h;
  const int L = h->d.L, I = h->d.I;
  const int kcap = (io.mem_rows + (io.own ? q.T : 0) + CA_BLK - 1) / CA_BLK * CA_BLK;  // <= SA_MAXK
  const size_t att_sa = (size_t)(16 + 2 * kcap) * KS * 2;
  // cross-attention: the whole padded source at once when it fits 3 blocks and the (episode, head)
  // units are few (one round of copies in flight per CTA); with many units, 2 blocks double-buffered
  // (smaller CTAs, more of them per SM)
  const bool ca_all = io.ca_rows <= CA_ALL_ROWS && q.B * NH <= CA_ALL_UNITS_PER_SM * h->sms;
  const int ca_cap = ca_all ? (io.ca_rows + CA_BLK - 1) / CA_BLK * CA_BLK : 2 * CA_BLK;
  const size_t att_ca = (size_t)(16 + 2 * ca_cap) * KS * 2;
  const uint16_t* memk_l = io.memk + (size_t)l * io.mem_rows * H;
  const uint16_t* memv_l = io.memv + (size_t)l * io.mem_rows * H;
  AttnParams ap;
  memset(&ap, 0, sizeof(ap));
  ap.y = h->y;
  ap.T = q.T;
  ap.qk_eps = h->d.qk_eps;
  ap.scale = 1.0f / sqrtf((float)HD);
  ap.lim_stride = io.lim_stride;
  // self-attention block
  seq_adarms(q, blk);
  seq_gemm(q, G_QKV, l, 0, h->qkv, 3 * H, nullptr);
  ap.src = h->qkv;
  ap.src_ld = 3 * H;
  ap.kb = memk_l;
  ap.vb = memv_l;
  ap.kv_ep = io.kvm_ep;
  ap.kv_rows = io.mem_rows;
  ap.lim = io.kv_start;
  ap.cos = io.sa_cos;
  ap.sin = io.sa_sin;
  ap.wq = h->nrm + (size_t)l * HD;
  ap.wk = h->nrm + (size_t)(L + l) * HD;
  ap.kcap = kcap;
  ap.own = io.own;
  ap.kv_input = io.sa_input;
  ap.frame_row0 = -1;
  if (io.frame_row0 >= 0) {
    ap.frame_row0 = io.frame_row0;
    ap.frame_rows = q.M;
    ap.mk_out = const_cast<uint16_t*>(memk_l);
    ap.mv_out = const_cast<uint16_t*>(memv_l);
  }
  if (q.err == cudaSuccess && q.st == MKX_OK)
    q.err = launch_pdl(bt_attention<true>, dim3(q.B * NH), dim3(32 * ATT_WARPS), att_sa, q.stream, ap);
  ap.frame_row0 = -1;
  seq_gemm(q, G_O, l, 1, h->h, H, blk + 2 * H);
  // cross-attention block
  seq_adarms(q, blk + 3 * H);
  seq_gemm(q, G_CAQ, l, 0, h->qkv, H, nullptr);  // the query in the qkv buffer, rows of H
  ap.src = h->qkv;
  ap.src_ld = H;
  ap.kb = io.kca + (size_t)l * io.ca_rows * H;
  ap.vb = io.vca + (size_t)l * io.ca_rows * H;
  ap.kv_ep = io.kvc_ep;
  ap.kv_rows = io.ca_rows;
  ap.lim = io.src_rows;
  ap.cos = io.ca_cos;
  ap.sin = io.ca_sin;
  ap.wq = h->nrm + (size_t)(2 * L + l) * HD;
  ap.wk = nullptr;
  ap.kv_input = io.ca_input;
  ap.kcap = ca_cap;
  ap.ca_all = ca_all ? 1 : 0;
  if (q.err == cudaSuccess && q.st == MKX_OK)
    q.err = launch_pdl(bt_attention<false>, dim3(q.B * NH), dim3(32 * ATT_WARPS), att_ca, q.stream, ap);
  seq_gemm(q, G_OCA, l, 1, h->h, H, blk + 5 * H);
  // MLP block
  seq_adarms(q, blk + 6 * H);
  seq_gemm(q, G_GU, l, 0, h->g, I, nullptr);
  seq_gemm(q, G_D, l, 2, h->h, H, blk + 8 * H);
}

mkx_status seq_finish(Seq& q, const char* what) {
  if (q.err != cudaSuccess) return batch_fail(q.err, what);
  if (q.st != MKX_OK) {
    snprintf(g_batch_err, sizeof(g_batch_err), "%s: tensor map or launch shape", what);
    return q.st;
  }
  return MKX_OK;
}
}  // namespace

extern "C" mkx_status mkx_batch_run(mkx_batch_handle* h, const mkx_batch_inputs* in, cudaStream_t stream) {
  if (!h || !in) return MKX_ERR_INVALID_ARG;
  const mkx_dims& d = h->d;
  if (in->B < 1 || in->B > h->max_ep || in->T < 1 || in->T > TPMAX || in->n_steps < 1 || in->action_dim < 1 ||
      in->action_dim > AO)
    return MKX_ERR_INVALID_ARG;
  if (in->mem_rows < 1 || in->mem_rows > 256 || in->ca_rows < 1 || in->ca_rows > 4096) return MKX_ERR_UNSUPPORTED;
  const void* ptrs[] = {in->x_in, in->x_out, in->mods, in->dt, in->memk, in->memv, in->kv_start, in->kca, in->vca,
                        in->src_rows, in->sa_cos, in->sa_sin, in->ca_cos, in->ca_sin};
  for (const void* q : ptrs)
    if (!q) return MKX_ERR_INVALID_ARG;
  const void* al16[] = {in->mods, in->memk, in->memv, in->kca, in->vca};
  for (const void* q : al16)
    if (reinterpret_cast<uintptr_t>(q) & 15u) return MKX_ERR_INVALID_ARG;
  const void* al8[] = {in->sa_cos, in->sa_sin, in->ca_cos, in->ca_sin};
  for (const void* q : al8)
    if (reinterpret_cast<uintptr_t>(q) & 7u) return MKX_ERR_INVALID_ARG;
  DeviceScope dev_scope(h->device);
  if (dev_scope.err != cudaSuccess) return batch_fail(dev_scope.err, "cudaSetDevice");
  const int L = d.L, A = d.A, T = in->T, B = in->B;
  const int MODW = 9 * L * H + 2 * H;
  Seq q = {h, stream, B, T, B * T, ((B * T + 15) / 16) * 16, (long long)(in->n_steps + 1) * MODW, cudaSuccess, MKX_OK};
  LayerIO io;
  memset(&io, 0, sizeof(io));
  io.memk = in->memk;
  io.memv = in->memv;
  io.kvm_ep = (long long)L * in->mem_rows * H;
  io.mem_rows = in->mem_rows;
  io.kv_start = in->kv_start;
  io.kca = in->kca;
  io.vca = in->vca;
  io.kvc_ep = (long long)L * in->ca_rows * H;
  io.ca_rows = in->ca_rows;
  io.src_rows = in->src_rows;
  io.lim_stride = 1;
  io.own = 1;
  io.sa_input = 1;  // the caller's memory and cross-attention K/V
  io.ca_input = 1;
  io.sa_cos = in->sa_cos;
  io.sa_sin = in->sa_sin;
  io.ca_cos = in->ca_cos;
  io.ca_sin = in->ca_sin;
  io.frame_row0 = -1;
  auto tail = [&](int first, int last, int s) {
    if (q.err != cudaSuccess) return;
    TailParams t;
    memset(&t, 0, sizeof(t));
    t.x_in = in->x_in;
    t.xs = h->xs;
    t.x_out = in->x_out;
    t.h = h->h;
    t.mfin = in->mods + (size_t)(1 + s) * MODW + (size_t)9 * L * H;
    t.ep_stride = q.ep_stride;
    t.dt = in->dt;
    t.win = h->win;
    t.bin = h->bin;
    t.wout = h->wout;
    t.bout = h->bout;
    t.T = T;
    t.A = A;
    t.adim = in->action_dim;
    t.first = first;
    t.last = last;
    t.eps = d.eps;
    q.err = launch_pdl(bt_tail, dim3(q.M), dim3(256), 0, stream, t);
  };
  cudaMemsetAsync(h->status, 0, sizeof(int), stream);
  tail(1, 0, 0);  // h0 = in-projection of x_in
  for (int s = 0; s < in->n_steps; ++s) {
    const uint16_t* mrow = in->mods + (size_t)(1 + s) * MODW;
    for (int l = 0; l < L; ++l) seq_layer(q, l, mrow + (size_t)9 * H * l, io);
    tail(0, s + 1 == in->n_steps, s);
  }
  return seq_finish(q, "mkx_batch_run");
}

extern "C" mkx_status mkx_batch_register_pass(mkx_batch_handle* h, const mkx_register_inputs* in, cudaStream_t stream) {
  if (!h || !in) return MKX_ERR_INVALID_ARG;
  const mkx_dims& d = h->d;
  if (in->R < 16 || in->R % 16 != 0 || in->R > 16 * h->max_ep || in->mem_rows < in->R || in->mem_rows > 256 ||
      in->ca_rows < 1 || in->ca_rows > 4096)
    return MKX_ERR_INVALID_ARG;
  const void* ptrs[] = {in->reg_in, in->memk, in->memv, in->kv_start, in->kca, in->vca, in->src_rows,
                        in->sa_cos, in->sa_sin, in->ca_cos, in->ca_sin};
  for (const void* q : ptrs)
    if (!q) return MKX_ERR_INVALID_ARG;
  const void* al16[] = {in->reg_in, in->memk, in->memv, in->kca, in->vca};
  for (const void* q : al16)
    if (reinterpret_cast<uintptr_t>(q) & 15u) return MKX_ERR_INVALID_ARG;
  const void* al8[] = {in->sa_cos, in->sa_sin, in->ca_cos, in->ca_sin};
  for (const void* q : al8)
    if (reinterpret_cast<uintptr_t>(q) & 7u) return MKX_ERR_INVALID_ARG;
  DeviceScope dev_scope(h->device);
  if (dev_scope.err != cudaSuccess) return batch_fail(dev_scope.err, "cudaSetDevice");
  const int L = d.L, R = in->R;
  // the register rows as R / 16 groups of 16 query rows sharing one memory and one source; plain
  // norms and residuals: one modulation row of zero scale / shift and unit gates for every group
  Seq q = {h, stream, R / 16, 16, R, R, 0, cudaSuccess, MKX_OK};
  LayerIO io;
  memset(&io, 0, sizeof(io));
  io.memk = in->memk;
  io.memv = in->memv;
  io.mem_rows = in->mem_rows;
  io.kv_start = in->kv_start;
  io.kca = in->kca;
  io.vca = in->vca;
  io.ca_rows = in->ca_rows;
  io.src_rows = in->src_rows;
  io.lim_stride = 0;
  io.own = 0;
  io.sa_input = 1;  // the memory rows below the frame; the frame's come from the QKV output (frame_row0)
  io.ca_input = 1;
  io.sa_cos = in->sa_cos;
  io.sa_sin = in->sa_sin;
  io.ca_cos = in->ca_cos;
  io.ca_sin = in->ca_sin;
  io.frame_row0 = in->mem_rows - R;
  cudaMemsetAsync(h->status, 0, sizeof(int), stream);
  q.err = cudaMemcpyAsync(h->h, in->reg_in, (size_t)R * H * 2, cudaMemcpyDeviceToDevice, stream);
  for (int l = 0; l < L; ++l) seq_layer(q, l, h->plain + (size_t)9 * H * l, io);
  return seq_finish(q, "mkx_batch_register_pass");
}

extern "C" const char* mkx_batch_last_cuda_error(void) { return g_batch_err; }

extern "C" mkx_status mkx_batch_copy_state(mkx_batch_handle* h, int which, void* dst, size_t bytes) {
  if (!h || !dst || which < 0 || which > 5) return MKX_ERR_INVALID_ARG;
  const int I = h->d.I;
  void* src[6] = {h->h, h->a, h->qkv, h->y, h->g, h->xs};
  const size_t cap[6] = {(size_t)h->Mp_max * H * 2, (size_t)h->Mp_max * H * 2, (size_t)h->Mp_max * 3 * H * 2,
                         (size_t)h->Mp_max * H * 2, (size_t)h->Mp_max * I * 2,
                         (size_t)h->max_ep * TPMAX * h->d.A * 4};
  if (bytes > cap[which]) return MKX_ERR_INVALID_ARG;
  DeviceScope dev_scope(h->device);
  if (dev_scope.err != cudaSuccess) return batch_fail(dev_scope.err, "cudaSetDevice");
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(dst, src[which], bytes, cudaMemcpyDeviceToDevice);
  return e == cudaSuccess ? MKX_OK : batch_fail(e, "mkx_batch_copy_state");
}

extern "C" mkx_status mkx_batch_last_error(mkx_batch_handle* h, int* code) {
  if (!h || !code) return MKX_ERR_INVALID_ARG;
  DeviceScope dev_scope(h->device);
  if (dev_scope.err != cudaSuccess) return batch_fail(dev_scope.err, "cudaSetDevice");
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(code, h->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return batch_fail(e, "mkx_batch_last_error");
  return *code ? MKX_ERR_DEVICE : MKX_OK;
}

extern "C" void mkx_batch_destroy(mkx_batch_handle* h) {
  if (!h) return;
  DeviceScope dev_scope(h->device);
  for (int g = 0; g < NGEMM; ++g) cudaFree(h->wpk[g]);
  void* bufs[] = {h->nrm, h->plain, h->win, h->bin, h->wout, h->bout, h->h, h->a, h->qkv, h->y, h->g,
                  h->xs, h->status};
  for (void* b : bufs) cudaFree(b);
  delete h;
}
