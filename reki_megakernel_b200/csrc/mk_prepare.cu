// Cross-attention K/V preparation ("register_prepare", restated; see include/mkx_prepare.h) on
// sm_100a as one tensor-core GEMM over all layers:
//
//   D[f, n] = sum_k Wkv[f, k] * src[n, k]      f over [L][K|V][768] (15,360 rows at REKI's sizes)
//
// One CTA per (128-feature tile, block of <= 256 tokens). Warp 0: producer into an mbarrier ring of up
// to 8 stages (the first ring of copies goes out right after the barriers are initialised, before
// the TMEM allocation): the W tile as one contiguous 16 KB bulk copy from a copy of W packed at create
// time in the 128-byte-swizzled K-major order the MMA reads (tile-contiguous, so HBM sees long
// bursts), the source rows by TMA with the same swizzle. Warp 1: allocates 256 TMEM columns and
// issues tcgen05.mma kind::f16 (M = 128, N = tokens, K = 16 per instruction, bf16 in, fp32
// accumulate in TMEM), committing each stage back to the producer. Warps 2-5 (one per TMEM lane
// quarter): read the accumulator with tcgen05.ld and transpose it through shared memory (reusing the
// drained stage ring). Then all 12 warps: in K tiles, one (token, head) row per thread for the head
// RMSNorm (1 + kn), written back in place; then, per lane, an 8-feature part of a token's rows of
// both heads: rotate-half RoPE in fp32 (partner dims from a shuffle, the RoPE rows loaded into a
// register ring ahead of time), one bf16 rounding, coalesced 16-byte stores of the [L][SP][NH][HD]
// outputs. Every wait is bounded by %globaltimer; after a timeout the CTA records the error, drains
// its copies and MMAs, frees TMEM and returns.
#include <cstdint>
#include <cstring>
#include <new>
#include <cuda.h>  // CUtensorMap and its enums (the encoder itself comes from cudaGetDriverEntryPoint)
#include <cuda_runtime.h>

#include "mkx_prepare.h"
#include "mkx_device.cuh"
#include "mkx_tma.cuh"

namespace mkxp {
using namespace mkx;

constexpr int BM = 128;             // output features per tile (UMMA M)
constexpr int BK = 64;              // K elements per stage: one 128-byte swizzle row
constexpr int MAXN = 256;           // tokens per tile (UMMA N)
constexpr int MAX_STAGES = 8;      // ring depth: as many stages as fit (weights in flight per SM)
constexpr int SMEM_BUDGET = 227 * 1024;
constexpr int NTHREADS = 384;       // warp 0 TMA, warp 1 TMEM + MMA, warps 2-5 TMEM read-back, all 12 epilogue
constexpr int TMEM_COLS = 256;
constexpr int TS = BM + 4;          // transposed tile: floats per token row (16-byte aligned rows)
constexpr int A_BYTES = BM * BK * 2;
constexpr int H = 768, NH = 12, HD = 64;
constexpr int TILES_PER_LAYER = 2 * H / BM;  // 6 K tiles then 6 V tiles

struct PrepParams {
  int S, SP, ntok, L, ktiles, stages;
  const uint16_t* wpk;  // packed W: [tile][kb][128 rows x 64] swizzled, 16 KB per (tile, kb)
  float eps;
  const float* kn;
  const float* cos;
  const float* sin;
  uint16_t* k_out;
  uint16_t* v_out;
  int* status;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity, unsigned long long limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > limit) return false;
  return true;
}

__device__ __forceinline__ void record(const PrepParams& p, int code) { atomicCAS(p.status, 0, code); }

extern __shared__ __align__(1024) char psmem[];

__global__ void __launch_bounds__(NTHREADS, 1)
    prep_kernel(const __grid_constant__ CUtensorMap ts, const __grid_constant__ PrepParams p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, tok0 = blockIdx.y * p.ntok;
  const int stage_bytes = A_BYTES + p.ntok * BK * 2;  // a multiple of 1024
  // every stage's A and B tile must start on a 1024-byte boundary (128-byte swizzle atoms): align the
  // ring inside the dynamic allocation, which is sized with 1 KB to spare
  char* ring = psmem + ((1024u - (smem_u32(psmem) & 1023u)) & 1023u);
  const int STAGES = p.stages;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + STAGES * stage_bytes);
  uint64_t* full = bars;
  uint64_t* empty = bars + MAX_STAGES;
  uint64_t* done = bars + 2 * MAX_STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * MAX_STAGES + 1);
  int* consumed_slot = reinterpret_cast<int*>(tmem_slot + 1);
  float* kn_s = reinterpret_cast<float*>(bars + 2 * MAX_STAGES + 4);  // [HD] K norm weights of the layer

  int issued = 0;  // producer (thread 0): k tiles whose copies have been issued
  auto issue = [&](int kb) {
    const int s = kb % STAGES;
    char* a = ring + s * stage_bytes;
    mbar_expect_tx(&full[s], (uint32_t)stage_bytes);
    bulk_g2s(a, p.wpk + ((size_t)tile * p.ktiles + kb) * (A_BYTES / 2), (uint32_t)A_BYTES, &full[s]);
    tma_load_2d(a + A_BYTES, &ts, kb * BK, tok0, &full[s]);
    issued = kb + 1;
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *consumed_slot = 0;
    fence_mbar_init();
    // the first ring of copies needs only these barriers: it goes out before the TMEM allocation and
    // the block barrier
    for (int kb = 0; kb < min(STAGES, p.ktiles); ++kb) issue(kb);
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  if (warp == 3 && lane < HD / 4)
    reinterpret_cast<float4*>(kn_s)[lane] =
        __ldg(reinterpret_cast<const float4*>(p.kn + (size_t)(tile / TILES_PER_LAYER) * HD) + lane);
  if (threadIdx.x == 64 && tile % TILES_PER_LAYER < TILES_PER_LAYER / 2) {
    // K tiles: the RoPE rows of this CTA's tokens are read only at the end; asking L2 for them now
    // takes their HBM latency off the epilogue
    const int nv = min(p.ntok, p.S - tok0);
    bulk_prefetch_l2(p.cos + (size_t)tok0 * HD, (uint32_t)(nv * HD * 4));
    bulk_prefetch_l2(p.sin + (size_t)tok0 * HD, (uint32_t)(nv * HD * 4));
  }
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // producer
    for (int kb = issued; kb < p.ktiles; ++kb) {
      const int s = kb % STAGES;
      if (!wait_bounded(&empty[s], ((kb / STAGES) & 1) ^ 1, p.timeout_ns)) {
        record(p, 0x100 | 1);
        break;
      }
      issue(kb);
    }
  } else if (warp == 1 && lane == 0) {
    // MMA issuer
    const uint32_t idesc = umma_idesc(BM, p.ntok);
    int kb = 0;
    for (; kb < p.ktiles; ++kb) {
      const int s = kb % STAGES;
      if (!wait_bounded(&full[s], (kb / STAGES) & 1, p.timeout_ns)) {
        record(p, 0x100 | 2);
        break;
      }
      tmem_fence_after();
      const uint32_t a = smem_u32(ring + s * stage_bytes), b = a + A_BYTES;
#pragma unroll
      for (int k = 0; k < BK / 16; ++k)
        umma_bf16(tmem, sw128_desc(a + 32 * k), sw128_desc(b + 32 * k), idesc, (kb | k) != 0 ? 1u : 0u);
      umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
    }
    *consumed_slot = kb;
    umma_commit(done);  // every MMA issued above has completed when `done` flips
  }
  // Epilogue, part 1 (warps 2-5, one per TMEM lane quarter): accumulator -> transposed fp32 tile
  // [token][feature] in the drained stage ring.
  float* tsm = reinterpret_cast<float*>(ring);
  bool ok = true;
  if (warp >= 2 && warp < 6) {
    ok = __all_sync(0xffffffffu, wait_bounded(done, 0, p.timeout_ns));  // warp-uniform for tcgen05.ld
    if (!ok && lane == 0) record(p, 0x100 | 3);
    tmem_fence_after();
    const int q = warp & 3, r = 32 * q + lane;  // this thread's accumulator row (feature)
    if (ok) {
      for (int c0 = 0; c0 < p.ntok; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)c0, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) tsm[(c0 + j) * TS + r] = __uint_as_float(v[j]);
      }
    }
    tmem_fence_before();
  }
  const int l = tile / TILES_PER_LAYER, within = tile % TILES_PER_LAYER;
  const bool is_k = within < TILES_PER_LAYER / 2;
  const int h0 = 2 * (within % (TILES_PER_LAYER / 2));
  const int nvalid = min(p.ntok, p.S - tok0);
  const int nch = 8 * nvalid, part = lane & 7;
  const int iters = nch > 32 * warp ? (nch - 32 * warp + NTHREADS - 1) / NTHREADS : 0;  // warp-uniform
  const float* cosb = p.cos + (size_t)tok0 * HD + 8 * part;
  const float* sinb = p.sin + (size_t)tok0 * HD + 8 * part;
  constexpr int RS = 4;  // RoPE ring slots
  float4 tb[RS][4];
  auto tload = [&](int i, float4 (&t)[4]) {
    const int c = 32 * warp + lane + i * NTHREADS;
    const size_t off = (size_t)(c < nch ? c >> 3 : 0) * HD;
    t[0] = __ldg(reinterpret_cast<const float4*>(cosb + off));
    t[1] = __ldg(reinterpret_cast<const float4*>(cosb + off) + 1);
    t[2] = __ldg(reinterpret_cast<const float4*>(sinb + off));
    t[3] = __ldg(reinterpret_cast<const float4*>(sinb + off) + 1);
  };
  if (is_k) {  // the RoPE ring's first loads go out before the barrier (global reads only)
#pragma unroll
    for (int u = 0; u < RS; ++u)
      if (u < iters) tload(u, tb[u]);
  }
  ok = __syncthreads_and(ok);  // all roles done; the tile is complete (or a wait failed)
  // Epilogue, part 2 (all 12 warps), in two passes over the transposed tile.
  // (a) K tiles: one (token, head) row of 64 features per thread, items taken head-major (consecutive
  //     threads read consecutive tokens' rows: no bank conflicts): head RMSNorm * (1 + kn) in fp32,
  //     the sum of squares formed in the order of a 16-lane butterfly over groups of 4 dims; the
  //     thread reads its row again and writes it back normalised (kn staged in shared memory).
  // (b) all tiles, after a barrier: one 8-feature part of a token's rows of both heads per lane, a
  //     warp covering four tokens' contiguous 256-byte (2 heads) output segments. K: rotate-half RoPE
  //     in fp32, the partner dims d +- 32 from lane ^ 4, the RoPE rows read from global memory
  //     (coalesced, once for both heads) into a 4-slot register ring whose first loads go out before
  //     the transposition barrier, so their L2 latency overlaps pass (a); V: as is. One bf16
  //     rounding, 16-byte stores.
  if (ok && is_k) {
    const float4* kn4 = reinterpret_cast<const float4*>(kn_s);
    for (int it = threadIdx.x; it < 2 * nvalid; it += NTHREADS) {
      const int hh = it >= nvalid ? 1 : 0, nl = it - hh * nvalid;
      float4* row = reinterpret_cast<float4*>(tsm + nl * TS + 64 * hh);
      float s[16];
#pragma unroll
      for (int g = 0; g < 16; ++g) {
        const float4 y = row[g];
        s[g] = fmaf(y.x, y.x, fmaf(y.y, y.y, fmaf(y.z, y.z, y.w * y.w)));
      }
#pragma unroll
      for (int g = 0; g < 8; ++g) s[g] += s[g + 8];
#pragma unroll
      for (int g = 0; g < 4; ++g) s[g] += s[g + 4];
#pragma unroll
      for (int g = 0; g < 2; ++g) s[g] += s[g + 2];
      const float rstd = rsqrtf((s[0] + s[1]) / (float)HD + p.eps);
#pragma unroll
      for (int g = 0; g < 16; ++g) {  // the row is the thread's own: read it again, normalise in place
        const float4 k4 = kn4[g];
        float4 y = row[g];
        y.x = y.x * rstd * (1.f + k4.x);
        y.y = y.y * rstd * (1.f + k4.y);
        y.z = y.z * rstd * (1.f + k4.z);
        y.w = y.w * rstd * (1.f + k4.w);
        row[g] = y;
      }
    }
  }
  __syncthreads();
  if (ok) {
    uint16_t* out = is_k ? p.k_out : p.v_out;
    const float sg = part < 4 ? -1.f : 1.f;  // rot[d] = -y[d + 32] for d < 32, y[d - 32] above
    for (int i0 = 0; i0 < iters; i0 += RS) {
#pragma unroll
      for (int u = 0; u < RS; ++u) {
        const int i = i0 + u;
        if (i >= iters) break;  // warp-uniform: the shuffles need all lanes
        const int c = 32 * warp + lane + i * NTHREADS;
        const bool valid = c < nch;
        const int nl = valid ? c >> 3 : 0;
        uint16_t* dst = out + (((size_t)l * p.SP + tok0 + nl) * NH + h0) * HD + 8 * part;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const float4* src = reinterpret_cast<const float4*>(tsm + nl * TS + 64 * hh + 8 * part);
          float4 a = src[0], b = src[1];
          if (is_k) {
            const float4 c0v = tb[u][0], c1v = tb[u][1], s0v = tb[u][2], s1v = tb[u][3];
            const float pa0 = __shfl_xor_sync(0xffffffffu, a.x, 4), pa1 = __shfl_xor_sync(0xffffffffu, a.y, 4);
            const float pa2 = __shfl_xor_sync(0xffffffffu, a.z, 4), pa3 = __shfl_xor_sync(0xffffffffu, a.w, 4);
            const float pb0 = __shfl_xor_sync(0xffffffffu, b.x, 4), pb1 = __shfl_xor_sync(0xffffffffu, b.y, 4);
            const float pb2 = __shfl_xor_sync(0xffffffffu, b.z, 4), pb3 = __shfl_xor_sync(0xffffffffu, b.w, 4);
            a = make_float4(fmaf(a.x, c0v.x, sg * pa0 * s0v.x), fmaf(a.y, c0v.y, sg * pa1 * s0v.y),
                            fmaf(a.z, c0v.z, sg * pa2 * s0v.z), fmaf(a.w, c0v.w, sg * pa3 * s0v.w));
            b = make_float4(fmaf(b.x, c1v.x, sg * pb0 * s1v.x), fmaf(b.y, c1v.y, sg * pb1 * s1v.y),
                            fmaf(b.z, c1v.z, sg * pb2 * s1v.z), fmaf(b.w, c1v.w, sg * pb3 * s1v.w));
          }
          if (valid)
            *reinterpret_cast<uint4*>(dst + hh * HD) =
                make_uint4(pack_bf2(a.x, a.y), pack_bf2(a.z, a.w), pack_bf2(b.x, b.y), pack_bf2(b.z, b.w));
        }
        if (is_k && i + RS < iters) tload(i + RS, tb[u]);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // after a failure: let every bulk copy this CTA issued land before its shared memory goes away
    for (int kb = *consumed_slot; kb < issued; ++kb)
      if (!wait_bounded(&full[kb % STAGES], (kb / STAGES) & 1, p.timeout_ns)) break;
  }
  if (warp == 1) {
    wait_bounded(done, 0, p.timeout_ns);  // no MMA may still write the accumulator
    tmem_fence_after();
    tmem_free(tmem, TMEM_COLS);
  }
}

// Packs W [rows][src_dim] into [tile][kb][128 x 64] blocks laid out as a 128-byte-swizzled K-major
// tile (16-byte chunk c of row r at r * 128 + (c ^ (r % 8)) * 16): what a TMA load with 128-byte
// swizzle would leave in shared memory, so a plain bulk copy of a block reproduces it.
__global__ void prep_pack_kernel(const uint16_t* __restrict__ w, uint16_t* __restrict__ out, int tiles, int ktiles,
                                 int src_dim) {
  const long long total = (long long)tiles * ktiles * BM * 8;  // 16-byte chunks
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(e & 7), r = (int)((e >> 3) % BM);
    const long long blk = e / (8 * BM);
    const int kb = (int)(blk % ktiles), tile = (int)(blk / ktiles);
    const uint4 v = *reinterpret_cast<const uint4*>(w + (size_t)(tile * BM + r) * src_dim + kb * BK + c * 8);
    *reinterpret_cast<uint4*>(reinterpret_cast<char*>(out) + blk * A_BYTES + r * 128 + ((c ^ (r & 7)) << 4)) = v;
  }
}

// ---------------------------------------------------------------------------------------------
}  // namespace mkxp

struct mkx_prep_handle {
  mkx_prep_dims d;
  int device;
  uint16_t* wpk;  // packed W (owned)
  float* kn;      // K norm weights (owned copy)
  int* status;
  unsigned long long timeout_ns;
  cudaStream_t last_stream;
};

using namespace mkxp;

extern "C" mkx_status mkx_prep_create(const mkx_prep_dims* dims, const uint16_t* wkv, const float* kn, int device,
                                      mkx_prep_handle** out) {
  if (!dims || !wkv || !kn || !out) return MKX_ERR_INVALID_ARG;
  *out = nullptr;
  const mkx_prep_dims d = *dims;
  if (d.H != H || d.NH != NH || d.HD != HD || d.L < 1 || d.L > 64 || d.src_dim < BK || d.src_dim % BK != 0)
    return MKX_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(wkv) & 15) != 0) return MKX_ERR_INVALID_ARG;
  mkx::DeviceScope dev_scope(device);
  if (dev_scope.err != cudaSuccess) return MKX_ERR_CUDA;
  mkx_prep_handle* h = new (std::nothrow) mkx_prep_handle();
  if (!h) return MKX_ERR_RESOURCES;
  memset(h, 0, sizeof(*h));
  h->d = d;
  h->device = device;
  h->timeout_ns = 2000000000ull;
  const int tiles = d.L * TILES_PER_LAYER, ktiles = d.src_dim / BK;
  const size_t wbytes = (size_t)tiles * ktiles * A_BYTES;
  bool ok = cudaMalloc(&h->wpk, wbytes) == cudaSuccess && cudaMalloc(&h->kn, (size_t)d.L * HD * 4) == cudaSuccess &&
            cudaMalloc(&h->status, sizeof(int)) == cudaSuccess && cudaMemset(h->status, 0, sizeof(int)) == cudaSuccess &&
            cudaMemcpy(h->kn, kn, (size_t)d.L * HD * 4, cudaMemcpyDeviceToDevice) == cudaSuccess &&
            cudaFuncSetAttribute(prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BUDGET) == cudaSuccess;
  if (ok) {
    prep_pack_kernel<<<1184, 256>>>(wkv, h->wpk, tiles, ktiles, d.src_dim);
    ok = cudaGetLastError() == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
  }
  if (!ok) {
    if (h->wpk) cudaFree(h->wpk);
    if (h->kn) cudaFree(h->kn);
    if (h->status) cudaFree(h->status);
    delete h;
    return MKX_ERR_CUDA;
  }
  *out = h;
  return MKX_OK;
}

extern "C" mkx_status mkx_prep_run(mkx_prep_handle* h, const uint16_t* src, int S, const float* cos,
                                   const float* sin, uint16_t* k_out, uint16_t* v_out, int SP, cudaStream_t stream) {
  if (!h || !src || !cos || !sin || !k_out || !v_out) return MKX_ERR_INVALID_ARG;
  if (S < 1 || S > 4096 || SP < S) return MKX_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(src) & 15) != 0 || (reinterpret_cast<uintptr_t>(k_out) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(v_out) & 15) != 0 || (reinterpret_cast<uintptr_t>(cos) & 15) != 0 ||
      (reinterpret_cast<uintptr_t>(sin) & 15) != 0)
    return MKX_ERR_INVALID_ARG;
  mkx::DeviceScope dev_scope(h->device);
  if (dev_scope.err != cudaSuccess) return MKX_ERR_CUDA;
  const int ntok = S >= MAXN ? MAXN : ((S + 15) / 16) * 16;
  CUtensorMap ts;
  if (!encode_bf16_sw128(&ts, src, (uint64_t)S, (uint64_t)h->d.src_dim, (uint32_t)ntok)) return MKX_ERR_CUDA;
  // as many ring stages as fit next to the alignment slack and the barriers (the transposed
  // accumulator tile reuses the ring; it always fits in 2 stages), at least 80 KB in total: at most
  // 2 CTAs per SM, so their 2 x 256 TMEM columns always fit the SM's 512 and no allocation waits
  const int stage_bytes = A_BYTES + ntok * BK * 2, slack = 1024 + 64 * 8;
  int stages = (SMEM_BUDGET - slack) / stage_bytes;
  if (stages > MAX_STAGES) stages = MAX_STAGES;
  int smem = stages * stage_bytes + slack;
  if (smem < 80 * 1024) smem = 80 * 1024;
  PrepParams p;
  memset(&p, 0, sizeof(p));
  p.S = S;
  p.SP = SP;
  p.ntok = ntok;
  p.L = h->d.L;
  p.ktiles = h->d.src_dim / BK;
  p.stages = stages;
  p.eps = h->d.eps;
  p.kn = h->kn;
  p.wpk = h->wpk;
  p.cos = cos;
  p.sin = sin;
  p.k_out = k_out;
  p.v_out = v_out;
  p.status = h->status;
  p.timeout_ns = h->timeout_ns;
  const dim3 grid(h->d.L * TILES_PER_LAYER, (S + ntok - 1) / ntok);
  prep_kernel<<<grid, NTHREADS, smem, stream>>>(ts, p);
  if (cudaGetLastError() != cudaSuccess) return MKX_ERR_CUDA;
  h->last_stream = stream;
  return MKX_OK;
}

extern "C" mkx_status mkx_prep_last_error(mkx_prep_handle* h, int* code) {
  if (!h || !code) return MKX_ERR_INVALID_ARG;
  mkx::DeviceScope dev_scope(h->device);
  if (dev_scope.err != cudaSuccess || cudaStreamSynchronize(h->last_stream) != cudaSuccess ||
      cudaMemcpy(code, h->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return MKX_ERR_CUDA;
  return MKX_OK;
}

extern "C" void mkx_prep_destroy(mkx_prep_handle* h) {
  if (!h) return;
  mkx::DeviceScope dev_scope(h->device);
  if (h->wpk) cudaFree(h->wpk);
  if (h->kn) cudaFree(h->kn);
  if (h->status) cudaFree(h->status);
  delete h;
}
