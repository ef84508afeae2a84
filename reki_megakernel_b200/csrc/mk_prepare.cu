// Cross-attention K/V preparation ("register_prepare", restated; see include/mkx_prepare.h) on
// sm_100a as one tensor-core GEMM over all layers:
//
//   D[f, n] = sum_k Wkv[f, k] * src[n, k]      f over [L][K|V][768] (15,360 rows at REKI's sizes)
//
// One CTA per (128-feature tile, block of <= 256 tokens). Warp 0: producer into an mbarrier ring of up
// to 8 stages: the W tile as one contiguous 16 KB bulk copy from a copy of W packed at create time in
// the 128-byte-swizzled K-major order the MMA reads (tile-contiguous, so HBM sees long bursts), the
// source rows by TMA with the same swizzle. Warp 1: allocates 256 TMEM columns and issues
// tcgen05.mma kind::f16 (M = 128, N = tokens, K = 16 per instruction, bf16 in, fp32 accumulate in
// TMEM), committing each stage back to the producer. Warps 2-5 (one per TMEM lane quarter): read the
// accumulator with tcgen05.ld, transpose it through shared memory (reusing the drained stage ring);
// then all 12 warps, per token, apply the K head RMSNorm (1 + kn) and rotate-half RoPE in fp32,
// round once to bf16 and store rows of the [L][SP][NH][HD] outputs (12 warps: the K tiles' norm and
// RoPE, with their table loads, took 5.4 us after a 14.8 us mainloop with 6). Every wait is bounded by %globaltimer; after a
// timeout the CTA records the error, drains its copies and MMAs, frees TMEM and returns.
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

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *consumed_slot = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = *tmem_slot;
  int issued = 0;

  if (warp == 0 && lane == 0) {
    // producer
    for (int kb = 0; kb < p.ktiles; ++kb) {
      const int s = kb % STAGES;
      if (kb >= STAGES && !wait_bounded(&empty[s], ((kb / STAGES) & 1) ^ 1, p.timeout_ns)) {
        record(p, 0x100 | 1);
        break;
      }
      char* a = ring + s * stage_bytes;
      mbar_expect_tx(&full[s], (uint32_t)stage_bytes);
      bulk_g2s(a, p.wpk + ((size_t)tile * p.ktiles + kb) * (A_BYTES / 2), (uint32_t)A_BYTES, &full[s]);
      tma_load_2d(a + A_BYTES, &ts, kb * BK, tok0, &full[s]);
      issued = kb + 1;
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
  ok = __syncthreads_and(ok);  // all roles done; the tile is complete (or a wait failed)
  // Epilogue, part 2 (all 12 warps): one (token, head) row per half-warp; lane j holds dims 4j..4j+3.
  // K: head RMSNorm (shuffle reduction over the 16 lanes) * (1 + kn), rotate-half RoPE (partner dims
  // d +- 32 sit in lane j ^ 8); V: as is. One bf16 rounding, 8-byte stores (128 B per row).
  if (ok) {
    const int l = tile / TILES_PER_LAYER, within = tile % TILES_PER_LAYER;
    const bool is_k = within < TILES_PER_LAYER / 2;
    const int h0 = 2 * (within % (TILES_PER_LAYER / 2));
    uint16_t* out = is_k ? p.k_out : p.v_out;
    const int half = lane >> 4, j = lane & 15;
    const float4 kn = __ldg(reinterpret_cast<const float4*>(p.kn + (size_t)l * HD) + j);
    const int nvalid = min(p.ntok, p.S - tok0);
    const int nitems = 2 * nvalid, nw = NTHREADS / 32;
    // item = 2 * token + head half; each warp takes two consecutive items per round
    auto tables = [&](int it, float4& c, float4& sn) {
      if (is_k && it < nitems) {
        const size_t n = (size_t)(tok0 + (it >> 1));
        c = __ldg(reinterpret_cast<const float4*>(p.cos + n * HD) + j);
        sn = __ldg(reinterpret_cast<const float4*>(p.sin + n * HD) + j);
      }
    };
    // rounds of this warp: items 2 * warp + half + 2 * nw * r; the cos/sin rows of round r + PF are
    // loaded while round r is processed (an L2 round trip spans several rounds)
    constexpr int PF = 8;
    const int rounds = nitems > 2 * warp ? (nitems - 2 * warp + 2 * nw - 1) / (2 * nw) : 0;
    const int it0 = 2 * warp + half;
    float4 c[PF], sn[PF];
#pragma unroll
    for (int u = 0; u < PF; ++u) {
      c[u] = sn[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      tables(it0 + 2 * nw * u, c[u], sn[u]);
    }
    for (int r0 = 0; r0 < rounds; r0 += PF) {
#pragma unroll
      for (int u = 0; u < PF; ++u) {
        const int r = r0 + u;
        if (r >= rounds) break;  // warp-uniform: the shuffles need all lanes
        const int it = it0 + 2 * nw * r;
        const bool valid = it < nitems;
        const int nl = it >> 1, hh = it & 1;
        float4 y = valid ? *reinterpret_cast<const float4*>(tsm + nl * TS + 64 * hh + 4 * j)
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        if (is_k) {
          float ss = fmaf(y.x, y.x, fmaf(y.y, y.y, fmaf(y.z, y.z, y.w * y.w)));
#pragma unroll
          for (int o = 8; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          const float rstd = rsqrtf(ss / (float)HD + p.eps);
          y.x = y.x * rstd * (1.f + kn.x);
          y.y = y.y * rstd * (1.f + kn.y);
          y.z = y.z * rstd * (1.f + kn.z);
          y.w = y.w * rstd * (1.f + kn.w);
          const float sg = j < 8 ? -1.f : 1.f;  // rot[d] = -y[d + 32] for d < 32, y[d - 32] above
          const float px = __shfl_xor_sync(0xffffffffu, y.x, 8), py = __shfl_xor_sync(0xffffffffu, y.y, 8);
          const float pz = __shfl_xor_sync(0xffffffffu, y.z, 8), pw = __shfl_xor_sync(0xffffffffu, y.w, 8);
          const float4 cc = c[u], ss4 = sn[u];
          y = make_float4(fmaf(y.x, cc.x, sg * px * ss4.x), fmaf(y.y, cc.y, sg * py * ss4.y),
                          fmaf(y.z, cc.z, sg * pz * ss4.z), fmaf(y.w, cc.w, sg * pw * ss4.w));
          tables(it + 2 * nw * PF, c[u], sn[u]);
        }
        if (valid) {
          uint2* dst = reinterpret_cast<uint2*>(out + (((size_t)l * p.SP + tok0 + nl) * NH + h0 + hh) * HD) + j;
          *dst = make_uint2(pack_bf2(y.x, y.y), pack_bf2(y.z, y.w));
        }
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
      (reinterpret_cast<uintptr_t>(v_out) & 15) != 0)
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
