// Per-step modulation rows ("_step_modulations", restated; see include/mkx_mods.h) on sm_100a.
//
// Two launches per call:
//   cond_kernel  a[s][h] = bf16(silu(8 (W_t temb_s + W_s state)))  for s < N (rows N..15 zero), and
//                dt = 1/N. 24 CTAs of 8 warps; the embedding in double (angles up to 1000 rad), then a
//                warp owns 4 columns h, keeps its W_t row slices in registers and reduces each (s, h)
//                dot product (fp32) across the lanes.
//   proj_kernel  mods[s][r] = bf16(W_m[r] . a[s] + b_m[r]): one persistent CTA of 16 warps per SM,
//                each CTA a contiguous run of 16-row m-tiles (balanced to within one m-tile per SM).
//                W_m was repacked at create time into mma.sync A-fragment order, so a lane's
//                fragment of one 16x16 block is one 16-byte non-caching load and a warp reads
//                512 contiguous bytes per block; k-blocks stream in chunks of 8, the next chunk in
//                flight while the current one is multiplied (mma.sync m16n8k16 bf16, fp32
//                accumulate) against a[16][768] held in shared memory. HBM-bound: the 108.5 MB of
//                W_m cross HBM once per call for all N steps.
#include <cstdint>
#include <cstring>
#include <new>
#include <cuda_runtime.h>

#include "mkx_mods.h"
#include "mkx_device.cuh"

namespace mkxm {
using namespace mkx;

constexpr int H = 768;
constexpr int NMAX = 16;               // steps per call: two n-tiles of 8
constexpr int KB = H / 16;             // 16-wide k-blocks per row
constexpr int CH = 8;                  // k-blocks per streamed chunk
constexpr int NCH = KB / CH;           // chunks per m-tile
constexpr int PW = 16, PT = PW * 32;   // projection: warps / threads per CTA
constexpr int AS = H + 8;              // shared activation row stride (bf16): conflict-free B fragments
constexpr int CW = 8, CT = CW * 32;    // conditioning: warps / threads per CTA
constexpr int CCOLS = 32;              // conditioning: columns h per CTA (4 per warp)
constexpr int TDIM_MAX = 512, SDIM_MAX = 64;
static_assert(KB % CH == 0, "chunks tile an m-tile");

// 16-byte read-only load that bypasses L1 (every W_m byte is used once per call).
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__global__ void __launch_bounds__(CT) cond_kernel(const float* __restrict__ w_t, const float* __restrict__ w_s,
                                                  const float* __restrict__ state, int N, int tdim, int sdim,
                                                  uint16_t* __restrict__ act, float* __restrict__ dt_out) {
  __shared__ float temb[NMAX * TDIM_MAX];  // [N][tdim]: cos half, then sin half
  const int half = tdim / 2;
  // The angles reach 1000 rad: computed (and reduced) in double, so the embedding carries only its
  // fp32 rounding (an fp32 angle would be off by ~2e-4 rad). N x tdim/2 values per CTA, negligible.
  for (int e = threadIdx.x; e < N * half; e += CT) {
    const int s = e / half, i = e - s * half;
    const double t = 1.0 - (double)s / (double)N;
    const double f = exp(-log(10000.0) * (double)i / (double)half);
    double sn, cs;
    sincos(1000.0 * t * f, &sn, &cs);
    temb[s * tdim + i] = (float)cs;
    temb[s * tdim + half + i] = (float)sn;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = tdim / 32;  // W_t values per lane
  for (int j = 0; j < CCOLS / CW; ++j) {
    const int h = blockIdx.x * CCOLS + warp + CW * j;
    float wr[TDIM_MAX / 32];
#pragma unroll
    for (int q = 0; q < TDIM_MAX / 32; ++q) wr[q] = q < per ? __ldg(w_t + (size_t)h * tdim + lane + 32 * q) : 0.f;
    const float st = lane < sdim ? __ldg(w_s + (size_t)h * sdim + lane) * __ldg(state + lane) : 0.f;
    const float st2 = lane + 32 < sdim ? __ldg(w_s + (size_t)h * sdim + lane + 32) * __ldg(state + lane + 32) : 0.f;
    for (int s = 0; s < NMAX; ++s) {
      float acc = 0.f;
      if (s < N) {
        acc = st + st2;
#pragma unroll
        for (int q = 0; q < TDIM_MAX / 32; ++q)
          if (q < per) acc = fmaf(wr[q], temb[s * tdim + lane + 32 * q], acc);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      }
      if (lane == 0) {
        const float e8 = 8.f * acc;
        const float a = s < N ? e8 / (1.f + expf(-e8)) : 0.f;
        act[s * H + h] = (uint16_t)(pack_bf2(a, 0.f) & 0xffffu);
      }
    }
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *dt_out = 1.f / (float)N;
}

__global__ void __launch_bounds__(PT, 1) proj_kernel(const uint4* __restrict__ wpk, const float* __restrict__ bias,
                                                     const uint16_t* __restrict__ act, int N, int MODW,
                                                     uint16_t* __restrict__ out) {
  __shared__ __align__(16) uint16_t xs[NMAX * AS];
  for (int e = threadIdx.x; e < NMAX * H / 8; e += PT) {
    const int row = e / (H / 8), c8 = e - row * (H / 8);
    *reinterpret_cast<uint4*>(xs + row * AS + c8 * 8) = *reinterpret_cast<const uint4*>(act + row * H + c8 * 8);
  }
  __syncthreads();
  const int MT = MODW / 16;
  const int mt0 = (int)((long long)blockIdx.x * MT / gridDim.x);
  const int mt1 = (int)((long long)(blockIdx.x + 1) * MT / gridDim.x);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, cc = lane & 3;
  const bool two = N > 8;
  const int nm = mt1 - mt0;
  const int mine = nm > warp ? (nm - warp + PW - 1) / PW : 0;  // m-tiles mt0 + warp + PW j
  const int nchunks = mine * NCH;
  const char* x0 = reinterpret_cast<const char*>(xs) + (size_t)g * AS * 2 + cc * 4;
  const char* x1 = x0 + (size_t)8 * AS * 2;
  auto chunk_src = [&](int c) {
    const int j = c / NCH, kc = c - j * NCH;
    const int mt = mt0 + warp + PW * j;
    return wpk + ((size_t)mt * KB + kc * CH) * 32 + lane;
  };
  float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
  auto epilogue = [&](int mt) {
    // d0: steps 2cc, 2cc+1 of rows g, g+8; d1: steps 8 + those. Lanes g and g ^ 1 hold adjacent
    // rows: the even-g lane stores the pair as one 32-bit word.
    const int r0 = mt * 16 + g;
    const float b0 = __ldg(bias + r0), b8 = __ldg(bias + r0 + 8);
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const float* d = h2 ? d1 : d0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int s = 8 * h2 + 2 * cc + (q & 1), r = r0 + (q >> 1) * 8;
        const float v = d[q] + ((q >> 1) ? b8 : b0);
        const float o = __shfl_xor_sync(0xffffffffu, v, 4);
        if ((g & 1) == 0 && s < N) *reinterpret_cast<uint32_t*>(out + (size_t)s * MODW + r) = pack_bf2(v, o);
      }
    }
  };
  auto compute = [&](const uint4 (&b)[CH], int c) {
    const int kc = c % NCH;
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      const int kb = kc * CH + i;
      mma_bf16(d0, b[i].x, b[i].y, b[i].z, b[i].w, lds32(x0 + kb * 32), lds32(x0 + kb * 32 + 16));
      if (two) mma_bf16(d1, b[i].x, b[i].y, b[i].z, b[i].w, lds32(x1 + kb * 32), lds32(x1 + kb * 32 + 16));
    }
    if (kc == NCH - 1) {
      epilogue(mt0 + warp + PW * (c / NCH));
#pragma unroll
      for (int q = 0; q < 4; ++q) d0[q] = d1[q] = 0.f;
    }
  };
  uint4 ba[CH], bb[CH];
  auto load = [&](uint4 (&b)[CH], int c) {
    const uint4* p = chunk_src(c);
#pragma unroll
    for (int i = 0; i < CH; ++i) b[i] = ldg_stream(p + i * 32);
  };
  if (nchunks > 0) load(ba, 0);
  for (int c = 0; c < nchunks; c += 2) {
    if (c + 1 < nchunks) load(bb, c + 1);
    compute(ba, c);
    if (c + 1 >= nchunks) break;
    if (c + 2 < nchunks) load(ba, c + 2);
    compute(bb, c + 1);
  }
}

// W_m [MODW][H] row-major -> fragment order: block (m-tile mt, k-block kb) is 32 lanes x 4 words;
// lane g*4 + cc holds {A[g][2cc..], A[g+8][2cc..], A[g][2cc+8..], A[g+8][2cc+8..]} (two bf16 each,
// lower k in the low half), the m16n8k16 A-fragment registers a0..a3.
__global__ void mods_pack_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int MODW) {
  const long long total = (long long)MODW * H;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(e / H), k = (int)(e - (long long)r * H);
    const int mt = r >> 4, rr = r & 15, kb = k >> 4, kk = k & 15;
    const int lane = (rr & 7) * 4 + ((kk & 7) >> 1);
    const int reg = (rr >> 3) + 2 * (kk >> 3);
    dst[((((long long)mt * KB + kb) * 32 + lane) * 4 + reg) * 2 + (kk & 1)] = src[e];
  }
}

}  // namespace mkxm

struct mkx_mods_handle {
  mkx_mods_dims d;
  int device;
  int MODW;
  int grid;
  float* w_t;      // owned copies
  float* w_s;
  uint16_t* wpk;   // W_m in fragment order
  float* b_m;
  uint16_t* act;   // [16][H] bf16 conditioning output
};

using namespace mkxm;

extern "C" int mkx_mods_width(const mkx_mods_handle* h) { return h ? h->MODW : 0; }

extern "C" mkx_status mkx_mods_input(mkx_mods_handle* h, uint16_t* dst, cudaStream_t stream) {
  if (!h || !dst) return MKX_ERR_INVALID_ARG;
  if (cudaSetDevice(h->device) != cudaSuccess ||
      cudaMemcpyAsync(dst, h->act, (size_t)NMAX * H * 2, cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
    return MKX_ERR_CUDA;
  return MKX_OK;
}

extern "C" mkx_status mkx_mods_create(const mkx_mods_dims* dims, const float* w_t, const float* w_s, const uint16_t* w_m,
                                      const float* b_m, int device, mkx_mods_handle** out) {
  if (!dims || !w_t || !w_s || !w_m || !b_m || !out) return MKX_ERR_INVALID_ARG;
  *out = nullptr;
  const mkx_mods_dims d = *dims;
  if (d.H != H || d.L < 1 || d.L > 64 || d.tdim < 64 || d.tdim > TDIM_MAX || d.tdim % 64 != 0 || d.sdim < 1 ||
      d.sdim > SDIM_MAX)
    return MKX_ERR_UNSUPPORTED;
  if (cudaSetDevice(device) != cudaSuccess) return MKX_ERR_CUDA;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return MKX_ERR_CUDA;
  mkx_mods_handle* h = new (std::nothrow) mkx_mods_handle();
  if (!h) return MKX_ERR_RESOURCES;
  memset(h, 0, sizeof(*h));
  h->d = d;
  h->device = device;
  h->MODW = 9 * d.L * H + 2 * H;
  h->grid = sms < h->MODW / 16 ? sms : h->MODW / 16;
  const size_t nt = (size_t)H * d.tdim, ns = (size_t)H * d.sdim, nm = (size_t)h->MODW * H;
  bool ok = cudaMalloc(&h->w_t, nt * 4) == cudaSuccess && cudaMalloc(&h->w_s, ns * 4) == cudaSuccess &&
            cudaMalloc(&h->wpk, nm * 2) == cudaSuccess && cudaMalloc(&h->b_m, (size_t)h->MODW * 4) == cudaSuccess &&
            cudaMalloc(&h->act, (size_t)NMAX * H * 2) == cudaSuccess &&
            cudaMemcpy(h->w_t, w_t, nt * 4, cudaMemcpyDeviceToDevice) == cudaSuccess &&
            cudaMemcpy(h->w_s, w_s, ns * 4, cudaMemcpyDeviceToDevice) == cudaSuccess &&
            cudaMemcpy(h->b_m, b_m, (size_t)h->MODW * 4, cudaMemcpyDeviceToDevice) == cudaSuccess;
  if (ok) {
    mods_pack_kernel<<<1184, 256>>>(w_m, h->wpk, h->MODW);
    ok = cudaGetLastError() == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
  }
  if (!ok) {
    mkx_mods_destroy(h);
    return MKX_ERR_CUDA;
  }
  *out = h;
  return MKX_OK;
}

extern "C" mkx_status mkx_mods_run(mkx_mods_handle* h, int N, const float* state, uint16_t* mods_out, float* dt_out,
                                   cudaStream_t stream) {
  if (!h || !state || !mods_out || !dt_out) return MKX_ERR_INVALID_ARG;
  if (N < 1 || N > NMAX) return MKX_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(mods_out) & 3) != 0) return MKX_ERR_INVALID_ARG;
  if (cudaSetDevice(h->device) != cudaSuccess) return MKX_ERR_CUDA;
  cond_kernel<<<H / CCOLS, CT, 0, stream>>>(h->w_t, h->w_s, state, N, h->d.tdim, h->d.sdim, h->act, dt_out);
  if (cudaGetLastError() != cudaSuccess) return MKX_ERR_CUDA;
  proj_kernel<<<h->grid, PT, 0, stream>>>(reinterpret_cast<const uint4*>(h->wpk), h->b_m, h->act, N, h->MODW, mods_out);
  if (cudaGetLastError() != cudaSuccess) return MKX_ERR_CUDA;
  return MKX_OK;
}

extern "C" void mkx_mods_destroy(mkx_mods_handle* h) {
  if (!h) return;
  cudaSetDevice(h->device);
  if (h->w_t) cudaFree(h->w_t);
  if (h->w_s) cudaFree(h->w_s);
  if (h->wpk) cudaFree(h->wpk);
  if (h->b_m) cudaFree(h->b_m);
  if (h->act) cudaFree(h->act);
  delete h;
}
