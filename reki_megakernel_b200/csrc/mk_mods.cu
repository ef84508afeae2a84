// Per-step modulation rows ("_step_modulations", restated; see include/mkx_mods.h) on sm_100a.
//
// Two launches per call:
//   cond_kernel  a[s][h] = bf16(silu(8 (W_t temb_s + W_s state)))  for s < N (rows N..15 zero), and
//                dt = 1/N. 96 CTAs of 8 warps, one column h per warp, the 16 step sums as independent
//                fp32 chains over a timestep-embedding table built once at create (in double: the
//                angles reach 1000 rad), then reduced across the lanes.
//   proj_kernel  mods[s][r] = bf16(W_m[r] . a[s] + b_m[r]): one persistent CTA of 16 warps per SM,
//                each CTA a contiguous run of 16-row m-tiles (balanced to within one m-tile per SM).
//                W_m was repacked at create time into mma.sync A-fragment order, so a lane's
//                fragment of one 16x16 block is one 16-byte non-caching load and a warp reads
//                512 contiguous bytes per block; k-blocks stream in chunks of 8, the next chunk in
//                flight while the current one is multiplied (mma.sync m16n8k16 bf16, fp32
//                accumulate) against a[16][768] held in shared memory. HBM-bound: the 108.5 MB of
//                W_m cross HBM once per call for all N steps. Launched as a programmatic dependent
//                of cond_kernel: each warp's first two chunks are in flight before it waits
//                (griddepcontrol.wait) for `act`.
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
constexpr int CH = 8;                  // projection: k-blocks per streamed chunk
constexpr int NCH = KB / CH;           // chunks per m-tile
constexpr int PW = 16, PT = PW * 32;   // projection: warps / threads per CTA
static_assert(KB % CH == 0, "chunks tile an m-tile");
constexpr int AS = H + 8;              // shared activation row stride (bf16): conflict-free B fragments
constexpr int CW = 8, CT = CW * 32;    // conditioning: warps (= columns h) / threads per CTA
constexpr int TDIM_MAX = 512, SDIM_MAX = 64;

// 16-byte read-only load that bypasses L1 (every W_m byte is used once per call).
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// Asks L2 to fetch `bytes` (a multiple of 16) from `src` (16-byte aligned); no data comes back.
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Timestep-embedding table of every step count, built once at create: temb[N - 1][s][tdim] =
// [cos(1000 t_s f_i) | sin(1000 t_s f_i)], t_s = 1 - s/N, f_i = 10000^(-i/(tdim/2)), in double
// (the angles reach 1000 rad), rounded once to fp32.
__global__ void temb_table_kernel(float* __restrict__ tab, int tdim) {
  const int half = tdim / 2;
  const int total = NMAX * NMAX * half;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
    const int i = e % half, s = (e / half) % NMAX, n = e / (half * NMAX) + 1;
    float* row = tab + ((size_t)(n - 1) * NMAX + s) * tdim;
    if (s >= n) {
      row[i] = 0.f;
      row[half + i] = 0.f;
      continue;
    }
    const double t = (double)(n - s) / (double)n;
    const double ang = 1000.0 * t * exp(-log(10000.0) * (double)i / (double)half);
    double sn, cs;
    sincos(ang, &sn, &cs);
    row[i] = (float)cs;
    row[half + i] = (float)sn;
  }
}

// Conditioning: warp w owns column h = 8 blockIdx.x + w; lane l holds W_t[h][l + 32 q]. The 16 step
// sums accumulate side by side (independent fp32 chains) over the table rows of this N (staged in
// shared memory), then reduce
// across the lanes; lane s finishes step s. Lets the projection launch at once (it streams W_m
// while this runs and waits for `act` only where it reads it).
__global__ void __launch_bounds__(CT) cond_kernel(const float* __restrict__ w_t, const float* __restrict__ w_s,
                                                  const float* __restrict__ state, const float* __restrict__ temb,
                                                  int N, int tdim, int sdim, uint16_t* __restrict__ act,
                                                  float* __restrict__ dt_out) {
  extern __shared__ float4 tsm4[];  // this N's table rows [N][tdim]
  float* tsm = reinterpret_cast<float*>(tsm4);
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x * CW + warp;
  const int per = tdim / 32;
  const float4* tb = reinterpret_cast<const float4*>(temb + (size_t)(N - 1) * NMAX * tdim);
  for (int e = threadIdx.x; e < N * tdim / 4; e += CT) tsm4[e] = __ldg(tb + e);
  float wr[TDIM_MAX / 32];
#pragma unroll
  for (int q = 0; q < TDIM_MAX / 32; ++q) wr[q] = q < per ? __ldg(w_t + (size_t)h * tdim + lane + 32 * q) : 0.f;
  float st = lane < sdim ? __ldg(w_s + (size_t)h * sdim + lane) * __ldg(state + lane) : 0.f;
  if (lane + 32 < sdim) st += __ldg(w_s + (size_t)h * sdim + lane + 32) * __ldg(state + lane + 32);
  __syncthreads();
  float acc[NMAX];
#pragma unroll
  for (int s = 0; s < NMAX; ++s) acc[s] = st;
#pragma unroll
  for (int q = 0; q < TDIM_MAX / 32; ++q) {
    if (q < per) {
#pragma unroll
      for (int s = 0; s < NMAX; ++s)
        if (s < N) acc[s] = fmaf(wr[q], tsm[s * tdim + lane + 32 * q], acc[s]);
    }
  }
  float mine = 0.f;
#pragma unroll
  for (int s = 0; s < NMAX; ++s) {
    if (s < N) {  // uniform
      float v = acc[s];
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == s) mine = v;
    }
  }
  if (lane < NMAX) {
    const float e8 = 8.f * mine;
    const float a = lane < N ? e8 / (1.f + expf(-e8)) : 0.f;
    act[lane * H + h] = (uint16_t)(pack_bf2(a, 0.f) & 0xffffu);
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *dt_out = 1.f / (float)N;
}

__global__ void __launch_bounds__(PT, 1) proj_kernel(const uint4* __restrict__ wpk, const float* __restrict__ bias,
                                                     const uint16_t* __restrict__ act, int N, int MODW,
                                                     uint16_t* __restrict__ out) {
  __shared__ __align__(16) uint16_t xs[NMAX * AS];
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
  // The first two chunks stream while the conditioning launch finishes (programmatic dependency);
  // `act` is read only after griddepcontrol.wait.
  if (nchunks > 0) load(ba, 0);
  if (nchunks > 1) load(bb, 1);
  if (lane == 0 && mine > 0) prefetch_l2(wpk + (size_t)(mt0 + warp) * KB * 32, KB * 512);  // first m-tile
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int e = threadIdx.x; e < NMAX * H / 8; e += PT) {
    const int row = e / (H / 8), c8 = e - row * (H / 8);
    *reinterpret_cast<uint4*>(xs + row * AS + c8 * 8) = *reinterpret_cast<const uint4*>(act + row * H + c8 * 8);
  }
  __syncthreads();
  for (int c = 0; c < nchunks; c += 2) {
    if (c > 0 && c + 1 < nchunks) load(bb, c + 1);
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
  float* temb;     // [16 step counts][16][tdim] fp32 timestep-embedding table
  int* status;     // device error word (a projection wait that ran out of time)
  unsigned long long timeout_ns;
  cudaStream_t last_stream;
};

using namespace mkxm;

extern "C" int mkx_mods_width(const mkx_mods_handle* h) { return h ? h->MODW : 0; }

extern "C" mkx_status mkx_mods_input(mkx_mods_handle* h, uint16_t* dst, cudaStream_t stream) {
  if (!h || !dst) return MKX_ERR_INVALID_ARG;
  mkx::DeviceScope dev_scope(h->device);
  if (dev_scope.err != cudaSuccess ||
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
  mkx::DeviceScope dev_scope(device);
  if (dev_scope.err != cudaSuccess) return MKX_ERR_CUDA;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return MKX_ERR_CUDA;
  mkx_mods_handle* h = new (std::nothrow) mkx_mods_handle();
  if (!h) return MKX_ERR_RESOURCES;
  memset(h, 0, sizeof(*h));
  h->d = d;
  h->device = device;
  h->MODW = 9 * d.L * H + 2 * H;
  h->grid = sms < h->MODW / 16 ? sms : h->MODW / 16;
  h->timeout_ns = 2000000000ull;
  const size_t nt = (size_t)H * d.tdim, ns = (size_t)H * d.sdim, nm = (size_t)h->MODW * H;
  bool ok = cudaMalloc(&h->w_t, nt * 4) == cudaSuccess && cudaMalloc(&h->w_s, ns * 4) == cudaSuccess &&
            cudaMalloc(&h->wpk, nm * 2) == cudaSuccess && cudaMalloc(&h->b_m, (size_t)h->MODW * 4) == cudaSuccess &&
            cudaMalloc(&h->act, (size_t)NMAX * H * 2) == cudaSuccess &&
            cudaMalloc(&h->temb, (size_t)NMAX * NMAX * d.tdim * 4) == cudaSuccess &&
            cudaMalloc(&h->status, sizeof(int)) == cudaSuccess && cudaMemset(h->status, 0, sizeof(int)) == cudaSuccess &&

            cudaMemcpy(h->w_t, w_t, nt * 4, cudaMemcpyDeviceToDevice) == cudaSuccess &&
            cudaMemcpy(h->w_s, w_s, ns * 4, cudaMemcpyDeviceToDevice) == cudaSuccess &&
            cudaMemcpy(h->b_m, b_m, (size_t)h->MODW * 4, cudaMemcpyDeviceToDevice) == cudaSuccess;
  if (ok) {
    mods_pack_kernel<<<1184, 256>>>(w_m, h->wpk, h->MODW);
    temb_table_kernel<<<64, 256>>>(h->temb, d.tdim);
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
  mkx::DeviceScope dev_scope(h->device);
  if (dev_scope.err != cudaSuccess) return MKX_ERR_CUDA;
  cond_kernel<<<H / CW, CT, (size_t)N * h->d.tdim * 4, stream>>>(h->w_t, h->w_s, state, h->temb, N, h->d.tdim, h->d.sdim, h->act, dt_out);
  if (cudaGetLastError() != cudaSuccess) return MKX_ERR_CUDA;
  // programmatic dependent launch: the projection may start while the conditioning runs
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(h->grid);
  cfg.blockDim = dim3(PT);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, proj_kernel, reinterpret_cast<const uint4*>(h->wpk), (const float*)h->b_m,
                         (const uint16_t*)h->act, N, h->MODW, mods_out) != cudaSuccess)
    return MKX_ERR_CUDA;
  h->last_stream = stream;
  return MKX_OK;
}

extern "C" mkx_status mkx_mods_last_error(mkx_mods_handle* h, int* code) {
  if (!h || !code) return MKX_ERR_INVALID_ARG;
  mkx::DeviceScope dev_scope(h->device);
  if (dev_scope.err != cudaSuccess || cudaStreamSynchronize(h->last_stream) != cudaSuccess ||
      cudaMemcpy(code, h->status, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return MKX_ERR_CUDA;
  return MKX_OK;
}

extern "C" void mkx_mods_destroy(mkx_mods_handle* h) {
  if (!h) return;
  mkx::DeviceScope dev_scope(h->device);
  if (h->w_t) cudaFree(h->w_t);
  if (h->w_s) cudaFree(h->w_s);
  if (h->wpk) cudaFree(h->wpk);
  if (h->b_m) cudaFree(h->b_m);
  if (h->act) cudaFree(h->act);
  if (h->status) cudaFree(h->status);
  if (h->temb) cudaFree(h->temb);
  delete h;
}
