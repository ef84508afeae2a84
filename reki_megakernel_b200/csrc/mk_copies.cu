// Host-to-device copy lists for callers whose inputs sit in pinned host memory (see include/mkx.h).
// A pitched copy moves the same row range of several consecutive layers with one copy-engine
// command: the per-command cost (~3.5 us here) is paid once per run of layers, not once per layer,
// while only the rows a launch reads cross the link.
#include <cstddef>
#include <cuda_runtime.h>

#include "mkx.h"

extern "C" mkx_status mkx_h2d_copies_2d(int n, void* const* dst, const size_t* dpitch, const void* const* src,
                                        const size_t* spitch, const size_t* width, const size_t* height,
                                        cudaStream_t stream) {
  if (n < 0 || (n > 0 && (!dst || !dpitch || !src || !spitch || !width || !height))) return MKX_ERR_INVALID_ARG;
  for (int i = 0; i < n; ++i)
    if (!dst[i] || !src[i] || height[i] < 1 || width[i] > dpitch[i] || width[i] > spitch[i]) return MKX_ERR_INVALID_ARG;
  for (int i = 0; i < n; ++i)
    if (cudaMemcpy2DAsync(dst[i], dpitch[i], src[i], spitch[i], width[i], height[i], cudaMemcpyHostToDevice, stream) !=
        cudaSuccess)
      return MKX_ERR_CUDA;
  return MKX_OK;
}
