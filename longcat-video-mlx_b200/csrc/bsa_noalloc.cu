// bsa_forward_noalloc: the full BSA call for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc or go through an allocator at the point where they run
// attention: code inside a region whose memory must be fixed in advance, embedders that own the
// whole device budget and forbid allocations from libraries, or hosts that bind this library
// without a device allocator of their own.  bsa_forward needs scratch for the pooled fp32 Q/K
// blocks and the fp32 block-score matrix, which its caller normally passes in.  This variant takes
// that scratch from a fixed array compiled into the library instead, so the caller only passes
// inputs and outputs.
//
// The array is a file-scope __device__ allocation of BSA_NOALLOC_SCRATCH_BYTES (16 MiB): every GPU
// that loads the library holds it until the process exits.  Requests that need more scratch
// (bsa_forward_scratch_bytes > 16 MiB) are rejected with BSA_ERR_SHAPE and a message.
//
// The array's device address is resolved once per device and cached for the life of the process.
// A device reset (cudaDeviceReset) is not supported: it reloads the module, and the cached address
// would then be stale.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <cuda_runtime.h>
#include "bsa_kernels.h"

namespace {

constexpr size_t kScratchBytes = BSA_NOALLOC_SCRATCH_BYTES;

// Shared by every call on a device.  On the host, `g_noalloc_scratch` names a host-side stand-in,
// not the device memory: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[64] = {};  // device address of g_noalloc_scratch, per device ordinal

}  // namespace

extern "C" int bsa_forward_noalloc(const void* q, const void* k, const void* v, int dtype, int B, int H, int S, int D,
                                   const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                                   int T, int Hl, int Wl, int cT, int cH, int cW, int topk, float sm_scale,
                                   const float* rope, int rope_dt, int rope_dh, int rope_dw, int rope_T,
                                   int rope_H, int rope_W, void* q_rot, void* k_rot, int32_t* block_indices,
                                   void* out, const int64_t* out_strides, void* stream) {
  // outputs are checked before the device is touched, so a rejected call has done nothing
  if (!q || !k || !v || !block_indices || !out || !q_strides || !k_strides || !v_strides || !out_strides)
    return bsa::set_error(BSA_ERR_ARG, "bsa_forward_noalloc: null pointer");
  const int64_t need = bsa_forward_scratch_bytes(B, H, S, D, cT, cH, cW);
  if (need > static_cast<int64_t>(kScratchBytes))
    return bsa::set_error(BSA_ERR_SHAPE,
                          "bsa_forward_noalloc: this call needs %lld bytes of scratch (pooled Q/K and score "
                          "matrix), above the library's fixed %zu-byte array; use bsa_forward with "
                          "caller-provided scratch",
                          static_cast<long long>(need), kScratchBytes);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return bsa::set_error(BSA_ERR_CUDA, "bsa_forward_noalloc: no current CUDA device");
  void* scratch = nullptr;
  {
    // one-time set-up per device, with that device current: resolve the array's device address
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p)
        return bsa::set_error(BSA_ERR_CUDA, "bsa_forward_noalloc: cudaGetSymbolAddress failed: %s",
                              cudaGetErrorString(e));
      g_scratch_ptr[dev] = p;
    }
    scratch = g_scratch_ptr[dev];
  }
  // Nothing in the scratch has to start at zero: the pooling kernels overwrite every pooled value
  // before the scoring kernel reads it, so the contents left by the previous call are never used.
  return bsa_forward(q, k, v, dtype, B, H, S, D, q_strides, k_strides, v_strides, T, Hl, Wl, cT, cH, cW, topk,
                     sm_scale, rope, rope_dt, rope_dh, rope_dw, rope_T, rope_H, rope_W, q_rot, k_rot, scratch,
                     block_indices, out, out_strides, stream);
}
