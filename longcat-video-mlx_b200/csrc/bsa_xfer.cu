// Peer exchange helpers for the sequence-parallel (Ulysses) path: device buffers that other
// processes on the node can map (CUDA IPC), and strided copies that the copy engines carry over
// NVLink.  The all-to-all around the BSA call moves [S/P, D] pieces of every head; a 2-D copy
// moves all heads of one peer in one call, and a copy engine does it without taking SMs from the
// attention kernel that runs meanwhile.
//
// These are the only entry points of the library that allocate device memory; the exchange
// allocates its persistent buffers once per process group and shape.
#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>
#include "bsa_b200.h"
#include "bsa_kernels.h"

extern "C" {

int bsa_ipc_alloc(int64_t bytes, void** ptr, unsigned char* handle) {
  if (!ptr || !handle || bytes <= 0) return bsa::set_error(BSA_ERR_ARG, "bsa_ipc_alloc: bad argument");
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, static_cast<size_t>(bytes)) != cudaSuccess)
    return bsa::set_error(BSA_ERR_CUDA, "bsa_ipc_alloc: cudaMalloc(%lld) failed: %s", static_cast<long long>(bytes),
                          cudaGetErrorString(cudaGetLastError()));
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    const cudaError_t e = cudaGetLastError();
    cudaFree(p);
    return bsa::set_error(BSA_ERR_CUDA, "bsa_ipc_alloc: cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == BSA_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return BSA_OK;
}

int bsa_ipc_free(void* ptr) {
  if (!ptr) return BSA_OK;
  if (cudaFree(ptr) != cudaSuccess)
    return bsa::set_error(BSA_ERR_CUDA, "bsa_ipc_free: %s", cudaGetErrorString(cudaGetLastError()));
  return BSA_OK;
}

int bsa_ipc_open(const unsigned char* handle, void** ptr) {
  if (!ptr || !handle) return bsa::set_error(BSA_ERR_ARG, "bsa_ipc_open: bad argument");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return bsa::set_error(BSA_ERR_CUDA, "bsa_ipc_open: %s", cudaGetErrorString(cudaGetLastError()));
  *ptr = p;
  return BSA_OK;
}

int bsa_ipc_close(void* ptr) {
  if (!ptr) return BSA_OK;
  if (cudaIpcCloseMemHandle(ptr) != cudaSuccess)
    return bsa::set_error(BSA_ERR_CUDA, "bsa_ipc_close: %s", cudaGetErrorString(cudaGetLastError()));
  return BSA_OK;
}

int bsa_copy_2d(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
                void* stream) {
  if (!dst || !src) return bsa::set_error(BSA_ERR_ARG, "bsa_copy_2d: null pointer");
  if (width < 0 || height < 0 || dpitch < width || spitch < width)
    return bsa::set_error(BSA_ERR_ARG, "bsa_copy_2d: bad extents");
  if (width == 0 || height == 0) return BSA_OK;
  if (cudaMemcpy2DAsync(dst, static_cast<size_t>(dpitch), src, static_cast<size_t>(spitch), static_cast<size_t>(width),
                        static_cast<size_t>(height), cudaMemcpyDefault,
                        static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return bsa::set_error(BSA_ERR_CUDA, "bsa_copy_2d: %s", cudaGetErrorString(cudaGetLastError()));
  return BSA_OK;
}

int bsa_copy_3d(void* dst, int64_t dpitch, int64_t dslice, const void* src, int64_t spitch, int64_t sslice,
                int64_t width, int64_t height, int64_t depth, void* stream) {
  if (depth == 1) return bsa_copy_2d(dst, dpitch, src, spitch, width, height, stream);
  if (!dst || !src) return bsa::set_error(BSA_ERR_ARG, "bsa_copy_3d: null pointer");
  if (width < 0 || height < 0 || depth < 0 || dpitch < width || spitch < width || dpitch <= 0 || spitch <= 0 ||
      dslice % dpitch || sslice % spitch || dslice < dpitch * height || sslice < spitch * height)
    return bsa::set_error(BSA_ERR_ARG, "bsa_copy_3d: bad extents");
  if (width == 0 || height == 0 || depth == 0) return BSA_OK;
  cudaMemcpy3DParms prm = {};
  prm.srcPtr = make_cudaPitchedPtr(const_cast<void*>(src), static_cast<size_t>(spitch), static_cast<size_t>(width),
                                   static_cast<size_t>(sslice / spitch));
  prm.dstPtr = make_cudaPitchedPtr(dst, static_cast<size_t>(dpitch), static_cast<size_t>(width),
                                   static_cast<size_t>(dslice / dpitch));
  prm.extent = make_cudaExtent(static_cast<size_t>(width), static_cast<size_t>(height), static_cast<size_t>(depth));
  prm.kind = cudaMemcpyDefault;
  if (cudaMemcpy3DAsync(&prm, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return bsa::set_error(BSA_ERR_CUDA, "bsa_copy_3d: %s", cudaGetErrorString(cudaGetLastError()));
  return BSA_OK;
}

int bsa_copy_3d_list(const int64_t* desc, int n, void* stream) {
  if (n < 0 || (n > 0 && !desc)) return bsa::set_error(BSA_ERR_ARG, "bsa_copy_3d_list: bad argument");
  for (int i = 0; i < n; ++i) {
    const int64_t* d = desc + 9 * static_cast<int64_t>(i);
    const int rc = bsa_copy_3d(reinterpret_cast<void*>(d[0]), d[1], d[2], reinterpret_cast<const void*>(d[3]), d[4],
                               d[5], d[6], d[7], d[8], stream);
    if (rc) return rc;
  }
  return BSA_OK;
}

}  // extern "C"
