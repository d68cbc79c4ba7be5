// peer.cu -- peer-memory plumbing for gathering o shards onto one GPU (C ABI, see bsattn.h).
//
// The attention kernel is persistent: one CTA per SM holding the whole register file and most of
// shared memory.  A gather done with kernels (NCCL send/recv) therefore waits until the attention
// launch ends.  Copy engines need no SM: the root rank exports its output allocation with CUDA
// IPC, every other rank maps it into its own device's context (peer access over NVLink) and
// enqueues device-to-peer copies of each finished chunk of heads while the next chunk computes.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "../../include/bsattn.h"

namespace bsattn_peer {

static_assert(sizeof(cudaIpcMemHandle_t) == BSATTN_IPC_HANDLE_BYTES, "IPC handle size");

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

// cuMemGetAddressRange through the runtime's driver entry point (no link against libcuda).
static AddressRangeFn address_range_fn() {
  static AddressRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddressRangeFn>(ptr);
  });
  return fn;
}

}  // namespace bsattn_peer

extern "C" {

int bsattn_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  if (!ptr || !handle || !offset) return BSATTN_E_NULL;
  bsattn_peer::AddressRangeFn range = bsattn_peer::address_range_fn();
  if (!range) return BSATTN_E_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return BSATTN_E_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return BSATTN_E_CUDA;
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return BSATTN_OK;
}

int bsattn_ipc_open(const void* handle, uint64_t offset, void** ptr) {
  if (!handle || !ptr) return BSATTN_E_NULL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return BSATTN_E_CUDA;
  *ptr = static_cast<char*>(base) + offset;
  return BSATTN_OK;
}

int bsattn_ipc_close(void* ptr, uint64_t offset) {
  if (!ptr) return BSATTN_E_NULL;
  return cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset) == cudaSuccess ? BSATTN_OK
                                                                                 : BSATTN_E_CUDA;
}

int bsattn_peer_copy(void* dst, const void* src, size_t bytes, void* stream) {
  if (!dst || !src) return BSATTN_E_NULL;
  if (bytes == 0) return BSATTN_OK;
  return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)) ==
                 cudaSuccess
             ? BSATTN_OK
             : BSATTN_E_CUDA;
}

}  // extern "C"
