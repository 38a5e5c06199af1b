// Host-only helpers of the C ABI: status strings, ABI version, record sizes.
#include "akv_common.cuh"

extern "C" const char *akv_status_string(int status) {
  switch (status) {
    case AKV_OK: return "ok";
    case AKV_ERR_INVALID: return "invalid argument (null pointer, size, alignment or dtype)";
    case AKV_ERR_UNSUPPORTED: return "unsupported geometry (head_dim must be 64 or 128; group a supported power of two)";
    case AKV_ERR_CUDA: return "CUDA launch error";
    case AKV_ERR_SCRATCH:
      return "request exceeds the fixed 8 MiB scratch of akv_packed_attention_static "
             "(akv_workspace_bytes of the call); use akv_packed_attention with a workspace";
    default: return "unknown status";
  }
}

// 3: V payloads stored in the bank-swizzled byte order (records of version 2 read differently).
// 4: exchange buffers hold both epoch parities (akv_exchange_bytes doubled);
//    akv_repack_pages takes the quantizer semantics, akv_unpack_pages the output dtype;
//    status words may live in mapped pinned host memory (akv_status_alloc).
extern "C" int akv_abi_version(void) { return 5; }

// The status word in mapped pinned host memory: kernels write it through the
// device address, the host reads it through the host address with no copy or
// synchronisation.
extern "C" int akv_status_alloc(void **host_ptr, void **dev_ptr) {
  if (!host_ptr || !dev_ptr) return AKV_ERR_INVALID;
  void *h = nullptr;
  if (cudaHostAlloc(&h, 64, cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) return AKV_ERR_CUDA;
  void *d = nullptr;
  if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess) {
    cudaFreeHost(h);
    return AKV_ERR_CUDA;
  }
  *(volatile int32_t *)h = 0;
  *host_ptr = h;
  *dev_ptr = d;
  return AKV_OK;
}

extern "C" int akv_status_free(void *host_ptr) {
  if (!host_ptr) return AKV_ERR_INVALID;
  return cudaFreeHost(host_ptr) == cudaSuccess ? AKV_OK : AKV_ERR_CUDA;
}

extern "C" int64_t akv_record_bytes(int head_dim, int group, int mode) {
  if (head_dim <= 0 || group <= 0 || (16 * head_dim) % group) return -1;
  if (mode < AKV_MODE_SKIP || mode > AKV_MODE_FP16) return -1;
  return akv::record_bytes(head_dim, group, mode);
}
