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
extern "C" int akv_abi_version(void) { return 3; }

extern "C" int64_t akv_record_bytes(int head_dim, int group, int mode) {
  if (head_dim <= 0 || group <= 0 || (16 * head_dim) % group) return -1;
  if (mode < AKV_MODE_SKIP || mode > AKV_MODE_FP16) return -1;
  return akv::record_bytes(head_dim, group, mode);
}
