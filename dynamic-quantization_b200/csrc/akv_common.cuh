// Shared device helpers for the packed-KV kernels (sm_100a).
//
// Page format and descriptor encoding are documented in include/anchorkv_b200.h.
// All PTX here is hand-written: bulk copies with mbarrier completion (the
// non-tensor TMA path), legacy-tensor-core mma.sync / movmatrix, and the
// bit tricks that turn packed integers into exact fp16 values.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "anchorkv_b200.h"

namespace akv {

constexpr int kBlock = 16;            // tokens per page (packed_decode.py:109, block=16)
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded waits give up after 2 s

// ---------------------------------------------------------------- page format
__host__ __device__ constexpr int mode_bits(int mode) {
  return mode == AKV_MODE_INT4 ? 4 : (mode == AKV_MODE_INT8 ? 8 : 16);
}
__host__ __device__ inline int desc_mode(int64_t d) { return (int)(d & 3); }
__host__ __device__ inline int desc_ntok(int64_t d) { return (int)((d >> 2) & 15) + 1; }
__host__ __device__ inline int64_t desc_offset(int64_t d) { return (int64_t)((uint64_t)d >> 8); }

// K (or V) payload bytes of one head record.
__host__ __device__ inline int64_t payload_bytes(int D, int mode) {
  return (int64_t)kBlock * D * mode_bits(mode) / 8;
}
// fp16 scales per K (or V) payload.
__host__ __device__ inline int64_t scale_count(int D, int group, int mode) {
  return mode == AKV_MODE_FP16 ? 0 : (int64_t)kBlock * D / group;
}
__host__ __device__ inline int64_t record_bytes(int D, int group, int mode) {
  if (mode == AKV_MODE_SKIP) return 0;
  int64_t b = 2 * payload_bytes(D, mode) + 4 * scale_count(D, group, mode);
  return (b + 15) & ~(int64_t)15;
}

// V payload byte order.  The 16-byte units of a V payload are permuted inside
// each 128-byte line: unit u of the line holding token row r is stored at
// u ^ S(r), with S chosen per row width (D * bits / 8 bytes) so that the
// decode's V fragment loads (lane (g, t) reads row 2t + {0, 1, 8, 9} at column
// g) land in 32 distinct banks.  S depends only on the line, so the map is an
// involution: the same function converts stored <-> row-major offsets.  K
// payloads and all scales stay row-major.
__host__ __device__ constexpr int v_swizzle_key(int row_bytes, int64_t o) {
  return row_bytes == 256   ? (int)(((o >> 9) & 1) | (((o >> 10) & 1) << 2))  // t = row/2 mod 4 -> {0,1,4,5}
         : row_bytes == 128 ? (int)((o >> 7) & 6)                              // row & 6
         : row_bytes == 64  ? (int)((o >> 6) & 6)                              // row & 6 (two rows per line)
                            : (int)((o >> 6) & 2);                             // (row >> 1) & 2 (four rows per line)
}
// Stored offset of row-major byte offset `o` of a V payload (and vice versa).
__host__ __device__ constexpr int64_t v_swizzle(int D, int mode, int64_t o) {
  return mode == AKV_MODE_SKIP ? o : o ^ ((int64_t)v_swizzle_key(D * mode_bits(mode) / 8, o) << 4);
}

// ------------------------------------------------------------------ PTX: sync
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking probe: has phase `parity` completed?
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Plain arrive (count 1) with release semantics.
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Wait for phase `parity` of an mbarrier; gives up after kWaitNs and returns
// false.  Plain try_wait may suspend the warp for a short hardware-defined time
// and returns as soon as the phase completes, so the hand-off stays prompt; the
// clock is read only every 256 probes.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitNs) return false;
  }
}
// Bulk (non-tensor TMA) copy global -> this CTA's shared memory, completing
// `bytes` of transaction count on `bar`.  Addresses 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// --------------------------------------------------------------- PTX: integer
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
// (a & b) ^ c in one LOP3.
__device__ __forceinline__ uint32_t and_xor(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6a;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ------------------------------------------------------------ PTX: f16x2 math
__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
// Pack two floats: lo -> bits 0-15, hi -> bits 16-31 (round to nearest even).
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Exact integer -> fp16 conversions by the magic-exponent trick: an fp16 with
// exponent field 0x19 (value 1024) has unit spacing, so OR-ing an offset-binary
// integer into its mantissa and subtracting the bias is exact.  Each half of
// the result holds one element.
//
// Nibbles at bits 0-3 and 16-19 (two's complement) -> (n_lo, n_hi).
__device__ __forceinline__ uint32_t int4_lo_to_f16x2(uint32_t w) {
  // (w & 0x000F000F) ^ 0x64086408: exponent 1024, nibble xor 8 -> 1024 + n + 8
  return hsub2(and_xor(w, 0x000F000Fu, 0x64086408u), 0x64086408u);  // - 1032
}
// Nibbles at bits 4-7 and 20-23 -> value 1024 + 16 (n + 8); * 1/16 - 72 = n.
__device__ __forceinline__ uint32_t int4_hi_to_f16x2(uint32_t w) {
  return hfma2(and_xor(w, 0x00F000F0u, 0x64806480u), 0x2C002C00u, 0xD480D480u);
}
// Signed bytes at bits 0-7 and 16-23 -> (n_lo, n_hi): 1024 + (n ^ 0x80) - 1152.
__device__ __forceinline__ uint32_t int8_to_f16x2(uint32_t w) {
  return hsub2(and_xor(w, 0x00FF00FFu, 0x64806480u), 0x64806480u);
}

// ------------------------------------------ programmatic dependent launch
// A kernel launched with programmatic stream serialization may start while its
// predecessor in the stream is still running; grid_dependency_wait() returns
// once that predecessor has completed and its memory is visible, and
// allow_dependents_launch() lets this kernel's own successor start early.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependents_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// --------------------------------------------------------- PTX: tensor cores
// D = A(16x16, row) * B(16x8, col) + D, f16 inputs, f32 accumulation.
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Transpose an 8x8 b16 matrix held in the mma fragment layout across the warp.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// ------------------------------------------------------------- dtype helpers
template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Record error bits in the caller's status word.  The word may be device
// memory or mapped pinned host memory (the Python layer keeps it there, so the
// host reads it without synchronising), so this is a plain read-OR-write, not
// an atomic (atomics on host memory are not portable across PCIe hosts): two
// different bits raised at the same moment may leave only one of them, but the
// word is nonzero after any error.  Only error paths call it.
__device__ __forceinline__ void set_status(int32_t *status, int bits) {
  if (!status) return;
  volatile int32_t *w = status;
  const int32_t v = *w;
  if ((v & bits) != bits) *w = v | bits;
  __threadfence_system();
}

// ----------------------------------------------------------- quantizer core
// One group's scale under the two reference semantics.  `divisor` is what the
// values are divided by; `stored` is the fp16 scale written to memory.
//   tensor (backend.py:216-219): s = amax > 0 ? amax/qmax : 1 (fp32); divide by s;
//                                store fp16(s).
//   page (packed_decode.py:61-62): s = fp16(max(amax/qmax, 2^-14)); divide by float(s).
struct GroupScale {
  float divisor;
  __half stored;
};
template <int SEM>
__device__ __forceinline__ GroupScale group_scale(float amax, float qmax) {
  GroupScale g;
  if (SEM == AKV_SEM_TENSOR) {
    const float s = amax > 0.f ? __fdiv_rn(amax, qmax) : 1.f;
    g.divisor = s;
    g.stored = __float2half_rn(s);
  } else {
    const float s = fmaxf(__fdiv_rn(amax, qmax), 6.103515625e-05f);
    g.stored = __float2half_rn(s);
    g.divisor = __half2float(g.stored);
  }
  return g;
}
// round-half-even(x / divisor) clamped to [-qmax, qmax] (torch.round + clamp).
__device__ __forceinline__ int quantize_value(float x, float divisor, float qmax) {
  float q = rintf(__fdiv_rn(x, divisor));
  q = fminf(fmaxf(q, -qmax), qmax);
  return (int)q;
}

}  // namespace akv
