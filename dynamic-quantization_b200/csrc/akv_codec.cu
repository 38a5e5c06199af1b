// Block codec kernels: symmetric INT8 / packed INT4 with fp16 absmax scales.
//
// Bit-exact with the reference quantizers (backend.py:183-226 quantize_tensor,
// packed_decode.py:48-67 pack_page) because every step is an IEEE operation
// with the same rounding: fp32 absmax, correctly rounded fp32 division
// (__fdiv_rn; this file must never be built with fast-math), round half to
// even (rintf), clamp, and fp16 round-to-nearest-even for the scales.  The
// page kernels move a 16-token slab per warp with 16-byte vector loads, keep
// the slab in registers, reduce the group absmax with warp shuffles and write
// coalesced payload words.
#include <algorithm>
#include <type_traits>

#include "akv_common.cuh"

namespace akv {

// ============================================================ flat tensors
// One warp per group of `group` consecutive elements (grid-stride).
template <typename T, int BITS, int SEM>
__global__ void __launch_bounds__(256) quantize_flat_kernel(const T *__restrict__ src, int64_t numel,
                                                            int64_t group, int64_t ngroups,
                                                            uint8_t *__restrict__ payload,
                                                            __half *__restrict__ scales) {
  const float qmax = BITS == 8 ? 127.f : 7.f;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  auto value = [&](int64_t e) -> float {
    if (e >= numel) return 0.f;  // zero padding of the tail group (backend.py:211-213)
    float x = to_f32<T>(src[e]);
    if (SEM == AKV_SEM_PAGE) x = __half2float(__float2half_rn(x));  // pack_page rounds to fp16 first
    return x;
  };
  for (int64_t g = warp; g < ngroups; g += nwarps) {
    const int64_t base = g * group;
    float amax = 0.f;
    for (int64_t i = lane; i < group; i += 32) amax = fmaxf(amax, fabsf(value(base + i)));
#pragma unroll
    for (int off = 16; off; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const GroupScale s = group_scale<SEM>(amax, qmax);
    if (BITS == 8) {
      int8_t *q = reinterpret_cast<int8_t *>(payload);
      for (int64_t i = lane; i < group; i += 32)
        q[base + i] = (int8_t)quantize_value(value(base + i), s.divisor, qmax);
    } else {
      for (int64_t i = lane; i < group / 2; i += 32) {
        const int lo = quantize_value(value(base + 2 * i), s.divisor, qmax);
        const int hi = quantize_value(value(base + 2 * i + 1), s.divisor, qmax);
        payload[base / 2 + i] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
      }
    }
    if (lane == 0) scales[g] = s.stored;
  }
}

template <typename T, int BITS>
__global__ void __launch_bounds__(256) dequantize_flat_kernel(const uint8_t *__restrict__ payload,
                                                              const __half *__restrict__ scales,
                                                              int64_t numel, int64_t group,
                                                              T *__restrict__ out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < numel; i += stride) {
    int q;
    if (BITS == 8) {
      q = (int)reinterpret_cast<const int8_t *>(payload)[i];
    } else {
      const int byte = payload[i >> 1];
      q = (i & 1) ? (byte >> 4) : (byte & 15);
      q = q >= 8 ? q - 16 : q;  // sign extension (backend.py:172)
    }
    out[i] = from_f32<T>((float)q * __half2float(scales[i / group]));
  }
}

// ============================================================ page records
// A slab is one (page, head, K-or-V) 16 x D fp16 tile.  Lane l of the warp owns
// elements 256*c + 8*l + [0, 8) for chunk c < D/16: one 16-byte fp16 vector per
// chunk, contiguous across the warp (512 bytes per load instruction).
template <int D>
struct Slab {
  static constexpr int kChunks = D / 16;
  static constexpr int kElems = kBlock * D;
};

// Byte XOR that turns the row-major offset of a lane's 8 elements of chunk c
// (elements 256c + 8 lane of a [16][D] slab) into their stored offset in a V
// payload: v_swizzle with the key worked out for these offsets (it depends on
// c alone for head_dim 128, on c and the lane for head_dim 64).
template <int D>
__device__ __forceinline__ int v_chunk_xor(int mode, int c, int lane) {
  int key;
  if constexpr (D == 128)
    key = mode == AKV_MODE_FP16 ? ((c & 1) | ((c & 2) << 1)) : ((2 * c) & 6);
  else
    key = mode == AKV_MODE_INT4 ? ((2 * c) & 2) : (((4 * c) & 4) | ((lane >> 3) & 2));
  return key << 4;
}

// The payload bytes of 8 consecutive elements (e = 256 c + 8 lane) of a record:
// FP16 all 16 bytes, INT8 8 bytes in .x / .y, INT4 4 bytes in .x.  `VPAY`: a V
// payload, stored in the swizzled byte order (v_swizzle).
template <int D, bool VPAY>
__device__ __forceinline__ uint4 record_raw8(int mode, const uint8_t *payload, int c, int lane) {
  const int e = 256 * c + 8 * lane;
  const int vx = VPAY ? v_chunk_xor<D>(mode, c, lane) : 0;
  if (mode == AKV_MODE_FP16) return *reinterpret_cast<const uint4 *>(payload + ((2 * e) ^ vx));
  if (mode == AKV_MODE_INT8) {
    const uint2 w = *reinterpret_cast<const uint2 *>(payload + (e ^ vx));
    return make_uint4(w.x, w.y, 0u, 0u);
  }
  return make_uint4(*reinterpret_cast<const uint32_t *>(payload + ((e / 2) ^ vx)), 0u, 0u, 0u);
}

// record_raw8 for all NC chunks of a slab, the mode tested once: the loads form
// one straight-line batch.
template <int D, int NC, bool VPAY>
__device__ __forceinline__ void slab_raw(int mode, const uint8_t *payload, int lane, uint4 (&raw)[NC]) {
  if (mode == AKV_MODE_FP16) {
#pragma unroll
    for (int c = 0; c < NC; ++c) raw[c] = record_raw8<D, VPAY>(AKV_MODE_FP16, payload, c, lane);
  } else if (mode == AKV_MODE_INT8) {
#pragma unroll
    for (int c = 0; c < NC; ++c) raw[c] = record_raw8<D, VPAY>(AKV_MODE_INT8, payload, c, lane);
  } else {
#pragma unroll
    for (int c = 0; c < NC; ++c) raw[c] = record_raw8<D, VPAY>(AKV_MODE_INT4, payload, c, lane);
  }
}

// The 8 integers of a raw INT8 / INT4 chunk.
__device__ __forceinline__ void raw8_ints(int mode, uint4 w, int (&q)[8]) {
  if (mode == AKV_MODE_INT8) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q[i] = (int)(int8_t)(w.x >> (8 * i));
      q[4 + i] = (int)(int8_t)(w.y >> (8 * i));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int n = (w.x >> (4 * i)) & 15;
      q[i] = n >= 8 ? n - 16 : n;
    }
  }
}

// A raw chunk dequantized to fp16 exactly as QuantizedPage.dense
// (packed_decode.py:34-45): fp16(int * float(scale)), `s` the element group's
// scale (unused for FP16 pages).
__device__ __forceinline__ uint4 raw8_to_f16(int mode, uint4 w, float s) {
  if (mode == AKV_MODE_FP16) return w;
  int q[8];
  raw8_ints(mode, w, q);
  uint32_t h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half lo = __float2half_rn((float)q[2 * i] * s);
    const __half hi = __float2half_rn((float)q[2 * i + 1] * s);
    h[i] = (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
  }
  return make_uint4(h[0], h[1], h[2], h[3]);
}

// A raw chunk as float values int * float(scale), before any rounding to fp16
// (PackedTensor.dequantize, backend.py:177-180, rounds once to the caller's
// dtype).  FP16 pages give their stored values.
__device__ __forceinline__ void raw8_to_f32(int mode, uint4 w, float s, float (&x)[8]) {
  if (mode == AKV_MODE_FP16) {
    const uint32_t h[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __half2float(__ushort_as_half((unsigned short)(h[i] & 0xffff)));
      x[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(h[i] >> 16)));
    }
    return;
  }
  int q[8];
  raw8_ints(mode, w, q);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = (float)q[i] * s;
}

// The scale of chunk c's elements of lane `lane` (groups of G elements).
template <int G>
__device__ __forceinline__ float chunk_scale(int mode, const __half *sc, int c, int lane) {
  return mode == AKV_MODE_FP16 ? 1.f : __half2float(sc[(256 * c + 8 * lane) / G]);
}

// Dequantize 8 consecutive elements of a record payload to fp16, exactly as
// QuantizedPage.dense (packed_decode.py:34-45): fp16(int * float(scale)).
template <int D, int G, bool VPAY>
__device__ __forceinline__ uint4 record_load8(int mode, const uint8_t *payload, const __half *sc,
                                              int c, int lane) {
  return raw8_to_f16(mode, record_raw8<D, VPAY>(mode, payload, c, lane), chunk_scale<G>(mode, sc, c, lane));
}

// ---- exact quantization of a page slab without a division per element
//
// round-half-even(x / s) for |x / s| <= qmax * (1 + 2^-11) (s is the group's
// absmax / qmax, possibly rounded down to fp16 by at most 2^-11): y = x * fl(1/s)
// is within 2^-16 of the exact quotient, so rounding y can differ from rounding
// x / s only when y lies within that distance of a half-integer.  Rounding is
// the 1.5 * 2^23 magic add (an RN addition), whose result t carries rint(y) as
// two's complement in its low mantissa bits.  A chunk where any lane sees a y
// within 2^-15 of a tie (about 1 chunk in 70 on random data) is redone with the
// correctly rounded division.  No clamp is needed on the fast path: |y| <=
// qmax + 0.07 rounds into [-qmax, qmax].
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23
constexpr float kTieGuard = 0.49996948242f;  // 0.5 - 2^-15

__device__ __forceinline__ uint32_t hmax2_u(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ float half_lo(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w & 0xffff))); }
__device__ __forceinline__ float half_hi(uint32_t w) { return __half2float(__ushort_as_half((unsigned short)(w >> 16))); }
// max |x| over the 8 fp16 values of a chunk, computed in fp16 (exact).
__device__ __forceinline__ float chunk_absmax(const uint4 &v) {
  const uint32_t m = hmax2_u(hmax2_u(v.x & 0x7fff7fffu, v.y & 0x7fff7fffu),
                             hmax2_u(v.z & 0x7fff7fffu, v.w & 0x7fff7fffu));
  return fmaxf(half_lo(m), half_hi(m));
}

// Quantize the 8 fp16 values of a chunk; returns their integers' low bytes in
// t[i] (bits 0-7 two's complement).
__device__ __forceinline__ void quantize_chunk(const uint4 &v, float s, float r, float qmax,
                                               uint32_t (&t)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  const uint64_t r2 = f2_pack(r, r), magic2 = f2_pack(kRoundMagic, kRoundMagic);
  bool tie = false;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t y = f2_mul(f2_pack(half_lo(w[i]), half_hi(w[i])), r2);
    const uint64_t tt = f2_add(y, magic2);
    const uint64_t d = f2_sub(y, f2_sub(tt, magic2));
    tie |= fabsf(f2_lo(d)) >= kTieGuard;
    tie |= fabsf(f2_hi(d)) >= kTieGuard;
    t[2 * i] = (uint32_t)tt;
    t[2 * i + 1] = (uint32_t)(tt >> 32);
  }
  if (__any_sync(0xffffffffu, tie)) {  // rare: recompute the chunk with the exact quotient
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float x = (i & 1) ? half_hi(w[i >> 1]) : half_lo(w[i >> 1]);
      const float q = fminf(fmaxf(rintf(__fdiv_rn(x, s)), -qmax), qmax);
      t[i] = __float_as_uint(q + kRoundMagic);
    }
  }
}

// Quantize one slab held in registers (v[c] = 8 fp16 values) into a record.
// `vpay`: a V payload, written in the swizzled byte order (v_swizzle); each
// lane's 16, 8 or 4 bytes stay inside one 16-byte unit, and a warp's store
// covers the same 128-byte lines as the row-major one.
template <int D, int G, int SEM>
__device__ __forceinline__ void store_slab(const uint4 (&v)[Slab<D>::kChunks], int mode,
                                           uint8_t *payload, __half *sc, int lane, bool vpay) {
  constexpr int NC = Slab<D>::kChunks;
  if (mode == AKV_MODE_FP16) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int vx = vpay ? v_chunk_xor<D>(mode, c, lane) : 0;
      *reinterpret_cast<uint4 *>(payload + ((512 * c + 16 * lane) ^ vx)) = v[c];
    }
    return;
  }
  const float qmax = mode == AKV_MODE_INT8 ? 127.f : 7.f;
  float lm[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) lm[c] = chunk_absmax(v[c]);
  // Group absmax: G/8 lanes share a group inside a chunk (G < 256), or
  // G/256 whole chunks share one (G >= 256).
  float gm[NC];
  if (G < 256) {
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float m = lm[c];
#pragma unroll
      for (int off = 1; off < G / 8; off <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      gm[c] = m;
    }
  } else {
    constexpr int CPG = G / 256 < NC ? G / 256 : NC;
#pragma unroll
    for (int c0 = 0; c0 < NC; c0 += CPG) {
      float m = 0.f;
#pragma unroll
      for (int c = c0; c < c0 + CPG; ++c) m = fmaxf(m, lm[c]);
#pragma unroll
      for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
#pragma unroll
      for (int c = c0; c < c0 + CPG; ++c) gm[c] = m;
    }
  }
  GroupScale gs{};
  float r = 0.f;
  constexpr int kGroupChunks = G >= 256 ? G / 256 : 1;  // chunks a group spans (a chunk holds 256 elements)
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    if (c % kGroupChunks == 0) {  // a new group starts in this chunk
      gs = group_scale<SEM>(gm[c], qmax);
      r = __frcp_rn(gs.divisor);
    }
    uint32_t t[8];
    quantize_chunk(v[c], gs.divisor, r, qmax, t);
    const int e = 256 * c + 8 * lane;
    const int vx = vpay ? v_chunk_xor<D>(mode, c, lane) : 0;
    if (mode == AKV_MODE_INT8) {
      const uint32_t w0 = prmt(prmt(t[0], t[1], 0x0040u), prmt(t[2], t[3], 0x0040u), 0x5410u);
      const uint32_t w1 = prmt(prmt(t[4], t[5], 0x0040u), prmt(t[6], t[7], 0x0040u), 0x5410u);
      *reinterpret_cast<uint2 *>(payload + (e ^ vx)) = make_uint2(w0, w1);
    } else {
      uint32_t pb[4];  // byte k: element 2k in the low nibble, 2k+1 in the high nibble
#pragma unroll
      for (int k = 0; k < 4; ++k) pb[k] = (t[2 * k] & 0x0fu) | ((t[2 * k + 1] << 4) & 0xf0u);
      *reinterpret_cast<uint32_t *>(payload + ((e / 2) ^ vx)) =
          prmt(prmt(pb[0], pb[1], 0x0040u), prmt(pb[2], pb[3], 0x0040u), 0x5410u);
    }
    if (e % G == 0) sc[e / G] = gs.stored;
  }
}

// Vector path for the common shapes: groups of G = 8 * L elements (L a power
// of two, 1..32) over a whole number of groups.  Thread t owns elements
// 8t .. 8t + 7 (one 16-byte load of fp16/bf16, two of fp32); the L lanes of a
// group are adjacent in a warp, so the group absmax is a shuffle reduction.
// Same arithmetic as quantize_flat_kernel: IEEE division per element.
template <typename T>
__device__ __forceinline__ void load8(const T *p, float (&x)[8]) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4 *>(p), b = *reinterpret_cast<const float4 *>(p + 4);
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
  } else {
    const uint4 w = *reinterpret_cast<const uint4 *>(p);
    const T *h = reinterpret_cast<const T *>(&w);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = to_f32<T>(h[i]);
  }
}

// Thread t's 8 integers (two's complement in their low bits) as payload bytes:
// INT8 one byte each, INT4 two per byte with the even element low.
template <int BITS>
__device__ __forceinline__ void store_quantized(const uint32_t (&q)[8], uint8_t *payload, int64_t t) {
  if (BITS == 8) {
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) w0 |= (q[i] & 255u) << (8 * i), w1 |= (q[4 + i] & 255u) << (8 * i);
    *reinterpret_cast<uint2 *>(payload + 8 * t) = make_uint2(w0, w1);
  } else {
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) w |= (q[i] & 15u) << (4 * i);
    *reinterpret_cast<uint32_t *>(payload + 4 * t) = w;
  }
}

template <typename T, int BITS, int SEM>
__global__ void __launch_bounds__(256) quantize_vec_kernel(const T *__restrict__ src, int64_t nthreads, int lanes,
                                                           uint8_t *__restrict__ payload, __half *__restrict__ scales) {
  const float qmax = BITS == 8 ? 127.f : 7.f;
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t0 = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) & ~(int64_t)31; t0 < nthreads; t0 += stride) {
    const int64_t t = t0 + lane;
    const bool active = t < nthreads;  // inactive lanes form whole groups (nthreads is a multiple of lanes)
    if constexpr (std::is_same<T, __half>::value) {
      // fp16 values: absmax in the fp16 domain and the exact reciprocal-multiply
      // rounding with its tie fallback (quantize_chunk), warp-collective
      const uint4 raw = active ? *reinterpret_cast<const uint4 *>(src + 8 * t) : make_uint4(0, 0, 0, 0);
      float amax = chunk_absmax(raw);
      for (int off = 1; off < lanes; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      const GroupScale g = group_scale<SEM>(amax, qmax);
      uint32_t q[8];
      quantize_chunk(raw, g.divisor, __frcp_rn(g.divisor), qmax, q);
      if (!active) continue;
      store_quantized<BITS>(q, payload, t);
      if ((t & (lanes - 1)) == 0) scales[t / lanes] = g.stored;
      continue;
    }
    float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (active) load8<T>(src + 8 * t, x);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (SEM == AKV_SEM_PAGE) x[i] = __half2float(__float2half_rn(x[i]));  // pack_page rounds to fp16 first
      amax = fmaxf(amax, fabsf(x[i]));
    }
    for (int off = 1; off < lanes; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if (!active) continue;
    const GroupScale g = group_scale<SEM>(amax, qmax);
    uint32_t q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = (uint32_t)quantize_value(x[i], g.divisor, qmax);
    store_quantized<BITS>(q, payload, t);
    if ((t & (lanes - 1)) == 0) scales[t / lanes] = g.stored;
  }
}

// Dequantize 8 elements per thread (group a multiple of 8: one scale each).
template <typename T, int BITS>
__global__ void __launch_bounds__(256) dequantize_vec_kernel(const uint8_t *__restrict__ payload,
                                                             const __half *__restrict__ scales, int64_t nthreads,
                                                             int64_t group8, T *__restrict__ out) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < nthreads; t += stride) {
    const float s = __half2float(scales[t / group8]);
    float y[8];
    if (BITS == 8) {
      const uint2 w = *reinterpret_cast<const uint2 *>(payload + 8 * t);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        y[i] = (float)(int)(int8_t)(w.x >> (8 * i)) * s;
        y[4 + i] = (float)(int)(int8_t)(w.y >> (8 * i)) * s;
      }
    } else {
      const uint32_t w = *reinterpret_cast<const uint32_t *>(payload + 4 * t);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int n = (w >> (4 * i)) & 15;
        y[i] = (float)(n >= 8 ? n - 16 : n) * s;  // sign extension (backend.py:172)
      }
    }
    if constexpr (sizeof(T) == 4) {
      float4 *o = reinterpret_cast<float4 *>(out + 8 * t);
      o[0] = make_float4(y[0], y[1], y[2], y[3]);
      o[1] = make_float4(y[4], y[5], y[6], y[7]);
    } else {
      uint4 w;
      T *h = reinterpret_cast<T *>(&w);
#pragma unroll
      for (int i = 0; i < 8; ++i) h[i] = from_f32<T>(y[i]);
      *reinterpret_cast<uint4 *>(out + 8 * t) = w;
    }
  }
}

// Descriptor check shared by the page kernels.
__device__ __forceinline__ bool page_in_arena(int64_t desc, int64_t page_bytes, int64_t arena_bytes) {
  const int64_t off = desc_offset(desc);
  return (off & 15) == 0 && off >= 0 && off + page_bytes <= arena_bytes;
}

// Pack (SRC_RECORD = false: dense fp16 source) or repack (SRC_RECORD = true:
// source records in the arena) one slab per warp.  A repack holds both the
// source record's reads and the destination's stores, so it runs 2 CTAs per
// SM (up to 128 registers) rather than 3 (85), where it would spill.
template <int D, int G, int SEM, bool SRC_RECORD>
__global__ void __launch_bounds__(256, SRC_RECORD ? 2 : 3) pack_pages_kernel(
    const __half *__restrict__ src_k, const __half *__restrict__ src_v, int64_t outer_stride,
    int64_t head_stride, int64_t blocks_per_row, const int64_t *__restrict__ src_desc,
    const int64_t *__restrict__ dst_desc, int64_t n_pages, uint8_t *__restrict__ arena,
    int64_t arena_bytes, int heads, int32_t *status) {
  constexpr int NC = Slab<D>::kChunks;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t items = n_pages * heads * 2;
  for (int64_t it = warp; it < items; it += nwarps) {
    const int kv = (int)(it & 1);
    const int h = (int)((it >> 1) % heads);
    const int64_t p = (it >> 1) / heads;
    const int64_t dd = dst_desc[p];
    const int dmode = desc_mode(dd);
    if (dmode == AKV_MODE_SKIP) continue;
    const int64_t drec = record_bytes(D, G, dmode);
    if (!page_in_arena(dd, drec * heads, arena_bytes)) {
      if (lane == 0) set_status(status, AKV_DEV_BAD_DESCRIPTOR);
      continue;
    }
    uint4 v[NC];
    if (SRC_RECORD) {
      const int64_t sd = src_desc[p];
      const int smode = desc_mode(sd);
      const int64_t srec = record_bytes(D, G, smode);
      if (smode == AKV_MODE_SKIP || !page_in_arena(sd, srec * heads, arena_bytes)) {
        if (lane == 0) set_status(status, AKV_DEV_BAD_DESCRIPTOR);
        continue;
      }
      const uint8_t *rec = arena + desc_offset(sd) + h * srec;
      const int64_t pb = payload_bytes(D, smode);
      const uint8_t *pay = rec + kv * pb;
      const __half *sc =
          reinterpret_cast<const __half *>(rec + 2 * pb) + kv * scale_count(D, G, smode);
      if (kv) {
#pragma unroll
        for (int c = 0; c < NC; ++c) v[c] = record_load8<D, G, true>(smode, pay, sc, c, lane);
      } else {
#pragma unroll
        for (int c = 0; c < NC; ++c) v[c] = record_load8<D, G, false>(smode, pay, sc, c, lane);
      }
    } else {
      const __half *src = (kv ? src_v : src_k) + (p / blocks_per_row) * outer_stride +
                          h * head_stride + (p % blocks_per_row) * (int64_t)kBlock * D;
#pragma unroll
      for (int c = 0; c < NC; ++c)
        v[c] = __ldg(reinterpret_cast<const uint4 *>(src + 256 * c + 8 * lane));
    }
    uint8_t *rec = arena + desc_offset(dd) + h * drec;
    const int64_t pb = payload_bytes(D, dmode);
    const int64_t ns = scale_count(D, G, dmode);
    __half *sc = reinterpret_cast<__half *>(rec + 2 * pb) + kv * ns;
    store_slab<D, G, SEM>(v, dmode, rec + kv * pb, sc, lane, kv == 1);
    if (kv == 1) {  // zero the record's alignment pad so records are deterministic
      const int64_t used = 2 * pb + 4 * ns;
      if (lane < drec - used) rec[used + lane] = 0;
    }
  }
}

// Dequantize records to dense [heads][n_pages * 16][D] in OutT: fp16 gives
// fp16(int * float(scale)) (QuantizedPage.dense, packed_decode.py:34-45);
// fp32 / bf16 round int * float(scale) once to that type
// (PackedTensor.dequantize, backend.py:177-180).
template <int D, int G, typename OutT>
__global__ void __launch_bounds__(256) unpack_pages_kernel(const int64_t *__restrict__ desc,
                                                           int64_t n_pages,
                                                           const uint8_t *__restrict__ arena,
                                                           int64_t arena_bytes, int heads,
                                                           OutT *__restrict__ out_k,
                                                           OutT *__restrict__ out_v,
                                                           int32_t *status) {
  constexpr int NC = Slab<D>::kChunks;
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t items = n_pages * heads * 2;
  for (int64_t it = warp; it < items; it += nwarps) {
    const int kv = (int)(it & 1);
    const int h = (int)((it >> 1) % heads);
    const int64_t p = (it >> 1) / heads;
    OutT *out = (kv ? out_v : out_k) + ((int64_t)h * n_pages + p) * kBlock * D;
    const int64_t d = desc[p];
    const int mode = desc_mode(d);
    const int64_t rb = record_bytes(D, G, mode);
    const bool ok = mode != AKV_MODE_SKIP && page_in_arena(d, rb * heads, arena_bytes);
    if (mode != AKV_MODE_SKIP && !ok && lane == 0) set_status(status, AKV_DEV_BAD_DESCRIPTOR);
    // Every chunk's payload load is issued before any is converted or stored, so
    // a warp keeps its whole slab in flight (one memory round trip per slab,
    // not one per chunk).
    uint4 raw[NC];
    float s[NC];
#pragma unroll
    for (int c = 0; c < NC; ++c) raw[c] = make_uint4(0u, 0u, 0u, 0u), s[c] = 0.f;
    if (ok) {
      const uint8_t *rec = arena + desc_offset(d) + h * rb;
      const int64_t pb = payload_bytes(D, mode);
      const __half *sc = reinterpret_cast<const __half *>(rec + 2 * pb) + kv * scale_count(D, G, mode);
      if (kv)
        slab_raw<D, NC, true>(mode, rec + pb, lane, raw);
      else
        slab_raw<D, NC, false>(mode, rec, lane, raw);
#pragma unroll
      for (int c = 0; c < NC; ++c) s[c] = chunk_scale<G>(mode, sc, c, lane);
    }
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      OutT *dst = out + 256 * c + 8 * lane;
      if constexpr (sizeof(OutT) == 2 && !std::is_same<OutT, __nv_bfloat16>::value) {
        *reinterpret_cast<uint4 *>(dst) = ok ? raw8_to_f16(mode, raw[c], s[c]) : make_uint4(0u, 0u, 0u, 0u);
      } else {
        float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (ok) raw8_to_f32(mode, raw[c], s[c], x);
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = from_f32<OutT>(x[i]);
      }
    }
  }
}

// ============================================================ token append
// Write `rows` decode-step token rows of K and V for every sequence of a batch
// into FP16 page records: sequence b's rows go to rows first_row .. of the page
// its table entry (or, for a fresh page, new_desc[b]) names.  One warp per
// (sequence, head, page row, K|V); a row is head_dim fp16 values, 8 bytes per
// lane.  K rows are stored row-major, V rows in the bank-swizzled order
// (v_swizzle keeps a row inside its own bytes, so an 8-byte chunk moves
// whole).  A fresh page's other rows are zeroed, as the reference's new pages
// start from zeros (packed_decode.py:141-146).  The entry's valid-token count
// becomes first_row + rows; its mode and offset do not change, so warps that
// read it while one warp rewrites it see the same page.
template <int D>
__global__ void __launch_bounds__(256) append_rows_kernel(
    const __half *__restrict__ src_k, const __half *__restrict__ src_v, int64_t sbs, int64_t shs, int64_t sts,
    int batch, int rows, int first_row, int64_t *table, int64_t table_stride, int page,
    const int64_t *__restrict__ new_desc, uint8_t *__restrict__ arena, int64_t arena_bytes, int heads,
    int32_t *status) {
  constexpr int LANES = D / 4;  // lanes holding 4 values (8 bytes) of a row
  constexpr int64_t RB = 2 * kBlock * D * 2;  // FP16 record: K and V payloads, no scales
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  // A fresh page has all of its 16 rows written (the new tokens, zeros
  // elsewhere); an existing page only the new rows.
  const int span = new_desc ? kBlock : rows;
  const int row0 = new_desc ? 0 : first_row;
  const int64_t items = (int64_t)batch * heads * span * 2;
  for (int64_t it = warp; it < items; it += nwarps) {
    const int kv = (int)(it & 1);
    const int r = row0 + (int)((it >> 1) % span);
    const int h = (int)((it >> 1) / span % heads);
    const int b = (int)((it >> 1) / span / heads);
    int64_t *entry = table + (int64_t)b * table_stride + page;
    const int64_t d = new_desc ? new_desc[b] : *entry;
    const bool lead = h == 0 && r == row0 && kv == 0;  // one warp per sequence
    if (desc_mode(d) != AKV_MODE_FP16 || !page_in_arena(d, RB * heads, arena_bytes)) {
      if (lane == 0 && lead) set_status(status, AKV_DEV_BAD_DESCRIPTOR);
      continue;
    }
    if (lane == 0 && lead)  // publish the new valid-token count (mode and offset unchanged)
      *entry = (d & ~((int64_t)15 << 2)) | ((int64_t)(first_row + rows - 1) << 2);
    const bool written = r >= first_row && r < first_row + rows;
    uint8_t *pay = arena + desc_offset(d) + h * RB + kv * (kBlock * D * 2);
    if (lane < LANES) {
      uint2 v = make_uint2(0u, 0u);
      if (written) {
        const __half *src = (kv ? src_v : src_k) + b * sbs + h * shs + (int64_t)(r - first_row) * sts;
        v = *reinterpret_cast<const uint2 *>(src + 4 * lane);
      }
      const int64_t o = (int64_t)r * (2 * D) + 8 * lane;
      *reinterpret_cast<uint2 *>(pay + (kv ? v_swizzle(D, AKV_MODE_FP16, o) : o)) = v;
    }
  }
}

// ================================================================ launchers
static int grid_for(int64_t warps_needed) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t blocks = (warps_needed + 7) / 8;  // 8 warps per 256-thread block
  return (int)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sms * 16));
}

static int launch_status() {
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_CUDA;
}

// G values the page kernels are instantiated for: 32, 64, 128 (per-row groups)
// and 16*D (one scale per 16-token slab, i.e. per block and KV head).
template <int D, template <int, int> class F, typename... Args>
static int dispatch_group(int group, Args... args) {
  switch (group) {
    case 32: return F<D, 32>::run(args...);
    case 64: return F<D, 64>::run(args...);
    case 128: return F<D, 128>::run(args...);
    case 16 * D: return F<D, 16 * D>::run(args...);
    default: return AKV_ERR_UNSUPPORTED;
  }
}

struct PackArgs {
  const void *src_k, *src_v;
  int64_t outer_stride, head_stride, blocks_per_row;
  const int64_t *src_desc, *dst_desc;
  int64_t n_pages;
  void *arena;
  int64_t arena_bytes;
  int heads, semantics;
  int32_t *status;
  cudaStream_t stream;
};

template <int D, int G>
struct PackLaunch {
  static int run(const PackArgs &a, bool repack) {
    const int grid = grid_for(a.n_pages * a.heads * 2);
#define AKV_PACK(SEM, REC)                                                                      \
  pack_pages_kernel<D, G, SEM, REC><<<grid, 256, 0, a.stream>>>(                                \
      (const __half *)a.src_k, (const __half *)a.src_v, a.outer_stride, a.head_stride,          \
      a.blocks_per_row, a.src_desc, a.dst_desc, a.n_pages, (uint8_t *)a.arena, a.arena_bytes, \
      a.heads, a.status)
    if (repack) {
      if (a.semantics == AKV_SEM_PAGE) AKV_PACK(AKV_SEM_PAGE, true);
      else AKV_PACK(AKV_SEM_TENSOR, true);
    } else {
      if (a.semantics == AKV_SEM_PAGE) AKV_PACK(AKV_SEM_PAGE, false);
      else AKV_PACK(AKV_SEM_TENSOR, false);
    }
#undef AKV_PACK
    return launch_status();
  }
};

struct UnpackArgs {
  const int64_t *desc;
  int64_t n_pages;
  const void *arena;
  int64_t arena_bytes;
  int heads;
  void *out_k, *out_v;
  int out_dtype;
  int32_t *status;
  cudaStream_t stream;
};

template <int D, int G>
struct UnpackLaunch {
  template <typename OutT>
  static void go(const UnpackArgs &a) {
    unpack_pages_kernel<D, G, OutT><<<grid_for(a.n_pages * a.heads * 2), 256, 0, a.stream>>>(
        a.desc, a.n_pages, (const uint8_t *)a.arena, a.arena_bytes, a.heads, (OutT *)a.out_k,
        (OutT *)a.out_v, a.status);
  }
  static int run(const UnpackArgs &a) {
    if (a.out_dtype == AKV_DTYPE_F16) go<__half>(a);
    else if (a.out_dtype == AKV_DTYPE_F32) go<float>(a);
    else go<__nv_bfloat16>(a);
    return launch_status();
  }
};

static bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace akv

using namespace akv;

extern "C" int akv_quantize(const void *src, int src_dtype, int64_t numel, int64_t group, int bits,
                            int semantics, void *payload, void *scales, void *stream) {
  if (!src || !payload || !scales || numel <= 0 || group <= 0) return AKV_ERR_INVALID;
  if (bits != 4 && bits != 8) return AKV_ERR_INVALID;
  if (bits == 4 && group % 2) return AKV_ERR_INVALID;
  if (semantics != AKV_SEM_TENSOR && semantics != AKV_SEM_PAGE) return AKV_ERR_INVALID;
  const int64_t ngroups = (numel + group - 1) / group;
  cudaStream_t s = (cudaStream_t)stream;
  // Vector path: a power-of-two group of 8..256 elements, whole groups,
  // 16-byte aligned source and naturally aligned payload.
  const bool pow2 = (group & (group - 1)) == 0;
  if (pow2 && group >= 8 && group <= 256 && numel % group == 0 && ((uintptr_t)src & 15) == 0 &&
      ((uintptr_t)payload & (bits == 8 ? 7 : 3)) == 0) {
    const int64_t nthreads = numel / 8;
    const int lanes = (int)(group / 8);
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((nthreads + 255) / 256, 148ll * 64));
#define AKV_QV(T, B, S)                                                                                  \
  quantize_vec_kernel<T, B, S><<<grid, 256, 0, s>>>((const T *)src, nthreads, lanes, (uint8_t *)payload, \
                                                    (__half *)scales)
#define AKV_QVB(T, S) \
  if (bits == 8) AKV_QV(T, 8, S); else AKV_QV(T, 4, S)
#define AKV_QVS(T) \
  if (semantics == AKV_SEM_TENSOR) { AKV_QVB(T, AKV_SEM_TENSOR); } else { AKV_QVB(T, AKV_SEM_PAGE); }
    switch (src_dtype) {
      case AKV_DTYPE_F32: AKV_QVS(float); break;
      case AKV_DTYPE_F16: AKV_QVS(__half); break;
      case AKV_DTYPE_BF16: AKV_QVS(__nv_bfloat16); break;
      default: return AKV_ERR_INVALID;
    }
#undef AKV_QVS
#undef AKV_QVB
#undef AKV_QV
    return launch_status();
  }
  const int grid = grid_for(ngroups);
#define AKV_Q(T, B, S)                                                                   \
  quantize_flat_kernel<T, B, S><<<grid, 256, 0, s>>>((const T *)src, numel, group, ngroups, \
                                                       (uint8_t *)payload, (__half *)scales)
#define AKV_QB(T, S) \
  if (bits == 8) AKV_Q(T, 8, S); else AKV_Q(T, 4, S)
#define AKV_QS(T) \
  if (semantics == AKV_SEM_TENSOR) { AKV_QB(T, AKV_SEM_TENSOR); } else { AKV_QB(T, AKV_SEM_PAGE); }
  switch (src_dtype) {
    case AKV_DTYPE_F32: AKV_QS(float); break;
    case AKV_DTYPE_F16: AKV_QS(__half); break;
    case AKV_DTYPE_BF16: AKV_QS(__nv_bfloat16); break;
    default: return AKV_ERR_INVALID;
  }
#undef AKV_QS
#undef AKV_QB
#undef AKV_Q
  return launch_status();
}

extern "C" int akv_dequantize(const void *payload, const void *scales, int64_t numel, int64_t group,
                              int bits, void *out, int out_dtype, void *stream) {
  if (!payload || !scales || !out || numel <= 0 || group <= 0) return AKV_ERR_INVALID;
  if (bits != 4 && bits != 8) return AKV_ERR_INVALID;
  cudaStream_t s = (cudaStream_t)stream;
  if (group % 8 == 0 && numel % 8 == 0 && ((uintptr_t)out & 15) == 0 &&
      ((uintptr_t)payload & (bits == 8 ? 7 : 3)) == 0) {  // vector path: 8 elements (one scale) per thread
    const int64_t nthreads = numel / 8;
    const int vgrid = (int)std::max<int64_t>(1, std::min<int64_t>((nthreads + 255) / 256, 148ll * 64));
#define AKV_DV(T)                                                                                              \
  if (bits == 8)                                                                                               \
    dequantize_vec_kernel<T, 8><<<vgrid, 256, 0, s>>>((const uint8_t *)payload, (const __half *)scales, nthreads, \
                                                      group / 8, (T *)out);                                     \
  else                                                                                                         \
    dequantize_vec_kernel<T, 4><<<vgrid, 256, 0, s>>>((const uint8_t *)payload, (const __half *)scales, nthreads, \
                                                      group / 8, (T *)out)
    switch (out_dtype) {
      case AKV_DTYPE_F32: AKV_DV(float); break;
      case AKV_DTYPE_F16: AKV_DV(__half); break;
      case AKV_DTYPE_BF16: AKV_DV(__nv_bfloat16); break;
      default: return AKV_ERR_INVALID;
    }
#undef AKV_DV
    return launch_status();
  }
  const int grid = grid_for((numel + 31) / 32);
#define AKV_D(T)                                                                           \
  if (bits == 8)                                                                           \
    dequantize_flat_kernel<T, 8><<<grid, 256, 0, s>>>((const uint8_t *)payload,            \
                                                       (const __half *)scales, numel, group, (T *)out); \
  else                                                                                     \
    dequantize_flat_kernel<T, 4><<<grid, 256, 0, s>>>((const uint8_t *)payload,            \
                                                       (const __half *)scales, numel, group, (T *)out)
  switch (out_dtype) {
    case AKV_DTYPE_F32: AKV_D(float); break;
    case AKV_DTYPE_F16: AKV_D(__half); break;
    case AKV_DTYPE_BF16: AKV_D(__nv_bfloat16); break;
    default: return AKV_ERR_INVALID;
  }
#undef AKV_D
  return launch_status();
}

static int check_page_geometry(int heads, int head_dim, int group) {
  if (heads <= 0) return AKV_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return AKV_ERR_UNSUPPORTED;
  if (group != 32 && group != 64 && group != 128 && group != 16 * head_dim) return AKV_ERR_UNSUPPORTED;
  return AKV_OK;
}

extern "C" int akv_pack_pages(const void *src_k, const void *src_v, int64_t outer_stride,
                              int64_t head_stride, int64_t blocks_per_row, int64_t n_pages,
                              const int64_t *dst_desc, void *arena, int64_t arena_bytes, int heads,
                              int head_dim, int group, int semantics, int32_t *dev_status,
                              void *stream) {
  if (int st = check_page_geometry(heads, head_dim, group)) return st;
  if (!src_k || !src_v || !dst_desc || !arena || n_pages < 0 || blocks_per_row <= 0) return AKV_ERR_INVALID;
  if (!aligned16(src_k) || !aligned16(src_v) || !aligned16(arena)) return AKV_ERR_INVALID;
  if ((outer_stride * 2) % 16 || (head_stride * 2) % 16) return AKV_ERR_INVALID;
  if (semantics != AKV_SEM_TENSOR && semantics != AKV_SEM_PAGE) return AKV_ERR_INVALID;
  if (n_pages == 0) return AKV_OK;
  PackArgs a{src_k, src_v, outer_stride, head_stride, blocks_per_row, nullptr, dst_desc, n_pages,
             arena, arena_bytes, heads, semantics, dev_status, (cudaStream_t)stream};
  return head_dim == 64 ? dispatch_group<64, PackLaunch>(group, a, false)
                        : dispatch_group<128, PackLaunch>(group, a, false);
}

extern "C" int akv_repack_pages(const int64_t *src_desc, const int64_t *dst_desc, int64_t n_pages,
                                void *arena, int64_t arena_bytes, int heads, int head_dim, int group,
                                int semantics, int32_t *dev_status, void *stream) {
  if (int st = check_page_geometry(heads, head_dim, group)) return st;
  if (!src_desc || !dst_desc || !arena || n_pages < 0 || !aligned16(arena)) return AKV_ERR_INVALID;
  if (semantics != AKV_SEM_TENSOR && semantics != AKV_SEM_PAGE) return AKV_ERR_INVALID;
  if (n_pages == 0) return AKV_OK;
  PackArgs a{nullptr, nullptr, 0, 0, 1, src_desc, dst_desc, n_pages, arena, arena_bytes, heads,
             semantics, dev_status, (cudaStream_t)stream};
  return head_dim == 64 ? dispatch_group<64, PackLaunch>(group, a, true)
                        : dispatch_group<128, PackLaunch>(group, a, true);
}

extern "C" int akv_unpack_pages(const int64_t *desc, int64_t n_pages, const void *arena,
                                int64_t arena_bytes, int heads, int head_dim, int group, void *out_k,
                                void *out_v, int out_dtype, int32_t *dev_status, void *stream) {
  if (int st = check_page_geometry(heads, head_dim, group)) return st;
  if (!desc || !arena || !out_k || !out_v || n_pages < 0) return AKV_ERR_INVALID;
  if (!aligned16(arena) || !aligned16(out_k) || !aligned16(out_v)) return AKV_ERR_INVALID;
  if (out_dtype != AKV_DTYPE_F16 && out_dtype != AKV_DTYPE_F32 && out_dtype != AKV_DTYPE_BF16)
    return AKV_ERR_INVALID;
  if (n_pages == 0) return AKV_OK;
  UnpackArgs a{desc, n_pages, arena, arena_bytes, heads, out_k, out_v, out_dtype, dev_status,
               (cudaStream_t)stream};
  return head_dim == 64 ? dispatch_group<64, UnpackLaunch>(group, a)
                        : dispatch_group<128, UnpackLaunch>(group, a);
}

extern "C" int akv_append_rows(const void *src_k, const void *src_v, int64_t src_batch_stride,
                               int64_t src_head_stride, int64_t src_token_stride, int batch, int rows,
                               int first_row, int64_t *table, int64_t table_stride, int page,
                               const int64_t *new_desc, void *arena, int64_t arena_bytes, int heads,
                               int head_dim, int32_t *dev_status, void *stream) {
  if (head_dim != 64 && head_dim != 128) return AKV_ERR_UNSUPPORTED;
  if (!src_k || !src_v || !table || !arena || batch <= 0 || heads <= 0 || page < 0) return AKV_ERR_INVALID;
  if (rows <= 0 || first_row < 0 || first_row + rows > kBlock || table_stride <= page) return AKV_ERR_INVALID;
  if (((uintptr_t)src_k & 7) || ((uintptr_t)src_v & 7) || !aligned16(arena)) return AKV_ERR_INVALID;
  if (src_batch_stride % 4 || src_head_stride % 4 || src_token_stride % 4) return AKV_ERR_INVALID;
  const int grid = grid_for((int64_t)batch * heads * (new_desc ? kBlock : rows) * 2);
  cudaStream_t s = (cudaStream_t)stream;
#define AKV_APPEND(D)                                                                                     \
  append_rows_kernel<D><<<grid, 256, 0, s>>>((const __half *)src_k, (const __half *)src_v, src_batch_stride, \
                                             src_head_stride, src_token_stride, batch, rows, first_row, table,  \
                                             table_stride, page, new_desc, (uint8_t *)arena, arena_bytes, heads, \
                                             dev_status)
  if (head_dim == 64) AKV_APPEND(64);
  else AKV_APPEND(128);
#undef AKV_APPEND
  return launch_status();
}
