// Paged split-K decode attention over mixed FP16/INT8/INT4 pages, and the
// log-sum-exp merge of its partial states.
//
// Reference: src/anchorkv/triton_decode.py:35-104 (one program per (query head,
// split), pages strided across splits, fp32 online softmax, fp16 rounding of
// dequantised values, LSE merge), whose numerics it reproduces with a
// different execution plan:
//
//  * one CTA per (split, KV head, sequence) serves every query head of that KV
//    head (the reference re-reads each KV page once per query head);
//  * each of the CTA's 4 warps streams its share of the split's pages through a
//    private 16 KB shared-memory ring with bulk copies (cp.async.bulk, mbarrier
//    completion, no multicast; one elected lane issues), skipping evicted or
//    invisible pages without reading them;
//  * a page's K/V are dequantised in registers straight into tensor-core
//    fragments (exact: the integer is formed in fp16 by an exponent trick and
//    multiplied by the fp16 scale with one rounding, matching
//    fp16(int * float(scale)) of packed_decode.py:45 / triton_decode.py:31);
//  * Q.K^T and P.V run as mma.sync m16n8k16 (f16 x f16 -> f32): 16 tokens x 8
//    query heads per page, so one page costs 2 * head_dim/16 MMAs;
//  * the online softmax is fp32 in base 2 with warp-shuffle max reductions and
//    lazy rescaling (the running max only moves when a page exceeds it by more
//    than 2^8, so P stays <= 256 in fp16);
//  * the CTA merges its warps in shared memory and writes one partial state
//    (acc[D], m, l) per (sequence, query head, split); a second kernel merges
//    splits (and, through akv_merge's state output, GPUs).
#include <math.h>

#include "akv_common.cuh"

namespace akv {

template <int D>
struct DecodeTraits {
  static constexpr int kWarps = 4;
  static constexpr int kThreads = kWarps * 32;
  static constexpr int kRing = 16384;  // bytes of ring per warp (power of two)
  static constexpr int kSlots = 8;     // records in flight per warp
  static constexpr int DK = D / 4;     // K dims a lane owns per row
  static constexpr int DV = D / 8;     // V dims a lane owns per row
  static constexpr int kTiles = D / 16;
  static constexpr int kSmem = kWarps * kRing + kWarps * kSlots * (8 + 4 + 4);
  static_assert(kWarps * 8 * (D + 2) * 4 <= kWarps * kRing, "merge scratch must fit in the rings");
};

struct DecodeParams {
  const uint8_t *arena;
  int64_t arena_bytes;
  const int64_t *table;
  int64_t table_stride;
  const int32_t *seq_blocks;
  int32_t max_blocks;
  const __half *q;
  int64_t q_bs, q_hs;
  int32_t q_heads, kv_heads, gqa, qgroups, splits, chunk, log2_group;
  float scale_log2;
  float *partials;
  int32_t *status;
};

__device__ __forceinline__ uint32_t rep_half(const __half *p) {
  const uint32_t u = __half_as_ushort(*p);
  return u | (u << 16);
}
__device__ __forceinline__ uint32_t pair_half(const __half *a, const __half *b) {
  return (uint32_t)__half_as_ushort(*a) | ((uint32_t)__half_as_ushort(*b) << 16);
}
// Selector putting byte s of A in byte 0 and byte s of B in byte 2.
__device__ __forceinline__ constexpr uint32_t sel8(int s) { return (uint32_t)(s | ((4 + s) << 8)); }

template <int N>
__device__ __forceinline__ void lds_words(const uint8_t *p, uint32_t (&w)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N / 4; ++i) {
      const uint4 v = *reinterpret_cast<const uint4 *>(p + 16 * i);
      w[4 * i] = v.x, w[4 * i + 1] = v.y, w[4 * i + 2] = v.z, w[4 * i + 3] = v.w;
    }
  } else if constexpr (N == 2) {
    const uint2 v = *reinterpret_cast<const uint2 *>(p);
    w[0] = v.x, w[1] = v.y;
  } else {
    static_assert(N == 1, "unsupported word count");
    w[0] = *reinterpret_cast<const uint32_t *>(p);
  }
}

// Scale indices a lane needs, fixed for the whole kernel (group is a power of
// two dividing 16*D): K rows gid and gid+8 at column t4*DK, V rows 2t4, 2t4+1,
// 2t4+8, 2t4+9 at column gid*DV.
struct ScaleIdx {
  int k0, k1, va, vb, vc, vd;
};

// ---------------------------------------------------------------- Q . K^T
// S[token][head] for the page's 16 tokens (rows gid, gid+8 of this lane) and
// query heads 2t4, 2t4+1.  The contraction dim is permuted identically in the
// K (A) and Q (B) fragments: k16 chunk c = 2j + hb takes, from the lane's 8-dim
// word group j, dims {2hb, 2hb+4} (fragment cols 2t4, 2t4+1) and
// {2hb+1, 2hb+5} (cols 2t4+8, 2t4+9).
template <int D, int MODE>
__device__ __forceinline__ void page_qk(const uint8_t *rec, const __half *ksc, const ScaleIdx &si,
                                        int gid, int t4, const uint32_t (&qf)[D / 16][2],
                                        float (&s)[4]) {
  using T = DecodeTraits<D>;
  constexpr int bits = mode_bits(MODE);
  constexpr int rowB = D * bits / 8;
  constexpr int W = T::DK * bits / 32;  // words of one row slice
  uint32_t r0[W], r1[W];
  lds_words<W>(rec + gid * rowB + t4 * (W * 4), r0);
  lds_words<W>(rec + (gid + 8) * rowB + t4 * (W * 4), r1);
  if constexpr (MODE == AKV_MODE_INT4) {
    const uint32_t sc0 = rep_half(ksc + si.k0), sc1 = rep_half(ksc + si.k1);
#pragma unroll
    for (int j = 0; j < W; ++j) {
      uint32_t x0 = r0[j], x1 = r1[j];
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        mma_16816(s, hmul2(int4_lo_to_f16x2(x0), sc0), hmul2(int4_lo_to_f16x2(x1), sc1),
                  hmul2(int4_hi_to_f16x2(x0), sc0), hmul2(int4_hi_to_f16x2(x1), sc1),
                  qf[2 * j + hb][0], qf[2 * j + hb][1]);
        x0 >>= 8, x1 >>= 8;
      }
    }
  } else if constexpr (MODE == AKV_MODE_INT8) {
    const uint32_t sc0 = rep_half(ksc + si.k0), sc1 = rep_half(ksc + si.k1);
#pragma unroll
    for (int j = 0; j < W / 2; ++j) {
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const uint32_t lo = sel8(2 * hb), hi = sel8(2 * hb + 1);
        mma_16816(s, hmul2(int8_to_f16x2(prmt(r0[2 * j], r0[2 * j + 1], lo)), sc0),
                  hmul2(int8_to_f16x2(prmt(r1[2 * j], r1[2 * j + 1], lo)), sc1),
                  hmul2(int8_to_f16x2(prmt(r0[2 * j], r0[2 * j + 1], hi)), sc0),
                  hmul2(int8_to_f16x2(prmt(r1[2 * j], r1[2 * j + 1], hi)), sc1),
                  qf[2 * j + hb][0], qf[2 * j + hb][1]);
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < W / 4; ++j) {
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const uint32_t a0 = r0[4 * j + hb], b0 = r0[4 * j + 2 + hb];
        const uint32_t a1 = r1[4 * j + hb], b1 = r1[4 * j + 2 + hb];
        mma_16816(s, prmt(a0, b0, 0x5410), prmt(a1, b1, 0x5410), prmt(a0, b0, 0x7632),
                  prmt(a1, b1, 0x7632), qf[2 * j + hb][0], qf[2 * j + hb][1]);
      }
    }
  }
}

// ------------------------------------------------------------------- P . V
// O^T[dim][head] += V^T[dim][token] * P^T[token][head].  The lane owns dims
// DV*gid + [0, DV): m-tile m's A rows gid / gid+8 are dims DV*gid + 2m / +2m+1;
// its k (token) columns 2t4, 2t4+1 / 2t4+8, 2t4+9 match the P fragment that
// movmatrix produced from the score accumulators.
template <int D, int MODE>
__device__ __forceinline__ void page_pv(const uint8_t *vrec, const __half *vsc, const ScaleIdx &si,
                                        int gid, int t4, uint32_t b0, uint32_t b1,
                                        float (&o)[D / 16][4]) {
  using T = DecodeTraits<D>;
  constexpr int bits = mode_bits(MODE);
  constexpr int rowB = D * bits / 8;
  constexpr int W = T::DV * bits / 32;
  uint32_t wa[W], wb[W], wc[W], wd[W];
  const uint8_t *base = vrec + gid * (W * 4);
  lds_words<W>(base + (2 * t4) * rowB, wa);
  lds_words<W>(base + (2 * t4 + 1) * rowB, wb);
  lds_words<W>(base + (2 * t4 + 8) * rowB, wc);
  lds_words<W>(base + (2 * t4 + 9) * rowB, wd);
  if constexpr (MODE == AKV_MODE_INT4) {
    const uint32_t sab = pair_half(vsc + si.va, vsc + si.vb);
    const uint32_t scd = pair_half(vsc + si.vc, vsc + si.vd);
#pragma unroll
    for (int q = 0; q < W; ++q) {
      const uint32_t xab = prmt(wa[q], wb[q], 0x5410), yab = prmt(wa[q], wb[q], 0x7632);
      const uint32_t xcd = prmt(wc[q], wd[q], 0x5410), ycd = prmt(wc[q], wd[q], 0x7632);
#pragma unroll
      for (int mm = 0; mm < 4; ++mm) {
        const uint32_t ab = (mm < 2 ? xab : yab) >> (8 * (mm & 1));
        const uint32_t cd = (mm < 2 ? xcd : ycd) >> (8 * (mm & 1));
        mma_16816(o[4 * q + mm], hmul2(int4_lo_to_f16x2(ab), sab), hmul2(int4_hi_to_f16x2(ab), sab),
                  hmul2(int4_lo_to_f16x2(cd), scd), hmul2(int4_hi_to_f16x2(cd), scd), b0, b1);
      }
    }
  } else if constexpr (MODE == AKV_MODE_INT8) {
    const uint32_t sab = pair_half(vsc + si.va, vsc + si.vb);
    const uint32_t scd = pair_half(vsc + si.vc, vsc + si.vd);
#pragma unroll
    for (int q = 0; q < W; ++q) {
#pragma unroll
      for (int mm = 0; mm < 2; ++mm) {
        const uint32_t lo = sel8(2 * mm), hi = sel8(2 * mm + 1);
        mma_16816(o[2 * q + mm], hmul2(int8_to_f16x2(prmt(wa[q], wb[q], lo)), sab),
                  hmul2(int8_to_f16x2(prmt(wa[q], wb[q], hi)), sab),
                  hmul2(int8_to_f16x2(prmt(wc[q], wd[q], lo)), scd),
                  hmul2(int8_to_f16x2(prmt(wc[q], wd[q], hi)), scd), b0, b1);
      }
    }
  } else {
#pragma unroll
    for (int m = 0; m < W; ++m)
      mma_16816(o[m], prmt(wa[m], wb[m], 0x5410), prmt(wa[m], wb[m], 0x7632),
                prmt(wc[m], wd[m], 0x5410), prmt(wc[m], wd[m], 0x7632), b0, b1);
  }
}

struct SoftmaxState {
  float m0, m1, l0, l1;  // heads 2t4, 2t4+1: running max (base 2) and this lane's sum
};

// Online softmax of one page's scores; returns the fp16 P fragments for P.V.
template <int D>
__device__ __forceinline__ void page_softmax(float (&s)[4], int ntok, int gid, float scale_log2,
                                             SoftmaxState &st, float (&o)[D / 16][4],
                                             uint32_t &b0, uint32_t &b1) {
  constexpr float kNegInf = -INFINITY;
  if (ntok < kBlock) {  // tokens past the page's valid count do not exist
    if (gid >= ntok) s[0] = s[1] = kNegInf;
    if (gid + 8 >= ntok) s[2] = s[3] = kNegInf;
  }
  float mx0 = fmaxf(s[0], s[2]), mx1 = fmaxf(s[1], s[3]);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
  }
  mx0 *= scale_log2, mx1 *= scale_log2;
  // Lazy rescale: keep the running max unless this page exceeds it by > 8
  // (P <= 2^8 in fp16 is exact enough and cannot overflow).
  const bool grow = mx0 > st.m0 + 8.f || mx1 > st.m1 + 8.f;
  if (__any_sync(0xffffffffu, grow)) {
    const float n0 = fmaxf(st.m0, mx0), n1 = fmaxf(st.m1, mx1);
    const float a0 = ex2(st.m0 - n0), a1 = ex2(st.m1 - n1);
    st.l0 *= a0, st.l1 *= a1;
#pragma unroll
    for (int m = 0; m < D / 16; ++m) o[m][0] *= a0, o[m][1] *= a1, o[m][2] *= a0, o[m][3] *= a1;
    st.m0 = n0, st.m1 = n1;
  }
  const float p0 = ex2(fmaf(s[0], scale_log2, -st.m0));
  const float p1 = ex2(fmaf(s[1], scale_log2, -st.m1));
  const float p2 = ex2(fmaf(s[2], scale_log2, -st.m0));
  const float p3 = ex2(fmaf(s[3], scale_log2, -st.m1));
  st.l0 += p0 + p2, st.l1 += p1 + p3;
  b0 = movmatrix_trans(pack_f16x2(p0, p1));
  b1 = movmatrix_trans(pack_f16x2(p2, p3));
}

template <int D, int MODE>
__device__ __forceinline__ void page_attend(uint8_t *rec, int ntok, int lane, int log2_group,
                                            const ScaleIdx &si, const uint32_t (&qf)[D / 16][2],
                                            float scale_log2, SoftmaxState &st,
                                            float (&o)[D / 16][4]) {
  constexpr int PB = kBlock * D * mode_bits(MODE) / 8;
  const int gid = lane >> 2, t4 = lane & 3;
  if (ntok < kBlock) {
    // Zero the V rows past the valid count so P=0 never meets a non-finite value.
    constexpr int rowB = D * mode_bits(MODE) / 8;
    for (int off = ntok * rowB + 4 * lane; off < PB; off += 128)
      *reinterpret_cast<uint32_t *>(rec + PB + off) = 0u;
    __syncwarp();
  }
  const __half *ksc = reinterpret_cast<const __half *>(rec + 2 * PB);
  const __half *vsc = ksc + ((kBlock * D) >> log2_group);
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  page_qk<D, MODE>(rec, ksc, si, gid, t4, qf, s);
  uint32_t b0, b1;
  page_softmax<D>(s, ntok, gid, scale_log2, st, o, b0, b1);
  page_pv<D, MODE>(rec + PB, vsc, si, gid, t4, b0, b1, o);
}

template <int D>
__global__ void __launch_bounds__(DecodeTraits<D>::kThreads, 3)
    decode_partials_kernel(const DecodeParams p) {
  using T = DecodeTraits<D>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, t4 = lane & 3;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y / p.qgroups, qg = blockIdx.y % p.qgroups;
  const int b = blockIdx.z;
  const int q0 = kvh * p.gqa + qg * 8;
  const int nq = min(8, p.gqa - qg * 8);
  const int nblk = p.seq_blocks ? min(p.seq_blocks[b], p.max_blocks) : p.max_blocks;
  const int lo = split * p.chunk, hi = min(lo + p.chunk, nblk);

  uint8_t *ring = smem + warp * T::kRing;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + T::kWarps * T::kRing) + warp * T::kSlots;
  uint32_t *slot_start = reinterpret_cast<uint32_t *>(smem + T::kWarps * T::kRing +
                                                      T::kWarps * T::kSlots * 8) + warp * T::kSlots;
  uint32_t *slot_meta = slot_start + T::kWarps * T::kSlots;

  // Query fragments (B operand of Q.K^T), permuted like the K fragments.
  uint32_t qf[T::kTiles][2];
  {
    uint32_t qw[T::DK / 2];
    if (gid < nq) {
      const __half *qp = p.q + (int64_t)b * p.q_bs + (int64_t)(q0 + gid) * p.q_hs + t4 * T::DK;
#pragma unroll
      for (int i = 0; i < T::DK / 8; ++i) {
        const uint4 v = __ldg(reinterpret_cast<const uint4 *>(qp) + i);
        qw[4 * i] = v.x, qw[4 * i + 1] = v.y, qw[4 * i + 2] = v.z, qw[4 * i + 3] = v.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < T::DK / 2; ++i) qw[i] = 0u;
    }
#pragma unroll
    for (int c = 0; c < T::kTiles; ++c) {
      const int j = c >> 1, hb = c & 1;
      qf[c][0] = prmt(qw[4 * j + hb], qw[4 * j + 2 + hb], 0x5410);
      qf[c][1] = prmt(qw[4 * j + hb], qw[4 * j + 2 + hb], 0x7632);
    }
  }
  const int lg = p.log2_group;
  ScaleIdx si;
  si.k0 = (gid * D + t4 * T::DK) >> lg;
  si.k1 = ((gid + 8) * D + t4 * T::DK) >> lg;
  si.va = ((2 * t4) * D + gid * T::DV) >> lg;
  si.vb = ((2 * t4 + 1) * D + gid * T::DV) >> lg;
  si.vc = ((2 * t4 + 8) * D + gid * T::DV) >> lg;
  si.vd = ((2 * t4 + 9) * D + gid * T::DV) >> lg;

  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < T::kSlots; ++i) mbar_init(smem_u32(&bars[i]), 1);
    fence_mbar_init();
  }
  __syncwarp();

  float o[T::kTiles][4];
#pragma unroll
  for (int m = 0; m < T::kTiles; ++m) o[m][0] = o[m][1] = o[m][2] = o[m][3] = 0.f;
  SoftmaxState st{-INFINITY, -INFINITY, 0.f, 0.f};

  const int64_t *trow = p.table + (int64_t)b * p.table_stride;
  const int64_t scale_bytes = (int64_t)2 * ((kBlock * D) >> lg);
  int pj = lo + warp;
  uint32_t head = 0, tail = 0;  // virtual byte counters of the ring
  int issued = 0, consumed = 0;
  bool timed_out = false;

  while (true) {
    // Producer: keep up to kSlots records in flight while the ring has room.
    while (issued - consumed < T::kSlots && pj < hi) {
      const int64_t d = __ldg(trow + pj);
      const int mode = desc_mode(d);
      if (mode == AKV_MODE_SKIP) {
        pj += T::kWarps;
        continue;
      }
      const int64_t pb = payload_bytes(D, mode);
      const uint32_t rb =
          (uint32_t)((2 * pb + (mode == AKV_MODE_FP16 ? 0 : 2 * scale_bytes) + 15) & ~(int64_t)15);
      const int64_t poff = desc_offset(d);
      if ((poff & 15) || poff < 0 || poff + (int64_t)p.kv_heads * rb > p.arena_bytes) {
        if (lane == 0) set_status(p.status, AKV_DEV_BAD_DESCRIPTOR);
        pj += T::kWarps;
        continue;
      }
      uint32_t start = head;
      const uint32_t phys = start & (T::kRing - 1);
      if (phys + rb > (uint32_t)T::kRing) start += T::kRing - phys;  // wrap to the next lap
      if (start + rb - tail > (uint32_t)T::kRing) break;              // wait for room
      const int slot = issued % T::kSlots;
      if (lane == 0) {
        slot_start[slot] = start;
        slot_meta[slot] = (uint32_t)mode | ((uint32_t)desc_ntok(d) << 8);
        fence_proxy_async_smem();  // prior generic reads of this space before the async write
        const uint32_t bar = smem_u32(&bars[slot]);
        mbar_expect_tx(bar, rb);
        bulk_g2s(smem_u32(ring + (start & (T::kRing - 1))), p.arena + poff + (int64_t)kvh * rb, rb, bar);
      }
      head = start + rb;
      ++issued;
      pj += T::kWarps;
    }
    __syncwarp();
    if (issued == consumed) break;
    // Consumer: the oldest record.
    const int slot = consumed % T::kSlots;
    if (!mbar_wait_bounded(smem_u32(&bars[slot]), (uint32_t)(consumed / T::kSlots) & 1u)) {
      timed_out = true;
      break;
    }
    const uint32_t meta = slot_meta[slot];
    uint8_t *rec = ring + (slot_start[slot] & (T::kRing - 1));
    const int ntok = (int)(meta >> 8);
    switch (meta & 3u) {
      case AKV_MODE_INT4:
        page_attend<D, AKV_MODE_INT4>(rec, ntok, lane, lg, si, qf, p.scale_log2, st, o);
        break;
      case AKV_MODE_INT8:
        page_attend<D, AKV_MODE_INT8>(rec, ntok, lane, lg, si, qf, p.scale_log2, st, o);
        break;
      default:
        page_attend<D, AKV_MODE_FP16>(rec, ntok, lane, lg, si, qf, p.scale_log2, st, o);
        break;
    }
    __syncwarp();
    ++consumed;
    tail = issued > consumed ? slot_start[consumed % T::kSlots] : head;
  }
  if (timed_out) {
    if (lane == 0) set_status(p.status, AKV_DEV_TIMEOUT);
    // Let the copies still in flight land (bounded) before the CTA exits.
    for (int k = consumed; k < issued; ++k)
      if (!mbar_wait_bounded(smem_u32(&bars[k % T::kSlots]), (uint32_t)(k / T::kSlots) & 1u)) break;
  }

  // ---- merge the 4 warps in shared memory, write one partial per query head
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    st.l0 += __shfl_xor_sync(0xffffffffu, st.l0, off);
    st.l1 += __shfl_xor_sync(0xffffffffu, st.l1, off);
  }
  __syncthreads();
  constexpr int RS = D + 2;
  float *red = reinterpret_cast<float *>(smem);
  float *mine = red + warp * 8 * RS;
  const int h0 = 2 * t4, h1 = 2 * t4 + 1;
#pragma unroll
  for (int m = 0; m < T::kTiles; ++m) {
    const int dd = T::DV * gid + 2 * m;
    mine[h0 * RS + dd] = o[m][0];
    mine[h1 * RS + dd] = o[m][1];
    mine[h0 * RS + dd + 1] = o[m][2];
    mine[h1 * RS + dd + 1] = o[m][3];
  }
  if (gid == 0) {
    mine[h0 * RS + D] = st.m0, mine[h0 * RS + D + 1] = st.l0;
    mine[h1 * RS + D] = st.m1, mine[h1 * RS + D + 1] = st.l1;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < nq * D; idx += T::kThreads) {
    const int n = idx / D, dd = idx % D;
    float mw[T::kWarps], top = -INFINITY;
#pragma unroll
    for (int w = 0; w < T::kWarps; ++w) {
      mw[w] = red[(w * 8 + n) * RS + D];
      top = fmaxf(top, mw[w]);
    }
    float acc = 0.f, den = 0.f;
#pragma unroll
    for (int w = 0; w < T::kWarps; ++w) {
      const float e = mw[w] == -INFINITY ? 0.f : ex2(mw[w] - top);
      acc += e * red[(w * 8 + n) * RS + dd];
      den += e * red[(w * 8 + n) * RS + D + 1];
    }
    float *out = p.partials + (((int64_t)b * p.q_heads + q0 + n) * p.splits + split) * RS;
    out[dd] = acc;
    if (dd == 0) out[D] = top, out[D + 1] = den;
  }
}

// One CTA of head_dim threads per (query head, sequence).
template <int D>
__global__ void __launch_bounds__(D) merge_kernel(const float *__restrict__ partials, int q_heads,
                                                  int splits, __half *__restrict__ out, int64_t obs,
                                                  int64_t ohs, float *__restrict__ state) {
  constexpr int RS = D + 2;
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const float *base = partials + ((int64_t)b * q_heads + h) * (int64_t)splits * RS;
  float top = -INFINITY;
  for (int s = 0; s < splits; ++s) top = fmaxf(top, base[s * RS + D]);
  float num = 0.f, den = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float m = base[s * RS + D];
    const float w = m == -INFINITY ? 0.f : ex2(m - top);  // empty split weighs 0 (triton_decode.py:78)
    num += w * base[s * RS + d];
    den += w * base[s * RS + D + 1];
  }
  if (out) out[(int64_t)b * obs + (int64_t)h * ohs + d] = __float2half_rn(den > 0.f ? num / den : 0.f);
  if (state) {
    float *st = state + ((int64_t)b * q_heads + h) * RS;
    st[d] = num;
    if (d == 0) st[D] = top, st[D + 1] = den;
  }
}

template <int D>
static int launch_decode(const DecodeParams &p, int batch, cudaStream_t stream) {
  using T = DecodeTraits<D>;
  if (cudaFuncSetAttribute(decode_partials_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           T::kSmem) != cudaSuccess)
    return AKV_ERR_CUDA;
  const dim3 grid(p.splits, p.kv_heads * p.qgroups, batch);
  decode_partials_kernel<D><<<grid, T::kThreads, T::kSmem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_CUDA;
}

static int ilog2_exact(int x) {
  int l = 0;
  while ((1 << l) < x) ++l;
  return (1 << l) == x ? l : -1;
}

}  // namespace akv

using namespace akv;

extern "C" int64_t akv_workspace_bytes(int batch, int q_heads, int splits, int head_dim) {
  if (batch <= 0 || q_heads <= 0 || splits <= 0 || head_dim <= 0) return 0;
  return (int64_t)batch * q_heads * splits * (head_dim + 2) * (int64_t)sizeof(float);
}

extern "C" int akv_decode_partials(const void *arena, int64_t arena_bytes, const int64_t *table,
                                   int64_t table_stride, const int32_t *seq_blocks,
                                   int32_t max_blocks, const void *query, int64_t q_batch_stride,
                                   int64_t q_head_stride, int32_t batch, int32_t q_heads,
                                   int32_t kv_heads, int32_t head_dim, int32_t group, float scale,
                                   int32_t splits, float *partials, int32_t *dev_status,
                                   void *stream) {
  if (!arena || !table || !query || !partials) return AKV_ERR_INVALID;
  if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || splits <= 0 || max_blocks < 0) return AKV_ERR_INVALID;
  if (q_heads % kv_heads) return AKV_ERR_INVALID;
  if (table_stride < max_blocks || arena_bytes < 0 || !isfinite(scale)) return AKV_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return AKV_ERR_UNSUPPORTED;
  const int lg = ilog2_exact(group);
  if (lg < 0 || group < head_dim / 4 || group > 16 * head_dim) return AKV_ERR_UNSUPPORTED;
  if (((uintptr_t)arena & 15) || ((uintptr_t)query & 15)) return AKV_ERR_INVALID;
  if (q_batch_stride % 8 || q_head_stride % 8) return AKV_ERR_INVALID;
  if (batch > 65535 || (int64_t)kv_heads * ((q_heads / kv_heads + 7) / 8) > 65535) return AKV_ERR_UNSUPPORTED;
  DecodeParams p;
  p.arena = (const uint8_t *)arena;
  p.arena_bytes = arena_bytes;
  p.table = table;
  p.table_stride = table_stride;
  p.seq_blocks = seq_blocks;
  p.max_blocks = max_blocks;
  p.q = (const __half *)query;
  p.q_bs = q_batch_stride;
  p.q_hs = q_head_stride;
  p.q_heads = q_heads;
  p.kv_heads = kv_heads;
  p.gqa = q_heads / kv_heads;
  p.qgroups = (p.gqa + 7) / 8;
  p.splits = splits;
  p.chunk = (max_blocks + splits - 1) / splits;
  p.log2_group = lg;
  p.scale_log2 = scale * 1.4426950408889634f;  // scores in base 2: exp(x) = 2^(x log2 e)
  p.partials = partials;
  p.status = dev_status;
  cudaStream_t s = (cudaStream_t)stream;
  return head_dim == 64 ? launch_decode<64>(p, batch, s) : launch_decode<128>(p, batch, s);
}

extern "C" int akv_merge(const float *partials, int32_t batch, int32_t q_heads, int32_t splits,
                         int32_t head_dim, void *out, int64_t out_batch_stride,
                         int64_t out_head_stride, float *state_out, void *stream) {
  if (!partials || (!out && !state_out)) return AKV_ERR_INVALID;
  if (batch <= 0 || q_heads <= 0 || splits <= 0 || batch > 65535) return AKV_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return AKV_ERR_UNSUPPORTED;
  const dim3 grid(q_heads, batch);
  cudaStream_t s = (cudaStream_t)stream;
  if (head_dim == 64)
    merge_kernel<64><<<grid, 64, 0, s>>>(partials, q_heads, splits, (__half *)out, out_batch_stride,
                                         out_head_stride, state_out);
  else
    merge_kernel<128><<<grid, 128, 0, s>>>(partials, q_heads, splits, (__half *)out,
                                           out_batch_stride, out_head_stride, state_out);
  return cudaGetLastError() == cudaSuccess ? AKV_OK : AKV_ERR_CUDA;
}

extern "C" int akv_packed_attention(const void *arena, int64_t arena_bytes, const int64_t *table,
                                    int64_t table_stride, const int32_t *seq_blocks,
                                    int32_t max_blocks, const void *query, int64_t q_batch_stride,
                                    int64_t q_head_stride, int32_t batch, int32_t q_heads,
                                    int32_t kv_heads, int32_t head_dim, int32_t group, float scale,
                                    int32_t splits, void *out, int64_t out_batch_stride,
                                    int64_t out_head_stride, void *workspace,
                                    int64_t workspace_bytes, int32_t *dev_status, void *stream) {
  if (!out || !workspace) return AKV_ERR_INVALID;
  if (workspace_bytes < akv_workspace_bytes(batch, q_heads, splits, head_dim)) return AKV_ERR_INVALID;
  int st = akv_decode_partials(arena, arena_bytes, table, table_stride, seq_blocks, max_blocks, query,
                               q_batch_stride, q_head_stride, batch, q_heads, kv_heads, head_dim,
                               group, scale, splits, (float *)workspace, dev_status, stream);
  if (st != AKV_OK) return st;
  return akv_merge((const float *)workspace, batch, q_heads, splits, head_dim, out, out_batch_stride,
                   out_head_stride, nullptr, stream);
}

// ===================================================== allocation-free variant
// akv_packed_attention_static: the same decode + merge, with the split-K
// partials in a fixed array compiled into this library instead of a workspace
// the caller allocates.  For callers that cannot allocate device memory: hosts
// that reserve all of HBM up front for their own pool (a serving engine's KV
// pool), latency-critical decode loops where cudaMalloc/cudaFree would
// synchronize the device, and bindings that hold raw pointers but no allocator.
//
// Every GPU that loads the library holds the array (kStaticScratchBytes) until
// the process exits.  All calls on a device share it and it keeps the last
// call's contents: each call rewrites every partial it reads before reading
// it, so nothing needs clearing, but calls whose kernels overlap on the GPU
// (different streams without ordering between them) race on it.
namespace akv {
constexpr int64_t kStaticScratchBytes = 8ll << 20;  // 8 MiB per GPU
static __device__ __align__(256) float g_static_partials[kStaticScratchBytes / sizeof(float)];
}  // namespace akv

#include <mutex>

namespace {
std::mutex g_static_mu;
void *g_static_ptr[256];  // device address of g_static_partials, per device ordinal
}  // namespace

extern "C" int64_t akv_static_scratch_bytes(void) { return akv::kStaticScratchBytes; }

extern "C" int akv_packed_attention_static(const void *arena, int64_t arena_bytes, const int64_t *table,
                                           int64_t table_stride, const int32_t *seq_blocks,
                                           int32_t max_blocks, const void *query, int64_t q_batch_stride,
                                           int64_t q_head_stride, int32_t batch, int32_t q_heads,
                                           int32_t kv_heads, int32_t head_dim, int32_t group, float scale,
                                           int32_t splits, void *out, int64_t out_batch_stride,
                                           int64_t out_head_stride, int32_t *dev_status, void *stream) {
  if (!out) return AKV_ERR_INVALID;
  const int64_t need = akv_workspace_bytes(batch, q_heads, splits, head_dim);
  if (need <= 0) return AKV_ERR_INVALID;
  if (need > akv::kStaticScratchBytes) return AKV_ERR_SCRATCH;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256) return AKV_ERR_CUDA;
  void *scratch = nullptr;
  {
    // First call on a device: look up the array's device address with that device current.
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_ptr[dev]) {
      void *p = nullptr;
      if (cudaGetSymbolAddress(&p, akv::g_static_partials) != cudaSuccess || !p) return AKV_ERR_CUDA;
      g_static_ptr[dev] = p;
    }
    scratch = g_static_ptr[dev];
  }
  return akv_packed_attention(arena, arena_bytes, table, table_stride, seq_blocks, max_blocks, query,
                              q_batch_stride, q_head_stride, batch, q_heads, kv_heads, head_dim, group,
                              scale, splits, out, out_batch_stride, out_head_stride, scratch, need,
                              dev_status, stream);
}
