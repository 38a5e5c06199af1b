// Paged decode attention over mixed FP16/INT8/INT4 pages (persistent stream-K),
// and the log-sum-exp merge of its partial states.
//
// Reference: src/anchorkv/triton_decode.py:35-104 (one program per (query head,
// split), pages strided across splits, fp32 online softmax, fp16 rounding of
// dequantised values, LSE merge), whose numerics it reproduces with a
// different execution plan:
//
//  * work is the flattened space of (sequence, KV head, query-head group, page)
//    items; every resident warp takes one contiguous range of it (stream-K), so
//    the load is balanced at page granularity and a warp's bulk-copy pipeline
//    stays full across sequence boundaries;
//  * each warp streams its own pages: it turns 32 page descriptors at a time
//    into ready records lane-parallel (one lane per page, descriptor loads a
//    window ahead, a ballot marks the pages to copy), skips evicted or
//    invisible pages without reading them, and bulk-copies each record
//    (cp.async.bulk, mbarrier completion, no multicast; lane 0 issues) into a
//    private 13 KB shared-memory ring the moment it frees room, so the copy
//    pipeline needs no hand-off between warps; an SM's 16 warps form one CTA,
//    so they share one scheduler age and finish together;
//  * V payloads are stored with their 16-byte units swizzled inside 128-byte
//    lines (v_swizzle), so the V fragment loads from the ring hit 32 banks;
//  * INT8 and INT4 pages travel in pairs (two pages of one item and mode, one
//    ring slot, one barrier, one softmax step), which halves the per-page
//    control work of the loop;
//  * a warp serves every query head of its KV head (up to 8 per pass; the
//    reference re-reads each KV page once per query head);
//  * a page's K/V are dequantised in registers straight into tensor-core
//    fragments (exact: the integer is formed in fp16 by an exponent trick and
//    multiplied by the fp16 scale with one rounding, matching
//    fp16(int * float(scale)) of packed_decode.py:45 / triton_decode.py:31),
//    for K and V alike;
//  * Q.K^T and P.V run as mma.sync m16n8k16 (f16 x f16 -> f32): 16 tokens x 8
//    query heads per page, 2 * head_dim/16 MMAs per page;
//  * the online softmax is fp32 in base 2; the running max only moves (one
//    warp vote, then a shuffle reduction) when a page exceeds it by more than
//    2^8, so P stays <= 256 in fp16 and most pages need no reduction at all;
//  * each warp writes one partial state (acc[D], m, l) per item it touched into
//    the caller's workspace; the merge kernel combines the few warps that
//    share an item.  The workspace starts with a header describing the
//    decomposition, so merging needs nothing but the workspace.
#include <math.h>

#include <string.h>

#include <algorithm>
#include <atomic>
#include <mutex>

#include "akv_common.cuh"

namespace akv {

// One CTA per SM, holding all of the SM's streaming warps (16 at 128
// registers).  The warp schedulers favour older CTAs: with four 4-warp CTAs
// per SM the youngest CTA's warps finished about 15 % after the oldest's on
// equal work, and that spread was the decode's tail.  Warps of one CTA share
// one age and finish together.  Small problems launch fewer warps per CTA so
// that every CTA still has an SM of its own.
template <int D>
struct DecodeTraits {
  static constexpr int kMaxWarps = 16;  // independent streaming warps per CTA, at most
  static constexpr int kMaxThreads = kMaxWarps * 32;
  static constexpr int kRing = 13312;   // bytes of ring per warp (3 INT4 page pairs)
  static constexpr int kSlots = 8;      // records in flight per warp
  static constexpr int DK = D / 4;      // K dims a lane owns per row
  static constexpr int DV = D / 8;      // V dims a lane owns per row
  static constexpr int kTiles = D / 16;
  // A warp's shared memory: its ring, then its slot barriers and records.
  static constexpr int kWarpBytes = kRing + kSlots * (8 + 4 + 4 + 4);
  static constexpr int kSmemMax = kMaxWarps * kWarpBytes;
  static_assert(kRing % 16 == 0 && kWarpBytes % 16 == 0, "rings stay 16-byte aligned");
  static_assert(kRing >= 4 * kBlock * D, "a ring must hold one FP16 record");
  // Two INT8 records with the finest scale group (32) form the largest pair.
  static_assert(kRing >= 2 * (2 * kBlock * D + 2 * (kBlock * D / 32) * 2 + 16), "a ring must hold a pair");
};

// Workspace header (int32 words), written by the decode kernel, read by merge.
enum HeaderField {
  kMagic, kWarpsF, kSmaxF, kRangeF, kMaxBlocksF, kItemsF, kKvHeadsF, kQGroupsF, kGqaF,
  kHeadDimF, kSlotHeadsF, kQHeadsF, kBatchF, kPartialsF, kHeaderWords
};
constexpr int32_t kHeaderMagic = 0x414b5633;  // "AKV3"
constexpr int64_t kHeaderBytes = 256;
// Workspace: the header, then the partial states (kPartialsF holds their
// offset in 4-byte words).

// Division by a per-launch constant d for dividends 0 <= n < 2^31:
// q = (umulhi(n, mul) + n) >> shift with shift = ceil(log2 d) and
// mul = floor(2^32 (2^shift - d) / d) + 1 (Granlund and Montgomery, "Division
// by invariant integers using multiplication", 1994).  Three instructions in
// place of a runtime integer division.
struct FastDiv {
  uint32_t mul, shift;
};
__device__ __forceinline__ int fdiv(int n, FastDiv f) {
  return (int)((__umulhi((uint32_t)n, f.mul) + (uint32_t)n) >> f.shift);
}
static FastDiv fast_div(uint32_t d) {  // d >= 1
  uint32_t shift = 0;
  while ((1ull << shift) < d) ++shift;
  const uint64_t mul = ((1ull << 32) * ((1ull << shift) - d)) / d + 1;
  return FastDiv{(uint32_t)mul, shift};
}

struct DecodeParams {
  const uint8_t *arena;
  int64_t arena_bytes;
  const int64_t *table;
  int64_t table_stride;
  const int32_t *seq_blocks;
  int32_t max_blocks;
  const __half *q;
  int64_t q_bs, q_hs;
  int32_t batch, q_heads, kv_heads, gqa, qgroups, items, log2_group;
  int32_t warps, range, smax, slot_heads;
  FastDiv fd_mb, fd_ipb, fd_qgroups;  // max_blocks, kv_heads * qgroups, qgroups
  float scale_log2;
  int32_t *header;
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
// 2t4+8, 2t4+9 at column gid*DV.  Two 16-bit indices per word.
struct ScaleIdx {
  uint32_t k, vab, vcd;
  uint32_t vo;  // the lane's stored V row-2t4 offset: INT4 bits 0-9, INT8 10-19, FP16 20-31
  __device__ __forceinline__ int k0() const { return (int)(k & 0xffff); }
  __device__ __forceinline__ int k1() const { return (int)(k >> 16); }
  __device__ __forceinline__ int va() const { return (int)(vab & 0xffff); }
  __device__ __forceinline__ int vb() const { return (int)(vab >> 16); }
  __device__ __forceinline__ int vc() const { return (int)(vcd & 0xffff); }
  __device__ __forceinline__ int vd() const { return (int)(vcd >> 16); }
};

// ---------------------------------------------------------------- Q . K^T
// S[token][head] for the page's 16 tokens (rows gid, gid+8 of this lane) and
// query heads 2t4, 2t4+1.  The contraction dim is permuted identically in the
// K (A) and Q (B) fragments: k16 chunk c = 2j + hb takes, from the lane's 8-dim
// word group j, dims {2hb, 2hb+4} (fragment cols 2t4, 2t4+1) and
// {2hb+1, 2hb+5} (cols 2t4+8, 2t4+9).  All chunks accumulate into one tile:
// the other page of a slot and the other warps hide the chain's latency, while
// two tiles cost a register quad and a sum per page (3 % slower on the mixed
// layer).
template <int D, int MODE, bool SLAB>
__device__ __forceinline__ void page_qk(const uint8_t *rec, const __half *ksc, const ScaleIdx &si,
                                        int gid, int t4, const uint32_t (&qf)[D / 16][2],
                                        float (&s)[4]) {
  using T = DecodeTraits<D>;
  constexpr int bits = mode_bits(MODE);
  constexpr int rowB = D * bits / 8;
  constexpr int W = T::DK * bits / 32;  // words of one row slice
  constexpr int NJ = D / 32;            // 8-dim word groups per slice
  constexpr int WJ = W / NJ;            // words per group (1, 2 or 4)
  constexpr bool WHOLE = W <= 8;        // narrow slices load at once, wide ones per group
  const uint8_t *row0 = rec + gid * rowB + t4 * (W * 4);
  const uint8_t *row1 = row0 + 8 * rowB;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  uint32_t sc0 = 0, sc1 = 0;
  if constexpr (MODE != AKV_MODE_FP16) {
    sc0 = rep_half(ksc + (SLAB ? 0 : si.k0()));
    sc1 = SLAB ? sc0 : rep_half(ksc + si.k1());
  }
  uint32_t a0w[WHOLE ? W : 1], a1w[WHOLE ? W : 1];
  if constexpr (WHOLE) {
    lds_words<W>(row0, a0w);
    lds_words<W>(row1, a1w);
  }
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    uint32_t r0[WJ], r1[WJ];
    if constexpr (WHOLE) {
#pragma unroll
      for (int i = 0; i < WJ; ++i) r0[i] = a0w[WJ * j + i], r1[i] = a1w[WJ * j + i];
    } else {
      lds_words<WJ>(row0 + 4 * WJ * j, r0);
      lds_words<WJ>(row1 + 4 * WJ * j, r1);
    }
    if constexpr (MODE == AKV_MODE_INT4) {
      uint32_t x0 = r0[0], x1 = r1[0];
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        mma_16816(acc, hmul2(int4_lo_to_f16x2(x0), sc0), hmul2(int4_lo_to_f16x2(x1), sc1),
                  hmul2(int4_hi_to_f16x2(x0), sc0), hmul2(int4_hi_to_f16x2(x1), sc1),
                  qf[2 * j + hb][0], qf[2 * j + hb][1]);
        x0 >>= 8, x1 >>= 8;
      }
    } else if constexpr (MODE == AKV_MODE_INT8) {
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const uint32_t lo = sel8(2 * hb), hi = sel8(2 * hb + 1);
        mma_16816(acc, hmul2(int8_to_f16x2(prmt(r0[0], r0[1], lo)), sc0),
                  hmul2(int8_to_f16x2(prmt(r1[0], r1[1], lo)), sc1),
                  hmul2(int8_to_f16x2(prmt(r0[0], r0[1], hi)), sc0),
                  hmul2(int8_to_f16x2(prmt(r1[0], r1[1], hi)), sc1),
                  qf[2 * j + hb][0], qf[2 * j + hb][1]);
      }
    } else {
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {
        const uint32_t a0 = r0[hb], b0 = r0[2 + hb], a1 = r1[hb], b1 = r1[2 + hb];
        mma_16816(acc, prmt(a0, b0, 0x5410), prmt(a1, b1, 0x5410), prmt(a0, b0, 0x7632),
                  prmt(a1, b1, 0x7632), qf[2 * j + hb][0], qf[2 * j + hb][1]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) s[i] = acc[i];
}

// ------------------------------------------------------------------- P . V
// O^T[dim][head] += V^T[dim][token] * P^T[token][head].  The lane owns dims
// DV*gid + [0, DV): m-tile m's A rows gid / gid+8 are dims DV*gid + 2m / +2m+1;
// its k (token) columns 2t4, 2t4+1 / 2t4+8, 2t4+9 match the P fragment that
// movmatrix produced from the score accumulators.
template <int D, int MODE, bool SLAB>
__device__ __forceinline__ void page_pv(const uint8_t *vrec, const __half *vsc, const ScaleIdx &si,
                                        int gid, int t4, uint32_t b0, uint32_t b1,
                                        float (&o)[D / 16][4]) {
  using T = DecodeTraits<D>;
  constexpr int bits = mode_bits(MODE);
  constexpr int rowB = D * bits / 8;
  constexpr int W = T::DV * bits / 32;        // words of one row slice
  constexpr int PARTS = W >= 8 ? 2 : 1;       // load wide slices in halves (fewer live registers)
  constexpr int WP = W / PARTS;
  constexpr int TP = (D / 16) / PARTS;        // m-tiles per part
  // Stored offsets of the lane's row slices in the swizzled V payload
  // (v_swizzle): row 2t4 is c0 (worked out once per kernel into si.vo for the
  // three modes); the second half of a 32-byte slice flips bit
  // 4; row 2t4+1 flips the row bit of a line holding two or four rows, or is
  // one row further; rows +8 are 8 rows further.  Within each phase of the
  // shared-memory load the lanes hit distinct banks.
  const int c0 = (int)((si.vo >> (MODE == AKV_MODE_INT4 ? 0 : (MODE == AKV_MODE_INT8 ? 10 : 20))) &
                        (MODE == AKV_MODE_FP16 ? 0xfffu : 0x3ffu));
  constexpr int kOddRow = rowB == 64 ? 64 : (rowB == 32 ? 32 : 0);
  auto sc = [](uint32_t x, uint32_t s) { return hmul2(x, s); };  // fp16(int * scale), one rounding
  uint32_t sab = 0, scd = 0;
  if constexpr (MODE != AKV_MODE_FP16) {
    if constexpr (SLAB) {
      sab = scd = rep_half(vsc);
    } else {
      sab = pair_half(vsc + si.va(), vsc + si.vb());
      scd = pair_half(vsc + si.vc(), vsc + si.vd());
    }
  }
#pragma unroll
  for (int part = 0; part < PARTS; ++part) {
    uint32_t wa[WP], wb[WP], wc[WP], wd[WP];
    static_assert(PARTS == 1 || 4 * WP == 16, "a slice half is one 16-byte unit");
    const int ca = c0 ^ (16 * part);
    const int cb = kOddRow ? (ca ^ kOddRow) : ca + rowB;
    lds_words<WP>(vrec + ca, wa);
    lds_words<WP>(vrec + cb, wb);
    lds_words<WP>(vrec + ca + 8 * rowB, wc);
    lds_words<WP>(vrec + cb + 8 * rowB, wd);
    float(&op)[TP][4] = *reinterpret_cast<float(*)[TP][4]>(&o[TP * part][0]);
    if constexpr (MODE == AKV_MODE_INT4) {
#pragma unroll
      for (int q = 0; q < WP; ++q) {
        const uint32_t xab = prmt(wa[q], wb[q], 0x5410), yab = prmt(wa[q], wb[q], 0x7632);
        const uint32_t xcd = prmt(wc[q], wd[q], 0x5410), ycd = prmt(wc[q], wd[q], 0x7632);
#pragma unroll
        for (int mm = 0; mm < 4; ++mm) {
          const uint32_t ab = (mm < 2 ? xab : yab) >> (8 * (mm & 1));
          const uint32_t cd = (mm < 2 ? xcd : ycd) >> (8 * (mm & 1));
          mma_16816(op[4 * q + mm], sc(int4_lo_to_f16x2(ab), sab), sc(int4_hi_to_f16x2(ab), sab),
                    sc(int4_lo_to_f16x2(cd), scd), sc(int4_hi_to_f16x2(cd), scd), b0, b1);
        }
      }
    } else if constexpr (MODE == AKV_MODE_INT8) {
#pragma unroll
      for (int q = 0; q < WP; ++q) {
#pragma unroll
        for (int mm = 0; mm < 2; ++mm) {
          const uint32_t lo = sel8(2 * mm), hi = sel8(2 * mm + 1);
          mma_16816(op[2 * q + mm], sc(int8_to_f16x2(prmt(wa[q], wb[q], lo)), sab),
                    sc(int8_to_f16x2(prmt(wa[q], wb[q], hi)), sab),
                    sc(int8_to_f16x2(prmt(wc[q], wd[q], lo)), scd),
                    sc(int8_to_f16x2(prmt(wc[q], wd[q], hi)), scd), b0, b1);
        }
      }
    } else {
#pragma unroll
      for (int m = 0; m < WP; ++m)
        mma_16816(op[m], prmt(wa[m], wb[m], 0x5410), prmt(wa[m], wb[m], 0x7632),
                  prmt(wc[m], wd[m], 0x5410), prmt(wc[m], wd[m], 0x7632), b0, b1);
    }
  }
}

struct SoftmaxState {
  float m0, m1, l0, l1;  // heads 2t4, 2t4+1: running max (base 2) and this lane's sum
};

// Online softmax step over one or two pages of one item (fp32, base 2).
// Returns the fp16 P fragments for P.V.  Scores are scaled before the max, so
// any sign of the softmax scale works.  The running max moves only when a score
// exceeds it by more than 2^8 (P <= 2^8 stays exact enough in fp16 and most
// pages need no reduction).  With NP = 2 the second page is skipped when `two`
// is false.
template <int D, int NP>
__device__ __forceinline__ void pages_softmax(float (&s)[NP][4], const int (&ntok)[NP], bool two,
                                              int gid, float scale_log2, SoftmaxState &st,
                                              float (&o)[D / 16][4], uint32_t (&b)[NP][2]) {
  constexpr float slack = 8.f;
  constexpr float kNegInf = -INFINITY;
  float x[NP][4];
  float mx0 = kNegInf, mx1 = kNegInf;
#pragma unroll
  for (int r = 0; r < NP; ++r) {
#pragma unroll
    for (int i = 0; i < 4; ++i) x[r][i] = s[r][i] * scale_log2;
    if (ntok[r] < kBlock) {  // tokens past the page's valid count do not exist
      if (gid >= ntok[r]) x[r][0] = x[r][1] = kNegInf;
      if (gid + 8 >= ntok[r]) x[r][2] = x[r][3] = kNegInf;
    }
    mx0 = fmaxf(mx0, fmaxf(x[r][0], x[r][2]));
    mx1 = fmaxf(mx1, fmaxf(x[r][1], x[r][3]));
  }
  // Lazy rescale: only then reduce the max across the lanes sharing a head.
  if (__any_sync(0xffffffffu, mx0 > st.m0 + slack || mx1 > st.m1 + slack)) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float n0 = fmaxf(st.m0, mx0), n1 = fmaxf(st.m1, mx1);
    const float a0 = ex2(st.m0 - n0), a1 = ex2(st.m1 - n1);
    st.l0 *= a0, st.l1 *= a1;
#pragma unroll
    for (int m = 0; m < D / 16; ++m) o[m][0] *= a0, o[m][1] *= a1, o[m][2] *= a0, o[m][3] *= a1;
    st.m0 = n0, st.m1 = n1;
  }
#pragma unroll
  for (int r = 0; r < NP; ++r) {
    if (r > 0 && !two) break;
    const float p0 = ex2(x[r][0] - st.m0), p1 = ex2(x[r][1] - st.m1);
    const float p2 = ex2(x[r][2] - st.m0), p3 = ex2(x[r][3] - st.m1);
    st.l0 += p0 + p2, st.l1 += p1 + p3;
    b[r][0] = movmatrix_trans(pack_f16x2(p0, p1));
    b[r][1] = movmatrix_trans(pack_f16x2(p2, p3));
  }
}

// Zero the V rows past a partial page's valid count, so that P = 0 never meets
// a non-finite value.  The V payload is swizzled inside 128-byte lines, which
// may hold several rows: every word from the line of row `ntok` on is zeroed
// when the row it stores (v_swizzle maps stored to row-major offsets) is past
// the count.
template <int D, int MODE>
__device__ __forceinline__ void zero_tail(uint8_t *rec, int ntok, int lane) {
  constexpr int PB = kBlock * D * mode_bits(MODE) / 8;
  constexpr int rowB = D * mode_bits(MODE) / 8;
  for (int off = ((ntok * rowB) & ~127) + 4 * lane; off < PB; off += 128)
    if ((int)v_swizzle(D, MODE, off) >= ntok * rowB) *reinterpret_cast<uint32_t *>(rec + PB + off) = 0u;
}

// One FP16 page.
template <int D, bool SLAB>
__device__ __forceinline__ void fp16_attend(uint8_t *rec, int ntok, int lane, const ScaleIdx &si,
                                            const uint32_t (&qf)[D / 16][2], float scale_log2,
                                            SoftmaxState &st, float (&o)[D / 16][4]) {
  constexpr int PB = kBlock * D * 2;
  const int gid = lane >> 2, t4 = lane & 3;
  if (ntok < kBlock) {
    zero_tail<D, AKV_MODE_FP16>(rec, ntok, lane);
    __syncwarp();
  }
  const ScaleIdx none{0, 0, 0, 0};
  float s[1][4];
  uint32_t b[1][2];
  const int nt[1] = {ntok};
  page_qk<D, AKV_MODE_FP16, SLAB>(rec, nullptr, none, gid, t4, qf, s[0]);
  pages_softmax<D, 1>(s, nt, false, gid, scale_log2, st, o, b);
  page_pv<D, AKV_MODE_FP16, SLAB>(rec + PB, nullptr, si, gid, t4, b[0][0], b[0][1], o);
}

// A slot of one or two INT8/INT4 pages of one item, adjacent in the ring
// (`rb` bytes apart), sharing one softmax step.  INT4 pages, the cheapest per
// instruction, run both pages' Q.K (and P.V) in line, which gives the warp
// schedulers two independent instruction streams; INT8 pages share one copy of
// the code in a two-trip loop, which keeps the kernel's instruction footprint
// small.  K and V are both dequantised exactly as fp16(int * float(scale)), the
// values the reference attends over: folding V's scale into the fp16 P fragment
// instead (one rounding of p * sV per term) was 1 % faster on the mixed layer
// but doubled the error tail of short sequences with outlier channels (66 of
// 16.7 M outputs beyond 2e-3 of the reference's fp16 SDPA over the same pages,
// against 0 without it).
template <int D, int MODE, bool SLAB>
__device__ __forceinline__ void slot_attend(uint8_t *rec, uint32_t rb, bool has2, int ntok0,
                                            int ntok1, int lane, int log2_group, const ScaleIdx &si,
                                            const uint32_t (&qf)[D / 16][2], float scale_log2,
                                            SoftmaxState &st, float (&o)[D / 16][4]) {
  constexpr int PB = kBlock * D * mode_bits(MODE) / 8;
  const int gid = lane >> 2, t4 = lane & 3;
  const int npages = has2 ? 2 : 1;
  if (ntok0 < kBlock || (has2 && ntok1 < kBlock)) {
    if (ntok0 < kBlock) zero_tail<D, MODE>(rec, ntok0, lane);
    if (has2 && ntok1 < kBlock) zero_tail<D, MODE>(rec + rb, ntok1, lane);
    __syncwarp();
  }
  const int vgap = SLAB ? 1 : ((kBlock * D) >> log2_group);  // K scales, then V scales
  float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  if constexpr (MODE == AKV_MODE_INT4) {  // both pages in line
    page_qk<D, MODE, SLAB>(rec, reinterpret_cast<const __half *>(rec + 2 * PB), si, gid, t4, qf, s[0]);
    if (has2) page_qk<D, MODE, SLAB>(rec + rb, reinterpret_cast<const __half *>(rec + rb + 2 * PB), si, gid, t4, qf, s[1]);
  } else {
#pragma unroll 1
  for (int r = 0; r < npages; ++r) {
    const uint8_t *pg = rec + r * rb;
    float sr[4];
    page_qk<D, MODE, SLAB>(pg, reinterpret_cast<const __half *>(pg + 2 * PB), si, gid, t4, qf, sr);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      s[0][i] = r ? s[0][i] : sr[i];
      s[1][i] = r ? sr[i] : s[1][i];
    }
  }
  }
  const int nt[2] = {ntok0, has2 ? ntok1 : 0};
  uint32_t b[2][2];
  pages_softmax<D, 2>(s, nt, has2, gid, scale_log2, st, o, b);
  if constexpr (MODE == AKV_MODE_INT4) {
    page_pv<D, MODE, SLAB>(rec + PB, reinterpret_cast<const __half *>(rec + 2 * PB) + vgap, si, gid, t4,
                                 b[0][0], b[0][1], o);
    if (has2)
      page_pv<D, MODE, SLAB>(rec + rb + PB, reinterpret_cast<const __half *>(rec + rb + 2 * PB) + vgap, si,
                                   gid, t4, b[1][0], b[1][1], o);
  } else {
#pragma unroll 1
  for (int r = 0; r < npages; ++r) {
    const uint8_t *pg = rec + r * rb;
    page_pv<D, MODE, SLAB>(pg + PB, reinterpret_cast<const __half *>(pg + 2 * PB) + vgap, si, gid, t4,
                                 r ? b[1][0] : b[0][0], r ? b[1][1] : b[0][1], o);
  }
  }
}

// Query words of this lane for item `item`: DK dims of query head (first head of
// the item's group + gid), zeros for lanes past the group's head count.
template <int D>
__device__ __forceinline__ void load_query(const DecodeParams &p, int item, int gid, int t4,
                                           uint32_t (&qw)[D / 8]) {
  constexpr int DK = D / 4;
  const int ipb = p.kv_heads * p.qgroups;
  const int b = item / ipb, r = item - b * ipb;
  const int kvh = r / p.qgroups, qg = r - kvh * p.qgroups;
  const int nq = min(8, p.gqa - 8 * qg);
  if (gid < nq) {
    const __half *qp = p.q + (int64_t)b * p.q_bs + (int64_t)(kvh * p.gqa + 8 * qg + gid) * p.q_hs + t4 * DK;
#pragma unroll
    for (int i = 0; i < DK / 8; ++i) {
      const uint4 v = __ldg(reinterpret_cast<const uint4 *>(qp) + i);
      qw[4 * i] = v.x, qw[4 * i + 1] = v.y, qw[4 * i + 2] = v.z, qw[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < DK / 2; ++i) qw[i] = 0u;
  }
}

// B fragments of Q.K^T from the query words, permuted like the K fragments.
template <int D>
__device__ __forceinline__ void query_fragments(const uint32_t (&qw)[D / 8], uint32_t (&qf)[D / 16][2]) {
#pragma unroll
  for (int c = 0; c < D / 16; ++c) {
    const int j = c >> 1, hb = c & 1;
    qf[c][0] = prmt(qw[4 * j + hb], qw[4 * j + 2 + hb], 0x5410);
    qf[c][1] = prmt(qw[4 * j + hb], qw[4 * j + 2 + hb], 0x7632);
  }
}

// SLAB: one scale per 16-token slab (group = 16 * head_dim), the
// per-block-per-KV-head layout; false: per-row groups (32/64/128).
template <int D, bool SLAB>
__global__ void __launch_bounds__(DecodeTraits<D>::kMaxThreads, 1)
    decode_streamk_kernel(const DecodeParams p) {
  using T = DecodeTraits<D>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, t4 = lane & 3;
  // Launched as a programmatic dependent: inputs (pages, table, queries) and the
  // workspace (a previous merge may still read it) are touched only after the
  // predecessor completes.  The merge that follows may launch right away; it
  // waits for this grid in turn.
  grid_dependency_wait();
  allow_dependents_launch();
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    int32_t *h = p.header;
    h[kMagic] = kHeaderMagic, h[kWarpsF] = p.warps, h[kSmaxF] = p.smax, h[kRangeF] = p.range;
    h[kMaxBlocksF] = p.max_blocks, h[kItemsF] = p.items, h[kKvHeadsF] = p.kv_heads;
    h[kQGroupsF] = p.qgroups, h[kGqaF] = p.gqa, h[kHeadDimF] = D, h[kSlotHeadsF] = p.slot_heads;
    h[kQHeadsF] = p.q_heads, h[kBatchF] = p.batch;
    h[kPartialsF] = (int32_t)((reinterpret_cast<const uint8_t *>(p.partials) -
                               reinterpret_cast<const uint8_t *>(p.header)) / 4);
  }
  const int gw = blockIdx.x * (blockDim.x >> 5) + warp;  // warps per CTA are chosen at launch
  const int mb = p.max_blocks;
  const int total = p.items * mb;
  const int e_begin = gw * p.range;
  const int e_end = min(e_begin + p.range, total);
  if (gw >= p.warps || e_begin >= e_end) return;  // whole warps only; no CTA-wide barriers below
  const int first_item = e_begin / mb, last_seg = (e_end - 1) / mb - first_item;
  const int ipb = p.kv_heads * p.qgroups;

  uint8_t *ring = smem + warp * T::kWarpBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(ring + T::kRing);
  uint32_t *slot_start = reinterpret_cast<uint32_t *>(ring + T::kRing + T::kSlots * 8);
  uint32_t *slot_meta = slot_start + T::kSlots;
  uint32_t *slot_phys = slot_meta + T::kSlots;

  const int lg = p.log2_group;
  ScaleIdx si;
  si.k = (uint32_t)((gid * D + t4 * T::DK) >> lg) | ((uint32_t)(((gid + 8) * D + t4 * T::DK) >> lg) << 16);
  si.vab = (uint32_t)(((2 * t4) * D + gid * T::DV) >> lg) |
           ((uint32_t)(((2 * t4 + 1) * D + gid * T::DV) >> lg) << 16);
  si.vcd = (uint32_t)(((2 * t4 + 8) * D + gid * T::DV) >> lg) |
           ((uint32_t)(((2 * t4 + 9) * D + gid * T::DV) >> lg) << 16);
  si.vo = (uint32_t)v_swizzle(D, AKV_MODE_INT4, (2 * t4) * (D / 2) + gid * (T::DV / 2)) |
          ((uint32_t)v_swizzle(D, AKV_MODE_INT8, (2 * t4) * D + gid * T::DV) << 10) |
          ((uint32_t)v_swizzle(D, AKV_MODE_FP16, (2 * t4) * (2 * D) + gid * (2 * T::DV)) << 20);
  const uint32_t scale_bytes = 2u * (uint32_t)((kBlock * D) >> lg);
  const uint32_t rb4 = (2u * (uint32_t)payload_bytes(D, AKV_MODE_INT4) + 2u * scale_bytes + 15u) & ~15u;
  const uint32_t rb8 = (2u * (uint32_t)payload_bytes(D, AKV_MODE_INT8) + 2u * scale_bytes + 15u) & ~15u;
  constexpr uint32_t rb16 = 2u * kBlock * D * 2u;

  if (lane == 0) {
#pragma unroll
    for (int i = 0; i < T::kSlots; ++i) mbar_init(smem_u32(&bars[i]), 1);
    fence_mbar_init();
  }
  __syncwarp();

  // ---- page windows: 32 consecutive flattened indices, one per lane.  The
  //      descriptor loads of the next window are issued a window ahead; when a
  //      window becomes current every lane turns its descriptor into a ready
  //      record (source offset, bytes, slot meta) and a ballot marks the pages
  //      to copy, so issuing a page is a find-first-set and three shuffles.
  auto fetch = [&](int w0, int64_t &raw, int &nb) {
    const int e = w0 + lane;
    raw = 0;
    nb = 0;
    if (e < e_end) {
      const int it = fdiv(e, p.fd_mb), bb = fdiv(it, p.fd_ipb);
      nb = p.seq_blocks ? min(__ldg(p.seq_blocks + bb), mb) : mb;
      raw = __ldg(p.table + (int64_t)bb * p.table_stride + (e - it * mb));
    }
  };
  // Per lane (one page of the window each): the record's source offset, the
  // bytes of the slot this lane leads (its record, or its record and its
  // partner's), the partner's source and the slot meta.  w_mask marks the
  // lanes that lead a slot; a follower travels with its leader.
  int64_t w_src = 0, w_src2 = 0;
  uint32_t w_need = 0, w_meta = 0, w_mask = 0;
  auto prepare = [&](int w0, int64_t raw, int nb) {
    const int e = w0 + lane;
    bool ok = false, first = false;
    int mode = AKV_MODE_SKIP;
    uint32_t rb = 0;
    if (e < e_end) {
      const int it = fdiv(e, p.fd_mb), j = e - it * mb;
      first = j == 0;
      mode = j < nb ? desc_mode(raw) : AKV_MODE_SKIP;
      rb = mode == AKV_MODE_FP16 ? rb16 : (mode == AKV_MODE_INT8 ? rb8 : rb4);
      const int64_t poff = desc_offset(raw);
      ok = mode != AKV_MODE_SKIP;
      if (ok && ((poff & 15) || poff + (int64_t)p.kv_heads * rb > p.arena_bytes)) {
        set_status(p.status, AKV_DEV_BAD_DESCRIPTOR);
        ok = false;
      }
      w_src = poff + (int64_t)fdiv(it - fdiv(it, p.fd_ipb) * ipb, p.fd_qgroups) * rb;
      w_meta = (uint32_t)mode | ((uint32_t)desc_ntok(raw) << 4) | ((uint32_t)(it - first_item) << 16);
    }
    // An INT8 or INT4 page pairs with the next page of its item and mode in
    // the window: in each (item, mode) group of lanes the 1st and 2nd pages
    // share a slot, the 3rd and 4th, ...; FP16 pages and an odd page out go
    // alone.  Item boundaries are the lanes whose page starts an item.
    const uint32_t m4 = __ballot_sync(0xffffffffu, ok && mode == AKV_MODE_INT4);
    const uint32_t m8 = __ballot_sync(0xffffffffu, ok && mode == AKV_MODE_INT8);
    const uint32_t bnd = __ballot_sync(0xffffffffu, first);
    const uint32_t self = 1u << lane, below = self - 1u, above = ~(below | self);
    const uint32_t lo_bnd = bnd & (below | self), hi_bnd = bnd & above;
    const uint32_t item = (lo_bnd ? 0xffffffffu << (31 - __clz(lo_bnd)) : 0xffffffffu) &
                          (hi_bnd ? (hi_bnd & (0u - hi_bnd)) - 1u : 0xffffffffu);
    const uint32_t group = (mode == AKV_MODE_INT4 ? m4 : (mode == AKV_MODE_INT8 ? m8 : 0u)) & item;
    const bool grouped = ok && (group & self);
    const bool follower = grouped && (__popc(group & below) & 1);
    const uint32_t next = group & above;
    const int partner = grouped && !follower && next ? __ffs(next) - 1 : lane;
    w_src2 = __shfl_sync(0xffffffffu, w_src, partner);
    const uint32_t pmeta = __shfl_sync(0xffffffffu, w_meta, partner);
    w_need = partner != lane ? 2u * rb : rb;
    if (partner != lane) w_meta |= 4u | (((pmeta >> 4) & 31u) << 9);
    w_mask = __ballot_sync(0xffffffffu, ok && !follower);
  };
  int win0 = e_begin;
  int64_t nxt_raw;
  int nxt_nb;
  {
    int64_t raw;
    int nb;
    fetch(win0, raw, nb);
    fetch(win0 + 32, nxt_raw, nxt_nb);
    prepare(win0, raw, nb);
  }

  uint32_t head = 0, tail = 0, head_p = 0;  // ring counters (virtual) and write position
  uint32_t issued = 0, consumed = 0;         // slots issued / consumed
  bool timed_out = false;

  uint32_t qf[T::kTiles][2];
  {
    uint32_t qw[D / 8];
    load_query<D>(p, first_item, gid, t4, qw);
    query_fragments<D>(qw, qf);
  }
  float o[T::kTiles][4];
#pragma unroll
  for (int m = 0; m < T::kTiles; ++m) o[m][0] = o[m][1] = o[m][2] = o[m][3] = 0.f;
  SoftmaxState st{-INFINITY, -INFINITY, 0.f, 0.f};
  int cur_seg = 0;

  auto finalize = [&](int seg) {
    float l0 = st.l0, l1 = st.l1;
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    const int item = first_item + seg;
    const int qg = (item % ipb) % p.qgroups;
    const int nq = min(8, p.gqa - 8 * qg);
    constexpr int PS = D + 4;  // partial row: acc[D], m, l, 2 pad (16-byte aligned rows)
    float *base = p.partials + ((int64_t)gw * p.smax + seg) * p.slot_heads * PS;
    // Scalar stores: the accumulators stay in the MMA's register quads (a
    // float2 pairing of (c0, c2) would fight that allocation on every page).
    const int h0 = 2 * t4, h1 = 2 * t4 + 1;
    if (h0 < nq) {
      float *row = base + h0 * PS + T::DV * gid;
#pragma unroll
      for (int m = 0; m < T::kTiles; ++m) row[2 * m] = o[m][0], row[2 * m + 1] = o[m][2];
      if (gid == 0) base[h0 * PS + D] = st.m0, base[h0 * PS + D + 1] = l0;
    }
    if (h1 < nq) {
      float *row = base + h1 * PS + T::DV * gid;
#pragma unroll
      for (int m = 0; m < T::kTiles; ++m) row[2 * m] = o[m][1], row[2 * m + 1] = o[m][3];
      if (gid == 0) base[h1 * PS + D] = st.m1, base[h1 * PS + D + 1] = l1;
    }
  };
  auto next_segment = [&]() {
    ++cur_seg;
#pragma unroll
    for (int m = 0; m < T::kTiles; ++m) o[m][0] = o[m][1] = o[m][2] = o[m][3] = 0.f;
    st = SoftmaxState{-INFINITY, -INFINITY, 0.f, 0.f};
    if (cur_seg <= last_seg) {  // each warp meets only a few items: load the next query directly
      uint32_t qw[D / 8];
      load_query<D>(p, first_item + cur_seg, gid, t4, qw);
      query_fragments<D>(qw, qf);
    }
  };

  while (true) {
    // Producer: keep up to kSlots records in flight while the ring has room.
    while (issued - consumed < T::kSlots) {
      if (w_mask == 0) {
        if (win0 + 32 >= e_end) break;  // no pages left
        win0 += 32;
        const int64_t raw = nxt_raw;
        const int nb = nxt_nb;
        fetch(win0 + 32, nxt_raw, nxt_nb);
        prepare(win0, raw, nb);
        continue;
      }
      const int k = __ffs(w_mask) - 1;  // the next slot's leading lane
      const uint32_t need = __shfl_sync(0xffffffffu, w_need, k);
      // Ring space: virtual byte counters (head, tail) grow monotonically (a
      // warp moves far less than 4 GB per launch) and measure occupancy; the
      // physical write position head_p is tracked beside them (no modulo).
      uint32_t start = head, start_p = head_p;
      if (issued == consumed && start_p != 0) {  // empty ring: restart at a lap boundary
        start += T::kRing - start_p;
        start_p = 0;
        tail = start;
      } else if (start_p + need > (uint32_t)T::kRing) {  // wrap to the next lap
        start += T::kRing - start_p;
        start_p = 0;
      }
      if (start + need - tail > (uint32_t)T::kRing) break;  // wait for room
      const uint32_t slot = issued % T::kSlots;
      if (lane == k) {  // the slot's leading lane holds its record(s) and issues the copies
        slot_start[slot] = start;
        slot_phys[slot] = start_p;
        slot_meta[slot] = w_meta;
        // No proxy fence before the copy: every generic read of this ring
        // space has returned its value (consumed by the page math) already.
        const uint32_t bar = smem_u32(&bars[slot]);
        mbar_expect_tx(bar, need);
        const bool pair = (w_meta & 4u) != 0;
        const uint32_t rb = pair ? need >> 1 : need;
        bulk_g2s(smem_u32(ring + start_p), p.arena + w_src, rb, bar);
        if (pair) bulk_g2s(smem_u32(ring + start_p + rb), p.arena + w_src2, rb, bar);
      }
      head = start + need;
      head_p = start_p + need;
      ++issued;
      w_mask &= w_mask - 1u;
    }
    __syncwarp();
    if (issued == consumed) break;
    // Consumer: the oldest record.
    const uint32_t slot = consumed % T::kSlots;
    if (!mbar_wait_bounded(smem_u32(&bars[slot]), (consumed / T::kSlots) & 1u)) {
      timed_out = true;
      break;
    }
    const uint32_t meta = slot_meta[slot];
    uint8_t *rec = ring + slot_phys[slot];
    const int seg = (int)(meta >> 16);
    while (cur_seg < seg) {
      finalize(cur_seg);
      next_segment();
    }
    const int ntok = (int)((meta >> 4) & 31), ntok1 = (int)((meta >> 9) & 31);
    const bool has2 = (meta & 4u) != 0;
    switch (meta & 3u) {
      case AKV_MODE_INT4:
        slot_attend<D, AKV_MODE_INT4, SLAB>(rec, rb4, has2, ntok, ntok1, lane, lg, si, qf, p.scale_log2, st, o);
        break;
      case AKV_MODE_INT8:
        slot_attend<D, AKV_MODE_INT8, SLAB>(rec, rb8, has2, ntok, ntok1, lane, lg, si, qf, p.scale_log2, st, o);
        break;
      default:
        fp16_attend<D, SLAB>(rec, ntok, lane, si, qf, p.scale_log2, st, o);
        break;
    }
    __syncwarp();
    ++consumed;
    tail = issued > consumed ? slot_start[consumed % T::kSlots] : head;
  }
  if (timed_out) {
    if (lane == 0) set_status(p.status, AKV_DEV_TIMEOUT);
    // Let the copies still in flight land (bounded) before the warp exits.
    for (uint32_t k = consumed; k < issued; ++k)
      if (!mbar_wait_bounded(smem_u32(&bars[k % T::kSlots]), (uint32_t)(k / T::kSlots) & 1u)) break;
  }
  // Items past the last record (or with no visible page) still get a partial.
  while (true) {
    finalize(cur_seg);
    if (cur_seg >= last_seg) break;
    next_segment();
  }
}

// The decomposition a merge reads back from the workspace header (the first
// 64 bytes, one vector load each for 16 lanes' worth of fields).
struct MergeGeom {
  const float *partials;
  int warps, smax, range, mb, kv_heads, qgroups, gqa, slot_heads;
};
template <int D>
__device__ __forceinline__ bool merge_geom(const int32_t *header, MergeGeom &g) {
  const int4 *hv = reinterpret_cast<const int4 *>(header);
  const int4 a = __ldcg(hv), b = __ldcg(hv + 1), c = __ldcg(hv + 2), d = __ldcg(hv + 3);
  const int f[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
  static_assert(kHeaderWords <= 16, "header fields fit one 64-byte read");
  g.partials = reinterpret_cast<const float *>(header + f[kPartialsF]);
  g.warps = f[kWarpsF], g.smax = f[kSmaxF], g.range = f[kRangeF], g.mb = f[kMaxBlocksF];
  g.kv_heads = f[kKvHeadsF], g.qgroups = f[kQGroupsF], g.gqa = f[kGqaF], g.slot_heads = f[kSlotHeadsF];
  return f[kMagic] == kHeaderMagic && f[kHeadDimF] == D;
}

// Write one merged row: the normalised fp16 output and/or the (acc, m, l) state.
template <int D>
__device__ __forceinline__ void store_row(int lane, int b, int h, int q_heads, float m, float l,
                                          const float (&acc)[D / 32], __half *out, int64_t obs, int64_t ohs,
                                          float *state) {
  constexpr int VEC = D / 32, RS = D + 2;
  if (out) {
    __half *o = out + (int64_t)b * obs + (int64_t)h * ohs + VEC * lane;
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) o[i] = __float2half_rn(acc[i] * inv);
  }
  if (state) {
    float *st = state + ((int64_t)b * q_heads + h) * RS;
#pragma unroll
    for (int i = 0; i < VEC; ++i) st[VEC * lane + i] = acc[i];
    if (lane == 0) st[D] = m, st[D + 1] = l;
  }
}

// Merge the partial states of the warps that touched each (sequence, query
// head) row, the online log-sum-exp of triton_decode._merge_parts
// (triton_decode.py:70-82).  One warp per row (a batch: each (sequence, KV
// head) spans a few warps): the row's contributors are loaded 8 at a time, so a
// row costs one L2 round trip per 8 contributors; each lane owns D/32 dims.
// Flattened work indices fit 31 bits (the plan checks), so int arithmetic.
template <int D>
__global__ void __launch_bounds__(128) merge_rows_kernel(const int32_t *__restrict__ header, int batch,
                                                         int q_heads, __half *__restrict__ out, int64_t obs,
                                                         int64_t ohs, float *__restrict__ state,
                                                         int32_t *status) {
  constexpr int PS = D + 4, VEC = D / 32, CB = 8;
  grid_dependency_wait();  // the decode grid that wrote the workspace has completed
  allow_dependents_launch();
  MergeGeom g;
  if (!merge_geom<D>(header, g)) {
    if (threadIdx.x == 0 && blockIdx.x == 0) set_status(status, AKV_DEV_BAD_DESCRIPTOR);
    return;
  }
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= batch * q_heads) return;
  const int b = row / q_heads, h = row - b * q_heads;
  const int kvh = h / g.gqa, r = h - kvh * g.gqa, qg = r >> 3, n = r & 7;
  const int item = (b * g.kv_heads + kvh) * g.qgroups + qg;
  float m = -INFINITY, l = 0.f, acc[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) acc[i] = 0.f;
  if (g.mb > 0) {
    const int w0 = item * g.mb / g.range;
    const int nc = min(((item + 1) * g.mb - 1) / g.range, g.warps - 1) - w0 + 1;
    int e = w0 * g.range, fi = e / g.mb;  // first entry of warp w0 + c, and its item
    e -= fi * g.mb;                       // ... as an offset into that item
    for (int c0 = 0; c0 < nc; c0 += CB) {
      float mw[CB], lw[CB], a[CB][VEC];
#pragma unroll
      for (int j = 0; j < CB; ++j) {
        mw[j] = -INFINITY;
        if (c0 + j < nc) {
          const int w = w0 + c0 + j;
          const float *pr = g.partials + ((int64_t)(w * g.smax + (item - fi)) * g.slot_heads + n) * PS;
          e += g.range;  // advance to warp w + 1
          while (e >= g.mb) e -= g.mb, ++fi;
          mw[j] = __ldcg(pr + D), lw[j] = __ldcg(pr + D + 1);
          if constexpr (VEC == 4) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(pr) + lane);
            a[j][0] = v.x, a[j][1] = v.y, a[j][2] = v.z, a[j][3] = v.w;
          } else {
            const float2 v = __ldcg(reinterpret_cast<const float2 *>(pr) + lane);
            a[j][0] = v.x, a[j][1] = v.y;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < CB; ++j) {
        if (mw[j] == -INFINITY) continue;  // an empty share weighs 0 (triton_decode.py:78)
        const float top = fmaxf(m, mw[j]);
        const float c = ex2(m - top), e2 = ex2(mw[j] - top);
        l = l * c + e2 * lw[j];
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] = acc[i] * c + e2 * a[j][i];
        m = top;
      }
    }
  }
  store_row<D>(lane, b, h, q_heads, m, l, acc, out, obs, ohs, state);
}

// Fold contributors w, w + stride, ... (<= w_end) of `item`, query head n of its
// group, into (m, l, acc).  Contributors are loaded CB at a time, all loads of a
// batch issued before any is combined, so a warp pays one L2 round trip per CB
// contributors; each contributor's first item advances incrementally.
template <int D>
__device__ __forceinline__ void fold_partials(const MergeGeom &g, int item, int n, int w, int w_end, int stride,
                                              int lane, float &m, float &l, float (&acc)[D / 32]) {
  constexpr int PS = D + 4, VEC = D / 32, CB = 4;
  if (w > w_end) return;
  int first = w * g.range / g.mb, rem = w * g.range - first * g.mb;
  const int step = stride * g.range, sq = step / g.mb, sr = step - sq * g.mb;
  for (; w <= w_end; w += CB * stride) {
    float mw[CB], lw[CB], a[CB][VEC];
#pragma unroll
    for (int j = 0; j < CB; ++j) {
      mw[j] = -INFINITY, lw[j] = 0.f;
#pragma unroll
      for (int i = 0; i < VEC; ++i) a[j][i] = 0.f;
      if (w + j * stride <= w_end) {
        const float *pr =
            g.partials + ((int64_t)((w + j * stride) * g.smax + (item - first)) * g.slot_heads + n) * PS;
        mw[j] = __ldcg(pr + D), lw[j] = __ldcg(pr + D + 1);
        if constexpr (VEC == 4) {
          const float4 v = __ldcg(reinterpret_cast<const float4 *>(pr) + lane);
          a[j][0] = v.x, a[j][1] = v.y, a[j][2] = v.z, a[j][3] = v.w;
        } else {
          const float2 v = __ldcg(reinterpret_cast<const float2 *>(pr) + lane);
          a[j][0] = v.x, a[j][1] = v.y;
        }
        first += sq, rem += sr;
        if (rem >= g.mb) rem -= g.mb, ++first;
      }
    }
#pragma unroll
    for (int j = 0; j < CB; ++j) {
      if (mw[j] == -INFINITY) continue;  // an empty share (or past w_end) weighs 0 (triton_decode.py:78)
      const float top = fmaxf(m, mw[j]);
      const float c = ex2(m - top), e = ex2(mw[j] - top);
      l = l * c + e * lw[j];
#pragma unroll
      for (int i = 0; i < VEC; ++i) acc[i] = acc[i] * c + e * a[j][i];
      m = top;
    }
  }
}

// The 32 entries (one per warp) that a CTA folds in shared memory.  Rows are
// padded to D + 1 floats, so the column a warp reduces spans all 32 banks.
template <int D>
struct FoldSmem {
  float acc[32][D + 1];
  float m[32], l[32];
  int bad;
};

// Fold the 32 entries of `sm` into one state: lane k of every warp weighs
// entry k, every warp reduces the max and the sum, and warp w reduces the VEC
// dims [VEC * w, VEC * w + VEC) (the dims lane w owns in a row): five shuffle
// steps per dim, instead of one warp walking the entries.  Every lane returns
// the row's max `top`, sum `den` and warp w's VEC accumulator sums `num`.
// An entry with max -inf (an empty share) weighs 0 (triton_decode.py:78).
template <int D>
__device__ __forceinline__ void cta_fold(const FoldSmem<D> &sm, int warp, int lane, float &top, float &den,
                                         float (&num)[D / 32]) {
  constexpr int VEC = D / 32;
  const float mk = sm.m[lane];
  top = mk;
#pragma unroll
  for (int o = 16; o; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, o));
  const float e = mk == -INFINITY ? 0.f : ex2(mk - top);
  den = e * sm.l[lane];
#pragma unroll
  for (int i = 0; i < VEC; ++i) num[i] = e * sm.acc[lane][VEC * warp + i];
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    den += __shfl_xor_sync(0xffffffffu, den, o);
#pragma unroll
    for (int i = 0; i < VEC; ++i) num[i] += __shfl_xor_sync(0xffffffffu, num[i], o);
  }
}

// The same merge for rows with hundreds of contributors (a long single
// sequence): one CTA of 32 warps per row, warp w folds contributors w, w+32, ...
// and the 32 warp states fold in shared memory (cta_fold).
template <int D>
__global__ void __launch_bounds__(1024) merge_wide_kernel(const int32_t *__restrict__ header, int q_heads,
                                                          __half *__restrict__ out, int64_t obs, int64_t ohs,
                                                          float *__restrict__ state, int32_t *status) {
  constexpr int VEC = D / 32, W = 32;
  __shared__ FoldSmem<D> sm;
  grid_dependency_wait();
  allow_dependents_launch();
  MergeGeom g;
  if (!merge_geom<D>(header, g)) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) set_status(status, AKV_DEV_BAD_DESCRIPTOR);
    return;
  }
  const int h = blockIdx.x, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = h / g.gqa, r = h - kvh * g.gqa, qg = r >> 3, n = r & 7;
  const int item = (b * g.kv_heads + kvh) * g.qgroups + qg;
  float m = -INFINITY, l = 0.f, acc[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) acc[i] = 0.f;
  if (g.mb > 0) {
    const int w0 = item * g.mb / g.range;
    fold_partials<D>(g, item, n, w0 + warp, min(((item + 1) * g.mb - 1) / g.range, g.warps - 1), W, lane, m, l,
                     acc);
  }
#pragma unroll
  for (int i = 0; i < VEC; ++i) sm.acc[warp][VEC * lane + i] = acc[i];
  if (lane == 0) sm.m[warp] = m, sm.l[warp] = l;
  __syncthreads();
  float top, den, num[VEC];
  cta_fold<D>(sm, warp, lane, top, den, num);
  // warp w writes dims [VEC w, VEC w + VEC), lane i < VEC dim VEC w + i
  if (lane < VEC) {
    float v = num[0];
#pragma unroll
    for (int i = 1; i < VEC; ++i)
      if (lane == i) v = num[i];
    if (out)
      out[(int64_t)b * obs + (int64_t)h * ohs + VEC * warp + lane] = __float2half_rn(v * (den > 0.f ? 1.f / den : 0.f));
    if (state) {
      float *st = state + ((int64_t)b * q_heads + h) * (D + 2);
      st[VEC * warp + lane] = v;
      if (warp == 0 && lane == 0) st[D] = top, st[D + 1] = den;
    }
  }
}

// ======================================== cross-GPU merge over peer memory
// One long sequence split over `world` GPUs: every rank decodes its page range
// into partial states, then this kernel, per (sequence, query head) row:
// (1) folds the rank's partials into `splits` part-states, one per CTA of the
//     row (CTA s folds contributors s*32 + w, stride 32 * splits),
// (2) stores each part-state into every rank's exchange buffer over NVLink
//     (plain 8-byte peer stores, each carrying its own epoch tag),
// (3) in the row's first CTA only, waits (bounded) until every part-state of
//     every rank carries this call's epoch, and (4) merges them into the output.
// The row's other CTAs store and exit, so no CTA waits on one that cannot run:
// a waiting CTA's siblings come right after it in launch order, and the host
// uses splits > 1 only while the whole grid fits the GPU at once.
//
// Exchange words.  Every value travels as one 64-bit word: the fp32 bits in the
// low half, the call's epoch in the high half.  A 64-bit store is single-copy
// atomic, so a reader that sees the epoch in a word holds that word's value of
// this call: no fence between the values and a flag, and no second trip over
// NVLink for the flag (the low-latency protocol of NCCL's LL fifo lines, at
// 64-bit granularity).  Buffer of one rank (akv_exchange_bytes): words
// [2][world][splits][rows][D + 2], slot [e & 1][r][s] holding rank r's part s
// of every row for the calls of epoch parity e & 1.  Buffers start zeroed;
// epochs start at 1, so no stale word matches.
//
// Two parities make consecutive calls safe without any extra handshake: rank
// A's call e + 2 writes the parity-(e & 1) slots again only after its call
// e + 1 finished, which needed every peer's call-(e + 1) parts of every row,
// and a peer publishes e + 1 only after its whole call-e grid (every read of
// the parity-(e & 1) slots) has completed: its decode of e + 1 waits for that
// grid, and its exchange of e + 1 waits for the decode.
constexpr int kMaxPeers = 8;
struct PeerBuffers {
  void *buf[kMaxPeers];
};

__device__ __forceinline__ void st_tagged(uint64_t *p, float a, float b, uint32_t epoch) {
  const uint64_t hi = (uint64_t)epoch << 32;
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(hi | __float_as_uint(a)),
               "l"(hi | __float_as_uint(b))
               : "memory");
}
// Load two tagged words; true when both carry `epoch`.
__device__ __forceinline__ bool ld_tagged(const uint64_t *p, uint32_t epoch, float &a, float &b) {
  uint64_t x, y;
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "l"(p) : "memory");
  a = __uint_as_float((uint32_t)x), b = __uint_as_float((uint32_t)y);
  return (uint32_t)(x >> 32) == epoch && (uint32_t)(y >> 32) == epoch;
}
// Exchange part-states per row: 4 CTAs per row while the grid stays within
// 128 CTAs (every B200 holds that many 1024-thread CTAs at once), else 1.
// world * splits <= 32 (at most 8 ranks): one waiting warp per part-state.
__host__ __device__ constexpr int exchange_splits(int64_t rows) { return rows <= 32 ? 4 : rows <= 64 ? 2 : 1; }

template <int D>
__global__ void __launch_bounds__(1024) merge_exchange_kernel(const int32_t *__restrict__ header, int q_heads,
                                                              int splits, const __grid_constant__ PeerBuffers peers,
                                                              int rank, int world,
                                                              uint32_t epoch, __half *__restrict__ out,
                                                              int64_t obs, int64_t ohs, int32_t *status) {
  constexpr int VEC = D / 32, W = 32, RW = D + 2;
  static_assert(VEC % 2 == 0, "values travel two words per store");
  __shared__ FoldSmem<D> sm;
  grid_dependency_wait();
  // The next kernel may be placed on SMs this grid leaves free once every CTA
  // of it has started; it still waits for this grid to complete.
  allow_dependents_launch();
  MergeGeom g;
  if (!merge_geom<D>(header, g)) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) set_status(status, AKV_DEV_BAD_DESCRIPTOR);
    return;
  }
  const int h = blockIdx.x / splits, s = blockIdx.x - h * splits, b = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = h / g.gqa, r = h - kvh * g.gqa, qg = r >> 3, n = r & 7;
  const int item = (b * g.kv_heads + kvh) * g.qgroups + qg;
  if (threadIdx.x == 0) sm.bad = 0;
  float m = -INFINITY, l = 0.f, acc[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) acc[i] = 0.f;
  if (g.mb > 0) {  // (1) this CTA's share of the rank's partials
    const int w0 = item * g.mb / g.range;
    fold_partials<D>(g, item, n, w0 + s * W + warp, min(((item + 1) * g.mb - 1) / g.range, g.warps - 1),
                     W * splits, lane, m, l, acc);
  }
#pragma unroll
  for (int i = 0; i < VEC; ++i) sm.acc[warp][VEC * lane + i] = acc[i];
  if (lane == 0) sm.m[warp] = m, sm.l[warp] = l;
  __syncthreads();
  float top, den, num[VEC];
  cta_fold<D>(sm, warp, lane, top, den, num);
  const int64_t rows = (int64_t)q_heads * gridDim.y, row = (int64_t)b * q_heads + h;
  const int64_t par = epoch & 1u;
  // (2) lane p of warp w stores dims [VEC w, VEC w + VEC) of this part, and
  // warp 0 its max and sum, into rank p's slot [parity][rank][s][row]
  if (lane < world) {
    uint64_t *dst = reinterpret_cast<uint64_t *>(peers.buf[lane]) +
                    (((par * world + rank) * splits + s) * rows + row) * RW;
#pragma unroll
    for (int i = 0; i < VEC; i += 2) st_tagged(dst + VEC * warp + i, num[i], num[i + 1], epoch);
    if (warp == 0) st_tagged(dst + D, top, den, epoch);
  }
  if (s != 0) return;  // the row's first CTA merges
  __syncthreads();     // every warp has read sm
  // (3) warp q waits (bounded) for part q % splits of rank q / splits
  const int parts = world * splits;
  float mq = -INFINITY, lq = 0.f, aq[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) aq[i] = 0.f;
  if (warp < parts) {
    const int src = warp / splits, sp = warp - src * splits;
    const uint64_t *st = reinterpret_cast<const uint64_t *>(peers.buf[rank]) +
                         (((par * world + src) * splits + sp) * rows + row) * RW;
    const uint64_t t0 = globaltimer();
    while (true) {
      bool got = ld_tagged(st + D, epoch, mq, lq);
#pragma unroll
      for (int i = 0; i < VEC; i += 2) got &= ld_tagged(st + VEC * lane + i, epoch, aq[i], aq[i + 1]);
      if (got) break;
      if (globaltimer() - t0 > kWaitNs) {
        sm.bad = 1;
        mq = -INFINITY;
        break;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < VEC; ++i) sm.acc[warp][VEC * lane + i] = aq[i];
  if (lane == 0) sm.m[warp] = mq, sm.l[warp] = lq;
  __syncthreads();
  if (sm.bad) {
    if (threadIdx.x == 0) set_status(status, AKV_DEV_TIMEOUT);
    return;
  }
  // (4) merge the world's parts; warp w writes output dims [VEC w, VEC w + VEC)
  cta_fold<D>(sm, warp, lane, top, den, num);
  if (lane < VEC) {
    float v = num[0];
#pragma unroll
    for (int i = 1; i < VEC; ++i)
      if (lane == i) v = num[i];
    out[(int64_t)b * obs + (int64_t)h * ohs + VEC * warp + lane] = __float2half_rn(v * (den > 0.f ? 1.f / den : 0.f));
  }
}

// Merge n already-merged states laid out [n][batch][q_heads][D+2] (e.g. gathered
// from n GPUs) into the normalised output.
template <int D>
__global__ void __launch_bounds__(256) merge_states_kernel(const float *__restrict__ states, int n,
                                                           int q_heads, int batch, __half *__restrict__ out,
                                                           int64_t obs, int64_t ohs) {
  // One warp per (sequence, query head) row, 8 rows per CTA; lane i owns dims
  // [VEC i, VEC i + VEC).  The states' maxima are loaded lane-parallel, then
  // the accumulators and sums 8 states at a time, every load of a batch issued
  // before any is used; each lane sums in state order as one thread per dim
  // would, so the result does not depend on the batching.
  constexpr int RS = D + 2, VEC = D / 32, SB = 8;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= (int64_t)batch * q_heads) return;
  const int b = (int)(row / q_heads), h = (int)(row - (int64_t)b * q_heads);
  const int64_t stride = (int64_t)batch * q_heads * RS;
  const float *base = states + row * RS;
  float top = -INFINITY;
  for (int s0 = 0; s0 < n; s0 += 32)
    if (s0 + lane < n) top = fmaxf(top, __ldg(base + (s0 + lane) * stride + D));
#pragma unroll
  for (int o = 16; o; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, o));
  float num[VEC], den = 0.f;
#pragma unroll
  for (int i = 0; i < VEC; ++i) num[i] = 0.f;
  for (int s0 = 0; s0 < n; s0 += SB) {
    float m[SB], l[SB], a[SB][VEC];
#pragma unroll
    for (int j = 0; j < SB; ++j) {
      m[j] = -INFINITY, l[j] = 0.f;
#pragma unroll
      for (int i = 0; i < VEC; ++i) a[j][i] = 0.f;
      if (s0 + j < n) {
        const float *st = base + (s0 + j) * stride;
        m[j] = __ldg(st + D), l[j] = __ldg(st + D + 1);
#pragma unroll
        for (int i = 0; i < VEC; ++i) a[j][i] = __ldg(st + VEC * lane + i);
      }
    }
#pragma unroll
    for (int j = 0; j < SB; ++j) {
      if (s0 + j >= n) break;
      const float wt = m[j] == -INFINITY ? 0.f : ex2(m[j] - top);
#pragma unroll
      for (int i = 0; i < VEC; ++i) num[i] += wt * a[j][i];
      den += wt * l[j];
    }
  }
  __half *o = out + (int64_t)b * obs + (int64_t)h * ohs + VEC * lane;
#pragma unroll
  for (int i = 0; i < VEC; ++i) o[i] = __float2half_rn(den > 0.f ? num[i] / den : 0.f);
}

// ------------------------------------------------------------------- host
struct Plan {
  int warps, range, smax, slot_heads, items, qgroups, ctas, wpc;  // wpc: warps per CTA
  int64_t bytes;
};
// Finest cut of the work the decode makes on its own: entries (pages of one
// item) a warp gets at least, against its fixed cost (query load, copy
// pipeline fill, partial write, one more merge contributor).
constexpr int64_t kMinPagesPerWarp = 16;

// CTAs of kMaxWarps warps the device holds at once (one per SM).  Constant per
// device, so it is worked out (and the kernels' shared-memory limit raised)
// once per device; later calls pay no CUDA queries for it.
template <int D>
static int device_ctas(int *out) {
  using T = DecodeTraits<D>;
  static std::atomic<int> cached[256];  // per device ordinal, 0 until worked out
  int dev = 0, sms = 0, per_sm = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return AKV_ERR_CUDA;
  const bool cacheable = dev >= 0 && dev < 256;
  if (cacheable) {
    const int c = cached[dev].load(std::memory_order_acquire);
    if (c > 0) {
      *out = c;
      return AKV_OK;
    }
  }
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return AKV_ERR_CUDA;
  int per_sm_slab = 0;
  if (cudaFuncSetAttribute(decode_streamk_kernel<D, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           T::kSmemMax) != cudaSuccess ||
      cudaFuncSetAttribute(decode_streamk_kernel<D, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           T::kSmemMax) != cudaSuccess)
    return AKV_ERR_CUDA;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_streamk_kernel<D, false>, T::kMaxThreads,
                                                    T::kSmemMax) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_slab, decode_streamk_kernel<D, true>,
                                                    T::kMaxThreads, T::kSmemMax) != cudaSuccess)
    return AKV_ERR_CUDA;
  per_sm = std::min(per_sm, per_sm_slab);  // both variants get the same decomposition
  if (per_sm < 1) return AKV_ERR_CUDA;
  *out = sms * per_sm;
  if (cacheable) cached[dev].store(sms * per_sm, std::memory_order_release);
  return AKV_OK;
}

// expand: cut finer than `splits` asks while the device has warps to spare
// (false: exactly min(resident warps, items * splits) pieces).
static int make_plan(int batch, int q_heads, int kv_heads, int head_dim, int max_blocks, int splits,
                     Plan *plan, bool expand = true) {
  if (batch <= 0 || q_heads <= 0 || kv_heads <= 0 || max_blocks < 0 || q_heads % kv_heads)
    return AKV_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return AKV_ERR_UNSUPPORTED;
  const int gqa = q_heads / kv_heads;
  Plan pl;
  pl.qgroups = (gqa + 7) / 8;
  pl.slot_heads = std::min(8, gqa);
  const int64_t items = (int64_t)batch * kv_heads * pl.qgroups;
  const int64_t total = items * max_blocks;
  if (items > (1 << 30) || total >= (1ll << 31)) return AKV_ERR_UNSUPPORTED;
  pl.items = (int)items;
  int dev_ctas = 0;
  const int st = head_dim == 64 ? device_ctas<64>(&dev_ctas) : device_ctas<128>(&dev_ctas);
  if (st != AKV_OK) return st;
  constexpr int kMaxWarps = DecodeTraits<128>::kMaxWarps;
  static_assert(DecodeTraits<64>::kMaxWarps == kMaxWarps, "one decomposition for both head dims");
  int64_t warps = (int64_t)dev_ctas * kMaxWarps;
  // splits > 0: at least that many pieces per item, and finer cuts (down to
  // kMinPagesPerWarp entries a warp) while the device has warps to spare.
  if (splits > 0)
    warps = std::min<int64_t>(warps, std::max<int64_t>(items * (int64_t)splits,
                                                       expand ? (total + kMinPagesPerWarp - 1) / kMinPagesPerWarp
                                                              : 0));
  warps = std::max<int64_t>(1, std::min<int64_t>(warps, std::max<int64_t>(total, 1)));
  const int64_t range = std::max<int64_t>(1, (total + warps - 1) / warps);
  warps = std::max<int64_t>(1, (total + range - 1) / range);
  pl.range = (int)range;
  pl.warps = (int)warps;
  pl.smax = max_blocks > 0 ? (int)(1 + (range - 1 + max_blocks - 1) / max_blocks) : 1;
  // One CTA per SM: spread fewer warps over as many SMs as they can use.
  pl.wpc = (int)std::min<int64_t>(kMaxWarps, (warps + dev_ctas - 1) / dev_ctas);
  pl.ctas = (int)((warps + pl.wpc - 1) / pl.wpc);
  pl.bytes = kHeaderBytes + (int64_t)pl.warps * pl.smax * pl.slot_heads * (head_dim + 4) * 4;
  *plan = pl;
  return AKV_OK;
}

static int ilog2_exact(int x) {
  int l = 0;
  while ((1 << l) < x) ++l;
  return (1 << l) == x ? l : -1;
}

}  // namespace akv

using namespace akv;

extern "C" int64_t akv_workspace_bytes(int batch, int q_heads, int kv_heads, int head_dim,
                                       int max_blocks, int splits) {
  Plan pl;
  if (make_plan(batch, q_heads, kv_heads, head_dim, max_blocks, splits, &pl) != AKV_OK) return -1;
  return pl.bytes;
}

namespace akv {
// Launch with programmatic stream serialization: the kernel may begin while its
// predecessor in the stream finishes (it calls grid_dependency_wait() before
// touching memory the predecessor may write or read).
template <typename... Params, typename... Args>
static cudaError_t launch_dependent(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Validate, plan and launch the decode kernel.
static int decode_launch(const void *arena, int64_t arena_bytes, const int64_t *table, int64_t table_stride,
                         const int32_t *seq_blocks, int32_t max_blocks, const void *query,
                         int64_t q_batch_stride, int64_t q_head_stride, int32_t batch, int32_t q_heads,
                         int32_t kv_heads, int32_t head_dim, int32_t group, float scale, int32_t splits,
                         void *workspace, int64_t workspace_bytes, int32_t *dev_status, cudaStream_t s) {
  if (!arena || !table || !query || !workspace) return AKV_ERR_INVALID;
  if (table_stride < max_blocks || arena_bytes < 0 || !isfinite(scale)) return AKV_ERR_INVALID;
  if (((uintptr_t)arena & 15) || ((uintptr_t)query & 15) || ((uintptr_t)workspace & 15))
    return AKV_ERR_INVALID;
  if (q_batch_stride % 8 || q_head_stride % 8) return AKV_ERR_INVALID;
  const int lg = ilog2_exact(group);
  if (lg < 0 || group < head_dim / 4 || group > 16 * head_dim) return AKV_ERR_UNSUPPORTED;
  Plan pl;
  if (int st = make_plan(batch, q_heads, kv_heads, head_dim, max_blocks, splits, &pl)) return st;
  // A workspace sized for exactly `splits` pieces per item (akv_workspace_bytes
  // sizes it for the finer cut) still runs, with that decomposition.
  if (workspace_bytes < pl.bytes &&
      make_plan(batch, q_heads, kv_heads, head_dim, max_blocks, splits, &pl, false) != AKV_OK)
    return AKV_ERR_INVALID;
  if (workspace_bytes < pl.bytes) return AKV_ERR_INVALID;
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
  p.batch = batch;
  p.q_heads = q_heads;
  p.kv_heads = kv_heads;
  p.gqa = q_heads / kv_heads;
  p.qgroups = pl.qgroups;
  p.items = pl.items;
  p.log2_group = lg;
  p.warps = pl.warps;
  p.range = pl.range;
  p.smax = pl.smax;
  p.slot_heads = pl.slot_heads;
  p.fd_mb = fast_div((uint32_t)std::max(max_blocks, 1));  // no page is divided when max_blocks is 0
  p.fd_ipb = fast_div((uint32_t)(kv_heads * pl.qgroups));
  p.fd_qgroups = fast_div((uint32_t)pl.qgroups);
  p.scale_log2 = scale * 1.4426950408889634f;  // scores in base 2: exp(x) = 2^(x log2 e)
  p.header = (int32_t *)workspace;
  p.partials = (float *)((uint8_t *)workspace + kHeaderBytes);
  p.status = dev_status;
  const bool slab = group == 16 * head_dim;
  cudaError_t err;
  if (head_dim == 64)
    err = launch_dependent(slab ? decode_streamk_kernel<64, true> : decode_streamk_kernel<64, false>, pl.ctas,
                           pl.wpc * 32, pl.wpc * DecodeTraits<64>::kWarpBytes, s, p);
  else
    err = launch_dependent(slab ? decode_streamk_kernel<128, true> : decode_streamk_kernel<128, false>, pl.ctas,
                           pl.wpc * 32, pl.wpc * DecodeTraits<128>::kWarpBytes, s, p);
  return err == cudaSuccess ? AKV_OK : AKV_ERR_CUDA;
}

// Merge launch.  The decode spreads all resident warps over the items, so few
// (sequence, head) rows mean many contributors per row (a long sequence: one
// CTA of 32 warps per row), many rows few contributors (one warp per row).
template <int D>
static cudaError_t merge_launch(const int32_t *header, int batch, int q_heads, __half *out, int64_t obs,
                                int64_t ohs, float *state, int32_t *status, cudaStream_t s) {
  const int rows = batch * q_heads;
  if (rows < 2 * 148)
    return launch_dependent(merge_wide_kernel<D>, dim3(q_heads, batch), 1024, 0, s, header, q_heads, out, obs,
                            ohs, state, status);
  return launch_dependent(merge_rows_kernel<D>, dim3((rows + 3) / 4), 128, 0, s, header, batch, q_heads, out,
                          obs, ohs, state, status);
}
}  // namespace akv

extern "C" int akv_decode_partials(const void *arena, int64_t arena_bytes, const int64_t *table,
                                   int64_t table_stride, const int32_t *seq_blocks,
                                   int32_t max_blocks, const void *query, int64_t q_batch_stride,
                                   int64_t q_head_stride, int32_t batch, int32_t q_heads,
                                   int32_t kv_heads, int32_t head_dim, int32_t group, float scale,
                                   int32_t splits, void *workspace, int64_t workspace_bytes,
                                   int32_t *dev_status, void *stream) {
  return decode_launch(arena, arena_bytes, table, table_stride, seq_blocks, max_blocks, query, q_batch_stride,
                       q_head_stride, batch, q_heads, kv_heads, head_dim, group, scale, splits, workspace,
                       workspace_bytes, dev_status, (cudaStream_t)stream);
}

extern "C" int akv_merge(const void *workspace, int32_t batch, int32_t q_heads, int32_t head_dim,
                         void *out, int64_t out_batch_stride, int64_t out_head_stride,
                         float *state_out, int32_t *dev_status, void *stream) {
  if (!workspace || (!out && !state_out)) return AKV_ERR_INVALID;
  if (batch <= 0 || q_heads <= 0 || batch > 65535 || (int64_t)batch * q_heads >= (1ll << 31))
    return AKV_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return AKV_ERR_UNSUPPORTED;
  const int32_t *header = (const int32_t *)workspace;
  cudaStream_t s = (cudaStream_t)stream;
  const cudaError_t err =
      head_dim == 64 ? merge_launch<64>(header, batch, q_heads, (__half *)out, out_batch_stride, out_head_stride,
                                        state_out, dev_status, s)
                     : merge_launch<128>(header, batch, q_heads, (__half *)out, out_batch_stride,
                                         out_head_stride, state_out, dev_status, s);
  return err == cudaSuccess ? AKV_OK : AKV_ERR_CUDA;
}

extern "C" int64_t akv_exchange_bytes(int32_t world, int32_t batch, int32_t q_heads, int32_t head_dim) {
  if (world <= 0 || world > kMaxPeers || batch <= 0 || q_heads <= 0 || (head_dim != 64 && head_dim != 128))
    return -1;
  const int64_t rows = (int64_t)batch * q_heads;
  return 2 * world * exchange_splits(rows) * rows * (head_dim + 2) * 8;  // both epoch parities, 8-byte words
}

extern "C" int akv_merge_exchange(const void *workspace, int32_t batch, int32_t q_heads, int32_t head_dim,
                                  void *const *peer_buffers, int32_t rank, int32_t world, uint32_t epoch,
                                  void *out, int64_t out_batch_stride, int64_t out_head_stride,
                                  int32_t *dev_status, void *stream) {
  if (!workspace || !peer_buffers || !out || epoch == 0) return AKV_ERR_INVALID;
  if (akv_exchange_bytes(world, batch, q_heads, head_dim) < 0 || rank < 0 || rank >= world || batch > 65535)
    return head_dim != 64 && head_dim != 128 ? AKV_ERR_UNSUPPORTED : AKV_ERR_INVALID;
  PeerBuffers peers = {};
  for (int r = 0; r < world; ++r) {
    if (!peer_buffers[r] || ((uintptr_t)peer_buffers[r] & 15)) return AKV_ERR_INVALID;
    peers.buf[r] = peer_buffers[r];
  }
  const int32_t *header = (const int32_t *)workspace;
  cudaStream_t s = (cudaStream_t)stream;
  const int splits = exchange_splits((int64_t)batch * q_heads);
  const dim3 grid(q_heads * splits, batch);
  const cudaError_t err =
      head_dim == 64 ? launch_dependent(merge_exchange_kernel<64>, grid, 1024, 0, s, header, (int)q_heads, splits,
                                        peers, (int)rank, (int)world, epoch, (__half *)out, out_batch_stride,
                                        out_head_stride, dev_status)
                     : launch_dependent(merge_exchange_kernel<128>, grid, 1024, 0, s, header, (int)q_heads, splits,
                                        peers, (int)rank, (int)world, epoch, (__half *)out, out_batch_stride,
                                        out_head_stride, dev_status);
  return err == cudaSuccess ? AKV_OK : AKV_ERR_CUDA;
}

extern "C" int akv_ipc_alloc(int64_t bytes, void **ptr, void *handle) {
  if (bytes <= 0 || !ptr || !handle) return AKV_ERR_INVALID;
  void *p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return AKV_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return AKV_ERR_CUDA;
  }
  static_assert(sizeof(h) == AKV_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return AKV_OK;
}

extern "C" int akv_ipc_open(const void *handle, void **ptr) {
  if (!handle || !ptr) return AKV_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? AKV_OK : AKV_ERR_CUDA;
}

extern "C" int akv_ipc_close(void *ptr) {
  if (!ptr) return AKV_ERR_INVALID;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? AKV_OK : AKV_ERR_CUDA;
}

extern "C" int akv_ipc_free(void *ptr) {
  if (!ptr) return AKV_ERR_INVALID;
  return cudaFree(ptr) == cudaSuccess ? AKV_OK : AKV_ERR_CUDA;
}

extern "C" int akv_merge_states(const float *states, int32_t n, int32_t batch, int32_t q_heads,
                                int32_t head_dim, void *out, int64_t out_batch_stride,
                                int64_t out_head_stride, void *stream) {
  if (!states || !out || n <= 0 || batch <= 0 || q_heads <= 0 || batch > 65535) return AKV_ERR_INVALID;
  if (head_dim != 64 && head_dim != 128) return AKV_ERR_UNSUPPORTED;
  const int64_t rows = (int64_t)batch * q_heads;
  const dim3 grid((unsigned)((rows + 7) / 8));
  cudaStream_t s = (cudaStream_t)stream;
  if (head_dim == 64)
    merge_states_kernel<64><<<grid, 256, 0, s>>>(states, n, q_heads, batch, (__half *)out,
                                                 out_batch_stride, out_head_stride);
  else
    merge_states_kernel<128><<<grid, 256, 0, s>>>(states, n, q_heads, batch, (__half *)out,
                                                  out_batch_stride, out_head_stride);
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
  if (!out) return AKV_ERR_INVALID;
  if (batch > 65535) return AKV_ERR_INVALID;
  const int st = akv_decode_partials(arena, arena_bytes, table, table_stride, seq_blocks, max_blocks, query,
                                     q_batch_stride, q_head_stride, batch, q_heads, kv_heads, head_dim, group,
                                     scale, splits, workspace, workspace_bytes, dev_status, stream);
  if (st != AKV_OK) return st;
  return akv_merge(workspace, batch, q_heads, head_dim, out, out_batch_stride, out_head_stride,
                   nullptr, dev_status, stream);
}

// ===================================================== allocation-free variant
// akv_packed_attention_static: the same decode + merge, with the partial
// states in a fixed array compiled into this library instead of a workspace
// the caller allocates.  For callers that cannot allocate device memory: hosts
// that reserve all of HBM up front for their own pool (a serving engine's KV
// pool), latency-critical decode loops where cudaMalloc/cudaFree would
// synchronize the device, and bindings that hold raw pointers but no allocator.
//
// Every GPU that loads the library holds the array (kStaticScratchBytes) until
// the process exits.  All calls on a device share it and it keeps the last
// call's contents: each call rewrites every partial it reads (and the header)
// before reading it, so nothing needs clearing, but calls whose kernels overlap
// on the GPU (different streams without ordering between them) race on it.
namespace akv {
constexpr int64_t kStaticScratchBytes = 8ll << 20;  // 8 MiB per GPU
static __device__ __align__(256) float g_static_partials[kStaticScratchBytes / sizeof(float)];
}  // namespace akv

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
  // The same plan akv_workspace_bytes sizes, with its own status on failure
  // (unsupported head_dim, invalid geometry, a CUDA query error), as
  // akv_packed_attention would report it.
  akv::Plan pl;
  if (int st = akv::make_plan(batch, q_heads, kv_heads, head_dim, max_blocks, splits, &pl)) return st;
  int64_t need = pl.bytes;
  if (need > akv::kStaticScratchBytes) {  // try exactly `splits` pieces per item, without the finer cut
    if (int st = akv::make_plan(batch, q_heads, kv_heads, head_dim, max_blocks, splits, &pl, false)) return st;
    if (pl.bytes > akv::kStaticScratchBytes) return AKV_ERR_SCRATCH;
    need = akv::kStaticScratchBytes;  // the decode picks the decomposition that fits
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 256) return AKV_ERR_CUDA;
  void *scratch = nullptr;
  {
    // First call on a device: look up the array's device address with that
    // device current.  The address is kept for the life of the process: a
    // cudaDeviceReset on that device unloads this module's copy of the array,
    // after which the kept address is stale and this entry point must not be
    // called on that device again.
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
