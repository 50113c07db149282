// Candidate decode and mixture kernels (HBM-bandwidth bound).
//
//   dequant_units_kernel: one packed candidate -> float32, element e of the
//       block stream to out[e], in the reference's exact operation order
//       (bit-exact).  One warp per 256-weight unit, lane i -> weights 8i..8i+7.
//   mix_units_kernel: W_mix[o, i] = sum_k p_k * W_k[o, i] -> bf16
//       [rows, ld_out]; columns >= cols (the zero padding of in_features)
//       are written as 0.  One thread per 32-weight sub-block: the sub-block's
//       scales are decoded once, then one packed FMA per two weights and
//       candidate.
//
// The dequant kernel stages a CTA's run of consecutive units into
// word-aligned shared-memory slots with aligned 32-bit loads (2-byte aligned
// GGUF blocks realigned with funnel shifts); the mix kernel copies each
// candidate's contiguous span of a block of units with one bulk copy and
// reads the fields of units that start inside a word through funnel shifts.
#pragma once

#include "formats.cuh"

namespace vq {

constexpr int kDecodeThreads = 256;
constexpr int kDecodeWarps = kDecodeThreads / 32;
constexpr int kDequantUnits = 16;  // units per CTA, dequant kernel
constexpr int kMixUnits = 32;      // units per CTA, mix kernel (8 sub-blocks each)

inline int stage_smem_bytes(const CandSet& cs, int units) {
  int s = 0;
  for (int k = 0; k < cs.K; ++k) s += units * unit_words(cs.fmt[k]) * 4;
  return s;
}

// Stage units [u0, u0 + nunits) of one candidate (`stream_bytes` long) into
// slots of `uw` words, kTPU threads per unit (kTPU * kWPT >= 68 words).
template <int kTPU, int kWPT>
__device__ __forceinline__ void stage_units(uint32_t* dst, const uint8_t* base, long long u0, int nunits, int ub,
                                            int uw, long long stream_bytes) {
  const int lu = threadIdx.x / kTPU;
  const int wl = threadIdx.x % kTPU;
  if (lu >= nunits) return;
  const long long start = (u0 + lu) * ub;
  const int n = static_cast<int>(min(static_cast<long long>(ub), stream_bytes - start));
  const uintptr_t a = reinterpret_cast<uintptr_t>(base + start);
  const uint32_t* s = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;
  const int nw = (n + 3) >> 2;
  uint32_t lo[kWPT], hi[kWPT];
#pragma unroll
  for (int j = 0; j < kWPT; ++j) {
    const int w = wl + kTPU * j;
    lo[j] = w < nw ? __ldg(s + w) : 0u;
    hi[j] = (w < nw && sh != 0u && 4 * w + 3 <= n) ? __ldg(s + w + 1) : 0u;
  }
#pragma unroll
  for (int j = 0; j < kWPT; ++j) {
    const int w = wl + kTPU * j;
    if (w < nw) dst[lu * uw + w] = __funnelshift_r(lo[j], hi[j], sh);
  }
}

// Exact decode of one candidate; total_elems need only be a multiple of the
// block size (Q8_0 tails are partial units).
__global__ void __launch_bounds__(kDecodeThreads) dequant_units_kernel(CandSet cs, long long total_elems,
                                                                       float* __restrict__ out, int* err) {
  extern __shared__ __align__(16) uint32_t stage[];
  const long long total_units = (total_elems + 255) / 256;
  const long long u0 = static_cast<long long>(blockIdx.x) * kDequantUnits;
  const int nunits = static_cast<int>(min(static_cast<long long>(kDequantUnits), total_units - u0));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int uw = unit_words(cs.fmt[0]);
  stage_units<16, 5>(stage, cs.ptr[0], u0, nunits, cs.ubytes[0], uw,
                     total_elems / block_elems(cs.fmt[0]) * block_bytes(cs.fmt[0]));
  __syncthreads();
  for (int lu = warp; lu < nunits; lu += kDecodeWarps) {
    float y[8];
    const bool ok = dec8(cs.fmt[0], stage + lu * uw, lane, y);
    if (!ok && lane == 0) report_error(err, kDevBadFormat, 0);
    const long long e = (u0 + lu) * 256 + 8 * lane;
    if (e >= total_elems) continue;
    float* dst = out + e;
    if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
      reinterpret_cast<float4*>(dst)[0] = make_float4(y[0], y[1], y[2], y[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(y[4], y[5], y[6], y[7]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) dst[j] = y[j];
    }
  }
}

// ---------------------------------------------------------------- mixture
// One mix CTA owns blocks of kMixUnits consecutive units and walks them with
// a stride of the grid (persistent).  Per block and candidate, one thread
// copies the contiguous span of the block's units into a shared-memory
// region with a single bulk copy (cp.async.bulk, completion counted on the
// stage's mbarrier); kMixStages stages keep the next blocks' copies in
// flight while the current one is mixed.  Units keep their byte layout in
// shared memory: a unit whose size is not a multiple of 4 (Q3_K, Q6_K) or
// whose stream base is not 16-byte aligned starts inside a word, and every
// field is read as the two aligned words that hold it, joined by one funnel
// shift that also applies the field's own bit shift.
constexpr int kMixStages = 2;

// Bytes of one candidate's region in a stage: the 16-byte aligned span of
// kMixUnits units plus 32 bytes, so that a field read at a unit's end never
// leaves the region.
__host__ __device__ inline int mix_region_bytes(int ub) { return ((kMixUnits * ub + 15) & ~15) + 32 + 16; }
inline int mix_stage_bytes(const CandSet& cs) {
  int s = 0;
  for (int k = 0; k < cs.K; ++k) s += mix_region_bytes(cs.ubytes[k]);
  return s;
}

// A unit in shared memory: `s` is the word holding its first byte, which is
// byte `delta` (0..3) of that word.
struct URef {
  const uint32_t* s;
  int delta;
  uint32_t sh;  // 8 * delta
  // unit bytes [4 i, 4 i + 4) shifted right by `extra` bits (extra < 8)
  __device__ __forceinline__ uint32_t wq(int i, int extra = 0) const {
    return __funnelshift_r(s[i], s[i + 1], sh + extra);
  }
  // the 32 bits at any unit byte `off`
  __device__ __forceinline__ uint32_t w(int off) const {
    const int o = off + delta;
    return __funnelshift_r(s[o >> 2], s[(o >> 2) + 1], 8 * (o & 3));
  }
  __device__ __forceinline__ uint32_t b16(int off) const { return w(off) & 0xFFFFu; }
  __device__ __forceinline__ uint32_t b8(int off) const { return w(off) & 0xFFu; }
};

// Scale and min of K-quant sub-block j from the 12-byte table at unit byte 4.
__device__ __forceinline__ void k4_scale_min_u(const URef& u, int j, uint32_t& sc, uint32_t& mn) {
  if (j < 4) {
    sc = u.b8(4 + j) & 63u;
    mn = u.b8(8 + j) & 63u;
  } else {
    const uint32_t hi = u.b8(8 + j);  // q[j + 4]
    sc = (hi & 15u) | ((u.b8(j) >> 6) << 4);
    mn = (hi >> 4) | ((u.b8(4 + j) >> 6) << 4);
  }
}

// Sub-block c (32 weights) of a unit as w = a[h] * q + b[h] (h = half of the
// sub-block), with the codes q + kSub - 2^23 one per byte of qb.  The same
// products, in the same order, as Chunk<F> (and so as the exact decoders up
// to the last rounding).
template <int F>
struct MixChunk;

template <>
struct MixChunk<kQ8_0> {
  static constexpr bool kMin = false;
  static constexpr float kSub = 8388736.0f;  // 2^23 + 128: int8 codes stored with the sign bit flipped
  __device__ __forceinline__ static void get(const URef& u, int c, float (&a)[2], float (&b)[2], uint32_t (&qb)[8]) {
    a[0] = a[1] = h2f(u.b16(34 * c));
    b[0] = b[1] = 0.f;
    const int o0 = 34 * c + 2 + u.delta;  // the block's codes
    const uint32_t* q = u.s + (o0 >> 2);
    const uint32_t shq = 8u * static_cast<uint32_t>(o0 & 3);
#pragma unroll
    for (int j = 0; j < 8; ++j) qb[j] = __funnelshift_r(q[j], q[j + 1], shq) ^ 0x80808080u;
  }
};

template <>
struct MixChunk<kQ4_K> {
  static constexpr bool kMin = true;
  static constexpr float kSub = 8388608.0f;
  __device__ __forceinline__ static void get(const URef& u, int c, float (&a)[2], float (&b)[2], uint32_t (&qb)[8]) {
    const uint32_t w0 = u.wq(0);
    uint32_t sc, mn;
    k4_scale_min_u(u, c, sc, mn);
    a[0] = a[1] = __fmul_rn(h2f(w0), u2f(sc));
    b[0] = b[1] = -__fmul_rn(h2f(w0 >> 16), u2f(mn));
#pragma unroll
    for (int j = 0; j < 8; ++j) qb[j] = u.wq(4 + 8 * (c >> 1) + j, 4 * (c & 1)) & 0x0F0F0F0Fu;
  }
};

template <>
struct MixChunk<kQ5_K> {
  static constexpr bool kMin = true;
  static constexpr float kSub = 8388608.0f;
  __device__ __forceinline__ static void get(const URef& u, int c, float (&a)[2], float (&b)[2], uint32_t (&qb)[8]) {
    const uint32_t w0 = u.wq(0);
    uint32_t sc, mn;
    k4_scale_min_u(u, c, sc, mn);
    a[0] = a[1] = __fmul_rn(h2f(w0), u2f(sc));
    b[0] = b[1] = -__fmul_rn(h2f(w0 >> 16), u2f(mn));
#pragma unroll
    for (int j = 0; j < 8; ++j)
      qb[j] = (u.wq(12 + 8 * (c >> 1) + j, 4 * (c & 1)) & 0x0F0F0F0Fu) | ((u.wq(4 + j, c) & 0x01010101u) << 4);
  }
};

template <>
struct MixChunk<kQ6_K> {
  static constexpr bool kMin = false;
  static constexpr float kSub = 8388640.0f;  // 2^23 + 32
  __device__ __forceinline__ static void get(const URef& u, int c, float (&a)[2], float (&b)[2], uint32_t (&qb)[8]) {
    const int h = c >> 2, g = c & 3;
    const float d = h2f(u.b16(208));
    const uint32_t sw = u.b16(192 + 8 * h + 2 * g);  // two int8 scales
    const int sc0 = static_cast<int>(static_cast<int8_t>(sw & 0xFFu));
    const int sc1 = static_cast<int>(static_cast<int8_t>((sw >> 8) & 0xFFu));
    a[0] = __fmul_rn(d, u2f(static_cast<uint32_t>(sc0 + 128)) - 128.0f);
    a[1] = __fmul_rn(d, u2f(static_cast<uint32_t>(sc1 + 128)) - 128.0f);
    b[0] = b[1] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      qb[j] = (u.wq(16 * h + 8 * (g & 1) + j, 4 * (g >> 1)) & 0x0F0F0F0Fu) |
              ((u.wq(32 + 8 * h + j, 2 * g) & 0x03030303u) << 4);
  }
};

template <>
struct MixChunk<kQ2_K> {
  static constexpr bool kMin = true;
  static constexpr float kSub = 8388608.0f;
  __device__ __forceinline__ static void get(const URef& u, int c, float (&a)[2], float (&b)[2], uint32_t (&qb)[8]) {
    const int h = c >> 2, sft = c & 3;
    const uint32_t sw = u.b16(2 * c);  // scale bytes 2c, 2c+1
    const uint32_t wd = u.wq(20);
    const float d = h2f(wd), dmin = h2f(wd >> 16);
    a[0] = __fmul_rn(d, u2f(sw & 15u));
    b[0] = -__fmul_rn(dmin, u2f((sw >> 4) & 15u));
    a[1] = __fmul_rn(d, u2f((sw >> 8) & 15u));
    b[1] = -__fmul_rn(dmin, u2f((sw >> 12) & 15u));
#pragma unroll
    for (int j = 0; j < 8; ++j) qb[j] = u.wq(4 + 8 * h + j, 2 * sft) & 0x03030303u;
  }
};

template <>
struct MixChunk<kQ3_K> {
  static constexpr bool kMin = false;
  static constexpr float kSub = 8388612.0f;  // 2^23 + 4
  __device__ __forceinline__ static void get(const URef& u, int c, float (&a)[2], float (&b)[2], uint32_t (&qb)[8]) {
    const int h = c >> 2, sft = c & 3;
    const float d = h2f(u.b16(108));
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int j16 = 2 * c + t;
      const uint32_t lo = (u.b8(96 + (j16 & 7)) >> (4 * (j16 >> 3))) & 15u;
      const uint32_t hi = (u.b8(104 + (j16 & 3)) >> (2 * (j16 >> 2))) & 3u;
      a[t] = __fmul_rn(d, u2f(lo | (hi << 4)) - 32.0f);
      b[t] = 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      qb[j] = (u.wq(8 + 8 * h + j, 2 * sft) & 0x03030303u) | ((u.wq(j, c) & 0x01010101u) << 2);
  }
};

template <>
struct MixChunk<kIQ4_XS> {
  static constexpr bool kMin = false;
  static constexpr float kSub = 8388736.0f;  // 2^23 + 128
  __device__ __forceinline__ static void get(const URef& u, int c, float (&a)[2], float (&b)[2], uint32_t (&qb)[8]) {
    const uint32_t w0 = u.wq(0);
    const uint32_t ls = ((u.b8(4 + (c >> 1)) >> (4 * (c & 1))) & 15u) | ((((w0 >> 16) >> (2 * c)) & 3u) << 4);
    a[0] = a[1] = __fmul_rn(h2f(w0), u2f(ls) - 32.0f);
    b[0] = b[1] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t w = u.wq(2 + 4 * c + j);  // elements 4j.. (low nibbles) and 16 + 4j.. (high)
      qb[j] = iq4nl4(w & 0x0F0F0F0Fu);
      qb[4 + j] = iq4nl4((w >> 4) & 0x0F0F0F0Fu);
    }
  }
};

// acc[j] holds elements 2j, 2j+1; w = (p_k a[h]) * q + p_k b[h], the b part
// kept per half in cst.
template <int F>
__device__ __forceinline__ void mix_chunk(const URef& u, int c, float pk, float2 (&acc)[16], float (&cst)[2]) {
  float a[2], b[2];
  uint32_t qb[8];
  MixChunk<F>::get(u, c, a, b, qb);
  const float2 pa[2] = {make_float2(pk * a[0], pk * a[0]), make_float2(pk * a[1], pk * a[1])};
  const float2 nsub = make_float2(-MixChunk<F>::kSub, -MixChunk<F>::kSub);
  if (MixChunk<F>::kMin) {
    cst[0] = fmaf(pk, b[0], cst[0]);
    cst[1] = fmaf(pk, b[1], cst[1]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 q01 = __fadd2_rn(make_float2(magic_byte(qb[j], 0), magic_byte(qb[j], 1)), nsub);
    const float2 q23 = __fadd2_rn(make_float2(magic_byte(qb[j], 2), magic_byte(qb[j], 3)), nsub);
    acc[2 * j] = __ffma2_rn(pa[j >> 2], q01, acc[2 * j]);
    acc[2 * j + 1] = __ffma2_rn(pa[j >> 2], q23, acc[2 * j + 1]);
  }
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
               : "memory");
}

// Issue the bulk copies of block `blk` of every candidate into stage buffer
// `buf`, completion on `bar` (one thread).
__device__ __forceinline__ void mix_issue(const CandSet& cs, uint8_t* buf, uint32_t bar, long long blk,
                                          long long total_units) {
  const long long u0 = blk * kMixUnits;
  const int nunits = static_cast<int>(min(static_cast<long long>(kMixUnits), total_units - u0));
  // the 16-byte aligned span of candidate k's units [u0, u0 + nunits)
  auto span = [&](int k, uintptr_t& a0) -> uint32_t {
    const int ub = cs.ubytes[k];
    const uintptr_t st = reinterpret_cast<uintptr_t>(cs.ptr[k]) + static_cast<uintptr_t>(u0) * ub;
    a0 = st & ~uintptr_t(15);
    return static_cast<uint32_t>(((st + static_cast<uintptr_t>(nunits) * ub + 15) & ~uintptr_t(15)) - a0);
  };
  uint32_t total = 0;
  for (int k = 0; k < cs.K; ++k) {
    uintptr_t a0;
    total += span(k, a0);
  }
  mbar_arrive_expect_tx(bar, total);
  int off = 0;
  for (int k = 0; k < cs.K; ++k) {
    uintptr_t a0;
    const uint32_t n = span(k, a0);
    bulk_g2s(smem_u32(buf + off), reinterpret_cast<const void*>(a0), n, bar);
    off += mix_region_bytes(cs.ubytes[k]);
  }
}

// W_mix[o, i] = sum_k p_k W_k[o, i] -> bf16 [rows, ld_out] for rows *
// units_per_row whole units; columns >= cols (the zero padding of
// in_features) are written as 0.  Thread (lu, c) of a block mixes sub-block
// c (32 weights) of unit lu over every candidate.
#ifndef VQ_MIX_MIN_BLOCKS
#define VQ_MIX_MIN_BLOCKS 3  // resident CTAs per SM the register budget is sized for
#endif
__global__ void __launch_bounds__(kDecodeThreads, VQ_MIX_MIN_BLOCKS)
    mix_units_kernel(CandSet cs, const float* __restrict__ probs, long long total_units, int units_per_row, int cols,
                     __nv_bfloat16* __restrict__ out, long long ld_out, int stage_bytes, int* err) {
  extern __shared__ __align__(128) uint8_t msmem[];
  __shared__ __align__(8) uint64_t bars[kMixStages];
  __shared__ float pk_s[kMaxCandidates];
  __shared__ int abort_flag;
  const long long nblocks = (total_units + kMixUnits - 1) / kMixUnits;
  const int tid = threadIdx.x;
  const int lu = tid >> 3, c = tid & 7;
  if (tid == 0) {
    for (int s = 0; s < kMixStages; ++s) mbar_init(smem_u32(&bars[s]), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (tid < cs.K) pk_s[tid] = __ldg(probs + tid);
  __syncthreads();
  if (tid == 0) {
    for (int s = 0; s < kMixStages; ++s) {
      const long long b = blockIdx.x + static_cast<long long>(s) * gridDim.x;
      if (b < nblocks) mix_issue(cs, msmem + s * stage_bytes, smem_u32(&bars[s]), b, total_units);
    }
  }
  bool fmt_ok = true;
  int it = 0;
  for (long long blk = blockIdx.x; blk < nblocks; blk += gridDim.x, ++it) {
    const int st = it % kMixStages;
    const uint32_t parity = static_cast<uint32_t>((it / kMixStages) & 1);
    const bool ok = mbar_wait(smem_u32(&bars[st]), parity, &abort_flag);
    if (!__syncthreads_and(ok)) {
      if (tid == 0) report_error(err, kDevWaitTimeout, 20);
      break;
    }
    const uint8_t* buf = msmem + st * stage_bytes;
    const long long u0 = blk * kMixUnits;
    const int nunits = static_cast<int>(min(static_cast<long long>(kMixUnits), total_units - u0));
    if (lu < nunits) {
      float2 acc[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) acc[j] = make_float2(0.f, 0.f);
      float cst[2] = {0.f, 0.f};
      int off = 0;
      for (int k = 0; k < cs.K; ++k) {
        const int ub = cs.ubytes[k];
        const int rel = static_cast<int>((reinterpret_cast<uintptr_t>(cs.ptr[k]) +
                                          static_cast<uintptr_t>(u0) * ub) & 15u) + lu * ub;
        const URef u{reinterpret_cast<const uint32_t*>(buf + off + (rel & ~3)), rel & 3,
                     8u * static_cast<uint32_t>(rel & 3)};
        const float pk = pk_s[k];
        switch (cs.fmt[k]) {
          case kQ8_0: mix_chunk<kQ8_0>(u, c, pk, acc, cst); break;
          case kQ2_K: mix_chunk<kQ2_K>(u, c, pk, acc, cst); break;
          case kQ3_K: mix_chunk<kQ3_K>(u, c, pk, acc, cst); break;
          case kQ4_K: mix_chunk<kQ4_K>(u, c, pk, acc, cst); break;
          case kQ5_K: mix_chunk<kQ5_K>(u, c, pk, acc, cst); break;
          case kQ6_K: mix_chunk<kQ6_K>(u, c, pk, acc, cst); break;
          case kIQ4_XS: mix_chunk<kIQ4_XS>(u, c, pk, acc, cst); break;
          default: fmt_ok = false;
        }
        off += mix_region_bytes(ub);
      }
      const long long uu = u0 + lu;
      const long long row = uu / units_per_row;
      const int col = static_cast<int>(uu - row * units_per_row) * 256 + 32 * c;
      __nv_bfloat16* dst = out + row * ld_out + col;
      if (col + 32 <= cols && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          __align__(16) __nv_bfloat162 hv[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 e = acc[4 * v + j];
            const float cs0 = cst[(8 * v + 2 * j) >> 4];
            hv[j] = __floats2bfloat162_rn(e.x + cs0, e.y + cs0);
          }
          reinterpret_cast<uint4*>(dst)[v] = *reinterpret_cast<const uint4*>(hv);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const long long c0 = col + 2 * j;
          const float cs0 = cst[(2 * j) >> 4];
          if (c0 < ld_out) dst[2 * j] = __float2bfloat16_rn(c0 < cols ? acc[j].x + cs0 : 0.f);
          if (c0 + 1 < ld_out) dst[2 * j + 1] = __float2bfloat16_rn(c0 + 1 < cols ? acc[j].y + cs0 : 0.f);
        }
      }
    }
    __syncthreads();  // every thread is done with this stage: refill it
    if (tid == 0) {
      const long long nb = blk + static_cast<long long>(kMixStages) * gridDim.x;
      if (nb < nblocks) mix_issue(cs, msmem + st * stage_bytes, smem_u32(&bars[st]), nb, total_units);
    }
  }
  if (!fmt_ok) report_error(err, kDevBadFormat, 1);
}

}  // namespace vq
