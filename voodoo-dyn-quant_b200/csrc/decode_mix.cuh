// Candidate decode and mixture kernels (HBM-bandwidth bound).
//
//   dequant: one packed candidate -> float32, element e of the block stream
//            to out[e] (bit-exact, reference operation order)
//   mix    : W_mix[o, i] = sum_k p_k * W_k[o, i] -> bf16 [rows, ld_out],
//            columns >= cols (the zero padding of in_features) written as 0.
//
// A CTA owns kUnitsPerCta consecutive 256-weight units of the row-major block
// stream.  It first stages every candidate's units into word-aligned
// shared-memory slots: thread t copies words (t % 16) + 16j of unit t / 16,
// so every thread has several independent aligned 32-bit loads in flight
// (2-byte aligned GGUF blocks are realigned with funnel shifts).  Then each
// warp decodes one unit per pass, lane i producing weights 8i..8i+7 for every
// candidate and writing 16-byte vectors.
#pragma once

#include "formats.cuh"

namespace vq {

constexpr int kUnitsPerCta = 16;
constexpr int kDecodeThreads = 256;
constexpr int kDecodeWarps = kDecodeThreads / 32;

inline int decode_smem_bytes(const CandSet& cs) {
  int s = 0;
  for (int k = 0; k < cs.K; ++k) s += kUnitsPerCta * unit_words(cs.fmt[k]) * 4;
  return s;
}

// Stage units [u0, u0 + nunits) of one candidate (stream of `stream_bytes`
// bytes) into slots of `uw` words.  Thread layout: 16 threads per unit.
__device__ __forceinline__ void stage_units_block(uint32_t* dst, const uint8_t* base, long long u0, int nunits,
                                                  int ub, int uw, long long stream_bytes) {
  const int lu = threadIdx.x >> 4;
  const int wl = threadIdx.x & 15;
  if (lu >= nunits) return;
  const long long start = (u0 + lu) * ub;
  const int n = static_cast<int>(min(static_cast<long long>(ub), stream_bytes - start));
  const uintptr_t a = reinterpret_cast<uintptr_t>(base + start);
  const uint32_t* s = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;
  const int nw = (n + 3) >> 2;
  uint32_t lo[5], hi[5];
#pragma unroll
  for (int j = 0; j < 5; ++j) {
    const int w = wl + 16 * j;
    lo[j] = w < nw ? __ldg(s + w) : 0u;
    hi[j] = (w < nw && sh != 0u && 4 * w + 3 <= n) ? __ldg(s + w + 1) : 0u;
  }
#pragma unroll
  for (int j = 0; j < 5; ++j) {
    const int w = wl + 16 * j;
    if (w < nw) dst[lu * uw + w] = __funnelshift_r(lo[j], hi[j], sh);
  }
}

template <int F>
__device__ __forceinline__ void mix_accum(const uint32_t* slot, int lane, float pk, float (&acc)[8], float& cst) {
  float a, b, q[8];
  Aff<F>::run(slot, lane, a, b, q);
  const float pa = pk * a;
  cst = fmaf(pk, b, cst);
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = fmaf(pa, q[j], acc[j]);
}

// kMix = false: K == 1, OutT = float, flat output (total_elems need only be a
//               multiple of the block size; Q8_0 tails are partial units).
// kMix = true : OutT = __nv_bfloat16, out[row * ld_out + col], whole units.
template <bool kMix, typename OutT>
__global__ void __launch_bounds__(kDecodeThreads) decode_units_kernel(CandSet cs, const float* __restrict__ probs,
                                                                      long long total_elems, int units_per_row,
                                                                      long long cols, OutT* __restrict__ out,
                                                                      long long ld_out, int* err) {
  extern __shared__ __align__(16) uint32_t stage[];
  const long long total_units = (total_elems + 255) / 256;
  const long long u0 = static_cast<long long>(blockIdx.x) * kUnitsPerCta;
  const int nunits = static_cast<int>(min(static_cast<long long>(kUnitsPerCta), total_units - u0));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  int o = 0;
  for (int k = 0; k < cs.K; ++k) {
    const int ub = cs.ubytes[k], uw = unit_words(cs.fmt[k]);
    const long long stream_bytes = total_elems / block_elems(cs.fmt[k]) * block_bytes(cs.fmt[k]);
    stage_units_block(stage + o, cs.ptr[k], u0, nunits, ub, uw, stream_bytes);
    o += kUnitsPerCta * uw;
  }
  __syncthreads();

  for (int lu = warp; lu < nunits; lu += kDecodeWarps) {
    const long long u = u0 + lu;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    bool ok = true;
    if (kMix) {
      float cst = 0.f;
      int so = 0;
      for (int k = 0; k < cs.K; ++k) {
        const int uw = unit_words(cs.fmt[k]);
        const uint32_t* slot = stage + so + lu * uw;
        const float pk = probs[k];
        switch (cs.fmt[k]) {
          case kQ8_0: mix_accum<kQ8_0>(slot, lane, pk, acc, cst); break;
          case kQ2_K: mix_accum<kQ2_K>(slot, lane, pk, acc, cst); break;
          case kQ3_K: mix_accum<kQ3_K>(slot, lane, pk, acc, cst); break;
          case kQ4_K: mix_accum<kQ4_K>(slot, lane, pk, acc, cst); break;
          case kQ5_K: mix_accum<kQ5_K>(slot, lane, pk, acc, cst); break;
          case kQ6_K: mix_accum<kQ6_K>(slot, lane, pk, acc, cst); break;
          case kIQ4_XS: mix_accum<kIQ4_XS>(slot, lane, pk, acc, cst); break;
          default: ok = false;
        }
        so += kUnitsPerCta * uw;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += cst;
    } else {
      float y[8];
      ok = dec8(cs.fmt[0], stage + lu * unit_words(cs.fmt[0]), lane, y);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = y[j];
    }
    if (!ok && lane == 0) report_error(err, kDevBadFormat, 0);
    if (kMix) {
      const long long row = u / units_per_row;
      const long long col = (u - row * units_per_row) * 256 + 8 * lane;
      OutT* dst = out + row * ld_out + col;
      if (col + 8 <= cols && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
        __align__(16) __nv_bfloat162 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
        *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(v);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const long long c = col + j;
          if (c < ld_out) dst[j] = __float2bfloat16_rn(c < cols ? acc[j] : 0.f);
        }
      }
    } else {
      const long long e = u * 256 + 8 * lane;
      if (e >= total_elems) continue;
      OutT* dst = out + e;
      if ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
        reinterpret_cast<float4*>(dst)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        reinterpret_cast<float4*>(dst)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) dst[j] = acc[j];
      }
    }
  }
}

}  // namespace vq
