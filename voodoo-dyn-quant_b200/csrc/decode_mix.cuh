// Candidate decode and mixture kernels (HBM-bandwidth bound).
//
//   dequant_units_kernel: one packed candidate -> float32, element e of the
//       block stream to out[e], in the reference's exact operation order
//       (bit-exact).  One warp per 256-weight unit, lane i -> weights 8i..8i+7.
//   mix_units_kernel: W_mix[o, i] = sum_k p_k * W_k[o, i] -> bf16
//       [rows, ld_out]; columns >= cols (the zero padding of in_features)
//       are written as 0.  One thread per 32-weight sub-block: the sub-block's
//       scales are decoded once, then one FMA per weight and candidate.
//
// Both stage a CTA's run of consecutive units into word-aligned shared-memory
// slots first (several independent aligned 32-bit loads in flight per thread;
// 2-byte aligned GGUF blocks are realigned with funnel shifts).
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

template <int F>
__device__ __forceinline__ void mix_chunk(const uint32_t* slot, int c, float pk, float (&acc)[32], float (&cst)[2]) {
  float a[2], b[2], q[32];
  Chunk<F>::run(slot, c, a, b, q);
  const float pa0 = pk * a[0], pa1 = pk * a[1];
  if (Chunk<F>::kMin) {
    cst[0] = fmaf(pk, b[0], cst[0]);
    cst[1] = fmaf(pk, b[1], cst[1]);
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) acc[j] = fmaf(j < 16 ? pa0 : pa1, q[j], acc[j]);
}

// rows * units_per_row units in total (whole units: padded cols % 256 == 0).
__global__ void __launch_bounds__(kDecodeThreads) mix_units_kernel(CandSet cs, const float* __restrict__ probs,
                                                                   long long total_units, int units_per_row,
                                                                   int cols, __nv_bfloat16* __restrict__ out,
                                                                   long long ld_out, int* err) {
  extern __shared__ __align__(16) uint32_t stage[];
  const long long u0 = static_cast<long long>(blockIdx.x) * kMixUnits;
  const int nunits = static_cast<int>(min(static_cast<long long>(kMixUnits), total_units - u0));
  int o = 0;
  for (int k = 0; k < cs.K; ++k) {
    const int uw = unit_words(cs.fmt[k]);
    stage_units<8, 9>(stage + o, cs.ptr[k], u0, nunits, cs.ubytes[k], uw, total_units * cs.ubytes[k]);
    o += kMixUnits * uw;
  }
  __syncthreads();

  const int lu = threadIdx.x >> 3, c = threadIdx.x & 7;
  if (lu >= nunits) return;
  float acc[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) acc[j] = 0.f;
  float cst[2] = {0.f, 0.f};
  bool ok = true;
  int so = 0;
  for (int k = 0; k < cs.K; ++k) {
    const int uw = unit_words(cs.fmt[k]);
    const uint32_t* slot = stage + so + lu * uw;
    const float pk = __ldg(probs + k);
    switch (cs.fmt[k]) {
      case kQ8_0: mix_chunk<kQ8_0>(slot, c, pk, acc, cst); break;
      case kQ2_K: mix_chunk<kQ2_K>(slot, c, pk, acc, cst); break;
      case kQ3_K: mix_chunk<kQ3_K>(slot, c, pk, acc, cst); break;
      case kQ4_K: mix_chunk<kQ4_K>(slot, c, pk, acc, cst); break;
      case kQ5_K: mix_chunk<kQ5_K>(slot, c, pk, acc, cst); break;
      case kQ6_K: mix_chunk<kQ6_K>(slot, c, pk, acc, cst); break;
      case kIQ4_XS: mix_chunk<kIQ4_XS>(slot, c, pk, acc, cst); break;
      default: ok = false;
    }
    so += kMixUnits * uw;
  }
  if (!ok) report_error(err, kDevBadFormat, 1);
  const long long u = u0 + lu;
  const long long row = u / units_per_row;
  const int col = static_cast<int>(u - row * units_per_row) * 256 + 32 * c;
  __nv_bfloat16* dst = out + row * ld_out + col;
  if (col + 32 <= cols && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      __align__(16) __nv_bfloat162 h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int e = 8 * v + 2 * j;
        h[j] = __floats2bfloat162_rn(acc[e] + cst[e >> 4], acc[e + 1] + cst[(e + 1) >> 4]);
      }
      reinterpret_cast<uint4*>(dst)[v] = *reinterpret_cast<const uint4*>(h);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const long long cc = col + j;
      if (cc < ld_out) dst[j] = __float2bfloat16_rn(cc < cols ? acc[j] + cst[j >> 4] : 0.f);
    }
  }
}

}  // namespace vq
