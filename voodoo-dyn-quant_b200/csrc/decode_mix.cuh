// Candidate decode and mixture kernels (HBM-bandwidth bound).
//
//   dequant: one packed candidate -> float32 [rows, padded_cols]   (bit-exact)
//   mix    : W_mix[o, i] = sum_k p_k * W_k[o, i] -> bf16 [rows, ld_out],
//            columns >= cols (the zero padding of in_features) written as 0.
//
// A CTA owns a run of kUnitsPerCta consecutive 256-weight units of the
// row-major block stream.  Because every candidate stores its blocks row-major
// and contiguously, that run is one contiguous byte span per candidate; the
// CTA stages the K spans in shared memory with 16-byte loads (each span starts
// on a 16-byte boundary since kUnitsPerCta * unit_bytes is a multiple of 16),
// then each warp decodes one unit per pass, lane i producing weights
// 8i..8i+7 for every candidate and writing 16-byte vectors.
#pragma once

#include "formats.cuh"

namespace vq {

constexpr int kUnitsPerCta = 16;
constexpr int kDecodeThreads = 256;

__device__ __forceinline__ void stage_span(uint8_t* dst, const uint8_t* src, int nbytes) {
  const bool vec = ((reinterpret_cast<uintptr_t>(src) | static_cast<uintptr_t>(nbytes)) & 15u) == 0;
  if (vec) {
    const uint4* s = reinterpret_cast<const uint4*>(src);
    uint4* d = reinterpret_cast<uint4*>(dst);
    for (int i = threadIdx.x; i < (nbytes >> 4); i += blockDim.x) d[i] = __ldg(s + i);
  } else {
    for (int i = threadIdx.x; i < nbytes; i += blockDim.x) dst[i] = src[i];
  }
}

// kMix = false: K must be 1, OutT = float; exact decode written flat
//               (element e of the block stream to out[e]); total_elems need
//               only be a multiple of the block size (Q8_0: 32).
// kMix = true : OutT = __nv_bfloat16, fp32 mixture rounded once to bf16, at
//               out[row * ld_out + col]; rows are whole units (padded cols
//               a multiple of 256).
template <bool kMix, typename OutT>
__global__ void __launch_bounds__(kDecodeThreads) decode_units_kernel(CandSet cs, const float* __restrict__ probs,
                                                                      long long total_elems, int units_per_row,
                                                                      long long cols, OutT* __restrict__ out,
                                                                      long long ld_out, int* err) {
  extern __shared__ __align__(16) uint8_t stage[];
  const long long total_units = (total_elems + 255) / 256;
  const long long u0 = static_cast<long long>(blockIdx.x) * kUnitsPerCta;
  const int nunits = static_cast<int>(min(static_cast<long long>(kUnitsPerCta), total_units - u0));

  int off[kMaxCandidates];
  int o = 0;
  for (int k = 0; k < cs.K; ++k) {
    off[k] = o;
    const long long span_end =
        min((u0 + nunits) * cs.ubytes[k], total_elems / block_elems(cs.fmt[k]) * block_bytes(cs.fmt[k]));
    stage_span(stage + o, cs.ptr[k] + u0 * cs.ubytes[k], static_cast<int>(span_end - u0 * cs.ubytes[k]));
    o += kUnitsPerCta * cs.ubytes[k];
  }
  float p[kMaxCandidates];
  if (kMix) {
    for (int k = 0; k < cs.K; ++k) p[k] = probs[k];
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int lu = warp; lu < nunits; lu += kDecodeThreads / 32) {
    const long long u = u0 + lu;
    const long long row = u / units_per_row;
    const long long col = (u - row * units_per_row) * 256 + 8 * lane;
    float acc[8];
    if (kMix) {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    }
    bool ok = true;
    for (int k = 0; k < cs.K; ++k) {
      float y[8];
      ok &= dec8(cs.fmt[k], stage + off[k] + lu * cs.ubytes[k], lane, y);
      if (kMix) {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = fmaf(p[k], y[j], acc[j]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = y[j];
      }
    }
    if (!ok && lane == 0) report_error(err, kDevBadFormat, 0);
    if (kMix) {
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

inline int decode_smem_bytes(const CandSet& cs) {
  int s = 0;
  for (int k = 0; k < cs.K; ++k) s += kUnitsPerCta * cs.ubytes[k];
  return s;
}

}  // namespace vq
