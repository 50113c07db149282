// Bit-exact GGUF block decoders for the candidate formats of the gated
// Linear.  A "unit" is 256 consecutive weights of one row: one super-block for
// the K-quants and IQ4_XS, eight 34-byte blocks for Q8_0.  dec8(unit, i, y)
// writes elements 8*i .. 8*i+7 of the unit (i in [0, 32)), so one warp decodes
// a whole unit with one call per lane.
//
// Every multiply/subtract is an explicitly rounded __fmul_rn / __fsub_rn in
// the order of the reference decoders (voodoo_quant/layers.py:62-213,
// voodoo_quant/quants/gpu_dequant.py:460-519; gguf-py 0.19.0 for Q2_K/Q3_K),
// so the compiler cannot contract them into FMAs and the float32 results are
// bit-identical to the reference.  All multi-byte fields sit at even offsets,
// so 2-byte alignment of each block is all that is assumed.
#pragma once

#include "common.cuh"

namespace vq {

// ggml type ids (public GGUF enumeration).
enum Format : int {
  kQ8_0 = 8,
  kQ2_K = 10,
  kQ3_K = 11,
  kQ4_K = 12,
  kQ5_K = 13,
  kQ6_K = 14,
  kIQ4_XS = 23,
};

__host__ __device__ inline int unit_bytes(int fmt) {
  switch (fmt) {
    case kQ8_0: return 272;  // 8 x 34
    case kQ2_K: return 84;
    case kQ3_K: return 110;
    case kQ4_K: return 144;
    case kQ5_K: return 176;
    case kQ6_K: return 210;
    case kIQ4_XS: return 136;
    default: return 0;
  }
}

__host__ __device__ inline int block_elems(int fmt) { return fmt == kQ8_0 ? 32 : 256; }
__host__ __device__ inline int block_bytes(int fmt) { return fmt == kQ8_0 ? 34 : unit_bytes(fmt); }

__device__ __forceinline__ float ld_f16(const uint8_t* p) {
  return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(p)));
}

// 6-bit scale/min pair j of the 12-byte Q4_K/Q5_K table (get_scale_min_k4).
__device__ __forceinline__ void k4_scale_min(const uint8_t* q, int j, int& sc, int& mn) {
  if (j < 4) {
    sc = q[j] & 63;
    mn = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 15) | ((q[j - 4] >> 6) << 4);
    mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

__device__ __forceinline__ void dec8_q8_0(const uint8_t* u, int i, float (&y)[8]) {
  const uint8_t* b = u + 34 * (i >> 2);
  const float d = ld_f16(b);
  const int8_t* qs = reinterpret_cast<const int8_t*>(b + 2 + 8 * (i & 3));
#pragma unroll
  for (int j = 0; j < 8; ++j) y[j] = __fmul_rn(static_cast<float>(qs[j]), d);
}

__device__ __forceinline__ void dec8_q4_k(const uint8_t* u, int i, float (&y)[8]) {
  const float d = ld_f16(u), dmin = ld_f16(u + 2);
  const int sb = i >> 2;  // 32-element sub-block
  int sc, mn;
  k4_scale_min(u + 4, sb, sc, mn);
  const float dl = __fmul_rn(d, static_cast<float>(sc));
  const float ml = __fmul_rn(dmin, static_cast<float>(mn));
  const uint8_t* qs = u + 16 + 32 * (sb >> 1) + 8 * (i & 3);
  const int sh = (sb & 1) * 4;
#pragma unroll
  for (int j = 0; j < 8; ++j) y[j] = __fsub_rn(__fmul_rn(dl, static_cast<float>((qs[j] >> sh) & 15)), ml);
}

__device__ __forceinline__ void dec8_q5_k(const uint8_t* u, int i, float (&y)[8]) {
  const float d = ld_f16(u), dmin = ld_f16(u + 2);
  const int sb = i >> 2;
  int sc, mn;
  k4_scale_min(u + 4, sb, sc, mn);
  const float dl = __fmul_rn(d, static_cast<float>(sc));
  const float ml = __fmul_rn(dmin, static_cast<float>(mn));
  const int l0 = 8 * (i & 3);
  const uint8_t* qh = u + 16 + l0;
  const uint8_t* qs = u + 48 + 32 * (sb >> 1) + l0;
  const int sh = (sb & 1) * 4;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int q = ((qs[j] >> sh) & 15) + 16 * ((qh[j] >> sb) & 1);
    y[j] = __fsub_rn(__fmul_rn(dl, static_cast<float>(q)), ml);
  }
}

__device__ __forceinline__ void dec8_q6_k(const uint8_t* u, int i, float (&y)[8]) {
  const int e0 = 8 * i;
  const int h = e0 >> 7, g = (e0 >> 5) & 3, l0 = e0 & 31;
  const uint8_t* ql = u + 64 * h + 32 * (g & 1) + l0;
  const uint8_t* qh = u + 128 + 32 * h + l0;
  const int8_t sc = reinterpret_cast<const int8_t*>(u + 192)[8 * h + (l0 >> 4) + 2 * g];
  const float d = ld_f16(u + 208);
  const float ds = __fmul_rn(d, static_cast<float>(sc));
  const int lsh = (g >> 1) * 4, hsh = 2 * g;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int q = ((ql[j] >> lsh) & 15) | (((qh[j] >> hsh) & 3) << 4);
    y[j] = __fmul_rn(ds, static_cast<float>(q - 32));
  }
}

__device__ __forceinline__ void dec8_q2_k(const uint8_t* u, int i, float (&y)[8]) {
  const int e0 = 8 * i;
  const int h = e0 >> 7, s = (e0 >> 5) & 3, l0 = e0 & 31;
  const int scb = u[e0 >> 4];
  const float d = ld_f16(u + 80), dmin = ld_f16(u + 82);
  const float dl = __fmul_rn(d, static_cast<float>(scb & 15));
  const float ml = __fmul_rn(dmin, static_cast<float>(scb >> 4));
  const uint8_t* qs = u + 16 + 32 * h + l0;
#pragma unroll
  for (int j = 0; j < 8; ++j) y[j] = __fsub_rn(__fmul_rn(dl, static_cast<float>((qs[j] >> (2 * s)) & 3)), ml);
}

__device__ __forceinline__ int q3k_scale(const uint8_t* sc12, int j) {
  const int lo = (sc12[j & 7] >> (4 * (j >> 3))) & 15;
  const int hi = (sc12[8 + (j & 3)] >> (2 * (j >> 2))) & 3;
  return (lo | (hi << 4)) - 32;
}

__device__ __forceinline__ void dec8_q3_k(const uint8_t* u, int i, float (&y)[8]) {
  const int e0 = 8 * i;
  const int h = e0 >> 7, s = (e0 >> 5) & 3, l0 = e0 & 31, hb = e0 >> 5;
  const float d = ld_f16(u + 108);
  const float dl = __fmul_rn(d, static_cast<float>(q3k_scale(u + 96, e0 >> 4)));
  const uint8_t* hm = u + l0;
  const uint8_t* qs = u + 32 + 32 * h + l0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int q = ((qs[j] >> (2 * s)) & 3) - 4 * (((hm[j] >> hb) & 1) ^ 1);
    y[j] = __fmul_rn(dl, static_cast<float>(q));
  }
}

__constant__ float kIQ4NL[16] = {-127.f, -104.f, -83.f, -65.f, -49.f, -35.f, -22.f, -10.f,
                                 1.f,    13.f,   25.f,  38.f,  53.f,  69.f,  89.f,  113.f};

__device__ __forceinline__ void dec8_iq4_xs(const uint8_t* u, int i, float (&y)[8]) {
  const int ib = i >> 2, part = i & 3;  // 32-element sub-block, quarter within it
  const float d = ld_f16(u);
  const int sh = *reinterpret_cast<const unsigned short*>(u + 2);
  const int ls = ((u[4 + (ib >> 1)] >> (4 * (ib & 1))) & 15) | (((sh >> (2 * ib)) & 3) << 4);
  const float dl = __fmul_rn(d, static_cast<float>(ls - 32));
  const uint8_t* qs = u + 8 + 16 * ib + 8 * (part & 1);
  const int nsh = (part >> 1) * 4;
#pragma unroll
  for (int j = 0; j < 8; ++j) y[j] = __fmul_rn(dl, kIQ4NL[(qs[j] >> nsh) & 15]);
}

// Decode elements 8*i..8*i+7 of a unit.  Returns false for an unknown format.
__device__ __forceinline__ bool dec8(int fmt, const uint8_t* unit, int i, float (&y)[8]) {
  switch (fmt) {
    case kQ8_0: dec8_q8_0(unit, i, y); return true;
    case kQ2_K: dec8_q2_k(unit, i, y); return true;
    case kQ3_K: dec8_q3_k(unit, i, y); return true;
    case kQ4_K: dec8_q4_k(unit, i, y); return true;
    case kQ5_K: dec8_q5_k(unit, i, y); return true;
    case kQ6_K: dec8_q6_k(unit, i, y); return true;
    case kIQ4_XS: dec8_iq4_xs(unit, i, y); return true;
    default:
#pragma unroll
      for (int j = 0; j < 8; ++j) y[j] = 0.f;
      return false;
  }
}

constexpr int kMaxCandidates = 8;

// A candidate set passed by value to kernels.
struct CandSet {
  const uint8_t* ptr[kMaxCandidates];
  int fmt[kMaxCandidates];
  int ubytes[kMaxCandidates];
  int K;
};

}  // namespace vq
