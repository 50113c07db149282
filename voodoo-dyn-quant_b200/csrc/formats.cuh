// Bit-exact GGUF block decoders for the candidate formats of the gated
// Linear.  A "unit" is 256 consecutive weights of one row: one super-block for
// the K-quants and IQ4_XS, eight 34-byte blocks for Q8_0.
//
// Decoders read a unit from a 4-byte aligned SHARED-memory slot (units are
// staged there by stage_unit_warp, which realigns 2-byte aligned GGUF blocks
// with funnel shifts), so every field is fetched with 32-bit loads.
// dec8<fmt>(slot, i, y) writes elements 8*i .. 8*i+7 of the unit (i in
// [0, 32)), so one warp decodes a whole unit with one call per lane.
//
// Every multiply/subtract is an explicitly rounded __fmul_rn / __fsub_rn in
// the order of the reference decoders (voodoo_quant/layers.py:62-213,
// voodoo_quant/quants/gpu_dequant.py:460-519; gguf-py 0.19.0 for Q2_K/Q3_K),
// so nothing is contracted into an FMA and the float32 results are
// bit-identical to the reference.  Small integers are converted to float with
// the exact identity float(0x4B000000 | q) - 2^23 = q (q < 2^23): one logic
// op and one add instead of a quarter-rate integer conversion.
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
// 32-bit words of a staged unit slot.
__host__ __device__ inline int unit_words(int fmt) { return (unit_bytes(fmt) + 3) / 4; }

constexpr int kMaxUnitWords = 68;  // Q8_0: 272 bytes

__device__ __forceinline__ float u2f(uint32_t q) {  // exact for q < 2^23
  return __uint_as_float(0x4B000000u | q) - 8388608.0f;
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

__device__ __forceinline__ uint32_t lw(const uint32_t* s, int word) { return s[word]; }

__device__ __forceinline__ uint32_t byte_of(const uint32_t* s, int off) {
  return (s[off >> 2] >> (8 * (off & 3))) & 0xFFu;
}

// Copy the `nbytes` (even) bytes at 2-byte aligned `src` into the 4-byte
// aligned slot `dst`, one output word per lane step.  Reads only aligned
// 32-bit words that contain at least one requested byte (so never a word
// outside the source allocation).
__device__ __forceinline__ void stage_unit_warp(uint32_t* dst, const uint8_t* src, int nbytes, int lane) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(src);
  const uint32_t* s = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;  // 0 or 16
  const int nw = (nbytes + 3) >> 2;
  for (int w = lane; w < nw; w += 32) {
    const uint32_t lo = __ldg(s + w);
    const uint32_t hi = (sh != 0u && 4 * w + 3 <= nbytes) ? __ldg(s + w + 1) : 0u;
    dst[w] = __funnelshift_r(lo, hi, sh);
  }
}

// Two consecutive 32-bit words starting at byte offset `off` (multiple of 4).
__device__ __forceinline__ void ld2(const uint32_t* s, int off, uint32_t& a, uint32_t& b) {
  a = s[off >> 2];
  b = s[(off >> 2) + 1];
}

// ---------------------------------------------------------------- decoders
template <int F>
struct Dec;

template <>
struct Dec<kQ8_0> {
  __device__ __forceinline__ static void run(const uint32_t* s, int i, float (&y)[8]) {
    const int b = i >> 2;
    const int dof = 34 * b;
    const float d = h2f(s[dof >> 2] >> (8 * (dof & 2)));
    const int off = dof + 2 + 8 * (i & 3);
    const int a = off & ~3;
    const uint32_t sh = static_cast<uint32_t>(off & 3) * 8u;
    const uint32_t w0 = s[a >> 2], w1 = s[(a >> 2) + 1];
    const uint32_t w2 = sh ? s[(a >> 2) + 2] : 0u;
    const uint32_t q0 = __funnelshift_r(w0, w1, sh), q1 = __funnelshift_r(w1, w2, sh);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t byte = ((j < 4 ? q0 : q1) >> (8 * (j & 3))) & 0xFFu;
      y[j] = __fmul_rn(u2f(byte ^ 0x80u) - 128.0f, d);
    }
  }
};

__device__ __forceinline__ void k4_scale_min_w(const uint32_t* s, int j, uint32_t& sc, uint32_t& mn) {
  // 12-byte table at byte 4: q[0..11] = bytes 4..15 (words 1..3)
  if (j < 4) {
    sc = byte_of(s, 4 + j) & 63u;
    mn = byte_of(s, 8 + j) & 63u;
  } else {
    const uint32_t hi = byte_of(s, 4 + j + 4);  // q[j+4]
    sc = (hi & 15u) | ((byte_of(s, 4 + j - 4) >> 6) << 4);
    mn = (hi >> 4) | ((byte_of(s, 4 + j) >> 6) << 4);
  }
}

template <>
struct Dec<kQ4_K> {
  __device__ __forceinline__ static void run(const uint32_t* s, int i, float (&y)[8]) {
    const uint32_t w0 = s[0];
    const float d = h2f(w0), dmin = h2f(w0 >> 16);
    const int sb = i >> 2;
    uint32_t sc, mn;
    k4_scale_min_w(s, sb, sc, mn);
    const float dl = __fmul_rn(d, u2f(sc));
    const float ml = __fmul_rn(dmin, u2f(mn));
    uint32_t a, b;
    ld2(s, 16 + 32 * (sb >> 1) + 8 * (i & 3), a, b);
    const uint32_t sh = (sb & 1) * 4;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t q = ((j < 4 ? a : b) >> (8 * (j & 3) + sh)) & 15u;
      y[j] = __fsub_rn(__fmul_rn(dl, u2f(q)), ml);
    }
  }
};

template <>
struct Dec<kQ5_K> {
  __device__ __forceinline__ static void run(const uint32_t* s, int i, float (&y)[8]) {
    const uint32_t w0 = s[0];
    const float d = h2f(w0), dmin = h2f(w0 >> 16);
    const int sb = i >> 2;
    uint32_t sc, mn;
    k4_scale_min_w(s, sb, sc, mn);
    const float dl = __fmul_rn(d, u2f(sc));
    const float ml = __fmul_rn(dmin, u2f(mn));
    const int l0 = 8 * (i & 3);
    uint32_t ha, hb, qa, qb;
    ld2(s, 16 + l0, ha, hb);
    ld2(s, 48 + 32 * (sb >> 1) + l0, qa, qb);
    const uint32_t sh = (sb & 1) * 4;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t bsh = 8 * (j & 3);
      const uint32_t q = (((j < 4 ? qa : qb) >> (bsh + sh)) & 15u) | ((((j < 4 ? ha : hb) >> (bsh + sb)) & 1u) << 4);
      y[j] = __fsub_rn(__fmul_rn(dl, u2f(q)), ml);
    }
  }
};

template <>
struct Dec<kQ6_K> {
  __device__ __forceinline__ static void run(const uint32_t* s, int i, float (&y)[8]) {
    const int h = i >> 4, g = (i >> 2) & 3, l0 = 8 * (i & 3);
    uint32_t la, lb, ha, hb;
    ld2(s, 64 * h + 32 * (g & 1) + l0, la, lb);
    ld2(s, 128 + 32 * h + l0, ha, hb);
    const int so = 192 + 8 * h + (l0 >> 4) + 2 * g;
    const int sc = static_cast<int>(static_cast<int8_t>(byte_of(s, so)));
    const float d = h2f(s[52]);  // byte 208
    const float ds = __fmul_rn(d, u2f(static_cast<uint32_t>(sc + 128)) - 128.0f);
    const uint32_t lsh = (g >> 1) * 4, hsh = 2 * g;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t bsh = 8 * (j & 3);
      const uint32_t q = (((j < 4 ? la : lb) >> (bsh + lsh)) & 15u) | ((((j < 4 ? ha : hb) >> (bsh + hsh)) & 3u) << 4);
      y[j] = __fmul_rn(ds, u2f(q) - 32.0f);
    }
  }
};

template <>
struct Dec<kQ2_K> {
  __device__ __forceinline__ static void run(const uint32_t* s, int i, float (&y)[8]) {
    const int h = i >> 4, sft = (i >> 2) & 3, l0 = 8 * (i & 3);
    const uint32_t scb = byte_of(s, i >> 1);
    const uint32_t wd = s[20];  // bytes 80..83: d, dmin
    const float dl = __fmul_rn(h2f(wd), u2f(scb & 15u));
    const float ml = __fmul_rn(h2f(wd >> 16), u2f(scb >> 4));
    uint32_t a, b;
    ld2(s, 16 + 32 * h + l0, a, b);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t q = ((j < 4 ? a : b) >> (8 * (j & 3) + 2 * sft)) & 3u;
      y[j] = __fsub_rn(__fmul_rn(dl, u2f(q)), ml);
    }
  }
};

template <>
struct Dec<kQ3_K> {
  __device__ __forceinline__ static void run(const uint32_t* s, int i, float (&y)[8]) {
    const int h = i >> 4, sft = (i >> 2) & 3, l0 = 8 * (i & 3), hbit = i >> 2;
    const int j16 = i >> 1;
    const uint32_t lo = (byte_of(s, 96 + (j16 & 7)) >> (4 * (j16 >> 3))) & 15u;
    const uint32_t hi = (byte_of(s, 104 + (j16 & 3)) >> (2 * (j16 >> 2))) & 3u;
    const float d = h2f(s[27]);  // byte 108
    const float dl = __fmul_rn(d, u2f(lo | (hi << 4)) - 32.0f);
    uint32_t ma, mb, qa, qb;
    ld2(s, l0, ma, mb);
    ld2(s, 32 + 32 * h + l0, qa, qb);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t bsh = 8 * (j & 3);
      const uint32_t low = ((j < 4 ? qa : qb) >> (bsh + 2 * sft)) & 3u;
      const uint32_t hb = ((j < 4 ? ma : mb) >> (bsh + hbit)) & 1u;
      y[j] = __fmul_rn(dl, u2f(low + 4u * hb) - 4.0f);  // low - 4 * (1 - hb)
    }
  }
};

// IQ4_NL code book packed as signed bytes (public GGUF constant).
__device__ __forceinline__ int8_t iq4nl(uint32_t idx) {
  constexpr uint32_t k0 = 0xBFAD9881u;  // -127 -104 -83 -65
  constexpr uint32_t k1 = 0xF6EADDCFu;  // -49 -35 -22 -10
  constexpr uint32_t k2 = 0x26190D01u;  // 1 13 25 38
  constexpr uint32_t k3 = 0x71594535u;  // 53 69 89 113
  const uint32_t lo = (idx & 8u) ? k2 : k0;
  const uint32_t hi = (idx & 8u) ? k3 : k1;
  return static_cast<int8_t>(__byte_perm(lo, hi, idx & 7u) & 0xFFu);
}

template <>
struct Dec<kIQ4_XS> {
  __device__ __forceinline__ static void run(const uint32_t* s, int i, float (&y)[8]) {
    const int ib = i >> 2, part = i & 3;
    const uint32_t w0 = s[0];
    const float d = h2f(w0);
    const uint32_t shv = w0 >> 16;
    const uint32_t ls = ((byte_of(s, 4 + (ib >> 1)) >> (4 * (ib & 1))) & 15u) | (((shv >> (2 * ib)) & 3u) << 4);
    const float dl = __fmul_rn(d, u2f(ls) - 32.0f);
    uint32_t a, b;
    ld2(s, 8 + 16 * ib + 8 * (part & 1), a, b);
    const uint32_t nsh = (part >> 1) * 4;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t idx = ((j < 4 ? a : b) >> (8 * (j & 3) + nsh)) & 15u;
      y[j] = __fmul_rn(dl, u2f(static_cast<uint32_t>(iq4nl(idx) + 128)) - 128.0f);
    }
  }
};

// ------------------------------------------ sub-block decoders (mix / gate-grad)
// Chunk<F>::qbytes(slot, c, a, b, qb) decodes elements 32c .. 32c+31 of a unit
// as exact small-integer codes packed one per byte, qb[j] byte i = code of
// element 4j + i plus a per-format bias, together with scale/offset pairs:
//   w[4j+i] = a[h] * (byte_i(qb[j]) + 2^23 - kSub) + b[h],   h = (4j+i) / 16
// (formats with one scale per 32 weights repeat the pair).  A byte becomes
// the float 2^23 + byte with one byte permute (exponent bits 0x4B), so
// subtracting kSub gives the code exactly.  a and b are the same float32
// products the exact decoders form (d*sc, -dmin*m), so a*q + b equals the
// exact decode up to its final rounding.  Chunk<F>::run returns the codes as
// floats.  The mixture and gate-gradient kernels (tolerance-checked) use this
// form: one FMA per weight, with the scale work done once per sub-block.
template <int F>
struct Chunk;

__device__ __forceinline__ void ld8(const uint32_t* s, int off, uint32_t (&w)[8]) {
#pragma unroll
  for (int j = 0; j < 8; ++j) w[j] = s[(off >> 2) + j];
}

// byte i of x as the float 2^23 + byte
__device__ __forceinline__ float magic_byte(uint32_t x, int i) {
  return __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7440u + i));
}

template <int F>
__device__ __forceinline__ void chunk_run(const uint32_t* s, int c, float (&a)[2], float (&b)[2], float (&q)[32]) {
  uint32_t qb[8];
  Chunk<F>::qbytes(s, c, a, b, qb);
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) q[4 * j + i] = magic_byte(qb[j], i) - Chunk<F>::kSub;
}

template <>
struct Chunk<kQ8_0> {
  static constexpr bool kMin = false;
  static constexpr float kSub = 8388736.0f;  // 2^23 + 128: int8 codes stored with the sign bit flipped
  __device__ __forceinline__ static void qbytes(const uint32_t* s, int c, float (&a)[2], float (&b)[2],
                                                uint32_t (&qb)[8]) {
    const int dof = 34 * c;
    a[0] = a[1] = h2f(s[dof >> 2] >> (8 * (dof & 2)));
    b[0] = b[1] = 0.f;
    const int off = dof + 2;
    const int al = off & ~3;
    const uint32_t sh = static_cast<uint32_t>(off & 3) * 8u;
    uint32_t w[9];
#pragma unroll
    for (int j = 0; j < 8; ++j) w[j] = s[(al >> 2) + j];
    w[8] = sh ? s[(al >> 2) + 8] : 0u;
#pragma unroll
    for (int j = 0; j < 8; ++j) qb[j] = __funnelshift_r(w[j], w[j + 1], sh) ^ 0x80808080u;
  }
  __device__ __forceinline__ static void run(const uint32_t* s, int c, float (&a)[2], float (&b)[2], float (&q)[32]) {
    chunk_run<kQ8_0>(s, c, a, b, q);
  }
};

template <>
struct Chunk<kQ4_K> {
  static constexpr bool kMin = true;
  static constexpr float kSub = 8388608.0f;
  __device__ __forceinline__ static void qbytes(const uint32_t* s, int c, float (&a)[2], float (&b)[2],
                                                uint32_t (&qb)[8]) {
    const uint32_t w0 = s[0];
    uint32_t sc, mn;
    k4_scale_min_w(s, c, sc, mn);
    a[0] = a[1] = __fmul_rn(h2f(w0), u2f(sc));
    b[0] = b[1] = -__fmul_rn(h2f(w0 >> 16), u2f(mn));
    uint32_t w[8];
    ld8(s, 16 + 32 * (c >> 1), w);
    const uint32_t sh = (c & 1) * 4;
#pragma unroll
    for (int j = 0; j < 8; ++j) qb[j] = (w[j] >> sh) & 0x0F0F0F0Fu;
  }
  __device__ __forceinline__ static void run(const uint32_t* s, int c, float (&a)[2], float (&b)[2], float (&q)[32]) {
    chunk_run<kQ4_K>(s, c, a, b, q);
  }
};

template <>
struct Chunk<kQ5_K> {
  static constexpr bool kMin = true;
  static constexpr float kSub = 8388608.0f;
  __device__ __forceinline__ static void qbytes(const uint32_t* s, int c, float (&a)[2], float (&b)[2],
                                                uint32_t (&qb)[8]) {
    const uint32_t w0 = s[0];
    uint32_t sc, mn;
    k4_scale_min_w(s, c, sc, mn);
    a[0] = a[1] = __fmul_rn(h2f(w0), u2f(sc));
    b[0] = b[1] = -__fmul_rn(h2f(w0 >> 16), u2f(mn));
    uint32_t w[8], h[8];
    ld8(s, 48 + 32 * (c >> 1), w);
    ld8(s, 16, h);
    const uint32_t sh = (c & 1) * 4;
#pragma unroll
    for (int j = 0; j < 8; ++j) qb[j] = ((w[j] >> sh) & 0x0F0F0F0Fu) | (((h[j] >> c) & 0x01010101u) << 4);
  }
  __device__ __forceinline__ static void run(const uint32_t* s, int c, float (&a)[2], float (&b)[2], float (&q)[32]) {
    chunk_run<kQ5_K>(s, c, a, b, q);
  }
};

template <>
struct Chunk<kQ6_K> {
  static constexpr bool kMin = false;
  static constexpr float kSub = 8388640.0f;  // 2^23 + 32
  __device__ __forceinline__ static void qbytes(const uint32_t* s, int c, float (&a)[2], float (&b)[2],
                                                uint32_t (&qb)[8]) {
    const int h = c >> 2, g = c & 3;
    const float d = h2f(s[52]);
    const int so = 192 + 8 * h + 2 * g;
    const uint32_t sw = s[so >> 2] >> (8 * (so & 3));  // two int8 scales (so is even)
    const int sc0 = static_cast<int>(static_cast<int8_t>(sw & 0xFFu));
    const int sc1 = static_cast<int>(static_cast<int8_t>((sw >> 8) & 0xFFu));
    a[0] = __fmul_rn(d, u2f(static_cast<uint32_t>(sc0 + 128)) - 128.0f);
    a[1] = __fmul_rn(d, u2f(static_cast<uint32_t>(sc1 + 128)) - 128.0f);
    b[0] = b[1] = 0.f;
    uint32_t l[8], hh[8];
    ld8(s, 64 * h + 32 * (g & 1), l);
    ld8(s, 128 + 32 * h, hh);
    const uint32_t lsh = (g >> 1) * 4, hsh = 2 * g;
#pragma unroll
    for (int j = 0; j < 8; ++j) qb[j] = ((l[j] >> lsh) & 0x0F0F0F0Fu) | (((hh[j] >> hsh) & 0x03030303u) << 4);
  }
  __device__ __forceinline__ static void run(const uint32_t* s, int c, float (&a)[2], float (&b)[2], float (&q)[32]) {
    chunk_run<kQ6_K>(s, c, a, b, q);
  }
};

template <>
struct Chunk<kQ2_K> {
  static constexpr bool kMin = true;
  static constexpr float kSub = 8388608.0f;
  __device__ __forceinline__ static void qbytes(const uint32_t* s, int c, float (&a)[2], float (&b)[2],
                                                uint32_t (&qb)[8]) {
    const int h = c >> 2, sft = c & 3;
    const uint32_t sw = s[c >> 1] >> (16 * (c & 1));  // scale bytes 2c, 2c+1
    const uint32_t wd = s[20];
    const float d = h2f(wd), dmin = h2f(wd >> 16);
    a[0] = __fmul_rn(d, u2f(sw & 15u));
    b[0] = -__fmul_rn(dmin, u2f((sw >> 4) & 15u));
    a[1] = __fmul_rn(d, u2f((sw >> 8) & 15u));
    b[1] = -__fmul_rn(dmin, u2f((sw >> 12) & 15u));
    uint32_t w[8];
    ld8(s, 16 + 32 * h, w);
#pragma unroll
    for (int j = 0; j < 8; ++j) qb[j] = (w[j] >> (2 * sft)) & 0x03030303u;
  }
  __device__ __forceinline__ static void run(const uint32_t* s, int c, float (&a)[2], float (&b)[2], float (&q)[32]) {
    chunk_run<kQ2_K>(s, c, a, b, q);
  }
};

template <>
struct Chunk<kQ3_K> {
  static constexpr bool kMin = false;
  static constexpr float kSub = 8388612.0f;  // 2^23 + 4
  __device__ __forceinline__ static void qbytes(const uint32_t* s, int c, float (&a)[2], float (&b)[2],
                                                uint32_t (&qb)[8]) {
    const int h = c >> 2, sft = c & 3;
    const float d = h2f(s[27]);
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const int j16 = 2 * c + t;
      const uint32_t lo = (byte_of(s, 96 + (j16 & 7)) >> (4 * (j16 >> 3))) & 15u;
      const uint32_t hi = (byte_of(s, 104 + (j16 & 3)) >> (2 * (j16 >> 2))) & 3u;
      a[t] = __fmul_rn(d, u2f(lo | (hi << 4)) - 32.0f);
      b[t] = 0.f;
    }
    uint32_t w[8], m[8];
    ld8(s, 32 + 32 * h, w);
    ld8(s, 0, m);
#pragma unroll
    for (int j = 0; j < 8; ++j) qb[j] = ((w[j] >> (2 * sft)) & 0x03030303u) | (((m[j] >> c) & 0x01010101u) << 2);
  }
  __device__ __forceinline__ static void run(const uint32_t* s, int c, float (&a)[2], float (&b)[2], float (&q)[32]) {
    chunk_run<kQ3_K>(s, c, a, b, q);
  }
};

// Four IQ4_NL codebook lookups at once: byte i of the result is
// kvalues[nibble i of the low nibbles of x] + 128 (x holds 4 indices, one per byte).
__device__ __forceinline__ uint32_t iq4nl4(uint32_t x) {
  constexpr uint32_t k0 = 0xBFAD9881u, k1 = 0xF6EADDCFu, k2 = 0x26190D01u, k3 = 0x71594535u;
  const uint32_t i3 = x & 0x07070707u;                                  // low 3 bits per byte
  const uint32_t sel = (i3 | (i3 >> 4)) & 0x00770077u;                  // bytes -> nibbles (pairs)
  const uint32_t sel16 = (sel & 0x77u) | ((sel >> 8) & 0x7700u);        // four 3-bit selectors
  const uint32_t lo = __byte_perm(k0, k1, sel16);
  const uint32_t hi = __byte_perm(k2, k3, sel16);
  const uint32_t m = ((x >> 3) & 0x01010101u) * 0xFFu;                  // bit 3 set -> high half
  return ((hi & m) | (lo & ~m)) ^ 0x80808080u;
}

template <>
struct Chunk<kIQ4_XS> {
  static constexpr bool kMin = false;
  static constexpr float kSub = 8388736.0f;  // 2^23 + 128
  __device__ __forceinline__ static void qbytes(const uint32_t* s, int c, float (&a)[2], float (&b)[2],
                                                uint32_t (&qb)[8]) {
    const uint32_t w0 = s[0];
    const uint32_t ls = ((byte_of(s, 4 + (c >> 1)) >> (4 * (c & 1))) & 15u) | ((((w0 >> 16) >> (2 * c)) & 3u) << 4);
    a[0] = a[1] = __fmul_rn(h2f(w0), u2f(ls) - 32.0f);
    b[0] = b[1] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t w = s[2 + 4 * c + j];  // bytes 8 + 16c + 4j ..: elements 4j.. (low) and 16 + 4j.. (high)
      qb[j] = iq4nl4(w & 0x0F0F0F0Fu);
      qb[4 + j] = iq4nl4((w >> 4) & 0x0F0F0F0Fu);
    }
  }
  __device__ __forceinline__ static void run(const uint32_t* s, int c, float (&a)[2], float (&b)[2], float (&q)[32]) {
    chunk_run<kIQ4_XS>(s, c, a, b, q);
  }
};

// Runtime dispatch (formats are uniform per candidate, so no divergence).
__device__ __forceinline__ bool dec8(int fmt, const uint32_t* slot, int i, float (&y)[8]) {
  switch (fmt) {
    case kQ8_0: Dec<kQ8_0>::run(slot, i, y); return true;
    case kQ2_K: Dec<kQ2_K>::run(slot, i, y); return true;
    case kQ3_K: Dec<kQ3_K>::run(slot, i, y); return true;
    case kQ4_K: Dec<kQ4_K>::run(slot, i, y); return true;
    case kQ5_K: Dec<kQ5_K>::run(slot, i, y); return true;
    case kQ6_K: Dec<kQ6_K>::run(slot, i, y); return true;
    case kIQ4_XS: Dec<kIQ4_XS>::run(slot, i, y); return true;
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
