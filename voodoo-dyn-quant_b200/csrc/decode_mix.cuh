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
// candidate's contiguous span with 16-byte cp.async and realigns only the
// units that are not word aligned.
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
// Shared-memory layout of one mix CTA (kMixUnits consecutive units): per
// candidate a raw region holding the 16-byte aligned span of its units'
// contiguous bytes (copied with cp.async), and, for a candidate whose units
// are not all 4-byte aligned there (2-byte multiple unit sizes, or a base
// pointer that is not 4-byte aligned), a region of word-aligned unit slots.
__host__ __device__ inline int mix_raw_bytes(int ub) { return (kMixUnits * ub + 32 + 15) & ~15; }
__host__ __device__ inline bool mix_realign(const CandSet& cs, int k) {
  return ((cs.ubytes[k] & 3) != 0) || ((reinterpret_cast<uintptr_t>(cs.ptr[k]) & 3u) != 0);
}
inline int mix_smem_bytes(const CandSet& cs) {
  int s = 0;
  for (int k = 0; k < cs.K; ++k) {
    s += mix_raw_bytes(cs.ubytes[k]);
    if (mix_realign(cs, k)) s += kMixUnits * unit_words(cs.fmt[k]) * 4;
  }
  return s;
}

// Per-candidate addressing of one block in the mix CTA's buffer (bytes):
// unit lu of the candidate is at slot + lu * stride, its raw bytes at
// raw + lu * ub.
struct MixCand {
  int fmt, slot, stride, raw, ub;
  float p;
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}

// acc2[j] holds elements 2j, 2j+1; w = (p_k a[h]) * q + p_k b[h] with the
// b part kept per half in cst.
template <int F>
__device__ __forceinline__ void mix_chunk(const uint32_t* slot, int c, float pk, uint64_t (&acc2)[16], float (&cst)[2]) {
  float a[2], b[2];
  uint32_t qb[8];
  Chunk<F>::qbytes(slot, c, a, b, qb);
  const uint64_t pa[2] = {f2pack(pk * a[0], pk * a[0]), f2pack(pk * a[1], pk * a[1])};
  const uint64_t nsub = f2pack(-Chunk<F>::kSub, -Chunk<F>::kSub);
  if (Chunk<F>::kMin) {
    cst[0] = fmaf(pk, b[0], cst[0]);
    cst[1] = fmaf(pk, b[1], cst[1]);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint64_t q01 = f2add(f2pack(magic_byte(qb[j], 0), magic_byte(qb[j], 1)), nsub);
    const uint64_t q23 = f2add(f2pack(magic_byte(qb[j], 2), magic_byte(qb[j], 3)), nsub);
    acc2[2 * j] = f2fma(pa[j >> 2], q01, acc2[2 * j]);
    acc2[2 * j + 1] = f2fma(pa[j >> 2], q23, acc2[2 * j + 1]);
  }
}

// Issue the cp.async copies of block `blk` (kMixUnits units) of every
// candidate into the raw regions of the buffer at `buf` (layout as above).
__device__ __forceinline__ void mix_issue(const CandSet& cs, uint8_t* buf, long long blk, long long total_units) {
  const long long u0 = blk * kMixUnits;
  const int nunits = static_cast<int>(min(static_cast<long long>(kMixUnits), total_units - u0));
  int off = 0;
  for (int k = 0; k < cs.K; ++k) {
    const int ub = cs.ubytes[k];
    const uintptr_t st = reinterpret_cast<uintptr_t>(cs.ptr[k]) + static_cast<uintptr_t>(u0) * ub;
    const uintptr_t a0 = st & ~uintptr_t(15);
    const int n16 = static_cast<int>((((st + static_cast<uintptr_t>(nunits) * ub + 15) & ~uintptr_t(15)) - a0) >> 4);
    for (int i = threadIdx.x; i < n16; i += kDecodeThreads)
      cp_async16(buf + off + 16 * i, reinterpret_cast<const void*>(a0 + 16 * static_cast<uintptr_t>(i)));
    off += mix_raw_bytes(ub);
    if (mix_realign(cs, k)) off += kMixUnits * unit_words(cs.fmt[k]) * 4;
  }
}

// rows * units_per_row units in total (whole units: padded cols % 256 == 0),
// in blocks of kMixUnits.  Persistent CTAs walk the blocks with a stride of
// the grid; with two buffers the copies of the next block are in flight while
// the current one is decoded.  One thread per 32-weight sub-block: its scales
// are decoded once per candidate, then one packed FMA per two weights.
#ifndef VQ_MIX_MIN_BLOCKS
#define VQ_MIX_MIN_BLOCKS 4  // resident CTAs per SM the register budget is sized for
#endif
__global__ void __launch_bounds__(kDecodeThreads, VQ_MIX_MIN_BLOCKS)
    mix_units_kernel(CandSet cs, const float* __restrict__ probs, long long total_units, int units_per_row, int cols,
                     __nv_bfloat16* __restrict__ out, long long ld_out, int buf_bytes, int nbuf, int* err) {
  extern __shared__ __align__(16) uint8_t msmem[];
  __shared__ MixCand meta[kMaxCandidates];
  const long long nblocks = (total_units + kMixUnits - 1) / kMixUnits;
  const int tid = threadIdx.x;
  const int lu = tid >> 3, c = tid & 7;
  bool ok = true;

  long long blk = blockIdx.x;
  if (blk < nblocks) mix_issue(cs, msmem, blk, total_units);
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int it = 0; blk < nblocks; blk += gridDim.x, ++it) {
    uint8_t* buf = msmem + (nbuf == 2 ? (it & 1) * buf_bytes : 0);
    if (nbuf == 2) {
      const long long nb = blk + gridDim.x;
      if (nb < nblocks) mix_issue(cs, msmem + ((it + 1) & 1) * buf_bytes, nb, total_units);
      asm volatile("cp.async.commit_group;\ncp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();

    const long long u0 = blk * kMixUnits;
    const int nunits = static_cast<int>(min(static_cast<long long>(kMixUnits), total_units - u0));
    // per-candidate unit addressing for this block, computed once
    if (tid == 0) {
      int off = 0;
      for (int k = 0; k < cs.K; ++k) {
        const int ub = cs.ubytes[k];
        const int delta = static_cast<int>((reinterpret_cast<uintptr_t>(cs.ptr[k]) + static_cast<uintptr_t>(u0) * ub) & 15u);
        MixCand m;
        m.fmt = cs.fmt[k];
        m.p = __ldg(probs + k);
        m.raw = off + delta;
        m.ub = ub;
        off += mix_raw_bytes(ub);
        if (mix_realign(cs, k)) {
          m.slot = off;
          m.stride = 4 * ((ub + 3) >> 2);
          off += kMixUnits * m.stride;
        } else {
          m.slot = m.raw;
          m.stride = ub;
        }
        meta[k] = m;
      }
    }
    __syncthreads();
    // word-align the units of candidates that need it (8 threads per unit)
    bool any = false;
    for (int k = 0; k < cs.K; ++k) {
      const MixCand m = meta[k];
      if (m.slot == m.raw) continue;
      any = true;
      if (lu < nunits) {
        const int uw = m.stride >> 2;
        const uint32_t* raw = reinterpret_cast<const uint32_t*>(buf + (m.raw & ~15));
        uint32_t* dst = reinterpret_cast<uint32_t*>(buf + m.slot) + lu * uw;
        const int b0 = (m.raw & 15) + lu * m.ub;
        const uint32_t sh = static_cast<uint32_t>(b0 & 3) * 8u;
        for (int w = c; w < uw; w += 8) {
          const int i = (b0 >> 2) + w;
          dst[w] = __funnelshift_r(raw[i], raw[i + 1], sh);
        }
      }
    }
    if (any) __syncthreads();

    if (lu < nunits) {
      uint64_t acc2[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) acc2[j] = 0ull;
      float cst[2] = {0.f, 0.f};
      for (int k = 0; k < cs.K; ++k) {
        const MixCand m = meta[k];
        const uint32_t* slot = reinterpret_cast<const uint32_t*>(buf + m.slot + lu * m.stride);
        switch (m.fmt) {
          case kQ8_0: mix_chunk<kQ8_0>(slot, c, m.p, acc2, cst); break;
          case kQ2_K: mix_chunk<kQ2_K>(slot, c, m.p, acc2, cst); break;
          case kQ3_K: mix_chunk<kQ3_K>(slot, c, m.p, acc2, cst); break;
          case kQ4_K: mix_chunk<kQ4_K>(slot, c, m.p, acc2, cst); break;
          case kQ5_K: mix_chunk<kQ5_K>(slot, c, m.p, acc2, cst); break;
          case kQ6_K: mix_chunk<kQ6_K>(slot, c, m.p, acc2, cst); break;
          case kIQ4_XS: mix_chunk<kIQ4_XS>(slot, c, m.p, acc2, cst); break;
          default: ok = false;
        }
      }
      float acc[32];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float2 v = f2unpack(acc2[j]);
        acc[2 * j] = v.x;
        acc[2 * j + 1] = v.y;
      }
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
    __syncthreads();  // this buffer is refilled two blocks from now (one, single-buffered)
    if (nbuf != 2) {
      const long long nb = blk + gridDim.x;
      if (nb < nblocks) mix_issue(cs, msmem, nb, total_units);
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (!ok) report_error(err, kDevBadFormat, 1);
}

}  // namespace vq
