// Chunked-vocab fused distillation loss (HBM-bandwidth bound).
//
// Per token row with student logits s[0..V), teacher logits t[0..V), target y
// and distillation temperature T (voodoo_quant/training/trainer.py:797-821,
// :2567-2575, vocab-parallel form :915-1066):
//
//   ce  = lse(s) - s[y]                               (0 when y < 0: ignored)
//   kl  = T^2 * sum_v p_v (log p_v - log q_v),  p = softmax(t/T), q = softmax(s/T)
//       = T^2 * ( A / Zt - lse(t/T) + lse(s/T) ),  A = sum_v e^{t_v/T - mt} (t_v - s_v)/T
//   d/ds_v = ce_w * (softmax(s)_v - [v == y]) + kl_w * T * (q_v - p_v)
//
// Pass 1 streams s and t once with online (max, sum-exp) pairs for s, s/T and
// t/T plus the running A; pass 2 re-reads the row (L2-resident: one CTA per
// SM holds at most a couple of rows in flight) to write the gradient.  Under
// vocab-parallel TP, pass 1 runs on each rank's shard (loss_stats_kernel),
// the per-row partial statistics are combined across ranks
// (loss_combine_kernel) and pass 2 runs on the shard (loss_grad_kernel).
#pragma once

#include "common.cuh"

namespace vq {
namespace loss {

constexpr int THREADS = 1024;
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kStats = 8;  // m1 z1 mq zq mt zt A sy  (sy = NaN when y is not in this shard)

struct MZ {  // running max and sum of exp(x - max)
  float m, z;
};

// e^x as one MUFU.EX2 (flush-to-zero: results below 2^-126 become 0, which
// only drops probabilities that are already negligible).
__device__ __forceinline__ float ex(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * kLog2e));
  return y;
}

__device__ __forceinline__ MZ mz_merge(MZ a, MZ b) {
  if (b.m == -INFINITY) return a;
  if (a.m == -INFINITY) return b;
  const float m = fmaxf(a.m, b.m);
  return {m, a.z * ex(a.m - m) + b.z * ex(b.m - m)};
}

struct RowAcc {
  MZ s1, sq, t;
  float a;  // sum e^{t/T - t.m} (t - s) / T
};

__device__ __forceinline__ void acc_init(RowAcc& r) {
  r.s1 = {-INFINITY, 0.f};
  r.sq = {-INFINITY, 0.f};
  r.t = {-INFINITY, 0.f};
  r.a = 0.f;
}

// Fold 8 values into a running (max, sum-exp): one rescale per 8 values.
__device__ __forceinline__ void mz_add8(MZ& r, const float (&x)[8]) {
  float mx = x[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) mx = fmaxf(mx, x[j]);
  const float m = fmaxf(r.m, mx);
  if (m == -INFINITY) return;
  float z = (r.m == -INFINITY) ? 0.f : r.z * ex(r.m - m);
#pragma unroll
  for (int j = 0; j < 8; ++j) z += ex(x[j] - m);
  r.m = m;
  r.z = z;
}

template <bool kT1>
__device__ __forceinline__ void acc_add8(RowAcc& r, const float (&s)[8], const float (&t)[8], float inv_t) {
  mz_add8(r.s1, s);
  float tt[8], d[8];
  if (!kT1) {
    float sq[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) sq[j] = s[j] * inv_t;
    mz_add8(r.sq, sq);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    tt[j] = kT1 ? t[j] : t[j] * inv_t;
    d[j] = kT1 ? (t[j] - s[j]) : (t[j] - s[j]) * inv_t;
  }
  float mx = tt[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) mx = fmaxf(mx, tt[j]);
  const float m = fmaxf(r.t.m, mx);
  if (m == -INFINITY) return;
  const float sc = (r.t.m == -INFINITY) ? 0.f : ex(r.t.m - m);
  float z = r.t.z * sc, a = r.a * sc;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float e = ex(tt[j] - m);
    z += e;
    a = fmaf(e, d[j], a);
  }
  r.t.m = m;
  r.t.z = z;
  r.a = a;
}

__device__ __forceinline__ RowAcc acc_merge(RowAcc x, RowAcc y) {
  RowAcc o;
  o.s1 = mz_merge(x.s1, y.s1);
  o.sq = mz_merge(x.sq, y.sq);
  const float m = fmaxf(x.t.m, y.t.m);
  const float fx = (x.t.m == -INFINITY) ? 0.f : ex(x.t.m - m);
  const float fy = (y.t.m == -INFINITY) ? 0.f : ex(y.t.m - m);
  o.t = {m, x.t.z * fx + y.t.z * fy};
  o.a = x.a * fx + y.a * fy;
  return o;
}

__device__ __forceinline__ RowAcc acc_shfl(const RowAcc& r, int o) {
  RowAcc x;
  x.s1.m = __shfl_xor_sync(0xffffffffu, r.s1.m, o);
  x.s1.z = __shfl_xor_sync(0xffffffffu, r.s1.z, o);
  x.sq.m = __shfl_xor_sync(0xffffffffu, r.sq.m, o);
  x.sq.z = __shfl_xor_sync(0xffffffffu, r.sq.z, o);
  x.t.m = __shfl_xor_sync(0xffffffffu, r.t.m, o);
  x.t.z = __shfl_xor_sync(0xffffffffu, r.t.z, o);
  x.a = __shfl_xor_sync(0xffffffffu, r.a, o);
  return x;
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 x = __bfloat1622float2(h[j]);
    f[2 * j] = x.x;
    f[2 * j + 1] = x.y;
  }
}

// Pass 1 over one row, reduced across the CTA (result valid in every thread).
// Vector path: 8 bf16 per 16-byte load, two vectors of s and t in flight per
// thread; the scalar tail (and unaligned rows) folds 8 at a time with -inf pad.
template <bool kT1>
__device__ RowAcc row_stats(const __nv_bfloat16* s, const __nv_bfloat16* t, int V, float inv_t, bool vec,
                            RowAcc* sh) {
  RowAcc r;
  acc_init(r);
  int done = 0;
  if (vec) {
    const int nv = V >> 3;
    const uint4* s4 = reinterpret_cast<const uint4*>(s);
    const uint4* t4 = reinterpret_cast<const uint4*>(t);
    int i = threadIdx.x;
    for (; i + THREADS < nv; i += 2 * THREADS) {
      const uint4 a0 = __ldg(s4 + i), b0 = __ldg(t4 + i);
      const uint4 a1 = __ldg(s4 + i + THREADS), b1 = __ldg(t4 + i + THREADS);
      float fs[8], ft[8];
      unpack8(a0, fs);
      unpack8(b0, ft);
      acc_add8<kT1>(r, fs, ft, inv_t);
      unpack8(a1, fs);
      unpack8(b1, ft);
      acc_add8<kT1>(r, fs, ft, inv_t);
    }
    if (i < nv) {
      float fs[8], ft[8];
      unpack8(__ldg(s4 + i), fs);
      unpack8(__ldg(t4 + i), ft);
      acc_add8<kT1>(r, fs, ft, inv_t);
    }
    done = nv << 3;
  }
  for (int i0 = done + 8 * threadIdx.x; i0 < V; i0 += 8 * THREADS) {
    float fs[8], ft[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const bool ok = i0 + j < V;
      fs[j] = ok ? __bfloat162float(s[i0 + j]) : -INFINITY;
      ft[j] = ok ? __bfloat162float(t[i0 + j]) : -INFINITY;
    }
    // padded lanes: s = t = -inf contribute e^-inf = 0; their (t - s) term is
    // multiplied by that 0 only if finite, so zero it explicitly
    RowAcc before = r;
    acc_add8<kT1>(r, fs, ft, inv_t);
    if (i0 + 8 > V) {
      // recompute A without the padded lanes (NaN from -inf - -inf)
      float a = 0.f;
      const float m = r.t.m;
      for (int j = 0; j < 8 && i0 + j < V; ++j) {
        const float tt = kT1 ? ft[j] : ft[j] * inv_t;
        const float d = kT1 ? (ft[j] - fs[j]) : (ft[j] - fs[j]) * inv_t;
        a = fmaf(ex(tt - m), d, a);
      }
      r.a = (before.t.m == -INFINITY ? 0.f : before.a * ex(before.t.m - m)) + a;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) r = acc_merge(r, acc_shfl(r, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sh[warp] = r;
  __syncthreads();
  if (warp == 0) {
    RowAcc x;
    if (lane < THREADS / 32) x = sh[lane]; else acc_init(x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = acc_merge(x, acc_shfl(x, o));
    if (lane == 0) sh[THREADS / 32] = x;
  }
  __syncthreads();
  RowAcc out = sh[THREADS / 32];
  __syncthreads();
  if (kT1) out.sq = out.s1;
  return out;
}

// Pass 2: gradient for one row (or one shard of a row).
template <bool kT1>
__device__ void row_grad(const __nv_bfloat16* s, const __nv_bfloat16* t, int V, long long y_local, float inv_t,
                         float lse1, float lseq, float lset, float ce_w, float klw_t, __nv_bfloat16* g, bool vec) {
  // d = ce_w * (e^{s - lse1} - [v==y]) + klw_t * (e^{s/T - lseq} - e^{t/T - lset})
  const float c1 = kT1 ? (ce_w + klw_t) : ce_w;
  auto grad1 = [&](float fs, float ft) {
    float d = c1 * ex(fs - lse1);
    if (!kT1) d = fmaf(klw_t, ex(fs * inv_t - lseq), d);
    d = fmaf(-klw_t, ex((kT1 ? ft : ft * inv_t) - lset), d);
    return d;
  };
  int done = 0;
  const int ybase = y_local >= 0 ? static_cast<int>(y_local >> 3) : -1;
  const int yoff = static_cast<int>(y_local & 7);
  if (vec) {
    const int nv = V >> 3;
    const uint4* s4 = reinterpret_cast<const uint4*>(s);
    const uint4* t4 = reinterpret_cast<const uint4*>(t);
    uint4* g4 = reinterpret_cast<uint4*>(g);
    for (int i = threadIdx.x; i < nv; i += THREADS) {
      float fs[8], ft[8];
      unpack8(__ldg(s4 + i), fs);
      unpack8(__ldg(t4 + i), ft);
      float d[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) d[j] = grad1(fs[j], ft[j]);
      if (i == ybase) {  // the target falls in this vector
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j == yoff) d[j] -= ce_w;
      }
      __align__(16) __nv_bfloat162 o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = __floats2bfloat162_rn(d[2 * j], d[2 * j + 1]);
      g4[i] = *reinterpret_cast<const uint4*>(o);
    }
    done = nv << 3;
  }
  for (int i = done + threadIdx.x; i < V; i += THREADS) {
    float d = grad1(__bfloat162float(s[i]), __bfloat162float(t[i]));
    if (i == y_local) d -= ce_w;
    g[i] = __float2bfloat16_rn(d);
  }
}

__device__ __forceinline__ float lse_of(MZ a) { return a.m + logf(a.z); }

// Single-GPU fused kernel: pass 1 + row loss + pass 2, persistent over rows.
template <bool kT1>
__global__ void __launch_bounds__(THREADS) loss_fused_kernel(
    const __nv_bfloat16* __restrict__ S, long long lds, const __nv_bfloat16* __restrict__ Tl, long long ldt,
    const long long* __restrict__ targets, int rows, int V, float temp, float ce_w, float kl_w,
    float* __restrict__ row_ce, float* __restrict__ row_kl, __nv_bfloat16* __restrict__ G, long long ldg,
    int vec) {
  __shared__ RowAcc sh[THREADS / 32 + 1];
  const float inv_t = 1.f / temp;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const __nv_bfloat16* s = S + static_cast<long long>(r) * lds;
    const __nv_bfloat16* t = Tl + static_cast<long long>(r) * ldt;
    const RowAcc a = row_stats<kT1>(s, t, V, inv_t, vec != 0, sh);
    const float lse1 = lse_of(a.s1), lseq = lse_of(a.sq), lset = lse_of(a.t);
    const long long y = targets[r];
    const bool valid = y >= 0 && y < V;
    if (threadIdx.x == 0) {
      row_ce[r] = valid ? lse1 - __bfloat162float(s[y]) : 0.f;
      row_kl[r] = temp * temp * (a.a / a.t.z - lset + lseq);
    }
    if (G != nullptr)
      row_grad<kT1>(s, t, V, valid ? y : -1, inv_t, lse1, lseq, lset, valid ? ce_w : 0.f, kl_w * temp,
                    G + static_cast<long long>(r) * ldg, vec != 0);
  }
}

// TP pass 1: per-row partial statistics of this rank's vocab shard.
template <bool kT1>
__global__ void __launch_bounds__(THREADS) loss_stats_kernel(const __nv_bfloat16* __restrict__ S, long long lds,
                                                             const __nv_bfloat16* __restrict__ Tl, long long ldt,
                                                             const long long* __restrict__ targets,
                                                             long long vocab_start, int rows, int V, float temp,
                                                             float* __restrict__ stats, int vec) {
  __shared__ RowAcc sh[THREADS / 32 + 1];
  const float inv_t = 1.f / temp;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const __nv_bfloat16* s = S + static_cast<long long>(r) * lds;
    const __nv_bfloat16* t = Tl + static_cast<long long>(r) * ldt;
    const RowAcc a = row_stats<kT1>(s, t, V, inv_t, vec != 0, sh);
    if (threadIdx.x == 0) {
      const long long y = targets[r] - vocab_start;
      float* o = stats + static_cast<long long>(r) * kStats;
      o[0] = a.s1.m; o[1] = a.s1.z; o[2] = a.sq.m; o[3] = a.sq.z;
      o[4] = a.t.m;  o[5] = a.t.z;  o[6] = a.a;
      o[7] = (targets[r] >= 0 && y >= 0 && y < V) ? __bfloat162float(s[y]) : __int_as_float(0x7fc00000);
    }
  }
}

// Combine [R, rows, kStats] partials (rank order) into per-row lse triples
// (lse1, lseq, lset, unused) and the row losses.
__global__ void loss_combine_kernel(const float* __restrict__ stats, int R, int rows, float temp,
                                    float* __restrict__ row_lse, float* __restrict__ row_ce,
                                    float* __restrict__ row_kl) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  RowAcc acc;
  acc_init(acc);
  float sy = __int_as_float(0x7fc00000);
  for (int k = 0; k < R; ++k) {
    const float* o = stats + (static_cast<long long>(k) * rows + r) * kStats;
    RowAcc x;
    x.s1 = {o[0], o[1]};
    x.sq = {o[2], o[3]};
    x.t = {o[4], o[5]};
    x.a = o[6];
    acc = acc_merge(acc, x);
    if (!isnan(o[7])) sy = o[7];
  }
  const float lse1 = lse_of(acc.s1), lseq = lse_of(acc.sq), lset = lse_of(acc.t);
  row_lse[4 * r + 0] = lse1;
  row_lse[4 * r + 1] = lseq;
  row_lse[4 * r + 2] = lset;
  row_lse[4 * r + 3] = isnan(sy) ? 0.f : 1.f;
  row_ce[r] = isnan(sy) ? 0.f : lse1 - sy;
  row_kl[r] = temp * temp * (acc.a / acc.t.z - lset + lseq);
}

// TP pass 2: gradient of this rank's shard given the global per-row lse.
template <bool kT1>
__global__ void __launch_bounds__(THREADS) loss_grad_kernel(const __nv_bfloat16* __restrict__ S, long long lds,
                                                            const __nv_bfloat16* __restrict__ Tl, long long ldt,
                                                            const long long* __restrict__ targets,
                                                            long long vocab_start, int rows, int V, float temp,
                                                            const float* __restrict__ row_lse, float ce_w,
                                                            float kl_w, __nv_bfloat16* __restrict__ G,
                                                            long long ldg, int vec) {
  const float inv_t = 1.f / temp;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const long long y = targets[r] - vocab_start;
    const bool mine = targets[r] >= 0 && y >= 0 && y < V;
    row_grad<kT1>(S + static_cast<long long>(r) * lds, Tl + static_cast<long long>(r) * ldt, V, mine ? y : -1,
                  inv_t, row_lse[4 * r], row_lse[4 * r + 1], row_lse[4 * r + 2],
                  targets[r] >= 0 ? ce_w : 0.f, kl_w * temp, G + static_cast<long long>(r) * ldg, vec != 0);
  }
}

}  // namespace loss
}  // namespace vq
