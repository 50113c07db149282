// Fused elementwise kernels of the Llama decoder block around the gated
// Linears of the distillation step (HBM-bandwidth bound, one pass each):
//
//   RMSNorm   y = w * bf16(x * rsqrt(mean(x^2) + eps))            (fwd)
//             dx = r * (g - n * mean(g * n)),  g = dy * w, n = x * r (bwd)
//   RoPE      out[:h] = x[:h] * cos[:h] - x[h:] * sin[:h]
//             out[h:] = x[h:] * cos[h:] + x[:h] * sin[h:]   (h = D/2, fwd)
//             dx[:h]  = g[:h] * cos[:h] + g[h:] * sin[h:]
//             dx[h:]  = g[h:] * cos[h:] - g[:h] * sin[:h]         (bwd)
//   SwiGLU    y = silu(a) * u,  da = dy * u * silu'(a),  du = dy * silu(a)
//
// The reference runs these as separate torch ops of the Hugging Face Llama
// block (LlamaRMSNorm.forward: fp32 cast, pow, mean, rsqrt, two multiplies;
// apply_rotary_pos_emb: rotate_half's neg + cat, two multiplies and an add
// on the transposed q/k views; act_fn(gate) * up), i.e. 3-6 HBM passes each
// plus their backward passes.  Here each is one pass of 16-byte vectors in
// fp32 registers with a single rounding to bf16.
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

namespace vq {
namespace blocks {

constexpr int kNormThreads = 128;
constexpr int kRopeThreads = 128;
constexpr int kEltThreads = 256;

struct V8 {  // 8 bf16 values widened to fp32
  float v[8];
};

__device__ __forceinline__ V8 widen8(const uint4& raw) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
  V8 r;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    r.v[2 * i] = f.x;
    r.v[2 * i + 1] = f.y;
  }
  return r;
}

__device__ __forceinline__ V8 load8(const __nv_bfloat16* p) { return widen8(*reinterpret_cast<const uint4*>(p)); }

__device__ __forceinline__ void store8(__nv_bfloat16* p, const V8& r) {
  uint4 raw;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(r.v[2 * i], r.v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = raw;
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Sum over the CTA (kNormThreads threads); every thread gets the total.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read by a previous call
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) t += red[w];
  return t;
}

// One CTA per row (grid-stride); a thread keeps VPT vectors of 8 in registers.
// kAdd: the input is the residual sum h = bf16(x + res) (a bf16 add, as the
// model's `residual + hidden_states`), written to h; the norm is taken of h.
template <int VPT, bool kAdd = false>
__global__ void __launch_bounds__(kNormThreads) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                                  const __nv_bfloat16* __restrict__ w, float eps,
                                                                  int rows, int D, __nv_bfloat16* __restrict__ y,
                                                                  long long ldy, float* __restrict__ rstd,
                                                                  const __nv_bfloat16* __restrict__ res = nullptr,
                                                                  long long ldres = 0,
                                                                  __nv_bfloat16* __restrict__ h = nullptr,
                                                                  long long ldh = 0) {
  __shared__ float red[kNormThreads / 32];
  const int nvec = D >> 3;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const __nv_bfloat16* xr = x + static_cast<long long>(row) * ldx;
    V8 v[VPT];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = threadIdx.x + j * kNormThreads;
      if (c < nvec) {
        v[j] = load8(xr + 8 * c);
        if (kAdd) {
          const V8 rv = load8(res + static_cast<long long>(row) * ldres + 8 * c);
#pragma unroll
          for (int i = 0; i < 8; ++i) v[j].v[i] = bf16_round(v[j].v[i] + rv.v[i]);
          store8(h + static_cast<long long>(row) * ldh + 8 * c, v[j]);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) ss = fmaf(v[j].v[i], v[j].v[i], ss);
      }
    }
    const float r = rsqrtf(block_sum(ss, red) / static_cast<float>(D) + eps);
    if (threadIdx.x == 0 && rstd != nullptr) rstd[row] = r;
    __nv_bfloat16* yr = y + static_cast<long long>(row) * ldy;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = threadIdx.x + j * kNormThreads;
      if (c < nvec) {
        const V8 wv = load8(w + 8 * c);
        V8 o;
#pragma unroll
        for (int i = 0; i < 8; ++i) o.v[i] = wv.v[i] * bf16_round(v[j].v[i] * r);
        store8(yr + 8 * c, o);
      }
    }
  }
}

// kAdd: dx = (the norm's input gradient) + dres in fp32, rounded once: the
// gradient of a residual sum h that feeds both the norm and a later add.
// x and dy stay in registers as raw bf16 between the two passes (4 registers
// per 8 values instead of 8), so more rows are in flight per SM; the second
// pass widens them again and recomputes x*r and dy*w exactly as the first.
template <int VPT, bool kAdd = false>
__global__ void __launch_bounds__(kNormThreads, VPT <= 4 ? 8 : 4) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                                  const __nv_bfloat16* __restrict__ dy, long long lddy,
                                                                  const __nv_bfloat16* __restrict__ w,
                                                                  const float* __restrict__ rstd, int rows, int D,
                                                                  __nv_bfloat16* __restrict__ dx, long long lddx,
                                                                  const __nv_bfloat16* __restrict__ dres = nullptr,
                                                                  long long lddres = 0) {
  __shared__ float red[kNormThreads / 32];
  const int nvec = D >> 3;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    const float r = rstd[row];
    const __nv_bfloat16* xr = x + static_cast<long long>(row) * ldx;
    const __nv_bfloat16* gr = dy + static_cast<long long>(row) * lddy;
    uint4 xq[VPT], gq[VPT];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = threadIdx.x + j * kNormThreads;
      if (c < nvec) {
        xq[j] = *reinterpret_cast<const uint4*>(xr + 8 * c);
        gq[j] = *reinterpret_cast<const uint4*>(gr + 8 * c);
      }
    }
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = threadIdx.x + j * kNormThreads;
      if (c < nvec) {
        const V8 n = widen8(xq[j]), g = widen8(gq[j]), wv = load8(w + 8 * c);
#pragma unroll
        for (int i = 0; i < 8; ++i) dot = fmaf(g.v[i] * wv.v[i], n.v[i] * r, dot);
      }
    }
    const float m = block_sum(dot, red) / static_cast<float>(D);
    __nv_bfloat16* dr = dx + static_cast<long long>(row) * lddx;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = threadIdx.x + j * kNormThreads;
      if (c < nvec) {
        const V8 n = widen8(xq[j]), g = widen8(gq[j]), wv = load8(w + 8 * c);
        V8 o;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float nn = n.v[i] * r, gg = g.v[i] * wv.v[i];
          o.v[i] = r * (gg - nn * m);
        }
        if (kAdd) {
          const V8 dv = load8(dres + static_cast<long long>(row) * lddres + 8 * c);
#pragma unroll
          for (int i = 0; i < 8; ++i) o.v[i] += dv.v[i];
        }
        store8(dr + 8 * c, o);
      }
    }
  }
}

struct RopeSide {            // one of q / k
  const __nv_bfloat16* in;   // [B, S, H, D] with strides (sb, ss, sh) elements, unit stride over D
  long long sb, ss, sh;
  int H;
  __nv_bfloat16* out;        // contiguous [B, S, H, D]
};

// One CTA per (b, s) position (grid-stride); a work item is 8 elements of
// the first half of one head and the matching 8 of the second half.
template <bool kBackward>
__global__ void __launch_bounds__(kRopeThreads) rope_kernel(RopeSide q, RopeSide k, const __nv_bfloat16* __restrict__ cos,
                                                            const __nv_bfloat16* __restrict__ sin, long long csb,
                                                            long long css, int B, int S, int D) {
  const int half = D >> 1;
  const int per_head = half >> 3;
  const int items = (q.H + k.H) * per_head;
  const long long positions = static_cast<long long>(B) * S;
  for (long long pos = blockIdx.x; pos < positions; pos += gridDim.x) {
    const int b = static_cast<int>(pos / S), s = static_cast<int>(pos % S);
    const __nv_bfloat16* cp = cos + b * csb + s * css;
    const __nv_bfloat16* sp = sin + b * csb + s * css;
    for (int it = threadIdx.x; it < items; it += kRopeThreads) {
      int h = it / per_head;
      const int c = (it - h * per_head) * 8;
      const RopeSide& side = h < q.H ? q : k;
      if (h >= q.H) h -= q.H;
      const __nv_bfloat16* src = side.in + b * side.sb + s * side.ss + h * side.sh;
      __nv_bfloat16* dst = side.out + ((pos * side.H + h) * static_cast<long long>(D));
      const V8 x1 = load8(src + c), x2 = load8(src + half + c);
      const V8 c1 = load8(cp + c), c2 = load8(cp + half + c);
      const V8 s1 = load8(sp + c), s2 = load8(sp + half + c);
      V8 o1, o2;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (kBackward) {
          o1.v[i] = fmaf(x1.v[i], c1.v[i], x2.v[i] * s2.v[i]);
          o2.v[i] = fmaf(x2.v[i], c2.v[i], -x1.v[i] * s1.v[i]);
        } else {
          o1.v[i] = fmaf(x1.v[i], c1.v[i], -x2.v[i] * s1.v[i]);
          o2.v[i] = fmaf(x2.v[i], c2.v[i], x1.v[i] * s2.v[i]);
        }
      }
      store8(dst + c, o1);
      store8(dst + half + c, o2);
    }
  }
}

__device__ __forceinline__ float sigmoidf_(float a) { return __fdividef(1.f, 1.f + __expf(-a)); }

template <bool kBackward>
__device__ __forceinline__ void swiglu_apply(const V8& av, const V8& uv, const V8& gv, __nv_bfloat16* out0,
                                             __nv_bfloat16* out1) {
  if (kBackward) {
    V8 da, du;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sg = sigmoidf_(av.v[j]);
      const float act = av.v[j] * sg;
      da.v[j] = gv.v[j] * uv.v[j] * (sg * (1.f + av.v[j] * (1.f - sg)));
      du.v[j] = gv.v[j] * act;
    }
    store8(out0, da);
    store8(out1, du);
  } else {
    V8 y;
#pragma unroll
    for (int j = 0; j < 8; ++j) y.v[j] = av.v[j] * sigmoidf_(av.v[j]) * uv.v[j];
    store8(out0, y);
  }
}

// Grid-stride over rows x (F / 8) vectors, two vectors per thread and
// iteration whose loads are all issued before either is computed; the
// (row, vector) position advances by the stride's quotient and remainder,
// with no division in the loop.
template <bool kBackward>
__global__ void __launch_bounds__(kEltThreads) swiglu_kernel(const __nv_bfloat16* __restrict__ a, long long lda,
                                                             const __nv_bfloat16* __restrict__ u, long long ldu,
                                                             const __nv_bfloat16* __restrict__ dy, long long lddy,
                                                             int rows, int F, __nv_bfloat16* __restrict__ out0,
                                                             __nv_bfloat16* __restrict__ out1, long long ldo) {
  const int nvec = F >> 3;
  const long long total = static_cast<long long>(rows) * nvec;
  const long long stride = static_cast<long long>(gridDim.x) * kEltThreads;
  const long long i0 = static_cast<long long>(blockIdx.x) * kEltThreads + threadIdx.x;
  if (i0 >= total) return;
  const long long dr = stride / nvec;
  const int dc = static_cast<int>(stride - dr * nvec);
  long long r = i0 / nvec;
  int c = static_cast<int>(i0 - r * nvec);
  for (long long i = i0; i < total; i += 2 * stride) {
    long long r2 = r + dr;
    int c2 = c + dc;
    if (c2 >= nvec) {
      c2 -= nvec;
      ++r2;
    }
    const bool second = i + stride < total;
    const V8 a0 = load8(a + r * lda + 8 * c), u0 = load8(u + r * ldu + 8 * c);
    V8 g0, a1, u1, g1;
    if (kBackward) g0 = load8(dy + r * lddy + 8 * c);
    if (second) {
      a1 = load8(a + r2 * lda + 8 * c2);
      u1 = load8(u + r2 * ldu + 8 * c2);
      if (kBackward) g1 = load8(dy + r2 * lddy + 8 * c2);
    }
    swiglu_apply<kBackward>(a0, u0, g0, out0 + r * ldo + 8 * c, kBackward ? out1 + r * ldo + 8 * c : nullptr);
    if (second)
      swiglu_apply<kBackward>(a1, u1, g1, out0 + r2 * ldo + 8 * c2, kBackward ? out1 + r2 * ldo + 8 * c2 : nullptr);
    r = r2 + dr;
    c = c2 + dc;
    if (c >= nvec) {
      c -= nvec;
      ++r;
    }
  }
}

}  // namespace blocks
}  // namespace vq

namespace vq {
namespace route {

constexpr int kThreads = 1024;
constexpr int kMaxKeys = 8;

// Stable counting sort of T keys in [0, K) by one CTA: order[pos] = i and
// inv[i] = pos for the element i that lands at position pos, group_off[k] =
// first position of key k (group_off[K] = T).  Keys >= K go to the last group.
// Thread t owns elements [t*E, (t+1)*E), so the per-thread counts, scanned
// over the threads, give every element its stable position.
__global__ void __launch_bounds__(kThreads) route_prep_kernel(const uint8_t* __restrict__ keys, long long T, int K,
                                                              long long* __restrict__ order, long long* __restrict__ inv,
                                                              int* __restrict__ group_off) {
  __shared__ int cnt[kMaxKeys][kThreads];  // per-thread counts, then their exclusive scan
  __shared__ int total[kMaxKeys];
  const int t = threadIdx.x;
  const long long E = (T + kThreads - 1) / kThreads;
  const long long b = t * E, e = b + E < T ? b + E : T;
  int c[kMaxKeys];
#pragma unroll
  for (int k = 0; k < kMaxKeys; ++k) c[k] = 0;
  for (long long i = b; i < e; ++i) {
    int k = keys[i];
    k = k < K ? k : K - 1;
#pragma unroll
    for (int q = 0; q < kMaxKeys; ++q) c[q] += (q == k);
  }
#pragma unroll
  for (int k = 0; k < kMaxKeys; ++k) cnt[k][t] = c[k];
  __syncthreads();
  // exclusive scan of each key's counts over the threads (one warp per key)
  const int warp = t >> 5, lane = t & 31;
  if (warp < K) {
    int run = 0;
    for (int base = 0; base < kThreads; base += 32) {
      const int v = cnt[warp][base + lane];
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      cnt[warp][base + lane] = run + x - v;
      run += __shfl_sync(0xffffffffu, x, 31);
    }
    if (lane == 0) total[warp] = run;
  }
  __syncthreads();
  int start[kMaxKeys];
  int acc = 0;
#pragma unroll
  for (int k = 0; k < kMaxKeys; ++k) {
    start[k] = acc + (k < K ? cnt[k][t] : 0);
    acc += k < K ? total[k] : 0;
  }
  if (t == 0) {
    int a = 0;
    for (int k = 0; k < K; ++k) {
      group_off[k] = a;
      a += total[k];
    }
    group_off[K] = a;
  }
  for (long long i = b; i < e; ++i) {
    int k = keys[i];
    k = k < K ? k : K - 1;
    int pos = 0;
#pragma unroll
    for (int q = 0; q < kMaxKeys; ++q)
      if (q == k) pos = start[q]++;
    order[pos] = i;
    inv[i] = pos;
  }
}

}  // namespace route
}  // namespace vq
