// Persistent, warp-specialised tcgen05 GEMM for the gated Linear.
//
//   D[M, N] = sum_k A[m, k] * B[n, k]      (bf16 operands, fp32 accumulate in TMEM)
//
// Operands are streamed by TMA in 128-byte-swizzled BK = 64 slices; either
// operand may be K-major (K contiguous) or MN-major (M/N contiguous), which
// covers the three GEMMs of the layer without any transpose copies:
//
//   forward   Y  = X  W^T : A = X  [T, Kin]  K-major,  B = W [N, Kin]  K-major
//   input grad dX = dY W  : A = dY [T, N]    K-major,  B = W [N, Kin]  MN-major
//   weight grad dW = dY^T X: A = dY [T, N]   MN-major, B = X [T, Kin]  MN-major
//
// Warp roles (256 threads): warp 0 issues TMA, warp 1 issues tcgen05.mma
// (one thread), warp 2 owns the TMEM allocation, warps 4-7 run the epilogue.
// The accumulator is double buffered in TMEM (2 x 256 fp32 columns) so the
// epilogue of tile i overlaps the main loop of tile i+1.  gemm_pair_kernel
// runs the same roles on a CTA pair (cta_group::2, 256-row tiles), with a
// second set of epilogue warps for the gate gradient, and optionally four
// more warps that decode and mix the B operand into shared memory instead of
// TMA (kMixB).
//
// Epilogues:
//   kEpiStoreBf16 : D -> bf16 C[M, N] (row-major, leading dimension ldc),
//                   through bulk tensor stores of 32 x 32 boxes where C allows.
//   kEpiGateGrad  : D is a 128 x 256 tile of dW; each epilogue thread owns one
//                   output row and dots it against the re-decoded candidate
//                   weights of the same 256-column unit, giving per-tile
//                   partial sums of g_k = <dW, W_k> that are written to
//                   partials[tile][warp][k] and reduced in fixed order by
//                   gategrad_reduce_kernel.  dW never reaches global memory.
//                   Several layers stacked by rows (q/k/v, gate/up) share one
//                   launch, each warp decoding its own layer's candidates.
//   kEpiSwiGLU    : paired kernel only; D holds 128 gate and the matching 128
//                   up outputs, the epilogue writes h = silu(gate) * up.
#pragma once

#include "common.cuh"
#include "decode_mix.cuh"
#include "formats.cuh"

namespace vq {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int THREADS = 256;
constexpr int A_STAGE = BM * BK * 2;  // 16 KiB
constexpr int B_STAGE = BN * BK * 2;  // 32 KiB
constexpr int TMEM_COLS = 512;        // two 256-column accumulators
constexpr int GROUP_N = 8;            // raster: tiles sweep M inside a band of 8 N-blocks

constexpr int kEpiStoreBf16 = 0;
constexpr int kEpiGateGrad = 1;
constexpr int kEpiSwiGLU = 2;  // paired kernel only: h = silu(gate) * up of a gate|up GEMM

// Shared memory: STAGES x (A, B) operand slices, the mbarriers, and for the
// gate-gradient epilogue one staging area per epilogue warp (32 rows x one
// candidate unit, row pitch kStagePitch words: odd, so the 32 rows of a warp
// fall in 32 different banks).  The dynamic shared-memory window starts
// 1024-byte aligned on sm_100 (checked at run time), as SWIZZLE_128B needs.
constexpr int kStagePitch = kMaxUnitWords + 1;  // 69 words
// Row pitch of the second gate-gradient epilogue set: the widest unit it may
// stage is Q6_K's 210 bytes = 53 words (odd, so again 32 distinct banks).
constexpr int kStagePitch1 = 53;
// One bulk-store buffer of the paired store epilogue: 32 rows x 32 bf16.
constexpr int kOutBufBytes = 32 * 32 * 2;
// Layers of one grouped gate-gradient launch (q/k/v, gate/up).
constexpr int kMaxGGroups = 4;

// Two floats rounded to bf16 (nearest even), packed low = a, high = b.
__device__ __forceinline__ uint32_t bf16x2_bits(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <int kEpi>
struct SmemLayout {
  static constexpr int a_off = 0;
  static constexpr int b_off = a_off + STAGES * A_STAGE;
  static constexpr int bar_off = b_off + STAGES * B_STAGE;      // 8-byte barriers
  static constexpr int n_bars = 2 * STAGES + 4;
  static constexpr int misc_off = bar_off + n_bars * 8;         // tmem base, abort flag
  static constexpr int stage_off = misc_off + 16;
  static constexpr int stage_words_per_warp = 32 * kStagePitch;
  static constexpr int stage_bytes = (kEpi == 1) ? 4 * stage_words_per_warp * 4 : 0;
  static constexpr int total = stage_off + stage_bytes;
};

struct Params {
  int M, N, K;
  int num_m_blk, num_n_blk, num_k_blk, num_tiles;
  // kEpiStoreBf16
  __nv_bfloat16* C;
  long long ldc;
  // paired store kernel: write C through the tensor map BMaps::c (32 x 32
  // boxes, 64-byte swizzle) instead of per-row 16-byte stores
  int tma_store;
  // decoded-B forward (paired kernel, kMixB): device float[K] mixture
  // weights of `cands`; valid columns = cols, units_per_row as above
  const float* mix_probs;
  // kEpiSwiGLU: B holds the gate rows [0, N) and the up rows [up_row,
  // up_row + N); a tile covers 128 output columns, the even CTA of the pair
  // loading gate rows and the odd one the matching up rows
  int up_row;
  // kEpiGateGrad: candidate rows = M (out features), valid columns = cols
  CandSet cands;
  int units_per_row;
  long long cols;
  float* partials;
  // paired gate-gradient kernel: bit k set = candidate k runs in the second
  // set of epilogue warps (never Q8_0, whose unit is too wide for its rows)
  int set1_mask;
  // stream-K tail (paired gate-gradient kernel only): when set, the tiles
  // left over after the full waves are split along K across all clusters;
  // pieces that do not start at k-block 0 write the partial slots that
  // follow the per-tile ones (sk_base), 16 per cluster.
  int stream_k;
  int sk_base;
  // grouped forward (paired kernel): rows [group_off[g], group_off[g + 1])
  // of A are multiplied with B_g; ngroups = 0 for a plain GEMM
  const int* group_off;
  int ngroups;
  // grouped gate gradient: gg_groups > 1 layers stacked by rows (dY's
  // columns), layer g owning rows [gg_row[g], gg_row[g + 1]) (multiples of
  // 32, so each epilogue warp's rows belong to one layer) with candidates
  // gg_ptr[g][k] of the formats in `cands`; partial slots hold gg_groups x K
  // values, layer g's at g * K, zero for the layers a warp does not cover
  int gg_groups;
  int gg_row[kMaxGGroups + 1];
  const uint8_t* gg_ptr[kMaxGGroups][kMaxCandidates];
  int* err;
};

constexpr int kMaxGroups = 8;

// B-operand tensor maps of a paired launch (one, or one per group), and the
// output map of the store epilogue (used when Params::tma_store is set).
template <int G>
struct BMaps {
  CUtensorMap m[G];
  CUtensorMap c;
};

// One unit of work of a persistent cluster: k-blocks [kb0, kb1) of a tile.
// piece >= 0 marks a stream-K piece (the cluster's first or second).
struct Seg {
  int tile, kb0, kb1, piece;
};

__device__ __forceinline__ void tile_coords(const Params& p, int tile, int& m_blk, int& n_blk) {
  const int band = GROUP_N * p.num_m_blk;
  const int g = tile / band;
  const int first_n = g * GROUP_N;
  const int gn = min(GROUP_N, p.num_n_blk - first_n);
  const int r = tile - g * band;
  m_blk = r / gn;
  n_blk = first_n + (r - m_blk * gn);
}

// Inverse of tile_coords.
__device__ __forceinline__ int tile_index(const Params& p, int m_blk, int n_blk) {
  const int g = n_blk / GROUP_N;
  const int first_n = g * GROUP_N;
  const int gn = min(GROUP_N, p.num_n_blk - first_n);
  return g * GROUP_N * p.num_m_blk + m_blk * gn + (n_blk - first_n);
}

// Segment i of cluster c out of C (the same sequence for every role).
__device__ __forceinline__ bool get_seg(const Params& p, int ntiles, int c, int C, int i, Seg& sg) {
  if (!p.stream_k) {
    const int tile = c + i * C;
    sg = {tile, 0, p.num_k_blk, -1};
    return tile < ntiles;
  }
  const int full = p.num_tiles / C;
  if (i < full) {
    sg = {c + i * C, 0, p.num_k_blk, -1};
    return true;
  }
  const int KB = p.num_k_blk;
  const int Gm = p.num_m_blk;
  if (full == 0 && Gm > 1 && p.num_n_blk <= C / Gm) {
    // Every tile split (fewer tiles than clusters): cluster c works on row
    // block c % Gm, and the clusters of the Gm row blocks that share an index
    // c / Gm walk the same (column block, k-block) range at the same time,
    // so each B k-slice is read from DRAM once for all row blocks.  A range
    // is at most one tile long (num_n_blk <= C / Gm), so it touches two tiles
    // at most.
    const int g = c % Gm, ic = c / Gm;
    const int Cg = C / Gm + (g < C % Gm ? 1 : 0);
    const long long Ug = static_cast<long long>(p.num_n_blk) * KB;
    const int lo = static_cast<int>(Ug * ic / Cg), hi = static_cast<int>(Ug * (ic + 1) / Cg);
    const int cut = (lo / KB + 1) * KB;
    const int j = i - full;
    if (j == 0 && lo < hi) {
      sg = {tile_index(p, g, lo / KB), lo % KB, (hi < cut ? hi : cut) - (lo / KB) * KB, 0};
      return true;
    }
    if (j == 1 && hi > cut) {
      sg = {tile_index(p, g, cut / KB), 0, hi - cut, 1};
      return true;
    }
    return false;
  }
  const long long U = static_cast<long long>(p.num_tiles - full * C) * KB;
  const int lo = static_cast<int>(U * c / C), hi = static_cast<int>(U * (c + 1) / C);
  const int j = i - full;
  const int cut = (lo / KB + 1) * KB;  // end of the tile the range starts in
  if (j == 0 && lo < hi) {
    sg = {full * C + lo / KB, lo % KB, (hi < cut ? hi : cut) - (lo / KB) * KB, 0};
    return true;
  }
  if (j == 1 && hi > cut) {
    sg = {full * C + cut / KB, 0, hi - cut, 1};
    return true;
  }
  return false;
}

// Stage this lane's unit (ub bytes at `unit`, 2-byte aligned) into its own
// slot row as ceil(ub / 4) aligned words.  The 16-byte aligned span around
// the unit is read with 16-byte loads (it never leaves the 16-byte granules
// that hold the unit's bytes) and realigned with funnel shifts; each lane
// stages and later decodes only its own row, so no warp synchronisation is
// needed between the two.
__device__ __forceinline__ void stage_row_lane(uint32_t* slot, const uint8_t* unit, int ub) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(unit);
  const uintptr_t a0 = a & ~uintptr_t(15);
  const int n16 = static_cast<int>((((a + ub + 15) & ~uintptr_t(15)) - a0) >> 4);
  const int d = static_cast<int>(a - a0);  // 0 .. 14, even
  const int dw = d >> 2;                   // first superset word of the unit
  const uint32_t sh = static_cast<uint32_t>(d & 2) * 8u;
  const int nw = (ub + 3) >> 2;
  const uint4* src = reinterpret_cast<const uint4*>(a0);
  if (d == 0 && (ub & 15) == 0) {  // 16-byte aligned unit of whole vectors: plain copy
#pragma unroll 1
    for (int t = 0; t < n16; ++t) {
      const uint4 v = __ldg(src + t);
      slot[4 * t] = v.x;
      slot[4 * t + 1] = v.y;
      slot[4 * t + 2] = v.z;
      slot[4 * t + 3] = v.w;
    }
    return;
  }
  // superset word g pairs with word g + 1: out[g - dw] = funnel(W[g], W[g + 1], sh)
  uint32_t prev = 0u;
#pragma unroll 1
  for (int t = 0; t < n16; ++t) {
    const uint4 v = __ldg(src + t);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    const int o0 = 4 * t - 1 - dw;  // output word completed by superset word 4t
    if (o0 >= 0 && o0 + 3 < nw) {   // interior vector: all four outputs in range
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        slot[o0 + i] = __funnelshift_r(prev, w[i], sh);
        prev = w[i];
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int o = o0 + i;
        if (o >= 0 && o < nw) slot[o] = __funnelshift_r(prev, w[i], sh);
        prev = w[i];
      }
    }
  }
  const int o = 4 * n16 - 1 - dw;
  if (o >= 0 && o < nw) slot[o] = __funnelshift_r(prev, 0u, sh);
}

// Dot of one dW row (256 TMEM columns at t_row, fp32) with the decoded unit
// in `slot` (this thread's row); columns at or beyond `cols` are skipped.
// Per 32-weight sub-block with w = a[h] * q + b[h] (h = half):
//   sum_j v_j w_j = sum_h a[h] * sum_{j in h} v_j q_j  (+ b[h] * sum_{j in h} v_j),
// with q_j = (2^23 + code byte) - kSub formed and accumulated as fp32 pairs.
// All 32 lanes must call it (tcgen05.ld is warp-collective).
template <int F>
__device__ __forceinline__ float row_dot(const uint32_t* slot, uint32_t t_row, long long colbase, long long cols,
                                         bool row_ok) {
  float s = 0.f;
  const uint64_t nsub = f2pack(-Chunk<F>::kSub, -Chunk<F>::kSub);
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    float v[32];
    tmem_ld_32cols(t_row + c * 32, v);
    const long long col0 = colbase + c * 32;
    if (row_ok && col0 < cols) {
      if (col0 + 32 > cols) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j >= cols) v[j] = 0.f;
      }
      float a[2], b[2];
      uint32_t qb[8];
      Chunk<F>::qbytes(slot, c, a, b, qb);
      uint64_t acc[2] = {0ull, 0ull}, vs[2] = {0ull, 0ull};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint64_t q01 = f2add(f2pack(magic_byte(qb[j], 0), magic_byte(qb[j], 1)), nsub);
        const uint64_t q23 = f2add(f2pack(magic_byte(qb[j], 2), magic_byte(qb[j], 3)), nsub);
        const uint64_t v01 = f2pack(v[4 * j], v[4 * j + 1]);
        const uint64_t v23 = f2pack(v[4 * j + 2], v[4 * j + 3]);
        acc[j >> 2] = f2fma(v01, q01, acc[j >> 2]);
        acc[j >> 2] = f2fma(v23, q23, acc[j >> 2]);
        if (Chunk<F>::kMin) {
          vs[j >> 2] = f2add(vs[j >> 2], v01);
          vs[j >> 2] = f2add(vs[j >> 2], v23);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float2 p = f2unpack(acc[h]);
        s = fmaf(a[h], p.x + p.y, s);
        if (Chunk<F>::kMin) {
          const float2 u = f2unpack(vs[h]);
          s = fmaf(b[h], u.x + u.y, s);
        }
      }
    }
  }
  return s;
}

// Store epilogue of one warp's 32 rows of a 128 x 256 accumulator tile
// through TMA: each 32-column slice is converted to bf16 into a 2 KB buffer
// in the 64-byte-swizzled layout of the output map's 32 x 32 box (16-byte
// chunk c of row r at r * 64 + ((c ^ (r >> 1) & 3) * 16), so each quarter-warp
// of 16-byte shared stores hits all 32 banks once) and written by one bulk
// tensor store from lane 0.  The warp's two buffers alternate (`it` counts
// the warp's slices); rows and columns past the map's extent are not written.
__device__ __forceinline__ void epilogue_store_tma(const Params& p, const CUtensorMap* tmc, uint8_t* bufs,
                                                   uint32_t t_row, int row0, int n_blk, int lane, uint32_t& it) {
  for (int c = 0; c < BN / 32; ++c) {
    const int col0 = n_blk * BN + c * 32;
    if (col0 >= p.N) break;  // uniform across the warp
    float v[32];
    tmem_ld_32cols(t_row + c * 32, v);
    uint8_t* buf = bufs + (it & 1u) * kOutBufBytes;
    if (lane == 0) bulk_wait_read<1>();  // the store that last read this buffer is done with it
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 q;
      q.x = bf16x2_bits(v[8 * j + 0], v[8 * j + 1]);
      q.y = bf16x2_bits(v[8 * j + 2], v[8 * j + 3]);
      q.z = bf16x2_bits(v[8 * j + 4], v[8 * j + 5]);
      q.w = bf16x2_bits(v[8 * j + 6], v[8 * j + 7]);
      *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = q;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmc, smem_u32(buf), col0, row0);
      bulk_commit();
    }
    ++it;
  }
}

// silu(g) * u with the operations, and the order, of the SwiGLU kernel.
__device__ __forceinline__ float silu_mul(float g, float u) {
  const float sg = __fdividef(1.f, 1.f + __expf(-g));
  return g * sg * u;
}

__device__ __forceinline__ float bf16_rn(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// SwiGLU epilogue of one warp's 32 rows: TMEM columns [0, 128) of the tile
// are gate outputs and [128, 256) the up outputs of the same 128 features
// (n_blk * 128 + j).  Each is rounded to bf16 first, as a GEMM writing
// gate|up in bf16 would, so h = bf16(silu(g) * u) equals the SwiGLU
// kernel's result on that output bit for bit.  Stored like the store
// epilogue: a bulk tensor store per 32 x 32 box, or row by row where the
// output map is not usable.
__device__ __forceinline__ void epilogue_swiglu(const Params& p, const CUtensorMap* tmc, uint8_t* bufs,
                                                uint32_t t_row, int row0, int n_blk, int lane, uint32_t& it) {
  const long long row = static_cast<long long>(row0) + lane;
  for (int c = 0; c < 4; ++c) {
    const int col0 = n_blk * 128 + c * 32;
    if (col0 >= p.N) break;  // uniform across the warp
    float g[32], u[32];
    tmem_ld_32cols(t_row + c * 32, g);
    tmem_ld_32cols(t_row + 128 + c * 32, u);
    uint32_t hb[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      hb[j] = bf16x2_bits(silu_mul(bf16_rn(g[2 * j]), bf16_rn(u[2 * j])),
                          silu_mul(bf16_rn(g[2 * j + 1]), bf16_rn(u[2 * j + 1])));
    if (p.tma_store) {
      uint8_t* buf = bufs + (it & 1u) * kOutBufBytes;
      if (lane == 0) bulk_wait_read<1>();  // the store that last read this buffer is done with it
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 4; ++j)
        *reinterpret_cast<uint4*>(buf + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) =
            make_uint4(hb[4 * j], hb[4 * j + 1], hb[4 * j + 2], hb[4 * j + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(tmc, smem_u32(buf), col0, row0);
        bulk_commit();
      }
      ++it;
    } else if (row < p.M) {
      __nv_bfloat16* dst = p.C + row * p.ldc + col0;
      if (col0 + 32 <= p.N && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          reinterpret_cast<uint4*>(dst)[j] = make_uint4(hb[4 * j], hb[4 * j + 1], hb[4 * j + 2], hb[4 * j + 3]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (col0 + j < p.N)
            dst[j] = __ushort_as_bfloat16(
                static_cast<unsigned short>((j & 1) ? hb[j >> 1] >> 16 : hb[j >> 1] & 0xFFFFu));
      }
    }
  }
}

// One row of a CTA's B half for k-block [k0, k0 + 64) of a mixed weight,
// decoded and mixed into shared memory by its own thread: W[nrow, k] =
// sum_k p_k decode(W_k)[nrow, k] with mix_units_kernel's arithmetic (the
// same candidate order, products and single bf16 rounding, so the tile
// equals the mix kernel's W_mix bit for bit), columns at or past `cols` and
// rows at or past N as zero.  Written in the 128-byte-swizzled K-major
// layout a TMA load of the tile would produce: 16-byte chunk j of row r at
// chunk j ^ (r & 7).  Each candidate unit is first staged into the thread's
// own slot row (16-byte loads that stay inside the unit's 16-byte granules).
__device__ __forceinline__ void mix_b_row(const Params& p, uint8_t* brow, uint32_t* slot_row, int nrow, int k0,
                                          int r7) {
  uint32_t packed[32];
  if (nrow < p.N) {
    const int c0 = (k0 & 255) >> 5;  // the k-block's first 32-weight sub-block of its unit
    const long long unit = static_cast<long long>(nrow) * p.units_per_row + (k0 >> 8);
    float2 acc0[16], acc1[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc0[j] = acc1[j] = make_float2(0.f, 0.f);
    float cst0[2] = {0.f, 0.f}, cst1[2] = {0.f, 0.f};
    for (int k = 0; k < p.cands.K; ++k) {
      const int ub = p.cands.ubytes[k];
      stage_row_lane(slot_row, p.cands.ptr[k] + unit * ub, ub);
      const URef u{slot_row, 0, 0u};
      const float pk = __ldg(p.mix_probs + k);
      switch (p.cands.fmt[k]) {
        case kQ8_0: mix_chunk<kQ8_0>(u, c0, pk, acc0, cst0); mix_chunk<kQ8_0>(u, c0 + 1, pk, acc1, cst1); break;
        case kQ2_K: mix_chunk<kQ2_K>(u, c0, pk, acc0, cst0); mix_chunk<kQ2_K>(u, c0 + 1, pk, acc1, cst1); break;
        case kQ3_K: mix_chunk<kQ3_K>(u, c0, pk, acc0, cst0); mix_chunk<kQ3_K>(u, c0 + 1, pk, acc1, cst1); break;
        case kQ4_K: mix_chunk<kQ4_K>(u, c0, pk, acc0, cst0); mix_chunk<kQ4_K>(u, c0 + 1, pk, acc1, cst1); break;
        case kQ5_K: mix_chunk<kQ5_K>(u, c0, pk, acc0, cst0); mix_chunk<kQ5_K>(u, c0 + 1, pk, acc1, cst1); break;
        case kQ6_K: mix_chunk<kQ6_K>(u, c0, pk, acc0, cst0); mix_chunk<kQ6_K>(u, c0 + 1, pk, acc1, cst1); break;
        case kIQ4_XS:
          mix_chunk<kIQ4_XS>(u, c0, pk, acc0, cst0);
          mix_chunk<kIQ4_XS>(u, c0 + 1, pk, acc1, cst1);
          break;
        default: break;  // the host checked every format
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int e0 = k0 + 2 * j, e1 = k0 + 32 + 2 * j;  // columns of acc0[j].x and acc1[j].x
      const float c0v = cst0[j >> 3], c1v = cst1[j >> 3];
      packed[j] = e0 < p.cols ? bf16x2_bits(acc0[j].x + c0v, e0 + 1 < p.cols ? acc0[j].y + c0v : 0.f) : 0u;
      packed[16 + j] = e1 < p.cols ? bf16x2_bits(acc1[j].x + c1v, e1 + 1 < p.cols ? acc1[j].y + c1v : 0.f) : 0u;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) packed[j] = 0u;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<uint4*>(brow + ((j ^ r7) << 4)) =
        make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
}

// Epilogue of one 128 x 256 accumulator tile held in this CTA's TMEM.
//   row0: first output row of this warp's 32 TMEM lanes; m128: index of the
//   128-row block (for the gate-gradient partial slots); stage: the
//   gate-gradient staging area (4 warps x 32 rows x kStagePitch words).
//   cand_set: -1 = every candidate, else only those of that epilogue set
//   (Params::set1_mask); pitch: words per staging row of this warp's set.
template <int kEpi>
__device__ __forceinline__ void epilogue_tile(const Params& p, uint8_t* stage, uint32_t t_row, long long row0,
                                              int m128, int n_blk, int wq, int lane, long long slot_override = -1,
                                              long long row_end = -1, int cand_set = -1, int pitch = kStagePitch) {
  const long long row = row0 + lane;
  const bool row_ok = row >= 0 && row < (row_end >= 0 ? row_end : static_cast<long long>(p.M));
  if (kEpi == kEpiStoreBf16) {
    for (int c = 0; c < BN / 32; ++c) {
      float v[32];
      tmem_ld_32cols(t_row + c * 32, v);
      const long long col0 = static_cast<long long>(n_blk) * BN + c * 32;
      if (row_ok && col0 < p.N) {
        __nv_bfloat16* dst = p.C + row * p.ldc + col0;
        if (col0 + 32 <= p.N && ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0)) {
          __align__(16) __nv_bfloat162 pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) pk[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
#pragma unroll
          for (int j = 0; j < 4; ++j) reinterpret_cast<uint4*>(dst)[j] = reinterpret_cast<const uint4*>(pk)[j];
        } else {
          for (int j = 0; j < 32 && col0 + j < p.N; ++j) dst[j] = __float2bfloat16_rn(v[j]);
        }
      }
    }
  } else {
    // Gate-gradient epilogue.  For each candidate: each thread stages its own
    // row's unit (one 256-column unit) into its shared slot row with 16-byte
    // loads, decodes it from there and dots it with the dW row read back from
    // TMEM; the warp then sums its 32 rows into one partial.
    uint32_t* slot_row = reinterpret_cast<uint32_t*>(stage) + (wq * 32 + lane) * pitch;
    const long long slot =
        slot_override >= 0 ? slot_override : (static_cast<long long>(m128) * p.num_n_blk + n_blk) * 4 + wq;
    const long long colbase = static_cast<long long>(n_blk) * BN;
    int gi = 0;  // layer of this warp's rows (grouped launch)
    long long lrow = row;
    if (p.gg_groups > 1) {
      while (gi + 1 < p.gg_groups && row0 >= p.gg_row[gi + 1]) ++gi;
      lrow = row - p.gg_row[gi];
    }
    const int KK = p.gg_groups > 1 ? p.gg_groups * p.cands.K : p.cands.K;
    const long long urow = (row_ok ? lrow : 0) * p.units_per_row + n_blk;
    for (int k = 0; k < p.cands.K; ++k) {
      if (cand_set >= 0 && ((p.set1_mask >> k) & 1) != cand_set) continue;
      const uint8_t* base = p.gg_groups > 1 ? p.gg_ptr[gi][k] : p.cands.ptr[k];
      stage_row_lane(slot_row, base + urow * p.cands.ubytes[k], p.cands.ubytes[k]);
      float s = 0.f;
      switch (p.cands.fmt[k]) {
        case kQ8_0: s = row_dot<kQ8_0>(slot_row, t_row, colbase, p.cols, row_ok); break;
        case kQ2_K: s = row_dot<kQ2_K>(slot_row, t_row, colbase, p.cols, row_ok); break;
        case kQ3_K: s = row_dot<kQ3_K>(slot_row, t_row, colbase, p.cols, row_ok); break;
        case kQ4_K: s = row_dot<kQ4_K>(slot_row, t_row, colbase, p.cols, row_ok); break;
        case kQ5_K: s = row_dot<kQ5_K>(slot_row, t_row, colbase, p.cols, row_ok); break;
        case kQ6_K: s = row_dot<kQ6_K>(slot_row, t_row, colbase, p.cols, row_ok); break;
        case kIQ4_XS: s = row_dot<kIQ4_XS>(slot_row, t_row, colbase, p.cols, row_ok); break;
        default: s = row_dot<kQ8_0>(slot_row, t_row, colbase, 0, false); break;  // keeps TMEM loads uniform
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) {
        float* dst = p.partials + slot * KK + k;
        for (int g = 0; g < KK / p.cands.K; ++g) dst[g * p.cands.K] = g == gi ? s : 0.f;
      }
      __syncwarp();
    }
  }
}

template <bool kAmn, bool kBmn, int kEpi>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, Params p) {
  using SL = SmemLayout<kEpi>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  if ((sbase & 1023u) != 0) {  // uniform across the CTA: nothing has started yet
    if (threadIdx.x == 0) report_error(p.err, kDevBadSmemAlign, 0);
    return;
  }
  const uint32_t bar0 = sbase + SL::bar_off;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + SL::misc_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + SL::misc_off + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 2) {
    tmem_alloc(smem_u32(tmem_holder), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      bool alive = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && alive; tile += gridDim.x) {
        int m_blk, n_blk;
        tile_coords(p, tile, m_blk, n_blk);
        for (int kb = 0; kb < p.num_k_blk; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag)) {
            report_error(p.err, kDevWaitTimeout, 1);
            alive = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(s), A_STAGE + B_STAGE);
          const uint32_t a_dst = sbase + SL::a_off + s * A_STAGE;
          const uint32_t b_dst = sbase + SL::b_off + s * B_STAGE;
          const int k0 = kb * BK;
          if (kAmn) {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * (64 * BK * 2), &tmA, full_bar(s), m_blk * BM + 64 * j, k0);
          } else {
            tma_load_2d(a_dst, &tmA, full_bar(s), k0, m_blk * BM);
          }
          if (kBmn) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * (64 * BK * 2), &tmB, full_bar(s), n_blk * BN + 64 * j, k0);
          } else {
            tma_load_2d(b_dst, &tmB, full_bar(s), k0, n_blk * BN);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN, kAmn, kBmn);
      uint32_t it = 0, local = 0;
      bool alive = true;
      for (int tile = blockIdx.x; tile < p.num_tiles && alive; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1u;
        if (!mbar_wait(tempty_bar(acc), aph ^ 1u, abort_flag)) {
          report_error(p.err, kDevWaitTimeout, 2);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = 0; kb < p.num_k_blk; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!mbar_wait(full_bar(s), ph, abort_flag)) {
            report_error(p.err, kDevWaitTimeout, 3);
            alive = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sbase + SL::a_off + s * A_STAGE;
          const uint32_t b_addr = sbase + SL::b_off + s * B_STAGE;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // K-major: +32 bytes per 16-element K step inside the swizzle row.
            // MN-major: +16 rows of 128 bytes per K step; MN atoms 64*BK*2 apart.
            const uint64_t adesc = kAmn ? smem_desc_sw128(a_addr + kk * 2048, 64 * BK * 2, 1024)
                                        : smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bdesc = kBmn ? smem_desc_sw128(b_addr + kk * 2048, 64 * BK * 2, 1024)
                                        : smem_desc_sw128(b_addr + kk * 32, 16, 1024);
            tc_mma_bf16(d_tmem, adesc, bdesc, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(empty_bar(s));  // frees this smem stage once its MMAs retire
        }
        if (!alive) break;
        tc_commit(tfull_bar(acc));  // accumulator ready for the epilogue
      }
    }
  } else if (warp >= 4) {
    // --------------------------------------------------------------- epilogue
    const int wq = warp & 3;  // TMEM lanes 32*wq .. 32*wq+31
    uint32_t local = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++local) {
      int m_blk, n_blk;
      tile_coords(p, tile, m_blk, n_blk);
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1u;
      if (!mbar_wait(tfull_bar(acc), aph, abort_flag)) {
        if (lane == 0) report_error(p.err, kDevWaitTimeout, 4);
        break;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(32 * wq) << 16) + acc * BN;

      epilogue_tile<kEpi>(p, smem + SL::stage_off, t_row, static_cast<long long>(m_blk) * BM + 32 * wq, m_blk,
                          n_blk, wq, lane);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}


// ===================================================================== 2-CTA
// The same GEMM on a CTA pair (cluster of 2, tcgen05 cta_group::2): a pair
// tile is 256 x 256; CTA r of the pair loads rows [128r, 128r + 128) of the
// A tile and rows [128r, 128r + 128) of the B tile (the MMA takes A split by M
// and B split by N across the pair), so each SM streams half of B and its
// shared memory feeds the tensor pipe at 8 KB per 256x256x16 step instead of
// 12 KB per 128x256x16.  One thread of the even CTA issues the MMAs; its
// commits arrive on both CTAs' barriers (tcgen05.commit multicast); both CTAs'
// TMA loads count on the even CTA's "full" barriers.  Each CTA's TMEM holds
// the fp32 accumulator of its own 128 rows, so the epilogue is unchanged.
constexpr int PA_STAGE = 128 * BK * 2;  // 16 KiB
constexpr int PB_STAGE = 128 * BK * 2;  // 16 KiB

// Per-epilogue shape of the paired kernel.  The gate-gradient epilogue
// (decode K candidates and dot them with the dW tile) would take longer than
// a tile's main loop with one warp per TMEM lane quarter, stalling the MMAs
// on the accumulator buffers; it runs two sets of four warps that split the
// candidates, and one pipeline stage fewer makes room for the second set's
// staging rows.
template <int kEpi>
struct PairCfg {
  static constexpr int kEpiSets = kEpi == kEpiGateGrad ? 2 : 1;
  static constexpr int kStages = kEpi == kEpiGateGrad ? 5 : 6;
  static constexpr int kThreads = 128 + 128 * kEpiSets;  // TMA, MMA, TMEM-owner, spare warp + epilogue sets
};

// kMixB: the B operand (the mixed weight) is decoded and mixed into shared
// memory by four producer warps per CTA instead of loaded by TMA; each of
// their threads stages one candidate unit at a time (kStagePitch words).
template <int kEpi, bool kMixB = false>
struct PairSmemLayout {
  static constexpr int kStages = kMixB ? 5 : PairCfg<kEpi>::kStages;
  static constexpr int a_off = 0;
  static constexpr int b_off = a_off + kStages * PA_STAGE;
  static constexpr int bar_off = b_off + kStages * PB_STAGE;
  static constexpr int n_bars = 2 * kStages + 4;
  static constexpr int misc_off = bar_off + n_bars * 8;  // tmem base, abort flag, group m-tile prefix
  static constexpr int grp_off = misc_off + 16;
  static constexpr int stage_off = misc_off + 64;
  static constexpr int stage1_off = stage_off + 4 * 32 * kStagePitch * 4;  // second set's rows
  static constexpr int stage_bytes = (kEpi == 1) ? 4 * 32 * (kStagePitch + kStagePitch1) * 4 : 0;
  // store epilogue: two 2 KB bulk-store buffers per epilogue warp, 1024-byte
  // aligned (the 64-byte swizzle pattern repeats every 512 bytes)
  static constexpr int out_off = (stage_off + 1023) & ~1023;
  static constexpr int out_bytes = (kEpi != kEpiGateGrad) ? 4 * 2 * kOutBufBytes : 0;
  static constexpr int mixb_off = out_off + out_bytes;
  static constexpr int mixb_bytes = kMixB ? 128 * kStagePitch * 4 : 0;
  static constexpr int total =
      kEpi != kEpiGateGrad ? mixb_off + mixb_bytes : stage_off + stage_bytes;
  static_assert(total <= 232448, "paired kernel shared memory above the 227 KB per-block limit");
};

// Grouped tile -> (group, first output row of the 256-row tile, column block),
// row-major within a group; mt[g] is the prefix of the groups' 256-row tiles.
__device__ __forceinline__ void group_tile(const Params& p, const int* mt, int tile, int& g, int& row_base,
                                           int& n_blk) {
  g = 0;
  while (g + 1 < p.ngroups && tile >= mt[g + 1] * p.num_n_blk) ++g;
  const int local = tile - mt[g] * p.num_n_blk;
  n_blk = local % p.num_n_blk;
  row_base = __ldg(p.group_off + g) + (local / p.num_n_blk) * 256;
}

template <bool kAmn, bool kBmn, int kEpi, int G = 1, bool kMixB = false>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(PairCfg<kEpi>::kThreads + (kMixB ? 128 : 0), 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ BMaps<G> tmB, Params p) {
  using SL = PairSmemLayout<kEpi, kMixB>;
  constexpr int NST = SL::kStages;
  constexpr int kSets = PairCfg<kEpi>::kEpiSets;
  static_assert(!kMixB || (!kAmn && !kBmn && kEpi == kEpiStoreBf16 && G == 1),
                "decoded B operand: forward store GEMM only");
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  if ((sbase & 1023u) != 0) {  // uniform in both CTAs: the layout is identical
    if (threadIdx.x == 0) report_error(p.err, kDevBadSmemAlign, 1);
    return;
  }
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t bar0 = sbase + SL::bar_off;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (NST + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * NST + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * NST + 2 + a); };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + SL::misc_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + SL::misc_off + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cluster_id = blockIdx.x >> 1, num_clusters = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(full_bar(s), kMixB ? 1 + 8 : 1);  // (kMixB: + 4 decoding warps x 2 CTAs)
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 8 * kSets);  // 4 epilogue warps per set x 2 CTAs (used in the even CTA)
    }
    *abort_flag = 0;
    if (G > 1) {  // 256-row tiles per group, from the device-side group offsets
      int* mt = reinterpret_cast<int*>(smem + SL::grp_off);
      mt[0] = 0;
      for (int g = 0; g < p.ngroups; ++g) {  // group sizes clamped to [0, M]: at most M/256 + G tiles
        int rows = __ldg(p.group_off + g + 1) - __ldg(p.group_off + g);
        rows = rows < 0 ? 0 : (rows > p.M ? p.M : rows);
        mt[g + 1] = mt[g] + (rows + 255) / 256;
      }
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    for (int g = 0; g < (G > 1 ? p.ngroups : 1); ++g) tma_prefetch_desc(&tmB.m[g]);
  }
  if (warp == 2) {
    tmem_alloc_pair(smem_u32(tmem_holder), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const int* mt = reinterpret_cast<const int*>(smem + SL::grp_off);
  const int ntiles = G > 1 ? mt[p.ngroups] * p.num_n_blk : p.num_tiles;
  // tile -> (B map, first output row of the 256-row tile, column block, end of its rows)
  auto coords = [&](int tile, const CUtensorMap*& bmap, int& row_base, int& n_blk, int& row_end, int& m_blk) {
    if (G > 1) {
      int g;
      group_tile(p, mt, tile, g, row_base, n_blk);
      bmap = &tmB.m[g];
      row_end = min(__ldg(p.group_off + g + 1), p.M);  // rows outside the group or the output are not stored
      m_blk = 0;
    } else {
      tile_coords(p, tile, m_blk, n_blk);
      bmap = &tmB.m[0];
      row_base = m_blk * 256;
      row_end = p.M;
    }
  };

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      uint32_t it = 0;
      bool alive = true;
      Seg sg;
      for (int si = 0; alive && get_seg(p, ntiles, cluster_id, num_clusters, si, sg); ++si) {
        int m_blk, n_blk, row_base, row_end;
        const CUtensorMap* bmap;
        coords(sg.tile, bmap, row_base, n_blk, row_end, m_blk);
        const int m0 = row_base + 128 * static_cast<int>(rank);
        const int n0 = kEpi == kEpiSwiGLU ? n_blk * 128 + (rank ? p.up_row : 0)
                                          : n_blk * BN + 128 * static_cast<int>(rank);
        for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++it) {
          const int s = it % NST;
          const uint32_t ph = (it / NST) & 1u;
          if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_flag)) {
            report_error(p.err, kDevWaitTimeout, 11);
            alive = false;
            break;
          }
          const uint32_t fb = map_to_rank(full_bar(s), 0);
          if (leader) mbar_arrive_expect_tx(full_bar(s), kMixB ? 2 * PA_STAGE : 2 * (PA_STAGE + PB_STAGE));
          const uint32_t a_dst = sbase + SL::a_off + s * PA_STAGE;
          const uint32_t b_dst = sbase + SL::b_off + s * PB_STAGE;
          const int k0 = kb * BK;
          if (kAmn) {
#pragma unroll
            for (int j = 0; j < 2; ++j) tma_load_2d_pair(a_dst + j * (64 * BK * 2), &tmA, fb, m0 + 64 * j, k0);
          } else {
            tma_load_2d_pair(a_dst, &tmA, fb, k0, m0);
          }
          if (kMixB) {
            // B is written by the decoding warps
          } else if (kBmn) {
#pragma unroll
            for (int j = 0; j < 2; ++j) tma_load_2d_pair(b_dst + j * (64 * BK * 2), bmap, fb, n0 + 64 * j, k0);
          } else {
            tma_load_2d_pair(b_dst, bmap, fb, k0, n0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer (even CTA)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(256, BN, kAmn, kBmn);
      uint32_t it = 0, local = 0;
      bool alive = true;
      Seg sg;
      for (int si = 0; alive && get_seg(p, ntiles, cluster_id, num_clusters, si, sg); ++si, ++local) {
        const int acc = local & 1;
        const uint32_t aph = (local >> 1) & 1u;
        if (!mbar_wait(tempty_bar(acc), aph ^ 1u, abort_flag)) {
          report_error(p.err, kDevWaitTimeout, 12);
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++it) {
          const int s = it % NST;
          const uint32_t ph = (it / NST) & 1u;
          if (!mbar_wait(full_bar(s), ph, abort_flag)) {
            report_error(p.err, kDevWaitTimeout, 13);
            alive = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sbase + SL::a_off + s * PA_STAGE;
          const uint32_t b_addr = sbase + SL::b_off + s * PB_STAGE;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t adesc = kAmn ? smem_desc_sw128(a_addr + kk * 2048, 64 * BK * 2, 1024)
                                        : smem_desc_sw128(a_addr + kk * 32, 16, 1024);
            const uint64_t bdesc = kBmn ? smem_desc_sw128(b_addr + kk * 2048, 64 * BK * 2, 1024)
                                        : smem_desc_sw128(b_addr + kk * 32, 16, 1024);
            tc_mma_bf16_pair(d_tmem, adesc, bdesc, idesc, (kb > sg.kb0 || kk > 0) ? 1u : 0u);
          }
          tc_commit_pair_mc(empty_bar(s), 0x3);  // frees stage s in both CTAs
        }
        if (!alive) break;
        tc_commit_pair_mc(tfull_bar(acc), 0x3);  // accumulators ready in both CTAs
      }
    }
  } else if (kMixB && warp >= 4 + 4 * kSets) {
    // ------------------------------------------------- B producer: decode + mix (both CTAs)
    const int dt = threadIdx.x - (4 + 4 * kSets) * 32;  // this thread's row of the CTA's 128-row B half
    uint32_t* slot_row = reinterpret_cast<uint32_t*>(smem + SL::mixb_off) + dt * kStagePitch;
    uint32_t it = 0;
    bool alive = true;
    Seg sg;
    for (int si = 0; alive && get_seg(p, ntiles, cluster_id, num_clusters, si, sg); ++si) {
      int m_blk, n_blk, row_base, row_end;
      const CUtensorMap* bmap;
      coords(sg.tile, bmap, row_base, n_blk, row_end, m_blk);
      const int nrow = n_blk * BN + 128 * static_cast<int>(rank) + dt;
      for (int kb = sg.kb0; kb < sg.kb1; ++kb, ++it) {
        const int s = it % NST;
        const uint32_t ph = (it / NST) & 1u;
        int ok = 1;
        if (lane == 0) ok = mbar_wait(empty_bar(s), ph ^ 1u, abort_flag) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);  // one decision for the whole warp
        __syncwarp();
        if (!ok) {
          if (lane == 0) report_error(p.err, kDevWaitTimeout, 16);
          alive = false;
          break;
        }
        mix_b_row(p, smem + SL::b_off + s * PB_STAGE + dt * 128, slot_row, nrow, kb * BK, dt & 7);
        fence_proxy_async_smem();  // the tensor cores read these rows through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_to_rank(full_bar(s), 0));
      }
    }
  } else if (warp >= 4) {
    // --------------------------------------------------------------- epilogue (both CTAs)
    const int wq = warp & 3;
    const int eset = (warp - 4) >> 2;  // epilogue set (TMEM lane quarter wq in either set)
    uint8_t* stage = smem + (eset ? SL::stage1_off : SL::stage_off);
    const int pitch = eset ? kStagePitch1 : kStagePitch;
    const uint32_t tempty_leader0 = map_to_rank(tempty_bar(0), 0);
    const uint32_t tempty_leader1 = map_to_rank(tempty_bar(1), 0);
    uint32_t local = 0, out_it = 0;
    bool sk_written[2] = {false, false};
    Seg sg;
    for (int si = 0; get_seg(p, ntiles, cluster_id, num_clusters, si, sg); ++si, ++local) {
      int m_blk, n_blk, row_base, row_end;
      const CUtensorMap* bmap;
      coords(sg.tile, bmap, row_base, n_blk, row_end, m_blk);
      const int acc = local & 1;
      const uint32_t aph = (local >> 1) & 1u;
      if (!mbar_wait(tfull_bar(acc), aph, abort_flag)) {
        if (lane == 0) report_error(p.err, kDevWaitTimeout, 14);
        break;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(32 * wq) << 16) + acc * BN;
      const int m128 = m_blk * 2 + static_cast<int>(rank);
      long long slot = -1;  // the tile's own slots unless a stream-K piece after the tile's first
      if (sg.piece >= 0 && sg.kb0 > 0) {
        slot = p.sk_base + ((static_cast<long long>(cluster_id) * 2 + sg.piece) * 2 + rank) * 4 + wq;
        sk_written[sg.piece] = true;
      }
      const int row0 = row_base + 128 * static_cast<int>(rank) + 32 * wq;
      // bulk stores clip at the output's last row, not at a group's end: a
      // warp whose rows straddle a group boundary stores row by row
      if (kEpi == kEpiSwiGLU)
        epilogue_swiglu(p, &tmB.c, smem + SL::out_off + wq * 2 * kOutBufBytes, t_row, row0, n_blk, lane, out_it);
      else if (kEpi == kEpiStoreBf16 && p.tma_store && (row_end == p.M || row0 + 32 <= row_end))
        epilogue_store_tma(p, &tmB.c, smem + SL::out_off + wq * 2 * kOutBufBytes, t_row, row0, n_blk, lane, out_it);
      else
        epilogue_tile<kEpi>(p, stage, t_row, row0, m128, n_blk, wq, lane, slot, row_end, kSets > 1 ? eset : -1,
                            pitch);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
    }
    if (kEpi != kEpiGateGrad && lane == 0) bulk_wait_all();  // no bulk store still reads shared memory
    if (kEpi == kEpiGateGrad && p.stream_k && lane == 0) {
      // stream-K slots this cluster did not fill read as zero in the reduction
      for (int j = 0; j < 2; ++j) {
        if (sk_written[j]) continue;
        const long long slot = p.sk_base + ((static_cast<long long>(cluster_id) * 2 + j) * 2 + rank) * 4 + wq;
        const int ng = p.gg_groups > 1 ? p.gg_groups : 1;
        for (int k = 0; k < p.cands.K; ++k)
          if (kSets == 1 || ((p.set1_mask >> k) & 1) == eset)
            for (int g = 0; g < ng; ++g) p.partials[(slot * ng + g) * p.cands.K + k] = 0.f;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA frees TMEM while the pair's MMAs or epilogues may still use it
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// grad_p[c / K * ld + c % K] = sum over slots (in slot order) of
// partials[slot][c], c < KK (KK = K, or layers x K for a grouped launch, each
// layer's K gradients written ld floats after the previous layer's), in fp64;
// a slot is one (tile, epilogue warp) pair.  One CTA per value; the
// per-thread strided sums and the tree below have a fixed shape, so the
// result is deterministic.
__global__ void __launch_bounds__(512) gategrad_reduce_kernel(const float* __restrict__ partials, int num_slots,
                                                              int KK, int K, long long ld, float* __restrict__ grad_p) {
  __shared__ double sh[512];
  const int k = blockIdx.x;
  double s = 0.0;
  for (int t = threadIdx.x; t < num_slots; t += blockDim.x)
    s += static_cast<double>(partials[static_cast<long long>(t) * KK + k]);
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) sh[threadIdx.x] += sh[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0) grad_p[(k / K) * ld + k % K] = static_cast<float>(sh[0]);
}

}  // namespace gemm
}  // namespace vq
