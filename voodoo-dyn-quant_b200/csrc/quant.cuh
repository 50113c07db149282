// Q8_0 quantiser on the GPU: float / bf16 weights -> GGUF Q8_0 blocks
// (2-byte fp16 scale d, then 32 int8 codes), byte-identical to ggml's
// reference rule as gguf-py restates it (quants.py Q8_0.quantize_blocks):
//   d  = max|x| / 127            (fp32 division)
//   id = d != 0 ? 1 / d : 0      (fp32 division)
//   q  = round-half-away(x * id) (fp32 product, C roundf)
//   d is stored as fp16, round to nearest even.
// Replaces libggml's quantize_q8_0 behind ggml.quantize_tensor
// (voodoo_quant/ggml.py:171-221), which builds the Q8_0 teacher
// (training/q8_teacher.py) and the Q8_0 candidates on the host.
#pragma once

#include "common.cuh"

namespace vq {
namespace quant {

constexpr int kQ8Threads = 256;

__device__ __forceinline__ float load_f32(const float* p) { return __ldg(p); }
__device__ __forceinline__ float load_f32(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// One warp per 32-element block, lane i owning element i; grid-stride over
// the rows * cols / 32 blocks in row-major order (the GGUF layout).
template <typename T>
__global__ void __launch_bounds__(kQ8Threads) q8_0_quantize_kernel(const T* __restrict__ w, long long rows,
                                                                  long long cols, long long ldw,
                                                                  uint8_t* __restrict__ out) {
  const long long per_row = cols / 32;
  const long long nblk = rows * per_row;
  const int lane = threadIdx.x & 31;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long b = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; b < nblk;
       b += nwarps) {
    const long long r = b / per_row;
    const long long c = (b - r * per_row) * 32 + lane;
    const float x = load_f32(w + r * ldw + c);
    float a = fabsf(x);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    const float d = a / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    const unsigned code = static_cast<uint8_t>(static_cast<int8_t>(static_cast<int>(roundf(x * id))));
    const unsigned bits = __half_raw(__float2half_rn(d)).x;  // every lane holds the same d
    // Byte j of the 34-byte block comes from lane j: the two scale bytes,
    // then the code of lane j - 2; lanes 0 and 1 also write the last two
    // codes.  Every byte is written once by one warp-wide store (coalesced).
    // (A variant where lane 0 stored both scale bytes after its own code
    // byte wrote a wrong low scale byte when built with nvcc 12.9 for sm_100a.)
    const unsigned up = __shfl_up_sync(0xffffffffu, code, 2);
    const unsigned tail = __shfl_sync(0xffffffffu, code, 30 + (lane & 1));
    const unsigned v = lane == 0 ? (bits & 0xffu) : lane == 1 ? (bits >> 8) : up;
    uint8_t* blk = out + b * 34;
    blk[lane] = static_cast<uint8_t>(v);
    if (lane < 2) blk[32 + lane] = static_cast<uint8_t>(tail);
  }
}

}  // namespace quant
}  // namespace vq
