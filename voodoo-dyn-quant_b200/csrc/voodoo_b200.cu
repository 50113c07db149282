// libvoodoo_b200: C-ABI entry points of the B200-native gated-candidate
// training step.  Declarations and the reference interface each one replaces
// are in include/voodoo_b200.h.  Conventions:
//   * every pointer argument is device memory unless documented otherwise;
//   * `stream` is a cudaStream_t (nullptr = legacy default stream);
//   * return 0 on success, a negative VQ_ERR_* code otherwise, with a message
//     available from vq_last_error() (thread-local);
//   * calls are asynchronous, never synchronise (except vq_device_error) and
//     never allocate: workspaces are passed in by the caller.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <atomic>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "formats.cuh"
#include "decode_mix.cuh"
#include "gemm_tc.cuh"
#include "loss.cuh"
#include "blocks.cuh"
#include "quant.cuh"
#include "../../include/voodoo_b200.h"

namespace {

thread_local char g_msg[512] = "ok";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(VQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define VQ_CUDA(call)                                   \
  do {                                                  \
    cudaError_t e_ = (call);                            \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
  } while (0)

__device__ int g_device_error;

int device_error_ptr(int** p) {
  VQ_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(p), g_device_error));
  return 0;
}

// Makes the device that owns `p` current (initialising its primary context on
// this thread, which driver-API calls such as cuTensorMapEncodeTiled need,
// e.g. on autograd worker threads) and restores the caller's device on exit.
class DeviceScope {
 public:
  explicit DeviceScope(const void* p) {
    cudaGetDevice(&prev_);
    int dev = prev_;
    cudaPointerAttributes a;
    if (p != nullptr && cudaPointerGetAttributes(&a, p) == cudaSuccess && a.type == cudaMemoryTypeDevice)
      dev = a.device;
    else
      cudaGetLastError();  // clear a sticky-free error from a host pointer query
    cudaSetDevice(dev);
    changed_ = dev != prev_;
  }
  ~DeviceScope() {
    if (changed_) cudaSetDevice(prev_);
  }

 private:
  int prev_ = 0;
  bool changed_ = false;
};

int sm_count(int* n) {
  int dev = 0;
  VQ_CUDA(cudaGetDevice(&dev));
  VQ_CUDA(cudaDeviceGetAttribute(n, cudaDevAttrMultiProcessorCount, dev));
  return 0;
}

// The driver's cuTensorMapEncodeTiled, looked up on first use (again after a
// failed lookup); an atomic, since calls may come from several threads.
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::atomic<PFN_cuTensorMapEncodeTiled_v12000> fn{nullptr};
  PFN_cuTensorMapEncodeTiled_v12000 f = fn.load(std::memory_order_acquire);
  if (f == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      f = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
      fn.store(f, std::memory_order_release);
    }
  }
  return f;
}

// Row-major bf16 matrix [rows][cols] with leading dimension ld (elements);
// TMA box = 64 columns (one 128-byte swizzle row) x box_rows rows.
int make_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld, int box_rows) {
  auto fn = encode_fn();
  if (fn == nullptr) return fail(VQ_ERR_CUDA, "cuTensorMapEncodeTiled unavailable from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0)
    return fail(VQ_ERR_INVALID, "matrix base pointer must be 16-byte aligned");
  if ((ld * 2) % 16 != 0) return fail(VQ_ERR_INVALID, "leading dimension %lld must be a multiple of 8 elements", ld);
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(VQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return 0;
}

// Output map of the paired store epilogue: bf16 C [rows][cols] (leading
// dimension ld) in 32 x 32 boxes with the 64-byte swizzle.  Returns false,
// and the epilogue stores row by row, where the bulk store cannot address C
// (base not 16-byte aligned, row pitch not a multiple of 16 bytes, C
// narrower or shorter than one box) or the driver declines the map.
bool make_out_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld) {
  auto fn = encode_fn();
  if (fn == nullptr || (reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * 2) % 16 != 0 || rows < 32 ||
      cols < 32)
    return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {32u, 32u};
  cuuint32_t estr[2] = {1u, 1u};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool known_format(int f) { return vq::unit_bytes(f) > 0; }

int build_candset(vq::CandSet* cs, int K, const int* types, const void* const* blocks) {
  if (K < 1 || K > vq::kMaxCandidates) return fail(VQ_ERR_INVALID, "number of candidates %d not in [1, %d]", K, vq::kMaxCandidates);
  if (types == nullptr || blocks == nullptr) return fail(VQ_ERR_INVALID, "null candidate type/pointer array");
  std::memset(cs, 0, sizeof(*cs));
  cs->K = K;
  for (int k = 0; k < K; ++k) {
    if (!known_format(types[k])) return fail(VQ_ERR_UNSUPPORTED, "unsupported ggml type %d for candidate %d", types[k], k);
    if (blocks[k] == nullptr) return fail(VQ_ERR_INVALID, "null block pointer for candidate %d", k);
    if ((reinterpret_cast<uintptr_t>(blocks[k]) & 1u) != 0)
      return fail(VQ_ERR_INVALID, "candidate %d blocks must be 2-byte aligned", k);
    cs->fmt[k] = types[k];
    cs->ubytes[k] = vq::unit_bytes(types[k]);
    cs->ptr[k] = static_cast<const uint8_t*>(blocks[k]);
  }
  return 0;
}

// Output rows are tiled by 256 on a CTA pair (tcgen05 cta_group::2) when M >
// 128, else by 128 on single CTAs.  `pair` reports the choice (the tensor
// map box of a K-major B operand and the gate-gradient slot count depend on it).
inline bool use_pair(long long M) { return M > vq::gemm::BM; }
// The gate-gradient GEMM always runs on CTA pairs: its stream-K split (the
// paired kernel's) then spreads even a few row blocks over every SM, where
// a 1-CTA launch of a 128-row layer (a KV projection's TP shard) would keep
// one SM per 256 columns busy.
inline bool gategrad_pair(long long) { return true; }

// Upper bound on CTA pairs of a paired launch (the stream-K partial slots of
// the gate-gradient workspace are sized for it).
constexpr int kMaxClusters = 128;

// SMs the gate-gradient GEMM leaves free (vq_set_gategrad_sm_reserve), for a
// collective that runs concurrently on another stream.
std::atomic<int> g_gategrad_sm_reserve{0};
// SMs the store-epilogue GEMMs (forward, dX) leave free (vq_set_gemm_sm_reserve).
std::atomic<int> g_gemm_sm_reserve{0};

inline int sm_reserve(int epi, int sms) {
  const int r = epi == vq::gemm::kEpiGateGrad   ? g_gategrad_sm_reserve.load(std::memory_order_relaxed)
                : epi == vq::gemm::kEpiStoreBf16 ? g_gemm_sm_reserve.load(std::memory_order_relaxed)
                                                 : 0;
  return r > 0 && r < sms - 2 ? r : 0;
}

// Gate-gradient partial slots the per-tile schedule writes.
inline long long gategrad_tile_slots(long long N, long long Kin) {
  const long long m128 = gategrad_pair(N) ? 2 * ((N + 255) / 256) : (N + vq::gemm::BM - 1) / vq::gemm::BM;
  return m128 * ((Kin + vq::gemm::BN - 1) / vq::gemm::BN) * 4;
}

// `used_slots` (gate-gradient launches): partial slots the launch writes.
template <bool kAmn, bool kBmn, int kEpi>
int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, vq::gemm::Params p, cudaStream_t st,
                long long* used_slots = nullptr) {
  using namespace vq::gemm;
  const bool pair = kEpi == vq::gemm::kEpiGateGrad ? gategrad_pair(p.M) : use_pair(p.M);
  p.num_m_blk = pair ? (p.M + 255) / 256 : (p.M + BM - 1) / BM;
  p.num_n_blk = (p.N + BN - 1) / BN;
  p.num_k_blk = (p.K + BK - 1) / BK;
  p.num_tiles = p.num_m_blk * p.num_n_blk;
  p.stream_k = 0;
  p.sk_base = 0;
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  if (used_slots != nullptr) *used_slots = gategrad_tile_slots(p.M, p.N);
  if (pair) {
    auto kern = gemm_pair_kernel<kAmn, kBmn, kEpi>;
    constexpr int smem = PairSmemLayout<kEpi>::total;
    VQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int avail = sms - sm_reserve(kEpi, sms);
    int clusters = p.num_tiles < avail / 2 ? p.num_tiles : avail / 2;
    // At most half as many gate-gradient tiles as pairs: split them all along
    // K over every pair (each piece decodes its tile's candidates again, so
    // a split pays only where it at least doubles the pairs at work).
    if (kEpi == kEpiGateGrad && 2 * p.num_tiles <= avail / 2) clusters = avail / 2;
    if (clusters > kMaxClusters) clusters = kMaxClusters;
    if (kEpi == kEpiGateGrad && p.num_tiles % clusters != 0 && (p.num_tiles > clusters || 2 * p.num_tiles <= clusters)) {
      // split the last, partial wave of tiles (or all of them) along K across every cluster
      p.stream_k = 1;
      p.sk_base = static_cast<int>(gategrad_tile_slots(p.M, p.N));
      if (used_slots != nullptr) *used_slots += 16LL * clusters;
    }
    BMaps<1> bm{};
    bm.m[0] = tb;
    p.tma_store = kEpi == kEpiStoreBf16 && make_out_map(&bm.c, p.C, p.M, p.N, p.ldc);
    kern<<<2 * clusters, PairCfg<kEpi>::kThreads, smem, st>>>(ta, bm, p);
  } else {
    auto kern = gemm_kernel<kAmn, kBmn, kEpi>;
    constexpr int smem = SmemLayout<kEpi>::total;
    VQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int avail = sms - sm_reserve(kEpi, sms);
    const int grid = p.num_tiles < avail ? p.num_tiles : avail;
    kern<<<grid, THREADS, smem, st>>>(ta, tb, p);
  }
  VQ_CUDA(cudaGetLastError());
  return 0;
}

// Candidates of the second gate-gradient epilogue set (bit k): greedy split
// by staged unit bytes plus a fixed per-candidate cost, largest first, with
// Q8_0 (too wide for the second set's staging rows) always in the first set.
inline int gategrad_set_split(int K, const int* types) {
  int order[8], cost[8];
  for (int k = 0; k < K; ++k) {
    order[k] = k;
    cost[k] = vq::unit_bytes(types[k]) + 96;
  }
  for (int i = 1; i < K; ++i)  // stable insertion sort by descending cost
    for (int j = i; j > 0 && cost[order[j]] > cost[order[j - 1]]; --j) {
      const int t = order[j];
      order[j] = order[j - 1];
      order[j - 1] = t;
    }
  int load[2] = {0, 0}, mask = 0;
  for (int i = 0; i < K; ++i) {
    const int k = order[i];
    const int set = (types[k] == vq::kQ8_0 || load[0] <= load[1]) ? 0 : 1;
    load[set] += cost[k];
    if (set) mask |= 1 << k;
  }
  return mask;
}

// Gate-gradient partial slots a workspace must hold: the per-tile slots plus,
// for paired launches, the stream-K slots (16 per cluster).
inline long long gategrad_slots(long long N, long long Kin) {
  return gategrad_tile_slots(N, Kin) + (gategrad_pair(N) ? 16LL * kMaxClusters : 0);
}

int check_matrix(const void* p, long long rows, long long cols, long long ld, const char* name) {
  if (rows < 0 || cols < 0) return fail(VQ_ERR_INVALID, "%s: negative shape", name);
  if (ld < cols) return fail(VQ_ERR_INVALID, "%s: leading dimension %lld < columns %lld", name, ld, cols);
  if (rows > 0 && cols > 0 && p == nullptr) return fail(VQ_ERR_INVALID, "%s: null pointer", name);
  return 0;
}

int zero_rows(void* p, long long rows, long long cols, long long ld, size_t elem, cudaStream_t st) {
  if (rows == 0 || cols == 0) return 0;
  VQ_CUDA(cudaMemset2DAsync(p, ld * elem, 0, cols * elem, rows, st));
  return 0;
}

// Scratch of vq_gategrad_noalloc, for callers that cannot allocate device
// memory (a plain C-FFI host without a device allocator, or a process whose
// memory pool owns the device).  Every GPU that loads this library holds it
// until exit.  In host code `g_gategrad_scratch` is only a stand-in symbol:
// its device address comes from cudaGetSymbolAddress, per device.
static __device__ __align__(256) float g_gategrad_scratch[VQ_GATEGRAD_NOALLOC_SCRATCH_BYTES / sizeof(float)];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch on the current device, looked up once per
// device (the first call on a device must come before any stream capture).
int noalloc_scratch(void** out) {
  int dev = 0;
  VQ_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(VQ_ERR_INVALID, "device ordinal %d beyond %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_gategrad_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(gate-grad scratch)");
    if (ptr == nullptr || reinterpret_cast<uintptr_t>(ptr) % 256 != 0)
      return fail(VQ_ERR_CUDA, "gate-grad scratch address %p is not 256-byte aligned", ptr);
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return 0;
}

}  // namespace

extern "C" {

const char* vq_last_error(void) { return g_msg; }

int vq_abi_version(void) { return VQ_ABI_VERSION; }

int vq_format_info(int ggml_type, int* block_elems, int* block_bytes) {
  if (!known_format(ggml_type)) return fail(VQ_ERR_UNSUPPORTED, "unsupported ggml type %d", ggml_type);
  if (block_elems) *block_elems = vq::block_elems(ggml_type);
  if (block_bytes) *block_bytes = vq::block_bytes(ggml_type);
  return 0;
}

int vq_device_error(void* stream, int* code) {
  DeviceScope scope(nullptr);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* dp = nullptr;
  if (int rc = device_error_ptr(&dp)) return rc;
  int h = 0;
  VQ_CUDA(cudaMemcpyAsync(&h, dp, sizeof(int), cudaMemcpyDeviceToHost, st));
  VQ_CUDA(cudaStreamSynchronize(st));
  VQ_CUDA(cudaMemsetAsync(dp, 0, sizeof(int), st));
  VQ_CUDA(cudaStreamSynchronize(st));
  if (code) *code = h;
  return 0;
}

int vq_dequant(int ggml_type, const void* blocks, int64_t rows, int64_t cols, float* out, void* stream) {
  DeviceScope scope(out);
  if (!known_format(ggml_type)) return fail(VQ_ERR_UNSUPPORTED, "unsupported ggml type %d", ggml_type);
  const int bs = vq::block_elems(ggml_type);
  if (rows < 0 || cols < 0) return fail(VQ_ERR_INVALID, "negative shape");
  if (cols % bs != 0) return fail(VQ_ERR_INVALID, "requires in_features %% %d == 0, got %lld", bs, (long long)cols);
  const long long total = static_cast<long long>(rows) * cols;
  if (total == 0) return 0;
  if (blocks == nullptr || out == nullptr) return fail(VQ_ERR_INVALID, "null pointer");
  vq::CandSet cs;
  const void* bl[1] = {blocks};
  if (int rc = build_candset(&cs, 1, &ggml_type, bl)) return rc;
  int* err = nullptr;
  if (int rc = device_error_ptr(&err)) return rc;
  const long long units = (total + 255) / 256;
  const long long grid = (units + vq::kDequantUnits - 1) / vq::kDequantUnits;
  if (grid > 0x7fffffffLL) return fail(VQ_ERR_INVALID, "tensor too large");
  vq::dequant_units_kernel<<<static_cast<unsigned>(grid), vq::kDecodeThreads,
                             vq::stage_smem_bytes(cs, vq::kDequantUnits), static_cast<cudaStream_t>(stream)>>>(
      cs, total, out, err);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_mix(int K, const int* types, const void* const* blocks, const float* probs, int64_t rows, int64_t padded_cols,
           int64_t cols, void* w_bf16, int64_t ldw, void* stream) {
  DeviceScope scope(w_bf16);
  vq::CandSet cs;
  if (int rc = build_candset(&cs, K, types, blocks)) return rc;
  if (rows < 0 || cols < 0 || padded_cols < cols) return fail(VQ_ERR_INVALID, "invalid shape");
  if (padded_cols % 256 != 0) return fail(VQ_ERR_INVALID, "padded in_features %lld must be a multiple of 256", (long long)padded_cols);
  if (ldw < cols || ldw > padded_cols) return fail(VQ_ERR_INVALID, "ldw %lld must be in [cols, padded_cols]", (long long)ldw);
  if (rows == 0 || padded_cols == 0) return 0;
  if (probs == nullptr || w_bf16 == nullptr) return fail(VQ_ERR_INVALID, "null pointer");
  int* err = nullptr;
  if (int rc = device_error_ptr(&err)) return rc;
  if (cols > 0x7fffffffLL) return fail(VQ_ERR_INVALID, "too many columns");
  const long long units = static_cast<long long>(rows) * (padded_cols / 256);
  const long long nblocks = (units + vq::kMixUnits - 1) / vq::kMixUnits;
  // Persistent CTAs, as many per SM as fit, each walking blocks of
  // kMixUnits units with kMixStages bulk-copy stages in flight.
  const int stage = vq::mix_stage_bytes(cs);
  const int smem = vq::kMixStages * stage;
  if (smem > 48 * 1024) VQ_CUDA(cudaFuncSetAttribute(vq::mix_units_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  int per_sm = 0;
  VQ_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, vq::mix_units_kernel, vq::kDecodeThreads, smem));
  if (per_sm < 1) return fail(VQ_ERR_INVALID, "mixture of %d candidates does not fit one SM", K);
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  const long long grid = std::min<long long>(nblocks, static_cast<long long>(sms) * per_sm);
  vq::mix_units_kernel<<<static_cast<unsigned>(grid), vq::kDecodeThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      cs, probs, units, static_cast<int>(padded_cols / 256), static_cast<int>(cols),
      static_cast<__nv_bfloat16*>(w_bf16), ldw, stage, err);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_linear_fwd(const void* x, int64_t T, int64_t Kin, int64_t ldx, const void* w, int64_t N, int64_t ldw, void* y,
                  int64_t ldy, void* stream) {
  DeviceScope scope(y);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_matrix(x, T, Kin, ldx, "x")) return rc;
  if (int rc = check_matrix(w, N, Kin, ldw, "w")) return rc;
  if (int rc = check_matrix(y, T, N, ldy, "y")) return rc;
  if (T == 0 || N == 0) return 0;
  if (Kin == 0) return zero_rows(y, T, N, ldy, 2, st);
  if (T > 0x7fffffff || N > 0x7fffffff || Kin > 0x7fffffff) return fail(VQ_ERR_INVALID, "dimension too large");
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, x, T, Kin, ldx, vq::gemm::BM)) return rc;
  if (int rc = make_map(&tb, w, N, Kin, ldw, use_pair(T) ? 128 : vq::gemm::BN)) return rc;
  vq::gemm::Params p{};
  p.M = static_cast<int>(T);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(Kin);
  p.C = static_cast<__nv_bfloat16*>(y);
  p.ldc = ldy;
  if (int rc = device_error_ptr(&p.err)) return rc;
  return launch_gemm<false, false, vq::gemm::kEpiStoreBf16>(ta, tb, p, st);
}

int vq_linear_dx(const void* dy, int64_t T, int64_t N, int64_t lddy, const void* w, int64_t Kin, int64_t ldw, void* dx,
                 int64_t lddx, void* stream) {
  DeviceScope scope(dx);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_matrix(dy, T, N, lddy, "dy")) return rc;
  if (int rc = check_matrix(w, N, Kin, ldw, "w")) return rc;
  if (int rc = check_matrix(dx, T, Kin, lddx, "dx")) return rc;
  if (T == 0 || Kin == 0) return 0;
  if (N == 0) return zero_rows(dx, T, Kin, lddx, 2, st);
  if (T > 0x7fffffff || N > 0x7fffffff || Kin > 0x7fffffff) return fail(VQ_ERR_INVALID, "dimension too large");
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, dy, T, N, lddy, vq::gemm::BM)) return rc;
  if (int rc = make_map(&tb, w, N, Kin, ldw, 64)) return rc;
  vq::gemm::Params p{};
  p.M = static_cast<int>(T);
  p.N = static_cast<int>(Kin);
  p.K = static_cast<int>(N);
  p.C = static_cast<__nv_bfloat16*>(dx);
  p.ldc = lddx;
  if (int rc = device_error_ptr(&p.err)) return rc;
  return launch_gemm<false, true, vq::gemm::kEpiStoreBf16>(ta, tb, p, st);
}

int vq_linear_fwd_swiglu(const void* x, int64_t T, int64_t Kin, int64_t ldx, const void* w, int64_t F, int64_t ldw,
                         void* h, int64_t ldh, void* stream) {
  DeviceScope scope(h);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_matrix(x, T, Kin, ldx, "x")) return rc;
  if (int rc = check_matrix(w, 2 * F, Kin, ldw, "w")) return rc;
  if (int rc = check_matrix(h, T, F, ldh, "h")) return rc;
  if (T == 0 || F == 0) return 0;
  if (Kin == 0) return zero_rows(h, T, F, ldh, 2, st);
  if (T > 0x7fffffff || 2 * F > 0x7fffffff || Kin > 0x7fffffff) return fail(VQ_ERR_INVALID, "dimension too large");
  if (!use_pair(T) || F % 128 != 0)
    return fail(VQ_ERR_UNSUPPORTED, "fused SwiGLU GEMM needs more than %d rows and a multiple of 128 features",
                vq::gemm::BM);
  using namespace vq::gemm;
  CUtensorMap ta;
  BMaps<1> bm{};
  if (int rc = make_map(&ta, x, T, Kin, ldx, BM)) return rc;
  if (int rc = make_map(&bm.m[0], w, 2 * F, Kin, ldw, 128)) return rc;
  Params p{};
  p.M = static_cast<int>(T);
  p.N = static_cast<int>(F);
  p.K = static_cast<int>(Kin);
  p.C = static_cast<__nv_bfloat16*>(h);
  p.ldc = ldh;
  p.up_row = static_cast<int>(F);
  p.num_m_blk = static_cast<int>((T + 255) / 256);
  p.num_n_blk = static_cast<int>(F / 128);
  p.num_k_blk = static_cast<int>((Kin + BK - 1) / BK);
  p.num_tiles = p.num_m_blk * p.num_n_blk;
  p.tma_store = make_out_map(&bm.c, h, T, F, ldh);
  if (int rc = device_error_ptr(&p.err)) return rc;
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  auto kern = gemm_pair_kernel<false, false, kEpiSwiGLU>;
  constexpr int smem = PairSmemLayout<kEpiSwiGLU>::total;
  VQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int avail = sms - sm_reserve(kEpiStoreBf16, sms);
  int clusters = p.num_tiles < avail / 2 ? p.num_tiles : avail / 2;
  if (clusters > kMaxClusters) clusters = kMaxClusters;
  kern<<<2 * clusters, PairCfg<kEpiSwiGLU>::kThreads, smem, st>>>(ta, bm, p);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_linear_fwd_grouped(const void* x, int64_t T, int64_t Kin, int64_t ldx, int G, const void* const* w,
                          int64_t N, int64_t ldw, const int* group_off, void* y, int64_t ldy, void* stream) {
  DeviceScope scope(y);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (G < 1 || G > vq::gemm::kMaxGroups) return fail(VQ_ERR_INVALID, "groups %d not in [1, %d]", G, vq::gemm::kMaxGroups);
  if (w == nullptr || group_off == nullptr) return fail(VQ_ERR_INVALID, "null weight array or group offsets");
  if (int rc = check_matrix(x, T, Kin, ldx, "x")) return rc;
  if (int rc = check_matrix(y, T, N, ldy, "y")) return rc;
  for (int g = 0; g < G; ++g)
    if (int rc = check_matrix(w[g], N, Kin, ldw, "w")) return rc;
  if (T == 0 || N == 0) return 0;
  if (Kin == 0) return zero_rows(y, T, N, ldy, 2, st);
  if (T > 0x7fffffff || N > 0x7fffffff || Kin > 0x7fffffff) return fail(VQ_ERR_INVALID, "dimension too large");
  if (!use_pair(T)) return fail(VQ_ERR_INVALID, "grouped GEMM needs more than %d rows", vq::gemm::BM);
  CUtensorMap ta;
  vq::gemm::BMaps<vq::gemm::kMaxGroups> bm{};
  if (int rc = make_map(&ta, x, T, Kin, ldx, vq::gemm::BM)) return rc;
  for (int g = 0; g < G; ++g)
    if (int rc = make_map(&bm.m[g], w[g], N, Kin, ldw, 128)) return rc;
  vq::gemm::Params p{};
  p.M = static_cast<int>(T);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(Kin);
  p.C = static_cast<__nv_bfloat16*>(y);
  p.ldc = ldy;
  p.group_off = group_off;
  p.ngroups = G;
  p.num_n_blk = static_cast<int>((N + vq::gemm::BN - 1) / vq::gemm::BN);
  p.num_k_blk = static_cast<int>((Kin + vq::gemm::BK - 1) / vq::gemm::BK);
  p.num_m_blk = static_cast<int>((T + 255) / 256) + G;  // upper bound on the groups' 256-row tiles
  p.num_tiles = p.num_m_blk * p.num_n_blk;              // the kernel counts the exact tiles itself
  p.tma_store = make_out_map(&bm.c, y, T, N, ldy);
  if (int rc = device_error_ptr(&p.err)) return rc;
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  auto kern = vq::gemm::gemm_pair_kernel<false, false, vq::gemm::kEpiStoreBf16, vq::gemm::kMaxGroups>;
  constexpr int smem = vq::gemm::PairSmemLayout<vq::gemm::kEpiStoreBf16>::total;
  VQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int clusters = p.num_tiles < sms / 2 ? p.num_tiles : sms / 2;
  kern<<<2 * clusters, vq::gemm::PairCfg<vq::gemm::kEpiStoreBf16>::kThreads, smem, st>>>(ta, bm, p);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_set_gategrad_sm_reserve(int sms) {
  if (sms < 0) return fail(VQ_ERR_INVALID, "negative SM count");
  g_gategrad_sm_reserve.store(sms, std::memory_order_relaxed);
  return 0;
}

int vq_set_gemm_sm_reserve(int sms) {
  if (sms < 0) return fail(VQ_ERR_INVALID, "negative SM count");
  g_gemm_sm_reserve.store(sms, std::memory_order_relaxed);
  return 0;
}

size_t vq_gategrad_workspace_bytes(int64_t N, int64_t Kin, int K) {
  if (N <= 0 || Kin <= 0 || K <= 0) return 0;
  return static_cast<size_t>(gategrad_slots(N, Kin)) * K * sizeof(float);
}

int vq_gategrad(const void* dy, int64_t lddy, const void* x, int64_t ldx, int64_t T, int64_t N, int64_t Kin, int K,
                const int* types, const void* const* blocks, int64_t padded_cols, void* workspace,
                size_t workspace_bytes, float* grad_probs, void* stream) {
  DeviceScope scope(grad_probs);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  vq::CandSet cs;
  if (int rc = build_candset(&cs, K, types, blocks)) return rc;
  if (int rc = check_matrix(dy, T, N, lddy, "dy")) return rc;
  if (int rc = check_matrix(x, T, Kin, ldx, "x")) return rc;
  if (grad_probs == nullptr) return fail(VQ_ERR_INVALID, "null grad_probs");
  if (padded_cols < Kin || padded_cols % 256 != 0)
    return fail(VQ_ERR_INVALID, "padded in_features %lld must be a multiple of 256 and >= %lld", (long long)padded_cols,
                (long long)Kin);
  if (T == 0 || N == 0 || Kin == 0) {
    VQ_CUDA(cudaMemsetAsync(grad_probs, 0, sizeof(float) * K, st));
    return 0;
  }
  if (T > 0x7fffffff || N > 0x7fffffff || Kin > 0x7fffffff) return fail(VQ_ERR_INVALID, "dimension too large");
  const size_t need = vq_gategrad_workspace_bytes(N, Kin, K);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(VQ_ERR_INVALID, "gate-grad workspace of %zu bytes required, got %zu", need, workspace_bytes);
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, dy, T, N, lddy, 64)) return rc;
  if (int rc = make_map(&tb, x, T, Kin, ldx, 64)) return rc;
  vq::gemm::Params p{};
  p.M = static_cast<int>(N);
  p.N = static_cast<int>(Kin);
  p.K = static_cast<int>(T);
  p.cands = cs;
  p.units_per_row = static_cast<int>(padded_cols / 256);
  p.cols = Kin;
  p.partials = static_cast<float*>(workspace);
  p.set1_mask = gategrad_set_split(K, types);
  if (int rc = device_error_ptr(&p.err)) return rc;
  long long used = 0;
  if (int rc = launch_gemm<true, true, vq::gemm::kEpiGateGrad>(ta, tb, p, st, &used)) return rc;
  const int slots = static_cast<int>(used);
  vq::gemm::gategrad_reduce_kernel<<<K, 512, 0, st>>>(p.partials, slots, K, K, K, grad_probs);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

size_t vq_gategrad_grouped_workspace_bytes(int64_t N_total, int64_t Kin, int G, int K) {
  if (N_total <= 0 || Kin <= 0 || G <= 0 || K <= 0) return 0;
  return static_cast<size_t>(gategrad_slots(N_total, Kin)) * G * K * sizeof(float);
}

int vq_gategrad_grouped(const void* dy, int64_t lddy, const void* x, int64_t ldx, int64_t T, int G,
                        const int64_t* rows, int64_t Kin, int K, const int* types, const void* const* blocks,
                        int64_t padded_cols, void* workspace, size_t workspace_bytes, float* grad_probs,
                        int64_t ld_grad, void* stream) {
  DeviceScope scope(grad_probs);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  using vq::gemm::kMaxGGroups;
  if (G < 1 || G > kMaxGGroups) return fail(VQ_ERR_INVALID, "layers %d not in [1, %d]", G, kMaxGGroups);
  if (rows == nullptr || blocks == nullptr) return fail(VQ_ERR_INVALID, "null row-count or block array");
  if (grad_probs == nullptr) return fail(VQ_ERR_INVALID, "null grad_probs");
  if (ld_grad < K) return fail(VQ_ERR_INVALID, "grad_probs row stride %lld < K = %d", (long long)ld_grad, K);
  vq::CandSet cs;
  if (int rc = build_candset(&cs, K, types, blocks)) return rc;
  int64_t N = 0;
  for (int g = 0; g < G; ++g) {
    if (rows[g] <= 0 || rows[g] % 32 != 0)
      return fail(VQ_ERR_INVALID, "layer %d: %lld rows, not a positive multiple of 32", g, (long long)rows[g]);
    vq::CandSet cg;
    if (int rc = build_candset(&cg, K, types, blocks + static_cast<size_t>(g) * K)) return rc;
    N += rows[g];
  }
  if (int rc = check_matrix(dy, T, N, lddy, "dy")) return rc;
  if (int rc = check_matrix(x, T, Kin, ldx, "x")) return rc;
  if (padded_cols < Kin || padded_cols % 256 != 0)
    return fail(VQ_ERR_INVALID, "padded in_features %lld must be a multiple of 256 and >= %lld", (long long)padded_cols,
                (long long)Kin);
  if (T == 0 || Kin == 0) {
    for (int g = 0; g < G; ++g) VQ_CUDA(cudaMemsetAsync(grad_probs + g * ld_grad, 0, sizeof(float) * K, st));
    return 0;
  }
  if (T > 0x7fffffff || N > 0x7fffffff || Kin > 0x7fffffff) return fail(VQ_ERR_INVALID, "dimension too large");
  const size_t need = vq_gategrad_grouped_workspace_bytes(N, Kin, G, K);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(VQ_ERR_INVALID, "grouped gate-grad workspace of %zu bytes required, got %zu", need, workspace_bytes);
  CUtensorMap ta, tb;
  if (int rc = make_map(&ta, dy, T, N, lddy, 64)) return rc;
  if (int rc = make_map(&tb, x, T, Kin, ldx, 64)) return rc;
  vq::gemm::Params p{};
  p.M = static_cast<int>(N);
  p.N = static_cast<int>(Kin);
  p.K = static_cast<int>(T);
  p.cands = cs;
  p.units_per_row = static_cast<int>(padded_cols / 256);
  p.cols = Kin;
  p.partials = static_cast<float*>(workspace);
  p.set1_mask = gategrad_set_split(K, types);
  p.gg_groups = G;
  p.gg_row[0] = 0;
  for (int g = 0; g < G; ++g) {
    p.gg_row[g + 1] = p.gg_row[g] + static_cast<int>(rows[g]);
    for (int k = 0; k < K; ++k) p.gg_ptr[g][k] = static_cast<const uint8_t*>(blocks[static_cast<size_t>(g) * K + k]);
  }
  if (int rc = device_error_ptr(&p.err)) return rc;
  long long used = 0;
  if (int rc = launch_gemm<true, true, vq::gemm::kEpiGateGrad>(ta, tb, p, st, &used)) return rc;
  vq::gemm::gategrad_reduce_kernel<<<G * K, 512, 0, st>>>(p.partials, static_cast<int>(used), G * K, K, ld_grad,
                                                          grad_probs);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_gategrad_noalloc(const void* dy, int64_t lddy, const void* x, int64_t ldx, int64_t T, int64_t N, int64_t Kin,
                        int K, const int* types, const void* const* blocks, int64_t padded_cols, float* grad_probs,
                        void* stream) {
  const size_t need = vq_gategrad_workspace_bytes(N, Kin, K);
  if (need > VQ_GATEGRAD_NOALLOC_SCRATCH_BYTES)
    return fail(VQ_ERR_INVALID,
                "gate-grad of a %lld x %lld layer with %d candidates needs %zu bytes of scratch; "
                "vq_gategrad_noalloc holds %zu (use vq_gategrad with a caller workspace)",
                (long long)N, (long long)Kin, K, need, (size_t)VQ_GATEGRAD_NOALLOC_SCRATCH_BYTES);
  if (grad_probs == nullptr) return fail(VQ_ERR_INVALID, "null grad_probs");
  DeviceScope scope(grad_probs);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  return vq_gategrad(dy, lddy, x, ldx, T, N, Kin, K, types, blocks, padded_cols, scratch,
                     VQ_GATEGRAD_NOALLOC_SCRATCH_BYTES, grad_probs, stream);
}

int vq_mixgemm_fwd(const void* x, int64_t T, int64_t Kin, int64_t ldx, int K, const int* types,
                   const void* const* blocks, const float* probs, int64_t N, int64_t padded_cols, void* w_mix,
                   int64_t ldw, void* y, int64_t ldy, void* stream) {
  if (int rc = vq_mix(K, types, blocks, probs, N, padded_cols, Kin, w_mix, ldw, stream)) return rc;
  return vq_linear_fwd(x, T, Kin, ldx, w_mix, N, ldw, y, ldy, stream);
}

int vq_mixgemm_fwd_fused(const void* x, int64_t T, int64_t Kin, int64_t ldx, int K, const int* types,
                         const void* const* blocks, const float* probs, int64_t N, int64_t padded_cols, void* y,
                         int64_t ldy, void* stream) {
  DeviceScope scope(y);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  vq::CandSet cs;
  if (int rc = build_candset(&cs, K, types, blocks)) return rc;
  if (probs == nullptr) return fail(VQ_ERR_INVALID, "null probs");
  if (int rc = check_matrix(x, T, Kin, ldx, "x")) return rc;
  if (int rc = check_matrix(y, T, N, ldy, "y")) return rc;
  if (padded_cols < Kin || padded_cols % 256 != 0)
    return fail(VQ_ERR_INVALID, "padded in_features %lld must be a multiple of 256 and >= %lld", (long long)padded_cols,
                (long long)Kin);
  if (T == 0 || N == 0) return 0;
  if (Kin == 0) return zero_rows(y, T, N, ldy, 2, st);
  if (T > 0x7fffffff || N > 0x7fffffff || Kin > 0x7fffffff) return fail(VQ_ERR_INVALID, "dimension too large");
  if (!use_pair(T)) return fail(VQ_ERR_UNSUPPORTED, "decoded-operand GEMM needs more than %d rows", vq::gemm::BM);
  using namespace vq::gemm;
  CUtensorMap ta;
  BMaps<1> bm{};
  if (int rc = make_map(&ta, x, T, Kin, ldx, BM)) return rc;
  Params p{};
  p.M = static_cast<int>(T);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(Kin);
  p.C = static_cast<__nv_bfloat16*>(y);
  p.ldc = ldy;
  p.cands = cs;
  p.units_per_row = static_cast<int>(padded_cols / 256);
  p.cols = Kin;
  p.mix_probs = probs;
  p.num_m_blk = static_cast<int>((T + 255) / 256);
  p.num_n_blk = static_cast<int>((N + BN - 1) / BN);
  p.num_k_blk = static_cast<int>((Kin + BK - 1) / BK);
  p.num_tiles = p.num_m_blk * p.num_n_blk;
  p.tma_store = make_out_map(&bm.c, y, T, N, ldy);
  if (int rc = device_error_ptr(&p.err)) return rc;
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  auto kern = gemm_pair_kernel<false, false, kEpiStoreBf16, 1, true>;
  constexpr int smem = PairSmemLayout<kEpiStoreBf16, true>::total;
  static_assert(smem <= 232448, "decoded-operand GEMM shared memory above the 227 KB per-block limit");
  VQ_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int avail = sms - sm_reserve(kEpiStoreBf16, sms);
  int clusters = p.num_tiles < avail / 2 ? p.num_tiles : avail / 2;
  if (clusters > kMaxClusters) clusters = kMaxClusters;
  kern<<<2 * clusters, PairCfg<kEpiStoreBf16>::kThreads + 128, smem, st>>>(ta, bm, p);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_mixgemm_dx(const void* dy, int64_t T, int64_t N, int64_t lddy, int K, const int* types,
                  const void* const* blocks, const float* probs, int64_t Kin, int64_t padded_cols, void* w_mix,
                  int64_t ldw, void* dx, int64_t lddx, void* stream) {
  if (int rc = vq_mix(K, types, blocks, probs, N, padded_cols, Kin, w_mix, ldw, stream)) return rc;
  return vq_linear_dx(dy, T, N, lddy, w_mix, Kin, ldw, dx, lddx, stream);
}

int vq_loss_fused(const void* s_logits, int64_t lds, const void* t_logits, int64_t ldt, const int64_t* targets,
                  int64_t rows, int64_t V, float temperature, float ce_weight, float kl_weight, float* row_ce,
                  float* row_kl, void* dlogits, int64_t ldg, void* stream) {
  DeviceScope scope(row_ce);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_matrix(s_logits, rows, V, lds, "student logits")) return rc;
  if (int rc = check_matrix(t_logits, rows, V, ldt, "teacher logits")) return rc;
  if (dlogits != nullptr) {
    if (int rc = check_matrix(dlogits, rows, V, ldg, "dlogits")) return rc;
  }
  if (!(temperature > 0.f)) return fail(VQ_ERR_INVALID, "temperature must be > 0");
  if (rows == 0) return 0;
  if (V <= 0 || V > 0x7fffffff || rows > 0x7fffffff) return fail(VQ_ERR_INVALID, "invalid vocabulary size");
  if (targets == nullptr || row_ce == nullptr || row_kl == nullptr) return fail(VQ_ERR_INVALID, "null pointer");
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  const int grid = static_cast<int>(rows < sms ? rows : sms);
  const bool vec = ((reinterpret_cast<uintptr_t>(s_logits) | reinterpret_cast<uintptr_t>(t_logits) |
                     reinterpret_cast<uintptr_t>(dlogits)) & 15u) == 0 &&
                   lds % 8 == 0 && ldt % 8 == 0 && (dlogits == nullptr || ldg % 8 == 0);
  const auto* S = static_cast<const __nv_bfloat16*>(s_logits);
  const auto* Tl = static_cast<const __nv_bfloat16*>(t_logits);
  auto* G = static_cast<__nv_bfloat16*>(dlogits);
  const auto* y = reinterpret_cast<const long long*>(targets);
  if (temperature == 1.0f)
    vq::loss::loss_fused_kernel<true><<<grid, vq::loss::THREADS, 0, st>>>(S, lds, Tl, ldt, y, (int)rows, (int)V, temperature,
                                                                          ce_weight, kl_weight, row_ce, row_kl, G, ldg, vec);
  else
    vq::loss::loss_fused_kernel<false><<<grid, vq::loss::THREADS, 0, st>>>(S, lds, Tl, ldt, y, (int)rows, (int)V, temperature,
                                                                           ce_weight, kl_weight, row_ce, row_kl, G, ldg, vec);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_loss_stats(const void* s_logits, int64_t lds, const void* t_logits, int64_t ldt, const int64_t* targets,
                  int64_t vocab_start, int64_t rows, int64_t V, float temperature, float* stats, void* stream) {
  DeviceScope scope(stats);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_matrix(s_logits, rows, V, lds, "student logits")) return rc;
  if (int rc = check_matrix(t_logits, rows, V, ldt, "teacher logits")) return rc;
  if (!(temperature > 0.f)) return fail(VQ_ERR_INVALID, "temperature must be > 0");
  if (rows == 0) return 0;
  if (V <= 0 || V > 0x7fffffff || rows > 0x7fffffff) return fail(VQ_ERR_INVALID, "invalid vocabulary size");
  if (targets == nullptr || stats == nullptr) return fail(VQ_ERR_INVALID, "null pointer");
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  const int grid = static_cast<int>(rows < sms ? rows : sms);
  const bool vec = ((reinterpret_cast<uintptr_t>(s_logits) | reinterpret_cast<uintptr_t>(t_logits)) & 15u) == 0 &&
                   lds % 8 == 0 && ldt % 8 == 0;
  const auto* S = static_cast<const __nv_bfloat16*>(s_logits);
  const auto* Tl = static_cast<const __nv_bfloat16*>(t_logits);
  const auto* y = reinterpret_cast<const long long*>(targets);
  if (temperature == 1.0f)
    vq::loss::loss_stats_kernel<true><<<grid, vq::loss::THREADS, 0, st>>>(S, lds, Tl, ldt, y, vocab_start, (int)rows,
                                                                          (int)V, temperature, stats, vec);
  else
    vq::loss::loss_stats_kernel<false><<<grid, vq::loss::THREADS, 0, st>>>(S, lds, Tl, ldt, y, vocab_start, (int)rows,
                                                                           (int)V, temperature, stats, vec);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_loss_combine(const float* stats, int ranks, int64_t rows, float temperature, float* row_lse, float* row_ce,
                    float* row_kl, void* stream) {
  DeviceScope scope(row_ce);
  if (ranks < 1) return fail(VQ_ERR_INVALID, "ranks must be >= 1");
  if (rows < 0 || rows > 0x7fffffff) return fail(VQ_ERR_INVALID, "invalid row count");
  if (rows == 0) return 0;
  if (!stats || !row_lse || !row_ce || !row_kl) return fail(VQ_ERR_INVALID, "null pointer");
  const int threads = 256;
  const int grid = static_cast<int>((rows + threads - 1) / threads);
  vq::loss::loss_combine_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(stats, ranks, (int)rows, temperature,
                                                                                      row_lse, row_ce, row_kl);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_loss_grad(const void* s_logits, int64_t lds, const void* t_logits, int64_t ldt, const int64_t* targets,
                 int64_t vocab_start, int64_t rows, int64_t V, float temperature, const float* row_lse,
                 float ce_weight, float kl_weight, void* dlogits, int64_t ldg, void* stream) {
  DeviceScope scope(dlogits);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (int rc = check_matrix(s_logits, rows, V, lds, "student logits")) return rc;
  if (int rc = check_matrix(t_logits, rows, V, ldt, "teacher logits")) return rc;
  if (int rc = check_matrix(dlogits, rows, V, ldg, "dlogits")) return rc;
  if (!(temperature > 0.f)) return fail(VQ_ERR_INVALID, "temperature must be > 0");
  if (rows == 0) return 0;
  if (V <= 0 || V > 0x7fffffff || rows > 0x7fffffff) return fail(VQ_ERR_INVALID, "invalid vocabulary size");
  if (targets == nullptr || row_lse == nullptr) return fail(VQ_ERR_INVALID, "null pointer");
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  const int grid = static_cast<int>(rows < sms ? rows : sms);
  const bool vec = ((reinterpret_cast<uintptr_t>(s_logits) | reinterpret_cast<uintptr_t>(t_logits) |
                     reinterpret_cast<uintptr_t>(dlogits)) & 15u) == 0 &&
                   lds % 8 == 0 && ldt % 8 == 0 && ldg % 8 == 0;
  const auto* S = static_cast<const __nv_bfloat16*>(s_logits);
  const auto* Tl = static_cast<const __nv_bfloat16*>(t_logits);
  auto* G = static_cast<__nv_bfloat16*>(dlogits);
  const auto* y = reinterpret_cast<const long long*>(targets);
  if (temperature == 1.0f)
    vq::loss::loss_grad_kernel<true><<<grid, vq::loss::THREADS, 0, st>>>(S, lds, Tl, ldt, y, vocab_start, (int)rows, (int)V,
                                                                         temperature, row_lse, ce_weight, kl_weight, G, ldg, vec);
  else
    vq::loss::loss_grad_kernel<false><<<grid, vq::loss::THREADS, 0, st>>>(S, lds, Tl, ldt, y, vocab_start, (int)rows, (int)V,
                                                                          temperature, row_lse, ce_weight, kl_weight, G, ldg, vec);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

}  // extern "C"

// ------------------------------------------------------------------ Llama block elementwise
namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_rows16(const void* p, long long rows, long long cols, long long ld, const char* name) {
  if (int rc = check_matrix(p, rows, cols, ld, name)) return rc;
  if (rows > 0 && cols > 0 && (!aligned16(p) || ld % 8 != 0))
    return fail(VQ_ERR_INVALID, "%s: base must be 16-byte aligned and the leading dimension a multiple of 8", name);
  return 0;
}

int grid_for(long long work, int per_sm) {
  int sms = 0;
  if (sm_count(&sms) != 0 || sms <= 0) sms = 148;
  const long long cap = static_cast<long long>(sms) * per_sm;
  return static_cast<int>(work < cap ? (work > 0 ? work : 1) : cap);
}

}  // namespace

extern "C" {

int vq_rmsnorm_fwd(const void* x, int64_t ldx, int64_t rows, int64_t D, const void* weight, float eps, void* y,
                   int64_t ldy, float* rstd, void* stream) {
  DeviceScope scope(y);
  if (D <= 0 || D % 8 != 0 || D > 8 * 8 * vq::blocks::kNormThreads)
    return fail(VQ_ERR_INVALID, "RMSNorm width %lld must be a positive multiple of 8 up to %d", (long long)D,
                8 * 8 * vq::blocks::kNormThreads);
  if (int rc = check_rows16(x, rows, D, ldx, "x")) return rc;
  if (int rc = check_rows16(y, rows, D, ldy, "y")) return rc;
  if (weight == nullptr || !aligned16(weight)) return fail(VQ_ERR_INVALID, "weight must be a 16-byte aligned pointer");
  if (rows == 0) return 0;
  if (rows > 0x7fffffff) return fail(VQ_ERR_INVALID, "too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int vpt = static_cast<int>((D / 8 + vq::blocks::kNormThreads - 1) / vq::blocks::kNormThreads);
  const int grid = grid_for(rows, 16);
  const auto* X = static_cast<const __nv_bfloat16*>(x);
  const auto* W = static_cast<const __nv_bfloat16*>(weight);
  auto* Y = static_cast<__nv_bfloat16*>(y);
  using namespace vq::blocks;
  if (vpt <= 1) rmsnorm_fwd_kernel<1><<<grid, kNormThreads, 0, st>>>(X, ldx, W, eps, (int)rows, (int)D, Y, ldy, rstd);
  else if (vpt <= 2) rmsnorm_fwd_kernel<2><<<grid, kNormThreads, 0, st>>>(X, ldx, W, eps, (int)rows, (int)D, Y, ldy, rstd);
  else if (vpt <= 4) rmsnorm_fwd_kernel<4><<<grid, kNormThreads, 0, st>>>(X, ldx, W, eps, (int)rows, (int)D, Y, ldy, rstd);
  else rmsnorm_fwd_kernel<8><<<grid, kNormThreads, 0, st>>>(X, ldx, W, eps, (int)rows, (int)D, Y, ldy, rstd);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_rmsnorm_bwd(const void* x, int64_t ldx, const void* dy, int64_t lddy, int64_t rows, int64_t D,
                   const void* weight, const float* rstd, void* dx, int64_t lddx, void* stream) {
  DeviceScope scope(dx);
  if (D <= 0 || D % 8 != 0 || D > 8 * 8 * vq::blocks::kNormThreads)
    return fail(VQ_ERR_INVALID, "RMSNorm width %lld must be a positive multiple of 8 up to %d", (long long)D,
                8 * 8 * vq::blocks::kNormThreads);
  if (int rc = check_rows16(x, rows, D, ldx, "x")) return rc;
  if (int rc = check_rows16(dy, rows, D, lddy, "dy")) return rc;
  if (int rc = check_rows16(dx, rows, D, lddx, "dx")) return rc;
  if (weight == nullptr || !aligned16(weight)) return fail(VQ_ERR_INVALID, "weight must be a 16-byte aligned pointer");
  if (rows == 0) return 0;
  if (rstd == nullptr) return fail(VQ_ERR_INVALID, "null rstd");
  if (rows > 0x7fffffff) return fail(VQ_ERR_INVALID, "too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int vpt = static_cast<int>((D / 8 + vq::blocks::kNormThreads - 1) / vq::blocks::kNormThreads);
  const int grid = grid_for(rows, 16);
  const auto* X = static_cast<const __nv_bfloat16*>(x);
  const auto* G = static_cast<const __nv_bfloat16*>(dy);
  const auto* W = static_cast<const __nv_bfloat16*>(weight);
  auto* DX = static_cast<__nv_bfloat16*>(dx);
  using namespace vq::blocks;
  if (vpt <= 1) rmsnorm_bwd_kernel<1><<<grid, kNormThreads, 0, st>>>(X, ldx, G, lddy, W, rstd, (int)rows, (int)D, DX, lddx);
  else if (vpt <= 2) rmsnorm_bwd_kernel<2><<<grid, kNormThreads, 0, st>>>(X, ldx, G, lddy, W, rstd, (int)rows, (int)D, DX, lddx);
  else if (vpt <= 4) rmsnorm_bwd_kernel<4><<<grid, kNormThreads, 0, st>>>(X, ldx, G, lddy, W, rstd, (int)rows, (int)D, DX, lddx);
  else rmsnorm_bwd_kernel<8><<<grid, kNormThreads, 0, st>>>(X, ldx, G, lddy, W, rstd, (int)rows, (int)D, DX, lddx);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_add_rmsnorm_fwd(const void* a, int64_t lda, const void* res, int64_t ldres, int64_t rows, int64_t D,
                       const void* weight, float eps, void* h, int64_t ldh, void* y, int64_t ldy, float* rstd,
                       void* stream) {
  DeviceScope scope(y);
  if (D <= 0 || D % 8 != 0 || D > 8 * 8 * vq::blocks::kNormThreads)
    return fail(VQ_ERR_INVALID, "RMSNorm width %lld must be a positive multiple of 8 up to %d", (long long)D,
                8 * 8 * vq::blocks::kNormThreads);
  if (int rc = check_rows16(a, rows, D, lda, "a")) return rc;
  if (int rc = check_rows16(res, rows, D, ldres, "res")) return rc;
  if (int rc = check_rows16(h, rows, D, ldh, "h")) return rc;
  if (int rc = check_rows16(y, rows, D, ldy, "y")) return rc;
  if (weight == nullptr || !aligned16(weight)) return fail(VQ_ERR_INVALID, "weight must be a 16-byte aligned pointer");
  if (rows == 0) return 0;
  if (rows > 0x7fffffff) return fail(VQ_ERR_INVALID, "too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int vpt = static_cast<int>((D / 8 + vq::blocks::kNormThreads - 1) / vq::blocks::kNormThreads);
  const int grid = grid_for(rows, 16);
  const auto* A = static_cast<const __nv_bfloat16*>(a);
  const auto* R = static_cast<const __nv_bfloat16*>(res);
  const auto* W = static_cast<const __nv_bfloat16*>(weight);
  auto* H = static_cast<__nv_bfloat16*>(h);
  auto* Y = static_cast<__nv_bfloat16*>(y);
  using namespace vq::blocks;
  const int n = static_cast<int>(rows), d = static_cast<int>(D);
  if (vpt <= 1) rmsnorm_fwd_kernel<1, true><<<grid, kNormThreads, 0, st>>>(A, lda, W, eps, n, d, Y, ldy, rstd, R, ldres, H, ldh);
  else if (vpt <= 2) rmsnorm_fwd_kernel<2, true><<<grid, kNormThreads, 0, st>>>(A, lda, W, eps, n, d, Y, ldy, rstd, R, ldres, H, ldh);
  else if (vpt <= 4) rmsnorm_fwd_kernel<4, true><<<grid, kNormThreads, 0, st>>>(A, lda, W, eps, n, d, Y, ldy, rstd, R, ldres, H, ldh);
  else rmsnorm_fwd_kernel<8, true><<<grid, kNormThreads, 0, st>>>(A, lda, W, eps, n, d, Y, ldy, rstd, R, ldres, H, ldh);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_rmsnorm_bwd_add(const void* x, int64_t ldx, const void* dy, int64_t lddy, const void* dres, int64_t lddres,
                       int64_t rows, int64_t D, const void* weight, const float* rstd, void* dx, int64_t lddx,
                       void* stream) {
  DeviceScope scope(dx);
  if (D <= 0 || D % 8 != 0 || D > 8 * 8 * vq::blocks::kNormThreads)
    return fail(VQ_ERR_INVALID, "RMSNorm width %lld must be a positive multiple of 8 up to %d", (long long)D,
                8 * 8 * vq::blocks::kNormThreads);
  if (int rc = check_rows16(x, rows, D, ldx, "x")) return rc;
  if (int rc = check_rows16(dy, rows, D, lddy, "dy")) return rc;
  if (int rc = check_rows16(dres, rows, D, lddres, "dres")) return rc;
  if (int rc = check_rows16(dx, rows, D, lddx, "dx")) return rc;
  if (weight == nullptr || !aligned16(weight)) return fail(VQ_ERR_INVALID, "weight must be a 16-byte aligned pointer");
  if (rows == 0) return 0;
  if (rstd == nullptr) return fail(VQ_ERR_INVALID, "null rstd");
  if (rows > 0x7fffffff) return fail(VQ_ERR_INVALID, "too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int vpt = static_cast<int>((D / 8 + vq::blocks::kNormThreads - 1) / vq::blocks::kNormThreads);
  const int grid = grid_for(rows, 16);
  const auto* X = static_cast<const __nv_bfloat16*>(x);
  const auto* G = static_cast<const __nv_bfloat16*>(dy);
  const auto* DR = static_cast<const __nv_bfloat16*>(dres);
  const auto* W = static_cast<const __nv_bfloat16*>(weight);
  auto* DX = static_cast<__nv_bfloat16*>(dx);
  using namespace vq::blocks;
  const int n = static_cast<int>(rows), d = static_cast<int>(D);
  if (vpt <= 1) rmsnorm_bwd_kernel<1, true><<<grid, kNormThreads, 0, st>>>(X, ldx, G, lddy, W, rstd, n, d, DX, lddx, DR, lddres);
  else if (vpt <= 2) rmsnorm_bwd_kernel<2, true><<<grid, kNormThreads, 0, st>>>(X, ldx, G, lddy, W, rstd, n, d, DX, lddx, DR, lddres);
  else if (vpt <= 4) rmsnorm_bwd_kernel<4, true><<<grid, kNormThreads, 0, st>>>(X, ldx, G, lddy, W, rstd, n, d, DX, lddx, DR, lddres);
  else rmsnorm_bwd_kernel<8, true><<<grid, kNormThreads, 0, st>>>(X, ldx, G, lddy, W, rstd, n, d, DX, lddx, DR, lddres);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_rope(const void* q, const int64_t* q_strides, int64_t Hq, const void* k, const int64_t* k_strides, int64_t Hk,
            const void* cos, const void* sin, const int64_t* cs_strides, int64_t B, int64_t S, int64_t D, int backward,
            void* q_out, void* k_out, void* stream) {
  DeviceScope scope(q_out);
  if (B < 0 || S < 0 || Hq < 0 || Hk < 0) return fail(VQ_ERR_INVALID, "negative shape");
  if (D <= 0 || D % 16 != 0) return fail(VQ_ERR_INVALID, "head dimension %lld must be a multiple of 16", (long long)D);
  if (B == 0 || S == 0 || Hq + Hk == 0) return 0;
  if (q_strides == nullptr || k_strides == nullptr || cs_strides == nullptr)
    return fail(VQ_ERR_INVALID, "null stride array");
  const void* ptrs[6] = {q, k, cos, sin, q_out, k_out};
  for (int i = 0; i < 6; ++i) {
    if ((i == 1 || i == 5) && Hk == 0) continue;
    if ((i == 0 || i == 4) && Hq == 0) continue;
    if (ptrs[i] == nullptr || !aligned16(ptrs[i])) return fail(VQ_ERR_INVALID, "pointer %d is null or not 16-byte aligned", i);
  }
  const int64_t st3[6] = {q_strides[0], q_strides[1], q_strides[2], k_strides[0], k_strides[1], k_strides[2]};
  for (int i = 0; i < 6; ++i)
    if (st3[i] < 0 || st3[i] % 8 != 0) return fail(VQ_ERR_INVALID, "q/k strides must be non-negative multiples of 8");
  if (cs_strides[0] < 0 || cs_strides[1] < 0 || cs_strides[0] % 8 != 0 || cs_strides[1] % 8 != 0)
    return fail(VQ_ERR_INVALID, "cos/sin strides must be non-negative multiples of 8");
  if (B * S > 0x7fffffffLL || Hq > 65535 || Hk > 65535) return fail(VQ_ERR_INVALID, "shape too large");
  vq::blocks::RopeSide qs{static_cast<const __nv_bfloat16*>(q), q_strides[0], q_strides[1], q_strides[2], (int)Hq,
                          static_cast<__nv_bfloat16*>(q_out)};
  vq::blocks::RopeSide ks{static_cast<const __nv_bfloat16*>(k), k_strides[0], k_strides[1], k_strides[2], (int)Hk,
                          static_cast<__nv_bfloat16*>(k_out)};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(B * S, 16);
  const auto* C = static_cast<const __nv_bfloat16*>(cos);
  const auto* Sn = static_cast<const __nv_bfloat16*>(sin);
  if (backward)
    vq::blocks::rope_kernel<true><<<grid, vq::blocks::kRopeThreads, 0, st>>>(qs, ks, C, Sn, cs_strides[0], cs_strides[1],
                                                                            (int)B, (int)S, (int)D);
  else
    vq::blocks::rope_kernel<false><<<grid, vq::blocks::kRopeThreads, 0, st>>>(qs, ks, C, Sn, cs_strides[0], cs_strides[1],
                                                                             (int)B, (int)S, (int)D);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_swiglu_fwd(const void* gate, int64_t ldg, const void* up, int64_t ldu, int64_t rows, int64_t F, void* y,
                  int64_t ldy, void* stream) {
  DeviceScope scope(y);
  if (F <= 0 || F % 8 != 0) return fail(VQ_ERR_INVALID, "SwiGLU width %lld must be a positive multiple of 8", (long long)F);
  if (int rc = check_rows16(gate, rows, F, ldg, "gate")) return rc;
  if (int rc = check_rows16(up, rows, F, ldu, "up")) return rc;
  if (int rc = check_rows16(y, rows, F, ldy, "y")) return rc;
  if (rows == 0) return 0;
  if (rows > 0x7fffffff) return fail(VQ_ERR_INVALID, "too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = grid_for((rows * (F / 8) + vq::blocks::kEltThreads - 1) / vq::blocks::kEltThreads, 8);
  vq::blocks::swiglu_kernel<false><<<grid, vq::blocks::kEltThreads, 0, st>>>(
      static_cast<const __nv_bfloat16*>(gate), ldg, static_cast<const __nv_bfloat16*>(up), ldu, nullptr, 0, (int)rows,
      (int)F, static_cast<__nv_bfloat16*>(y), nullptr, ldy);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_swiglu_bwd(const void* gate, int64_t ldg, const void* up, int64_t ldu, const void* dy, int64_t lddy, int64_t rows,
                  int64_t F, void* dgate, void* dup, int64_t ldo, void* stream) {
  DeviceScope scope(dgate);
  if (F <= 0 || F % 8 != 0) return fail(VQ_ERR_INVALID, "SwiGLU width %lld must be a positive multiple of 8", (long long)F);
  if (int rc = check_rows16(gate, rows, F, ldg, "gate")) return rc;
  if (int rc = check_rows16(up, rows, F, ldu, "up")) return rc;
  if (int rc = check_rows16(dy, rows, F, lddy, "dy")) return rc;
  if (int rc = check_rows16(dgate, rows, F, ldo, "dgate")) return rc;
  if (int rc = check_rows16(dup, rows, F, ldo, "dup")) return rc;
  if (rows == 0) return 0;
  if (rows > 0x7fffffff) return fail(VQ_ERR_INVALID, "too many rows");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = grid_for((rows * (F / 8) + vq::blocks::kEltThreads - 1) / vq::blocks::kEltThreads, 8);
  vq::blocks::swiglu_kernel<true><<<grid, vq::blocks::kEltThreads, 0, st>>>(
      static_cast<const __nv_bfloat16*>(gate), ldg, static_cast<const __nv_bfloat16*>(up), ldu,
      static_cast<const __nv_bfloat16*>(dy), lddy, (int)rows, (int)F, static_cast<__nv_bfloat16*>(dgate),
      static_cast<__nv_bfloat16*>(dup), ldo);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

}  // extern "C"

extern "C" {

int vq_route_prep(const void* keys, int64_t T, int K, int64_t* order, int64_t* inv, int* group_off, void* stream) {
  DeviceScope scope(order);
  if (K < 1 || K > vq::route::kMaxKeys) return fail(VQ_ERR_INVALID, "groups %d not in [1, %d]", K, vq::route::kMaxKeys);
  if (T < 0) return fail(VQ_ERR_INVALID, "negative length");
  if (group_off == nullptr) return fail(VQ_ERR_INVALID, "null group offsets");
  if (T > 0 && (keys == nullptr || order == nullptr || inv == nullptr)) return fail(VQ_ERR_INVALID, "null pointer");
  if (T > (1LL << 30)) return fail(VQ_ERR_INVALID, "too many elements");
  vq::route::route_prep_kernel<<<1, vq::route::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(keys), T, K, reinterpret_cast<long long*>(order), reinterpret_cast<long long*>(inv),
      group_off);
  VQ_CUDA(cudaGetLastError());
  return 0;
}

int vq_quantize(int ggml_type, const void* w, int w_dtype, int64_t rows, int64_t cols, int64_t ldw, void* out,
                void* stream) {
  DeviceScope scope(out);
  if (ggml_type != vq::kQ8_0) return fail(VQ_ERR_UNSUPPORTED, "GPU quantiser: ggml type %d not supported (Q8_0 only)", ggml_type);
  if (w_dtype != 0 && w_dtype != 1) return fail(VQ_ERR_INVALID, "weight dtype %d (0 = float32, 1 = bfloat16)", w_dtype);
  if (rows < 0 || cols < 0) return fail(VQ_ERR_INVALID, "negative shape");
  if (cols % 32 != 0) return fail(VQ_ERR_INVALID, "requires in_features %% 32 == 0, got %lld", (long long)cols);
  if (ldw < cols) return fail(VQ_ERR_INVALID, "leading dimension %lld < %lld", (long long)ldw, (long long)cols);
  const long long nblk = static_cast<long long>(rows) * (cols / 32);
  if (nblk == 0) return 0;
  if (w == nullptr || out == nullptr) return fail(VQ_ERR_INVALID, "null pointer");
  int sms = 0;
  if (int rc = sm_count(&sms)) return rc;
  const long long warps_per_cta = vq::quant::kQ8Threads / 32;
  long long grid = (nblk + warps_per_cta - 1) / warps_per_cta;
  if (grid > 16LL * sms) grid = 16LL * sms;  // grid-stride beyond 16 resident CTAs per SM
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (w_dtype == 0)
    vq::quant::q8_0_quantize_kernel<float><<<static_cast<unsigned>(grid), vq::quant::kQ8Threads, 0, st>>>(
        static_cast<const float*>(w), rows, cols, ldw, static_cast<uint8_t*>(out));
  else
    vq::quant::q8_0_quantize_kernel<__nv_bfloat16><<<static_cast<unsigned>(grid), vq::quant::kQ8Threads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(w), rows, cols, ldw, static_cast<uint8_t*>(out));
  VQ_CUDA(cudaGetLastError());
  return 0;
}

}  // extern "C"

