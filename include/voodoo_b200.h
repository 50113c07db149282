/*
 * voodoo_b200.h -- C ABI of libvoodoo_b200.so, the B200 (sm_100a) kernels of
 * the gated-candidate training step of Voodoo dynamic quantisation.
 *
 * Conventions
 *   - Every pointer is DEVICE memory unless a comment says "host".
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - Matrices are row-major; `ld*` are leading dimensions in ELEMENTS.
 *     bf16 matrices used as GEMM operands need a 16-byte aligned base and a
 *     leading dimension that is a multiple of 8.
 *   - Packed candidates are GGUF block streams, rows contiguous, exactly the
 *     layout ggml's quantize_* writes ([rows * cols / block_elems, block_bytes]
 *     uint8).  Formats are ggml type ids: Q8_0 = 8, Q2_K = 10, Q3_K = 11,
 *     Q4_K = 12, Q5_K = 13, Q6_K = 14, IQ4_XS = 23.
 *   - Return 0 on success or a negative VQ_ERR_* code; vq_last_error() gives a
 *     thread-local message.  No C++ exception crosses this boundary.
 *   - Calls only enqueue work on `stream`: they never synchronise (except
 *     vq_device_error) and never allocate; scratch space is caller-provided.
 *   - Thread-safe for distinct streams.  The one process-wide state is the
 *     pair of SM reserves (vq_set_gategrad_sm_reserve, vq_set_gemm_sm_reserve):
 *     read when a GEMM is launched, they set how many SMs its persistent grid
 *     leaves free, never what it computes.
 */
#ifndef VOODOO_B200_H
#define VOODOO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VQ_ABI_VERSION 1

#define VQ_OK 0
#define VQ_ERR_INVALID (-1)     /* bad shape, alignment, null pointer, ... (Python: ValueError)   */
#define VQ_ERR_CUDA (-2)        /* CUDA runtime / driver failure          (Python: RuntimeError) */
#define VQ_ERR_UNSUPPORTED (-3) /* unknown or unsupported ggml type       (Python: ValueError)   */

/* Message of the last failing call on this thread. */
const char* vq_last_error(void);

/* VQ_ABI_VERSION of the loaded library. */
int vq_abi_version(void);

/* Block geometry of a ggml type.  Replaces the QuantTypeInfo lookup
 * voodoo_quant/ggml.py:158-168 (get_quant_info) for the supported formats. */
int vq_format_info(int ggml_type, int* block_elems /* host */, int* block_bytes /* host */);

/* Synchronise `stream`, then return and clear the device error word in *code
 * (host): 0 = none; (1 << 16 | where) = an mbarrier wait gave up after its
 * time limit; (2 << 16) = a kernel met an unknown format. */
int vq_device_error(void* stream, int* code /* host */);

/* K0 -- bit-exact dequantisation of one packed candidate into float32
 * out[rows, cols] (cols = padded in_features, a multiple of the block size).
 * Replaces dequantize_tensor_gpu, voodoo_quant/layers.py:298-319 (per-format
 * decoders layers.py:62-213, quants/gpu_dequant.py:460-519) and the libggml
 * call ggml.dequantize_tensor, voodoo_quant/ggml.py:224-269. */
int vq_dequant(int ggml_type, const void* blocks, int64_t rows, int64_t cols, float* out, void* stream);

/* K1a -- softmax candidate mixture W_mix = sum_k probs[k] * W_k, accumulated
 * in fp32 from the bit-exact decodes and rounded once to bf16 into
 * w_bf16[rows, ldw]; columns in [cols, ldw) are written as zero.
 * types/blocks are HOST arrays of K entries (ggml ids / device pointers),
 * probs is a device float[K]; padded_cols is a multiple of 256.
 * Replaces _MixedWeightFunction.forward, voodoo_quant/layers.py:336-352,
 * _MixedWeightFunctionLazy.forward :502-580 and get_mixed_weight :1474-1535. */
int vq_mix(int K, const int* types, const void* const* blocks, const float* probs, int64_t rows,
           int64_t padded_cols, int64_t cols, void* w_bf16, int64_t ldw, void* stream);

/* K1b -- y[T, N] = x[T, Kin] * w[N, Kin]^T (bf16 in, fp32 accumulate in TMEM,
 * bf16 out), persistent tcgen05 GEMM.  Replaces F.linear(x, mixed),
 * voodoo_quant/layers.py:1730-1731. */
int vq_linear_fwd(const void* x, int64_t T, int64_t Kin, int64_t ldx, const void* w, int64_t N, int64_t ldw,
                  void* y, int64_t ldy, void* stream);

/* K1 with the SwiGLU of a Llama MLP in its epilogue: h[T, F] =
 * silu(x w_gate^T) * (x w_up^T), w[2F, Kin] holding the gate rows then the up
 * rows.  Each gate/up output is rounded to bf16 before the activation, so h
 * equals a gate|up GEMM into bf16 followed by vq_swiglu_fwd bit for bit;
 * the [T, 2F] gate|up output is never written.  T > 128, F a multiple of
 * 128 (VQ_ERR_UNSUPPORTED otherwise).  For forward-only (teacher) MLPs:
 * replaces Q8Linear.forward for gate_proj and up_proj
 * (voodoo_quant/training/q8_teacher.py:101-128) and the act_fn(gate) * up of
 * the Hugging Face LlamaMLP.forward (transformers modeling_llama.py:183)
 * around them. */
int vq_linear_fwd_swiglu(const void* x, int64_t T, int64_t Kin, int64_t ldx, const void* w, int64_t F, int64_t ldw,
                         void* h, int64_t ldh, void* stream);

/* K2 -- dx[T, Kin] = dy[T, N] * w[N, Kin] (w read MN-major by TMA, no
 * transpose copy).  Replaces the input-gradient half of F.linear's autograd
 * in MixedQuantLinear.forward, voodoo_quant/layers.py:1731. */
int vq_linear_dx(const void* dy, int64_t T, int64_t N, int64_t lddy, const void* w, int64_t Kin, int64_t ldw,
                 void* dx, int64_t lddx, void* stream);

/* Bytes of scratch vq_gategrad needs for an [N, Kin] layer with K candidates. */
size_t vq_gategrad_workspace_bytes(int64_t N, int64_t Kin, int K);

/* K3 -- grad_probs[k] = <dy^T x, W_k> over the first Kin columns, for the K
 * packed candidates (types/blocks HOST arrays, padded_cols = padded
 * in_features).  dW = dy^T x is accumulated tile by tile in TMEM and reduced
 * against re-decoded candidate tiles in the GEMM epilogue; it is never
 * written to memory.  Fixed-order (deterministic) reduction.
 * Replaces _MixedWeightFunction.backward, voodoo_quant/layers.py:355-363
 * (and _MixedWeightFunctionLazy.backward :583-667) together with the weight
 * gradient of F.linear that feeds it. */
int vq_gategrad(const void* dy, int64_t lddy, const void* x, int64_t ldx, int64_t T, int64_t N, int64_t Kin, int K,
                const int* types, const void* const* blocks, int64_t padded_cols, void* workspace,
                size_t workspace_bytes, float* grad_probs, void* stream);

/* Bytes of scratch vq_gategrad_grouped needs for G layers of N_total rows in
 * all, Kin columns, K candidates each. */
size_t vq_gategrad_grouped_workspace_bytes(int64_t N_total, int64_t Kin, int G, int K);

/* K3 for G <= 4 gated Linears that read the same input x (q/k/v, gate/up):
 * one gate-gradient GEMM over dy [T, N_total], whose columns are the layers'
 * outputs side by side (layer g: rows[g] columns, a multiple of 32), with
 * layer g's K candidates at blocks[g * K + k] (the same K formats `types` for
 * every layer).  grad_probs[g * ld_grad + k] = <dy_g^T x, W_{g,k}>.  Results
 * equal G vq_gategrad calls up to the order of fp32 partial sums.  Batches the
 * per-layer _MixedWeightFunction.backward of voodoo_quant/layers.py:355-363
 * for layers whose forwards share one input. */
int vq_gategrad_grouped(const void* dy, int64_t lddy, const void* x, int64_t ldx, int64_t T, int G,
                        const int64_t* rows, int64_t Kin, int K, const int* types, const void* const* blocks,
                        int64_t padded_cols, void* workspace, size_t workspace_bytes, float* grad_probs,
                        int64_t ld_grad, void* stream);

/* PTQR grouping in one launch: the stable counting sort of T routing keys
 * (uint8, values in [0, K), K <= 8): order[p] = i and inv[i] = p (int64) for
 * the element i placed at position p, group_off[K + 1] (int32) the first
 * position of each candidate's group.  Replaces the per-candidate nonzero
 * selections of _RoutedMixedLinear.forward, voodoo_quant/layers.py:390-396. */
int vq_route_prep(const void* keys, int64_t T, int K, int64_t* order, int64_t* inv, int* group_off, void* stream);

/* Number of SMs later vq_gategrad / vq_gategrad_noalloc launches leave free
 * (process-wide; 0 = use every SM).  A caller that has a collective in flight
 * on another stream while the gate-gradient GEMM runs (the TP input-gradient
 * all-reduce) reserves the SMs the collective's kernel needs, so the two
 * actually run concurrently: the persistent GEMM otherwise occupies every SM
 * and the collective waits for it.  No counterpart in the reference (its
 * all-reduces are synchronous). */
int vq_set_gategrad_sm_reserve(int sms);

/* The same for the store-epilogue GEMMs (vq_linear_fwd, vq_linear_dx,
 * vq_mixgemm_fwd): a caller that splits dX into row chunks and all-reduces
 * chunk i while chunk i + 1 is computed leaves the collective its SMs.  No
 * counterpart in the reference. */
int vq_set_gemm_sm_reserve(int sms);

/* GPU quantiser: weights [rows, ldw] (w_dtype 0 = float32, 1 = bfloat16;
 * cols a multiple of 32) -> packed blocks out (rows * cols / 32 blocks of
 * block_bytes).  Q8_0 (ggml type 8) only: byte-identical to ggml's
 * reference rule (d = max|x| / 127 stored as fp16, q = roundf(x / d)).
 * Replaces libggml's quantize_q8_0 behind ggml.quantize_tensor,
 * voodoo_quant/ggml.py:171-221 (Q8_0 teacher, training/q8_teacher.py:101-128,
 * and Q8_0 candidates, layers.py:1301-1340).  Other types return
 * VQ_ERR_UNSUPPORTED. */
int vq_quantize(int ggml_type, const void* w, int w_dtype, int64_t rows, int64_t cols, int64_t ldw, void* out,
                void* stream);

/* K1 for the per-token routed (PTQR) forward: rows of x are grouped by
 * candidate, rows [group_off[g], group_off[g + 1]) use weight w[g] (w a HOST
 * array of G <= 8 device pointers to bf16 [N, ldw]; group_off a DEVICE int
 * array of G + 1 ascending offsets from 0 to T).  The kernel reads the
 * offsets itself, so the caller needs no host copy of the group sizes.
 * T > 128.  Replaces the per-candidate matmuls of _RoutedMixedLinear.forward,
 * voodoo_quant/layers.py:384-401. */
int vq_linear_fwd_grouped(const void* x, int64_t T, int64_t Kin, int64_t ldx, int G, const void* const* w,
                          int64_t N, int64_t ldw, const int* group_off, void* y, int64_t ldy, void* stream);

/* Largest scratch vq_gategrad_noalloc can use: 4 MiB, which covers every
 * unsharded layer up to a 152064 x 5120 vocabulary projection with 7
 * candidates (vq_gategrad_workspace_bytes gives the need of a shape). */
#define VQ_GATEGRAD_NOALLOC_SCRATCH_BYTES (4u << 20)

/* vq_gategrad without a workspace argument, for callers that cannot allocate
 * device memory: a host that binds this library over a plain C FFI and has no
 * device allocator to hand it, or a process whose memory pool (a framework's
 * caching allocator) owns the device memory, so that a cudaMalloc beside the
 * pool would fail or split it.  No counterpart in the reference (its gate
 * gradient is plain torch autograd).
 *   - Scratch is one file-scope device array of
 *     VQ_GATEGRAD_NOALLOC_SCRATCH_BYTES, held on every GPU that loads the
 *     library until the process exits.  Shapes whose
 *     vq_gategrad_workspace_bytes exceeds it are rejected (VQ_ERR_INVALID)
 *     before anything runs; use vq_gategrad with a workspace for those.
 *   - The array's memory is committed when the CUDA driver loads this
 *     library's device code on a device, which happens lazily, at the first
 *     call of any vq_* entry point that launches work there.  A process whose
 *     pool will take nearly all device memory should make one such call on
 *     each device before the pool reserves its memory.
 *   - The first call on a device looks up the array's device address with
 *     that device current (the device of grad_probs) and keeps it for the
 *     process; make that first call before any stream capture on the device.
 *     The address is not looked up again, so a process that resets a device
 *     (cudaDeviceReset) must not call this entry point on it afterwards.
 *   - Every call shares the array.  Nothing in it needs to start at zero: a
 *     call that completes writes every partial slot it reads back.  A call
 *     whose kernel gave up on a bounded wait (vq_device_error non-zero) may
 *     sum partials an earlier call left, so its result is valid only while
 *     vq_device_error reads 0.  Calls that overlap on the GPU (other streams,
 *     other threads) race on the array: order them.
 *   - Allocates nothing: no cudaMalloc, cudaFree or allocating library call.
 * Arguments, results and errors are those of vq_gategrad. */
int vq_gategrad_noalloc(const void* dy, int64_t lddy, const void* x, int64_t ldx, int64_t T, int64_t N, int64_t Kin,
                        int K, const int* types, const void* const* blocks, int64_t padded_cols, float* grad_probs,
                        void* stream);

/* K1 convenience: vq_mix into w_mix[N, ldw] followed by vq_linear_fwd. */
int vq_mixgemm_fwd(const void* x, int64_t T, int64_t Kin, int64_t ldx, int K, const int* types,
                   const void* const* blocks, const float* probs, int64_t N, int64_t padded_cols, void* w_mix,
                   int64_t ldw, void* y, int64_t ldy, void* stream);

/* K1 as ONE kernel: y[T, N] = x[T, Kin] * W_mix^T with W_mix = sum_k
 * probs[k] * W_k decoded and mixed by producer warps straight into the
 * GEMM's shared-memory operand tiles (no W_mix in HBM).  Each B tile is
 * decoded again for every 256-row tile of x, so the decode work grows with T
 * / 256; the result equals vq_mix followed by vq_linear_fwd bit for bit.
 * T > 128 (VQ_ERR_UNSUPPORTED otherwise).  Replaces _MixedWeightFunction.forward
 * + F.linear, voodoo_quant/layers.py:336-352,1730-1731, as one launch. */
int vq_mixgemm_fwd_fused(const void* x, int64_t T, int64_t Kin, int64_t ldx, int K, const int* types,
                         const void* const* blocks, const float* probs, int64_t N, int64_t padded_cols, void* y,
                         int64_t ldy, void* stream);

/* K2 convenience: vq_mix into w_mix[N, ldw] followed by vq_linear_dx, i.e.
 * dx[T, Kin] = dy[T, N] * (sum_k probs[k] W_k).  For callers that keep no
 * W_mix between the forward and the backward (the reference re-mixes in its
 * backward, _MixedWeightFunctionLazy.backward, voodoo_quant/layers.py:
 * 582-667, then multiplies through F.linear's autograd, :1731). */
int vq_mixgemm_dx(const void* dy, int64_t T, int64_t N, int64_t lddy, int K, const int* types,
                  const void* const* blocks, const float* probs, int64_t Kin, int64_t padded_cols, void* w_mix,
                  int64_t ldw, void* dx, int64_t lddx, void* stream);

/* K4 -- fused chunked-vocab CE + KL(teacher || student) on bf16 logits.
 * Per row r: row_ce[r] = lse(s) - s[y] (0 when targets[r] < 0) and
 * row_kl[r] = T^2 * KL(softmax(t/T) || softmax(s/T)); when dlogits != NULL it
 * also writes d/ds = ce_weight * (softmax(s) - onehot(y))
 *                  + kl_weight * T * (softmax(s/T) - softmax(t/T))
 * (the gradient of ce_weight * sum(row_ce) + kl_weight * sum(row_kl)).
 * targets are int64 token ids.  Replaces the loss of
 * voodoo_quant/training/trainer.py:2567-2575 and _chunked_forward_loss
 * :797-821. */
int vq_loss_fused(const void* s_logits, int64_t lds, const void* t_logits, int64_t ldt, const int64_t* targets,
                  int64_t rows, int64_t V, float temperature, float ce_weight, float kl_weight, float* row_ce,
                  float* row_kl, void* dlogits, int64_t ldg, void* stream);

/* K4, vocab-parallel pass 1: per-row partial statistics float[rows, 8] of this
 * rank's vocab shard [vocab_start, vocab_start + V).  Replaces the per-chunk
 * _global_lse MAX/SUM all-reduce inputs of _tp_vocab_parallel_losses,
 * voodoo_quant/training/trainer.py:974-996. */
int vq_loss_stats(const void* s_logits, int64_t lds, const void* t_logits, int64_t ldt, const int64_t* targets,
                  int64_t vocab_start, int64_t rows, int64_t V, float temperature, float* stats, void* stream);

/* K4, combine: stats[ranks, rows, 8] (all ranks' partials, rank order) ->
 * row_lse[rows, 4] (lse(s), lse(s/T), lse(t/T), target-found flag), row_ce,
 * row_kl.  Replaces the cross-rank logsumexp of trainer.py:974-996 and the
 * partial-loss all-reduce :1061-1064. */
int vq_loss_combine(const float* stats, int ranks, int64_t rows, float temperature, float* row_lse,
                    float* row_ce, float* row_kl, void* stream);

/* K4, vocab-parallel pass 2: the gradient of this rank's logits shard given
 * the global row_lse.  Replaces the per-chunk backward of
 * _tp_vocab_parallel_losses, trainer.py:1041-1046. */
int vq_loss_grad(const void* s_logits, int64_t lds, const void* t_logits, int64_t ldt, const int64_t* targets,
                 int64_t vocab_start, int64_t rows, int64_t V, float temperature, const float* row_lse,
                 float ce_weight, float kl_weight, void* dlogits, int64_t ldg, void* stream);

/* ---- Llama decoder-block elementwise work of the distillation step ----
 * The reference's step runs the Hugging Face Llama block around the gated
 * Linears (voodoo_quant/training/trainer.py:2538-2556 calls the student and
 * teacher models); these replace that block's torch elementwise ops, one HBM
 * pass each, bf16 in and out with fp32 arithmetic.  Row-major operands need a
 * 16-byte aligned base and a leading dimension that is a multiple of 8. */

/* y = w * bf16(x * rsqrt(mean(x^2) + eps)) per row of x[rows, D] (D % 8 == 0,
 * D <= 8192, weight bf16[D]); rstd[rows] (float, may be NULL) keeps
 * rsqrt(mean(x^2) + eps) for the backward.  Replaces LlamaRMSNorm.forward
 * (transformers models/llama/modeling_llama.py). */
int vq_rmsnorm_fwd(const void* x, int64_t ldx, int64_t rows, int64_t D, const void* weight, float eps, void* y,
                   int64_t ldy, float* rstd, void* stream);

/* dx = r * (g - n * mean(g * n)) with g = dy * w and n = x * r, r = rstd[row].
 * The weight gradient is not produced (the step trains only the gates). */
int vq_rmsnorm_bwd(const void* x, int64_t ldx, const void* dy, int64_t lddy, int64_t rows, int64_t D,
                   const void* weight, const float* rstd, void* dx, int64_t lddx, void* stream);

/* Residual add fused into the RMSNorm that follows it: h = a + res (bf16
 * add), y = weight * bf16(h * rsqrt(mean(h^2) + eps)); h, y and rstd are
 * written.  Replaces `hidden_states = residual + hidden_states;
 * post_attention_layernorm(hidden_states)` of Hugging Face
 * LlamaDecoderLayer.forward in the student/teacher models the step runs
 * (trainer.py:2538-2556). */
int vq_add_rmsnorm_fwd(const void* a, int64_t lda, const void* res, int64_t ldres, int64_t rows, int64_t D,
                       const void* weight, float eps, void* h, int64_t ldh, void* y, int64_t ldy, float* rstd,
                       void* stream);

/* Its backward: dx = (RMSNorm input gradient of dy at x = h) + dres in fp32,
 * rounded once to bf16 -- the gradient of both a and res, where dres is the
 * gradient reaching h through the later residual add. */
int vq_rmsnorm_bwd_add(const void* x, int64_t ldx, const void* dy, int64_t lddy, const void* dres, int64_t lddres,
                       int64_t rows, int64_t D, const void* weight, const float* rstd, void* dx, int64_t lddx,
                       void* stream);

/* Rotary embedding of q [B, S, Hq, D] and k [B, S, Hk, D] in one launch
 * (unit stride over D; HOST arrays q_strides/k_strides = {b, s, h} and
 * cs_strides = {b, s} in elements, multiples of 8) with cos/sin [B, S, D];
 * writes contiguous [B, S, H, D] outputs.  backward != 0 applies the
 * transposed rotation (the input gradient).  D % 16 == 0.  Replaces
 * apply_rotary_pos_emb / rotate_half (transformers modeling_llama.py). */
int vq_rope(const void* q, const int64_t* q_strides, int64_t Hq, const void* k, const int64_t* k_strides, int64_t Hk,
            const void* cos, const void* sin, const int64_t* cs_strides, int64_t B, int64_t S, int64_t D, int backward,
            void* q_out, void* k_out, void* stream);

/* y = silu(gate) * up over [rows, F] (F % 8 == 0).  Replaces
 * LlamaMLP.forward's act_fn(gate_proj(x)) * up_proj(x) product. */
int vq_swiglu_fwd(const void* gate, int64_t ldg, const void* up, int64_t ldu, int64_t rows, int64_t F, void* y,
                  int64_t ldy, void* stream);

/* dgate = dy * up * silu'(gate), dup = dy * silu(gate); both outputs share ldo. */
int vq_swiglu_bwd(const void* gate, int64_t ldg, const void* up, int64_t ldu, const void* dy, int64_t lddy, int64_t rows,
                  int64_t F, void* dgate, void* dup, int64_t ldo, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VOODOO_B200_H */
