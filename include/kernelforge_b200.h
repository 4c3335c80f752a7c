/*
 * kernelforge_b200.h -- C ABI of the B200-native KernelForge hot path.
 *
 * Every entry point takes raw device pointers, sizes and strides (in ELEMENTS), a cudaStream_t
 * passed as `void*` (NULL = legacy default stream), and returns a kf_status. No compute entry
 * point allocates device memory, synchronises the host, or keeps a pointer past the call: the
 * caller owns every buffer, including the workspace where one is needed (the diagnostic
 * kf_query_device_error synchronises; kf_sana_linattn_fwd_noalloc uses a built-in array). Launches are asynchronous
 * on `stream`; a kernel-side failure (a bounded wait that timed out) is recorded in a device
 * error word that kf_query_device_error() reads.
 *
 * The Python modules under kernelforge_b200/ (rmsnorm/, SANA_LinearAttention/,
 * flash_attention_jvp/) keep the reference's call signatures and call these functions.
 * Each declaration names the reference interface it replaces (path:line in zzd1992/KernelForge).
 */
#ifndef KERNELFORGE_B200_H_
#define KERNELFORGE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Element types (the reference's dtype strings "float" / "float16" / "bfloat16"). */
typedef enum {
  KF_DTYPE_F32 = 0,
  KF_DTYPE_F16 = 1,
  KF_DTYPE_BF16 = 2
} kf_dtype;

typedef enum {
  KF_OK = 0,
  KF_ERR_INVALID_ARGUMENT = 1,   /* bad size / stride / null pointer */
  KF_ERR_UNSUPPORTED = 2,        /* dtype or shape outside the supported domain */
  KF_ERR_MISALIGNED = 3,         /* pointer or stride alignment the kernel needs is missing */
  KF_ERR_WORKSPACE = 4,          /* workspace missing or too small */
  KF_ERR_CUDA = 5,               /* a CUDA runtime call or launch failed */
  KF_ERR_DEVICE_TIMEOUT = 6      /* a kernel's bounded wait expired (see kf_query_device_error) */
} kf_status;

/* Human-readable name of a kf_status value (static storage). */
const char* kf_status_string(int status);

/* ABI version: bumped whenever a signature below changes. */
int kf_abi_version(void);

/*
 * Reads (and clears) the device error words of every kernel module on the current device,
 * after synchronising `stream`. *code receives 0 when no kernel reported a failure, else the
 * kf_status of the first failure. Host-synchronising: a diagnostic, not a hot-path call.
 */
int kf_query_device_error(void* stream, int* code);

/*
 * Self-test of the failure-detection path. No counterpart in the reference. Launches one warp
 * that waits on an mbarrier nothing arrives on, through the bounded wait every kernel here uses:
 * after the library's 4 s bound it records KF_ERR_DEVICE_TIMEOUT (6) and returns, so the next
 * kf_query_device_error reports 6 and the context stays usable. Diagnostic only: it occupies
 * one SM for 4 s.
 */
int kf_selftest_bounded_wait(void* stream);

/* ------------------------------------------------------------------------------------------
 * RMSNorm forward.
 * Replaces rms_norm(batch, seq_len, dim, eps, dtype) -> kernel(X, Weight) -> Output
 * (rmsnorm/custom.py:11-75) and computes RMSNorm.forward (rmsnorm/original.py:40-52):
 *   y[r, :] = cast(cast(x[r, :] * rsqrt(mean(x[r, :]^2) + eps)) * weight)
 * with fp32 statistics and the reference's double rounding for 16-bit dtypes.
 * x, y: `rows` rows of `dim` elements, row strides x_row_stride / y_row_stride (elements).
 * weight: `dim` elements, or NULL for no weight (the no-weight comparator of
 * rmsnorm/original.py:55-78). x, weight, y share `dtype`. rows == 0 is a no-op.
 * ---------------------------------------------------------------------------------------- */
int kf_rmsnorm_fwd(const void* x, const void* weight, void* y,
                   int64_t rows, int64_t dim, int64_t x_row_stride, int64_t y_row_stride,
                   float eps, int dtype, void* stream);

/*
 * RMSNorm backward. No counterpart in the reference, whose RMSNorm is forward-only
 * (rmsnorm/README.md:5). Gradients of kf_rmsnorm_fwd's y = cast(cast(x r) w),
 * r = 1 / sqrt(mean(x^2) + eps), with the casts taken as identities (as torch autograd does):
 *   dx = r (dy w) - x r^3 ((dy w) . x) / dim          (fp32, rounded to dtype)
 *   dweight = sum over rows of dy cast(x r)            (fp32, summed in a fixed order)
 * x, dy, dx: `rows` rows of `dim` elements with their own row strides (elements). weight and
 * dweight: `dim` elements, both NULL for no weight (then dx = r dy - x r^3 (dy . x) / dim).
 * With a weight, `workspace` (kf_rmsnorm_bwd_workspace_size(dim) bytes, 16-byte aligned,
 * contents ignored) holds the per-CTA dweight partials. rows == 0 writes zeros to dweight.
 */
size_t kf_rmsnorm_bwd_workspace_size(int64_t dim);
int kf_rmsnorm_bwd(const void* x, const void* weight, const void* dy, void* dx, void* dweight,
                   void* workspace, size_t workspace_bytes, int64_t rows, int64_t dim,
                   int64_t x_row_stride, int64_t dy_row_stride, int64_t dx_row_stride, float eps,
                   int dtype, void* stream);

/* ------------------------------------------------------------------------------------------
 * SANA ReLU linear attention over packed QKV.
 * Replaces qkv_attn_matmul(batch, heads, dim, seq_len, eps, dtype, output_dtype,
 * reduce_splits) -> run(qkv) (SANA_LinearAttention/custom.py:340-388) and computes
 * LiteLA.attn_matmul (SANA_LinearAttention/original.py:99-117) on the packed layout:
 *   qkv [batch, seq_len, 3, heads*dim] (contiguous; q, k, v along axis 2)
 *   out [batch, seq_len, heads*dim] in out_dtype
 *   VK_h = sum_t v_t relu(k_t)^T,  ksum_h = sum_t relu(k_t)           (fp32 accumulation)
 *   out[t, h*dim + r] = (VK_h relu(q_t))_r / (ksum_h . relu(q_t) + eps)
 * `splits` picks the schedule of the bf16/fp16 head_dim-32 path:
 *   0       automatic: the one-launch path when its CTAs fill the GPU's SMs or outnumber
 *           the split path's producer CTAs (with clusters, only for token shares of 1024-4096
 *           per CTA), else the split path with a default split count;
 *   -1      the one-launch path: each CTA owns whole (batch, head) units, reduces K^T V and
 *           ksum in shared memory and writes the output (the workspace is not touched); with
 *           fewer units than SMs, a thread-block cluster of up to 8 CTAs shares each unit,
 *           splitting its tokens and summing the CTAs' K^T V and ksum over distributed shared
 *           memory in a fixed order;
 *   s > 0   the split path: the token axis in s chunks whose fp32 partials go through the
 *           workspace to a tcgen05 epilogue launch.
 * Other shapes (fp32 input, other head dims) keep fp32 partials in the workspace and reduce them
 * in the last CTA to arrive (per-head arrival counters). Size the workspace with
 * kf_sana_linattn_workspace_size and zero-fill it once before its first use; every call leaves
 * it ready for the next one. Calls that share a workspace must be ordered on one stream.
 * dim must divide 128 (the reference's constraint, custom.py:350-351).
 * ---------------------------------------------------------------------------------------- */
size_t kf_sana_linattn_workspace_size(int64_t batch, int64_t heads, int64_t dim, int64_t seq_len,
                                      int64_t splits);

int kf_sana_linattn_fwd(const void* qkv, void* out, void* workspace, size_t workspace_bytes,
                        int64_t batch, int64_t heads, int64_t dim, int64_t seq_len, int64_t splits,
                        float eps, int in_dtype, int out_dtype, void* stream);

/*
 * kf_sana_linattn_fwd after LiteLA's qk_norm (SANA_LinearAttention/original.py:92-96, 127-128):
 * q and k each pass through an RMSNorm over the heads*dim channels of their token
 * (rmsnorm/original.py:40-52, y = cast(cast(x r) w), r = 1/sqrt(mean(x^2) + norm_eps) in fp32)
 * before the attention. Replaces the q_norm / k_norm calls of LiteLA.forward; the reference's
 * custom kernels have no such form (they reject qk_norm). One launch computes r for every
 * token's q and k into the workspace; the attention kernels then apply the norm to q and k as
 * they read them, so no normalised copy is written. q_weight / k_weight: [heads*dim] in
 * in_dtype, 16-byte aligned. The workspace is kf_sana_linattn_qknorm_workspace_size bytes (the
 * kf_sana_linattn_fwd layout followed by 8 bytes per token, rounded up to 128 tokens per batch)
 * and may be shared with kf_sana_linattn_fwd. Other arguments as for kf_sana_linattn_fwd.
 */
size_t kf_sana_linattn_qknorm_workspace_size(int64_t batch, int64_t heads, int64_t dim, int64_t seq_len,
                                             int64_t splits);

int kf_sana_linattn_qknorm_fwd(const void* qkv, void* out, void* workspace, size_t workspace_bytes,
                               int64_t batch, int64_t heads, int64_t dim, int64_t seq_len, int64_t splits,
                               float eps, const void* q_weight, const void* k_weight, float norm_eps,
                               int in_dtype, int out_dtype, void* stream);

/*
 * The schedule kf_sana_linattn_fwd runs for these arguments on the current CUDA device, without
 * launching anything (16-byte aligned qkv and out assumed). No counterpart in the reference.
 *   *launches       kernel launches per call (1: the one-launch path; 2: the other paths);
 *   *ctas_per_unit  on the one-launch path, the CTAs that share one (batch, head) unit: 1, or
 *                   the size of the thread-block cluster that splits its tokens (used when
 *                   batch*heads is below the SM count); 0 on the other paths.
 */
int kf_sana_linattn_plan(int64_t batch, int64_t heads, int64_t dim, int64_t seq_len, int64_t splits,
                         int in_dtype, int64_t* launches, int64_t* ctas_per_unit);

/*
 * kf_sana_linattn_fwd without a workspace, for callers that cannot allocate device memory
 * (code running inside another runtime's memory manager or allocator hook, or under a fixed
 * memory budget). No counterpart in the reference. It allocates nothing: its scratch is a
 * file-scope device array of kf_sana_noalloc_scratch_bytes() bytes (16 MiB), which every GPU
 * that loads the library holds until exit. The caller still passes qkv and out.
 * - `splits` means what it means for kf_sana_linattn_fwd, and the schedule is the one
 *   kf_sana_linattn_plan reports: 0 automatic, -1 the one-launch path (which needs no
 *   scratch), s > 0 the split path with s chunks. The one difference: when the split path's
 *   partials for the requested (or default) split count do not fit the array, fewer splits
 *   are used, down to 1; the result stays within the same tolerance, but the fp32 summation
 *   order differs from kf_sana_linattn_fwd with the same `splits`.
 * - Shapes whose scratch does not fit even with one split are rejected with KF_ERR_WORKSPACE
 *   before any launch (the bf16/fp16 head_dim-32 split path needs batch*heads*4224 bytes per
 *   split; shapes the automatic schedule sends to the one-launch path are never rejected).
 * - The array's device address belongs to a CUDA context. The first call in a context (the
 *   first call on each device, and the first after a cudaDeviceReset or on another context)
 *   loads the library's module there if needed and looks the address up
 *   (cudaGetSymbolAddress); make that first call outside any stream capture.
 * - Every call shares the one array: calls that overlap on the GPU (other streams, other
 *   threads) race. Order them on one stream. The arrival counters are zeroed by each call.
 */
int kf_sana_linattn_fwd_noalloc(const void* qkv, void* out, int64_t batch, int64_t heads,
                                int64_t dim, int64_t seq_len, int64_t splits, float eps,
                                int in_dtype, int out_dtype, void* stream);

/* Size in bytes of the fixed scratch array used by kf_sana_linattn_fwd_noalloc. */
size_t kf_sana_noalloc_scratch_bytes(void);

/* ------------------------------------------------------------------------------------------
 * Projection GEMM with a fused bias (SANA's QKV and output projections).
 * Replaces the reference's _qkv_projection(batch, seq_len, channels, dtype) -> kernel(X, WeightT)
 * (SANA_LinearAttention/custom.py:23-85) and the bias-fused _output_projection -> kernel(X,
 * WeightT, Bias) (custom.py:457-523), i.e. the nn.Linear layers of LiteLA.forward
 * (original.py:122, 143):
 *   y[r, o] = sum_i x[r, i] * W[o, i] (+ bias[o])          fp32 accumulation, one rounding
 * x: [rows, in_features]; y: [rows, out_features]; bias: [out_features] or NULL; all contiguous,
 * one dtype. weight_layout 0: W as nn.Linear stores it, [out_features, in_features]; 1: the
 * reference's prepacked WeightT, [in_features, out_features]. With a packed QKV weight
 * (out_features = 3 * channels) y is the packed [batch, seq_len, 3, channels] layout that
 * kf_sana_linattn_fwd reads.
 * fp16/bf16 run on the tcgen05 tensor cores and need in_features and out_features to be
 * multiples of 8 and 16-byte aligned pointers; fp32 runs fp32 FMAs (no TF32), any shape.
 * rows == 0 is a no-op. Deterministic.
 * ---------------------------------------------------------------------------------------- */
int kf_linear_fwd(const void* x, const void* weight, const void* bias, void* y, int64_t rows,
                  int64_t in_features, int64_t out_features, int weight_layout, int dtype, void* stream);

/* ------------------------------------------------------------------------------------------
 * SANA linear attention fused with its QKV projection (heads of 32 channels, no qk_norm).
 * Replaces the grouped kernels of GroupedFull64QOutLiteLA.grouped_attention
 * (SANA_LinearAttention/custom.py:595-868: grouped_full64_kv_vk_producer and
 * partial_reduce_joint_qout, which the reference writes for B=1, N=1024, C=1152 only), for any
 * batch, seq_len and channels (a multiple of 32, at least 64):
 *   qkv = x W^T (+ bias), rounded to dtype, as LiteLA.forward's self.qkv (original.py:122)
 *   out = LiteLA.attn_matmul of that qkv (original.py:99-117), in dtype
 * without writing q, k or v: a first launch projects K and V and accumulates each split's
 * [K^T V ; sum relu(K)] into the workspace; a second projects Q and writes out.
 * x: [batch, seq_len, channels]; qkv_weight: [3*channels, channels] (nn.Linear layout);
 * qkv_bias: [3*channels] or NULL; out: [batch, seq_len, channels]; dtype bf16 (as the
 * reference's grouped kernels; other dtypes return KF_ERR_UNSUPPORTED); x,
 * qkv_weight, out and workspace 16-byte aligned. Size the workspace with
 * kf_sana_proj_attn_workspace_size (fp32 partials; nothing needs zeroing). Deterministic.
 * ---------------------------------------------------------------------------------------- */
size_t kf_sana_proj_attn_workspace_size(int64_t batch, int64_t seq_len, int64_t channels);

int kf_sana_proj_attn_fwd(const void* x, const void* qkv_weight, const void* qkv_bias, void* out,
                          void* workspace, size_t workspace_bytes, int64_t batch, int64_t seq_len,
                          int64_t channels, float eps, int dtype, void* stream);

/* ------------------------------------------------------------------------------------------
 * FlashAttention forward and forward-mode JVP.
 * Layout: q, tq, out, tangent_out [batch, q_len, q_heads, head_dim]; k, v, tk, tv
 * [batch, k_len, kv_heads, head_dim]; all contiguous, 16-byte aligned, `dtype` fp16 or bf16.
 * lse: fp32 [batch, q_heads, q_len], natural log; +inf for a row that sees no key.
 * head_dim: a multiple of 8, at most 256; q_heads a multiple of kv_heads (GQA / MQA).
 * causal: key j is visible to query i iff j <= i + k_len - q_len (bottom-right aligned).
 * softmax_scale: finite and positive (the reference default is head_dim^-1/2).
 * A NULL tangent (tq / tk / tv) is a zero tangent; its GEMM is skipped.
 * Deterministic: no atomics; the same inputs give bitwise-identical outputs.
 * ---------------------------------------------------------------------------------------- */

/* O and LSE. Replaces the native forward that FlashAttentionFunction.forward calls
 * (_flash_attn_forward, flash_attention_jvp/custom.py:230-239). */
int kf_fa_fwd(const void* q, const void* k, const void* v, void* out, float* lse,
              int64_t batch, int64_t q_len, int64_t k_len, int64_t q_heads, int64_t kv_heads,
              int64_t head_dim, float softmax_scale, int causal, int dtype, void* stream);

/* Standalone JVP from a cached O / LSE:
 *   tO = P tV + H V - rowsum(H) * O,  P = exp(scale * Q K^T - LSE),
 *   H = P * scale * (tQ K^T + Q tK^T).
 * Replaces _attention_jvp_kernel(...)(Q, K, V, TQ, TK, TV, O, LSE) -> TO and the
 * kernelforge::flash_attention_jvp operator (flash_attention_jvp/custom.py:12-157). */
int kf_fa_jvp(const void* q, const void* k, const void* v, const void* tq, const void* tk,
              const void* tv, const void* out, const float* lse, void* tangent_out,
              int64_t batch, int64_t q_len, int64_t k_len, int64_t q_heads, int64_t kv_heads,
              int64_t head_dim, float softmax_scale, int causal, int dtype, void* stream);

/* One-pass forward + JVP (O, LSE and tO with online recurrences; six GEMMs per key tile).
 * Replaces the native forward followed by the JVP launch that torch.func.jvp of
 * flash_attention performs (flash_attention_jvp/custom.py:226-291), fused as
 * flash-attention-jvp-derivation.md sections 7-8 describe. For head dims above 128 (tensor
 * memory holds O's accumulator or tO's, not both) it runs the forward and then the standalone
 * JVP on the same stream; with every tangent NULL, the forward and tO = 0. */
int kf_fa_fwd_jvp(const void* q, const void* k, const void* v, const void* tq, const void* tk,
                  const void* tv, void* out, float* lse, void* tangent_out,
                  int64_t batch, int64_t q_len, int64_t k_len, int64_t q_heads, int64_t kv_heads,
                  int64_t head_dim, float softmax_scale, int causal, int dtype, void* stream);

/* Backward (reverse-mode VJP) from the saved O and LSE:
 *   P = exp(scale * Q K^T - LSE), dP = dO V^T, dS = P * (dP - rowsum(dO * O)),
 *   dQ = scale * dS K, dK = scale * dS^T Q, dV = P^T dO   (GQA: summed over the group).
 * Replaces flash_attn's _flash_attn_backward called by FlashAttentionFunction.backward
 * (flash_attention_jvp/custom.py:255-266), including its `deterministic` flag. dq / dk / dv are
 * written in full. The workspace (kf_fa_bwd_workspace_size bytes for the same head_dim and
 * deterministic, 16-byte aligned, contents ignored) holds two fp32 row statistics per (batch,
 * head, query), padded to a multiple of 128 queries: -LSE log2(e) and -rowsum(dO * O); with
 * deterministic = 0 and head_dim <= 128 also the fp32 dQ sums (64 or 128 per row).
 * deterministic = 0: head dims up to 128 run one kernel for dQ, dK and dV whose dQ partials are
 *   summed at L2, so dq may differ in the last bit from run to run (dk, dv do not), as with
 *   flash_attn's deterministic=False, which the reference passes.
 * deterministic != 0 (and head dims 136..256): separate dQ and dK / dV kernels, no atomics,
 *   bitwise reproducible. */
size_t kf_fa_bwd_workspace_size(int64_t batch, int64_t q_heads, int64_t q_len, int64_t head_dim,
                                int deterministic);
int kf_fa_bwd(const void* q, const void* k, const void* v, const void* out, const void* dout,
              const float* lse, void* dq, void* dk, void* dv, void* workspace, size_t workspace_bytes,
              int64_t batch, int64_t q_len, int64_t k_len, int64_t q_heads, int64_t kv_heads,
              int64_t head_dim, float softmax_scale, int causal, int deterministic, int dtype,
              void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* KERNELFORGE_B200_H_ */
