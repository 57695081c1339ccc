/*
 * fni8_b200.h -- C ABI of the B200 (sm_100a) W8A8 matmul path for fni8-serve.
 *
 * fni8-serve (Python) reaches its kernels through the external `fni8` package:
 *   fni8.linear(x, qt, bias=)           fni8serve/layers/linear.py:69
 *   fni8.rmsnorm(x, w, eps, residual=, unit_offset=)   fni8serve/layers/norm.py:51
 *   fni8.act_and_mul(x, "silu"|"gelu_tanh")            fni8serve/layers/activation.py:24,40
 *   the per-expert GatedMLP loop of SparseMoE          fni8serve/models/moe.py:97-105
 * This header is the native boundary underneath a drop-in `fni8` Python package: plain
 * pointers, element counts and an opaque CUDA stream (`void* stream`, a cudaStream_t;
 * NULL means the legacy default stream). No torch or C++ types cross it.
 *
 * Conventions
 *  - Every function returns an int status (FNI8_OK == 0). On failure nothing has been
 *    launched, and fni8_last_error_message() describes the problem (thread-local).
 *  - All tensors are dense row-major with the innermost dimension contiguous.
 *  - Activations: dtype FNI8_F16 or FNI8_BF16. Weights: int8 [N, K] (out_features x
 *    in_features, K contiguous) with one fp32 scale per output row (`per_row_i8`).
 *  - Per-token activation quantisation: scale[m] = absmax(x[m, :]) / 127 (fp32),
 *    q = round_half_even(x * (127 / absmax)) clamped to [-127, 127] (one reciprocal
 *    per row, fp32); an all-zero row gets scale 0 and q = 0.
 *  - Dequant epilogue (fp32, evaluated left to right, no fused multiply-add):
 *    y = (float(acc) * a_scale[m]) * w_scale[n] (+ bias[n]) (+ residual[m, n]),
 *    rounded once to the output dtype.
 *  - K must be a multiple of 16 for the GEMMs (TMA row-stride rule); the quantisers
 *    accept any K. A caller with other K pads K with zeros in both operands (exact:
 *    zero channels change neither the int32 sums nor a token's absmax).
 *  - Calls are asynchronous on `stream`, allocate nothing and never synchronise, so
 *    they can be captured into a CUDA graph. Calls that share a workspace must not
 *    overlap on the GPU.
 *  - Any host thread may call any entry point, concurrently with others: the one-time
 *    setup (kernel attributes, cluster-occupancy plans, the tensor-map encoder) is
 *    guarded, and the error message is per thread.
 */
#ifndef FNI8_B200_H
#define FNI8_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FNI8_ABI_VERSION 1

#if defined(__GNUC__)
#define FNI8_API __attribute__((visibility("default")))
#else
#define FNI8_API
#endif

enum fni8_status {
  FNI8_OK = 0,
  FNI8_ERR_INVALID = 1,       /* bad pointer, shape, dtype or flag */
  FNI8_ERR_UNSUPPORTED = 2,   /* valid request this build does not implement */
  FNI8_ERR_ALIGN = 3,         /* pointer / stride alignment the kernels need */
  FNI8_ERR_CUDA = 4,          /* a CUDA runtime call failed */
  FNI8_ERR_WORKSPACE = 5,     /* workspace missing or too small */
  FNI8_ERR_DEVICE_TIMEOUT = 6 /* a bounded device-side wait gave up (fni8_device_status) */
};

enum fni8_dtype { FNI8_F16 = 0, FNI8_BF16 = 1, FNI8_F32 = 2, FNI8_I32 = 3, FNI8_I8 = 4 };
enum fni8_act { FNI8_ACT_SILU = 0, FNI8_ACT_GELU_TANH = 1 };
enum fni8_scoring { FNI8_SCORE_SOFTMAX = 0, FNI8_SCORE_SIGMOID = 1 };
/* GEMM kernel selection (fni8_gemm_w8a8_ex). AUTO picks by shape. */
enum fni8_gemm_path {
  FNI8_PATH_AUTO = 0,   /* by shape, from B200 measurements */
  FNI8_PATH_TILE = 1,   /* tcgen05 tile kernel, 128-row activation tiles */
  FNI8_PATH_STREAM = 2, /* swap-AB stream-K kernel for M <= 256 (uses the workspace) */
  FNI8_PATH_FUSED = 3,  /* reserved: not built (returns FNI8_ERR_UNSUPPORTED) */
  FNI8_PATH_SPLITK = 4  /* swap-AB cluster split-K kernel for M <= 256 (uses the workspace) */
};

/* ------------------------------------------------------------------ library */
FNI8_API int fni8_abi_version(void);
FNI8_API const char* fni8_status_string(int status);
FNI8_API const char* fni8_last_error_message(void);
/* Reads and clears the device-side watchdog words of the current device. *code_out
 * receives 0 when no bounded wait has timed out since the last call. Synchronises.
 * A non-zero code (returned with FNI8_ERR_DEVICE_TIMEOUT) means a kernel left its loop
 * early and its results are void; the call then re-zeroes the built-in scratch of
 * fni8_gemm_w8a8_noalloc on the current device. A caller-provided GEMM workspace may
 * hold partial sums of the abandoned kernel: zero it again (fni8_workspace_init)
 * before its next use. */
FNI8_API int fni8_device_status(int* code_out);
/* Test hook for the failure-detection path (no counterpart in the reference, whose
 * kernels have no bounded waits): launches one warp on `stream` that waits on a device
 * flag nothing ever sets. The wait gives up after wait_us microseconds (1 .. 1000000),
 * records watchdog code 0x2F0 for fni8_device_status and the kernel ends; with
 * dirty_scratch == 0 no GPU state beyond the status word changes. Otherwise the warp first fills the
 * built-in scratch of fni8_gemm_w8a8_noalloc with non-zero words, as a stream-K
 * reduction abandoned by a timed-out wait would leave it, so a test can check that
 * fni8_device_status restores it. Any in-flight call of fni8_gemm_w8a8_noalloc on the
 * device races with it. */
FNI8_API int fni8_watchdog_selftest(int64_t wait_us, int dirty_scratch, void* stream);

/* ------------------------------------------------------------------ quantisers */
/* Per-token absmax int8 quantisation of x[M, K]: the activation stage inside
 * fni8.linear (fni8serve/layers/linear.py:2-13,69). */
FNI8_API int fni8_quantize_rows_i8(const void* x, int dtype, int64_t M, int64_t K, int8_t* q, float* scale,
                          void* stream);

/* fni8_quantize_rows_i8 over the first *rows_dev rows of x[M, K] (M is their upper bound;
 * the count lives in device memory, e.g. the rows an expert-parallel rank received; rows past
 * it are left untouched). K a multiple of 8 (<= 16384), 16-byte aligned rows. */
FNI8_API int fni8_quantize_rows_i8_rows(const void* x, int dtype, int64_t M, int64_t K, const int32_t* rows_dev,
                                        int8_t* q, float* scale, void* stream);

/* RMSNorm over the last dim: replaces fni8.rmsnorm (fni8serve/layers/norm.py:38-58).
 * y = dtype((x_f32 * (1/sqrt(mean(x_f32^2) + eps))) * g), g = w or (1 + w) when
 * unit_offset. With residual != NULL the input is x + residual (rounded to dtype), which
 * is also written to residual_out. */
FNI8_API int fni8_rmsnorm(const void* x, const void* residual, const void* weight, int dtype, int64_t M, int64_t K,
                 float eps, int unit_offset, void* out, void* residual_out, void* stream);

/* Fused RMSNorm -> per-token int8 quantisation (one pass over HBM). Emits the int8 rows
 * and scales exactly as fni8_quantize_rows_i8 would on the rounded RMSNorm output;
 * `out` (the rounded normed rows) is optional (NULL skips the store). */
FNI8_API int fni8_rmsnorm_quant_i8(const void* x, const void* residual, const void* weight, int dtype, int64_t M,
                          int64_t K, float eps, int unit_offset, void* out, void* residual_out, int8_t* q,
                          float* scale, void* stream);

/* act(x[:, :I]) * x[:, I:] for x[M, 2I]: replaces fni8.act_and_mul
 * (fni8serve/layers/activation.py:21-25,37-41): act(gate) in fp32 rounded to dtype, times
 * up in fp32, rounded to dtype (the reference's F.silu(gate) * up on fp16 tensors). */
FNI8_API int fni8_act_and_mul(const void* x, int dtype, int act, int64_t M, int64_t I, void* out, void* stream);

/* Fused act_and_mul -> per-token int8 quantisation of the rounded result (the input of
 * down_proj in GatedMLP.forward, fni8serve/layers/mlp.py:39-40). */
FNI8_API int fni8_act_and_mul_quant_i8(const void* x, int dtype, int act, int64_t M, int64_t I, int8_t* q, float* scale,
                              void* stream);
/* Both at once: out[M, I] = act_and_mul(x) and its per-token int8 rows q[M, I] / scale[M]
 * (the q of fni8_act_and_mul_quant_i8), in one pass over x. fni8.act_and_mul uses it to hand
 * the int8 rows to the down projection that consumes `out` (GatedMLP.forward,
 * fni8serve/layers/mlp.py:39-40). */
FNI8_API int fni8_act_and_mul_dual(const void* x, int dtype, int act, int64_t M, int64_t I, void* out, int8_t* q,
                                   float* scale, void* stream);
/* fni8_act_and_mul_quant_i8 over the first *rows_dev rows of x[M, 2I] (M is their upper
 * bound; the count lives in device memory, e.g. the rows an expert-parallel rank received;
 * rows past it are left untouched). */
FNI8_API int fni8_act_and_mul_quant_i8_rows(const void* x, int dtype, int act, int64_t M, int64_t I,
                                            const int32_t* rows_dev, int8_t* q, float* scale, void* stream);

/* ------------------------------------------------------------------ dense GEMM */
/* Bytes of workspace fni8_gemm_w8a8* may use for an M x N x K problem (0 when none). */
FNI8_API size_t fni8_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);
/* Zero a workspace once before first use; the GEMM kernels leave it zeroed again. */
FNI8_API int fni8_workspace_init(void* workspace, size_t bytes, void* stream);

/* out[M, N] = dequant(a[M, K] . w[N, K]^T): the int8 GEMM + epilogue inside
 * fni8.linear (fni8serve/layers/linear.py:67-69). bias [N] and residual [M, N] are
 * optional and in out_dtype (F16 or BF16). */
FNI8_API int fni8_gemm_w8a8(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                   const void* bias, const void* residual, void* out, int out_dtype, int64_t M, int64_t N,
                   int64_t K, void* workspace, size_t workspace_bytes, void* stream);

/* Same with an explicit kernel choice (enum fni8_gemm_path). */
FNI8_API int fni8_gemm_w8a8_ex(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                      const void* bias, const void* residual, void* out, int out_dtype, int64_t M, int64_t N,
                      int64_t K, int path, void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free form of fni8_gemm_w8a8 for decode-sized problems. No counterpart in
 * the reference. For callers that cannot allocate device memory (an engine that has
 * reserved all of HBM up front, or a host reaching this library through a bare FFI with
 * no device allocator): instead of a caller-provided workspace it uses a 4 MiB scratch
 * array built into the library, which every GPU that loads the library holds until the
 * process exits. Takes M <= 32 rows (larger M, or an N/K split that would need more than
 * 4 MiB, returns FNI8_ERR_UNSUPPORTED) and calls no allocator. The first call on a device
 * looks up the array's address and zeroes it on `stream`; make that first call before
 * any stream capture. CUDA loads a library's modules lazily by default, so the array's
 * 4 MiB are taken on a device at that first call (or the first use of any stream-K
 * kernel there): make it before the engine reserves all of HBM, or run with
 * CUDA_MODULE_LOADING=EAGER. All calls on a device share the array: calls that overlap on
 * the GPU (other streams, other threads) race and must be serialised by the caller. The
 * kernels leave the array zeroed after every completed call; after a watchdog timeout
 * fni8_device_status zeroes it again. */
FNI8_API int fni8_gemm_w8a8_noalloc(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                                    const void* bias, const void* residual, void* out, int out_dtype, int64_t M,
                                    int64_t N, int64_t K, void* stream);

/* GatedMLP's gate_up projection with act_and_mul applied in the GEMM epilogue
 * (fni8serve/layers/mlp.py:39-40 with layers/activation.py:21-45): w_gu [2I, K] int8 holds
 * the gate rows [0, I) and the up rows [I, 2I) in gate_up_weight's merge order
 * (fni8serve/models/weights.py:49-50), s_gu [2I] their fp32 scales. out[M, I] =
 * act(gate) * up in out_dtype, equal bit for bit to fni8_gemm_w8a8 into [M, 2I] followed
 * by fni8_act_and_mul, without the [M, 2I] intermediate. act: FNI8_ACT_SILU or
 * FNI8_ACT_GELU_TANH. I must be a multiple of 128 (FNI8_ERR_UNSUPPORTED otherwise), out
 * 16-byte aligned. Tile kernel: meant for prefill-sized M. */
FNI8_API int fni8_gemm_w8a8_act(const int8_t* a, const float* a_scale, const int8_t* w_gu, const float* s_gu, int act,
                                void* out, int out_dtype, int64_t M, int64_t I, int64_t K, void* stream);

/* Raw int32 accumulators acc[M, N] = a . w^T (the int8 x int8 -> int32 matmul of the
 * reference's gemm_w8a8; used for the bit-exact check). */
FNI8_API int fni8_gemm_w8a8_i32(const int8_t* a, const int8_t* w, int32_t* acc, int64_t M, int64_t N, int64_t K, int path,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Whole fni8.linear(x, qt, bias=) (fni8serve/layers/linear.py:67-69) for per_row_i8:
 * quantise x[M, K] per token into q_scratch[M, K] / s_scratch[M], then the W8A8 GEMM
 * with dequant epilogue into out[M, N] (dtype of x). `workspace` is the zero-maintained
 * GEMM workspace (fni8_gemm_workspace_bytes). */
FNI8_API int fni8_linear_w8a8(const void* x, int dtype, const int8_t* w, const float* w_scale, const void* bias,
                              void* out, int64_t M, int64_t N, int64_t K, int8_t* q_scratch, float* s_scratch,
                              void* workspace, size_t workspace_bytes, void* stream);
/* Same with an explicit kernel choice (enum fni8_gemm_path). */
FNI8_API int fni8_linear_w8a8_ex(const void* x, int dtype, const int8_t* w, const float* w_scale, const void* bias,
                                 void* out, int64_t M, int64_t N, int64_t K, int8_t* q_scratch, float* s_scratch,
                                 int path, void* workspace, size_t workspace_bytes, void* stream);

/* W4A8: int8 activations a[M, K] (+ per-token scale) x 4-bit weights — the per_group_i4 /
 * int4 QTensor of fni8serve (layers/linear.py:33-45, convert.py:69-80): w4[N, K/2] bytes,
 * element 2j of a row in the low nibble of byte j, signed two's complement; w_scale[N, K/g]
 * fp32 per group of g input channels. out[m, n] = dtype((sum_g float(acc_g[m, n]) *
 * w_scale[n, g]) * a_scale[m] (+ bias[n])), acc_g the exact int32 sum over group g.
 * Takes group_size 128 and K a multiple of 128 (FNI8_ERR_UNSUPPORTED otherwise); the
 * workspace is the zero-maintained GEMM workspace (fni8_gemm_workspace_bytes). The fp32
 * sum over the groups of a split K range is formed per K slice, then over the slices in
 * order: the result can differ from a one-pass sum in the last fp16 bit. */
FNI8_API int fni8_gemm_w4a8(const int8_t* a, const float* a_scale, const uint8_t* w4, const float* w_scale,
                            int64_t group_size, const void* bias, void* out, int out_dtype, int64_t M, int64_t N,
                            int64_t K, void* workspace, size_t workspace_bytes, void* stream);
/* fni8.linear(x, qt, bias=) for per_group_i4 / int4 weights: per-token int8 quantisation of
 * x into q_scratch / s_scratch, then fni8_gemm_w4a8. */
FNI8_API int fni8_linear_w4a8(const void* x, int dtype, const uint8_t* w4, const float* w_scale, int64_t group_size,
                              const void* bias, void* out, int64_t M, int64_t N, int64_t K, int8_t* q_scratch,
                              float* s_scratch, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ MoE */
/* Router scores -> top-k (SparseMoE.forward routing, fni8serve/models/moe.py:65-95):
 * softmax over all E (or sigmoid + optional selection bias added for the choice only),
 * optional group-limited selection (n_groups > 0), top-k (ties -> lower expert id),
 * optional renormalisation (sum clamped to >= 1e-9), times `scaling`, then rounded to
 * weight_dtype (FNI8_F16 / FNI8_BF16, as the reference casts to x.dtype; FNI8_F32 keeps
 * fp32). E <= 1024, top_k <= 32. */
FNI8_API int fni8_moe_route(const float* logits, int64_t T, int64_t E, int64_t top_k, int scoring, const float* sel_bias,
                   int64_t n_groups, int64_t topk_group, int norm_topk, float scaling, int weight_dtype,
                   int32_t* topi, float* topw, void* stream);

/* Stable grouping of the T*k (token, slot) pairs by expert: counts[E], offsets[E+1]
 * (exclusive scan), row_of_slot[T*k] (slot = t*k + j -> grouped row; -1 for an expert id
 * outside [0, E), which is dropped) and slot_of_row[offsets[E]]. Rows of one expert keep
 * slot order, so the grouping is deterministic. Uses fni8_moe_plan_workspace_bytes(T*k, E)
 * bytes of workspace (no zeroing needed). E <= 1024. */
FNI8_API size_t fni8_moe_plan_workspace_bytes(int64_t n_slots, int64_t E);
FNI8_API int fni8_moe_plan(const int32_t* topi, int64_t n_slots, int64_t E, int32_t* counts, int32_t* offsets,
                  int32_t* row_of_slot, int32_t* slot_of_row, void* workspace, size_t workspace_bytes,
                  void* stream);

/* Per-token int8 quantisation of x[T, K] (as fni8_quantize_rows_i8) whose rows go straight
 * to the expert-grouped order of fni8_moe_plan: token t's codes are written to row
 * row_of_slot[t * top_k + j] of q_out (and its scale to scale_out) for every slot j the plan
 * placed (entries < 0 are skipped). The quantise-then-gather of the reference's
 * `xf[tok_idx]` (fni8serve/models/moe.py:103) in one pass over x. K % 16 == 0, K <= 16384,
 * 16-byte aligned rows. */
FNI8_API int fni8_moe_quantize_scatter_i8(const void* x, int dtype, int64_t T, int64_t K, const int32_t* row_of_slot,
                                          int64_t top_k, int8_t* q_out, float* scale_out, void* stream);

/* q_out[r] = q[slot_of_row[r] / top_k], scale_out likewise (int8 row gather). */
FNI8_API int fni8_moe_gather_rows_i8(const int8_t* q, const float* scale, const int32_t* slot_of_row, int64_t R, int64_t K,
                            int64_t top_k, int8_t* q_out, float* scale_out, void* stream);

/* Grouped W8A8 GEMM over S row segments of a[R, K]: segment s covers rows
 * [seg_off[s], seg_off[s] + seg_cnt[s]) and multiplies them by expert seg_expert[s] of
 * w[E, N, K] (scales w_scale[E, N]); out[R, N] in out_dtype. The per-expert GEMMs of
 * the SparseMoE loop (fni8serve/models/moe.py:99-105) in one persistent launch.
 * The segment arrays live in device memory (S <= 512). */
FNI8_API int fni8_grouped_gemm_w8a8(const int8_t* a, const float* a_scale, int64_t R, const int8_t* w, const float* w_scale,
                           int64_t E, int64_t N, int64_t K, const int32_t* seg_expert, const int32_t* seg_off,
                           const int32_t* seg_cnt, int64_t S, void* out, int out_dtype, void* stream);

/* The grouped gate_up projection of the expert loop with act_and_mul in its epilogue:
 * segment s multiplies rows [seg_off[s], seg_off[s] + seg_cnt[s]) of a[R, K] by expert
 * seg_expert[s] of w_gu [E, 2I, K] (gate rows [0, I), up rows [I, 2I) per expert, fp32
 * scales s_gu [E, 2I]) and writes act(gate) * up to out[R, I] (the GatedMLP inside each
 * expert, fni8serve/models/moe.py:103, layers/mlp.py:39-40); equal bit for bit to
 * fni8_grouped_gemm_w8a8 into [R, 2I] followed by fni8_act_and_mul. I % 128 == 0. */
FNI8_API int fni8_grouped_gemm_w8a8_act(const int8_t* a, const float* a_scale, int64_t R, const int8_t* w_gu,
                                        const float* s_gu, int64_t E, int64_t I, int64_t K, const int32_t* seg_expert,
                                        const int32_t* seg_off, const int32_t* seg_cnt, int64_t S, int act, void* out,
                                        int out_dtype, void* stream);

/* fni8_grouped_gemm_w8a8 whose output rows go to other buffers: row r (of a segment) is
 * stored as row (row_tag[r] & 0xFFFFFF) of peer_out[row_tag[r] >> 24], a [peer_rows, N]
 * buffer of that rank mapped into this process (fni8_ipc_open; this rank's own at its
 * index). With the tags of fni8_ep_dispatch_i8, the down projection of an expert-parallel
 * layer stores each expert output straight into its source rank's back buffer over NVLink, tile
 * by tile while later tiles compute: the return step of fni8_ep_return fused into the GEMM
 * epilogue. Rows leave 4 rows x 128 contiguous bytes per store instruction; a tag outside
 * the buffers is skipped and reported by fni8_device_status. out_dtype F16 or BF16,
 * N % 64 == 0. */
FNI8_API int fni8_grouped_gemm_w8a8_scatter(const int8_t* a, const float* a_scale, int64_t R, const int8_t* w,
                                            const float* w_scale, int64_t E, int64_t N, int64_t K,
                                            const int32_t* seg_expert, const int32_t* seg_off,
                                            const int32_t* seg_cnt, int64_t S, const int32_t* row_tag,
                                            void* const* peer_out, int64_t world, int64_t peer_rows, int out_dtype,
                                            void* stream);

/* out[t] = sum_j topw[t, j] * y[row_of_slot[t*k + j]] in fp32, rounded once: the
 * weighted index_add_ combine (fni8serve/models/moe.py:97,105). */
FNI8_API int fni8_moe_combine(const void* y, int dtype, const int32_t* row_of_slot, const float* topw, int64_t T,
                     int64_t top_k, int64_t H, void* out, void* stream);
/* Routed-expert block of SparseMoE on one GPU (fni8serve/models/moe.py:97-105) given
 * the routing: quantise x, group, gate_up grouped GEMM, act_and_mul + quant, down
 * grouped GEMM, weighted combine. w_gu [E, 2I, H], w_dn [E, H, I] int8 with per-row
 * fp32 scales s_gu [E, 2I], s_dn [E, H]. */
FNI8_API size_t fni8_moe_experts_workspace_bytes(int64_t T, int64_t H, int64_t top_k, int64_t E, int64_t I);
FNI8_API int fni8_moe_experts_w8a8(const void* x, int dtype, int64_t T, int64_t H, const int32_t* topi, const float* topw,
                          int64_t top_k, const int8_t* w_gu, const float* s_gu, const int8_t* w_dn,
                          const float* s_dn, int64_t E, int64_t I, int act, void* out, void* workspace,
                          size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------ expert-parallel exchange
 * New capability: the reference runs every expert on one GPU (fni8serve/models/moe.py:99-105)
 * and forbids tensor parallelism (fni8serve/config.py:40-45). One process per GPU; rows move
 * between GPUs as stores into peer memory mapped with CUDA IPC. No function here waits on
 * another GPU: after each exchange the caller orders the ranks with a collective on the
 * same stream (every rank passes it only once every rank's exchange has completed). */
#define FNI8_IPC_HANDLE_BYTES 64
/* cudaMalloc'd, zeroed device buffer of `bytes` and its IPC handle (FNI8_IPC_HANDLE_BYTES
 * bytes into `handle`); fni8_ipc_free releases it. */
FNI8_API int fni8_ipc_alloc(size_t bytes, void** ptr, void* handle);
FNI8_API int fni8_ipc_free(void* ptr);
/* Map a peer process's buffer from its handle (peer access enabled on first use);
 * fni8_ipc_close unmaps it. */
FNI8_API int fni8_ipc_open(const void* handle, void** ptr);
FNI8_API int fni8_ipc_close(void* ptr);

/* Barrier of the `world` ranks of one node over peer memory, on `stream` (no host wait):
 * each rank passes it once every rank has reached it, and then sees every store into its
 * memory that the other ranks' kernels issued before their barrier. peer_flags: `world`
 * pointers to each rank's flag words (world uint32 in memory mapped with fni8_ipc_open,
 * zeroed once; this rank's own at index rank); epoch: a uint32 counter in this rank's
 * device memory, zeroed once (every rank runs the same sequence of barriers). With n > 0
 * the barrier also all-gathers n int32 words: src [n] of this rank lands at words
 * [rank * n, rank * n + n) of every rank's peer_dst buffer. A rank that has not arrived
 * after wait_us microseconds (1 .. 1e6) is reported by fni8_device_status and the kernel
 * returns; no GPU waits for good. Replaces an NCCL all_reduce / all_gather used only as a
 * barrier between the kernels of an expert-parallel or column-parallel layer. */
FNI8_API int fni8_peer_barrier(void* const* peer_flags, int64_t world, int64_t rank, uint32_t* epoch,
                               const int32_t* src, int64_t n, void* const* peer_dst, int64_t wait_us, void* stream);

/* Expert ids through a placement: out[i] = map[ids[i]] for ids[i] in [0, E), else ids[i]
 * (n ids, map [E]). With map[e] = the slot (rank * E/world + local index) that a
 * load-balanced placement gives expert e, the routing of every token addresses the ranks'
 * local experts; out may equal ids. */
FNI8_API int fni8_moe_map_ids(const int32_t* ids, int64_t n, const int32_t* map, int64_t E, int32_t* out,
                              void* stream);

/* Placement of one exchange on the device, from cnt_all [world, E] (rows each source rank
 * sends to each expert; expert e lives on rank e / (E / world)): rank d's receive buffer
 * holds its local experts one after another, each expert's rows ordered by source rank.
 * Writes dst_base [world * E/world] (where this rank's rows of (owner d, local expert el)
 * start in d's buffer, as fni8_ep_dispatch_i8 takes it), this rank's received segments
 * seg_off / seg_cnt [E/world] and their total n_recv [1]. One small kernel. */
FNI8_API int fni8_ep_placement(const int32_t* cnt_all, int64_t world, int64_t rank, int64_t E, int32_t* dst_base,
                               int32_t* seg_off, int32_t* seg_cnt, int32_t* n_recv, void* stream);

/* Dispatch: the sorted rows of fni8_moe_plan (slot_of_row, offsets[E + 1]) to the ranks
 * owning their experts (expert e lives on rank e / (E / world)). Row r of local expert el
 * of rank d goes to position dst_base[d * (E / world) + el] + (r - offsets[e]) of rank d's
 * receive buffers: the int8 row q[slot / top_k] (H bytes) into peer_q[d], its scale into
 * peer_scale[d] and the tag (rank << 24 | r) into peer_tag[d]. peer_* are `world` device
 * pointers (this rank's own buffers at index rank); cap_rows is the rows each receive
 * buffer holds (a row past it is skipped and reported by fni8_device_status); max_rows
 * bounds the sorted rows (T * top_k, < 2^24). */
FNI8_API int fni8_ep_dispatch_i8(const int8_t* q, const float* scale, const int32_t* slot_of_row,
                                 const int32_t* offsets, int64_t E, int64_t world, int64_t rank, int64_t top_k,
                                 int64_t H, const int32_t* dst_base, void* const* peer_q, void* const* peer_scale,
                                 void* const* peer_tag, int64_t cap_rows, int64_t max_rows, void* stream);
/* Return: row i < *n_recv of y[cap_rows, H] (dtype) goes to row (tag[i] & 0xFFFFFF) of the
 * back buffer of rank tag[i] >> 24 (peer_back: `world` device pointers to [back_rows, H]
 * buffers): the source's sorted row r, so that rank combines its tokens with
 * fni8_moe_combine over its own row_of_slot. */
FNI8_API int fni8_ep_return(const void* y, int dtype, const int32_t* n_recv, int64_t cap_rows, const int32_t* tag,
                            int64_t H, int64_t world, void* const* peer_back, int64_t back_rows, void* stream);

/* ------------------------------------------------------------------ column-parallel linear
 * New capability (the reference forbids tensor parallelism, fni8serve/config.py:40-45): a
 * dense W8A8 linear with its output channels sharded over the ranks, each rank's slice
 * all-gathered into every rank's full output without a separate collective.
 *
 * y = dequant(a[M, K] . w[N, K]^T) for this rank's N output columns (the fni8_gemm_w8a8
 * epilogue: a_scale [M], w_scale [N], optional bias [N]; out_dtype F16 or BF16), with element
 * (m, n) stored to element (m, col_off + n) of every buffer peer_out[0 .. n_peers) (row stride
 * ld elements; this rank's own buffer and its NVLink peers' buffers mapped with
 * fni8_ipc_open, n_peers <= 8). Prefill sizes run the tile GEMM with these stores in its
 * epilogue, so the slices cross NVLink tile by tile while later tiles compute; decode sizes
 * run the split-K GEMM into tmp [M, N] (tmp_bytes >= M * N * 2) and then one kernel that
 * copies it into the buffers. ws / ws_bytes: the GEMM workspace (fni8_gemm_workspace_bytes,
 * zeroed once). Buffers 16-byte aligned, ld and col_off multiples of 8, N a multiple of 64,
 * K of 16. No rank is waited for: the caller orders the ranks (a collective on the same
 * stream) before any of them reads its buffer. */
FNI8_API int fni8_gemm_w8a8_peer_cols(const int8_t* a, const float* a_scale, const int8_t* w, const float* w_scale,
                                      const void* bias, int out_dtype, int64_t M, int64_t N, int64_t K,
                                      void* const* peer_out, int n_peers, int64_t ld, int64_t col_off, void* tmp,
                                      size_t tmp_bytes, void* ws, size_t ws_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FNI8_B200_H */
