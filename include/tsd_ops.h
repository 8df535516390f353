/* tsd_ops.h — operator-level C-ABI of libtsd_b200 (device pointers, caller's stream).
 *
 * The kernels the MM-DiT forward is built from, exposed for parity tests and for callers that
 * assemble their own graphs. Each replaces a GGML node group of src/mmdit.cpp in
 * pwilkin/thinksound.cpp (cited per entry). All pointers are device memory; `stream` is a
 * cudaStream_t (NULL = legacy default stream); calls are asynchronous. `err` is an optional
 * device int that a kernel sets to a non-zero code if one of its bounded waits expires.
 * Return: TSD_OK or a TSD_ERR_* code from tsd.h.
 */
#ifndef TSD_OPS_H
#define TSD_OPS_H

#include <stdint.h>

#ifndef TSD_API
#if defined(__GNUC__)
#define TSD_API __attribute__((visibility("default")))
#else
#define TSD_API
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Epilogue modes of tsd_op_gemm. */
#define TSD_EPI_STORE 0       /* out = act(acc + bias), f32 or bf16 */
#define TSD_EPI_SWIGLU 1      /* out[f] = silu(acc[2f]) * acc[2f+1]: W rows alternate w1 / w3; no bias */
#define TSD_EPI_GATE_RESID 2  /* resid += gate * (acc + bias) */
#define TSD_ACT_NONE 0
#define TSD_ACT_SILU 1

/* tcgen05 GEMM / implicit conv (replaces `lin` mmdit.cpp:12-16, `conv1d_f32`/`conv_cl` :20-34,
 * SwiGLU of `convmlp`/`mlp` :39-52, gate+residual :231,:234):
 *   acc[b][t][m] = sum_tap sum_k X[b][t + tap - pad][k] * W[m][tap*K_in + k]
 * W bf16 [M][taps*K_in]; X bf16 rows with the given row / batch strides (elements);
 * out row index b*S + t. M multiple of 128 (256 for SWIGLU), K_in multiple of 64.
 * GATE_RESID reads gate row (out row / gate_div): 1 for a per-token gate, S for one per item.
 * Split-K (max_splits > 1) needs scratch from the caller: `ws` (ws_floats floats) for partial
 * tiles and `counters` (n_counters ints, zero before the first call; the kernel leaves them
 * zero). Partials are summed in a fixed order, so results do not depend on timing. With
 * ws == NULL the GEMM runs without splitting K. */
TSD_API int tsd_op_gemm(const void * W, int M, int K_in, int taps, int pad, const void * X, int nbatch, int S,
                int64_t x_row_stride, int64_t x_batch_stride, int mode, int act, const float * bias, int m_valid,
                void * out, int out_bf16, int64_t ldo, float * resid, int64_t ldr, const float * gate, int64_t ldg,
                int gate_div, int max_splits, float * ws, int64_t ws_floats, int * counters, int n_counters,
                int * err, void * stream);

/* tsd_op_gemm for callers that cannot allocate device memory (no counterpart in the
 * reference): same arguments, and the same tiling and results as tsd_op_gemm given
 * TSD_GEMM_STATIC_WS_FLOATS floats and TSD_GEMM_STATIC_COUNTERS counters of scratch, but that
 * scratch is a pair of fixed file-scope device arrays in the library (8 MB + 32 KB, held by
 * every GPU that loads the library until exit), so the call performs no cudaMalloc/cudaFree.
 * Shapes whose best split-K plan would need more scratch run with fewer K splits (the planner
 * keeps every plan within the arrays); a plan beyond them is rejected with TSD_ERR_ARG and a
 * message. The first call on a device (and the first after its context is recreated) looks up
 * the arrays' addresses: make it before any stream capture. All calls on a device share the
 * arrays, which keep the last call's contents: calls that overlap on the GPU race. */
#define TSD_GEMM_STATIC_WS_FLOATS 2097152
#define TSD_GEMM_STATIC_COUNTERS 8192
TSD_API int tsd_op_gemm_static(const void * W, int M, int K_in, int taps, int pad, const void * X, int nbatch, int S,
                               int64_t x_row_stride, int64_t x_batch_stride, int mode, int act, const float * bias,
                               int m_valid, void * out, int out_bf16, int64_t ldo, float * resid, int64_t ldr,
                               const float * gate, int64_t ldg, int gate_div, int max_splits, int * err, void * stream);

/* The tiling tsd_op_gemm would choose for a GEMM shape given `ws_floats` / `n_counters` of
 * scratch (no launch; for tests and tuning). out[0] token tile, out[1] K splits, out[2] 1 for
 * CTA pairs, out[3] 1 if the splits reduce inside a thread-block cluster (no scratch), out[4]
 * scratch floats the plan needs (non-zero only for split-K through global memory), out[5] 1 if,
 * with one tile per CTA, the split that completes a tile last gathers the other splits' partials
 * from the scratch into its shared memory (else a reducer reads them there). Needs the GPU the
 * GEMM would run on to be current (cluster occupancy is a property of the device). */
TSD_API int tsd_op_gemm_plan(int M, int K_in, int taps, int nbatch, int S, int max_splits, int64_t ws_floats,
                             int n_counters, int64_t out[6]);

/* The head-parallel arrival wait (tsd_hp_* in tsd.h) as an operator: one warp waits until
 * counters[r] >= *epoch * ctas for every rank r != rank of `world`, bounded by the wait limit
 * (tsd_set_wait_limit); on expiry it sets *err (if non-NULL) to a non-zero code and returns.
 * counters and epoch are device memory. Used to test the error path of the exchange. */
TSD_API int tsd_op_peer_wait(const uint32_t * counters, const uint32_t * epoch, int rank, int world, uint32_t ctas,
                             int * err, void * stream);

/* Few-token GEMV with weights in their stored ggml type (0 F32, 30 BF16, 8 Q8_0), N <= 8
 * (the [H,1]-column mul_mats of mmdit.cpp:158-160,185-192,209). W2 != NULL: SwiGLU pair. */
TSD_API int tsd_op_gemv(const void * W, int ggml_type, const void * W2, int M, int K, const float * x, int64_t ldx, int N,
                const float * bias, int act, int round_bf16, void * y, int y_bf16, int64_t ldy, void * stream);

/* tcgen05 flash attention (replaces `attention` mmdit.cpp:85-94): Q, K, V fp16 [B*nh][S][64];
 * out bf16 token-major out[b][t][h*64+d] with row stride ldo (elements). */
TSD_API int tsd_op_attention(const void * Q, const void * K, const void * V, int B, int nh, int S, void * out, int64_t ldo,
                     int * err, void * stream);

/* tsd_op_attention with f32 output (same kernel and arithmetic; the output is not rounded to
 * bf16), for parity checks of the attention itself. out[b][t][h*64+d], row stride ldo. */
TSD_API int tsd_op_attention_f32(const void * Q, const void * K, const void * V, int B, int nh, int S, float * out,
                                 int64_t ldo, int * err, void * stream);

/* LayerNorm (eps 1e-5, no affine) + modulate x*(1+scale)+shift (mmdit.cpp:55-59,218,232):
 * x f32 [rows][H] -> y bf16; shift/scale row = row (per_token) or row / rows_per_item. */
TSD_API int tsd_op_ln_modulate(const float * x, int rows, int H, const float * shift, const float * scale, int64_t ld_mod,
                       int per_token, int rows_per_item, void * y, void * stream);

/* split_qkv + QK RMSNorm (eps 1e-6, gain) + RoPE NORMAL + F16 cast (mmdit.cpp:67-100,219-223):
 * qkv f32 [B][S][3H] with Q|K|V column blocks -> fp16 head-major [B][nh][Sj][64] at row s_off. */
TSD_API int tsd_op_qk_norm_rope(const float * qkv, int B, int S, int H, int nh, const float * q_gain, const float * k_gain,
                        int rope, float freq_scale, float theta, void * Q, void * K, void * V, int Sj, int s_off,
                        void * stream);

/* Per-op profile of one forward on device-resident inputs (arguments as tsd_forward_device, in
 * tsd.h): the forward's ops run one by one with CUDA events between them (no graph) and, for
 * up to max_ops ops, report kind (0 tcgen05 GEMM, 1 GEMV, 2 attention, 3 other kernel,
 * 4 memset/copy), kernel launches, milliseconds, algorithmic FLOPs and bytes.
 * *n_ops receives the number of ops of the forward. */
struct tsd_model;
TSD_API int tsd_forward_profile(struct tsd_model * m, int B, const float * latent, int64_t T, const float * t,
                                const float * clip_f, int64_t clip_S, const float * sync_f, int64_t sync_S,
                                const float * text_f, int64_t text_S, const float * t5, int64_t t5_S,
                                const float * global_text, float * flow_out, void * stream, int max_ops, int * n_ops,
                                int * kind, int * launches, float * ms, double * flops, double * bytes);
/* Label of op i of the model's current forward plan (stage, kind, GEMM shape and grid), or
 * NULL if there is no plan or i is out of range. Valid until the plan is rebuilt. */
TSD_API const char * tsd_plan_op_label(struct tsd_model * m, int i);

#ifdef __cplusplus
}
#endif

#endif /* TSD_OPS_H */
