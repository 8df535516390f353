// kernels.h — host-side launch interface of the sm_100a kernels (internal to libtsd_b200).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace tsd {

// Host-side setter of one translation unit's copy of the device wait limit (common.cuh);
// every copy registers itself at load time (list kept in capi.cu, used by tsd_set_wait_limit).
using WaitLimitSetter = cudaError_t (*)(unsigned long long);
int register_wait_limit_setter(WaitLimitSetter fn);

// ---------------------------------------------------------------------------------------------
// tcgen05 GEMM:  out[b][t][m] = epi( sum_tap sum_k  X[b][t + tap - pad][k] * W[m][tap*K_in + k] )
//   W: bf16, [M rows][taps*K_in] (tap-major columns), via a 2-D tensor map (box 64 x 128*numA).
//   X: bf16 activations, [nbatch][S][K_in] with arbitrary row / batch strides, via a 3-D tensor
//      map (box 64 x BN x 1). Rows outside [0, S) of an item read as zero (conv padding).
// Persistent CTAs walk 128-feature x BN-token output tiles (SwiGLU: 64 w1 + 64 w3 rows per tile).
// ---------------------------------------------------------------------------------------------
enum EpiMode : int {
    EPI_STORE = 0,       // out = act(acc + bias)                       (f32 or bf16)
    EPI_SWIGLU = 1,      // out = silu(acc_w1) * acc_w3                  (bf16)
    EPI_GATE_RESID = 2,  // resid += gate * (acc + bias)                 (f32)
    EPI_QKV = 3,         // per-head RMSNorm (Q, K) + RoPE, fp16 head-major Q / K / V (no split-K)
};
enum Act : int { ACT_NONE = 0, ACT_SILU = 1 };

struct GemmParams {
    int M;             // weight rows (multiple of 128; one A tile = 128 rows)
    int mblocks;       // M / 128
    int order;         // tile walk: 0 m-block-major, 1 token-tile-major
    int S;             // tokens per batch item
    int nbatch;
    int K_in;          // input features per tap (multiple of 64)
    int taps, pad;
    int BN;            // token tile (multiple of 16, <= 256)
    int n_tiles;       // ceil(S / BN)
    int splits;        // split-K factor
    int stages;        // operand ring depth (set by gemm_plan from BN)
    int kpb;           // K blocks of 64 per operand stage (1 or 2; 2 halves the TMA instructions per K)
    int a_q8;          // weights are planar Q8_0 (int8 [M][K] + f16 scales [K/32][M]), dequantised in smem
    int mode, act;
    int m_valid;       // features >= m_valid are not stored (zero-padded weight rows)
    const float * bias;
    void * out; int out_bf16; long long ldo;       // out row = b*S + t
    int out_cblk; long long out_cstride;           // column blocking: feature m at (m / cblk) * cstride + m % cblk
    float * resid; long long ldr;
    const float * gate; long long ldg; int gate_div;   // gate row = out row / gate_div
    float * ws;        // split-K partials [out tile][split][BN][128] (splits > 1 and not csplit)
    int * counters;    // per out tile arrival counters, zero between launches
    int * err;
    // set by gemm_finalize:
    int vec;           // output buffers allow the split-K reducer's vector accesses
    int epi_tma;       // epilogue moves output (GATE_RESID: residual / gate) tiles with TMA
    int csplit;        // split-K through the cluster's shared memory (one wave; cluster = the splits of a tile)
    int pair;          // CTA pairs (cta_group::2): 256 weight rows x BN tokens per pair, each CTA loading its
                       // 128 rows and half the tokens; m-blocks even, no Q8_0 A, tile walk m-block-major
    int gather;        // split-K through the global workspace with one tile per CTA: the split that completes
                       // a tile last gathers the other partials into its idle operand stages
    int ipt;           // batch items per token tile: > 1 puts several short items side by side in one tile
                       // (single CTAs, no split), each in `bni` rows, so a weight tile is read once for all
    int bni;           // token rows per item of a multi-item tile (a multiple of 16, >= S)
    int groups;        // token tiles along the batch: nbatch, or ceil(nbatch / ipt)
    // EPI_QKV: W rows are [Q | K | V] (H each, feature = head * 64 + d); out row = item * s_item + t
    __half * q_out, * k_out, * v_out;   // [item][nh][Sj][64], this stream's tokens at s_off
    const float * qg, * kg;             // RMSNorm gains [64]
    const float2 * rope;                // (cos, sin) [s_item][32], or null (no RoPE)
    int hidden, nh, Sj, s_off, s_item;
};

struct GemmLaunch {
    CUtensorMap tmA, tmB;   // weights, activations
    CUtensorMap tmO, tmG;   // epilogue: output (GATE_RESID: residual) and per-token gate tiles
    CUtensorMap tmV;        // EPI_QKV: tmO / tmG / tmV = the stream's Q / K / V rows
    CUtensorMap tmS;        // planar Q8_0 weights: the scale plane (tmA then maps the int8 plane)
    GemmParams p;
    dim3 grid;          // persistent: min(tiles, SMs) CTAs
    bool finalized = false;
};

// Programmatic dependent launch on (default) unless TSD_NO_PDL is set to a non-zero value.
bool pdl_enabled();
// Launch with programmatic dependent launch (PDL) when enabled: the kernel may be scheduled while
// its predecessor in the stream finishes; it calls pdl_wait() before it touches global memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args &&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
}

// Tensor-map helpers (driver entry point resolved at first use).
bool make_tmap_2d(CUtensorMap * m, const void * ptr, CUtensorMapDataType dt, int esize,
                  uint64_t d0, uint64_t d1, uint64_t stride1_bytes, uint32_t b0, uint32_t b1);
bool make_tmap_3d(CUtensorMap * m, const void * ptr, CUtensorMapDataType dt, int esize,
                  uint64_t d0, uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
                  uint32_t b0, uint32_t b1, uint32_t b2);

// Fill `L` for a GEMM; returns false on unsupported arguments. W: bf16 [M][taps*K_in], or with
// q8_scales, the int8 plane of planar Q8_0 weights (taps == 1) and q8_scales = [K_in/32][M] f16.
// swiglu: W rows alternate w1 / w3
// (row 2f = w1 of feature f, row 2f + 1 = w3 of f) and the output has M / 2 features. Split-K (max_splits > 1) is
// reduces through the cluster's shared memory when the split tiles fit one wave (unless
// allow_cluster is false), else through a global workspace, used only if ws_floats / n_counters
// can hold the partials; the caller then sets p.ws and p.counters (counters zeroed once; the
// kernel leaves them zero).
bool gemm_plan(GemmLaunch & L, const void * W, int M, int K_in, int taps, int pad, int swiglu,
               const void * X, int nbatch, int S, long long x_row_stride, long long x_batch_stride,
               int num_sms, int max_splits, long long ws_floats = 0, int n_counters = 0, bool allow_cluster = true,
               int force_bn = 0, int force_splits = 0, const void * q8_scales = nullptr, int force_pair = -1);
// Up to max_out feasible (token tile, K splits, CTA pair) choices for a GEMM shape, best first by
// the cost model; force_bn / force_splits / force_pair in gemm_plan select one of them (plan-time
// autotuning). force_pair: -1 the model's choice, 0 single CTAs only, 1 the best pair choice.
int gemm_candidates(int M, int K_in, int taps, int nbatch, int S, int num_sms, int max_splits, long long ws_floats,
                    int n_counters, bool allow_cluster, int max_out, int * bn, int * splits, int * pair = nullptr);
// Workspace floats a planned launch needs (0 when it does not split K).
long long gemm_ws_floats(const GemmLaunch & L);
// After the epilogue fields of L.p are set: encode the epilogue tensor maps (TMA stores where the
// output layout allows them, plain stores otherwise). gemm_launch finalizes a copy if needed.
void gemm_finalize(GemmLaunch & L);
cudaError_t gemm_launch(const GemmLaunch & L, cudaStream_t st);

// ---------------------------------------------------------------------------------------------
// GEMV for a handful of tokens (N <= 8): y[n][m] = act(sum_k x[n][k] * W[m][k] + bias[m]),
// weights in their stored ggml type (0 f32, 30 bf16, 8 q8_0), read once from HBM.
// dual: W2 given -> y = silu(W x) * (W2 x) (SwiGLU pair, no bias).
// round_bf16: round x to bf16 first (what the reference's mul_mat does for BF16 weights).
// ---------------------------------------------------------------------------------------------
cudaError_t gemv_launch(const void * W, int wtype, const void * W2, int M, int K, const float * x,
                        long long ldx, int N, const float * bias, int act, int round_bf16,
                        void * y, int y_bf16, long long ldy, cudaStream_t st, int * err = nullptr);

// ---------------------------------------------------------------------------------------------
// Attention (tcgen05): O = softmax(Q K^T * scale) V per (batch, head); Q, K, V fp16
// [B*nh][S][64] (head-major). O written bf16 token-major: out[b][t][h*64 + d], row stride ldo.
// ---------------------------------------------------------------------------------------------
constexpr int kMaxHpRanks = 8;
struct AttnLaunch {
    CUtensorMap tmQ, tmK, tmV;
    int S, nh, B;
    long long ldo;
    void * out;
    int * err;
    float scale;
    bool out_f32 = false;   // f32 output (parity tests) instead of bf16
};
bool attn_plan(AttnLaunch & L, const void * Q, const void * K, const void * V, int B, int nh, int S,
               void * out, long long ldo, int * err, bool out_f32 = false);
cudaError_t attn_launch(const AttnLaunch & L, cudaStream_t st);

// ---------------------------------------------------------------------------------------------
// Elementwise / normalisation kernels
// ---------------------------------------------------------------------------------------------
// y = LN(x) * (1 + scale) + shift, LN eps 1e-5 without affine; x f32 [rows][H];
// shift/scale rows: row (per_token) or row / rows_per_item. y bf16 [rows][H].
cudaError_t ln_modulate(const float * x, int rows, int H, const float * shift, const float * scale,
                        long long ld_mod, int per_token, int rows_per_item, __nv_bfloat16 * y, cudaStream_t st);
// qkv f32 [B][S][3H] (Q|K|V column blocks) -> RMSNorm(q,k)*gain, RoPE (if fscale > 0), fp16
// head-major at sequence offset s_off of joint buffers [B][nh][Sj][64].
// (cos, sin) of the RoPE angles fscale * (pos * theta^(-2i/64)), pos < S, i < 32 (ggml rope NORMAL).
cudaError_t rope_table(int S, float fscale, float theta, float2 * tab, cudaStream_t st);
cudaError_t qk_norm_rope(const float * qkv, int B, int S, int H, int nh, const float * qg, const float * kg,
                         int rope, float fscale, float theta, __half * Q, __half * K, __half * V, int Sj, int s_off,
                         cudaStream_t st);
cudaError_t latent_to_tokens(const float * lat, int B, int C, int T, __nv_bfloat16 * y, cudaStream_t st);
cudaError_t sync_prep(const float * sync, int B, int S, int C, const float * pos_emb, __nv_bfloat16 * y, cudaStream_t st);
cudaError_t text_prep(const float * text, int text_S, int text_dim, const float * t5, int t5_S, int t5_dim,
                      int B, __nv_bfloat16 * y, cudaStream_t st);
cudaError_t timestep_embed(const float * t, int B, int H, float max_period, float * y, cudaStream_t st);
cudaError_t seq_mean(const float * x, int B, int S, int H, float * y, cudaStream_t st);
cudaError_t add_vec(const float * a, const float * b, int n, float * y, cudaStream_t st);
// ext[b][t] = sync[b][floor((t+0.5)*sync_S/T)] + gc[b]; sext = bf16(silu(ext)); sgc = silu(gc)
cudaError_t build_extended(const float * sync, int sync_S, const float * gc, int B, int T, int H,
                           float * ext, __nv_bfloat16 * sext, float * sgc, cudaStream_t st);
cudaError_t cast_f32_bf16(const float * x, long long n, __nv_bfloat16 * y, cudaStream_t st);
// y = bf16(silu(x)) (the adaLN GEMM operand build_extended writes; rebuilt after a teacher-forced ext)
cudaError_t silu_cast_bf16(const float * x, long long n, __nv_bfloat16 * y, cudaStream_t st);
// CFG combine + Euler update on [B2][T][L] flows: pairs (cond = item 2p, uncond = 2p+1);
// x [P][L][T] (t fastest) += dt * (u + (c - u) * cfg); optionally also store v into flow0.
cudaError_t cfg_euler(const float * flow, int P, int T, int L, float cfg, float dt, float * x, float * flow0,
                      cudaStream_t st);
// Pack x [P][L][T] into both halves of the batched latent input [2P][L][T].
cudaError_t dup_latent(const float * x, int P, int L, int T, float * lat2, cudaStream_t st);

}  // namespace tsd
