// tsd_oracle.cpp — CPU oracle for the MM-DiT hot path.
//
// TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
// leg may load this library, and only as the checker or the timed CPU reference. The product
// (thinksound.cpp_b200/) never links or calls it.
//
// What it restates: pwilkin/thinksound.cpp src/mmdit.cpp — ts_dit::forward (:119-342) and
// ts_dit::sample (:344-376) — together with the semantics of the GGML ops that file calls
// (ggml_mul_mat, ggml_im2col, ggml_norm, ggml_rms_norm, ggml_rope_ext NORMAL,
// ggml_flash_attn_ext, ggml_get_rows, ggml_pad, ggml_concat, ggml_mean, ggml_silu).
// GGML itself (ggml-org/ggml, an un-vendored git submodule; the reference's docs pin the
// llama.cpp build at commit 911b67a60) is absent, so its op semantics are restated from the
// published definitions of those ops.
//
// PARITY UNPINNED: the reference's golden GGUFs (convert/dump_dit_golden.py,
// dump_dit_debug*.py) were never committed and the reference cannot be built here (empty GGML
// submodule), so no reference output exists to pin this restatement against. It is
// cross-checked instead against an independent PyTorch restatement (tests/torch_ref.py).
//
// Two numeric modes (bit flags of `mode`):
//   TSO_EMU_ACT  — round every mul_mat activation operand to the weight's vec-dot type the way
//                  GGML's CPU backend does (BF16 weights -> BF16 activations, F16 -> F16,
//                  Q8_0 -> Q8_0 blocks of 32 with an fp16 scale). mmdit.cpp:12-25.
//   TSO_EMU_KV16 — round Q, K and V to F16 before attention (mmdit.cpp:88-90: K/V are cast to
//                  F16; GGML's flash-attn converts Q to the K type for its dot products).
// mode 0 is the exact FP32 restatement with dequantised weights.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>
#include <algorithm>
#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" {
typedef void (*tso_dbg_cb)(void * ud, const char * name, const float * data, int64_t n);
}

namespace {

enum { GT_F32 = 0, GT_F16 = 1, GT_Q8_0 = 8, GT_BF16 = 30 };
enum { TSO_EMU_ACT = 1, TSO_EMU_KV16 = 2 };

// ---- scalar conversions (IEEE round-to-nearest-even) ----
inline float bf16_round(float x) {
    uint32_t u; memcpy(&u, &x, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return x;              // NaN stays NaN
    u += 0x7fffu + ((u >> 16) & 1u);
    u &= 0xffff0000u;
    float r; memcpy(&r, &u, 4); return r;
}
inline uint16_t f32_to_f16_bits(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t exp = (int32_t)((x >> 23) & 0xff) - 127 + 15;
    uint32_t mant = x & 0x7fffffu;
    if (((x >> 23) & 0xff) == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0));
    if (exp >= 31) return (uint16_t)(sign | 0x7c00u);
    if (exp <= 0) {
        if (exp < -10) return (uint16_t) sign;
        mant |= 0x800000u;
        int shift = 14 - exp;
        uint32_t half = mant >> shift;
        uint32_t rem = mant & ((1u << shift) - 1), mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (half & 1u))) half++;
        return (uint16_t)(sign | half);
    }
    uint32_t half = sign | ((uint32_t) exp << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (half & 1u))) half++;
    return (uint16_t) half;
}
inline float f16_bits_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu, mant = h & 0x3ffu, x;
    if (exp == 0) {
        if (mant == 0) x = sign;
        else { exp = 127 - 15 + 1; while (!(mant & 0x400u)) { mant <<= 1; exp--; } mant &= 0x3ffu; x = sign | (exp << 23) | (mant << 13); }
    } else if (exp == 31) x = sign | 0x7f800000u | (mant << 13);
    else x = sign | ((exp + 127 - 15) << 23) | (mant << 13);
    float f; memcpy(&f, &x, 4); return f;
}
inline float f16_round(float x) { return f16_bits_to_f32(f32_to_f16_bits(x)); }
inline float bf16_bits_to_f32(uint16_t b) { uint32_t u = (uint32_t) b << 16; float f; memcpy(&f, &u, 4); return f; }

struct Tensor {
    int type = GT_F32;
    int64_t ne[4] = {1, 1, 1, 1};
    std::vector<float> f;        // dequantised values, ggml memory order (ne0 fastest)
    int64_t n() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
};

struct Model {
    int hidden = 1024, n_head = 16, head_dim = 64, depth = 21, fused_depth = 14, latent_dim = 64;
    float rope_theta = 10000.f, t_max_period = 1.f;
    std::unordered_map<std::string, Tensor> w;
    const Tensor & need(const std::string & n) const {
        auto it = w.find(n);
        if (it == w.end()) { fprintf(stderr, "tso: missing tensor %s\n", n.c_str()); throw 1; }
        return it->second;
    }
};

// Activation rounding applied by GGML's CPU mul_mat to src1 (the activations) when the
// weight's vec_dot_type is not F32 (ggml.c: src1 is converted with from_float of vec_dot_type).
void round_activations(std::vector<float> & x, int64_t rows, int64_t K, int wtype) {
    if (wtype == GT_BF16) { for (auto & v : x) v = bf16_round(v); return; }
    if (wtype == GT_F16)  { for (auto & v : x) v = f16_round(v); return; }
    if (wtype == GT_Q8_0) {
        // quantize_row_q8_0: per 32-block, d = amax/127, q = round(x/d), d stored as fp16.
        for (int64_t r = 0; r < rows; ++r)
            for (int64_t b0 = 0; b0 < K; b0 += 32) {
                float * p = &x[r * K + b0];
                int64_t nb = std::min<int64_t>(32, K - b0);
                float amax = 0.f;
                for (int64_t i = 0; i < nb; ++i) amax = std::max(amax, std::fabs(p[i]));
                const float d = amax / 127.f, id = d ? 1.f / d : 0.f;
                const float dq = f16_round(d);
                for (int64_t i = 0; i < nb; ++i) p[i] = roundf(p[i] * id) * dq;
            }
    }
}

// Y[n][m] = sum_k X[n][k] * W[m][k] (+ bias[m]). X [N][K], W [M][K] (ggml ne = [K, M]).
void gemm_nt(const float * X, int64_t N, const float * W, int64_t M, int64_t K,
             const float * bias, float * Y) {
    const int64_t MB = 8, NB = 4;
    const int64_t nmb = (M + MB - 1) / MB, nnb = (N + NB - 1) / NB;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t job = 0; job < nmb * nnb; ++job) {
        const int64_t m0 = (job % nmb) * MB, n0 = (job / nmb) * NB;
        const int64_t m1 = std::min(M, m0 + MB), n1 = std::min(N, n0 + NB);
        for (int64_t m = m0; m < m1; ++m) {
            const float * w = W + m * K;
            for (int64_t n = n0; n < n1; ++n) {
                const float * x = X + n * K;
                float acc = 0.f;
#pragma omp simd reduction(+:acc)
                for (int64_t k = 0; k < K; ++k) acc += x[k] * w[k];
                Y[n * M + m] = acc + (bias ? bias[m] : 0.f);
            }
        }
    }
}

struct Ctx {
    const Model & M;
    int mode;
    tso_dbg_cb cb; void * ud;
    void dbg(const char * name, const std::vector<float> & v) const { if (cb) cb(ud, name, v.data(), (int64_t) v.size()); }

    // lin (mmdit.cpp:12-16): y = mul_mat(w, x) + b. x [N][K] token-major -> [N][M].
    std::vector<float> lin(const std::string & wn, const std::string & bn, const std::vector<float> & x, int64_t N) const {
        const Tensor & W = M.need(wn);
        const int64_t K = W.ne[0], Mo = W.ne[1];
        const float * b = bn.empty() ? nullptr : M.need(bn).f.data();
        std::vector<float> xr(x.begin(), x.begin() + N * K);
        if (mode & TSO_EMU_ACT) round_activations(xr, N, K, W.type);
        std::vector<float> y((size_t)(N * Mo));
        gemm_nt(xr.data(), N, W.f.data(), Mo, K, b, y.data());
        return y;
    }
    // conv1d_f32 + conv_cl (mmdit.cpp:20-34): stride 1, padding p, dilation 1.
    // im2col column index ic*K + k holds x[t + k - p][ic] (zero outside [0, N)).
    std::vector<float> conv(const std::string & wn, const std::string & bn, const std::vector<float> & x, int64_t N, int p) const {
        const Tensor & W = M.need(wn);
        const int64_t KK = W.ne[0], IC = W.ne[1], OC = W.ne[2];
        std::vector<float> cols((size_t)(N * IC * KK), 0.f);
        for (int64_t t = 0; t < N; ++t)
            for (int64_t ic = 0; ic < IC; ++ic)
                for (int64_t k = 0; k < KK; ++k) {
                    int64_t s = t + k - p;
                    cols[(size_t)(t * IC * KK + ic * KK + k)] = (s >= 0 && s < N) ? x[(size_t)(s * IC + ic)] : 0.f;
                }
        if (mode & TSO_EMU_ACT) round_activations(cols, N, IC * KK, W.type);
        const float * b = bn.empty() ? nullptr : M.need(bn).f.data();
        std::vector<float> y((size_t)(N * OC));
        gemm_nt(cols.data(), N, W.f.data(), OC, IC * KK, b, y.data());
        return y;
    }
    static void silu_(std::vector<float> & v) { for (auto & x : v) x = x / (1.0f + expf(-x)); }
    // convmlp (mmdit.cpp:39-44) and mlp (:47-52): w2(silu(w1 x) * w3 x)
    std::vector<float> convmlp(const std::string & p, const std::vector<float> & x, int64_t N) const {
        auto h1 = conv(p + ".w1.weight", "", x, N, 1);
        auto h3 = conv(p + ".w3.weight", "", x, N, 1);
        silu_(h1); for (size_t i = 0; i < h1.size(); ++i) h1[i] *= h3[i];
        return conv(p + ".w2.weight", "", h1, N, 1);
    }
    std::vector<float> mlp(const std::string & p, const std::vector<float> & x, int64_t N) const {
        auto h1 = lin(p + ".w1.weight", "", x, N);
        auto h3 = lin(p + ".w3.weight", "", x, N);
        silu_(h1); for (size_t i = 0; i < h1.size(); ++i) h1[i] *= h3[i];
        return lin(p + ".w2.weight", "", h1, N);
    }
    // layernorm (mmdit.cpp:59, ggml_norm eps 1e-5, no affine) then modulate (:55-57)
    // x*(scale+1)+shift; shift/scale rows indexed per token (per_token) or broadcast.
    std::vector<float> ln_modulate(const std::vector<float> & x, int64_t N, int64_t H,
                                   const float * shift, const float * scale, int64_t mod_stride) const {
        std::vector<float> y((size_t)(N * H));
        for (int64_t n = 0; n < N; ++n) {
            const float * r = &x[(size_t)(n * H)];
            double s = 0; for (int64_t i = 0; i < H; ++i) s += r[i];
            const float mean = (float)(s / H);
            double v = 0; for (int64_t i = 0; i < H; ++i) { float d = r[i] - mean; v += (double) d * d; }
            const float rstd = 1.0f / sqrtf((float)(v / H) + 1e-5f);
            const float * sh = shift + n * mod_stride; const float * sc = scale + n * mod_stride;
            for (int64_t i = 0; i < H; ++i) y[(size_t)(n * H + i)] = ((r[i] - mean) * rstd) * (sc[i] + 1.0f) + sh[i];
        }
        return y;
    }
    // rmsnorm_w (mmdit.cpp:78-80) per head over head_dim, eps 1e-6, times gain g[hd]
    void rmsnorm_heads(std::vector<float> & q, int64_t N, int nh, int hd, const float * g) const {
        for (int64_t n = 0; n < N; ++n)
            for (int h = 0; h < nh; ++h) {
                float * r = &q[(size_t)(n * nh * hd + h * hd)];
                double s = 0; for (int d = 0; d < hd; ++d) s += (double) r[d] * r[d];
                const float sc = 1.0f / sqrtf((float)(s / hd) + 1e-6f);
                for (int d = 0; d < hd; ++d) r[d] = (r[d] * sc) * g[d];
            }
    }
    // rope (mmdit.cpp:96-100): GGML_ROPE_TYPE_NORMAL — adjacent pairs (2i, 2i+1),
    // theta = pos * freq_scale * base^(-2i/hd), ext_factor 0, attn_factor 1.
    void rope(std::vector<float> & q, int64_t N, int nh, int hd, float fscale) const {
        for (int64_t n = 0; n < N; ++n)
            for (int i = 0; i < hd / 2; ++i) {
                const float theta = fscale * ((float) n * powf(M.rope_theta, -2.0f * i / (float) hd));
                const float c = cosf(theta), s = sinf(theta);
                for (int h = 0; h < nh; ++h) {
                    float * r = &q[(size_t)(n * nh * hd + h * hd + 2 * i)];
                    const float x0 = r[0], x1 = r[1];
                    r[0] = x0 * c - x1 * s;
                    r[1] = x0 * s + x1 * c;
                }
            }
    }
    // attention (mmdit.cpp:85-94): softmax(Q K^T / sqrt(hd)) V per head, no mask.
    // q,k,v,out token-major [S][H], column index d + hd*h.
    std::vector<float> attention(std::vector<float> q, std::vector<float> k, std::vector<float> v, int64_t S, int nh, int hd) const {
        if (mode & TSO_EMU_KV16) { for (auto & x : q) x = f16_round(x); for (auto & x : k) x = f16_round(x); for (auto & x : v) x = f16_round(x); }
        const int64_t H = (int64_t) nh * hd;
        const float scale = 1.0f / sqrtf((float) hd);
        std::vector<float> o((size_t)(S * H));
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
        for (int h = 0; h < nh; ++h)
            for (int64_t i = 0; i < S; ++i) {
                std::vector<float> s((size_t) S);
                const float * qi = &q[(size_t)(i * H + h * hd)];
                float mx = -INFINITY;
                for (int64_t j = 0; j < S; ++j) {
                    const float * kj = &k[(size_t)(j * H + h * hd)];
                    float acc = 0.f;
                    for (int d = 0; d < hd; ++d) acc += qi[d] * kj[d];
                    s[j] = acc * scale; mx = std::max(mx, s[j]);
                }
                double sum = 0;
                for (int64_t j = 0; j < S; ++j) { s[j] = expf(s[j] - mx); sum += s[j]; }
                float * oi = &o[(size_t)(i * H + h * hd)];
                for (int d = 0; d < hd; ++d) oi[d] = 0.f;
                for (int64_t j = 0; j < S; ++j) {
                    const float * vj = &v[(size_t)(j * H + h * hd)];
                    for (int d = 0; d < hd; ++d) oi[d] += s[j] * vj[d];
                }
                const float inv = (float)(1.0 / sum);
                for (int d = 0; d < hd; ++d) oi[d] *= inv;
            }
        return o;
    }

    struct Pre {   // pre_attn outputs (mmdit.cpp:203-225)
        std::vector<float> mod, q, k, v, xn;   // mod [Nmod][n*H]
        int64_t mod_stride = 0;                 // 0: broadcast one row; else n*H per token
        int nchunk = 6;
    };
    // cond [Nc][H] with Nc == N (per-token, latent) or 1 (global_c).
    Pre pre_attn(const std::string & bp, const std::vector<float> & x, int64_t N,
                 const std::vector<float> & cond, int64_t Nc, bool rope_on, float fscale, bool pre_only) const {
        const int64_t H = M.hidden; const int nh = M.n_head, hd = M.head_dim;
        Pre P;
        std::vector<float> sc = cond; silu_(sc);
        P.mod = lin(bp + ".adaLN_modulation.1.weight", bp + ".adaLN_modulation.1.bias", sc, Nc);
        P.nchunk = pre_only ? 2 : 6;
        const int64_t row = (int64_t) P.nchunk * H;
        P.mod_stride = (Nc == 1) ? 0 : row;
        P.xn = ln_modulate(x, N, H, P.mod.data() + 0 * H, P.mod.data() + 1 * H, P.mod_stride);
        auto qkv = lin(bp + ".attn.qkv.weight", bp + ".attn.qkv.bias", P.xn, N);
        // split_qkv (mmdit.cpp:67-76): feature f = 3*c + j, j = 0 (q), 1 (k), 2 (v)
        P.q.resize((size_t)(N * H)); P.k.resize((size_t)(N * H)); P.v.resize((size_t)(N * H));
        for (int64_t n = 0; n < N; ++n)
            for (int64_t c = 0; c < H; ++c) {
                P.q[(size_t)(n * H + c)] = qkv[(size_t)(n * 3 * H + 3 * c + 0)];
                P.k[(size_t)(n * H + c)] = qkv[(size_t)(n * 3 * H + 3 * c + 1)];
                P.v[(size_t)(n * H + c)] = qkv[(size_t)(n * 3 * H + 3 * c + 2)];
            }
        rmsnorm_heads(P.q, N, nh, hd, M.need(bp + ".attn.q_norm.weight").f.data());
        rmsnorm_heads(P.k, N, nh, hd, M.need(bp + ".attn.k_norm.weight").f.data());
        if (rope_on) { rope(P.q, N, nh, hd, fscale); rope(P.k, N, nh, hd, fscale); }
        return P;
    }
    // post_attn (mmdit.cpp:226-235)
    // `attn_name`: stage name of the residual stream after the attention half (gate_msa * out-proj
    // added, :231), before the FFN half.
    void post_attn(const std::string & bp, std::vector<float> & x, int64_t N, const std::vector<float> & ao,
                   const Pre & P, bool is_text, const std::string & attn_name) const {
        const int64_t H = M.hidden;
        auto l1 = is_text ? lin(bp + ".linear1.weight", bp + ".linear1.bias", ao, N)
                          : conv(bp + ".linear1.weight", bp + ".linear1.bias", ao, N, 1);
        const float * gate_msa = P.mod.data() + 2 * H;
        for (int64_t n = 0; n < N; ++n)
            for (int64_t i = 0; i < H; ++i) x[(size_t)(n * H + i)] += l1[(size_t)(n * H + i)] * gate_msa[n * P.mod_stride + i];
        dbg(attn_name.c_str(), x);
        auto r = ln_modulate(x, N, H, P.mod.data() + 3 * H, P.mod.data() + 4 * H, P.mod_stride);
        auto f = is_text ? mlp(bp + ".ffn", r, N) : convmlp(bp + ".ffn", r, N);
        const float * gate_mlp = P.mod.data() + 5 * H;
        for (int64_t n = 0; n < N; ++n)
            for (int64_t i = 0; i < H; ++i) x[(size_t)(n * H + i)] += f[(size_t)(n * H + i)] * gate_mlp[n * P.mod_stride + i];
    }

    // ts_dit::forward (mmdit.cpp:119-342) for one batch item.
    // latent [latent_dim][T] (t fastest); clip_f [clip_S][1024]; sync_f [sync_S][768];
    // text_f [text_S][1024]; t5 [t5_S][t5_dim]; global_text [1024]. flow out [T][latent_dim].
    void forward(const float * latent, int64_t T, float t, const float * clip_f, int64_t clip_S,
                 const float * sync_f, int64_t sync_S, const float * text_f, int64_t text_S,
                 const float * t5, int64_t t5_S, const float * gtext, float * flow_out) const {
        const int64_t H = M.hidden; const int nh = M.n_head, hd = M.head_dim, L = M.latent_dim;
        const int n_joint = M.depth - M.fused_depth;
        // audio_input_proj (:150-155)
        std::vector<float> lat0((size_t)(T * L));
        for (int64_t c = 0; c < L; ++c) for (int64_t tt = 0; tt < T; ++tt) lat0[(size_t)(tt * L + c)] = latent[c * T + tt];
        auto lat = conv("audio_input_proj.0.weight", "audio_input_proj.0.bias", lat0, T, 1);
        silu_(lat);
        lat = convmlp("audio_input_proj.2", lat, T);
        dbg("x_in", lat);
        // timestep embedding (:305-313) and t_embed mlp (:158-161)
        std::vector<float> temb((size_t) H);
        {
            const int half = (int)(H / 2);
            const float fscale_t = 10000.0f / M.t_max_period;
            for (int kk = 0; kk < half; ++kk) {
                const float fr = fscale_t * powf(10000.0f, -2.0f * kk / (float) H);
                temb[kk] = cosf(t * fr); temb[half + kk] = sinf(t * fr);
            }
        }
        auto te = lin("t_embed.mlp.0.weight", "t_embed.mlp.0.bias", temb, 1);
        silu_(te);
        te = lin("t_embed.mlp.2.weight", "t_embed.mlp.2.bias", te, 1);
        dbg("t_emb", te);
        // clip (:165-167)
        const int64_t CD = M.need("clip_input_proj.0.weight").ne[0];
        std::vector<float> cin(clip_f, clip_f + clip_S * CD);
        auto clip = lin("clip_input_proj.0.weight", "clip_input_proj.0.bias", cin, clip_S);
        silu_(clip);
        clip = convmlp("clip_input_proj.2", clip, clip_S);
        // sync (:168-177): + sync_pos_emb per 8-frame segment, conv k7 p3, silu, convmlp, get_rows
        const Tensor & spe = M.need("sync_pos_emb");
        const int64_t SD = spe.ne[0];
        std::vector<float> sy(sync_f, sync_f + sync_S * SD);
        for (int64_t s = 0; s < sync_S; ++s) for (int64_t c = 0; c < SD; ++c) sy[(size_t)(s * SD + c)] += spe.f[(size_t)((s % 8) * SD + c)];
        auto sync = conv("sync_input_proj.0.weight", "sync_input_proj.0.bias", sy, sync_S, 3);
        silu_(sync);
        sync = convmlp("sync_input_proj.2", sync, sync_S);
        std::vector<float> sync_t((size_t)(T * H));
        for (int64_t i = 0; i < T; ++i) {
            int64_t si = (int64_t) floorf(((float) i + 0.5f) * (float) sync_S / (float) T);   // :319
            memcpy(&sync_t[(size_t)(i * H)], &sync[(size_t)(si * H)], sizeof(float) * H);
        }
        // text (:178-183): pad text_f [text_S][1024] to t5 width, concat t5 along the sequence
        const int64_t TD = M.need("text_input_proj.0.weight").ne[0];    // 2048
        const int64_t St = text_S + t5_S;
        const int64_t XD = 1024;
        std::vector<float> tcat((size_t)(St * TD), 0.f);
        for (int64_t s = 0; s < text_S; ++s) memcpy(&tcat[(size_t)(s * TD)], text_f + s * XD, sizeof(float) * XD);
        memcpy(&tcat[(size_t)(text_S * TD)], t5, sizeof(float) * t5_S * TD);
        auto text = lin("text_input_proj.0.weight", "text_input_proj.0.bias", tcat, St);
        silu_(text);
        text = mlp("text_input_proj.2", text, St);
        // conditioning vectors (:185-200)
        std::vector<float> gt(gtext, gtext + XD);
        auto text_fc = lin("text_cond_proj.weight", "text_cond_proj.bias", gt, 1);
        std::vector<float> cmean((size_t) H, 0.f);
        for (int64_t i = 0; i < H; ++i) { double s = 0; for (int64_t n = 0; n < clip_S; ++n) s += clip[(size_t)(n * H + i)]; cmean[i] = (float)(s / clip_S); }
        auto clip_fc = lin("clip_cond_proj.weight", "clip_cond_proj.bias", cmean, 1);
        dbg("clip_fc", clip_fc); dbg("text_fc", text_fc);
        std::vector<float> gsum((size_t) H);
        for (int64_t i = 0; i < H; ++i) gsum[i] = clip_fc[i] + text_fc[i];
        auto gc = mlp("global_cond_mlp", gsum, 1);
        dbg("gcmlp", gc);
        for (int64_t i = 0; i < H; ++i) gc[i] += te[i];
        std::vector<float> ext((size_t)(T * H));
        for (int64_t n = 0; n < T; ++n) for (int64_t i = 0; i < H; ++i) ext[(size_t)(n * H + i)] = sync_t[(size_t)(n * H + i)] + gc[i];
        dbg("clip_pp", clip); dbg("text_pp", text); dbg("global_c", gc); dbg("extended_c", ext);

        // joint blocks (:237-272)
        const float clip_fscale = (float) T / (float) clip_S;
        for (int i = 0; i < n_joint; ++i) {
            const std::string jb = "joint_blocks." + std::to_string(i);
            const bool pre_only = (i == n_joint - 1);
            Pre pl = pre_attn(jb + ".latent_block", lat, T, ext, T, true, 1.0f, false);
            Pre pc = pre_attn(jb + ".clip_block", clip, clip_S, gc, 1, true, clip_fscale, pre_only);
            Pre pt = pre_attn(jb + ".text_block", text, St, gc, 1, false, 1.0f, pre_only);
            if (i == 0) dbg("text_xn", pt.xn);
            const int64_t S = T + clip_S + St;
            std::vector<float> Q, K, V;
            for (const Pre * p : {&pl, &pc, &pt}) { Q.insert(Q.end(), p->q.begin(), p->q.end()); K.insert(K.end(), p->k.begin(), p->k.end()); V.insert(V.end(), p->v.begin(), p->v.end()); }
            if (i == 0) { dbg("a0_q", Q); dbg("a0_k", K); dbg("a0_v", V); }
            auto ao = attention(Q, K, V, S, nh, hd);
            if (i == 0) dbg("a0_out", ao);
            std::vector<float> ao_l(ao.begin(), ao.begin() + T * H);
            std::vector<float> ao_c(ao.begin() + T * H, ao.begin() + (T + clip_S) * H);
            std::vector<float> ao_t(ao.begin() + (T + clip_S) * H, ao.end());
            // per-block stage names (the GPU library reports the same ones)
            const std::string bi = "blk" + std::to_string(i);
            post_attn(jb + ".latent_block", lat, T, ao_l, pl, false, bi + "_attn_lat");
            if (!pre_only) {
                post_attn(jb + ".clip_block", clip, clip_S, ao_c, pc, false, bi + "_attn_clip");
                post_attn(jb + ".text_block", text, St, ao_t, pt, true, bi + "_attn_text");
            }
            dbg((bi + "_lat").c_str(), lat); dbg((bi + "_clip").c_str(), clip); dbg((bi + "_text").c_str(), text);
            if (i == 0) { dbg("jb0_lat", lat); dbg("jb0_clip", clip); dbg("jb0_text", text); }
        }
        dbg("after_joint", lat);
        // fused blocks (:274-282)
        for (int i = 0; i < M.fused_depth; ++i) {
            const std::string fb = "fused_blocks." + std::to_string(i);
            Pre p = pre_attn(fb, lat, T, ext, T, true, 1.0f, false);
            auto ao = attention(p.q, p.k, p.v, T, nh, hd);
            const std::string bi = "blk" + std::to_string(n_joint + i);
            post_attn(fb, lat, T, ao, p, false, bi + "_attn_lat");
            dbg((bi + "_lat").c_str(), lat);
        }
        dbg("after_fused", lat);
        // final layer (:284-290)
        std::vector<float> sext = ext; silu_(sext);
        auto fmod = lin("final_layer.adaLN_modulation.1.weight", "final_layer.adaLN_modulation.1.bias", sext, T);
        auto fx = ln_modulate(lat, T, H, fmod.data(), fmod.data() + H, 2 * H);
        auto flow = conv("final_layer.conv.weight", "final_layer.conv.bias", fx, T, 3);
        dbg("flow_cl", flow);
        memcpy(flow_out, flow.data(), sizeof(float) * T * L);
    }
};

} // namespace

struct tso_model { Model m; };

extern "C" {

tso_model * tso_model_new(int hidden, int n_head, int depth, int fused_depth, int latent_dim,
                          float rope_theta, float t_max_period) {
    tso_model * p = new tso_model();
    p->m.hidden = hidden; p->m.n_head = n_head; p->m.head_dim = hidden / n_head;
    p->m.depth = depth; p->m.fused_depth = fused_depth; p->m.latent_dim = latent_dim;
    p->m.rope_theta = rope_theta; p->m.t_max_period = t_max_period;
    return p;
}

void tso_model_free(tso_model * p) { delete p; }

// Register one tensor (ggml type id, ggml ne order, raw ggml bytes). Returns 0 on success.
int tso_model_set(tso_model * p, const char * name, int type, const int64_t * ne, const void * data) {
    Tensor t; t.type = type;
    for (int i = 0; i < 4; ++i) t.ne[i] = ne[i] > 0 ? ne[i] : 1;
    const int64_t n = t.n();
    t.f.resize((size_t) n);
    if (type == GT_F32) memcpy(t.f.data(), data, sizeof(float) * n);
    else if (type == GT_F16) { auto s = (const uint16_t *) data; for (int64_t i = 0; i < n; ++i) t.f[i] = f16_bits_to_f32(s[i]); }
    else if (type == GT_BF16) { auto s = (const uint16_t *) data; for (int64_t i = 0; i < n; ++i) t.f[i] = bf16_bits_to_f32(s[i]); }
    else if (type == GT_Q8_0) {
        if (t.ne[0] % 32) return -2;
        auto s = (const uint8_t *) data;
        for (int64_t b = 0; b < n / 32; ++b) {
            const uint8_t * blk = s + b * 34;
            uint16_t dh; memcpy(&dh, blk, 2);
            const float d = f16_bits_to_f32(dh);
            for (int i = 0; i < 32; ++i) t.f[(size_t)(b * 32 + i)] = (float)(int8_t) blk[2 + i] * d;
        }
    } else return -1;
    p->m.w[name] = std::move(t);
    return 0;
}

int tso_forward(const tso_model * p, int mode, const float * latent, int64_t T, float t,
                const float * clip_f, int64_t clip_S, const float * sync_f, int64_t sync_S,
                const float * text_f, int64_t text_S, const float * t5, int64_t t5_S,
                const float * gtext, float * flow_out, tso_dbg_cb cb, void * ud) {
    if (!p || T <= 0 || clip_S <= 0 || sync_S <= 0 || sync_S % 8 || text_S < 0 || t5_S < 0) return -1;
    try {
        Ctx c{p->m, mode, cb, ud};
        c.forward(latent, T, t, clip_f, clip_S, sync_f, sync_S, text_f, text_S, t5, t5_S, gtext, flow_out);
    } catch (...) { return -2; }
    return 0;
}

// ts_dit::sample (mmdit.cpp:344-376): Euler over t = 1 - s/steps with CFG
// v = u + (c - u) * cfg. Uncond uses empty_string_feat / empty_t5_feat and a zero global
// vector. noise/out [latent_dim][T] (t fastest); flow0 [latent_dim][T] or null.
int tso_sample(const tso_model * p, int mode, const float * noise, int64_t T,
               const float * clip_f, int64_t clip_S, const float * sync_f, int64_t sync_S,
               const float * text_f, int64_t text_S, const float * t5, int64_t t5_S,
               const float * gtext, int steps, float cfg, float * out, float * flow0) {
    if (!p || steps <= 0) return -1;
    try {
        const Model & M = p->m;
        const int L = M.latent_dim;
        const Tensor & es = M.need("empty_string_feat");
        const Tensor & et = M.need("empty_t5_feat");
        if (es.n() < text_S * 1024 || et.n() < t5_S * M.need("text_input_proj.0.weight").ne[0]) return -3;
        std::vector<float> zeros(1024, 0.f);
        std::vector<float> x(noise, noise + T * L), fc((size_t)(T * L)), fu((size_t)(T * L));
        Ctx c{M, mode, nullptr, nullptr};
        for (int s = 0; s < steps; ++s) {
            const float t_curr = 1.0f - (float) s / steps, t_prev = 1.0f - (float)(s + 1) / steps;
            const float dt = t_prev - t_curr;
            c.forward(x.data(), T, t_curr, clip_f, clip_S, sync_f, sync_S, text_f, text_S, t5, t5_S, gtext, fc.data());
            c.forward(x.data(), T, t_curr, clip_f, clip_S, sync_f, sync_S, es.f.data(), text_S, et.f.data(), t5_S, zeros.data(), fu.data());
            for (int64_t cc = 0; cc < L; ++cc)
                for (int64_t tt = 0; tt < T; ++tt) {
                    const float fcv = fc[(size_t)(cc + L * tt)], fuv = fu[(size_t)(cc + L * tt)];
                    const float v = fuv + (fcv - fuv) * cfg;
                    if (s == 0 && flow0) flow0[tt + T * cc] = v;
                    x[(size_t)(tt + T * cc)] += dt * v;
                }
        }
        memcpy(out, x.data(), sizeof(float) * T * L);
    } catch (...) { return -2; }
    return 0;
}

int tso_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

} // extern "C"
