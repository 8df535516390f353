// model.cu — DiT weight store: GGUF reader, device upload, one-time repack for the kernels.
//
// Mirrors the reference's loading path (src/common/ts_model.cpp:13-41: metadata, device
// allocation, per-tensor read + upload; ts_dit::load mmdit.cpp:105-117: hparams from dit.*
// keys) without GGML. Tensor names, ggml types (F32, F16, BF16, Q8_0) and shapes are those of
// convert/convert_thinksound.py and convert/quantize_gguf.py. After upload the projection
// weights are repacked once into the layouts the kernels read:
//   * conv weights ggml [K, IC, OC] -> bf16 [OC][K*IC] (tap-major, one K-block per tap);
//   * qkv rows f = 3c + j (split_qkv, mmdit.cpp:67-76) -> [Q rows | K rows | V rows];
//   * SwiGLU w1 / w3 -> one matrix whose rows alternate (w1 row f, w3 row f, w1 row f + 1, ...);
//   * every per-token adaLN weight (joint latent blocks, fused blocks, final layer) stacked
//     into one matrix, so all of them run as one GEMM per forward;
//   * F32 / F16 / Q8_0 projection weights are converted to bf16 for the tensor cores.
// Few-token weights (t_embed, cond projections, global_cond_mlp, clip/text adaLN) stay in
// their stored type for the weight-streaming GEMV.
#include "runtime.h"

#include <initializer_list>

#include <cstring>
#include <fstream>

namespace tsd {

size_t ggml_nbytes(int type, int64_t n) {
    switch (type) {
        case GT_F32: return (size_t)n * 4;
        case GT_F16:
        case GT_BF16: return (size_t)n * 2;
        case GT_Q8_0: return (size_t)(n / 32) * 34;
        default: return 0;
    }
}

namespace {

__device__ __forceinline__ float load_elem(const void * src, int type, long long e) {
    switch (type) {
        case GT_F32: return reinterpret_cast<const float *>(src)[e];
        case GT_F16: return __half2float(reinterpret_cast<const __half *>(src)[e]);
        case GT_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(src)[e]);
        default: {
            const uint8_t * blk = reinterpret_cast<const uint8_t *>(src) + (e / 32) * 34;
            const __half d = *reinterpret_cast<const __half *>(blk);
            return (float)(int8_t)blk[2 + (e & 31)] * __half2float(d);
        }
    }
}

// dst[r][tap*K_in + ic] = src(row rowmap[r], ic, tap); rowmap -1 -> zero row, -2 -> untouched.
__global__ void repack_kernel(__nv_bfloat16 * dst, long long dst_ld, const int * rowmap, int rows, const void * src,
                              int src_type, int K_in, int taps) {
    const long long kt = (long long)K_in * taps;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * kt) return;
    const int r = (int)(i / kt);
    const long long kk = i % kt;
    const int tap = (int)(kk / K_in), ic = (int)(kk % K_in);
    const int sr = rowmap ? rowmap[r] : r;
    if (sr == -2) return;
    float v = 0.f;
    if (sr >= 0) v = load_elem(src, src_type, (long long)sr * kt + (long long)ic * taps + tap);
    dst[(long long)r * dst_ld + kk] = __float2bfloat16_rn(v);
}

// Q8_0 rows -> the GEMM's planar form: q[r][k] = quant of source row rowmap[r], qs[k/32][r] = its
// block scale (rowmap -1: zero row, -2: untouched). One thread per (row, 32-block).
__global__ void repack_q8_kernel(int8_t * q, __half * qs, long long qs_ld, const int * rowmap, int rows,
                                 const uint8_t * src, int K) {
    const int nb = K / 32;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)rows * nb) return;
    const int r = (int)(i / nb), b = (int)(i - (long long)r * nb);
    const int sr = rowmap ? rowmap[r] : r;
    if (sr == -2) return;
    int8_t * dq = q + (long long)r * K + b * 32;
    if (sr < 0) {
        for (int e = 0; e < 32; ++e) dq[e] = 0;
        qs[(long long)b * qs_ld + r] = __float2half(0.f);
        return;
    }
    const uint8_t * blk = src + ((long long)sr * nb + b) * 34;
    for (int e = 0; e < 32; ++e) dq[e] = (int8_t)blk[2 + e];
    qs[(long long)b * qs_ld + r] = *reinterpret_cast<const __half *>(blk);
}

__global__ void to_f32_kernel(const void * src, int type, long long n, float * dst) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = load_elem(src, type, i);
}

}  // namespace

Model::~Model() {
    plan.reset();
    if (device >= 0) cudaSetDevice(device);
    hp_release(*this);
    for (auto & kv : raw)
        if (kv.second.d) cudaFree(kv.second.d);
    for (void * p : allocs) cudaFree(p);
    if (h_err) cudaFreeHost(h_err);
}

void * Model::dalloc(size_t bytes) {
    void * p = nullptr;
    if (cudaMalloc(&p, bytes < 256 ? 256 : bytes) != cudaSuccess) return nullptr;
    allocs.push_back(p);
    return p;
}

int model_set_tensor(Model & m, const char * name, int type, const int64_t ne[4], const void * data, size_t nbytes) {
    if (!name || !data || m.finalized) return m.finalized ? TSD_ERR_STATE : TSD_ERR_ARG;
    RawTensor t;
    t.type = type;
    for (int i = 0; i < 4; ++i) t.ne[i] = ne[i] > 0 ? ne[i] : 1;
    t.nbytes = ggml_nbytes(type, t.n());
    if (!t.nbytes) return TSD_ERR_UNSUPPORTED;
    if (type == GT_Q8_0 && t.ne[0] % 32) return TSD_ERR_UNSUPPORTED;
    if (nbytes != t.nbytes) {
        fprintf(stderr, "tsd: tensor '%s': %zu bytes given, %zu expected\n", name, nbytes, t.nbytes);
        return TSD_ERR_ARG;
    }
    TSD_CUDA_TRY(cudaSetDevice(m.device));
    auto old = m.raw.find(name);
    if (old != m.raw.end()) {
        cudaFree(old->second.d);
        m.raw.erase(old);
    }
    TSD_CUDA_TRY(cudaMalloc(&t.d, t.nbytes));
    TSD_CUDA_TRY(cudaMemcpy(t.d, data, t.nbytes, cudaMemcpyDefault));
    if (t.n() <= (1 << 20)) {
        t.host.resize(t.nbytes);
        TSD_CUDA_TRY(cudaMemcpy(t.host.data(), t.d, t.nbytes, cudaMemcpyDeviceToHost));
    }
    m.raw[name] = std::move(t);
    return TSD_OK;
}

namespace {

struct Finalizer {
    Model & m;
    std::vector<std::string> consumed;   // raw tensors fully repacked (freed at the end)
    int rc = TSD_OK;

    const RawTensor * need(const std::string & n) {
        const RawTensor * t = m.get(n);
        if (!t && rc == TSD_OK) {
            fprintf(stderr, "tsd: required tensor missing: '%s'\n", n.c_str());
            rc = TSD_ERR_MISSING;
        }
        return t;
    }
    float * bias_f32(const std::string & n, const std::vector<int> * perm = nullptr, int pad_to = 0) {
        const RawTensor * t = need(n);
        if (!t) return nullptr;
        if (t->type != GT_F32 || t->host.empty()) { rc = TSD_ERR_UNSUPPORTED; return nullptr; }
        const float * src = reinterpret_cast<const float *>(t->host.data());
        const int n_out = std::max<int>((int)t->n(), pad_to);
        std::vector<float> h((size_t)n_out, 0.f);
        for (int i = 0; i < (int)t->n(); ++i) h[i] = src[perm ? (*perm)[i] : i];
        float * d = reinterpret_cast<float *>(m.dalloc(h.size() * 4));
        if (!d || cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) { rc = TSD_ERR_CUDA; return nullptr; }
        return d;
    }
    // Planar Q8_0 for the GEMM (TSD_Q8_IN_KERNEL=1) when every source is Q8_0 with one tap (the
    // reference quantises only 2-D weights; convolution weights stay F32): the weights stay resident
    // at 34 bytes per 32 and the GEMM's converter warps dequantise each tile in shared memory.
    // Default: widen to bf16 at load. The in-kernel path keeps 47% less weight memory resident and
    // gives identical results, but its conversion (two warps per stage, six in a CTA with a single
    // tile) still costs ~1.3x the widened step at config 4.
    bool q8_gemm(std::initializer_list<const RawTensor *> ts, int taps, int K_in) {
        const char * e = getenv("TSD_Q8_IN_KERNEL");
        if (!(e && *e == '1') || taps != 1 || K_in % 64) return false;
        for (const RawTensor * t : ts)
            if (!t || t->type != GT_Q8_0) return false;
        return true;
    }
    bool alloc_q8(GW & g, long long rows, int K) {
        g.q = reinterpret_cast<int8_t *>(m.dalloc((size_t)rows * K));
        g.qs = reinterpret_cast<__half *>(m.dalloc((size_t)rows * (K / 32) * 2));
        if (!g.q || !g.qs) { rc = TSD_ERR_CUDA; return false; }
        return true;
    }
    bool repack_q8(int8_t * q, __half * qs, long long qs_ld, const std::vector<int> & rowmap, const RawTensor * t, int K) {
        int * dmap = nullptr;
        if (cudaMalloc(&dmap, rowmap.size() * 4) != cudaSuccess) { rc = TSD_ERR_CUDA; return false; }
        cudaMemcpy(dmap, rowmap.data(), rowmap.size() * 4, cudaMemcpyHostToDevice);
        const long long n = (long long)rowmap.size() * (K / 32);
        repack_q8_kernel<<<(unsigned)((n + 255) / 256), 256>>>(q, qs, qs_ld, dmap, (int)rowmap.size(),
                                                               reinterpret_cast<const uint8_t *>(t->d), K);
        cudaError_t e = cudaDeviceSynchronize();
        cudaFree(dmap);
        if (e != cudaSuccess) { rc = TSD_ERR_CUDA; return false; }
        return true;
    }
    bool repack(__nv_bfloat16 * dst, long long dst_ld, const std::vector<int> & rowmap, const RawTensor * t, int K_in,
                int taps) {
        int * dmap = nullptr;
        if (cudaMalloc(&dmap, rowmap.size() * 4) != cudaSuccess) { rc = TSD_ERR_CUDA; return false; }
        cudaMemcpy(dmap, rowmap.data(), rowmap.size() * 4, cudaMemcpyHostToDevice);
        const long long n = (long long)rowmap.size() * K_in * taps;
        repack_kernel<<<(unsigned)((n + 255) / 256), 256>>>(dst, dst_ld, dmap, (int)rowmap.size(), t->d, t->type, K_in, taps);
        cudaError_t e = cudaDeviceSynchronize();
        cudaFree(dmap);
        if (e != cudaSuccess) { rc = TSD_ERR_CUDA; return false; }
        return true;
    }
    // Plain projection: 2-D [K_in, M] (taps = 1) or conv [taps, K_in, M]; M padded to 128.
    GW proj(const std::string & p, bool has_bias, int taps, int pad) {
        GW g;
        const RawTensor * t = need(p + ".weight");
        if (!t) return g;
        const int M = (int)(taps == 1 ? t->ne[1] : t->ne[2]);
        const int K_in = (int)(taps == 1 ? t->ne[0] : t->ne[1]);
        if (taps > 1 && t->ne[0] != taps) { fprintf(stderr, "tsd: %s: kernel size %lld != %d\n", p.c_str(), (long long)t->ne[0], taps); rc = TSD_ERR_ARG; return g; }
        const int Mp = (M + 127) / 128 * 128;
        g.M = Mp; g.K_in = K_in; g.taps = taps; g.pad = pad; g.m_valid = M;
        std::vector<int> map(Mp);
        for (int r = 0; r < Mp; ++r) map[r] = r < M ? r : -1;
        if (q8_gemm({t}, taps, K_in)) {
            if (!alloc_q8(g, Mp, K_in)) return g;
            repack_q8(g.q, g.qs, Mp, map, t, K_in);
        } else {
            g.w = reinterpret_cast<__nv_bfloat16 *>(m.dalloc((size_t)Mp * taps * K_in * 2));
            if (!g.w) { rc = TSD_ERR_CUDA; return g; }
            repack(g.w, (long long)taps * K_in, map, t, K_in, taps);
        }
        if (has_bias) g.bias = bias_f32(p + ".bias", nullptr, Mp);
        consumed.push_back(p + ".weight");
        return g;
    }
    // qkv: output rows f = 3c + j -> j*H + c (Q | K | V blocks).
    GW qkv(const std::string & p) {
        GW g;
        const RawTensor * t = need(p + ".weight");
        if (!t) return g;
        const int H = m.H;
        if (t->ne[0] != H || t->ne[1] != 3 * H) { rc = TSD_ERR_ARG; return g; }
        std::vector<int> map(3 * H);
        for (int j = 0; j < 3; ++j)
            for (int c = 0; c < H; ++c) map[j * H + c] = 3 * c + j;
        g.M = 3 * H; g.K_in = H; g.taps = 1; g.pad = 0; g.m_valid = 3 * H;
        if (q8_gemm({t}, 1, H)) {
            if (!alloc_q8(g, 3 * H, H)) return g;
            repack_q8(g.q, g.qs, 3 * H, map, t, H);
        } else {
            g.w = reinterpret_cast<__nv_bfloat16 *>(m.dalloc((size_t)3 * H * H * 2));
            if (!g.w) { rc = TSD_ERR_CUDA; return g; }
            repack(g.w, H, map, t, H, 1);
        }
        g.bias = bias_f32(p + ".bias", &map);
        consumed.push_back(p + ".weight");
        return g;
    }
    // SwiGLU pair: w1, w3 ([K_in, F] or [taps, K_in, F]) as one matrix with alternating rows.
    GW w13(const std::string & p, int taps, int pad) {
        GW g;
        const RawTensor * t1 = need(p + ".w1.weight");
        const RawTensor * t3 = need(p + ".w3.weight");
        if (!t1 || !t3) return g;
        const int F = (int)(taps == 1 ? t1->ne[1] : t1->ne[2]);
        const int K_in = (int)(taps == 1 ? t1->ne[0] : t1->ne[1]);
        if (F % 64) { fprintf(stderr, "tsd: %s: FFN width %d not a multiple of 64\n", p.c_str(), F); rc = TSD_ERR_UNSUPPORTED; return g; }
        g.M = 2 * F; g.K_in = K_in; g.taps = taps; g.pad = pad; g.m_valid = 2 * F;
        std::vector<int> m1(2 * F, -2), m3(2 * F, -2);
        for (int f = 0; f < F; ++f) { m1[2 * f] = f; m3[2 * f + 1] = f; }
        if (q8_gemm({t1, t3}, taps, K_in)) {
            if (!alloc_q8(g, 2 * F, K_in)) return g;
            repack_q8(g.q, g.qs, 2 * F, m1, t1, K_in);
            repack_q8(g.q, g.qs, 2 * F, m3, t3, K_in);
        } else {
            g.w = reinterpret_cast<__nv_bfloat16 *>(m.dalloc((size_t)2 * F * taps * K_in * 2));
            if (!g.w) { rc = TSD_ERR_CUDA; return g; }
            repack(g.w, (long long)taps * K_in, m1, t1, K_in, taps);
            repack(g.w, (long long)taps * K_in, m3, t3, K_in, taps);
        }
        consumed.push_back(p + ".w1.weight");
        consumed.push_back(p + ".w3.weight");
        return g;
    }
    VW vw(const std::string & p, bool has_bias) {
        VW v;
        const RawTensor * t = need(p + ".weight");
        if (!t) return v;
        if (t->type == GT_F16) {   // the GEMV reads F32 / BF16 / Q8_0; widen F16 once
            float * d = reinterpret_cast<float *>(m.dalloc((size_t)t->n() * 4));
            to_f32_kernel<<<(unsigned)((t->n() + 255) / 256), 256>>>(t->d, t->type, t->n(), d);
            v.w = d; v.type = GT_F32;
        } else {
            v.w = t->d; v.type = t->type;
        }
        v.K = (int)t->ne[0]; v.M = (int)t->ne[1];
        if (has_bias) v.bias = bias_f32(p + ".bias");
        return v;
    }
    const float * gain(const std::string & n) {
        const RawTensor * t = need(n);
        if (!t) return nullptr;
        if (t->type != GT_F32 || t->n() != 64) { rc = TSD_ERR_UNSUPPORTED; return nullptr; }
        return reinterpret_cast<const float *>(t->d);
    }

    void run() {
        Model & M = m;
        M.H = M.hp.hidden;
        M.nh = M.hp.n_head;
        M.L = M.hp.latent_dim;
        if (M.H % 128 || M.nh <= 0 || M.H / M.nh != 64 || M.H != M.nh * 64) {
            fprintf(stderr, "tsd: unsupported hidden %d / heads %d (head_dim must be 64, hidden a multiple of 128)\n", M.H, M.nh);
            rc = TSD_ERR_UNSUPPORTED;
            return;
        }
        const int n_joint = M.hp.depth - M.hp.fused_depth;
        if (n_joint < 1 || M.hp.fused_depth < 0) { rc = TSD_ERR_ARG; return; }
        const RawTensor * f1 = need("audio_input_proj.2.w1.weight");
        if (!f1) return;
        M.F = (int)f1->ne[2];
        // ---- pre-processing (mmdit.cpp:150-200) ----
        M.ap0 = proj("audio_input_proj.0", true, 3, 1);
        M.ap13 = w13("audio_input_proj.2", 3, 1);
        M.ap2 = proj("audio_input_proj.2.w2", false, 3, 1);
        M.te0 = vw("t_embed.mlp.0", true);
        M.te2 = vw("t_embed.mlp.2", true);
        M.cp0 = proj("clip_input_proj.0", true, 1, 0);
        M.cp13 = w13("clip_input_proj.2", 3, 1);
        M.cp2 = proj("clip_input_proj.2.w2", false, 3, 1);
        const RawTensor * pe = need("sync_pos_emb");
        if (pe) {
            M.sync_dim = (int)pe->ne[0];
            if (pe->type != GT_F32 || pe->ne[1] != 8) { rc = TSD_ERR_UNSUPPORTED; return; }
            M.sync_pe = reinterpret_cast<const float *>(pe->d);
        }
        M.sp0 = proj("sync_input_proj.0", true, 7, 3);
        M.sp13 = w13("sync_input_proj.2", 3, 1);
        M.sp2 = proj("sync_input_proj.2.w2", false, 3, 1);
        M.tp0 = proj("text_input_proj.0", true, 1, 0);
        M.tp13 = w13("text_input_proj.2", 1, 0);
        M.tp2 = proj("text_input_proj.2.w2", false, 1, 0);
        M.tcp = vw("text_cond_proj", true);
        M.ccp = vw("clip_cond_proj", true);
        {
            VW a = vw("global_cond_mlp.w1", false), b = vw("global_cond_mlp.w3", false);
            M.gc13 = a; M.gc13.w2 = b.w;
            if (a.type != b.type) { rc = TSD_ERR_UNSUPPORTED; return; }
        }
        M.gc2 = vw("global_cond_mlp.w2", false);
        if (rc) return;
        M.clip_dim = M.cp0.K_in;
        M.t5_dim = M.tp0.K_in;
        M.text_dim = M.tcp.K;
        if (M.clip_dim % 64 || M.sync_dim % 64 || M.t5_dim % 64 || M.text_dim > M.t5_dim || M.L % 64) {
            rc = TSD_ERR_UNSUPPORTED;
            return;
        }
        // ---- stacked per-token adaLN (joint latent blocks, fused blocks, final layer) ----
        struct AdaSrc { std::string name; long long off; int rows; };
        std::vector<AdaSrc> ada;
        long long rows = 0;
        auto add_ada = [&](const std::string & p) -> long long {
            const RawTensor * t = need(p + ".weight");
            if (!t) return 0;
            const long long off = rows;
            ada.push_back({p, off, (int)t->ne[1]});
            rows += t->ne[1];
            return off;
        };
        M.joint.resize(n_joint);
        for (int i = 0; i < n_joint; ++i) {
            const bool pre_only = (i == n_joint - 1);
            const std::string jb = "joint_blocks." + std::to_string(i);
            const char * names[3] = {".latent_block", ".clip_block", ".text_block"};
            for (int s = 0; s < 3; ++s) {
                StreamW & w = M.joint[i][s];
                const std::string p = jb + names[s];
                w.present = true;
                w.pre_only = (s > 0) && pre_only;
                w.conv = (s != 2);
                if (s == 0) { w.ada_off = add_ada(p + ".adaLN_modulation.1"); w.ada_rows = 6 * M.H; }
                else w.ada = vw(p + ".adaLN_modulation.1", true);
                w.qkv = qkv(p + ".attn.qkv");
                w.qg = gain(p + ".attn.q_norm.weight");
                w.kg = gain(p + ".attn.k_norm.weight");
                if (!w.pre_only) {
                    const int taps = w.conv ? 3 : 1, pad = w.conv ? 1 : 0;
                    w.l1 = proj(p + ".linear1", true, taps, pad);
                    w.w13 = w13(p + ".ffn", taps, pad);
                    w.w2 = proj(p + ".ffn.w2", false, taps, pad);
                }
            }
        }
        // The clip / text adaLN of every joint block reads the same [H] conditioning (global_c),
        // so their weights are stacked row-wise, in their stored type, into one matrix that one
        // GEMV launch per forward streams (mmdit.cpp:209 for the clip and text blocks).
        if (!rc) {
            long long ct_rows = 0;
            int ct_type = -1;
            bool ok = true;
            for (auto & blk : M.joint)
                for (int s = 1; s < 3; ++s) {
                    const VW & v = blk[s].ada;
                    if (!v.w || !v.bias || v.w2 || v.K != M.H || (ct_type >= 0 && v.type != ct_type)) ok = false;
                    ct_type = v.type;
                    ct_rows += v.M;
                }
            if (ok && ct_rows > 0) {
                const size_t rowb = ggml_nbytes(ct_type, M.H);
                auto * w = reinterpret_cast<uint8_t *>(M.dalloc((size_t)ct_rows * rowb));
                auto * b = reinterpret_cast<float *>(M.dalloc((size_t)ct_rows * 4));
                if (!w || !b) { rc = TSD_ERR_CUDA; return; }
                long long off = 0;
                for (int i = 0; i < (int)M.joint.size(); ++i)
                    for (int s = 1; s < 3; ++s) {
                        StreamW & st = M.joint[i][s];
                        if (cudaMemcpy(w + off * rowb, st.ada.w, (size_t)st.ada.M * rowb, cudaMemcpyDeviceToDevice) != cudaSuccess ||
                            cudaMemcpy(b + off, st.ada.bias, (size_t)st.ada.M * 4, cudaMemcpyDeviceToDevice) != cudaSuccess) {
                            rc = TSD_ERR_CUDA;
                            return;
                        }
                        st.ada_ct_off = off;
                        off += st.ada.M;
                        consumed.push_back("joint_blocks." + std::to_string(i) + (s == 1 ? ".clip_block" : ".text_block") +
                                           ".adaLN_modulation.1.weight");
                    }
                M.ada_ct.w = w; M.ada_ct.type = ct_type; M.ada_ct.M = (int)ct_rows; M.ada_ct.K = M.H; M.ada_ct.bias = b;
            }
        }
        M.fused.resize(M.hp.fused_depth);
        for (int i = 0; i < M.hp.fused_depth; ++i) {
            StreamW & w = M.fused[i];
            const std::string p = "fused_blocks." + std::to_string(i);
            w.present = true; w.conv = true;
            w.ada_off = add_ada(p + ".adaLN_modulation.1"); w.ada_rows = 6 * M.H;
            w.qkv = qkv(p + ".attn.qkv");
            w.qg = gain(p + ".attn.q_norm.weight");
            w.kg = gain(p + ".attn.k_norm.weight");
            w.l1 = proj(p + ".linear1", true, 3, 1);
            w.w13 = w13(p + ".ffn", 3, 1);
            w.w2 = proj(p + ".ffn.w2", false, 3, 1);
        }
        M.final_ada_off = add_ada("final_layer.adaLN_modulation.1");
        M.fconv = proj("final_layer.conv", true, 7, 3);
        if (rc) return;
        for (const auto & a : ada)
            if (a.rows != (a.name.rfind("final_layer", 0) == 0 ? 2 : 6) * M.H) {
                fprintf(stderr, "tsd: %s has %d rows\n", a.name.c_str(), a.rows);
                rc = TSD_ERR_ARG;
                return;
            }
        // rows is a multiple of 128 because H is.
        M.ada_lat.M = (int)rows; M.ada_lat.K_in = M.H; M.ada_lat.taps = 1; M.ada_lat.m_valid = (int)rows;
        bool ada_q8 = !ada.empty();
        for (const auto & a : ada) ada_q8 = ada_q8 && q8_gemm({need(a.name + ".weight")}, 1, M.H);
        if (ada_q8) {
            if (!alloc_q8(M.ada_lat, rows, M.H)) return;
        } else {
            M.ada_lat.w = reinterpret_cast<__nv_bfloat16 *>(M.dalloc((size_t)rows * M.H * 2));
            if (!M.ada_lat.w) { rc = TSD_ERR_CUDA; return; }
        }
        std::vector<float> hb((size_t)rows, 0.f);
        for (const auto & a : ada) {
            const RawTensor * t = need(a.name + ".weight");
            std::vector<int> map(a.rows);
            for (int r = 0; r < a.rows; ++r) map[r] = r;
            if (ada_q8) repack_q8(M.ada_lat.q + a.off * M.H, M.ada_lat.qs + a.off, rows, map, t, M.H);
            else repack(M.ada_lat.w + a.off * M.H, M.H, map, t, M.H, 1);
            consumed.push_back(a.name + ".weight");
            const RawTensor * b = need(a.name + ".bias");
            if (!b || b->type != GT_F32 || b->host.empty()) { rc = rc ? rc : TSD_ERR_UNSUPPORTED; return; }
            memcpy(&hb[a.off], b->host.data(), (size_t)a.rows * 4);
        }
        M.ada_lat.bias = reinterpret_cast<float *>(M.dalloc(hb.size() * 4));
        if (!M.ada_lat.bias || cudaMemcpy(M.ada_lat.bias, hb.data(), hb.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
            rc = TSD_ERR_CUDA;
            return;
        }
        // learned empties used by the sampler (mmdit.cpp:350-353)
        need("empty_string_feat");
        need("empty_t5_feat");
    }
};

}  // namespace

int model_finalize(Model & m) {
    if (m.finalized) return TSD_ERR_STATE;
    TSD_CUDA_TRY(cudaSetDevice(m.device));
    Finalizer f{m};
    f.run();
    if (f.rc) return f.rc;
    TSD_CUDA_TRY(cudaDeviceSynchronize());
    for (const auto & n : f.consumed) {
        auto it = m.raw.find(n);
        if (it != m.raw.end() && it->second.d) { cudaFree(it->second.d); it->second.d = nullptr; }
    }
    m.d_err = reinterpret_cast<int *>(m.dalloc(256));
    if (!m.d_err) return TSD_ERR_CUDA;
    TSD_CUDA_TRY(cudaMemset(m.d_err, 0, 256));
    if (!m.h_err) TSD_CUDA_TRY(cudaHostAlloc(reinterpret_cast<void **>(&m.h_err), sizeof(int), cudaHostAllocDefault));
    m.finalized = true;
    return TSD_OK;
}

// ---------------------------------------------------------------------------------------------
// GGUF (v2/v3) reader: header, key/values, tensor infos, aligned data section.
// ---------------------------------------------------------------------------------------------
namespace {

struct Reader {
    std::ifstream f;
    bool ok = true;
    template <class T> T rd() {
        T v{};
        f.read(reinterpret_cast<char *>(&v), sizeof(T));
        if (!f) ok = false;
        return v;
    }
    std::string str() {
        const uint64_t n = rd<uint64_t>();
        if (!ok || n > (1u << 24)) { ok = false; return {}; }
        std::string s(n, '\0');
        f.read(&s[0], (std::streamsize)n);
        if (!f) ok = false;
        return s;
    }
};

enum { GG_U8, GG_I8, GG_U16, GG_I16, GG_U32, GG_I32, GG_F32, GG_BOOL, GG_STR, GG_ARR, GG_U64, GG_I64, GG_F64 };

struct KV { int type = -1; double num = 0; };

bool skip_value(Reader & r, int type) {
    switch (type) {
        case GG_U8: case GG_I8: case GG_BOOL: r.rd<uint8_t>(); break;
        case GG_U16: case GG_I16: r.rd<uint16_t>(); break;
        case GG_U32: case GG_I32: case GG_F32: r.rd<uint32_t>(); break;
        case GG_U64: case GG_I64: case GG_F64: r.rd<uint64_t>(); break;
        case GG_STR: r.str(); break;
        case GG_ARR: {
            const int at = (int)r.rd<uint32_t>();
            const uint64_t n = r.rd<uint64_t>();
            for (uint64_t i = 0; i < n && r.ok; ++i) skip_value(r, at);
            break;
        }
        default: return false;
    }
    return r.ok;
}

bool read_scalar(Reader & r, int type, KV & kv) {
    kv.type = type;
    switch (type) {
        case GG_U8: kv.num = r.rd<uint8_t>(); break;
        case GG_I8: kv.num = r.rd<int8_t>(); break;
        case GG_BOOL: kv.num = r.rd<uint8_t>() ? 1 : 0; break;
        case GG_U16: kv.num = r.rd<uint16_t>(); break;
        case GG_I16: kv.num = r.rd<int16_t>(); break;
        case GG_U32: kv.num = r.rd<uint32_t>(); break;
        case GG_I32: kv.num = r.rd<int32_t>(); break;
        case GG_F32: kv.num = r.rd<float>(); break;
        case GG_U64: kv.num = (double)r.rd<uint64_t>(); break;
        case GG_I64: kv.num = (double)r.rd<int64_t>(); break;
        case GG_F64: kv.num = r.rd<double>(); break;
        default: kv.type = -1; return skip_value(r, type);
    }
    return r.ok;
}

}  // namespace

int model_load_gguf(const char * path, int device, Model ** out) {
    Reader r;
    r.f.open(path, std::ios::binary);
    if (!r.f) { fprintf(stderr, "tsd: cannot open '%s'\n", path); return TSD_ERR_IO; }
    char magic[4];
    r.f.read(magic, 4);
    if (!r.f || memcmp(magic, "GGUF", 4) != 0) { fprintf(stderr, "tsd: '%s' is not a GGUF file\n", path); return TSD_ERR_IO; }
    const uint32_t version = r.rd<uint32_t>();
    if (version < 2 || version > 3) { fprintf(stderr, "tsd: unsupported GGUF version %u\n", version); return TSD_ERR_IO; }
    const uint64_t n_tensors = r.rd<uint64_t>(), n_kv = r.rd<uint64_t>();
    std::unordered_map<std::string, KV> kvs;
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        std::string key = r.str();
        const int type = (int)r.rd<uint32_t>();
        KV kv;
        if (!read_scalar(r, type, kv)) break;
        kvs[key] = kv;
    }
    struct TI { std::string name; int64_t ne[4]; int type; uint64_t off; };
    std::vector<TI> tis;
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        TI ti;
        ti.name = r.str();
        const uint32_t nd = r.rd<uint32_t>();
        if (nd > 4) { r.ok = false; break; }
        for (int d = 0; d < 4; ++d) ti.ne[d] = 1;
        for (uint32_t d = 0; d < nd; ++d) ti.ne[d] = (int64_t)r.rd<uint64_t>();
        ti.type = (int)r.rd<uint32_t>();
        ti.off = r.rd<uint64_t>();
        tis.push_back(ti);
    }
    if (!r.ok) { fprintf(stderr, "tsd: truncated GGUF header in '%s'\n", path); return TSD_ERR_IO; }
    uint64_t align = 32;
    if (kvs.count("general.alignment") && kvs["general.alignment"].num > 0) align = (uint64_t)kvs["general.alignment"].num;
    const uint64_t hdr_end = (uint64_t)r.f.tellg();
    const uint64_t data_off = (hdr_end + align - 1) / align * align;

    auto geti = [&](const char * k, int def) -> int {
        auto it = kvs.find(k);
        if (it == kvs.end()) return def;
        const int t = it->second.type;   // get_i32 accepts i32 / u32 / i64 / bool (ts_model.cpp:119-129)
        if (t == GG_I32 || t == GG_U32 || t == GG_I64 || t == GG_BOOL) return (int)it->second.num;
        return def;
    };
    auto getf = [&](const char * k, float def) -> float {
        auto it = kvs.find(k);
        if (it == kvs.end()) return def;
        const int t = it->second.type;   // get_f32 accepts f32 / f64 / i32 (ts_model.cpp:131-140)
        if (t == GG_F32 || t == GG_F64 || t == GG_I32) return (float)it->second.num;
        return def;
    };
    tsd_hparams hp;
    hp.hidden = geti("dit.hidden_dim", 1024);
    hp.n_head = geti("dit.num_heads", 16);
    hp.depth = geti("dit.depth", 21);
    hp.fused_depth = geti("dit.fused_depth", 14);
    hp.latent_dim = geti("dit.latent_dim", 64);
    hp.rope_theta = getf("dit.rope_theta", 10000.f);
    hp.t_max_period = getf("dit.t_embed_max_period", 1.f);

    // every tensor's type and byte range are checked against the file before any device work,
    // so a truncated or inconsistent file fails as TSD_ERR_IO without touching the GPU (the
    // reference's loader fails on its first short read, ts_model.cpp:33-35)
    r.f.clear();
    r.f.seekg(0, std::ios::end);
    const uint64_t file_size = (uint64_t)r.f.tellg();
    for (const TI & ti : tis) {
        for (int d = 0; d < 4; ++d)
            if (ti.ne[d] < 1 || ti.ne[d] > (int64_t(1) << 40)) {
                fprintf(stderr, "tsd: tensor '%s' has a bad shape in '%s'\n", ti.name.c_str(), path);
                return TSD_ERR_IO;
            }
        const size_t nb = ggml_nbytes(ti.type, ti.ne[0] * ti.ne[1] * ti.ne[2] * ti.ne[3]);
        if (!nb) { fprintf(stderr, "tsd: tensor '%s' has unsupported type %d\n", ti.name.c_str(), ti.type); return TSD_ERR_UNSUPPORTED; }
        if (ti.off > file_size || data_off + ti.off + nb > file_size) {
            fprintf(stderr, "tsd: truncated GGUF '%s': tensor '%s' needs bytes up to %llu of a %llu-byte file\n", path,
                    ti.name.c_str(), (unsigned long long)(data_off + ti.off + nb), (unsigned long long)file_size);
            return TSD_ERR_IO;
        }
    }

    std::unique_ptr<Model> m(new Model());
    m->hp = hp;
    m->device = device;
    if (cudaSetDevice(device) != cudaSuccess) return TSD_ERR_CUDA;
    cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, device);
    std::vector<uint8_t> buf;
    for (const TI & ti : tis) {
        const int64_t n = ti.ne[0] * ti.ne[1] * ti.ne[2] * ti.ne[3];
        const size_t nb = ggml_nbytes(ti.type, n);
        if (!nb) { fprintf(stderr, "tsd: tensor '%s' has unsupported type %d\n", ti.name.c_str(), ti.type); return TSD_ERR_UNSUPPORTED; }
        buf.resize(nb);
        r.f.clear();
        r.f.seekg((std::streamoff)(data_off + ti.off));
        r.f.read(reinterpret_cast<char *>(buf.data()), (std::streamsize)nb);
        if (!r.f) { fprintf(stderr, "tsd: read failed for tensor '%s'\n", ti.name.c_str()); return TSD_ERR_IO; }
        const int rc = model_set_tensor(*m, ti.name.c_str(), ti.type, ti.ne, buf.data(), nb);
        if (rc) return rc;
    }
    const int rc = model_finalize(*m);
    if (rc) return rc;
    *out = m.release();
    return TSD_OK;
}

}  // namespace tsd
