// dit.cu — forward plan of the MM-DiT velocity evaluation on one B200.
//
// Restates ts_dit::forward (src/mmdit.cpp:119-342) as a fixed sequence of kernel launches over
// buffers allocated once per input shape (B, T, clip_S, sync_S, text_S, t5_S). The plan is
// built once (tensor maps encoded, grids chosen) and replayed; replays are captured into a
// CUDA graph. Token-major activations everywhere: x[b][t][H] f32 residual streams, bf16 GEMM
// operands, fp16 head-major Q/K/V shared by the three streams of a joint block.
#include "runtime.h"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <tuple>

namespace tsd {

Plan::~Plan() {
    for (cudaGraphExec_t g : graph)
        if (g) cudaGraphExecDestroy(g);
    for (cudaStream_t q : side)
        if (q) cudaStreamDestroy(q);
    for (cudaEvent_t e : events) cudaEventDestroy(e);
    if (copy_st) cudaStreamDestroy(copy_st);
    for (cudaEvent_t e : in_ev)
        if (e) cudaEventDestroy(e);
    if (prev_done) cudaEventDestroy(prev_done);
    for (void * p : allocs) cudaFree(p);
}

namespace {

struct Builder {
    Model & m;
    Plan & P;
    Builder(Model & m_, Plan & P_) : m(m_), P(P_) {
        const char * a = getenv("TSD_AUTOTUNE");
        autotune = a && *a == '1';
        tune_log = getenv("TSD_DEBUG_PLAN") != nullptr;
    }
    int rc = TSD_OK;
    std::string tag = "pre";   // label prefix of the ops being added
    // Split-K scratch shared by all GEMMs of the plan (they run one after another).
    static constexpr long long kWsFloats = 8ll << 20;   // 32 MB of partial tiles
    static constexpr int kCounters = 1 << 16;
    float * ws = nullptr;                  // per lane: concurrent GEMMs must not share split-K scratch
    int * counters = nullptr;
    float * ws_lane[1 + kSideLanes] = {};
    int * counters_lane[1 + kSideLanes] = {};
    int lane = 0;                          // lane of the ops being added
    bool inv = false;                      // the ops being added are conditioning-only
    // Optional plan-time autotuning of the GEMM tiling (TSD_AUTOTUNE=1): per distinct shape the
    // cost model's best few (token tile, K splits) choices are timed on the plan's own buffers
    // and the fastest kept. Off by default: the number of K splits sets the summation order, so
    // timing-noise-driven choices would make results differ (at bf16 rounding level) from run to
    // run; the model's choice is a fixed function of the shape. Decisions are kept process-wide
    // so that all plans of one process agree. Inputs hold whatever the buffers hold at build time:
    // the kernels' speed does not depend on the values, and every buffer they write is rewritten
    // by the forward itself.
    using TuneKey = std::tuple<int, int, int, int, int, int, int, int, int, int>;
    static std::map<TuneKey, std::tuple<int, int, int>> & tuned_cache() {
        static std::map<TuneKey, std::tuple<int, int, int>> c;
        return c;
    }
    cudaStream_t tune_st = nullptr;
    bool autotune = false, tune_log = false;
    ~Builder() { if (tune_st) cudaStreamDestroy(tune_st); }

    // Milliseconds per launch of L (1 warm-up, then 3 timed launches), or -1 on a launch error.
    float time_gemm(const GemmLaunch & L) {
        if (!tune_st && cudaStreamCreateWithFlags(&tune_st, cudaStreamNonBlocking) != cudaSuccess) return -1.f;
        cudaEvent_t e0, e1;
        if (cudaEventCreate(&e0) != cudaSuccess) return -1.f;
        if (cudaEventCreate(&e1) != cudaSuccess) { cudaEventDestroy(e0); return -1.f; }
        float ms = -1.f;
        bool ok = gemm_launch(L, tune_st) == cudaSuccess && cudaEventRecord(e0, tune_st) == cudaSuccess;
        for (int i = 0; ok && i < 3; ++i) ok = gemm_launch(L, tune_st) == cudaSuccess;
        ok = ok && cudaEventRecord(e1, tune_st) == cudaSuccess && cudaEventSynchronize(e1) == cudaSuccess &&
             cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess;
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        if (!ok) { cudaGetLastError(); return -1.f; }
        return ms / 3.f;
    }

    template <class T> T * alloc(size_t n) {
        void * p = nullptr;
        if (cudaMalloc(&p, std::max<size_t>(n * sizeof(T), 256)) != cudaSuccess) {
            rc = TSD_ERR_CUDA;
            return nullptr;
        }
        P.allocs.push_back(p);
        return reinterpret_cast<T *>(p);
    }
    void op(std::function<cudaError_t(cudaStream_t)> fn, int kind = OP_ELEM, double flops = 0, double bytes = 0,
            int launches = 1) {
        Op o;
        o.fn = std::move(fn);
        o.kind = kind; o.flops = flops; o.bytes = bytes; o.launches = launches;
        o.lane = lane;
        o.invariant = inv;
        o.label = tag + (kind == OP_GEMM ? " gemm" : kind == OP_GEMV ? " gemv" : kind == OP_ATTN ? " attn" : kind == OP_COPY ? " copy" : " elem");
        P.ops.push_back(std::move(o));
    }
    // Lane markers (see Op): fork lets the side lanes start after everything lane 0 has queued,
    // join makes lane 0 wait for everything the side lanes have queued.
    void mark(int sync) {
        Op o;
        o.sync = sync;
        o.kind = OP_COPY;
        o.launches = 0;
        o.label = sync == 1 ? "fork" : "join";
        P.ops.push_back(std::move(o));
    }
    // This lane's next ops read input group `g` (graph replay: wait for its copy to land).
    void wait_input(int g) {
        Op o;
        o.sync = 3;
        o.input = g;
        o.kind = OP_COPY;
        o.launches = 0;
        o.lane = lane;
        o.label = "wait input";
        P.ops.push_back(std::move(o));
    }
    void copy(void * dst, const void * src, size_t bytes) {
        op([=](cudaStream_t st) { return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, st); }, OP_COPY, 0,
           2.0 * bytes);
    }
    void snap(const std::string & name, const void * ptr, long long n, int kind = 0, int B = 0, int nh = 0, int S = 0,
              bool inject = false) {
        if (!P.ops.empty()) P.ops.back().snaps.push_back(Snap{name, ptr, n, kind, B, nh, S, inject});
    }
    // A residual stream at a block boundary: reported, and offered for teacher forcing.
    void inject_point(const std::string & name, float * ptr, long long n,
                      std::function<cudaError_t(cudaStream_t)> after_inject = {}) {
        snap(name, ptr, n, 0, 0, 0, 0, true);
        if (!P.ops.empty()) P.ops.back().snaps.back().after_inject = std::move(after_inject);
    }

    // GEMM over activations X [nbatch][S][K_in] (row stride xrs, batch stride xbs, elements).
    void gemm(const GW & w, const void * X, int nbatch, int S, long long xrs, long long xbs, int mode, int act,
              void * out, int out_bf16, long long ldo, float * resid = nullptr, long long ldr = 0,
              const float * gate = nullptr, long long ldg = 0, int gate_div = 1, int swiglu = 0, int max_splits = 8,
              int out_cblk = 0, long long out_cstride = 0) {
        if (rc) return;
        // Linear layers over a contiguous batch run as one long token sequence.
        // (not the QKV projection: its epilogue stores per item, clipped at the stream's length)
        if (mode != EPI_QKV && w.taps == 1 && xbs == (long long)S * xrs && nbatch > 1) { S *= nbatch; nbatch = 1; }
        GemmLaunch L;
        const int M = w.M;
        int force_bn = 0, force_sp = 0, force_pair = -1;
        const TuneKey key{m.device, M, w.K_in, w.taps, nbatch, S, mode, act, out_bf16, max_splits};
        auto & tuned = tuned_cache();
        auto hit = autotune ? tuned.find(key) : tuned.end();
        if (autotune && hit != tuned.end()) {
            std::tie(force_bn, force_sp, force_pair) = hit->second;
        }
        const void * Wp = w.q ? static_cast<const void *>(w.q) : static_cast<const void *>(w.w);
        if (!gemm_plan(L, Wp, M, w.K_in, w.taps, w.pad, swiglu, X, nbatch, S, xrs, xbs, m.num_sms, max_splits,
                       kWsFloats, kCounters, true, force_bn, force_sp, w.qs, force_pair)) {
            fprintf(stderr, "tsd: gemm plan failed (M %d K %d taps %d S %d)\n", M, w.K_in, w.taps, S);
            rc = TSD_ERR_ARG;
            return;
        }
        GemmParams & p = L.p;
        p.mode = mode; p.act = act;
        p.m_valid = swiglu ? w.M / 2 : w.m_valid;
        p.bias = w.bias;
        p.out = out; p.out_bf16 = out_bf16; p.ldo = ldo;
        p.out_cblk = out_cblk; p.out_cstride = out_cstride;
        p.resid = resid; p.ldr = ldr; p.gate = gate; p.ldg = ldg; p.gate_div = gate_div;
        p.ws = ws_lane[lane]; p.counters = counters_lane[lane];
        p.err = m.d_err;
        if (mode == EPI_QKV) {
            p.q_out = qspec.q; p.k_out = qspec.k; p.v_out = qspec.v;
            p.qg = qspec.qg; p.kg = qspec.kg; p.rope = qspec.rope;
            p.hidden = qspec.hidden; p.nh = qspec.nh; p.Sj = qspec.Sj; p.s_off = qspec.s_off; p.s_item = qspec.s_item;
        }
        gemm_finalize(L);
        if (autotune && hit == tuned.end()) {
            int bns[8], sps[8], prs[8];
            const int nc = gemm_candidates(M, w.K_in, w.taps, nbatch, S, m.num_sms, max_splits, kWsFloats, kCounters,
                                           true, 8, bns, sps, prs);
            float best = time_gemm(L);
            std::tuple<int, int, int> pick{L.p.BN, L.p.splits, L.p.pair};
            if (tune_log) fprintf(stderr, "tsd tune: M=%d K=%d taps=%d nb=%d S=%d mode=%d: model BN=%d sp=%d pair=%d %.1f us", M,
                                  w.K_in, w.taps, nbatch, S, mode, L.p.BN, L.p.splits, L.p.pair, best * 1000.f);
            for (int i = 1; i < nc; ++i) {
                GemmLaunch C = L;
                if (!gemm_plan(C, Wp, M, w.K_in, w.taps, w.pad, swiglu, X, nbatch, S, xrs, xbs, m.num_sms, max_splits,
                               kWsFloats, kCounters, true, bns[i], sps[i], w.qs, prs[i]))
                    continue;
                const GemmParams & q = L.p;   // same epilogue, new tiling
                GemmParams & cp = C.p;
                const int BN = cp.BN, nt = cp.n_tiles, sp = cp.splits, cs = cp.csplit, order = cp.order, st = cp.stages;
                const int aq8 = cp.a_q8, pr = cp.pair, kpb = cp.kpb, ga = cp.gather, ipt = cp.ipt, bni = cp.bni;
                const int groups = cp.groups;
                cp = q;
                cp.BN = BN; cp.n_tiles = nt; cp.splits = sp; cp.csplit = cs; cp.order = order; cp.stages = st;
                cp.a_q8 = aq8; cp.pair = pr; cp.kpb = kpb;   // the tiling fields that go with C's tensor maps
                cp.gather = ga; cp.ipt = ipt; cp.bni = bni; cp.groups = groups;
                gemm_finalize(C);
                const float t = time_gemm(C);
                if (tune_log) fprintf(stderr, " | BN=%d sp=%d pair=%d %.1f us", BN, sp, pr, t * 1000.f);
                if (t > 0.f && (best < 0.f || t < best)) { best = t; pick = {BN, sp, pr}; L = C; }
            }
            if (tune_log) fprintf(stderr, " -> BN=%d sp=%d pair=%d\n", std::get<0>(pick), std::get<1>(pick), std::get<2>(pick));
            tuned[key] = pick;
        }
        const double n_tok = (double)nbatch * S, kdim = (double)w.taps * w.K_in;
        const double flops = 2.0 * (swiglu ? 2 * p.m_valid : p.m_valid) * n_tok * kdim;
        const double bytes = (w.q ? 34.0 / 32.0 : 2.0) * M * kdim + 2.0 * n_tok * w.K_in +
                             n_tok * (mode == EPI_GATE_RESID ? 12.0 : (out_bf16 ? 2.0 : 4.0)) * p.m_valid;
        op([L](cudaStream_t st) { return gemm_launch(L, st); }, OP_GEMM, flops, bytes);
        char buf[160];
        snprintf(buf, sizeof buf, " M=%d N=%d K=%d taps=%d BN=%d grid=%ux%ux%u mode=%d%s%s", p.m_valid, nbatch * S,
                 w.taps * w.K_in, w.taps, p.BN, L.grid.x, L.grid.y, L.grid.z, mode, p.epi_tma ? " tma" : "",
                 p.a_q8 ? " q8" : "");
        P.ops.back().label += buf;
    }
    // QKV projection whose epilogue applies the per-head RMSNorm (Q, K) and RoPE (rope != null)
    // and writes fp16 Q / K / V head-major at this stream's offset in the joint sequence
    // (replaces qk_norm_rope after a plain f32 QKV GEMM).
    struct QkvSpec {
        __half * q = nullptr, * k = nullptr, * v = nullptr;
        const float * qg = nullptr, * kg = nullptr;
        const float2 * rope = nullptr;
        int Sj = 0, s_off = 0, s_item = 0;
        int hidden = 0, nh = 0;      // rows per Q / K / V section, heads stored
    } qspec;
    // Head-parallel plans use this rank's slice of the QKV rows (sections of hpar.sec rows, nl
    // heads each) in place of the full weight.
    void gemm_qkv(const StreamW & w, const GW * slice, const void * X, int nbatch, int S, const float2 * rope,
                  __half * Q, __half * K, __half * V, int Sj, int s_off) {
        qspec.q = Q; qspec.k = K; qspec.v = V; qspec.qg = w.qg; qspec.kg = w.kg; qspec.rope = rope;
        qspec.Sj = Sj; qspec.s_off = s_off; qspec.s_item = S;
        qspec.hidden = slice ? m.hpar.sec : m.H;
        qspec.nh = slice ? m.hpar.nl : m.nh;
        gemm(slice ? *slice : w.qkv, X, nbatch, S, m.H, (long long)S * m.H, EPI_QKV, ACT_NONE, nullptr, 0, 0, nullptr, 0,
             nullptr, 0, 1, 0, /*max_splits=*/1);
    }
    // Attention of one layer; returns the buffer the out-projection reads (the full [B][S][H]
    // attention output). Head-parallel: this rank's heads into the layer's exchange buffer, this
    // rank's column block pushed into every peer's copy of that buffer, then a wait for the
    // peers' blocks.
    __nv_bfloat16 * attention(const __half * Q, const __half * K, const __half * V, int B, int S, __nv_bfloat16 * ao,
                              int * err) {
        const int H = m.H;
        HeadParallel & hp = m.hpar;
        AttnLaunch A;
        if (!hp.connected) {
            if (!attn_plan(A, Q, K, V, B, m.nh, S, ao, H, err)) { rc = TSD_ERR_ARG; return ao; }
            op([A](cudaStream_t st) { return attn_launch(A, st); }, OP_ATTN, 4.0 * B * m.nh * 64.0 * S * S,
               6.0 * B * m.nh * 64.0 * S + 2.0 * B * S * H);
            return ao;
        }
        const long long off = hp_carve(m, (size_t)B * S * H * 2);
        const int slot = hp_next_slot(m);
        if (off < 0 || slot < 0) {
            fprintf(stderr, "tsd: head-parallel exchange arena exhausted (give tsd_hp_init a larger arena)\n");
            rc = TSD_ERR_ARG;
            return ao;
        }
        auto * X = reinterpret_cast<__nv_bfloat16 *>(hp.arena + off);
        const long long col = (long long)hp.h0 * 64;    // this rank's columns of the [B][S][H] rows
        if (!attn_plan(A, Q, K, V, B, hp.nl, S, X + col, H, err)) { rc = TSD_ERR_ARG; return ao; }
        __nv_bfloat16 * pdst[kMaxHpRanks] = {};
        unsigned * pflag[kMaxHpRanks] = {};
        int np = 0;
        for (int r = 0; r < hp.world; ++r) {
            if (r == hp.rank) continue;
            pdst[np] = reinterpret_cast<__nv_bfloat16 *>(hp.peer[r] + off);
            pflag[np] = hp_counter(m, r, slot, hp.rank);
            ++np;
        }
        op([A](cudaStream_t st) { return attn_launch(A, st); }, OP_ATTN, 4.0 * B * hp.nl * 64.0 * S * S,
           6.0 * B * hp.nl * 64.0 * S + 2.0 * B * S * H);
        // this rank's column block of every row, pushed into the peers' buffers over NVLink
        const int rows = B * S, c0 = hp.h0 * 64, nc = hp.nl * 64;
        std::array<__nv_bfloat16 *, kMaxHpRanks> d;
        std::array<unsigned *, kMaxHpRanks> f;
        for (int k = 0; k < kMaxHpRanks; ++k) { d[k] = pdst[k]; f[k] = pflag[k]; }
        const __nv_bfloat16 * src = X;
        op([=](cudaStream_t st) { return hp_push_launch(src, d.data(), f.data(), np, rows, H, c0, nc, st); },
           OP_COPY, 0, 2.0 * rows * nc * np);
        const unsigned ctas = (unsigned)hp_push_ctas(rows);
        const unsigned * counters = hp_counter(m, hp.rank, slot, 0);
        const unsigned * epoch = epoch_ptr;
        const int rank = hp.rank, world = hp.world;
        op([=](cudaStream_t st) { return hp_wait_launch(counters, epoch, rank, world, ctas, err, st); });
        return X;
    }
    unsigned * epoch_ptr = nullptr;
    // Few-token GEMV over B items (chunks of 8 tokens). With more than 8 tokens a GEMV would
    // stream the weight once per chunk of 8, so a single BF16 weight (the GEMV also rounds x to
    // bf16 for it) runs on the tensor-core GEMM instead, after a cast of x to bf16.
    void gemv(const VW & w, const float * x, long long ldx, int N, int act, float * y, long long ldy, int y_bf16 = 0) {
        if (rc) return;
        if (N > 8 && w.type == GT_BF16 && !w.w2 && w.M % 128 == 0 && w.K % 64 == 0 && ldx == w.K) {
            auto * xb = alloc<__nv_bfloat16>((size_t)N * w.K);
            if (rc) return;
            const long long n = (long long)N * w.K;
            op([=](cudaStream_t st) { return cast_f32_bf16(x, n, xb, st); });
            GW g;
            g.w = const_cast<__nv_bfloat16 *>(static_cast<const __nv_bfloat16 *>(w.w));
            g.M = w.M; g.K_in = w.K; g.taps = 1; g.pad = 0; g.m_valid = w.M;
            g.bias = const_cast<float *>(w.bias);
            gemm(g, xb, 1, N, w.K, (long long)N * w.K, EPI_STORE, act, y, y_bf16, ldy);
            return;
        }
        const VW wc = w;
        int * const err = m.d_err;
        op([wc, x, ldx, N, act, y, ldy, y_bf16, err](cudaStream_t st) {
            for (int n0 = 0; n0 < N; n0 += 8) {
                const int nn = std::min(8, N - n0);
                cudaError_t e = gemv_launch(wc.w, wc.type, wc.w2, wc.M, wc.K, x + n0 * ldx, ldx, nn, wc.bias, act,
                                            wc.type == GT_BF16, y_bf16 ? (void *)((__nv_bfloat16 *)y + n0 * ldy) : (void *)(y + n0 * ldy),
                                            y_bf16, ldy, st, err);
                if (e != cudaSuccess) return e;
            }
            return cudaSuccess;
        }, OP_GEMV, 2.0 * w.M * w.K * N * (w.w2 ? 2 : 1),
           (double)ggml_nbytes(w.type, (long long)w.M * w.K) * (w.w2 ? 2 : 1) * ((N + 7) / 8) + 4.0 * N * (w.K + w.M),
           (N + 7) / 8);
    }

    void build() {
        const Shape & sh = P.sh;
        const int B = sh.B, T = sh.T, H = m.H, F = m.F, L = m.L, nh = m.nh;
        const int cS = sh.clip_S, yS = sh.sync_S;
        const int St = sh.text_S + sh.t5_S, Sj = T + cS + St;
        const int maxS = std::max(std::max(T, cS), std::max(yS, St));
        P.St = St; P.Sj = Sj; P.maxS = maxS;
        const int R = m.ada_lat.M;
        // ---- buffers ----
        P.lat_in = alloc<float>((size_t)B * L * T);
        P.clip_in = alloc<float>((size_t)B * cS * m.clip_dim);
        P.sync_in = alloc<float>((size_t)B * yS * m.sync_dim);
        P.text_in = alloc<float>((size_t)B * std::max(1, sh.text_S) * m.text_dim);
        P.t5_in = alloc<float>((size_t)B * std::max(1, sh.t5_S) * m.t5_dim);
        P.gtext_in = alloc<float>((size_t)B * m.text_dim);
        P.t_in = alloc<float>((size_t)B);
        P.flow = alloc<float>((size_t)B * T * L);
        auto * lat_tok = alloc<__nv_bfloat16>((size_t)B * T * L);
        auto * clip_tok = alloc<__nv_bfloat16>((size_t)B * cS * m.clip_dim);
        auto * sync_tok = alloc<__nv_bfloat16>((size_t)B * yS * m.sync_dim);
        auto * text_tok = alloc<__nv_bfloat16>((size_t)B * St * m.t5_dim);
        auto * a1 = alloc<__nv_bfloat16>((size_t)B * maxS * H);
        auto * hbuf = alloc<__nv_bfloat16>((size_t)B * maxS * F);
        auto * xn = alloc<__nv_bfloat16>((size_t)B * maxS * H);
        // per-lane copies for the joint blocks, whose three streams run on their own lanes
        __nv_bfloat16 * xn_l[3] = {xn, alloc<__nv_bfloat16>((size_t)B * maxS * H), alloc<__nv_bfloat16>((size_t)B * maxS * H)};
        __nv_bfloat16 * hb_l[3] = {hbuf, alloc<__nv_bfloat16>((size_t)B * maxS * F), alloc<__nv_bfloat16>((size_t)B * maxS * F)};
        __nv_bfloat16 * a1_l[3] = {a1, alloc<__nv_bfloat16>((size_t)B * maxS * H), alloc<__nv_bfloat16>((size_t)B * maxS * H)};
        float * x_lat = alloc<float>((size_t)B * T * H);
        float * x_clip = alloc<float>((size_t)B * cS * H);
        float * x_text = alloc<float>((size_t)B * St * H);
        float * x_clip0 = alloc<float>((size_t)B * cS * H);     // projected clip / text tokens: kept
        float * x_text0 = alloc<float>((size_t)B * St * H);     // across replays, copied into x_clip / x_text
        float * sync_out = alloc<float>((size_t)B * yS * H);
        float * temb = alloc<float>((size_t)B * H);
        float * te1 = alloc<float>((size_t)B * H);
        float * te = alloc<float>((size_t)B * H);
        float * text_fc = alloc<float>((size_t)B * H);
        float * cmean = alloc<float>((size_t)B * H);
        float * clip_fc = alloc<float>((size_t)B * H);
        float * gsum = alloc<float>((size_t)B * H);
        float * gch = alloc<float>((size_t)B * F);
        float * gcm = alloc<float>((size_t)B * H);
        float * gc = alloc<float>((size_t)B * H);
        float * sgc = alloc<float>((size_t)B * H);
        float * ext = alloc<float>((size_t)B * T * H);
        auto * sext = alloc<__nv_bfloat16>((size_t)B * T * H);
        float * mod_lat = alloc<float>((size_t)B * T * R);
        float * mod_c = alloc<float>((size_t)B * 6 * H);
        float * mod_ct = alloc<float>((size_t)B * std::max(1, m.ada_ct.M));
        float * mod_t = alloc<float>((size_t)B * 6 * H);
        const bool hpm = m.hpar.connected;
        const int nhl = hpm ? m.hpar.nl : nh;             // heads this rank computes
        auto * Qb = alloc<__half>((size_t)B * nhl * Sj * 64);
        auto * Kb = alloc<__half>((size_t)B * nhl * Sj * 64);
        auto * Vb = alloc<__half>((size_t)B * nhl * Sj * 64);
        auto * ao = alloc<__nv_bfloat16>((size_t)B * Sj * H);
        auto * rope_lat = alloc<float2>((size_t)T * 32);     // RoPE (cos, sin): latent positions, scale 1
        auto * rope_clip = alloc<float2>((size_t)cS * 32);   // clip positions, scale T / clip_S
        ws = alloc<float>((size_t)kWsFloats * (1 + kSideLanes));
        counters = alloc<int>((size_t)kCounters * (1 + kSideLanes));
        if (rc) return;
        if (cudaMemset(counters, 0, sizeof(int) * kCounters * (1 + kSideLanes)) != cudaSuccess) { rc = TSD_ERR_CUDA; return; }
        for (int l = 0; l <= kSideLanes; ++l) {
            ws_lane[l] = ws + (size_t)l * kWsFloats;
            counters_lane[l] = counters + (size_t)l * kCounters;
        }
        P.counters = counters;
        P.n_counters = kCounters * (1 + kSideLanes);
        int * err = m.d_err;
        // Per-token adaLN output is column-blocked: chunk k of the stacked weight rows is one
        // contiguous [B*T][H] plane at mod_lat + k * BTH (row stride H), so each block's
        // shift / scale / gate rows are dense and page-local.
        const long long BTH = (long long)B * T * H;
        // Values the op closures need, copied out of the plan and model: the closures outlive
        // this builder, so they must not reach P or m through the builder's `this`.
        float * const lat_in = P.lat_in, * const t_in = P.t_in, * const clip_in = P.clip_in;
        float * const sync_in = P.sync_in, * const text_in = P.text_in, * const t5_in = P.t5_in;
        const int clip_dim = m.clip_dim, sync_dim = m.sync_dim, text_dim = m.text_dim, t5_dim = m.t5_dim;
        const float * const sync_pe = m.sync_pe;
        const int text_S = sh.text_S, t5_S = sh.t5_S;
        const float theta = m.hp.rope_theta;
        // step-invariant RoPE tables, built once with the plan
        if (rope_table(T, 1.0f, theta, rope_lat, 0) != cudaSuccess ||
            rope_table(cS, (float)T / (float)cS, theta, rope_clip, 0) != cudaSuccess ||
            cudaStreamSynchronize(0) != cudaSuccess) {
            rc = TSD_ERR_CUDA;
            return;
        }

        op([err](cudaStream_t st) { return cudaMemsetAsync(err, 0, sizeof(int), st); }, OP_COPY, 0, 0, 0);
        if (hpm) {   // this plan's forward counter, read by its head-parallel waits
            const int pi = hp_next_plan(m);
            if (pi < 0) { rc = TSD_ERR_ARG; return; }
            unsigned * const ep = hp_epoch(m, pi);
            epoch_ptr = ep;
            op([ep](cudaStream_t st) { return hp_epoch_launch(ep, st); });
        }

        // The input projections are independent chains: audio, t-embed and sync on lane 0, clip
        // on lane 1, text on lane 2 (each lane with its own a1 / hbuf), joined before the
        // conditioning vectors that combine them. The clip, sync and text chains and the global
        // conditioning MLP depend on the conditioning inputs only (marked `inv`): their results
        // (x_clip0, x_text0, sync_out, gcm) are written by nothing else, so a replay with the same
        // conditioning may skip them; the per-step copies into the residual streams stay.
        mark(1);
        // ---- audio_input_proj (mmdit.cpp:150-155) ----
        tag = "pre.audio";
        wait_input(IN_LAT);
        op([=](cudaStream_t st) { return latent_to_tokens(lat_in, B, L, T, lat_tok, st); });
        gemm(m.ap0, lat_tok, B, T, L, (long long)T * L, EPI_STORE, ACT_SILU, a1, 1, H);
        gemm(m.ap13, a1, B, T, H, (long long)T * H, EPI_SWIGLU, ACT_NONE, hbuf, 1, F, nullptr, 0, nullptr, 0, 1, 1);
        gemm(m.ap2, hbuf, B, T, F, (long long)T * F, EPI_STORE, ACT_NONE, x_lat, 0, H);
        snap("x_in", x_lat, (long long)B * T * H);
        // ---- t_embed (mmdit.cpp:157-161, 305-313) ----
        tag = "pre.temb";
        const float maxp = m.hp.t_max_period;
        op([=](cudaStream_t st) { return timestep_embed(t_in, B, H, maxp, temb, st); });
        gemv(m.te0, temb, H, B, ACT_SILU, te1, H);
        gemv(m.te2, te1, H, B, ACT_NONE, te, H);
        snap("t_emb", te, (long long)B * H);
        // ---- clip (mmdit.cpp:164-167) ----
        tag = "pre.clip";
        lane = 1;
        wait_input(IN_CLIP);
        inv = true;
        op([=](cudaStream_t st) { return cast_f32_bf16(clip_in, (long long)B * cS * clip_dim, clip_tok, st); });
        gemm(m.cp0, clip_tok, B, cS, m.clip_dim, (long long)cS * m.clip_dim, EPI_STORE, ACT_SILU, a1_l[1], 1, H);
        gemm(m.cp13, a1_l[1], B, cS, H, (long long)cS * H, EPI_SWIGLU, ACT_NONE, hb_l[1], 1, F, nullptr, 0, nullptr, 0, 1, 1);
        gemm(m.cp2, hb_l[1], B, cS, F, (long long)cS * F, EPI_STORE, ACT_NONE, x_clip0, 0, H);
        snap("clip_pp", x_clip0, (long long)B * cS * H);
        inv = false;
        copy(x_clip, x_clip0, (size_t)B * cS * H * sizeof(float));
        lane = 0;
        // ---- sync (mmdit.cpp:168-177) ----
        tag = "pre.sync";
        wait_input(IN_SYNC);
        inv = true;
        op([=](cudaStream_t st) { return sync_prep(sync_in, B, yS, sync_dim, sync_pe, sync_tok, st); });
        gemm(m.sp0, sync_tok, B, yS, m.sync_dim, (long long)yS * m.sync_dim, EPI_STORE, ACT_SILU, a1, 1, H);
        gemm(m.sp13, a1, B, yS, H, (long long)yS * H, EPI_SWIGLU, ACT_NONE, hbuf, 1, F, nullptr, 0, nullptr, 0, 1, 1);
        gemm(m.sp2, hbuf, B, yS, F, (long long)yS * F, EPI_STORE, ACT_NONE, sync_out, 0, H);
        inv = false;
        // ---- text (mmdit.cpp:178-183) ----
        tag = "pre.text";
        lane = 2;
        wait_input(IN_TEXT);
        inv = true;
        op([=](cudaStream_t st) {
            return text_prep(text_in, text_S, text_dim, t5_in, t5_S, t5_dim, B, text_tok, st);
        });
        gemm(m.tp0, text_tok, B, St, m.t5_dim, (long long)St * m.t5_dim, EPI_STORE, ACT_SILU, a1_l[2], 1, H);
        gemm(m.tp13, a1_l[2], B, St, H, (long long)St * H, EPI_SWIGLU, ACT_NONE, hb_l[2], 1, F, nullptr, 0, nullptr, 0, 1, 1);
        gemm(m.tp2, hb_l[2], B, St, F, (long long)St * F, EPI_STORE, ACT_NONE, x_text0, 0, H);
        snap("text_pp", x_text0, (long long)B * St * H);
        inv = false;
        copy(x_text, x_text0, (size_t)B * St * H * sizeof(float));
        lane = 0;
        mark(2);
        // ---- conditioning vectors (mmdit.cpp:184-200) ----
        tag = "pre.cond";
        wait_input(IN_GTEXT);
        inv = true;
        gemv(m.tcp, P.gtext_in, m.text_dim, B, ACT_NONE, text_fc, H);
        snap("text_fc", text_fc, (long long)B * H);
        op([=](cudaStream_t st) { return seq_mean(x_clip0, B, cS, H, cmean, st); });
        gemv(m.ccp, cmean, H, B, ACT_NONE, clip_fc, H);
        snap("clip_fc", clip_fc, (long long)B * H);
        op([=](cudaStream_t st) { return add_vec(clip_fc, text_fc, B * H, gsum, st); });
        gemv(m.gc13, gsum, H, B, ACT_NONE, gch, F);
        gemv(m.gc2, gch, F, B, ACT_NONE, gcm, H);
        snap("gcmlp", gcm, (long long)B * H);
        inv = false;
        op([=](cudaStream_t st) { return add_vec(gcm, te, B * H, gc, st); });
        inject_point("global_c", gc, (long long)B * H);
        op([=](cudaStream_t st) { return build_extended(sync_out, yS, gc, B, T, H, ext, sext, sgc, st); });
        // a teacher-forced ext also replaces the adaLN GEMM's operand bf16(silu(ext)) derived from it
        inject_point("extended_c", ext, (long long)B * T * H,
                     [=](cudaStream_t st) { return silu_cast_bf16(ext, (long long)B * T * H, sext, st); });
        // ---- every per-token adaLN of the step in one GEMM (mmdit.cpp:209, 285); on a side lane
        // beside it, every clip / text adaLN of the step in one GEMV ----
        tag = "adaln";
        const int R_ct = m.ada_ct.w ? m.ada_ct.M : 0;
        if (R_ct) {
            mark(1);
            lane = 1;
            gemv(m.ada_ct, sgc, H, B, ACT_NONE, mod_ct, R_ct);
            lane = 0;
        }
        gemm(m.ada_lat, sext, B, T, H, (long long)T * H, EPI_STORE, ACT_NONE, mod_lat, 0, H, nullptr, 0, nullptr, 0, 1, 0,
             8, H, BTH);
        if (R_ct) mark(2);
        (void)R;

        // ---- joint blocks (mmdit.cpp:237-272) ----
        // A stream's adaLN chunk k (shift, scale, gate_msa, shift_mlp, scale_mlp, gate_mlp) is at
        // mod + k * cs with row stride ld: latent rows per token (cs = BTH, ld = H), clip / text
        // one row per item (cs = H, ld = 6H or 2H).
        const int n_joint = (int)m.joint.size();
        float * xs[3] = {x_lat, x_clip, x_text};
        const int Ss[3] = {T, cS, St};
        const int soff[3] = {0, T, T + cS};
        float * modc[3] = {nullptr, mod_c, mod_t};
        // The three streams of a joint block are independent except at the attention: stream s
        // runs on lane s (its own CUDA stream in the captured graph), joined before the
        // attention and forked after it.
        mark(1);
        const char * const sname[3] = {"lat", "clip", "text"};
        for (int i = 0; i < n_joint; ++i) {
            const auto & blk = m.joint[i];
            for (int s = 0; s < 3; ++s)
                inject_point("blk" + std::to_string(i) + "_in_" + sname[s], xs[s], (long long)B * Ss[s] * H);
            const float * mods[3];
            long long lds[3], css[3];
            for (int s = 0; s < 3; ++s) {
                const StreamW & w = blk[s];
                const int S = Ss[s];
                lane = s;
                __nv_bfloat16 * const xn = xn_l[s];
                tag = "j" + std::to_string(i) + (s == 0 ? ".lat" : s == 1 ? ".clip" : ".text");
                if (s == 0) { mods[s] = mod_lat + (w.ada_off / H) * BTH; lds[s] = H; css[s] = BTH; }
                else if (R_ct) {   // this stream's rows of the stacked clip / text adaLN output
                    lds[s] = R_ct;
                    css[s] = H;
                    mods[s] = mod_ct + w.ada_ct_off;
                } else {
                    lds[s] = (long long)(w.pre_only ? 2 : 6) * H;
                    css[s] = H;
                    gemv(w.ada, sgc, H, B, ACT_NONE, modc[s], lds[s]);
                    mods[s] = modc[s];
                }
                const float * mod = mods[s];
                const long long ld = lds[s], cs = css[s];
                op([=](cudaStream_t st) { return ln_modulate(xs[s], B * S, H, mod, mod + cs, ld, s == 0, S, xn, st); });
                if (i == 0 && s == 2) snap("text_xn", xn, (long long)B * S * H, 1);
                gemm_qkv(w, hpm ? &m.hpar.joint_qkv[i][s] : nullptr, xn, B, S,
                         s == 0 ? rope_lat : s == 1 ? rope_clip : nullptr, Qb, Kb, Vb, Sj, soff[s]);
            }
            if (i == 0) {   // (head-parallel: this rank's heads)
                snap("a0_q", Qb, (long long)B * Sj * nhl * 64, 2, B, nhl, Sj);
                snap("a0_k", Kb, (long long)B * Sj * nhl * 64, 2, B, nhl, Sj);
                snap("a0_v", Vb, (long long)B * Sj * nhl * 64, 2, B, nhl, Sj);
            }
            lane = 0;
            mark(2);
            tag = "j" + std::to_string(i);
            __nv_bfloat16 * const aoj = attention(Qb, Kb, Vb, B, Sj, ao, err);
            if (rc) return;
            if (i == 0) snap("a0_out", aoj, (long long)B * Sj * H, 1);
            mark(1);
            for (int s = 0; s < 3; ++s) {
                const StreamW & w = blk[s];
                if (w.pre_only) continue;
                const int S = Ss[s];
                lane = s;
                __nv_bfloat16 * const xn = xn_l[s];
                __nv_bfloat16 * const hbuf = hb_l[s];
                tag = "j" + std::to_string(i) + (s == 0 ? ".lat" : s == 1 ? ".clip" : ".text");
                const float * mod = mods[s];
                const long long ld = lds[s], cs = css[s];
                const int gdiv = (s == 0) ? 1 : S;
                gemm(w.l1, aoj + (long long)soff[s] * H, B, S, H, (long long)Sj * H, EPI_GATE_RESID, ACT_NONE, nullptr, 0, 0,
                     xs[s], H, mod + 2 * cs, ld, gdiv);
                snap("blk" + std::to_string(i) + "_attn_" + sname[s], xs[s], (long long)B * S * H);
                inject_point("blk" + std::to_string(i) + "_mid_" + sname[s], xs[s], (long long)B * S * H);
                op([=](cudaStream_t st) { return ln_modulate(xs[s], B * S, H, mod + 3 * cs, mod + 4 * cs, ld, s == 0, S, xn, st); });
                gemm(w.w13, xn, B, S, H, (long long)S * H, EPI_SWIGLU, ACT_NONE, hbuf, 1, F, nullptr, 0, nullptr, 0, 1, 1);
                gemm(w.w2, hbuf, B, S, F, (long long)S * F, EPI_GATE_RESID, ACT_NONE, nullptr, 0, 0, xs[s], H, mod + 5 * cs,
                     ld, gdiv);
            }
            lane = 0;
            for (int s = 0; s < 3; ++s) snap("blk" + std::to_string(i) + "_" + sname[s], xs[s], (long long)B * Ss[s] * H);
            if (i == 0) {
                snap("jb0_lat", x_lat, (long long)B * T * H);
                snap("jb0_clip", x_clip, (long long)B * cS * H);
                snap("jb0_text", x_text, (long long)B * St * H);
            }
        }
        lane = 0;
        mark(2);
        snap("after_joint", x_lat, (long long)B * T * H);
        // ---- fused blocks (mmdit.cpp:274-282) ----
        int fi = 0;
        for (const StreamW & w : m.fused) {
            const int fidx = fi;
            tag = "f" + std::to_string(fi++);
            const float * mod = mod_lat + (w.ada_off / H) * BTH;
            const long long ld = H, cs = BTH;
            const std::string bi = "blk" + std::to_string(n_joint + fidx);
            inject_point(bi + "_in_lat", x_lat, (long long)B * T * H);
            op([=](cudaStream_t st) { return ln_modulate(x_lat, B * T, H, mod, mod + cs, ld, 1, T, xn, st); });
            gemm_qkv(w, hpm ? &m.hpar.fused_qkv[fidx] : nullptr, xn, B, T, rope_lat, Qb, Kb, Vb, T, 0);
            __nv_bfloat16 * const aof = attention(Qb, Kb, Vb, B, T, ao, err);
            if (rc) return;
            gemm(w.l1, aof, B, T, H, (long long)T * H, EPI_GATE_RESID, ACT_NONE, nullptr, 0, 0, x_lat, H, mod + 2 * cs, ld, 1);
            snap(bi + "_attn_lat", x_lat, (long long)B * T * H);
            inject_point(bi + "_mid_lat", x_lat, (long long)B * T * H);
            op([=](cudaStream_t st) { return ln_modulate(x_lat, B * T, H, mod + 3 * cs, mod + 4 * cs, ld, 1, T, xn, st); });
            gemm(w.w13, xn, B, T, H, (long long)T * H, EPI_SWIGLU, ACT_NONE, hbuf, 1, F, nullptr, 0, nullptr, 0, 1, 1);
            gemm(w.w2, hbuf, B, T, F, (long long)T * F, EPI_GATE_RESID, ACT_NONE, nullptr, 0, 0, x_lat, H, mod + 5 * cs, ld, 1);
            snap(bi + "_lat", x_lat, (long long)B * T * H);
        }
        snap("after_fused", x_lat, (long long)B * T * H);
        // ---- final layer (mmdit.cpp:284-290) ----
        tag = "final";
        inject_point("final_in_lat", x_lat, (long long)B * T * H);
        const float * fmod = mod_lat + (m.final_ada_off / H) * BTH;
        op([=](cudaStream_t st) { return ln_modulate(x_lat, B * T, H, fmod, fmod + BTH, H, 1, T, xn, st); });
        gemm(m.fconv, xn, B, T, H, (long long)T * H, EPI_STORE, ACT_NONE, P.flow, 0, L);
        snap("flow_cl", P.flow, (long long)B * T * L);
    }
};

void to_host_f32(const Snap & s, std::vector<float> & out) {
    out.resize((size_t)s.n);
    if (s.kind == 0) {
        cudaMemcpy(out.data(), s.ptr, (size_t)s.n * 4, cudaMemcpyDeviceToHost);
    } else if (s.kind == 1) {
        std::vector<uint16_t> h((size_t)s.n);
        cudaMemcpy(h.data(), s.ptr, (size_t)s.n * 2, cudaMemcpyDeviceToHost);
        for (long long i = 0; i < s.n; ++i) { uint32_t u = (uint32_t)h[i] << 16; memcpy(&out[i], &u, 4); }
    } else {
        std::vector<__half> h((size_t)s.n);
        cudaMemcpy(h.data(), s.ptr, (size_t)s.n * 2, cudaMemcpyDeviceToHost);
        const int H = s.nh * 64;
        for (int b = 0; b < s.B; ++b)
            for (int hh = 0; hh < s.nh; ++hh)
                for (int t = 0; t < s.S; ++t)
                    for (int d = 0; d < 64; ++d)
                        out[((size_t)b * s.S + t) * H + hh * 64 + d] =
                            __half2float(h[(((size_t)b * s.nh + hh) * s.S + t) * 64 + d]);
    }
}

}  // namespace

int plan_build(Model & m, const Shape & sh, std::unique_ptr<Plan> & out) {
    if (sh.B < 1 || sh.T < 1 || sh.clip_S < 1 || sh.sync_S < 8 || sh.sync_S % 8 || sh.text_S < 0 || sh.t5_S < 0 ||
        sh.text_S + sh.t5_S < 1)
        return TSD_ERR_ARG;
    TSD_CUDA_TRY(cudaSetDevice(m.device));
    std::unique_ptr<Plan> p(new Plan());
    p->sh = sh;
    Builder b{m, *p};
    b.build();
    if (b.rc) return b.rc;
    // overlapped input staging: the copy stream and the per-group events exist before the first
    // capture, so every captured graph holds the waits on them
    TSD_CUDA_TRY(cudaStreamCreateWithFlags(&p->copy_st, cudaStreamNonBlocking));
    for (cudaEvent_t & e : p->in_ev) TSD_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    TSD_CUDA_TRY(cudaEventCreateWithFlags(&p->prev_done, cudaEventDisableTiming));
    out = std::move(p);
    return TSD_OK;
}

// Op-by-op execution on one stream: the inputs of every group have landed first.
static cudaError_t wait_all_inputs(Plan & p, cudaStream_t st) {
    for (cudaEvent_t e : p.in_ev)
        if (e) {
            const cudaError_t r = cudaStreamWaitEvent(st, e, 0);
            if (r != cudaSuccess) return r;
        }
    return cudaSuccess;
}

int plan_profile(Model & m, Plan & p, cudaStream_t st, std::vector<float> & ms) {
    (void)m;
    TSD_CUDA_TRY(wait_all_inputs(p, st));
    std::vector<cudaEvent_t> ev(p.ops.size() + 1);
    for (auto & e : ev) TSD_CUDA_TRY(cudaEventCreate(&e));
    int rc = TSD_OK;
    cudaError_t ce = cudaEventRecord(ev[0], st);
    for (size_t i = 0; i < p.ops.size() && ce == cudaSuccess; ++i) {
        if (p.ops[i].fn) ce = p.ops[i].fn(st);     // lane markers have no work
        if (ce == cudaSuccess) ce = cudaEventRecord(ev[i + 1], st);
    }
    if (ce == cudaSuccess) ce = cudaEventSynchronize(ev.back());
    ms.assign(p.ops.size(), 0.f);
    if (ce == cudaSuccess)
        for (size_t i = 0; i < p.ops.size(); ++i) cudaEventElapsedTime(&ms[i], ev[i], ev[i + 1]);
    else {
        fprintf(stderr, "tsd: profile: %s\n", cudaGetErrorString(ce));
        rc = TSD_ERR_CUDA;
    }
    for (auto & e : ev) cudaEventDestroy(e);
    return rc;
}

int plan_run(Model & m, Plan & p, cudaStream_t st, tsd_dbg_fn dbg, void * ud, bool reuse_cond, tsd_inject_fn inject) {
    (void)m;
    if (dbg || inject) {
        TSD_CUDA_TRY(wait_all_inputs(p, st));
        std::vector<float> h;
        for (const Op & o : p.ops) {
            if (o.fn) TSD_CUDA_TRY(o.fn(st));
            if (!o.snaps.empty()) {
                TSD_CUDA_TRY(cudaStreamSynchronize(st));
                for (const Snap & s : o.snaps) {
                    if (!dbg && !s.inject) continue;
                    to_host_f32(s, h);
                    if (dbg) dbg(ud, s.name.c_str(), h.data(), (int64_t)h.size());
                    if (s.inject && inject && s.kind == 0 && inject(ud, s.name.c_str(), h.data(), (int64_t)h.size())) {
                        // on the plan's stream and waited for: a synchronous copy from pageable memory may
                        // return before its DMA lands and is not ordered against a non-blocking stream
                        TSD_CUDA_TRY(cudaMemcpyAsync(const_cast<void *>(s.ptr), h.data(), (size_t)s.n * 4,
                                                     cudaMemcpyHostToDevice, st));
                        if (s.after_inject) TSD_CUDA_TRY(s.after_inject(st));
                        TSD_CUDA_TRY(cudaStreamSynchronize(st));
                    }
                }
            }
        }
        return TSD_OK;
    }
    const int gi = reuse_cond ? 1 : 0;
    if (!p.graph[gi] || p.graph_stream[gi] != st) {
        if (p.graph[gi]) { cudaGraphExecDestroy(p.graph[gi]); p.graph[gi] = nullptr; }
        cudaStreamCaptureStatus cs;
        TSD_CUDA_TRY(cudaStreamIsCapturing(st, &cs));
        const bool can_capture = (st != nullptr) && cs == cudaStreamCaptureStatusNone;
        if (!can_capture) {
            TSD_CUDA_TRY(wait_all_inputs(p, st));
            for (const Op & o : p.ops)
                if (o.fn && !(reuse_cond && o.invariant)) TSD_CUDA_TRY(o.fn(st));
            return TSD_OK;
        }
        // side lanes and one event per fork / two per join, created once per plan
        size_t need_ev = 0;
        for (const Op & o : p.ops) need_ev += o.sync == 1 ? 1 : o.sync == 2 ? kSideLanes : 0;
        for (int l = 0; l < kSideLanes; ++l)
            if (!p.side[l]) TSD_CUDA_TRY(cudaStreamCreateWithFlags(&p.side[l], cudaStreamNonBlocking));
        while (p.events.size() < need_ev) {
            cudaEvent_t ev;
            TSD_CUDA_TRY(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
            p.events.push_back(ev);
        }
        cudaGraph_t g;
        TSD_CUDA_TRY(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
        cudaError_t e = cudaSuccess;
        size_t ev = 0;
        for (const Op & o : p.ops) {
            if (o.sync == 1) {            // fork: side lanes continue after lane 0's work so far
                e = cudaEventRecord(p.events[ev], st);
                for (int l = 0; e == cudaSuccess && l < kSideLanes; ++l) e = cudaStreamWaitEvent(p.side[l], p.events[ev], 0);
                ++ev;
            } else if (o.sync == 2) {     // join: lane 0 continues after the side lanes' work
                for (int l = 0; e == cudaSuccess && l < kSideLanes; ++l) {
                    e = cudaEventRecord(p.events[ev + l], p.side[l]);
                    if (e == cudaSuccess) e = cudaStreamWaitEvent(st, p.events[ev + l], 0);
                }
                ev += kSideLanes;
            } else if (o.sync == 3) {     // input group: an external wait on its copy event
                if (p.in_ev[o.input])
                    e = cudaStreamWaitEvent(o.lane == 0 ? st : p.side[o.lane - 1], p.in_ev[o.input],
                                            cudaEventWaitExternal);
            } else if (!(reuse_cond && o.invariant)) {
                e = o.fn(o.lane == 0 ? st : p.side[o.lane - 1]);
            }
            if (e != cudaSuccess) break;
        }
        cudaError_t e2 = cudaStreamEndCapture(st, &g);
        if (e != cudaSuccess || e2 != cudaSuccess) {
            if (e2 == cudaSuccess) cudaGraphDestroy(g);
            fprintf(stderr, "tsd: graph capture failed: %s\n", cudaGetErrorString(e != cudaSuccess ? e : e2));
            return TSD_ERR_CUDA;
        }
        e = cudaGraphInstantiate(&p.graph[gi], g, 0);
        cudaGraphDestroy(g);
        TSD_CUDA_TRY(e);
        p.graph_stream[gi] = st;
    }
    TSD_CUDA_TRY(cudaGraphLaunch(p.graph[gi], st));
    return TSD_OK;
}

}  // namespace tsd
