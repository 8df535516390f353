// gemm_tc.cu — persistent tcgen05 / TMEM / TMA GEMM for the MM-DiT projections (sm_100a).
//
// Replaces the reference's ggml_mul_mat (src/mmdit.cpp:12-16 `lin`) and the im2col+mul_mat
// convolution (`conv1d_f32`, :20-25): a conv with k taps is an implicit GEMM whose K loop runs
// over (tap, input-feature block) and whose activation tile for tap k is the token window
// shifted by k - pad (TMA zero-fills rows outside the batch item, which is the conv padding).
// The adaLN gate + residual add (:231, :234) and SwiGLU (:42-43, :50-51) are fused into the
// epilogue, so no separate elementwise kernel touches HBM for them.
//
// Persistent CTAs (at most one per SM) walk output tiles of 128 weight rows x BN tokens (x a K
// split), m-block-major so CTAs running at the same time share weight tiles through L2. Warps 0
// and 7 issue the weight tiles and warp 6 the token tiles into a ring of 3-8 stages (one TMA box
// of one or two K blocks per operand per stage), warp 1 owns TMEM and issues tcgen05.mma into one
// of two 256-column accumulators, warps 2-5 drain the other accumulator (thread = output
// feature) while the next tile accumulates. A second instance of each kernel runs CTA pairs
// (cta_group::2, 256 weight rows per pair, each CTA loading half of the token tile). SwiGLU
// weight rows alternate w1 / w3 of one feature, so h1 and h3 of a feature sit in neighbouring
// TMEM lanes (= neighbouring threads) and the epilogue pairs them with one register exchange.
// Launched with programmatic dependent launch: weight tiles of the first stages are requested
// before the kernel waits for the activations its predecessor writes.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <vector>
#include <cstdio>
#include <cstdlib>

namespace tsd {

namespace {

constexpr int kMaxStages = 8;              // operand ring depth: as many stages as fit the area
constexpr int kStageArea = 4 * (128 * 128 + 256 * 128);   // 192 KB: 4 stages at BN = 256
constexpr int kABytes = 128 * 128;          // 128 rows x 64 bf16
constexpr int kTmemCols = 512;              // two 256-column fp32 accumulators
constexpr int kQ8Bytes = 9216;             // Q8_0 A path, per stage: int8 tile 128 x 64 + scales 2 x 128 f16 (padded)
constexpr int kThreads = 256;              // warps: 0 TMA, 1 MMA, 2-5 epilogue, 6-7 Q8_0 converters
constexpr int kEBufBytes = 16384;          // epilogue staging buffer (x2): 32 tokens x 128 f32
constexpr int kSmemBytes = kStageArea + 2 * kEBufBytes + 1024 /*align*/ + 256 /*barriers*/;

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// Token columns the epilogue finishes at a time: the tile, or one item of a multi-item tile.
__device__ __forceinline__ int epi_bn(const GemmParams & p) { return p.ipt > 1 ? p.bni : p.BN; }

struct TileCoord { int mb, b, t0, kb_begin, kb_end, split, otile; };

// Tile t -> (m-block, batch item, first token, K range). Consecutive t share the m-block.
// CTA pairs walk pair tiles: tile t covers m-blocks 2 * (t / per_mb) + {0, 1}, `prank` picks
// this CTA's.
__device__ __forceinline__ TileCoord decode(const GemmParams & p, int t, int nkb, int prank = 0) {
    TileCoord c;
    int nt;
    if (p.order == 0) {           // m-block-major: consecutive tiles share the weight tile
        const int per_mb = p.groups * p.n_tiles * p.splits;
        c.mb = t / per_mb;
        const int rem = t - c.mb * per_mb;
        if (p.pair) c.mb = 2 * c.mb + prank;
        nt = rem / p.splits;
        c.split = rem - nt * p.splits;
    } else {                      // token-tile-major: consecutive tiles share the activation tile
        c.mb = t % p.mblocks;
        const int r = t / p.mblocks;
        const int ntt = p.groups * p.n_tiles;
        nt = r % ntt;
        c.split = r / ntt;
    }
    const int g = nt / p.n_tiles;                     // batch group (one item unless ipt > 1)
    c.b = g * p.ipt;                                  // first item of the tile
    c.t0 = (nt - g * p.n_tiles) * p.BN;               // (0 in a multi-item tile: n_tiles = 1)
    c.otile = c.mb * (p.groups * p.n_tiles) + nt;     // output tile (all K splits of it)
    c.kb_begin = (int)((long long)nkb * c.split / p.splits);
    c.kb_end = (int)((long long)nkb * (c.split + 1) / p.splits);
    return c;
}

// Epilogue kinds, fixed at compile time so that each kernel instance holds only its own
// straight-line epilogue (with every variant in one body, the skipped branches of a 32-way
// unrolled loop made the executed path a sparse walk through tens of KB of code and the
// epilogue warps stalled on instruction fetch).
enum EpiKind : int { EK_F32 = 0, EK_BF16, EK_F32_SILU, EK_BF16_SILU, EK_SWIGLU_F32, EK_SWIGLU_BF16, EK_GATE, EK_QKV, EK_COUNT };
template <int EK> struct Epi {
    static constexpr bool gate = EK == EK_GATE;
    static constexpr bool qkv = EK == EK_QKV;
    static constexpr bool swiglu = EK == EK_SWIGLU_F32 || EK == EK_SWIGLU_BF16;
    static constexpr bool bf16 = EK == EK_BF16 || EK == EK_BF16_SILU || EK == EK_SWIGLU_BF16;
    static constexpr bool silu = EK == EK_F32_SILU || EK == EK_BF16_SILU;
};

// SiLU in the epilogue: the fast form where the result is rounded to bf16, exact f32 otherwise.
template <bool BF16> __device__ __forceinline__ float silu_out(float x) { return BF16 ? silu_fast(x) : silu_f(x); }

template <bool BF16> __device__ __forceinline__ void put(void * out, long long i, float v) {
    if (BF16) reinterpret_cast<__nv_bfloat16 *>(out)[i] = __float2bfloat16_rn(v);
    else reinterpret_cast<float *>(out)[i] = v;
}

struct EpiCtx {
    int m;               // output feature of this thread
    bool m_ok;           // m is stored by this thread
    float bias;
    int ncols;           // valid token columns of the tile
    long long row_base;  // output row of the tile's first token
    long long col;       // output column offset of feature m (after column blocking)
};

// STORE: thread = feature e.m, 32 token columns j0.. of it; every warp store writes 32
// consecutive features of one output row.
template <int EK>
__device__ __forceinline__ void emit_store(const GemmParams & p, const EpiCtx & e, int j0, const uint32_t (&v)[32]) {
    if (!e.m_ok) return;
    const int ncols = e.ncols - j0;
    const long long base = (e.row_base + j0) * p.ldo + e.col;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        float val = __uint_as_float(v[j]) + e.bias;
        if (Epi<EK>::silu) val = silu_out<Epi<EK>::bf16>(val);
        if (j < ncols) put<Epi<EK>::bf16>(p.out, base + (long long)j * p.ldo, val);
    }
}

// SWIGLU: tile rows alternate w1 / w3 of one feature, so lanes 2i and 2i+1 hold h1 and h3 of
// feature e.m. One exchange gives the even lane h3 of columns 0-15 and the odd lane h1 of
// columns 16-31; each lane then finishes 16 of the 32 columns.
template <int EK>
__device__ __forceinline__ void emit_swiglu(const GemmParams & p, const EpiCtx & e, int j0, const uint32_t (&w)[32],
                                            int lane) {
    const bool odd = lane & 1;
    float o[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const float lo = __uint_as_float(w[j]), hi = __uint_as_float(w[j + 16]);
        const float r = __shfl_xor_sync(0xffffffffu, odd ? lo : hi, 1);
        const float h1 = odd ? r : lo, h3 = odd ? hi : r;
        o[j] = silu_out<Epi<EK>::bf16>(h1) * h3;
    }
    if (!e.m_ok) return;
    const int c0 = j0 + (odd ? 16 : 0);
    const int ncols = e.ncols - c0;
    const long long base = (e.row_base + c0) * p.ldo + e.col;
#pragma unroll
    for (int j = 0; j < 16; ++j)
        if (j < ncols) put<Epi<EK>::bf16>(p.out, base + (long long)j * p.ldo, o[j]);
}

// TMA epilogue, STORE / SWIGLU: write one 32-token chunk into the staging buffer, laid out as
// the output box [token][feature] (128 features; SwiGLU 64), f32 or bf16.
template <int EK>
__device__ __forceinline__ void stage_chunk(const EpiCtx & e, const uint32_t (&v)[32], int ml, int lane, uint8_t * sbuf) {
    if (Epi<EK>::swiglu) {
        const bool odd = lane & 1;
        const int f = ml >> 1;                       // output feature within the tile
        const int r0 = odd ? 16 : 0;                 // tokens of this lane
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const float lo = __uint_as_float(v[j]), hi = __uint_as_float(v[j + 16]);
            const float r = __shfl_xor_sync(0xffffffffu, odd ? lo : hi, 1);
            const float h1 = odd ? r : lo, h3 = odd ? hi : r;
            const float o = silu_out<Epi<EK>::bf16>(h1) * h3;
            if (Epi<EK>::bf16) reinterpret_cast<__nv_bfloat16 *>(sbuf)[(r0 + j) * 64 + f] = __float2bfloat16_rn(o);
            else reinterpret_cast<float *>(sbuf)[(r0 + j) * 64 + f] = o;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            float val = __uint_as_float(v[j]) + e.bias;
            if (Epi<EK>::silu) val = silu_out<Epi<EK>::bf16>(val);
            if (Epi<EK>::bf16) reinterpret_cast<__nv_bfloat16 *>(sbuf)[j * 128 + ml] = __float2bfloat16_rn(val);
            else reinterpret_cast<float *>(sbuf)[j * 128 + ml] = val;
        }
    }
}

// One 32-token chunk through the staging buffer: wait until the store that last read the
// buffer is done, fill it, hand it to the TMA (thread 64 issues the stores: rows 0-15 and, if
// inside the tile, rows 16-31).
template <int EK>
__device__ __forceinline__ void tma_chunk(const GemmParams & p, const CUtensorMap * tmO, const EpiCtx & e, int j0,
                                          const uint32_t (&v)[32], int ml, int lane, uint8_t * ebuf, int & gc,
                                          int c0o, int cb, int b, int t0) {
    uint8_t * sbuf = ebuf + (gc & 1) * kEBufBytes;
    if (gc >= 2 && threadIdx.x == 64) bulk_wait_read<1>();
    epi_bar();
    stage_chunk<EK>(e, v, ml, lane, sbuf);
    fence_proxy_async_smem();
    epi_bar();
    if (threadIdx.x == 64) {
        constexpr int rowb = (Epi<EK>::swiglu ? 64 : 128) * (Epi<EK>::bf16 ? 2 : 4);
        tma_store_4d(tmO, sbuf, c0o, t0 + j0, b, cb);
        if (j0 + 16 < epi_bn(p)) tma_store_4d(tmO, sbuf + 16 * rowb, c0o, t0 + j0 + 16, b, cb);
        bulk_commit();
    }
    ++gc;
}

// TMA epilogue, GATE_RESID: request the residual (and per-token gate) tile of 16 tokens into
// staging buffer g & 1 (residual [16][128] f32, gate behind it). Thread 64 only.
// Gate + residual epilogue, 16 tokens a step, through staging buffer g & 1 =
// [increments 16 x 128 f32 | per-token gate 16 x 128 f32]. The residual is never loaded: the
// increments gate * (acc + bias) go out by a TMA reduce-add into the residual (each element gets
// exactly one f32 add, so the result equals x + increment computed in registers). Thread 64
// loads the gate tiles (two steps ahead), thread 96 issues the reduce-adds: a TMA instruction
// costs its issuing thread ~300 cycles, so the two streams run on threads of different warps.
__device__ __forceinline__ void gate_issue(const CUtensorMap * tmG, uint64_t * ebar, uint8_t * ebuf, int g, int m0, int t,
                                           int b) {
    uint64_t * bar = &ebar[g & 1];
    mbar_arrive_expect_tx(bar, 8192u);
    tma_load_4d(ebuf + (g & 1) * kEBufBytes + 8192, tmG, bar, m0, t, b, 0);
}
// One step: this thread's feature of 16 tokens (v = accumulator sums, gv = per-item gate when the
// gate is not per token). t = the step's first token; t2 = the token of the step two ahead, or
// -1. Returns false if the gate tile did not arrive in time.
__device__ __forceinline__ bool gate_step(const GemmParams & p, const EpiCtx & e, const CUtensorMap * tmO,
                                          const CUtensorMap * tmG, bool gtile, uint64_t * ebar, uint8_t * ebuf, int gs,
                                          int & gl, const float (&v)[16], const float (&gv)[16], int ml, int m0, int t,
                                          int t2, int b) {
    float * dbuf = reinterpret_cast<float *>(ebuf + (gs & 1) * kEBufBytes);
    const float * gr = dbuf + 16 * 128;
    if (gtile && !__all_sync(0xffffffffu, mbar_wait(&ebar[gs & 1], (gs >> 1) & 1, nullptr, p.err, DEV_TIMEOUT_ACC)))
        return false;
#pragma unroll
    for (int j = 0; j < 16; ++j) dbuf[j * 128 + ml] = (gtile ? gr[j * 128 + ml] : gv[j]) * (v[j] + e.bias);
    fence_proxy_async_smem();
    if (threadIdx.x == 96) bulk_wait_read<0>();     // the previous reduce has read the buffer written next step
    epi_bar();
    if (threadIdx.x == 96) {
        tma_reduce_add_4d(tmO, dbuf, m0, t, b, 0);
        bulk_commit();
    }
    if (threadIdx.x == 64 && gtile && t2 >= 0) {
        gate_issue(tmG, ebar, ebuf, gl, m0, t2, b);
        ++gl;
    }
    return true;
}

// QKV: RMSNorm over each head's 64 features (Q, K), RoPE on feature pairs (2i, 2i+1), fp16
// into the head-major joint Q / K / V. Thread = feature; a head spans this warp and warp q ^ 1.
// For 32 token columns the per-token sums of squares are reduced across the warp's lanes by a
// transposing butterfly (lane j ends with token j's sum, 31 shuffles), exchanged with the
// partner warp through shared memory (`red`, two buffers used alternately by the chunks that
// take the barrier: `nqk` counts those, so two uses of a buffer always have a barrier between
// them), and broadcast.
// The float operations follow qk_norm_rope_kernel: (x * rstd) * g, then x0 cos - x1 sin,
// x0 sin + x1 cos.
// (cos, sin) of pair d / 2 for the 32 token columns from j0 of the tile (RoPE table rows).
__device__ __forceinline__ void rope_load(const GemmParams & p, const EpiCtx & e, const TileCoord & c, int j0, int d,
                                          float2 (&cs)[32]) {
    const float2 * r = p.rope + (long long)(c.t0 + j0) * 32 + (d >> 1);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        cs[j] = make_float2(1.f, 0.f);
        if (j0 + j < e.ncols) cs[j] = __ldg(r + j * 32);
    }
}

// TMA_ONLY: the caller's kernel form always has the TMA epilogue maps (p.epi_tma).
template <bool TMA_ONLY>
__device__ __forceinline__ void emit_qkv(const GemmParams & p, const EpiCtx & e, const TileCoord & c, int j0,
                                         const uint32_t (&w)[32], int ml, int lane, int q, uint8_t * ebuf, int & nqk,
                                         int & gs, const CUtensorMap * tmQ, const CUtensorMap * tmK,
                                         const CUtensorMap * tmV, float2 (&cs)[32]) {
    // reduction exchange in the upper half of staging buffer 0 (staging uses the lower 8 KB)
    float * red = reinterpret_cast<float *>(ebuf + 8192);
    const int f0 = c.mb * 128;
    const int which = f0 / p.hidden;                    // 0 Q, 1 K, 2 V
    const int cf = f0 - which * p.hidden + ml;          // head * 64 + d
    const int h = cf >> 6, d = cf & 63;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(w[j]) + e.bias;
    if (which < 2) {
        float a[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) a[j] = v[j] * v[j];
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
            const bool up = lane & off;
#pragma unroll
            for (int i = 0; i < off; ++i) {
                const float send = up ? a[i] : a[i + off];
                const float keep = up ? a[i + off] : a[i];
                a[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
            }
        }
        float * rr = red + (nqk++ & 1) * 128;           // [warp quadrant][token]
        rr[q * 32 + lane] = a[0];
        epi_bar();
        const float tot = rr[q * 32 + lane] + rr[(q ^ 1) * 32 + lane];
        float * rsd = red + 256 + q * 32;               // this warp's rstd per token (warp-private)
        rsd[lane] = 1.0f / sqrtf(tot / 64.0f + 1e-6f);  // rstd of token `lane`
        __syncwarp();
        const float g = (which == 0 ? p.qg : p.kg)[d];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = (v[j] * rsd[j]) * g;
        __syncwarp();                                   // rsd is rewritten by the next chunk
        if (p.rope) {
            // cs holds this chunk's (cos, sin), loaded during the previous chunk (or before the
            // accumulator was ready); the next chunk's are requested right after use
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float o = __shfl_xor_sync(0xffffffffu, v[j], 1);
                v[j] = (d & 1) ? o * cs[j].y + v[j] * cs[j].x : v[j] * cs[j].x - o * cs[j].y;
            }
            if (j0 + 32 < epi_bn(p)) rope_load(p, e, c, j0 + 32, d, cs);
        }
    }
    if (TMA_ONLY || p.epi_tma) {
        // this warp pair's head: [32 tokens][64] fp16 in the staging buffer, then two 16-token
        // TMA boxes per head (the second only inside the tile); tokens past the stream's length
        // are clipped. The four boxes are issued by lane 0 of the four epilogue warps (a TMA
        // instruction costs its issuing thread ~300 cycles), each committing one group per chunk;
        // each issuer waits for its own stores of two chunks ago before the buffer is rewritten.
        uint8_t * sbuf = ebuf + (gs & 1) * kEBufBytes;
        if (gs >= 2 && lane == 0) bulk_wait_read<1>();
        epi_bar();
        __half * hb = reinterpret_cast<__half *>(sbuf + (ml >> 6) * 4096);
#pragma unroll
        for (int j = 0; j < 32; ++j) hb[j * 64 + d] = __float2half_rn(v[j]);
        fence_proxy_async_smem();
        epi_bar();
        if (lane == 0) {
            const CUtensorMap * tm = which == 0 ? tmQ : which == 1 ? tmK : tmV;
            const int h0 = (f0 - which * p.hidden) >> 6;
            const int hh = q >> 1, half = q & 1;       // this warp's box: head hh, tokens half * 16 ..
            if (half == 0 || j0 + 16 < epi_bn(p))
                tma_store_4d(tm, sbuf + hh * 4096 + half * 2048, 0, c.t0 + j0 + half * 16, h0 + hh, c.b);
            bulk_commit();
        }
        ++gs;
        return;
    }
    __half * dst = which == 0 ? p.q_out : which == 1 ? p.k_out : p.v_out;
    long long row = e.row_base + j0;
    int b = (int)(row / p.s_item), t = (int)(row - (long long)b * p.s_item);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        // h >= nh: a padding head of a head-parallel slice (zero weight rows), not stored
        if (j0 + j < e.ncols && h < p.nh) dst[(((long long)b * p.nh + h) * p.Sj + p.s_off + t) * 64 + d] = __float2half_rn(v[j]);
        if (++t == p.s_item) { t = 0; ++b; }
    }
}

// GATE_RESID loads: gate and residual of 16 token columns of feature e.m. `g` / `gpos` walk the
// gate rows (gate row = output row / gate_div) column by column.
struct GateCursor {
    const float * g;
    int gpos;
};
__device__ __forceinline__ void gate_load16(const GemmParams & p, const EpiCtx & e, int c0, GateCursor & gc,
                                            float (&gv)[16], float (&xv)[16]) {
    const float * x = p.resid + (e.row_base + c0) * p.ldr + e.m;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        gv[j] = 0.f; xv[j] = 0.f;
        if (e.m_ok && c0 + j < e.ncols) { gv[j] = __ldg(gc.g); xv[j] = x[(long long)j * p.ldr]; }
        if (++gc.gpos == p.gate_div) { gc.gpos = 0; gc.g += p.ldg; }
    }
}
__device__ __forceinline__ void gate_store16(const GemmParams & p, const EpiCtx & e, int c0, const uint32_t (&v)[16],
                                             const float (&gv)[16], const float (&xv)[16]) {
    if (!e.m_ok) return;
    float * x = p.resid + (e.row_base + c0) * p.ldr + e.m;
#pragma unroll
    for (int j = 0; j < 16; ++j)
        if (c0 + j < e.ncols) x[(long long)j * p.ldr] = xv[j] + gv[j] * (__uint_as_float(v[j]) + e.bias);
}

// Split-K reduction + epilogue of one output tile by the CTA that completed it last.
// Partials are [split][BN][128] floats. Warp w of the 4 epilogue warps takes rows j = w, w+4,
// ...; lane l owns tile rows 4l..4l+3, so every access is a coalesced 512-byte row and the
// loads of all splits are in flight together. Sum order is split 0, 1, 2, ... Outputs go out
// as vectors when p.vec says the buffers allow it and every value of the vector is stored.
template <int EK>
__device__ __forceinline__ void store_one(const GemmParams & p, long long row, int m, float a, float bias) {
    if (Epi<EK>::gate) {
        float * dst = p.resid + row * p.ldr + m;
        *dst += p.gate[(row / p.gate_div) * p.ldg + m] * (a + bias);
        return;
    }
    float v = a + bias;
    if (Epi<EK>::silu) v = silu_out<Epi<EK>::bf16>(v);
    const long long col = p.out_cblk ? (long long)(m / p.out_cblk) * p.out_cstride + m % p.out_cblk : m;
    put<Epi<EK>::bf16>(p.out, row * p.ldo + col, v);
}

template <int EK>
__device__ __forceinline__ void finish_row(const GemmParams & p, long long row, int mo, bool vec, const float4 & a4,
                                           const float (&bias)[4], const float4 & g, const float4 & x0) {
    const float a[4] = {a4.x, a4.y, a4.z, a4.w};
    const long long col = p.out_cblk ? (long long)(mo / p.out_cblk) * p.out_cstride + mo % p.out_cblk : mo;
    if (Epi<EK>::swiglu) {
        const float o0 = silu_out<Epi<EK>::bf16>(a[0]) * a[1], o1 = silu_out<Epi<EK>::bf16>(a[2]) * a[3];
        if (vec) {
            if (Epi<EK>::bf16)
                *reinterpret_cast<__nv_bfloat162 *>(reinterpret_cast<__nv_bfloat16 *>(p.out) + row * p.ldo + col) =
                    __floats2bfloat162_rn(o0, o1);
            else
                *reinterpret_cast<float2 *>(reinterpret_cast<float *>(p.out) + row * p.ldo + col) = make_float2(o0, o1);
        } else {
            store_one<EK>(p, row, mo, o0, 0.f);
            if (mo + 1 < p.m_valid) store_one<EK>(p, row, mo + 1, o1, 0.f);
        }
    } else if (!vec) {
#pragma unroll
        for (int e = 0; e < 4; ++e) if (mo + e < p.m_valid) store_one<EK>(p, row, mo + e, a[e], bias[e]);
    } else if (Epi<EK>::gate) {
        float4 x = x0;
        x.x += g.x * (a[0] + bias[0]); x.y += g.y * (a[1] + bias[1]);
        x.z += g.z * (a[2] + bias[2]); x.w += g.w * (a[3] + bias[3]);
        *reinterpret_cast<float4 *>(p.resid + row * p.ldr + mo) = x;
    } else {
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) { v[e] = a[e] + bias[e]; if (Epi<EK>::silu) v[e] = silu_out<Epi<EK>::bf16>(v[e]); }
        if (Epi<EK>::bf16) {
            __nv_bfloat162 * o = reinterpret_cast<__nv_bfloat162 *>(reinterpret_cast<__nv_bfloat16 *>(p.out) + row * p.ldo + col);
            o[0] = __floats2bfloat162_rn(v[0], v[1]);
            o[1] = __floats2bfloat162_rn(v[2], v[3]);
        } else {
            *reinterpret_cast<float4 *>(reinterpret_cast<float *>(p.out) + row * p.ldo + col) = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
}

// Rows are taken 4 per warp at a time (j = j0 + 4r): their gate / residual loads and then,
// split by split, their partial loads are all in flight together, so a group costs about one
// memory round trip per split instead of one per row.
template <int EK>
__device__ __forceinline__ void reduce_tile(const GemmParams & p, const TileCoord & c, int ew, int lane) {
    constexpr int R = 4;
    const int ncols = min(p.BN, p.S - c.t0);
    const size_t sstride = (size_t)p.BN * 128;                  // floats per split
    const float * base = p.ws + (size_t)c.otile * p.splits * sstride + lane * 4;
    // first output feature of this lane: SwiGLU rows (h1, h3, h1, h3) are features 2l, 2l + 1
    const int nf = Epi<EK>::swiglu ? 2 : 4;
    const int mo = Epi<EK>::swiglu ? c.mb * 64 + lane * 2 : c.mb * 128 + lane * 4;
    if (mo >= p.m_valid) return;                                // no stored feature (no collectives below)
    const bool vec = p.vec && mo + nf - 1 < p.m_valid;
    float bias[4] = {0.f, 0.f, 0.f, 0.f};
    if (!Epi<EK>::swiglu && p.bias) {
#pragma unroll
        for (int e = 0; e < 4; ++e) if (mo + e < p.m_valid) bias[e] = p.bias[mo + e];
    }
    const long long row0 = (long long)c.b * p.S + c.t0;
    for (int j0 = ew; j0 < ncols; j0 += 4 * R) {
        float4 acc[R], g[R], x[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
            g[r] = acc[r]; x[r] = acc[r];
            const int j = j0 + 4 * r;
            if (Epi<EK>::gate && vec && j < ncols) {
                g[r] = __ldg(reinterpret_cast<const float4 *>(p.gate + ((row0 + j) / p.gate_div) * p.ldg + mo));
                x[r] = *reinterpret_cast<const float4 *>(p.resid + (row0 + j) * p.ldr + mo);
            }
        }
        for (int s = 0; s < p.splits; ++s) {
            float4 part[R];
#pragma unroll
            for (int r = 0; r < R; ++r)
                if (j0 + 4 * r < ncols)
                    part[r] = __ldcg(reinterpret_cast<const float4 *>(base + s * sstride + (size_t)(j0 + 4 * r) * 128));
#pragma unroll
            for (int r = 0; r < R; ++r)
                if (j0 + 4 * r < ncols) {
                    acc[r].x += part[r].x; acc[r].y += part[r].y; acc[r].z += part[r].z; acc[r].w += part[r].w;
                }
        }
#pragma unroll
        for (int r = 0; r < R; ++r)
            if (j0 + 4 * r < ncols) finish_row<EK>(p, row0 + j0 + 4 * r, mo, vec, acc[r], bias, g[r], x[r]);
    }
}

// Split-K inside a cluster (one CTA per split, cluster rank = split). The tile's rows are cut
// into per-rank slices of whole 16-row blocks; rank r finishes rows [lo(r), hi(r)).
__device__ __forceinline__ int slice_lo(int r, int BN, int splits) { return 16 * (r * (BN >> 4) / splits); }
__device__ __forceinline__ int slice_rows_max(int BN, int splits) { return 16 * (((BN >> 4) + splits - 1) / splits); }

// This CTA's slice, 16 rows at a time: sum the ranks' partials in rank order (own rows from
// `part`, the others from the receive slots the peers filled), apply the epilogue and write the
// 16 rows out (TMA store from a staging buffer, or plain stores). Thread = tile row ml.
template <int EK>
__device__ __forceinline__ void finish_slice(const GemmParams & p, const CUtensorMap * tmO, const CUtensorMap * tmG,
                                             const TileCoord & c, const EpiCtx & e, const float * part,
                                             const float * recv, int rows_max, int rank, int lo, int hi, int ml,
                                             int lane, uint8_t * ebuf, uint64_t * ebar, int & gs, int & gl) {
    const bool tma = p.epi_tma;
    const int m0 = Epi<EK>::swiglu ? c.mb * 64 : c.mb * 128;
    const int cb = p.out_cblk ? m0 / p.out_cblk : 0;
    const int c0o = m0 - cb * p.out_cblk;
    const int nsteps = (hi - lo) >> 4;
    if (Epi<EK>::gate) {
        GateCursor gcur{nullptr, 0};
        const long long rr = e.row_base + lo;
        const long long grow = rr / p.gate_div;
        gcur.g = p.gate + grow * p.ldg + e.m;
        gcur.gpos = (int)(rr - grow * p.gate_div);
        const bool gtile = p.gate_div == 1;
        if (tma) {
            // gate tiles by TMA two steps ahead, residual updates by TMA reduce-add (gate_step)
            if (threadIdx.x == 64 && gtile)
                for (int k = 0; k < 2 && k < nsteps; ++k, ++gl) gate_issue(tmG, ebar, ebuf, gl, m0, c.t0 + lo + 16 * k, c.b);
            for (int k = 0; k < nsteps; ++k, ++gs) {
                const int r0 = lo + 16 * k;
                float gv[16];
                if (!gtile) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        gv[j] = 0.f;
                        if (e.m_ok && r0 + j < e.ncols) gv[j] = __ldg(gcur.g);
                        if (++gcur.gpos == p.gate_div) { gcur.gpos = 0; gcur.g += p.ldg; }
                    }
                }
                float acc[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[j] = 0.f;
                for (int sp = 0; sp < p.splits; ++sp) {
                    const float * src = sp == rank ? part + (size_t)r0 * 128
                                                   : recv + ((size_t)(sp < rank ? sp : sp - 1) * rows_max + (r0 - lo)) * 128;
#pragma unroll
                    for (int j = 0; j < 16; ++j) acc[j] += src[j * 128 + ml];
                }
                if (!gate_step(p, e, tmO, tmG, gtile, ebar, ebuf, gs, gl, acc, gv, ml, m0, c.t0 + r0,
                               k + 2 < nsteps ? c.t0 + r0 + 32 : -1, c.b))
                    return;
            }
            return;
        }
        // no tensor maps: residual and gate rows straight from global memory, the next step's
        // loaded while this one is summed (each thread owns one feature: coalesced accesses)
        float ga[16], xa[16], gb[16], xb[16];
        gate_load16(p, e, lo, gcur, ga, xa);
        for (int k = 0; k < nsteps; ++k) {
            const int r0 = lo + 16 * k;
            uint32_t v[16];
            {
                float acc[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[j] = 0.f;
                for (int sp = 0; sp < p.splits; ++sp) {
                    const float * src = sp == rank ? part + (size_t)r0 * 128
                                                   : recv + ((size_t)(sp < rank ? sp : sp - 1) * rows_max + (r0 - lo)) * 128;
#pragma unroll
                    for (int j = 0; j < 16; ++j) acc[j] += src[j * 128 + ml];
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = __float_as_uint(acc[j]);
            }
            if (k + 1 < nsteps) gate_load16(p, e, r0 + 16, gcur, gb, xb);
            gate_store16(p, e, r0, v, ga, xa);
#pragma unroll
            for (int j = 0; j < 16; ++j) { ga[j] = gb[j]; xa[j] = xb[j]; }
        }
        return;
    }
    for (int k = 0; k < nsteps; ++k) {
        const int r0 = lo + 16 * k;                           // first tile row (token) of this step
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = 0.f;
        for (int s = 0; s < p.splits; ++s) {
            const float * src = s == rank ? part + (size_t)r0 * 128
                                          : recv + ((size_t)(s < rank ? s : s - 1) * rows_max + (r0 - lo)) * 128;
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] += src[j * 128 + ml];
        }
        // STORE / SWIGLU: out row values of this thread's feature
        float o[16];
        bool mine = true;                                     // this thread holds an output value
        if (Epi<EK>::swiglu) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float r = __shfl_xor_sync(0xffffffffu, acc[j], 1);
                o[j] = silu_out<Epi<EK>::bf16>(acc[j]) * r;                    // valid on even lanes (h1 row)
            }
            mine = !(lane & 1);
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                o[j] = acc[j] + e.bias;
                if (Epi<EK>::silu) o[j] = silu_out<Epi<EK>::bf16>(o[j]);
            }
        }
        if (tma) {
            uint8_t * sbuf = ebuf + (gs & 1) * kEBufBytes;
            if (gs >= 2 && threadIdx.x == 64) bulk_wait_read<1>();
            epi_bar();
            const int fw = Epi<EK>::swiglu ? 64 : 128;
            const int f = Epi<EK>::swiglu ? (ml >> 1) : ml;
            if (mine) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    if (Epi<EK>::bf16) reinterpret_cast<__nv_bfloat16 *>(sbuf)[j * fw + f] = __float2bfloat16_rn(o[j]);
                    else reinterpret_cast<float *>(sbuf)[j * fw + f] = o[j];
                }
            }
            fence_proxy_async_smem();
            epi_bar();
            if (threadIdx.x == 64) {
                tma_store_4d(tmO, sbuf, c0o, c.t0 + r0, c.b, cb);
                bulk_commit();
            }
            ++gs;
        } else if (mine && e.m_ok) {
            const long long base = (e.row_base + r0) * p.ldo + e.col;
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (r0 + j < e.ncols) put<Epi<EK>::bf16>(p.out, base + (long long)j * p.ldo, o[j]);
        }
    }
}

// 16 Q8_0 weights (one 16-byte chunk of a row) -> 16 bf16 w = bf16(q * d): each byte becomes the
// f32 2^23 + 128 + q by a byte permute into the mantissa (after flipping its sign bit), an f32x2
// subtract leaves q exactly, an f32x2 multiply gives q * d exactly (8 x 11 significant bits), and
// one conversion per pair rounds to bf16: the same bits as the load-time widening.
__device__ __forceinline__ void q8_chunk_to_bf16(const uint4 & u, float d, uint32_t (&o)[8]) {
    const uint32_t w4[4] = {u.x ^ 0x80808080u, u.y ^ 0x80808080u, u.z ^ 0x80808080u, u.w ^ 0x80808080u};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float f0 = __uint_as_float(__byte_perm(w4[i], 0x4B000000u, 0x7650u + 2 * h));
            const float f1 = __uint_as_float(__byte_perm(w4[i], 0x4B000000u, 0x7650u + 2 * h + 1));
            uint32_t r;
            asm("{\n\t.reg .b64 a, m, s, t;\n\t"
                "mov.b64 a, {%1, %2};\n\t"
                "mov.b64 m, {%3, %3};\n\t"
                "mov.b64 s, {%4, %4};\n\t"
                "add.rn.f32x2 t, a, m;\n\t"
                "mul.rn.f32x2 t, t, s;\n\t"
                "{\n\t.reg .f32 lo, hi;\n\t"
                "mov.b64 {lo, hi}, t;\n\t"
                "cvt.rn.bf16x2.f32 %0, hi, lo;\n\t}\n\t}"
                : "=r"(r) : "f"(f0), "f"(f1), "f"(-8388736.0f), "f"(d));
            o[2 * i + h] = r;
        }
    }
}

// PAIR: the CTA-pair form (cta_group::2). A kernel holding cta_group::2 instructions must be
// launched in clusters of an even size, so the single-CTA form is a separate instance.
// FORM bits: 1 the multi-item form (several batch items per token tile, p.ipt > 1); 2 a workspace
// split-K whose last split gathers the partials (p.gather); 4 planar Q8_0 weights converted in
// shared memory (p.a_q8); 8 split-K inside a cluster (p.csplit); 16 a workspace split-K reduced
// by the last split's reducer; 32 an epilogue without TMA maps (p.epi_tma false: plain stores),
// which the other forms leave out. Separate instances, so that the common form (0, no split) runs
// straight-line code: compiled into one kernel, the other forms' loops and branches cost every
// GEMM 1-2% (measured).
template <int EK, bool PAIR, int FORM>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmG,
               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmS, const GemmParams p) {
    constexpr bool MI = (FORM & 1) != 0, GATHER = (FORM & 2) != 0, Q8 = (FORM & 4) != 0;
    constexpr bool CSPLIT = (FORM & 8) != 0, WSRED = (FORM & 16) != 0, PLAIN = (FORM & 32) != 0;
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t * ebuf = smem + kStageArea;                       // epilogue staging [2][kEBufBytes]
    uint64_t * full = reinterpret_cast<uint64_t *>(ebuf + 2 * kEBufBytes);
    uint64_t * empty = full + kMaxStages;
    uint64_t * acc_full = empty + kMaxStages;  // [2]
    uint64_t * acc_empty = acc_full + 2;       // [2]
    uint64_t * ebar = acc_empty + 2;           // [2] residual / gate tile loads (GATE_RESID, TMA epilogue)
    uint64_t * cbar = ebar + 2;                // [3] cluster split-K: slice rows received / own copies
                                               //     landed at the peers / peers ready to receive
    uint64_t * rfull = cbar + 3;               // [kMaxStages] Q8_0: raw int8 tile + scales landed
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(rfull + kMaxStages);
    volatile int * s_abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int * s_last = s_abort + 1;       // split-K: this CTA reduces the tile

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kpt = p.K_in >> 6;
    const int nkb = p.taps * kpt;
    const int kpb = p.kpb;                       // K blocks per stage (a K step); kpt % kpb == 0
    const int nks = nkb / kpb;                   // K steps; tile K ranges are in K steps
    // CTA pairs: consecutive cluster ranks 2j (leader) and 2j + 1 share pair tiles
    const uint32_t crank = (PAIR || CSPLIT) ? cluster_ctarank() : 0u;
    const int prank = PAIR ? (int)(crank & 1u) : 0;           // this CTA's half of the pair tile
    const uint32_t lead = crank & ~1u;                           // cluster rank of the pair leader
    const int srank = PAIR ? (int)(crank >> 1) : (int)crank;   // cluster split-K: this CTA's split
    const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int tstep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
    const int num_tiles = (PAIR ? p.mblocks >> 1 : p.mblocks) * p.groups * p.n_tiles * p.splits;
    const int bh = PAIR ? p.BN >> 1 : p.BN;                   // token rows of B this CTA loads
    // one stage: kpb A atoms (bf16 128 x 64, SW128) | kpb B atoms (bh x 64) | Q8_0 path (kpb = 1):
    // int8 tile + scales; a multiple of 1024 bytes, so every stage's SW128 atoms stay aligned
    const uint32_t b_bytes = (uint32_t)(bh * 128);                   // one B atom
    const int sbytes = kpb * (kABytes + (int)b_bytes) + (Q8 ? kQ8Bytes : 0);
    const int nst = p.stages;                   // ring depth, <= kMaxStages, nst * sbytes <= kStageArea
    // Q8_0: warps 6-7 convert each stage's int8 tile; a CTA with a single tile (no epilogue to
    // overlap with a later main loop) puts its four epilogue warps on the conversion as well
    const bool q8_single = Q8 && tile0 + tstep >= num_tiles;
    const int q8_conv_warps = q8_single ? 6 : 2;
    // Q8_0 conversion of every stage of this CTA's tiles by converter thread `cid` of `ncv`:
    // 16-byte units u = row * 4 + chunk of the 128 x 64 int8 tile, each to two 16-byte chunks of
    // the bf16 A tile in the 128-byte-swizzled layout TMA would have written (16-byte chunk j of
    // row r at r * 128 + ((j ^ (r & 7)) << 4)); then one arrival per warp on the stage's barrier.
    const auto convert_q8 = [&](int cid, int ncv) {
        int s = 0;
        uint32_t ph = 0;
        for (int t = tile0; t < num_tiles; t += tstep) {
            const TileCoord c = decode(p, t, nks, prank);    // kpb = 1 on this path
            bool ok = true;
            for (int kb = c.kb_begin; kb < c.kb_end; ++kb) {
                if (!mbar_wait(&rfull[s], ph, s_abort, p.err, DEV_TIMEOUT_FULL)) { ok = false; break; }
                uint8_t * sa = smem + s * sbytes;
                const uint8_t * raw = sa + kABytes + p.BN * 128;
                const __half * sc = reinterpret_cast<const __half *>(raw + 128 * 64);
                for (int u = cid; u < 512; u += ncv) {
                    const int r = u >> 2, jj = u & 3;
                    const uint4 q = reinterpret_cast<const uint4 *>(raw + r * 64)[jj];
                    uint32_t o[8];
                    q8_chunk_to_bf16(q, __half2float(sc[(jj >> 1) * 128 + r]), o);
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int j = jj * 2 + half;
                        *reinterpret_cast<uint4 *>(sa + r * 128 + ((j ^ (r & 7)) << 4)) =
                            make_uint4(o[4 * half], o[4 * half + 1], o[4 * half + 2], o[4 * half + 3]);
                    }
                }
                fence_proxy_async_smem();       // the MMA reads the tile through the async proxy
                __syncwarp();
                if ((threadIdx.x & 31) == 0) mbar_arrive(&full[s]);
                if (++s == nst) { s = 0; ph ^= 1; }
            }
            if (!ok) break;
        }
    };

    if (threadIdx.x == 0) {
        // full: the producer's expect_tx (+ both converter warps' arrivals on the Q8_0 path)
        for (int s = 0; s < kMaxStages; ++s) {
            mbar_init(&full[s], Q8 ? 1 + q8_conv_warps : 1); mbar_init(&empty[s], 1); mbar_init(&rfull[s], 1);
        }
        // acc_empty: the four epilogue warps (of both CTAs of a pair, on the leader's)
        for (int s = 0; s < 2; ++s) { mbar_init(&acc_full[s], 1); mbar_init(&acc_empty[s], PAIR ? 8 : 4); mbar_init(&ebar[s], 1); }
        mbar_init(&cbar[0], 1);
        for (int s = 1; s < 3; ++s) mbar_init(&cbar[s], CSPLIT ? p.splits - 1 : 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) { tma_prefetch(&tmA); tma_prefetch(&tmB); }
    if (threadIdx.x == 64 && p.epi_tma) {
        tma_prefetch(&tmO);
        if ((Epi<EK>::gate && p.gate_div == 1) || Epi<EK>::qkv) tma_prefetch(&tmG);
        if (Epi<EK>::qkv) tma_prefetch(&tmV);
    }
    if (warp == 1) {
        if constexpr (PAIR) { tmem_alloc_pair(tmem_slot, kTmemCols); tmem_relinquish_pair(); }
        else { tmem_alloc(tmem_slot, kTmemCols); tmem_relinquish(); }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // pairs / cluster split-K: every CTA's barriers are initialised before any other CTA of the
    // cluster signals them; cbar[0] then expects the bytes of this split's slice from each of
    // the other splits
    if (CSPLIT || PAIR) cluster_sync_all();
    if (CSPLIT && threadIdx.x == 64) {
        const int rows = slice_lo(srank + 1, p.BN, p.splits) - slice_lo(srank, p.BN, p.splits);
        mbar_arrive_expect_tx(&cbar[0], (uint32_t)((p.splits - 1) * rows * 512));
    }
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();

    // ---------------- TMA producers ----------------
    // A TMA instruction costs its issuing thread ~300 cycles whatever the box size, and an
    // integer division ~120, against 310-520 cycles of MMAs per K block: one thread issuing both
    // tiles of every K block (and dividing to find the conv tap) bound the mainloop. So a stage
    // holds kpb = 2 K blocks where K allows (one 3-D / 4-D box per operand per stage), the weight
    // tiles (A) are issued by two threads (warps 0 and 7, alternate stages) and the activation
    // tiles (B) by a third (warp 6), each walking K by increments. On the Q8_0 path warps 6-7
    // convert and warp 0 issues everything. Weight tiles of the first stages do not depend on
    // earlier kernels: they are requested before the wait for the predecessor grid.
    // role bit 1: A (weights; arms `full` with the stage's bytes), bit 2: B (activations);
    // A of K step `it` is issued by the part with it % a_parts == a_part.
    const auto produce = [&](const int role, const int a_part, const int a_parts) {
        const bool do_a = role & 1, do_b = role & 2;
        const uint32_t stage_tx = (uint32_t)kpb * (kABytes + b_bytes) * (PAIR ? 2u : 1u);
        const auto issue_a = [&](int st, int kb, int ya) {
            uint8_t * sa = smem + st * sbytes;
            if (Q8) {
                uint8_t * raw = sa + kABytes + p.BN * 128;
                mbar_arrive_expect_tx(&rfull[st], 128 * 64 + 2 * 128 * 2);
                tma_load_2d(raw, &tmA, &rfull[st], kb * 64, ya);
                tma_load_2d(raw + 128 * 64, &tmS, &rfull[st], ya, kb * 2);
            } else if constexpr (PAIR) {
                // both CTAs' tiles count on the leader's barrier, which the leader arms
                if (prank == 0) mbar_arrive_expect_tx(&full[st], stage_tx);
                tma_load_3d_pair(sa, &tmA, mapa_shared(smem_u32(&full[st]), lead), 0, ya, kb);
            } else {
                mbar_arrive_expect_tx(&full[st], stage_tx);
                tma_load_3d(sa, &tmA, &full[st], 0, ya, kb);
            }
        };
        const auto issue_b = [&](int st, int kc, int yb, int b) {
            uint8_t * sb = smem + st * sbytes + kpb * kABytes;
            if (Q8) mbar_arrive_expect_tx(&full[st], b_bytes);
            // multi-item tile: one box per K atom holding bni token rows of each of this CTA's items,
            // item after item (a pair: the leader the first ipt / 2 items, the peer the rest), so
            // the items' rows form one operand of ipt * bni rows for a single MMA; rows past an
            // item's end and items past the batch read the fill value zero
            if constexpr (PAIR) {
                if (MI) {
                    for (int j = 0; j < kpb; ++j)
                        tma_load_4d_pair(sb + (size_t)j * b_bytes, &tmB, mapa_shared(smem_u32(&full[st]), lead), 0,
                                         yb, kc + j, b + prank * (p.ipt >> 1));
                } else {
                    tma_load_4d_pair(sb, &tmB, mapa_shared(smem_u32(&full[st]), lead), 0, yb, kc, b);
                }
            } else {
                if (MI) {
                    for (int j = 0; j < kpb; ++j) tma_load_4d(sb + (size_t)j * b_bytes, &tmB, &full[st], 0, yb, kc + j, b);
                } else {
                    tma_load_4d(sb, &tmB, &full[st], 0, yb, kc, b);
                }
            }
        };
        const int amask = a_parts - 1;                       // a_parts is 1 or 2
        int pre = 0;
        if (do_a) {
            for (int t = tile0; t < num_tiles && pre < nst; t += tstep) {
                const TileCoord c = decode(p, t, nks, prank);
                for (int ks = c.kb_begin; ks < c.kb_end && pre < nst; ++ks, ++pre)
                    if ((pre & amask) == a_part) issue_a(pre, ks * kpb, c.mb * 128);
            }
        }
        if (do_b) pdl_wait();
        int it = 0;
        int s = 0;                 // ring slot of `it`, and the parity of its use (it / nst) & 1
        uint32_t ph = 0;
        for (int t = tile0; t < num_tiles && !*s_abort; t += tstep) {
            const TileCoord c = decode(p, t, nks, prank);
            const int kb0 = c.kb_begin * kpb;
            const int tap = kb0 / kpt;                       // conv tap and K block within it
            int kc = kb0 - tap * kpt;
            // first token row of the B tile (a multi-item pair tile: whole items on each CTA)
            int yb = c.t0 + (MI ? 0 : prank * bh) + tap - p.pad;
            const int ya = c.mb * 128;
            bool ok = true;
            for (int ks = c.kb_begin; ks < c.kb_end; ++ks, ++it) {
                const int cs = s;
                const uint32_t cph = ph;
                if (++s == nst) { s = 0; ph ^= 1; }
                const bool a_now = do_a && it >= pre && (it & amask) == a_part;   // first stages went out early
                if (it >= nst && (a_now || do_b) && !mbar_wait(&empty[cs], cph ^ 1, s_abort, p.err, DEV_TIMEOUT_EMPTY)) {
                    ok = false;
                    break;
                }
                if (a_now) issue_a(cs, ks * kpb, ya);
                if (do_b) issue_b(cs, kc, yb, c.b);
                kc += kpb;
                if (kc == kpt) { kc = 0; ++yb; }              // next tap: the token window moves by one
            }
            if (!ok) break;
        }
        if (*s_abort && !PAIR) {
            // Let this thread's copies still in flight land before the CTA exits (one deadline).
            const int issued = it > pre ? it : pre;
            const unsigned long long t_start = globaltimer();
            for (int i = (issued > nst ? issued - nst : 0); i < issued; ++i) {
                uint64_t * bar = (Q8 && do_a) ? &rfull[i % nst] : &full[i % nst];
                while (!mbar_try_wait(bar, (i / nst) & 1) && globaltimer() - t_start < wait_ns()) {}
            }
        }
    };

    if (warp == 0 || (!Q8 && warp >= 6)) {
        // one call site for every producer thread (one inlined copy of the loop): warp 0 weight
        // tiles of even K steps (Q8_0: every tile of both operands), warp 6 the activation
        // tiles, warp 7 the weight tiles of odd K steps
        if (lane == 0) produce(Q8 ? 3 : warp == 6 ? 2 : 1, warp == 7 ? 1 : 0, Q8 ? 1 : 2);
    } else if (warp == 1) {
        if (lane == 0 && prank == 0) {
            // ---------------- MMA issuer (a pair's leader issues for both CTAs) ----------------
            // (a multi-item tile: N = ipt * bni, every item's rows in one MMA)
            const uint32_t idesc = make_idesc_f16(PAIR ? 256 : 128, p.BN, true);
            const uint16_t pmask = (uint16_t)(3u << lead);
            int it = 0, lt = 0;
            int s = 0;                 // ring slot of `it` and the parity of its fill
            uint32_t ph = 0;
            bool ok = true;
            for (int t = tile0; ok && t < num_tiles; t += tstep, ++lt) {
                const TileCoord c = decode(p, t, nks, prank);
                const int buf = lt & 1;
                if (lt >= 2) {
                    const uint32_t par = ((lt >> 1) & 1) ^ 1;
                    if (!(PAIR ? mbar_wait_cluster(&acc_empty[buf], par, p.err, DEV_TIMEOUT_ACC)
                                 : mbar_wait(&acc_empty[buf], par, s_abort, p.err, DEV_TIMEOUT_ACC)))
                        break;
                }
                tc_fence_after();
                const uint32_t dacc = tmem + buf * 256;
                for (int kb = c.kb_begin; kb < c.kb_end; ++kb, ++it) {
                    const int cs = s;
                    if (!mbar_wait(&full[cs], ph, s_abort, p.err, DEV_TIMEOUT_FULL)) { ok = false; break; }
                    if (++s == nst) { s = 0; ph ^= 1; }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + cs * sbytes);
                    for (int j = 0; j < kpb; ++j) {
                        const uint64_t adesc = make_sdesc_sw128(sa + j * kABytes);
                        const uint64_t bdesc = make_sdesc_sw128(sa + kpb * kABytes + j * b_bytes);
                        const uint32_t acc0 = (kb > c.kb_begin || j > 0) ? 1u : 0u;
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            if constexpr (PAIR) umma_f16_ss_pair(dacc, adesc + 2 * kk, bdesc + 2 * kk, idesc, (acc0 | kk) ? 1u : 0u);
                            else umma_f16_ss(dacc, adesc + 2 * kk, bdesc + 2 * kk, idesc, (acc0 | kk) ? 1u : 0u);
                        }
                    }
                    if constexpr (PAIR) umma_commit_pair(&empty[cs], pmask);
                    else umma_commit(&empty[cs]);
                }
                if constexpr (PAIR) umma_commit_pair(&acc_full[buf], pmask);
                else umma_commit(&acc_full[buf]);
            }
        }
    } else if (warp >= 6) {
        // ---------------- Q8_0 converters (warps 6, 7) ----------------
        if constexpr (Q8) convert_q8((warp - 6) * 32 + lane, 32 * q8_conv_warps);
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        if (q8_single) convert_q8(64 + (warp - 2) * 32 + lane, 32 * q8_conv_warps);
        pdl_wait();
        const int q = warp & 3;                       // TMEM lane quadrant of this warp
        const int ml = q * 32 + lane;                 // TMEM lane = weight row within the tile
        int gs = 0;                                   // staging-buffer uses so far (buffer gs & 1)
        int nqk = 0;                                  // QKV: chunks that took the RMS exchange barrier
        int gl = 0;                                   // thread 64: residual / gate loads issued
        int lt = 0;
        // TMEM buffer `buf` is free again: on the pair leader's barrier for both CTAs
        const auto release_acc = [&](int buf) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (PAIR && prank) mbar_arrive_remote(mapa_shared(smem_u32(&acc_empty[buf]), lead));
                else mbar_arrive(&acc_empty[buf]);
            }
        };
        const int ebn = MI ? p.bni : p.BN;            // token columns finished at a time
        for (int t = tile0; t < num_tiles; t += tstep, ++lt) {
            TileCoord c = decode(p, t, nks, prank);      // (a multi-item tile advances c.b per item)
            const int buf = lt & 1;
            EpiCtx e;
            // output feature of this thread (SwiGLU: rows 2i / 2i + 1 are w1 / w3 of feature i)
            e.m = Epi<EK>::swiglu ? c.mb * 64 + (ml >> 1) : c.mb * 128 + ml;
            e.m_ok = e.m < p.m_valid;
            e.bias = (p.bias && e.m_ok && !Epi<EK>::swiglu) ? p.bias[e.m] : 0.f;
            e.ncols = min(ebn, p.S - c.t0);
            e.row_base = (long long)c.b * p.S + c.t0;
            e.col = p.out_cblk ? (long long)(e.m / p.out_cblk) * p.out_cstride + e.m % p.out_cblk : e.m;
            constexpr bool whole = !CSPLIT && !WSRED;         // this CTA finishes whole tiles
            const bool tma = whole && !PLAIN;                 // (forms without PLAIN: p.epi_tma)
            const bool tma_gate = p.epi_tma && (whole || CSPLIT);             // residual / gate maps exist
            const int m0 = Epi<EK>::swiglu ? c.mb * 64 : c.mb * 128;    // first output feature of the tile
            const int cb = p.out_cblk ? m0 / p.out_cblk : 0;              // its column block (output map dim 3)
            const int c0o = m0 - cb * p.out_cblk;
            const int nsteps = ebn >> 4;                                  // GATE_RESID: 16-token steps
            const bool gtile = p.gate_div == 1;                           // per-token gate (else one per item)
            // gate + residual of the first columns are fetched while the accumulator fills
            GateCursor gcur{nullptr, 0};
            float ga[16], xa[16], gb[16], xb[16];
            // (GATE_RESID) the gate rows this CTA will read, into L2; the first gate / residual
            // tiles of a whole-tile epilogue in flight
            const auto gate_prologue = [&]() {
                if (Epi<EK>::gate && tma_gate && gtile && threadIdx.x == 64) {
                    // (the per-token gate planes are not L2-resident)
                    int lo = 0, hi = e.ncols;
                    if (CSPLIT) { lo = slice_lo(srank, p.BN, p.splits); hi = min(slice_lo(srank + 1, p.BN, p.splits), e.ncols); }
                    for (int t = lo + 32; t < hi; t += 16) tma_prefetch_l2_4d(&tmG, m0, c.t0 + t, c.b, 0);
                }
                if (Epi<EK>::gate && whole) {
                    if (tma) {
                        if (!gtile) {                                         // gate rows walked by a cursor
                            const long long grow = e.row_base / p.gate_div;
                            gcur.g = p.gate + grow * p.ldg + e.m;
                            gcur.gpos = (int)(e.row_base - grow * p.gate_div);
                        }
                        if (threadIdx.x == 64 && gtile) {
                            for (int s2 = 0; s2 < 2 && s2 < nsteps; ++s2, ++gl)
                                gate_issue(&tmG, ebar, ebuf, gl, m0, c.t0 + 16 * s2, c.b);
                        }
                    } else {
                        const long long grow = e.row_base / p.gate_div;
                        gcur.g = p.gate + grow * p.ldg + e.m;
                        gcur.gpos = (int)(e.row_base - grow * p.gate_div);
                        gate_load16(p, e, 0, gcur, ga, xa);
                    }
                }
            };
            // while the accumulator fills (a gathering split learns only afterwards whether it
            // finishes the tile)
            if constexpr (!GATHER) gate_prologue();
            float2 rcs[32];                                               // QKV: RoPE (cos, sin) of a chunk
            if (Epi<EK>::qkv && p.rope && c.mb * 128 < 2 * p.hidden)
                rope_load(p, e, c, 0, (c.mb * 128 - (c.mb * 128 / p.hidden) * p.hidden + ml) & 63, rcs);
            // warp-uniform outcome: tcgen05.ld below is warp-collective
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (lt >> 1) & 1, s_abort, p.err, DEV_TIMEOUT_ACC)))
                break;
            tc_fence_after();
            const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + buf * 256;
            if constexpr (GATHER) {
                // Split-K through the global workspace, one tile per CTA (the operand stages are
                // idle now). Every split but the last to complete the tile stores its partial tile
                // and leaves; the last one (it skips its own store when the others are all in
                // already) brings the other partials into its stages with bulk copies, adds them
                // to its accumulator in TMEM in split order (the same sum as the reducer of the
                // workspace path) and finishes the tile as an unsplit one.
                int * ctr = p.counters + c.otile;
                if (threadIdx.x == 64) *s_last = ld_acquire_gpu(ctr) == p.splits - 1 ? 2 : 0;
                epi_bar();
                const bool early = *s_last == 2;
                if (!early) {
                    float * wsp = p.ws + ((size_t)(c.otile * p.splits + c.split) * p.BN) * 128 + ml;
                    for (int j0 = 0; j0 < p.BN; j0 += 32) {
                        float v[32];
                        tmem_ld32(trow + j0, v);
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j0 + j < p.BN) __stcg(wsp + (size_t)(j0 + j) * 128, v[j]);
                    }
                    __threadfence();
                    epi_bar();
                    if (threadIdx.x == 64) *s_last = atomicAdd(ctr, 1) == p.splits - 1 ? 1 : 0;
                    epi_bar();
                }
                if (*s_last == 0) {            // another split finishes this tile
                    release_acc(buf);
                    epi_bar();                 // every thread has read s_last
                    continue;
                }
                if (threadIdx.x == 64) {
                    __threadfence();           // acquire the other splits' partial tiles ...
                    fence_proxy_async_all();   // ... for the bulk copies
                    *ctr = 0;                  // ready for the next launch
                    mbar_arrive_expect_tx(&cbar[0], (uint32_t)(p.splits - 1) * (uint32_t)p.BN * 512u);
                    for (int sp = 0, k = 0; sp < p.splits; ++sp)
                        if (sp != c.split)
                            bulk_load_g2s(smem + (size_t)(k++) * p.BN * 512,
                                          p.ws + ((size_t)(c.otile * p.splits + sp) * p.BN) * 128,
                                          (uint32_t)p.BN * 512u, &cbar[0]);
                }
                if (!__all_sync(0xffffffffu, mbar_wait(&cbar[0], 0, s_abort, p.err, DEV_TIMEOUT_FULL))) {
                    release_acc(buf);
                    break;
                }
                const float * parts = reinterpret_cast<const float *>(smem);   // [splits - 1][BN][128]
                for (int j0 = 0; j0 < p.BN; j0 += 16) {
                    float own[16], a[16];
                    tmem_ld16(trow + j0, own);
#pragma unroll
                    for (int j = 0; j < 16; ++j) a[j] = 0.f;
                    for (int sp = 0, k = 0; sp < p.splits; ++sp) {
                        if (sp == c.split) {
#pragma unroll
                            for (int j = 0; j < 16; ++j) a[j] += own[j];
                        } else {
                            const float * src = parts + ((size_t)(k++) * p.BN + j0) * 128 + ml;
#pragma unroll
                            for (int j = 0; j < 16; ++j) a[j] += src[j * 128];
                        }
                    }
                    tmem_st16(trow + j0, a);
                }
                tmem_wait_st();
                gate_prologue();
            }
            if constexpr (whole) {
                bool failed = false;
                // one pass per item of a multi-item tile (item it in accumulator columns it * bni ..)
                for (int it = 0; it < (MI ? p.ipt : 1) && !failed; ++it) {
                if (MI && it > 0) {
                    if (++c.b >= p.nbatch) break;
                    e.row_base = (long long)c.b * p.S + c.t0;
                    gate_prologue();
                    if (Epi<EK>::qkv && p.rope && c.mb * 128 < 2 * p.hidden)
                        rope_load(p, e, c, 0, (c.mb * 128 - (c.mb * 128 / p.hidden) * p.hidden + ml) & 63, rcs);
                }
                const uint32_t trow_i = MI ? trow + (uint32_t)(it * p.bni) : trow;
                if (Epi<EK>::gate && tma) {
                    // gate tiles of 16 tokens by TMA two steps ahead, residual updates by TMA
                    // reduce-add (gate_step)
                    for (int s2 = 0; s2 < nsteps; ++s2, ++gs) {
                        float v[16], gv[16];
                        if (!gtile) {
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                gv[j] = 0.f;
                                if (e.m_ok && 16 * s2 + j < e.ncols) gv[j] = __ldg(gcur.g);
                                if (++gcur.gpos == p.gate_div) { gcur.gpos = 0; gcur.g += p.ldg; }
                            }
                        }
                        tmem_ld16(trow_i + 16 * s2, v);
                        if (!gate_step(p, e, &tmO, &tmG, gtile, ebar, ebuf, gs, gl, v, gv, ml, m0, c.t0 + 16 * s2,
                                       s2 + 2 < nsteps ? c.t0 + 16 * (s2 + 2) : -1, c.b)) {
                            failed = true;
                            break;
                        }
                    }
                } else if (Epi<EK>::gate) {
                    // The next chunk's TMEM load and its gate / residual loads are in flight
                    // while this chunk's results are stored.
                    uint32_t va[16], vb[16];
                    tmem_ld16_async(trow_i, va);
                    tmem_wait_ld(va);
                    for (int c0 = 0; c0 < ebn; c0 += 32) {
                        const bool nb = c0 + 16 < ebn;
                        if (nb) { gate_load16(p, e, c0 + 16, gcur, gb, xb); tmem_ld16_async(trow_i + c0 + 16, vb); }
                        gate_store16(p, e, c0, va, ga, xa);
                        if (!nb) break;
                        tmem_wait_ld(vb);
                        const bool na = c0 + 32 < ebn;
                        if (na) { gate_load16(p, e, c0 + 32, gcur, ga, xa); tmem_ld16_async(trow_i + c0 + 32, va); }
                        gate_store16(p, e, c0 + 16, vb, gb, xb);
                        if (!na) break;
                        tmem_wait_ld(va);
                    }
                } else {
                    // One call site per epilogue body keeps the instruction footprint small (a
                    // TMEM load is ~50 cycles; prefetching it would double the inlined code).
                    for (int j0 = 0; j0 < ebn; j0 += 32) {
                        uint32_t v[32];
                        tmem_ld32_async(trow_i + j0, v);
                        tmem_wait_ld(v);
                        if (Epi<EK>::qkv) emit_qkv<!PLAIN>(p, e, c, j0, v, ml, lane, q, ebuf, nqk, gs, &tmO, &tmG, &tmV, rcs);
                        else if (tma) tma_chunk<EK>(p, &tmO, e, j0, v, ml, lane, ebuf, gs, c0o, cb, c.b, c.t0);
                        else if (Epi<EK>::swiglu) emit_swiglu<EK>(p, e, j0, v, lane);
                        else emit_store<EK>(p, e, j0, v);
                    }
                }
                }
                release_acc(buf);
                if (failed) break;
            } else if constexpr (CSPLIT) {
                // Split-K inside the cluster (one tile per CTA; the operand stages are idle now):
                // partial tile -> own shared memory; the row slices the other ranks finish are
                // pushed into their receive slots by bulk copies that complete on their barrier;
                // then this CTA's slice is summed over all ranks and finished.
                // splits are ranks 0..splits-1 (pairs: cluster rank 2 * split + prank)
                const int rank = srank;
                const auto crk = [&](int d) { return (uint32_t)(PAIR ? 2 * d + prank : d); };
                const int rows_max = slice_rows_max(p.BN, p.splits);
                const int lo = slice_lo(rank, p.BN, p.splits), hi = slice_lo(rank + 1, p.BN, p.splits);
                float * part = reinterpret_cast<float *>(smem);                  // [BN][128]
                float * recv = part + (size_t)p.BN * 128;                         // [splits - 1][rows_max][128]
                if (threadIdx.x == 64) {     // the MMAs are done: this CTA's stages may now be written by peers
                    for (int d = 0; d < p.splits; ++d)
                        if (d != rank) mbar_arrive_remote(mapa_shared(smem_u32(&cbar[2]), crk(d)));
                }
                // TMEM -> partial tile, 16 columns at a time with the next load in flight (BN % 16 == 0)
                {
                    uint32_t va[16], vb[16];
                    tmem_ld16_async(trow, va);
                    tmem_wait_ld(va);
                    for (int j0 = 0; j0 < p.BN; j0 += 32) {
                        const bool nb = j0 + 16 < p.BN;
                        if (nb) tmem_ld16_async(trow + j0 + 16, vb);
#pragma unroll
                        for (int j = 0; j < 16; ++j) part[(j0 + j) * 128 + ml] = __uint_as_float(va[j]);
                        if (!nb) break;
                        tmem_wait_ld(vb);
                        const bool na = j0 + 32 < p.BN;
                        if (na) tmem_ld16_async(trow + j0 + 32, va);
#pragma unroll
                        for (int j = 0; j < 16; ++j) part[(j0 + 16 + j) * 128 + ml] = __uint_as_float(vb[j]);
                        if (!na) break;
                        tmem_wait_ld(va);
                    }
                }
                release_acc(buf);
                fence_proxy_async_smem();
                epi_bar();
                // push once every peer's stages are free (a timed-out wait sends nothing)
                if (threadIdx.x == 64 && mbar_wait_cluster(&cbar[2], 0, p.err, DEV_TIMEOUT_CLUSTER)) {
                    for (int d = 0; d < p.splits; ++d) {
                        if (d == rank) continue;
                        const int dlo = slice_lo(d, p.BN, p.splits), dhi = slice_lo(d + 1, p.BN, p.splits);
                        if (dhi <= dlo) continue;
                        const int slot = rank < d ? rank : rank - 1;          // this rank's slot at d
                        const uint32_t dst = mapa_shared(smem_u32(recv + (size_t)slot * rows_max * 128), crk(d));
                        bulk_copy_to_peer(dst, part + (size_t)dlo * 128, (uint32_t)(dhi - dlo) * 512u,
                                          mapa_shared(smem_u32(&cbar[0]), crk(d)));
                    }
                }
                // the other ranks' rows of this slice have landed (byte count on cbar[0])
                if (__all_sync(0xffffffffu, mbar_wait_cluster(&cbar[0], 0, p.err, DEV_TIMEOUT_CLUSTER))) {
                    if (threadIdx.x == 64) {                                       // tell the senders
                        for (int d = 0; d < p.splits; ++d)
                            if (d != rank) mbar_arrive_remote(mapa_shared(smem_u32(&cbar[1]), crk(d)));
                    }
                    finish_slice<EK>(p, &tmO, &tmG, c, e, part, recv, rows_max, rank, lo, hi, ml, lane, ebuf, ebar, gs, gl);
                }
                // this CTA's outgoing copies have landed at every peer before it exits
                __all_sync(0xffffffffu, mbar_wait_cluster(&cbar[1], 0, p.err, DEV_TIMEOUT_CLUSTER));
            } else {
                // Split-K, deterministic: every split stores its partial tile; the CTA that
                // completes the tile last sums the partials in split order and runs the epilogue.
                float * wsp = p.ws + ((size_t)(c.otile * p.splits + c.split) * p.BN) * 128 + ml;
                for (int j0 = 0; j0 < p.BN; j0 += 32) {
                    float v[32];
                    tmem_ld32(trow + j0, v);
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j0 + j < p.BN) __stcg(wsp + (size_t)(j0 + j) * 128, v[j]);
                }
                release_acc(buf);
                __threadfence();
                epi_bar();
                if (threadIdx.x == 64) *s_last = (atomicAdd(&p.counters[c.otile], 1) == p.splits - 1);
                epi_bar();
                if (*s_last) {
                    __threadfence();
                    reduce_tile<EK>(p, c, q, lane);
                    if (threadIdx.x == 64) p.counters[c.otile] = 0;   // ready for the next launch
                }
                epi_bar();   // every thread has read s_last before the next tile rewrites it
            }
        }
        if (threadIdx.x == 64) {
            // loads issued but not consumed (a wait gave up): let them land before the CTA exits
            for (int g = gs; g < gl; ++g) {
                const unsigned long long t_start = globaltimer();
                while (!mbar_try_wait(&ebar[g & 1], (g >> 1) & 1) && globaltimer() - t_start < wait_ns()) {}
            }
            bulk_wait<0>();                           // TMA stores complete before exit
        }
        if (threadIdx.x == 96) bulk_wait<0>();      // gate epilogue: this thread's reduce-adds complete
        if (Epi<EK>::qkv && lane == 0) bulk_wait<0>();   // QKV: every epilogue warp's stores complete
    }
    tc_fence_before();
    __syncwarp();
    // a pair's CTAs signal each other's barriers and the leader's MMAs read the peer's shared
    // memory and write its tensor memory: neither leaves before both are done
    if (PAIR) cluster_sync_all();
    else __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR) tmem_dealloc_pair(tmem, kTmemCols);
        else tmem_dealloc(tmem, kTmemCols);
    }
}

typedef CUresult (*PFN_encodeTiled_t)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                      const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled_t encode_fn() {
    static PFN_encodeTiled_t fn = nullptr;
    if (!fn) {
        void * ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_encodeTiled_t>(ptr);
    }
    return fn;
}

}  // namespace

bool pdl_enabled() {
    static int on = -1;
    if (on < 0) {
        const char * e = getenv("TSD_NO_PDL");
        on = (e && *e && *e != '0') ? 0 : 1;
    }
    return on == 1;
}

bool make_tmap_2d(CUtensorMap * m, const void * ptr, CUtensorMapDataType dt, int esize, uint64_t d0, uint64_t d1,
                  uint64_t stride1_bytes, uint32_t b0, uint32_t b1) {
    auto fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15) || (stride1_bytes & 15) || (b0 * esize) % 16) return false;
    cuuint64_t dims[2] = {d0, d1};
    cuuint64_t strides[1] = {stride1_bytes};
    cuuint32_t box[2] = {b0, b1};
    cuuint32_t es[2] = {1, 1};
    CUtensorMapSwizzle sw = (b0 * esize == 128) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
    return fn(m, dt, 2, const_cast<void *>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_tmap_3d(CUtensorMap * m, const void * ptr, CUtensorMapDataType dt, int esize, uint64_t d0, uint64_t d1,
                  uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2) {
    auto fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15) || (stride1_bytes & 15) || (stride2_bytes & 15) ||
        (b0 * esize) % 16)
        return false;
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
    cuuint32_t box[3] = {b0, b1, b2};
    cuuint32_t es[3] = {1, 1, 1};
    CUtensorMapSwizzle sw = (b0 * esize == 128) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
    return fn(m, dt, 3, const_cast<void *>(ptr), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Clusters of `cs` CTAs of this kernel that can be resident at once (0 if unknown), cached per
// device. One CTA fills an SM, so this is set by how SMs group into GPCs.
static int max_active_clusters(int cs) {
    static int cache[64][9];
    static bool done[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || cs < 1 || cs > 8) return 0;
    if (!done[dev]) {
        done[dev] = true;
        cudaFuncSetAttribute(gemm_tc_kernel<EK_F32, false, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        for (int k = 1; k <= 8; ++k) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)(k * (sms / k)), 1, 1);
            cfg.blockDim = dim3(kThreads, 1, 1);
            cfg.dynamicSmemBytes = kSmemBytes;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = (unsigned)k; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = 1;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<EK_F32, false, 0>, &cfg) != cudaSuccess) {
                cudaGetLastError();
                n = 0;
            }
            cache[dev][k] = n;
        }
    }
    return cache[dev][cs];
}

// Tile / split / pair choice from a cost model of the kernel's time in SM cycles, built on
// single-thread issue costs measured on B200: a TMA instruction costs its issuing thread ~300
// cycles, a K=16 MMA at M=128 takes max(65, N / 2) cycles, and the MMA issuer loses ~250 cycles
// at each stage's barrier wait unless enough MMA work is queued. A CTA's time is its K blocks
// times the per-stage maximum of those, over the waves of CTAs, plus the exposed epilogue of
// the last tile (~20 B / cycle of output). Split-K trades a reduction for parallelism: within
// one wave the splits of a tile form a cluster and reduce through distributed shared memory
// (~2000 cycles + the slice rows); beyond one wave they reduce through the global workspace,
// whose last-arriving CTA was measured at ~40000 cycles.
struct TileChoice {
    double cost;
    int BN, splits, pair;
    int ipt = 1;       // batch items per token tile (BN = ipt x the item's rows when > 1)
};
// CTA pairs (cta_group::2) halve the token bytes each SM draws: a pair computes 256 weight
// rows x BN tokens, each CTA loading its 128 weight rows and BN / 2 tokens. They need an even
// m-block count, a cluster of 2 (x the splits for a cluster split-K) and bf16 weights.
static bool pairs_enabled() {       // read per plan: tests compare both forms in one process
    const char * e = getenv("TSD_NO_PAIR");
    return !(e && *e && *e != '0');
}
// Split-K inside a thread-block cluster (no scratch) unless TSD_NO_CLUSTER_SPLIT is set to a
// non-zero value (tests: exercises the split-K that reduces through caller scratch). Read per plan.
static bool cluster_split_enabled() {
    const char * e = getenv("TSD_NO_CLUSTER_SPLIT");
    return !(e && *e && *e != '0');
}
// Workspace split-K in which the split that completes a tile last gathers the other partial
// tiles into its operand stages (one tile per CTA; the stages hold splits - 1 partials).
// TSD_NO_GATHER_SPLIT=1 leaves the reduction to the last split's reducer reading the workspace.
static bool gather_split_ok(int bn, int sp) {
    const char * e = getenv("TSD_NO_GATHER_SPLIT");
    if (e && *e && *e != '0') return false;
    return (long long)(sp - 1) * bn * 512 <= (long long)kStageArea;
}
// Several short batch items in one token tile (TSD_NO_MULTI_ITEM=1: one item per tile).
static bool multi_item_enabled() {
    const char * e = getenv("TSD_NO_MULTI_ITEM");
    return !(e && *e && *e != '0');
}
// Rows per item of a multi-item tile for items of S tokens, and whether `ipt` of them fit: the
// epilogue reads the accumulator of an item in 32-column chunks, so the last item's chunks must
// stay inside the tile's 256 TMEM columns (which also keeps the one MMA's N = ipt * bni <= 256).
static int item_rows(int S) { return (S + 15) / 16 * 16; }
static bool multi_item_fits(int S, int ipt) {
    const int bni = item_rows(S);
    return ipt >= 2 && S <= 128 && (ipt - 1) * bni + (bni + 31) / 32 * 32 <= 256;
}
// Every feasible (BN, splits, pair, items per tile), cheapest first by the model.
static std::vector<TileChoice> tile_choices(int S, int nbatch, int mblocks, int nkb, int num_sms, int max_splits,
                                            long long ws_floats, int n_counters, bool allow_cluster, bool allow_pair,
                                            bool k128, bool q8) {
    std::vector<TileChoice> out;
    for (int pair = 0; pair <= 1; ++pair) {
        if (pair && (!allow_pair || !allow_cluster || mblocks % 2 || !pairs_enabled() || max_active_clusters(2) < 1))
            continue;
        const int cpt = pair ? 2 : 1;                         // CTAs per tile
        for (int bn = 16; bn <= 256; bn += 16) {
            const int nt = (S + bn - 1) / bn;
            if (nt > 1 && ((S + nt - 1) / nt + 15) / 16 * 16 < bn) continue;   // a smaller bn gives the same count
            const long long otiles = (long long)(mblocks / cpt) * nbatch * nt;  // output tiles (pair tiles)
            for (int sp = 1; sp <= std::min(8, std::max(1, max_splits)); ++sp) {   // reducers sum <= 8 partials
                if (sp > 1 && nkb / sp < 4) break;
                const long long ctas = otiles * sp * cpt;
                bool cluster = allow_cluster && cluster_split_enabled() && sp > 1 && ctas <= num_sms && cpt * sp <= 8;
                if (cluster) {   // partial tile + receive slots fit the operand stages; clusters co-resident
                    const int rows_max = 16 * (((bn >> 4) + sp - 1) / sp);
                    const int mac = max_active_clusters(cpt * sp);
                    cluster = (long long)bn * 512 + (long long)(sp - 1) * rows_max * 512 <= (long long)kStageArea &&
                              mac > 0 && otiles <= mac;
                }
                if (sp > 1 && !cluster && (pair || otiles * cpt > n_counters || otiles * cpt * sp * bn * 128 > ws_floats))
                    continue;                                  // pairs split K only inside the cluster
                const long long slots = pair ? std::min<long long>(num_sms & ~1, 2ll * max_active_clusters(2)) : num_sms;
                const long long waves = (ctas + slots - 1) / slots;
                const double kb = (double)nkb / sp;                          // K blocks per tile
                const double kb_bytes = 16384.0 + 128.0 * bn / cpt;          // per CTA and K block
                const double tile_bytes = kb * kb_bytes;
                const long long wave_ctas = std::min<long long>(ctas, slots);
                // per stage of kpb K blocks: the MMAs (a K=16 MMA takes max(65, N / 2) cycles, N the
                // instruction's N: BN, also for pairs), plus what the issuer loses at its barrier
                // wait (~250 cycles, hidden only behind enough queued MMA work); at least one TMA
                // instruction of the B issuer (~300 cycles each). Per SM intake <= ~110 B / cycle.
                const int b_atom = (int)(128 * bn / cpt);
                const int kpb = (k128 && !q8 && kStageArea / (2 * (kABytes + b_atom)) >= 3 && nkb % (2 * sp) == 0 &&
                                 nkb / (2 * sp) >= 2) ? 2 : 1;
                const double mi = std::max(65.0, bn / 2.0);
                const double ex = 4.0 * kpb * mi;
                const double idle = kpb == 1 ? std::max(250.0 - (mi >= 100.0 ? ex - 260.0 : 0.0), 0.0) : (mi < 100.0 ? 244.0 : 0.0);
                const double t_stage = std::max(ex + idle, q8 ? 600.0 : 300.0);
                const double t_sm = kb * std::max(t_stage / kpb, kb_bytes / 110.0);
                const double t_l2 = (double)wave_ctas * tile_bytes / 12000.0;
                const double epi = bn * 128.0 * 4.0 / 20.0;
                // workspace split-K: the last split reduces alone (~40000 cycles), or, with one tile
                // per CTA, gathers the partials by bulk copy (~3000 cycles + ~5 per partial column)
                // and then runs the whole tile's epilogue, which a cluster split-K shares out among
                // the splits (measured: the gathering form of a tiling trails its cluster form)
                const bool gather = sp > 1 && !cluster && !pair && ctas <= num_sms && gather_split_ok(bn, sp);
                const double reduce = sp == 1 ? 0.0 : cluster ? 2000.0 + bn * 512.0 * 2.0 / 100.0
                                                    : gather ? 3000.0 + 5.0 * sp * bn + epi * (sp - 1) : 40000.0;
                const double cost = (double)waves * (std::max(t_sm, t_l2) + 3000.0) + epi + reduce;
                out.push_back({cost, bn, sp, pair});
            }
        }
    }
    // Multi-item tiles (short conv streams: items of <= 128 tokens): ipt items side by side, each
    // in bni rows, so every weight tile is read once for all of them instead of once per item.
    // No split. The token-tile issuer sends one box per K atom holding all of the CTA's items
    // (~500 cycles each), and per K=16 step one MMA covers every item (N = ipt bni). A CTA pair
    // takes an even number of items: each CTA loads half of them.
    const bool pairs_ok = allow_pair && allow_cluster && mblocks % 2 == 0 && pairs_enabled() && max_active_clusters(2) >= 1;
    if (nbatch >= 2 && multi_item_enabled())
        for (int pair = 0; pair <= (pairs_ok ? 1 : 0); ++pair)
            for (int ipt = 2; ipt <= nbatch && multi_item_fits(S, ipt); ++ipt) {
                if (pair && ipt % 2) continue;
                const int cpt = pair ? 2 : 1;
                const int bni = item_rows(S), bn = ipt * bni;
                const long long otiles = (long long)(mblocks / cpt) * ((nbatch + ipt - 1) / ipt);   // (pair tiles)
                const long long slots = pair ? std::min<long long>(num_sms & ~1, 2ll * max_active_clusters(2)) : num_sms;
                const long long waves = (otiles * cpt + slots - 1) / slots;
                const double kb = nkb;
                const int b_atom = 128 * bn / cpt;
                const double kb_bytes = 16384.0 + b_atom;
                const int kpb = (k128 && !q8 && kStageArea / (2 * (kABytes + b_atom)) >= 3 && nkb % 2 == 0 && nkb / 2 >= 2) ? 2 : 1;
                const int nst = std::min(kMaxStages, kStageArea / (kpb * (kABytes + b_atom) + (q8 ? kQ8Bytes : 0)));
                const double ex = 4.0 * kpb * std::max(65.0, bn / 2.0);
                // one token box per K atom; a stage comes back after the load latency (~2550
                // cycles under load) plus the MMAs that hold it, nst stages in flight
                const double t_stage = std::max(std::max(std::max(ex, 500.0 * kpb), (2550.0 + ex) / nst),
                                                q8 ? 600.0 : 300.0);
                const double t_sm = kb * std::max(t_stage / kpb, kb_bytes / 110.0);
                const double t_l2 = (double)std::min<long long>(otiles * cpt, slots) * kb * kb_bytes / 12000.0;
                const double epi = bn * 128.0 * 4.0 / 20.0;
                TileChoice t{(double)waves * (std::max(t_sm, t_l2) + 3000.0) + epi, bn, 1, pair};
                t.ipt = ipt;
                out.push_back(t);
            }
    std::stable_sort(out.begin(), out.end(), [](const TileChoice & a, const TileChoice & b) { return a.cost < b.cost; });
    return out;
}

int gemm_candidates(int M, int K_in, int taps, int nbatch, int S, int num_sms, int max_splits, long long ws_floats,
                    int n_counters, bool allow_cluster, int max_out, int * bn, int * splits, int * pair) {
    if (M % 128 || K_in % 64 || taps < 1 || S < 1 || nbatch < 1) return 0;
    const auto c = tile_choices(S, nbatch, M / 128, taps * (K_in / 64), num_sms, max_splits, ws_floats, n_counters,
                                allow_cluster, true, K_in % 128 == 0, false);
    int n = 0;
    for (const TileChoice & t : c) {
        if (n >= max_out) break;
        bn[n] = t.BN;
        splits[n] = t.splits;
        if (pair) pair[n] = t.pair;
        ++n;
    }
    return n;
}

long long gemm_ws_floats(const GemmLaunch & L) {
    const GemmParams & p = L.p;
    return p.splits > 1 && !p.csplit ? (long long)p.mblocks * p.groups * p.n_tiles * p.splits * p.BN * 128 : 0;
}

static bool make_tmap_4d(CUtensorMap * m, const void * ptr, CUtensorMapDataType dt, int esize, const uint64_t (&d)[4],
                         const uint64_t (&stride_bytes)[3], const uint32_t (&box)[4], bool sw128);

bool gemm_plan(GemmLaunch & L, const void * W, int M, int K_in, int taps, int pad, int swiglu, const void * X,
               int nbatch, int S, long long x_row_stride, long long x_batch_stride, int num_sms, int max_splits,
               long long ws_floats, int n_counters, bool allow_cluster, int force_bn, int force_splits,
               const void * q8_scales, int force_pair) {
    if (M % 128 || K_in % 64 || taps < 1 || S < 1 || nbatch < 1) return false;
    if (q8_scales && taps != 1) return false;
    GemmParams & p = L.p;
    p = GemmParams{};
    L.finalized = false;
    p.M = M; p.S = S; p.nbatch = nbatch; p.K_in = K_in; p.taps = taps; p.pad = pad;
    p.mblocks = M / 128;
    p.gate_div = 1;
    const int nkb = taps * (K_in / 64);
    {
        // the model's best choice, or the requested one if it is among the feasible choices
        // the same choice as for bf16 weights (the Q8_0 path must sum in the same order)
        const auto c = tile_choices(S, nbatch, p.mblocks, nkb, num_sms, max_splits, ws_floats, n_counters, allow_cluster,
                                    q8_scales == nullptr && force_pair != 0, K_in % 128 == 0, false);
        if (c.empty()) return false;
        TileChoice t = c[0];
        if (force_pair < 0 && getenv("TSD_FORCE_PAIR")) force_pair = 1;   // tests: exercise the pair form
        if (force_pair == 1)          // the model's best pair choice
            for (const TileChoice & x : c)
                if (x.pair) { t = x; break; }
        if (force_bn <= 0 && getenv("TSD_FORCE_MULTI_ITEM"))   // tests: the best multi-item choice (a pair
            for (const TileChoice & x : c)                    // one with TSD_FORCE_PAIR), if any
                if (x.ipt > 1 && (force_pair != 1 || x.pair)) { t = x; break; }
        for (const TileChoice & x : c)
            if (force_bn > 0 && x.BN == force_bn && x.splits == force_splits && (force_pair < 0 || x.pair == force_pair)) {
                t = x;
                break;
            }
        p.BN = t.BN;
        p.ipt = t.ipt;
        p.bni = t.ipt > 1 ? item_rows(S) : t.BN;
        p.n_tiles = t.ipt > 1 ? 1 : (S + t.BN - 1) / t.BN;
        p.groups = (nbatch + t.ipt - 1) / t.ipt;
        p.splits = t.splits;
        p.pair = t.pair;
        p.a_q8 = q8_scales != nullptr;
        // two K blocks per stage when K allows (no stage straddles a conv tap), each split keeps
        // whole stages, and at least 3 stages fit; else one
        const int b_atom = (p.pair ? p.BN / 2 : p.BN) * 128;
        const int st2 = kStageArea / (2 * (kABytes + b_atom));
        p.kpb = (!p.a_q8 && K_in % 128 == 0 && st2 >= 3 && nkb % (2 * p.splits) == 0 && nkb / (2 * p.splits) >= 2) ? 2 : 1;
        p.stages = std::min(kMaxStages, kStageArea / (p.kpb * (kABytes + b_atom) + (p.a_q8 ? kQ8Bytes : 0)));
    }
    if (getenv("TSD_DEBUG_PLAN")) {
        fprintf(stderr, "tsd plan: M=%d K=%d taps=%d nbatch=%d S=%d -> BN=%d tiles/item=%d items/tile=%d splits=%d pair=%d kpb=%d stages=%d | max active clusters",
                M, K_in, taps, nbatch, S, p.BN, p.n_tiles, p.ipt, p.splits, p.pair, p.kpb, p.stages);
        for (int k = 2; k <= 8; ++k) fprintf(stderr, " %d:%d", k, max_active_clusters(k));
        fprintf(stderr, "\n");
    }
    p.m_valid = swiglu ? M / 2 : M;
    {
        const char * o = getenv("TSD_TILE_ORDER");
        p.order = (o && *o == '1') ? 1 : 0;
    }
    const long long tiles = (long long)p.mblocks * p.groups * p.n_tiles * p.splits;   // CTA tiles
    const int cpt = p.pair ? 2 : 1;
    // one wave of split tiles: the splits of an output tile run as one cluster (rank = split,
    // which m-block-major order makes consecutive; pairs: rank = 2 * split + half)
    {
        const int rows_max = 16 * (((p.BN >> 4) + p.splits - 1) / p.splits);
        const int mac = p.splits > 1 && cpt * p.splits <= 8 ? max_active_clusters(cpt * p.splits) : 0;
        p.csplit = allow_cluster && cluster_split_enabled() && p.splits > 1 && tiles <= num_sms && mac > 0 &&
                   (long long)(p.mblocks / cpt) * p.groups * p.n_tiles <= mac &&
                   (long long)p.BN * 512 + (long long)(p.splits - 1) * rows_max * 512 <= (long long)kStageArea;
    }
    if (p.csplit || p.pair) p.order = 0;
    {
        long long g = std::min<long long>(tiles, num_sms);
        if (p.pair && !p.csplit) g = std::min<long long>(g, 2ll * max_active_clusters(2)) & ~1ll;   // whole pairs, co-resident
        L.grid = dim3((unsigned)g, 1, 1);
    }
    // workspace split-K with one tile per CTA: the last split gathers the partials (gather_split_ok)
    p.gather = p.splits > 1 && !p.csplit && !p.pair && tiles <= (long long)L.grid.x && gather_split_ok(p.BN, p.splits);
    if (q8_scales) {
        // int8 plane: 64 x 128 boxes (64-byte rows, no swizzle); scales: 128 rows x 2 blocks
        if (!make_tmap_2d(&L.tmA, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)K_in, (uint64_t)M, (uint64_t)K_in, 64,
                          128) ||
            !make_tmap_2d(&L.tmS, q8_scales, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (uint64_t)M, (uint64_t)K_in / 32,
                          (uint64_t)M * 2, 128, 2))
            return false;
    } else if (!make_tmap_3d(&L.tmA, W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 64, (uint64_t)M, (uint64_t)nkb,
                             (uint64_t)taps * K_in * 2, 128, 64, 128, (uint32_t)p.kpb))
        return false;   // weights as [K atom][row][64]: one box = kpb atoms of 128 rows
    {
        // activations as [item][K atom][token][64]: one box = kpb atoms of the B tile's tokens
        const uint64_t d[4] = {64, (uint64_t)S, (uint64_t)(K_in / 64), (uint64_t)nbatch};
        const uint64_t st[3] = {(uint64_t)x_row_stride * 2, 128, (uint64_t)x_batch_stride * 2};
        // (a multi-item tile: one K atom of bni rows of each of this CTA's items per box)
        const int mi_items = p.ipt > 1 ? (p.pair ? p.ipt / 2 : p.ipt) : 1;
        const uint32_t box[4] = {64, (uint32_t)(p.ipt > 1 ? p.bni : p.pair ? p.BN / 2 : p.BN),
                                 (uint32_t)(p.ipt > 1 ? 1 : p.kpb), (uint32_t)mi_items};
        if (!make_tmap_4d(&L.tmB, X, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, d, st, box, true)) return false;
    }
    return true;
}

static bool make_tmap_4d(CUtensorMap * m, const void * ptr, CUtensorMapDataType dt, int esize, const uint64_t (&d)[4],
                         const uint64_t (&stride_bytes)[3], const uint32_t (&box)[4], bool sw128) {
    auto fn = encode_fn();
    if (!fn || (reinterpret_cast<uintptr_t>(ptr) & 15) || (box[0] * esize) % 16) return false;
    for (int i = 0; i < 3; ++i)
        if (stride_bytes[i] % 16 || stride_bytes[i] >= (1ull << 40)) return false;
    cuuint64_t dims[4] = {d[0], d[1], d[2], d[3]};
    cuuint64_t strides[3] = {stride_bytes[0], stride_bytes[1], stride_bytes[2]};
    cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
    cuuint32_t es[4] = {1, 1, 1, 1};
    return fn(m, dt, 4, const_cast<void *>(ptr), dims, strides, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              sw128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

void gemm_finalize(GemmLaunch & L) {
    GemmParams & p = L.p;
    const auto al = [](const void * q, unsigned a) { return (reinterpret_cast<uintptr_t>(q) & (a - 1)) == 0; };
    // vector accesses in the split-K reducer (4 consecutive features; 2 for SwiGLU), if aligned
    const int nv = p.mode == EPI_SWIGLU ? 2 : 4;
    const unsigned ob = (unsigned)nv * (p.out_bf16 ? 2u : 4u);
    p.vec = p.mode == EPI_GATE_RESID
                ? (al(p.resid, 16) && al(p.gate, 16) && p.ldr % 4 == 0 && p.ldg % 4 == 0)
                : (al(p.out, ob) && p.ldo % nv == 0 && (p.out_cblk == 0 || (p.out_cblk % nv == 0 && p.out_cstride % nv == 0)));
    // TMA epilogue: output (or residual / gate) as [features][S][nbatch][column blocks]; boxes of
    // 128 (SwiGLU 64) features x 16 tokens. Tokens past S and features past m_valid are clipped.
    p.epi_tma = 0;
    const uint64_t S = (uint64_t)p.S, nb = (uint64_t)p.nbatch;
    if (p.mode == EPI_QKV) {
        // the stream's rows of Q / K / V: [item][head][token < s_item][64] fp16, token stride 64,
        // head stride Sj * 64, item stride nh * Sj * 64, based at token s_off
        const uint64_t d[4] = {64, (uint64_t)p.s_item, (uint64_t)p.nh, nb};
        const uint64_t st[3] = {128, (uint64_t)p.Sj * 128, (uint64_t)p.nh * p.Sj * 128};
        const uint32_t box[4] = {64, 16, 1, 1};
        const long long off = (long long)p.s_off * 64;
        p.epi_tma = p.nbatch * p.S == p.nbatch * p.s_item &&
                    make_tmap_4d(&L.tmO, p.q_out + off, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, d, st, box, false) &&
                    make_tmap_4d(&L.tmG, p.k_out + off, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, d, st, box, false) &&
                    make_tmap_4d(&L.tmV, p.v_out + off, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, d, st, box, false);
    } else if (p.mode == EPI_GATE_RESID) {
        const bool gtile = p.gate_div == 1;
        {
            const uint64_t d[4] = {(uint64_t)p.m_valid, S, nb, 1};
            const uint64_t sr[3] = {(uint64_t)p.ldr * 4, S * p.ldr * 4, S * nb * p.ldr * 4};
            const uint64_t sg[3] = {(uint64_t)p.ldg * 4, S * p.ldg * 4, S * nb * p.ldg * 4};
            const uint32_t box[4] = {128, 16, 1, 1};
            p.epi_tma = make_tmap_4d(&L.tmO, p.resid, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, d, sr, box, false) &&
                        (!gtile || make_tmap_4d(&L.tmG, p.gate, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, d, sg, box, false));
        }
    } else {
        const int es = p.out_bf16 ? 2 : 4;
        const uint32_t fw = p.mode == EPI_SWIGLU ? 64 : 128;
        const CUtensorMapDataType dt = p.out_bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
        const uint32_t box[4] = {fw, 16, 1, 1};
        if (p.out_cblk == 0) {
            const uint64_t d[4] = {(uint64_t)p.m_valid, S, nb, 1};
            const uint64_t st[3] = {(uint64_t)p.ldo * es, S * p.ldo * es, S * nb * p.ldo * es};
            p.epi_tma = make_tmap_4d(&L.tmO, p.out, dt, es, d, st, box, false);
        } else if (p.out_cblk % fw == 0 && p.m_valid % p.out_cblk == 0) {
            const uint64_t d[4] = {(uint64_t)p.out_cblk, S, nb, (uint64_t)(p.m_valid / p.out_cblk)};
            const uint64_t st[3] = {(uint64_t)p.ldo * es, S * p.ldo * es, (uint64_t)p.out_cstride * es};
            p.epi_tma = make_tmap_4d(&L.tmO, p.out, dt, es, d, st, box, false);
        }
    }
    if (getenv("TSD_NO_TMA_EPILOGUE")) p.epi_tma = 0;
    L.finalized = true;
}

namespace {
template <int EK, bool PAIR, int FORM>
cudaError_t launch_form(cudaLaunchConfig_t & cfg, const GemmLaunch & L, const GemmParams & p) {
    static bool attr = false;   // per instance
    if (!attr) {
        cudaError_t e =
            cudaFuncSetAttribute(gemm_tc_kernel<EK, PAIR, FORM>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<EK, PAIR, FORM>, L.tmA, L.tmB, L.tmO, L.tmG, L.tmV, L.tmS, p);
}
template <int EK> cudaError_t launch_kind(cudaLaunchConfig_t & cfg, const GemmLaunch & L, const GemmParams & p) {
    // (Q8_0 weights never pair; pairs split K only inside a cluster; multi-item tiles never split)
    if (!p.epi_tma && (p.splits == 1 || p.gather)) {   // whole tiles through plain stores
        const int f = 32 | (p.ipt > 1 ? 1 : 0) | (p.gather ? 2 : 0) | (p.a_q8 ? 4 : 0);
        switch (f) {
            case 32: return p.pair ? launch_form<EK, true, 32>(cfg, L, p) : launch_form<EK, false, 32>(cfg, L, p);
            case 33: return p.pair ? launch_form<EK, true, 33>(cfg, L, p) : launch_form<EK, false, 33>(cfg, L, p);
            case 34: return launch_form<EK, false, 34>(cfg, L, p);
            case 36: return launch_form<EK, false, 36>(cfg, L, p);
            case 37: return launch_form<EK, false, 37>(cfg, L, p);
            default: return launch_form<EK, false, 38>(cfg, L, p);
        }
    }
    if (p.a_q8) {
        if (p.ipt > 1) return launch_form<EK, false, 5>(cfg, L, p);
        if (p.splits > 1)
            return p.csplit ? launch_form<EK, false, 12>(cfg, L, p)
                            : p.gather ? launch_form<EK, false, 6>(cfg, L, p) : launch_form<EK, false, 20>(cfg, L, p);
        return launch_form<EK, false, 4>(cfg, L, p);
    }
    if (p.ipt > 1) return p.pair ? launch_form<EK, true, 1>(cfg, L, p) : launch_form<EK, false, 1>(cfg, L, p);
    if (p.splits > 1) {
        if (p.csplit) return p.pair ? launch_form<EK, true, 8>(cfg, L, p) : launch_form<EK, false, 8>(cfg, L, p);
        return p.gather ? launch_form<EK, false, 2>(cfg, L, p) : launch_form<EK, false, 16>(cfg, L, p);
    }
    return p.pair ? launch_form<EK, true, 0>(cfg, L, p) : launch_form<EK, false, 0>(cfg, L, p);
}
}  // namespace

cudaError_t gemm_launch(const GemmLaunch & L0, cudaStream_t st) {
    GemmLaunch Lf;
    if (!L0.finalized) { Lf = L0; gemm_finalize(Lf); }
    const GemmLaunch & L = L0.finalized ? L0 : Lf;
    const GemmParams & p = L.p;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = L.grid;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    int na = 0;
    if (pdl_enabled()) {
        at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (p.csplit || p.pair) {
        at[na].id = cudaLaunchAttributeClusterDimension;
        at[na].val.clusterDim.x = (unsigned)((p.pair ? 2 : 1) * (p.csplit ? p.splits : 1));
        at[na].val.clusterDim.y = 1;
        at[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = at;
    cfg.numAttrs = na;
    if (p.mode == EPI_QKV && p.splits != 1) return cudaErrorInvalidValue;
    switch (p.mode) {
        case EPI_QKV: return launch_kind<EK_QKV>(cfg, L, p);
        case EPI_GATE_RESID: return launch_kind<EK_GATE>(cfg, L, p);
        case EPI_SWIGLU: return p.out_bf16 ? launch_kind<EK_SWIGLU_BF16>(cfg, L, p) : launch_kind<EK_SWIGLU_F32>(cfg, L, p);
        default:
            if (p.act == ACT_SILU) return p.out_bf16 ? launch_kind<EK_BF16_SILU>(cfg, L, p) : launch_kind<EK_F32_SILU>(cfg, L, p);
            return p.out_bf16 ? launch_kind<EK_BF16>(cfg, L, p) : launch_kind<EK_F32>(cfg, L, p);
    }
}

}  // namespace tsd
