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
// split), m-block-major so CTAs running at the same time share weight tiles through L2. Warp 0
// issues TMA into a 4-stage ring, warp 1 owns TMEM and issues tcgen05.mma into one of two
// 256-column accumulators, warps 2-5 drain the other accumulator (thread = output feature)
// while the next tile accumulates. SwiGLU weights are interleaved in 64-row blocks (w1 rows,
// then the matching w3 rows), so a tile holds h1 in TMEM lanes 0-63 and h3 in lanes 64-127;
// the epilogue pairs them through shared memory. Launched with programmatic dependent launch:
// weight tiles of the first stages are requested before the kernel waits for the activations
// its predecessor writes.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>

namespace tsd {

namespace {

constexpr int kStages = 4;
constexpr int kABytes = 128 * 128;          // 128 rows x 64 bf16
constexpr int kBBytesMax = 256 * 128;       // 256 tokens x 64 bf16
constexpr int kStageBytes = kABytes + kBBytesMax;
constexpr int kXStride = 33;                // SwiGLU exchange row stride (floats), conflict-free
constexpr int kXBytes = 64 * kXStride * 4;
constexpr int kTmemCols = 512;              // two 256-column fp32 accumulators
constexpr int kSmemBytes = kStages * kStageBytes + kXBytes + 1024 /*align*/ + 256 /*barriers*/;

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

struct TileCoord { int mb, b, t0, kb_begin, kb_end, split, otile; };

// Tile t -> (m-block, batch item, first token, K range). Consecutive t share the m-block.
__device__ __forceinline__ TileCoord decode(const GemmParams & p, int t, int nkb) {
    TileCoord c;
    int nt;
    if (p.order == 0) {           // m-block-major: consecutive tiles share the weight tile
        const int per_mb = p.nbatch * p.n_tiles * p.splits;
        c.mb = t / per_mb;
        const int rem = t - c.mb * per_mb;
        nt = rem / p.splits;
        c.split = rem - nt * p.splits;
    } else {                      // token-tile-major: consecutive tiles share the activation tile
        c.mb = t % p.mblocks;
        const int r = t / p.mblocks;
        const int ntt = p.nbatch * p.n_tiles;
        nt = r % ntt;
        c.split = r / ntt;
    }
    c.b = nt / p.n_tiles;
    c.t0 = (nt - c.b * p.n_tiles) * p.BN;
    c.otile = c.mb * (p.nbatch * p.n_tiles) + nt;     // output tile (all K splits of it)
    c.kb_begin = (int)((long long)nkb * c.split / p.splits);
    c.kb_end = (int)((long long)nkb * (c.split + 1) / p.splits);
    return c;
}

struct EpiCtx {
    int m;               // output feature of this thread
    bool m_ok;           // m is stored by this thread
    float bias;
    int ncols;           // valid token columns of the tile
    long long row_base;  // output row of the tile's first token
    long long col;       // output column offset of feature m (after column blocking)
};

// Epilogue of one 32-column chunk of final accumulator values v (thread = feature e.m).
// Fully unrolled and predicated so v[] stays in registers (a partially unrolled loop with an
// early exit made the compiler spill it to local memory).
__device__ __forceinline__ void emit_chunk(const GemmParams & p, const EpiCtx & e, int j0, float (&v)[32], float * xbuf,
                                           int q, int lane, bool swiglu) {
    if (swiglu) {
        if (q >= 2) {
#pragma unroll
            for (int j = 0; j < 32; ++j) xbuf[((q - 2) * 32 + lane) * kXStride + j] = v[j];
        }
        epi_bar();
        if (q < 2) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = silu_f(v[j]) * xbuf[(q * 32 + lane) * kXStride + j];
        }
        epi_bar();
    }
    if (!e.m_ok) return;
    const long long row0 = e.row_base + j0;
    const int ncols = e.ncols - j0;
    if (p.mode == EPI_GATE_RESID) {
        // All gate and residual loads of the chunk are issued before any store: with the
        // read-modify-write interleaved, possible aliasing serialised 32 memory round trips.
        float * dst = p.resid + row0 * p.ldr + e.m;
        const long long grow = row0 / p.gate_div;        // gate row of token row0
        int gpos = (int)(row0 - grow * p.gate_div);      // position inside that gate row
        const float * g = p.gate + grow * p.ldg + e.m;
        float gv[32], xv[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            gv[j] = 0.f; xv[j] = 0.f;
            if (j < ncols) { gv[j] = __ldg(g); xv[j] = dst[(long long)j * p.ldr]; }
            if (++gpos == p.gate_div) { gpos = 0; g += p.ldg; }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < ncols) dst[(long long)j * p.ldr] = xv[j] + gv[j] * (v[j] + e.bias);
    } else if (p.out_bf16) {
        __nv_bfloat16 * o = reinterpret_cast<__nv_bfloat16 *>(p.out) + row0 * p.ldo + e.col;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            float val = v[j] + e.bias;
            if (p.act == ACT_SILU) val = silu_f(val);
            if (j < ncols) o[(long long)j * p.ldo] = __float2bfloat16_rn(val);
        }
    } else {
        float * o = reinterpret_cast<float *>(p.out) + row0 * p.ldo + e.col;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            float val = v[j] + e.bias;
            if (p.act == ACT_SILU) val = silu_f(val);
            if (j < ncols) o[(long long)j * p.ldo] = val;
        }
    }
}

__global__ void __launch_bounds__(192, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float * xbuf = reinterpret_cast<float *>(smem + kStages * kStageBytes);
    uint64_t * full = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes + kXBytes);
    uint64_t * empty = full + kStages;
    uint64_t * acc_full = empty + kStages;     // [2]
    uint64_t * acc_empty = acc_full + 2;       // [2]
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    volatile int * s_abort = reinterpret_cast<volatile int *>(tmem_slot + 1);
    volatile int * s_last = s_abort + 1;       // split-K: this CTA reduces the tile

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kpt = p.K_in >> 6;
    const int nkb = p.taps * kpt;
    const int num_tiles = p.mblocks * p.nbatch * p.n_tiles * p.splits;
    const uint32_t tx_bytes = (uint32_t)(kABytes + p.BN * 128);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int s = 0; s < 2; ++s) { mbar_init(&acc_full[s], 1); mbar_init(&acc_empty[s], 4); }
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) { tma_prefetch(&tmA); tma_prefetch(&tmB); }
    if (warp == 1) { tmem_alloc(tmem_slot, kTmemCols); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_launch_dependents();

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            // Weight tiles of the first stages do not depend on earlier kernels: request them
            // before waiting for the predecessor grid; their activation tiles follow the wait.
            int pre = 0;
            for (int t = blockIdx.x; t < num_tiles && pre < kStages; t += gridDim.x) {
                const TileCoord c = decode(p, t, nkb);
                for (int kb = c.kb_begin; kb < c.kb_end && pre < kStages; ++kb, ++pre) {
                    mbar_arrive_expect_tx(&full[pre], tx_bytes);
                    tma_load_2d(smem + pre * kStageBytes, &tmA, &full[pre], kb * 64, c.mb * 128);
                }
            }
            pdl_wait();
            int it = 0;
            for (int t = blockIdx.x; t < num_tiles && !*s_abort; t += gridDim.x) {
                const TileCoord c = decode(p, t, nkb);
                for (int kb = c.kb_begin; kb < c.kb_end; ++kb, ++it) {
                    const int s = it % kStages;
                    uint8_t * sa = smem + s * kStageBytes;
                    const int tap = kb / kpt, kc = kb - tap * kpt;
                    if (it < pre) {       // A already requested
                        tma_load_3d(sa + kABytes, &tmB, &full[s], kc * 64, c.t0 + tap - p.pad, c.b);
                        continue;
                    }
                    if (it >= kStages &&
                        !mbar_wait(&empty[s], ((it / kStages) & 1) ^ 1, s_abort, p.err, DEV_TIMEOUT_EMPTY))
                        break;
                    mbar_arrive_expect_tx(&full[s], tx_bytes);
                    tma_load_2d(sa, &tmA, &full[s], kb * 64, c.mb * 128);
                    tma_load_3d(sa + kABytes, &tmB, &full[s], kc * 64, c.t0 + tap - p.pad, c.b);
                }
            }
            if (*s_abort) {
                // Let the copies still in flight land before the CTA exits.
                const int issued = it > pre ? it : pre;
                for (int i = (issued > kStages ? issued - kStages : 0); i < issued; ++i) {
                    const unsigned long long t_start = globaltimer();
                    while (!mbar_try_wait(&full[i % kStages], (i / kStages) & 1) && globaltimer() - t_start < kWaitNs) {}
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            const uint32_t idesc = make_idesc_f16(128, p.BN, true);
            int it = 0, lt = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < num_tiles; t += gridDim.x, ++lt) {
                const TileCoord c = decode(p, t, nkb);
                const int buf = lt & 1;
                if (lt >= 2 && !mbar_wait(&acc_empty[buf], ((lt >> 1) & 1) ^ 1, s_abort, p.err, DEV_TIMEOUT_ACC)) break;
                tc_fence_after();
                const uint32_t dacc = tmem + buf * 256;
                for (int kb = c.kb_begin; kb < c.kb_end; ++kb, ++it) {
                    const int s = it % kStages;
                    if (!mbar_wait(&full[s], (it / kStages) & 1, s_abort, p.err, DEV_TIMEOUT_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(smem + s * kStageBytes);
                    const uint64_t adesc = make_sdesc_sw128(sa);
                    const uint64_t bdesc = make_sdesc_sw128(sa + kABytes);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_f16_ss(dacc, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb > c.kb_begin || kk > 0) ? 1u : 0u);
                    umma_commit(&empty[s]);
                }
                umma_commit(&acc_full[buf]);
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        pdl_wait();
        const int q = warp & 3;                       // TMEM lane quadrant of this warp
        const int ml = q * 32 + lane;                 // TMEM lane = weight row within the tile
        const bool swiglu = p.mode == EPI_SWIGLU;
        int lt = 0;
        for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++lt) {
            const TileCoord c = decode(p, t, nkb);
            const int buf = lt & 1;
            // warp-uniform outcome: tcgen05.ld below is warp-collective
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[buf], (lt >> 1) & 1, s_abort, p.err, DEV_TIMEOUT_ACC)))
                break;
            tc_fence_after();
            const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + buf * 256;
            EpiCtx e;
            // output feature of this thread (SwiGLU: lanes 0-63 carry h1 of features mb*64 + lane)
            e.m = swiglu ? c.mb * 64 + ml : c.mb * 128 + ml;
            e.m_ok = swiglu ? (q < 2 && e.m < p.m_valid) : (e.m < p.m_valid);
            e.bias = (p.bias && e.m_ok && !swiglu) ? p.bias[e.m] : 0.f;
            e.ncols = min(p.BN, p.S - c.t0);
            e.row_base = (long long)c.b * p.S + c.t0;
            e.col = p.out_cblk ? (long long)(e.m / p.out_cblk) * p.out_cstride + e.m % p.out_cblk : e.m;
            if (p.splits == 1) {
                for (int j0 = 0; j0 < p.BN; j0 += 32) {
                    float v[32];
                    tmem_ld32(trow + j0, v);
                    emit_chunk(p, e, j0, v, xbuf, q, lane, swiglu);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[buf]);
            } else {
                // Split-K, deterministic: every split stores its partial tile; the CTA that
                // completes the tile last sums the partials in split order and runs the epilogue.
                float * wsp = p.ws + ((size_t)(c.otile * p.splits + c.split) * p.BN) * 128 + ml;
                for (int j0 = 0; j0 < p.BN; j0 += 32) {
                    float v[32];
                    tmem_ld32(trow + j0, v);
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j0 + j < p.BN) wsp[(size_t)(j0 + j) * 128] = v[j];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acc_empty[buf]);
                __threadfence();
                epi_bar();
                if (threadIdx.x == 64) *s_last = (atomicAdd(&p.counters[c.otile], 1) == p.splits - 1);
                epi_bar();
                if (*s_last) {
                    __threadfence();
                    const float * base = p.ws + (size_t)c.otile * p.splits * p.BN * 128 + ml;
                    for (int j0 = 0; j0 < p.BN; j0 += 32) {
                        float v[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = 0.f;
                        for (int s = 0; s < p.splits; ++s) {
                            const float * src = base + ((size_t)s * p.BN + j0) * 128;
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (j0 + j < p.BN) v[j] += src[(size_t)j * 128];
                        }
                        emit_chunk(p, e, j0, v, xbuf, q, lane, swiglu);
                    }
                    if (threadIdx.x == 64) p.counters[c.otile] = 0;   // ready for the next launch
                }
                epi_bar();   // every thread has read s_last before the next tile rewrites it
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
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

// Tile / split choice from a small cost model of one SM's work per K block of 64: MMA about
// 2*BN cycles, operand fill about (16 KB + 128 B * BN) / 96 B per cycle, whichever is larger,
// plus a fixed cost per tile wave (pipeline fill, last epilogue) and, for split-K, the partial
// tile round trip through the workspace. Split-K adds parallelism when there are fewer output
// tiles than SMs; ws_floats / n_counters bound it.
static void choose_tiles(int S, int nbatch, int mblocks, int nkb, int num_sms, int max_splits, long long ws_floats,
                         int n_counters, int & BN, int & n_tiles, int & splits) {
    double best = 1e30;
    BN = 16; n_tiles = (S + 15) / 16; splits = 1;
    for (int bn = 16; bn <= 256; bn += 16) {
        const int nt = (S + bn - 1) / bn;
        if (nt > 1 && ((S + nt - 1) / nt + 15) / 16 * 16 < bn) continue;   // a smaller bn gives the same count
        const long long otiles = (long long)mblocks * nbatch * nt;
        for (int sp = 1; sp <= std::max(1, max_splits); ++sp) {
            if (sp > 1 && (nkb / sp < 4 || otiles > n_counters || otiles * sp * bn * 128 > ws_floats)) break;
            const long long tiles = otiles * sp;
            const long long waves = (tiles + num_sms - 1) / num_sms;
            const double per_kb = std::max(2.0 * bn, (16384.0 + 128.0 * bn) / 96.0);
            const double reduce = sp > 1 ? (double)bn * 128 * 4 * (sp + 1) / 64.0 : 0.0;   // bytes / (B/cycle)
            const double cost = (double)waves * ((double)nkb / sp * per_kb + 2000.0 + reduce);
            if (cost < best - 1e-9) { best = cost; BN = bn; n_tiles = nt; splits = sp; }
        }
    }
}

long long gemm_ws_floats(const GemmLaunch & L) {
    const GemmParams & p = L.p;
    return p.splits > 1 ? (long long)p.mblocks * p.nbatch * p.n_tiles * p.splits * p.BN * 128 : 0;
}

bool gemm_plan(GemmLaunch & L, const void * W, int M, int K_in, int taps, int pad, int swiglu, const void * X,
               int nbatch, int S, long long x_row_stride, long long x_batch_stride, int num_sms, int max_splits,
               long long ws_floats, int n_counters) {
    if (M % 128 || K_in % 64 || taps < 1 || S < 1 || nbatch < 1) return false;
    GemmParams & p = L.p;
    p = GemmParams{};
    p.M = M; p.S = S; p.nbatch = nbatch; p.K_in = K_in; p.taps = taps; p.pad = pad;
    p.mblocks = M / 128;
    p.gate_div = 1;
    const int nkb = taps * (K_in / 64);
    choose_tiles(S, nbatch, p.mblocks, nkb, num_sms, max_splits, ws_floats, n_counters, p.BN, p.n_tiles, p.splits);
    p.m_valid = swiglu ? M / 2 : M;
    {
        const char * o = getenv("TSD_TILE_ORDER");
        p.order = (o && *o == '1') ? 1 : 0;
    }
    const long long tiles = (long long)p.mblocks * nbatch * p.n_tiles * p.splits;
    L.grid = dim3((unsigned)std::min<long long>(tiles, num_sms), 1, 1);
    if (!make_tmap_2d(&L.tmA, W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)taps * K_in, (uint64_t)M,
                      (uint64_t)taps * K_in * 2, 64, 128))
        return false;
    if (!make_tmap_3d(&L.tmB, X, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)K_in, (uint64_t)S, (uint64_t)nbatch,
                      (uint64_t)x_row_stride * 2, (uint64_t)x_batch_stride * 2, 64, p.BN, 1))
        return false;
    return true;
}

cudaError_t gemm_launch(const GemmLaunch & L, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = L.grid;
    cfg.blockDim = dim3(192, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemm_tc_kernel, L.tmA, L.tmB, L.p);
}

}  // namespace tsd
