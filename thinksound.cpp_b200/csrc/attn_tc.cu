// attn_tc.cu — tcgen05 flash attention for the MM-DiT joint and fused blocks (sm_100a).
//
// Replaces the reference's `attention` (src/mmdit.cpp:85-94): softmax(Q K^T / sqrt(64)) V per
// head with no mask, K and V in F16 (:89-90) and F32 softmax/accumulation
// (ggml_flash_attn_ext_set_prec F32, :92). Q, K, V arrive fp16 head-major
// [B*nh][S][64]; for the joint blocks S is the [latent | clip | text] concatenation
// (:251-254), which the QKV producers write in place, so no concat/split copies exist.
//
// One CTA per (128-query tile, batch*head), two CTAs per SM: each takes 256 TMEM columns (S
// 0-127, O 128-191, P 192-255) and ~84 KB of shared memory (Q, a 2-stage K / V ring), so one
// CTA's softmax overlaps the other's MMAs and a joint layer's 192 CTAs run as one wave.
// Warp 0: TMA (Q once, 128-row K and V chunks). Warp 1: TMEM owner + MMA issuer: S_j = Q K_j^T
// (M=128, N=128) into the S columns, then, once the softmax has read S_j, S_{j+1} while the
// softmax of chunk j runs, and O += P_j V_j with P_j taken from tensor memory as the MMA's A
// operand (V an MN-major shared-memory operand). Warps 2-9: online softmax, two warps per TMEM
// lane quadrant: a query row (TMEM lane) is shared by two threads, each taking 64 of a chunk's
// 128 key columns. Only the chunk max is exchanged (once per chunk, through shared memory); each
// half keeps its own running sum under the common max and the two are added at the end. P_j
// goes to tensor memory as fp16 pairs (tcgen05.st), never through shared memory. The running max
// is updated lazily: while a chunk's max stays within 2^8 of it, the stale max is kept (P <= 256,
// exact in the final O / l), so O is rescaled in TMEM (32 of its 64 columns per half) only when
// the max jumps; the final 1/l scale and the token-major store out[b][t][h*64 + d] are split the
// same way.
#include "common.cuh"
#include "kernels.h"

namespace tsd {

namespace {

constexpr int kQT = 128, kKV = 128, kHD = 64, kStages = 2;
constexpr int kTileBytes = 128 * 128;               // 128 rows x 64 fp16
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTileBytes;            // [kStages]
constexpr int kOffV = kOffK + kStages * kTileBytes;  // [kStages]
constexpr int kOffRed = kOffV + kStages * kTileBytes;   // [3][2 halves][128 rows] f32: maxima (2 parities), sums
constexpr int kOffBar = kOffRed + 3 * 2 * 128 * 4;
constexpr int kSmemBytes = kOffBar + 256 + 1024;
constexpr int kThreads = 320;                        // warps: 0 TMA, 1 MMA, 2-9 softmax
constexpr uint32_t kTmemCols = 256;                  // two CTAs per SM share the 512 columns
constexpr uint32_t kColO = 128, kColP = 192;
constexpr float kLazyMax = 8.0f;                     // log2 of the largest P kept under a stale max

struct AttnArgs {
    int S, nh;
    long long ldo;
    void * out;            // bf16, or f32 when out_f32
    int * err;
    float scale_log2;
    int out_f32;
};

__device__ __forceinline__ void soft_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__global__ void __launch_bounds__(kThreads, 2)
attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, const AttnArgs a) {
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t * bars = reinterpret_cast<uint64_t *>(smem + kOffBar);
    uint64_t * q_full = bars + 0;
    uint64_t * kv_full = bars + 1;          // [2]
    uint64_t * kv_empty = bars + 3;         // [2]
    uint64_t * s_full = bars + 5;           // S_j in TMEM
    uint64_t * s_free = bars + 6;           // the softmax has read S_j (256 arrivals)
    uint64_t * p_full = bars + 7;           // P_j in TMEM (256 arrivals)
    uint64_t * pv_done = bars + 8;          // O += P_j V_j complete (P and O may be touched again)
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(bars + 9);
    volatile int * s_abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * kQT;
    const int bh = blockIdx.y;
    const int S = a.S;
    const int nchunks = (S + kKV - 1) / kKV;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < kStages; ++s) { mbar_init(&kv_full[s], 1); mbar_init(&kv_empty[s], 1); }
        mbar_init(s_full, 1);
        mbar_init(s_free, 256);
        mbar_init(p_full, 256);
        mbar_init(pv_done, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) { tma_prefetch(&tmQ); tma_prefetch(&tmK); tma_prefetch(&tmV); }
    if (warp == 1) { tmem_alloc(tmem_slot, kTmemCols); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();   // launched with PDL: the Q / K / V writers have finished after this

    if (warp == 0) {
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, kTileBytes);
            tma_load_3d(smem + kOffQ, &tmQ, q_full, 0, q0, bh);
            int issued = 0;
            for (int j = 0; j < nchunks; ++j, ++issued) {
                const int s = j % kStages;
                if (j >= kStages && !mbar_wait(&kv_empty[s], ((j / kStages) & 1) ^ 1, s_abort, a.err, DEV_TIMEOUT_ATTN))
                    break;
                mbar_arrive_expect_tx(&kv_full[s], 2 * kTileBytes);
                tma_load_3d(smem + kOffK + s * kTileBytes, &tmK, &kv_full[s], 0, j * kKV, bh);
                tma_load_3d(smem + kOffV + s * kTileBytes, &tmV, &kv_full[s], 0, j * kKV, bh);
            }
            if (*s_abort) {   // let the copies still in flight land before the CTA exits
                const unsigned long long t0 = globaltimer();
                while (!mbar_try_wait(q_full, 0) && globaltimer() - t0 < wait_ns()) {}
                for (int i = (issued > kStages ? issued - kStages : 0); i < issued; ++i) {
                    const unsigned long long t1 = globaltimer();
                    while (!mbar_try_wait(&kv_full[i % kStages], (i / kStages) & 1) && globaltimer() - t1 < wait_ns()) {}
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc_s = make_idesc_f16(128, kKV, false, false);
            const uint32_t idesc_o = make_idesc_f16(128, kHD, false, true);
            const uint64_t qd = make_sdesc_sw128(smem_u32(smem + kOffQ));
            bool ok = mbar_wait(q_full, 0, s_abort, a.err, DEV_TIMEOUT_ATTN);
            const auto issue_s = [&](int j) -> bool {
                const int s = j % kStages;
                if (!mbar_wait(&kv_full[s], (j / kStages) & 1, s_abort, a.err, DEV_TIMEOUT_ATTN)) return false;
                tc_fence_after();
                const uint64_t kd = make_sdesc_sw128(smem_u32(smem + kOffK + s * kTileBytes));
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) umma_f16_ss(tmem, qd + 2 * kk, kd + 2 * kk, idesc_s, kk > 0);
                umma_commit(s_full);
                return true;
            };
            if (ok) ok = issue_s(0);
            for (int j = 0; ok && j < nchunks; ++j) {
                // S_{j+1} once the softmax has read S_j (it then overlaps the softmax of chunk j)
                if (j + 1 < nchunks) {
                    if (!mbar_wait(s_free, j & 1, s_abort, a.err, DEV_TIMEOUT_ATTN) || !issue_s(j + 1)) { ok = false; break; }
                }
                if (!mbar_wait(p_full, j & 1, s_abort, a.err, DEV_TIMEOUT_ATTN)) { ok = false; break; }
                tc_fence_after();
                const uint32_t vb = smem_u32(smem + kOffV + (j % kStages) * kTileBytes);
#pragma unroll
                for (int kk = 0; kk < 8; ++kk)
                    umma_f16_ts(tmem + kColO, tmem + kColP + 8 * kk, make_sdesc_sw128(vb + kk * 2048), idesc_o,
                                (j > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&kv_empty[j % kStages]);
                umma_commit(pv_done);
            }
            if (!ok) { umma_commit(s_full); umma_commit(pv_done); }   // no waiter depends on unissued MMAs
        }
    } else {
        // ---------------- softmax + epilogue (warps 2..9) ----------------
        const int q = warp & 3;
        const int half = (warp - 2) >> 2;             // key columns half * 64 .. + 63 of each chunk
        const int r = q * 32 + lane;                   // query row within the tile (TMEM lane)
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
        float * red = reinterpret_cast<float *>(smem + kOffRed);
        float m_run = -INFINITY, l_run = 0.f;
        // A failed (timed-out) wait leaves `ok` false for the whole warp; the warp still takes every
        // named barrier below (one per chunk and one at the end), so the other seven never block.
        // The waits carry no shared abort flag: each warp gives up only on its own deadline.
        bool ok = true;
        for (int j = 0; j < nchunks; ++j) {
            const int valid = S - j * kKV - half * 64;   // columns >= valid are padding keys
            float mx = -INFINITY;
            uint32_t w[32];                            // columns 32-63 of this half, kept from pass 1
            if (ok) ok = __all_sync(0xffffffffu, mbar_wait(s_full, j & 1, nullptr, a.err, DEV_TIMEOUT_ATTN));
            if (ok) {
                tc_fence_after();
                // pass 1: the row max of this half's 64 scores (masking only in the ragged last chunk)
                float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
                uint32_t u[32];
                tmem_ld32_async(lane_base + half * 64, u);
                tmem_ld32_async(lane_base + half * 64 + 32, w);
                tmem_wait_ld(u);
                tmem_wait_ld(w);
                if (valid >= 64) {
#pragma unroll
                    for (int i = 0; i < 32; ++i)
                        m4[i & 3] = max3(m4[i & 3], __uint_as_float(u[i]), __uint_as_float(w[i]));
                } else {
#pragma unroll
                    for (int i = 0; i < 32; ++i) {
                        if (i < valid) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(u[i]));
                        if (32 + i < valid) m4[(i + 2) & 3] = fmaxf(m4[(i + 2) & 3], __uint_as_float(w[i]));
                    }
                }
                mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * a.scale_log2;
            }
            float * rm = red + ((j & 1) * 2) * 128;     // this chunk's maxima [half][row]
            rm[half * 128 + r] = mx;
            soft_bar();
            if (!ok) continue;
            const float mc = fmaxf(mx, rm[(half ^ 1) * 128 + r]);   // chunk max of the row (both halves)
            // both halves of a row hold the same m_run and mc, so they take the same branch
            const bool grow = mc > m_run + kLazyMax;
            const float m_new = grow ? mc : m_run;
            const float alpha = grow ? ex2_approx(m_run - m_new) : 1.0f;   // 0 on the first chunk
            if (j > 0) {
                // PV_{j-1} must be done with P (rewritten below) and O (rescaled here)
                ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (j - 1) & 1, nullptr, a.err, DEV_TIMEOUT_ATTN));
                if (!ok) continue;
                tc_fence_after();
                if (__any_sync(0xffffffffu, grow)) {   // rows that keep their max scale by 1
#pragma unroll
                    for (int c0 = 0; c0 < 32; c0 += 16) {  // 16 columns at a time: few live registers
                        float o[16];
                        tmem_ld16(lane_base + kColO + half * 32 + c0, o);
#pragma unroll
                        for (int i = 0; i < 16; ++i) o[i] *= alpha;
                        tmem_st16(lane_base + kColO + half * 32 + c0, o);
                    }
                }
            }
            // pass 2: P = 2^(s * scale - m), fp16 pairs (key 2c in the low half) into the P columns;
            // one exponential in four on the FMA pipes (exp2_poly), the rest on the SFU
            float2 r01 = make_float2(0.f, 0.f), r23 = make_float2(0.f, 0.f);   // partial row sums
            const float nm = -m_new;
            const float2 sc2 = make_float2(a.scale_log2, a.scale_log2), nm2 = make_float2(nm, nm);
            {
                // columns 0-31 are read again (the last read of S_j: S_{j+1} may then overwrite it,
                // and runs while the exponentials below are computed); columns 32-63 are in w
                uint32_t u[32];
                tmem_ld32_async(lane_base + half * 64, u);
                tmem_wait_ld(u);
                tc_fence_before();
                mbar_arrive(s_free);
                const auto piece = [&](const uint32_t (&v)[32], int c0) {
                    const int vlim = valid - c0;       // columns >= vlim of this piece are padding keys
#pragma unroll
                    for (int c1 = 0; c1 < 32; c1 += 16) {
                        uint32_t pk[8];
#pragma unroll
                        for (int c = 0; c < 8; ++c) {
                            const int i0 = c1 + 2 * c;
                            // s * scale - m for the column pair (one packed FMA)
                            float2 x = fma2(make_float2(__uint_as_float(v[i0]), __uint_as_float(v[i0 + 1])), sc2, nm2);
                            if (vlim < 32) {           // only in the ragged last chunk
                                if (i0 >= vlim) x.x = -INFINITY;
                                if (i0 + 1 >= vlim) x.y = -INFINITY;
                            }
                            const float p0 = ex2_approx(x.x);
                            const float p1 = (i0 & 2) ? exp2_poly(x.y) : ex2_approx(x.y);
                            if (c & 1) r23 = add2(r23, make_float2(p0, p1));
                            else r01 = add2(r01, make_float2(p0, p1));
                            const __half2 h2 = __floats2half2_rn(p0, p1);
                            pk[c] = *reinterpret_cast<const uint32_t *>(&h2);
                        }
                        tmem_st8_u(lane_base + kColP + half * 32 + (c0 + c1) / 2, pk);
                    }
                };
                piece(u, 0);
                piece(w, 32);
            }
            l_run = l_run * alpha + ((r01.x + r01.y) + (r23.x + r23.y));
            m_run = m_new;
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(p_full);
        }
        const int jl = nchunks - 1;
        const bool fin = ok && __all_sync(0xffffffffu, mbar_wait(pv_done, jl & 1, nullptr, a.err, DEV_TIMEOUT_ATTN));
        // both halves' sums under the common max
        float * rl = red + 4 * 128;
        rl[half * 128 + r] = l_run;
        soft_bar();
        if (fin) {
            const float inv = 1.0f / (l_run + rl[(half ^ 1) * 128 + r]);
            tc_fence_after();
            const int t = q0 + r;
            const int b = bh / a.nh, h = bh % a.nh;
            float o[32];
            tmem_ld32(lane_base + kColO + half * 32, o);
            if (t < S && a.out_f32) {
                float * dst = reinterpret_cast<float *>(a.out) + ((long long)b * S + t) * a.ldo + h * kHD + half * 32;
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    *reinterpret_cast<float4 *>(dst + e * 4) =
                        make_float4(o[e * 4] * inv, o[e * 4 + 1] * inv, o[e * 4 + 2] * inv, o[e * 4 + 3] * inv);
            } else if (t < S) {
                __nv_bfloat16 * dst = reinterpret_cast<__nv_bfloat16 *>(a.out) + ((long long)b * S + t) * a.ldo + h * kHD + half * 32;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    uint4 u4;
                    __nv_bfloat162 * p2 = reinterpret_cast<__nv_bfloat162 *>(&u4);
#pragma unroll
                    for (int i = 0; i < 4; ++i) p2[i] = __floats2bfloat162_rn(o[e * 8 + 2 * i] * inv, o[e * 8 + 2 * i + 1] * inv);
                    *reinterpret_cast<uint4 *>(dst + e * 8) = u4;
                }
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

}  // namespace

bool attn_plan(AttnLaunch & L, const void * Q, const void * K, const void * V, int B, int nh, int S, void * out,
               long long ldo, int * err, bool out_f32) {
    if (S < 1 || B < 1 || nh < 1 || (ldo % 8) || (reinterpret_cast<uintptr_t>(out) & 15)) return false;
    L.out_f32 = out_f32;
    const uint64_t rows = S, heads = (uint64_t)B * nh;
    bool ok = make_tmap_3d(&L.tmQ, Q, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kHD, rows, heads, kHD * 2, rows * kHD * 2, kHD, kQT, 1) &&
              make_tmap_3d(&L.tmK, K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kHD, rows, heads, kHD * 2, rows * kHD * 2, kHD, kKV, 1) &&
              make_tmap_3d(&L.tmV, V, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, kHD, rows, heads, kHD * 2, rows * kHD * 2, kHD, kKV, 1);
    L.S = S; L.nh = nh; L.B = B; L.ldo = ldo; L.out = out; L.err = err;
    L.scale = 1.0f / 8.0f;
    return ok;
}

cudaError_t attn_launch(const AttnLaunch & L, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
        // all of the SM's unified L1 / shared storage as shared memory: two CTAs per SM
        cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
        attr = true;
    }
    AttnArgs a;
    a.S = L.S; a.nh = L.nh; a.ldo = L.ldo; a.out = L.out; a.err = L.err; a.out_f32 = L.out_f32 ? 1 : 0;
    a.scale_log2 = L.scale * 1.4426950408889634f;
    dim3 grid((L.S + kQT - 1) / kQT, L.B * L.nh);
    launch_pdl(attn_tc_kernel, dim3(grid), dim3(kThreads), kSmemBytes, st, L.tmQ, L.tmK, L.tmV, a);
    return cudaGetLastError();
}

}  // namespace tsd
