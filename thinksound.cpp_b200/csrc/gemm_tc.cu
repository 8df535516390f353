// gemm_tc.cu — tcgen05 / TMEM / TMA GEMM for the MM-DiT projections (sm_100a).
//
// Replaces the reference's ggml_mul_mat (src/mmdit.cpp:12-16 `lin`) and the im2col+mul_mat
// convolution (`conv1d_f32`, :20-25): a conv with k taps is an implicit GEMM whose K loop runs
// over (tap, input-feature block) and whose activation tile for tap k is the token window
// shifted by k - pad (TMA zero-fills rows outside the batch item, which is the conv padding).
// The adaLN gate + residual add (:231, :234) and SwiGLU (:42-43, :50-51) are fused into the
// epilogue, so no separate elementwise kernel touches HBM for them.
//
// CTA = 6 warps: warp 0 issues TMA, warp 1 owns TMEM and issues tcgen05.mma (one elected
// thread), warps 2-5 run the epilogue (one TMEM lane quadrant each; thread = output feature).
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cstdio>

namespace tsd {

namespace {

constexpr int kABytes = 128 * 128;          // 128 rows x 64 bf16
constexpr int kBBytesMax = 256 * 128;       // 256 tokens x 64 bf16
template <int kNumA> struct GemmCfg {
    static constexpr int kStages = kNumA == 1 ? 4 : 3;
    static constexpr int kStageBytes = kNumA * kABytes + kBBytesMax;
    static constexpr int kTmemCols = kNumA == 1 ? 256 : 512;
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 256 /*barriers*/;
};

template <int kNumA>
__global__ void __launch_bounds__(192, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
    using C = GemmCfg<kNumA>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t * full = reinterpret_cast<uint64_t *>(smem + C::kStages * C::kStageBytes);
    uint64_t * empty = full + C::kStages;
    uint64_t * acc_full = empty + C::kStages;
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
    volatile int * s_abort = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int mb = blockIdx.x;
    const int b = blockIdx.y / p.n_tiles, tile = blockIdx.y % p.n_tiles;
    const int t0 = tile * p.BN;
    const int kpt = p.K_in >> 6;
    const int nkb = p.taps * kpt;
    const int split = blockIdx.z;
    const int kb_begin = (int)((long long)nkb * split / p.splits);
    const int kb_end = (int)((long long)nkb * (split + 1) / p.splits);
    const uint32_t tx_bytes = (uint32_t)(kNumA * kABytes + p.BN * 128);

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(acc_full, 1);
        *s_abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) { tma_prefetch(&tmA); tma_prefetch(&tmB); }
    if (warp == 1) { tmem_alloc(tmem_slot, C::kTmemCols); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int issued = 0;
            for (int kb = kb_begin; kb < kb_end; ++kb, ++issued) {
                const int s = issued % C::kStages;
                if (issued >= C::kStages &&
                    !mbar_wait(&empty[s], ((issued / C::kStages) & 1) ^ 1, s_abort, p.err, DEV_TIMEOUT_EMPTY))
                    break;
                uint8_t * sa = smem + s * C::kStageBytes;
                uint8_t * sb = sa + kNumA * kABytes;
                const int tap = kb / kpt, kc = kb - tap * kpt;
                mbar_arrive_expect_tx(&full[s], tx_bytes);
                tma_load_2d(sa, &tmA, &full[s], kb * 64, mb * 128 * kNumA);
                tma_load_3d(sb, &tmB, &full[s], kc * 64, t0 + tap - p.pad, b);
            }
            if (*s_abort) {
                // Let the copies still in flight land before the CTA exits.
                for (int i = (issued > C::kStages ? issued - C::kStages : 0); i < issued; ++i) {
                    const int s = i % C::kStages;
                    const unsigned long long t_start = globaltimer();
                    while (!mbar_try_wait(&full[s], (i / C::kStages) & 1) && globaltimer() - t_start < kWaitNs) {}
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            const uint32_t idesc = make_idesc_f16(128, p.BN, true);
            int i = 0;
            for (int kb = kb_begin; kb < kb_end; ++kb, ++i) {
                const int s = i % C::kStages;
                if (!mbar_wait(&full[s], (i / C::kStages) & 1, s_abort, p.err, DEV_TIMEOUT_FULL)) break;
                tc_fence_after();
                const uint32_t sa = smem_u32(smem + s * C::kStageBytes);
                const uint64_t bdesc = make_sdesc_sw128(sa + kNumA * kABytes);
#pragma unroll
                for (int a = 0; a < kNumA; ++a) {
                    const uint64_t adesc = make_sdesc_sw128(sa + a * kABytes);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma_f16_ss(tmem + a * 256, adesc + 2 * kk, bdesc + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(acc_full);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;                       // TMEM lane quadrant of this warp
        const int m = mb * 128 + q * 32 + lane;       // output feature of this thread
        // warp-uniform outcome: tcgen05.ld below is warp-collective
        if (__all_sync(0xffffffffu, mbar_wait(acc_full, 0, s_abort, p.err, DEV_TIMEOUT_ACC))) {
            tc_fence_after();
            const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
            const bool m_ok = m < p.m_valid;
            const float bias = (p.bias && m_ok && (p.mode != EPI_GATE_RESID || split == 0)) ? p.bias[m] : 0.f;
            const int ncols = min(p.BN, p.S - t0);
            for (int j0 = 0; j0 < p.BN; j0 += 32) {
                float v[32];
                tmem_ld32(trow + j0, v);
                if (p.mode == EPI_SWIGLU) {
                    float v3[32];
                    tmem_ld32(trow + 256 + j0, v3);
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = silu_f(v[j]) * v3[j];
                }
                if (!m_ok) continue;
#pragma unroll 4
                for (int j = 0; j < 32; ++j) {
                    const int jj = j0 + j;
                    if (jj >= ncols) break;
                    const long long row = (long long)b * p.S + t0 + jj;
                    if (p.mode == EPI_GATE_RESID) {
                        const float g = p.gate[(row / p.gate_div) * p.ldg + m];
                        float * dst = p.resid + row * p.ldr + m;
                        const float val = g * (v[j] + bias);
                        if (p.splits > 1) atomicAdd(dst, val);
                        else *dst += val;
                    } else {
                        float val = v[j] + bias;
                        if (p.act == ACT_SILU) val = silu_f(val);
                        if (p.out_bf16) reinterpret_cast<__nv_bfloat16 *>(p.out)[row * p.ldo + m] = __float2bfloat16_rn(val);
                        else reinterpret_cast<float *>(p.out)[row * p.ldo + m] = val;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, C::kTmemCols);
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

template <int kNumA> void set_smem_attr() {
    static bool done = false;
    if (!done) {
        cudaFuncSetAttribute(gemm_tc_kernel<kNumA>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<kNumA>::kSmemBytes);
        done = true;
    }
}

}  // namespace

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

// Token-tile choice: fewest tiles of <= 256 tokens, then split further while the grid covers
// less than one wave of SMs (a smaller tile re-reads weights from L2, not HBM).
static void choose_tiles(int S, int nbatch, int mblocks, int num_sms, int & BN, int & n_tiles) {
    n_tiles = (S + 255) / 256;
    BN = ((S + n_tiles - 1) / n_tiles + 15) / 16 * 16;
    while ((long long)mblocks * nbatch * n_tiles < (long long)num_sms * 9 / 10 && BN > 48) {
        const int nt = n_tiles + 1;
        const int bn = ((S + nt - 1) / nt + 15) / 16 * 16;
        if (bn >= BN) break;
        n_tiles = nt;
        BN = bn;
    }
    n_tiles = (S + BN - 1) / BN;
}

bool gemm_plan(GemmLaunch & L, const void * W, int M, int K_in, int taps, int pad, int numA, const void * X, int nbatch,
               int S, long long x_row_stride, long long x_batch_stride, int num_sms, int max_splits) {
    if (M % (128 * numA) || K_in % 64 || taps < 1 || S < 1 || nbatch < 1 || (numA != 1 && numA != 2)) return false;
    GemmParams & p = L.p;
    p = GemmParams{};
    p.M = M; p.S = S; p.nbatch = nbatch; p.K_in = K_in; p.taps = taps; p.pad = pad;
    const int mblocks = M / (128 * numA);
    choose_tiles(S, nbatch, mblocks, num_sms, p.BN, p.n_tiles);
    const int nkb = taps * (K_in / 64);
    p.splits = 1;
    const long long ctas = (long long)mblocks * nbatch * p.n_tiles;
    if (max_splits > 1 && ctas < num_sms * 3 / 4) {
        int s = (int)std::min<long long>(max_splits, (num_sms + ctas - 1) / ctas);
        s = std::min(s, nkb / 8);
        p.splits = std::max(1, s);
    }
    p.m_valid = M;
    L.numA = numA;
    L.grid = dim3(mblocks, nbatch * p.n_tiles, p.splits);
    if (!make_tmap_2d(&L.tmA, W, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)taps * K_in, (uint64_t)M,
                      (uint64_t)taps * K_in * 2, 64, 128 * numA))
        return false;
    if (!make_tmap_3d(&L.tmB, X, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)K_in, (uint64_t)S, (uint64_t)nbatch,
                      (uint64_t)x_row_stride * 2, (uint64_t)x_batch_stride * 2, 64, p.BN, 1))
        return false;
    return true;
}

cudaError_t gemm_launch(const GemmLaunch & L, cudaStream_t st) {
    if (L.numA == 1) {
        set_smem_attr<1>();
        gemm_tc_kernel<1><<<L.grid, 192, GemmCfg<1>::kSmemBytes, st>>>(L.tmA, L.tmB, L.p);
    } else {
        set_smem_attr<2>();
        gemm_tc_kernel<2><<<L.grid, 192, GemmCfg<2>::kSmemBytes, st>>>(L.tmA, L.tmB, L.p);
    }
    return cudaGetLastError();
}

}  // namespace tsd
