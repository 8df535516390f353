// gemv.cu — weight-streaming GEMV for the few-token projections (sm_100a, CUDA cores).
//
// The reference runs these as ggml_mul_mat with a single column (src/mmdit.cpp:158-160
// t_embed, :185-192 text/clip cond projections and global_cond_mlp, :209 adaLN of the clip and
// text streams, whose conditioning is the [H,1] global_c). With N = B (a handful of tokens)
// they are bound by reading the weights once from HBM, so they use CUDA cores and read the
// weights in their stored ggml type: F32, BF16, or Q8_0 blocks (fp16 scale + 32 int8), which
// are dequantised in registers. One warp per output feature; the x rows come from L1/L2.
#include "common.cuh"
#include "kernels.h"

namespace tsd {

namespace {

constexpr int kMaxN = 8;

__device__ __forceinline__ float rnd_bf16(float v, int r) { return r ? __bfloat162float(__float2bfloat16_rn(v)) : v; }

// Accumulate one 8-element chunk [k, k+8) of row w for all tokens.
template <int WT>
__device__ __forceinline__ void load_w8(const void * W, long long row, int K, int k, float (&w)[8]) {
    if constexpr (WT == 30) {   // BF16
        const uint4 u = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(W) + row * K + k);
        const __nv_bfloat162 * h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) { float2 f = __bfloat1622float2(h[i]); w[2 * i] = f.x; w[2 * i + 1] = f.y; }
    } else if constexpr (WT == 0) {  // F32
        const float4 * p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(W) + row * K + k);
        const float4 a = p[0], b = p[1];
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
    } else {                          // Q8_0: block of 32 = 2-byte fp16 scale + 32 int8
        const uint8_t * blk = reinterpret_cast<const uint8_t *>(W) + (row * (K / 32) + k / 32) * 34;
        const float d = __half2float(*reinterpret_cast<const __half *>(blk));
        const int off = 2 + (k & 31);
        // 8 int8 at a 2-byte-aligned address: four 16-bit loads.
        const uint16_t * q16 = reinterpret_cast<const uint16_t *>(blk + off);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint16_t v = q16[i];
            w[2 * i] = (float)(int8_t)(v & 0xff) * d;
            w[2 * i + 1] = (float)(int8_t)(v >> 8) * d;
        }
    }
}

template <int WT, bool kDual>
__global__ void __launch_bounds__(256)
gemv_kernel(const void * __restrict__ W, const void * __restrict__ W2, int M, int K, const float * __restrict__ x,
            long long ldx, int N, const float * __restrict__ bias, int act, int round_bf16, void * y, int y_bf16,
            long long ldy) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m = blockIdx.x * 8 + warp;
    if (m >= M) return;
    float acc[kMaxN], acc2[kMaxN];
#pragma unroll
    for (int n = 0; n < kMaxN; ++n) { acc[n] = 0.f; acc2[n] = 0.f; }
    for (int k = lane * 8; k < K; k += 256) {
        float w[8], w2[8];
        load_w8<WT>(W, m, K, k, w);
        if constexpr (kDual) load_w8<WT>(W2, m, K, k, w2);
#pragma unroll
        for (int n = 0; n < kMaxN; ++n) {
            if (n >= N) break;
            const float4 * xp = reinterpret_cast<const float4 *>(x + n * ldx + k);
            const float4 a = xp[0], b = xp[1];
            const float xv[8] = {rnd_bf16(a.x, round_bf16), rnd_bf16(a.y, round_bf16), rnd_bf16(a.z, round_bf16),
                                 rnd_bf16(a.w, round_bf16), rnd_bf16(b.x, round_bf16), rnd_bf16(b.y, round_bf16),
                                 rnd_bf16(b.z, round_bf16), rnd_bf16(b.w, round_bf16)};
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                acc[n] = fmaf(w[i], xv[i], acc[n]);
                if constexpr (kDual) acc2[n] = fmaf(w2[i], xv[i], acc2[n]);
            }
        }
    }
#pragma unroll
    for (int n = 0; n < kMaxN; ++n) {
        if (n >= N) break;
        float a = acc[n], a2 = acc2[n];
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            a += __shfl_xor_sync(0xffffffffu, a, o);
            if constexpr (kDual) a2 += __shfl_xor_sync(0xffffffffu, a2, o);
        }
        if (lane == 0) {
            float v;
            if constexpr (kDual) v = silu_f(a) * a2;
            else {
                v = a + (bias ? bias[m] : 0.f);
                if (act == ACT_SILU) v = silu_f(v);
            }
            if (y_bf16) reinterpret_cast<__nv_bfloat16 *>(y)[n * ldy + m] = __float2bfloat16_rn(v);
            else reinterpret_cast<float *>(y)[n * ldy + m] = v;
        }
    }
}

template <int WT>
cudaError_t launch_wt(const void * W, const void * W2, int M, int K, const float * x, long long ldx, int N,
                      const float * bias, int act, int round_bf16, void * y, int y_bf16, long long ldy, cudaStream_t st) {
    dim3 grid((M + 7) / 8);
    if (W2) launch_pdl(gemv_kernel<WT, true>, dim3(grid), dim3(256), 0, st, W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy);
    else launch_pdl(gemv_kernel<WT, false>, dim3(grid), dim3(256), 0, st, W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy);
    return cudaGetLastError();
}

}  // namespace

cudaError_t gemv_launch(const void * W, int wtype, const void * W2, int M, int K, const float * x, long long ldx, int N,
                        const float * bias, int act, int round_bf16, void * y, int y_bf16, long long ldy,
                        cudaStream_t st, int * /*err: these kernels have no waits*/) {
    if (N < 1 || N > kMaxN || K % 32 || (ldx & 3)) return cudaErrorInvalidValue;
    switch (wtype) {
        case 0: return launch_wt<0>(W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy, st);
        case 30: return launch_wt<30>(W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy, st);
        case 8: return launch_wt<8>(W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace tsd
