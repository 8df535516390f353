// gemv.cu — weight-streaming GEMV for the few-token projections (sm_100a, CUDA cores).
//
// The reference runs these as ggml_mul_mat with a single column (src/mmdit.cpp:158-160
// t_embed, :185-192 text/clip cond projections and global_cond_mlp, :209 adaLN of the clip and
// text streams, whose conditioning is the [H,1] global_c). With N = B (a handful of tokens)
// they are bound by reading the weights once from HBM, so they use CUDA cores and read the
// weights in their stored ggml type: F32, BF16, or Q8_0 blocks (fp16 scale + 32 int8), which
// are decoded on the fly. Warps own output features; the x rows come from L1/L2.
#include "common.cuh"
#include "kernels.h"

namespace tsd {

namespace {

constexpr int kMaxN = 8;

// bf16 round-to-nearest-even of a finite f32 in integer ops (the conversion instruction issues
// on the narrow conversion pipe, and this runs for every x value a chunk reads).
__device__ __forceinline__ float rne_bf16(float v) {
    const uint32_t u = __float_as_uint(v);
    return __uint_as_float((u + 0x7fffu + ((u >> 16) & 1u)) & 0xffff0000u);
}

// Four int8 of a 32-bit word as exact f32 without the conversion pipe: byte b becomes the f32
// whose bits are 0x4B0000 | (b ^ 0x80), i.e. 2^23 + 128 + b, and 2^23 + 128 is subtracted.
__device__ __forceinline__ void s8x4_to_f32(uint32_t w, float * f) {
    const uint32_t x = w ^ 0x80808080u;
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7650u + i)) - 8388736.0f;
}

// Weights of one 8-weight chunk as f32 (Q8_0: the integer values, scale in *d).
__device__ __forceinline__ void bf16x8_to_f32(const uint4 & u, float (&w)[8]) {
    const uint32_t v[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) { w[2 * i] = __uint_as_float(v[i] << 16); w[2 * i + 1] = __uint_as_float(v[i] & 0xffff0000u); }
}
__device__ __forceinline__ void q8_chunk(const uint8_t * blk, int sub, float (&w)[8], float & d) {
    // blk: a 34-byte Q8_0 block (2-byte aligned); sub: which 8 of its 32 values
    d = __half2float(*reinterpret_cast<const __half *>(blk));
    const uint16_t * q16 = reinterpret_cast<const uint16_t *>(blk + 2 + sub * 8);
    s8x4_to_f32((uint32_t)q16[0] | ((uint32_t)q16[1] << 16), w);
    s8x4_to_f32((uint32_t)q16[2] | ((uint32_t)q16[3] << 16), w + 4);
}

// x[n][k .. k+8) as f32, rounded to bf16 when the weights are BF16 (GGML's mul_mat converts
// the activations to the weights' vec-dot type).
__device__ __forceinline__ void load_x8(const float * x, int round, float (&xv)[8]) {
    const float4 a = reinterpret_cast<const float4 *>(x)[0], b = reinterpret_cast<const float4 *>(x)[1];
    xv[0] = a.x; xv[1] = a.y; xv[2] = a.z; xv[3] = a.w; xv[4] = b.x; xv[5] = b.y; xv[6] = b.z; xv[7] = b.w;
    if (round) {
#pragma unroll
        for (int i = 0; i < 8; ++i) xv[i] = rne_bf16(xv[i]);
    }
}

// acc += w . xv over one chunk. Q8_0 sums q_i * x_i and applies the block scale once per chunk.
template <int WT>
__device__ __forceinline__ float chunk_dot(const float (&w)[8], float d, const float (&xv)[8], float acc) {
    if constexpr (WT == 8) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) s = fmaf(w[i], xv[i], s);
        return fmaf(d, s, acc);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) acc = fmaf(w[i], xv[i], acc);
        return acc;
    }
}

// Weights of chunk [k, k+8) of row `row`, read directly from global memory (per-chunk form).
template <int WT>
__device__ __forceinline__ void load_w8(const void * W, long long row, int K, int k, float (&w)[8], float & d) {
    if constexpr (WT == 30) {
        bf16x8_to_f32(*reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(W) + row * K + k), w);
        d = 1.f;
    } else if constexpr (WT == 0) {
        const float4 * p = reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(W) + row * K + k);
        const float4 a = p[0], b = p[1];
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w; w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
        d = 1.f;
    } else {
        q8_chunk(reinterpret_cast<const uint8_t *>(W) + (row * (K / 32) + k / 32) * 34, (k & 31) >> 3, w, d);
    }
}

__device__ __forceinline__ void store_out(float a, float a2, bool dual, int m, int n, const float * bias, int act,
                                          void * y, int y_bf16, long long ldy) {
    float v;
    if (dual) v = silu_f(a) * a2;
    else {
        v = a + (bias ? bias[m] : 0.f);
        if (act == ACT_SILU) v = silu_f(v);
    }
    if (y_bf16) reinterpret_cast<__nv_bfloat16 *>(y)[n * ldy + m] = __float2bfloat16_rn(v);
    else reinterpret_cast<float *>(y)[n * ldy + m] = v;
}

// Per-chunk form: one warp per output row, each lane walks its chunks (lane + 32 j) and waits
// for each chunk's loads before the next. Used when K % 256 != 0 or an operand is not 16-byte
// aligned; it sums in the same order as the streaming form below.
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
        float w[8], w2[8], d, d2 = 1.f;
        load_w8<WT>(W, m, K, k, w, d);
        if constexpr (kDual) load_w8<WT>(W2, m, K, k, w2, d2);
#pragma unroll
        for (int n = 0; n < kMaxN; ++n) {
            if (n >= N) break;
            float xv[8];
            load_x8(x + n * ldx + k, round_bf16, xv);
            acc[n] = chunk_dot<WT>(w, d, xv, acc[n]);
            if constexpr (kDual) acc2[n] = chunk_dot<WT>(w2, d2, xv, acc2[n]);
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
        if (lane == 0) store_out(a, a2, kDual, m, n, bias, act, y, y_bf16, ldy);
    }
}

// ---------------------------------------------------------------------------------------------
// Streaming form (K % 256 == 0, 16-byte-aligned operands). A warp owns R rows and issues every
// 16-byte load of a phase of those rows (1024 weights: 2 KB BF16, 1088 B Q8_0; 512 F32 weights)
// before the first FMA, so several KB per warp are in flight; the x values of a chunk are loaded
// and rounded once for all R rows. Q8_0 rows are 16-byte aligned when K % 256 == 0 (K/32 * 34
// bytes), so a phase is read as plain 16-byte words, parked in the warp's shared-memory slot and
// decoded there (34-byte blocks straddle the words). A lane owns the same chunks (lane + 32 j)
// in the same order as in gemv_kernel, so both forms give bit-identical sums.
constexpr int kStreamWarps = 4;

template <int WT>
struct StreamPhase {
    static constexpr int kWeights = WT == 0 ? 512 : 1024;     // weights of a row per phase
    static constexpr int kChunks = kWeights / 256;             // 8-weight chunks per lane per phase
    static constexpr int kBytes = WT == 8 ? kWeights / 32 * 34 : kWeights * (WT == 0 ? 4 : 2);
    static constexpr int kU4 = (kBytes / 16 + 31) / 32;        // 16-byte loads per lane per phase
};

template <int WT>
__device__ __forceinline__ void stream_load(const void * W, long long row, int K, int k0, int nchunk, int lane,
                                            uint4 (&raw)[StreamPhase<WT>::kU4]) {
    const uint8_t * base = reinterpret_cast<const uint8_t *>(W) +
                           (WT == 8 ? (row * (K / 32) + k0 / 32) * 34 : (row * K + k0) * (WT == 0 ? 4 : 2));
    const uint4 * p = reinterpret_cast<const uint4 *>(base);
    if constexpr (WT == 0) {   // F32: a chunk is two words, kept together in raw[2j], raw[2j+1]
#pragma unroll
        for (int j = 0; j < StreamPhase<WT>::kChunks; ++j)
            if (lane + 32 * j < nchunk) {
                raw[2 * j] = __ldg(p + 2 * (lane + 32 * j));
                raw[2 * j + 1] = __ldg(p + 2 * (lane + 32 * j) + 1);
            }
    } else {                   // BF16: word = chunk; Q8_0: the phase's bytes in order
        const int n16 = WT == 8 ? nchunk / 4 * 34 / 16 : nchunk;
#pragma unroll
        for (int j = 0; j < StreamPhase<WT>::kU4; ++j)
            if (lane + 32 * j < n16) raw[j] = __ldg(p + lane + 32 * j);
    }
}

// Phase-local chunk j of this lane from the staged words (BF16 / F32: registers; Q8_0: the slot).
template <int WT>
__device__ __forceinline__ void stream_chunk(const uint4 (&raw)[StreamPhase<WT>::kU4], const uint8_t * slot, int lane,
                                             int j, float (&w)[8], float & d) {
    if constexpr (WT == 30) {
        bf16x8_to_f32(raw[j], w);
        d = 1.f;
    } else if constexpr (WT == 0) {
        const float * f = reinterpret_cast<const float *>(&raw[2 * j]);
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = f[i];
        d = 1.f;
    } else {
        const int c = lane + 32 * j;
        q8_chunk(slot + (c >> 2) * 34, c & 3, w, d);
    }
}

template <int WT, bool kDual, int NMAX, int R>
__global__ void __launch_bounds__(kStreamWarps * 32)
gemv_stream_kernel(const void * __restrict__ W, const void * __restrict__ W2, int M, int K, const float * __restrict__ x,
                   long long ldx, int N, const float * __restrict__ bias, int act, int round_bf16, void * y, int y_bf16,
                   long long ldy) {
    using PH = StreamPhase<WT>;
    constexpr int kSlots = R * (kDual ? 2 : 1);            // staged row phases per warp (Q8_0)
    __shared__ __align__(16) uint8_t q8s[WT == 8 ? kStreamWarps * kSlots : 1][WT == 8 ? PH::kBytes : 16];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = (blockIdx.x * kStreamWarps + warp) * R;
    long long rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) rows[r] = min(m0 + r, M - 1);   // a tail warp re-reads row M-1 (not stored)
    // The weights are constant: the first phase is requested before waiting for the previous
    // kernel (launched with PDL), so its DRAM latency overlaps that kernel's tail.
    uint4 raw[R][PH::kU4], raw2[R][PH::kU4];
    const int nchunk0 = min(PH::kWeights, K) / 8;
    if (m0 < M) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            stream_load<WT>(W, rows[r], K, 0, nchunk0, lane, raw[r]);
            if constexpr (kDual) stream_load<WT>(W2, rows[r], K, 0, nchunk0, lane, raw2[r]);
        }
    }
    pdl_wait();
    pdl_launch_dependents();
    if (m0 >= M) return;   // whole warps only: the __syncwarp()s below stay warp-uniform
    float acc[R][NMAX], acc2[R][NMAX];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int n = 0; n < NMAX; ++n) { acc[r][n] = 0.f; acc2[r][n] = 0.f; }
    for (int k0 = 0; k0 < K; k0 += PH::kWeights) {
        const int nchunk = min(PH::kWeights, K - k0) / 8;   // a multiple of 32
        if (k0 > 0) {
#pragma unroll
            for (int r = 0; r < R; ++r) {
                stream_load<WT>(W, rows[r], K, k0, nchunk, lane, raw[r]);
                if constexpr (kDual) stream_load<WT>(W2, rows[r], K, k0, nchunk, lane, raw2[r]);
            }
        }
        if constexpr (WT == 8) {
            const int n16 = nchunk / 4 * 34 / 16;
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int j = 0; j < PH::kU4; ++j)
                    if (lane + 32 * j < n16) {
                        reinterpret_cast<uint4 *>(q8s[warp * kSlots + r])[lane + 32 * j] = raw[r][j];
                        if constexpr (kDual) reinterpret_cast<uint4 *>(q8s[warp * kSlots + R + r])[lane + 32 * j] = raw2[r][j];
                    }
            __syncwarp();
        }
#pragma unroll
        for (int j = 0; j < PH::kChunks; ++j) {
            if (lane + 32 * j >= nchunk) break;   // nchunk % 32 == 0: uniform across the warp
            const int k = k0 + 8 * (lane + 32 * j);
            float w[R][8], w2[R][8], d[R], d2[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                stream_chunk<WT>(raw[r], q8s[WT == 8 ? warp * kSlots + r : 0], lane, j, w[r], d[r]);
                if constexpr (kDual) stream_chunk<WT>(raw2[r], q8s[WT == 8 ? warp * kSlots + R + r : 0], lane, j, w2[r], d2[r]);
            }
#pragma unroll
            for (int n = 0; n < NMAX; ++n) {
                if (n >= N) break;
                float xv[8];
                load_x8(x + n * ldx + k, round_bf16, xv);
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    acc[r][n] = chunk_dot<WT>(w[r], d[r], xv, acc[r][n]);
                    if constexpr (kDual) acc2[r][n] = chunk_dot<WT>(w2[r], d2[r], xv, acc2[r][n]);
                }
            }
        }
        if constexpr (WT == 8) __syncwarp();   // the slots are rewritten by the next phase
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int n = 0; n < NMAX; ++n) {
            if (n >= N) break;
            float a = acc[r][n], a2 = acc2[r][n];
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                a += __shfl_xor_sync(0xffffffffu, a, o);
                if constexpr (kDual) a2 += __shfl_xor_sync(0xffffffffu, a2, o);
            }
            if (lane == 0 && m0 + r < M) store_out(a, a2, kDual, m0 + r, n, bias, act, y, y_bf16, ldy);
        }
}

template <int WT, bool kDual, int R>
void launch_stream(const void * W, const void * W2, int M, int K, const float * x, long long ldx, int N,
                   const float * bias, int act, int round_bf16, void * y, int y_bf16, long long ldy, cudaStream_t st) {
    const dim3 grid((M + kStreamWarps * R - 1) / (kStreamWarps * R)), block(kStreamWarps * 32);
    if (N <= 2)
        launch_pdl(gemv_stream_kernel<WT, kDual, 2, R>, grid, block, 0, st, W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy);
    else
        launch_pdl(gemv_stream_kernel<WT, kDual, kMaxN, R>, grid, block, 0, st, W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy);
}

template <int WT>
cudaError_t launch_wt(const void * W, const void * W2, int M, int K, const float * x, long long ldx, int N,
                      const float * bias, int act, int round_bf16, void * y, int y_bf16, long long ldy, cudaStream_t st) {
    const bool aligned = (reinterpret_cast<uintptr_t>(W) & 15) == 0 && (reinterpret_cast<uintptr_t>(W2) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    if (K % 256 == 0 && aligned) {
        if (W2) launch_stream<WT, true, 1>(W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy, st);
        else launch_stream<WT, false, 2>(W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy, st);
    } else {
        const dim3 grid((M + 7) / 8);
        if (W2) launch_pdl(gemv_kernel<WT, true>, grid, dim3(256), 0, st, W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy);
        else launch_pdl(gemv_kernel<WT, false>, grid, dim3(256), 0, st, W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t gemv_launch(const void * W, int wtype, const void * W2, int M, int K, const float * x, long long ldx, int N,
                        const float * bias, int act, int round_bf16, void * y, int y_bf16, long long ldy,
                        cudaStream_t st, int * /*err: these kernels have no waits*/) {
    if (N < 1 || N > kMaxN || K % 32 || (ldx & 3)) return cudaErrorInvalidValue;
    // x rows and BF16 / F32 weights are read as 16-byte words, Q8_0 blocks as 2-byte halves
    const uintptr_t wa = wtype == 8 ? 1 : 15;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(W) & wa) ||
        (reinterpret_cast<uintptr_t>(W2) & wa))
        return cudaErrorInvalidValue;
    switch (wtype) {
        case 0: return launch_wt<0>(W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy, st);
        case 30: return launch_wt<30>(W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy, st);
        case 8: return launch_wt<8>(W, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy, st);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace tsd
