// elementwise.cu — normalisation, RoPE and layout kernels of the MM-DiT forward (sm_100a).
//
// These replace the reference's non-GEMM GGML nodes (src/mmdit.cpp): ggml_norm + modulate
// (:55-59), split_qkv + rms_norm + rope + the F16 cast of K/V (:67-100), and the small
// pre-processing ops (:150-200: transposes, sync positional add, text pad/concat, timestep
// embedding :305-313, sequence mean, nearest-exact sync gather :319). Each is one pass over
// its tensor; all accumulate in f32.
#include "common.cuh"
#include "kernels.h"

namespace tsd {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One warp per row. Two-pass mean / variance (population), eps 1e-5, no affine.
// One CTA per row (token): each thread keeps up to kLnVec float4 of the row in registers, so x is
// read once; mean, then the sum of squared deviations (two passes over registers, as
// ggml_norm computes them), then LN(x) * (1 + scale) + shift written bf16.
constexpr int kLnVec = 4;
__device__ __forceinline__ float block_sum(float v, float * red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();                       // red[] free from a previous use
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t += red[i];
    return t;
}
__global__ void ln_modulate_kernel(const float * __restrict__ x, int rows, int H, const float * __restrict__ shift,
                                   const float * __restrict__ scale, long long ld_mod, int per_token, int rows_per_item,
                                   __nv_bfloat16 * __restrict__ y) {
    __shared__ float red[32];
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const int row = blockIdx.x;
    const int n4 = H >> 2;
    const float4 * xr = reinterpret_cast<const float4 *>(x + (long long)row * H);
    const long long mrow = per_token ? row : row / rows_per_item;
    const float4 * sh = reinterpret_cast<const float4 *>(shift + mrow * ld_mod);
    const float4 * sc = reinterpret_cast<const float4 *>(scale + mrow * ld_mod);
    float4 v[kLnVec], a[kLnVec], c[kLnVec];
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < kLnVec; ++k) {
        const int i = threadIdx.x + k * blockDim.x;
        if (i < n4) {
            v[k] = xr[i]; a[k] = sh[i]; c[k] = sc[i];
            s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
        }
    }
    const float mean = block_sum(s, red) / (float)H;
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < kLnVec; ++k) {
        const int i = threadIdx.x + k * blockDim.x;
        if (i < n4) {
            const float d0 = v[k].x - mean, d1 = v[k].y - mean, d2 = v[k].z - mean, d3 = v[k].w - mean;
            ss += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
        }
    }
    const float rstd = 1.0f / sqrtf(block_sum(ss, red) / (float)H + 1e-5f);
    __nv_bfloat162 * yr = reinterpret_cast<__nv_bfloat162 *>(y + (long long)row * H);
#pragma unroll
    for (int k = 0; k < kLnVec; ++k) {
        const int i = threadIdx.x + k * blockDim.x;
        if (i < n4) {
            const float o0 = ((v[k].x - mean) * rstd) * (c[k].x + 1.0f) + a[k].x;
            const float o1 = ((v[k].y - mean) * rstd) * (c[k].y + 1.0f) + a[k].y;
            const float o2 = ((v[k].z - mean) * rstd) * (c[k].z + 1.0f) + a[k].z;
            const float o3 = ((v[k].w - mean) * rstd) * (c[k].w + 1.0f) + a[k].w;
            yr[2 * i] = __floats2bfloat162_rn(o0, o1);
            yr[2 * i + 1] = __floats2bfloat162_rn(o2, o3);
        }
    }
}

// One warp per (item, token, head); lane owns dims 2*lane, 2*lane+1 (one RoPE pair).
__global__ void qk_norm_rope_kernel(const float * __restrict__ qkv, int B, int S, int H, int nh,
                                    const float * __restrict__ qg, const float * __restrict__ kg, int rope, float fscale,
                                    float theta, __half * __restrict__ Q, __half * __restrict__ K,
                                    __half * __restrict__ V, int Sj, int s_off) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= (long long)B * S * nh) return;
    const int h = (int)(w % nh);
    const long long bt = w / nh;
    const int t = (int)(bt % S), b = (int)(bt / S);
    const float * row = qkv + bt * 3LL * H + h * 64 + 2 * lane;
    float2 q = *reinterpret_cast<const float2 *>(row);
    float2 k = *reinterpret_cast<const float2 *>(row + H);
    const float2 v = *reinterpret_cast<const float2 *>(row + 2 * H);
    const float rq = 1.0f / sqrtf(warp_sum(q.x * q.x + q.y * q.y) / 64.0f + 1e-6f);
    const float rk = 1.0f / sqrtf(warp_sum(k.x * k.x + k.y * k.y) / 64.0f + 1e-6f);
    q.x = (q.x * rq) * qg[2 * lane]; q.y = (q.y * rq) * qg[2 * lane + 1];
    k.x = (k.x * rk) * kg[2 * lane]; k.y = (k.y * rk) * kg[2 * lane + 1];
    if (rope) {
        const float ang = fscale * ((float)t * powf(theta, -2.0f * (float)lane / 64.0f));
        float sn, cs;
        sincosf(ang, &sn, &cs);
        q = make_float2(q.x * cs - q.y * sn, q.x * sn + q.y * cs);
        k = make_float2(k.x * cs - k.y * sn, k.x * sn + k.y * cs);
    }
    const long long o = (((long long)b * nh + h) * Sj + s_off + t) * 64 + 2 * lane;
    *reinterpret_cast<__half2 *>(Q + o) = __floats2half2_rn(q.x, q.y);
    *reinterpret_cast<__half2 *>(K + o) = __floats2half2_rn(k.x, k.y);
    *reinterpret_cast<__half2 *>(V + o) = __floats2half2_rn(v.x, v.y);
}

// The angle expression of qk_norm_rope_kernel, tabulated once per plan for the QKV GEMM epilogue.
__global__ void rope_table_kernel(int S, float fscale, float theta, float2 * __restrict__ tab) {
    pdl_wait();                // launched with PDL: earlier kernels are done with `tab`
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= S * 32) return;
    const int t = i >> 5, p = i & 31;
    const float ang = fscale * ((float)t * powf(theta, -2.0f * (float)p / 64.0f));
    float sn, cs;
    sincosf(ang, &sn, &cs);
    tab[i] = make_float2(cs, sn);
}

__global__ void latent_to_tokens_kernel(const float * __restrict__ lat, int B, int C, int T, __nv_bfloat16 * __restrict__ y) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)B * C * T) return;
    const int c = (int)(i % C);
    const long long bt = i / C;
    const int t = (int)(bt % T), b = (int)(bt / T);
    y[i] = __float2bfloat16_rn(lat[((long long)b * C + c) * T + t]);
}

__global__ void sync_prep_kernel(const float * __restrict__ sync, int B, int S, int C, const float * __restrict__ pe,
                                 __nv_bfloat16 * __restrict__ y) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)B * S * C) return;
    const int c = (int)(i % C);
    const int s = (int)((i / C) % S);
    y[i] = __float2bfloat16_rn(sync[i] + pe[(s % 8) * C + c]);
}

__global__ void text_prep_kernel(const float * __restrict__ text, int text_S, int text_dim, const float * __restrict__ t5,
                                 int t5_S, int t5_dim, int B, __nv_bfloat16 * __restrict__ y) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const int St = text_S + t5_S;
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)B * St * t5_dim) return;
    const int c = (int)(i % t5_dim);
    const long long bs = i / t5_dim;
    const int s = (int)(bs % St), b = (int)(bs / St);
    float v;
    if (s < text_S) v = c < text_dim ? text[((long long)b * text_S + s) * text_dim + c] : 0.f;
    else v = t5[((long long)b * t5_S + (s - text_S)) * t5_dim + c];
    y[i] = __float2bfloat16_rn(v);
}

__global__ void timestep_embed_kernel(const float * __restrict__ t, int B, int H, float max_period, float * __restrict__ y) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int half = H / 2;
    if (i >= B * half) return;
    const int b = i / half, k = i % half;
    const float fr = (10000.0f / max_period) * powf(10000.0f, -2.0f * (float)k / (float)H);
    float sn, cs;
    sincosf(t[b] * fr, &sn, &cs);
    y[(long long)b * H + k] = cs;
    y[(long long)b * H + half + k] = sn;
}

__global__ void seq_mean_kernel(const float * __restrict__ x, int B, int S, int H, float * __restrict__ y) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * H) return;
    const int b = i / H, h = i % H;
    float s = 0.f;
    for (int t = 0; t < S; ++t) s += x[((long long)b * S + t) * H + h];
    y[i] = s / (float)S;
}

__global__ void add_vec_kernel(const float * a, const float * b, int n, float * y) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = a[i] + b[i];
}

__global__ void build_extended_kernel(const float * __restrict__ sync, int sync_S, const float * __restrict__ gc, int B,
                                      int T, int H, float * __restrict__ ext, __nv_bfloat16 * __restrict__ sext) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)B * T * H) return;
    const int h = (int)(i % H);
    const long long bt = i / H;
    const int t = (int)(bt % T), b = (int)(bt / T);
    const int si = (int)floorf(((float)t + 0.5f) * (float)sync_S / (float)T);
    const float v = sync[((long long)b * sync_S + si) * H + h] + gc[(long long)b * H + h];
    ext[i] = v;
    sext[i] = __float2bfloat16_rn(silu_f(v));
}

__global__ void silu_vec_kernel(const float * __restrict__ x, int n, float * __restrict__ y) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = silu_f(x[i]);
}

__global__ void cast_kernel(const float * __restrict__ x, long long n, __nv_bfloat16 * __restrict__ y) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __float2bfloat16_rn(x[i]);
}

__global__ void cfg_euler_kernel(const float * __restrict__ flow, int P, int T, int L, float cfg, float dt,
                                 float * __restrict__ x, float * __restrict__ flow0) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)P * L * T) return;
    const int t = (int)(i % T);
    const int c = (int)((i / T) % L);
    const int p = (int)(i / ((long long)T * L));
    const float fc = flow[(((long long)2 * p) * T + t) * L + c];
    const float fu = flow[(((long long)2 * p + 1) * T + t) * L + c];
    const float v = fu + (fc - fu) * cfg;
    if (flow0) flow0[i] = v;
    x[i] += dt * v;
}

__global__ void dup_latent_kernel(const float * __restrict__ x, int P, int L, int T, float * __restrict__ lat2) {
    pdl_wait();                // launched with PDL: the predecessor's writes are visible after this
    pdl_launch_dependents();   // let the next kernel in the stream start its prologue
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long per = (long long)L * T;
    if (i >= (long long)P * per) return;
    const long long p = i / per, r = i % per;
    lat2[(2 * p) * per + r] = x[i];
    lat2[(2 * p + 1) * per + r] = x[i];
}

inline unsigned nblk(long long n, int bs) { return (unsigned)((n + bs - 1) / bs); }

}  // namespace

cudaError_t ln_modulate(const float * x, int rows, int H, const float * shift, const float * scale, long long ld_mod,
                        int per_token, int rows_per_item, __nv_bfloat16 * y, cudaStream_t st) {
    if (H % 4 || (ld_mod % 4)) return cudaErrorInvalidValue;
    // threads: the row's float4 count spread over at most kLnVec per thread, whole warps, <= 1024
    const int n4 = H / 4;
    int threads = (n4 + kLnVec - 1) / kLnVec;
    threads = (threads + 31) / 32 * 32;
    if (threads > 1024 || (long long)threads * kLnVec < n4) return cudaErrorInvalidValue;
    launch_pdl(ln_modulate_kernel, dim3(rows), dim3(threads), 0, st, x, rows, H, shift, scale, ld_mod, per_token, rows_per_item, y);
    return cudaGetLastError();
}

cudaError_t qk_norm_rope(const float * qkv, int B, int S, int H, int nh, const float * qg, const float * kg, int rope,
                         float fscale, float theta, __half * Q, __half * K, __half * V, int Sj, int s_off, cudaStream_t st) {
    if (H != nh * 64) return cudaErrorInvalidValue;
    launch_pdl(qk_norm_rope_kernel, dim3(nblk((long long)B * S * nh, 8)), dim3(256), 0, st, qkv, B, S, H, nh, qg, kg, rope, fscale, theta, Q, K,
                                                                       V, Sj, s_off);
    return cudaGetLastError();
}

cudaError_t rope_table(int S, float fscale, float theta, float2 * tab, cudaStream_t st) {
    launch_pdl(rope_table_kernel, dim3(nblk((long long)S * 32, 256)), dim3(256), 0, st, S, fscale, theta, tab);
    return cudaGetLastError();
}

cudaError_t latent_to_tokens(const float * lat, int B, int C, int T, __nv_bfloat16 * y, cudaStream_t st) {
    launch_pdl(latent_to_tokens_kernel, dim3(nblk((long long)B * C * T, 256)), dim3(256), 0, st, lat, B, C, T, y);
    return cudaGetLastError();
}

cudaError_t sync_prep(const float * sync, int B, int S, int C, const float * pos_emb, __nv_bfloat16 * y, cudaStream_t st) {
    launch_pdl(sync_prep_kernel, dim3(nblk((long long)B * S * C, 256)), dim3(256), 0, st, sync, B, S, C, pos_emb, y);
    return cudaGetLastError();
}

cudaError_t text_prep(const float * text, int text_S, int text_dim, const float * t5, int t5_S, int t5_dim, int B,
                      __nv_bfloat16 * y, cudaStream_t st) {
    launch_pdl(text_prep_kernel, dim3(nblk((long long)B * (text_S + t5_S) * t5_dim, 256)), dim3(256), 0, st, text, text_S, text_dim, t5, t5_S,
                                                                                         t5_dim, B, y);
    return cudaGetLastError();
}

cudaError_t timestep_embed(const float * t, int B, int H, float max_period, float * y, cudaStream_t st) {
    launch_pdl(timestep_embed_kernel, dim3(nblk((long long)B * (H / 2), 256)), dim3(256), 0, st, t, B, H, max_period, y);
    return cudaGetLastError();
}

cudaError_t seq_mean(const float * x, int B, int S, int H, float * y, cudaStream_t st) {
    launch_pdl(seq_mean_kernel, dim3(nblk((long long)B * H, 256)), dim3(256), 0, st, x, B, S, H, y);
    return cudaGetLastError();
}

cudaError_t add_vec(const float * a, const float * b, int n, float * y, cudaStream_t st) {
    launch_pdl(add_vec_kernel, dim3(nblk(n, 256)), dim3(256), 0, st, a, b, n, y);
    return cudaGetLastError();
}

cudaError_t build_extended(const float * sync, int sync_S, const float * gc, int B, int T, int H, float * ext,
                           __nv_bfloat16 * sext, float * sgc, cudaStream_t st) {
    launch_pdl(build_extended_kernel, dim3(nblk((long long)B * T * H, 256)), dim3(256), 0, st, sync, sync_S, gc, B, T, H, ext, sext);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    launch_pdl(silu_vec_kernel, dim3(nblk((long long)B * H, 256)), dim3(256), 0, st, gc, B * H, sgc);
    return cudaGetLastError();
}

__global__ void silu_cast_kernel(const float * __restrict__ x, long long n, __nv_bfloat16 * __restrict__ y) {
    pdl_wait();
    pdl_launch_dependents();
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = __float2bfloat16_rn(silu_f(x[i]));
}

cudaError_t silu_cast_bf16(const float * x, long long n, __nv_bfloat16 * y, cudaStream_t st) {
    launch_pdl(silu_cast_kernel, dim3(nblk(n, 256)), dim3(256), 0, st, x, n, y);
    return cudaGetLastError();
}

cudaError_t cast_f32_bf16(const float * x, long long n, __nv_bfloat16 * y, cudaStream_t st) {
    launch_pdl(cast_kernel, dim3(nblk(n, 256)), dim3(256), 0, st, x, n, y);
    return cudaGetLastError();
}

cudaError_t cfg_euler(const float * flow, int P, int T, int L, float cfg, float dt, float * x, float * flow0,
                      cudaStream_t st) {
    launch_pdl(cfg_euler_kernel, dim3(nblk((long long)P * L * T, 256)), dim3(256), 0, st, flow, P, T, L, cfg, dt, x, flow0);
    return cudaGetLastError();
}

cudaError_t dup_latent(const float * x, int P, int L, int T, float * lat2, cudaStream_t st) {
    launch_pdl(dup_latent_kernel, dim3(nblk((long long)P * L * T, 256)), dim3(256), 0, st, x, P, L, T, lat2);
    return cudaGetLastError();
}

}  // namespace tsd
