// gemm_static.cu — tsd_op_gemm_static: the projection GEMM (gemm_tc.cu) for callers that
// cannot allocate device memory.
//
// The GEMM splits K across CTAs for few-token, long-K shapes. Within one wave the splits of a
// tile reduce through the cluster's shared memory and need no scratch; beyond it they need
// scratch in global memory: partial tiles plus per-tile arrival counters. tsd_op_gemm takes that
// scratch from the caller; this variant takes it from two file-scope __device__ arrays of fixed
// size instead (TSD_GEMM_STATIC_WS_FLOATS floats and TSD_GEMM_STATIC_COUNTERS ints), so it calls
// no cudaMalloc / cudaFree and no allocating library routine. Every GPU that loads the library
// holds the arrays (8 MB + 32 KB) until the process exits. The tiling is chosen exactly as
// tsd_op_gemm chooses it when given scratch of that size, so plans that split K through global
// memory always fit the arrays (and shapes that do not split, or split inside a cluster, use
// none of it).
//
// Host code cannot use the array names as device addresses (in host code they name host-side
// stand-ins), so the first call on each device looks the addresses up with
// cudaGetSymbolAddress while that device is current, and later calls reuse them as long as the
// device's CUDA context is the same one (after a context is destroyed and recreated, e.g. by
// cudaDeviceReset, the module is loaded anew and the addresses are looked up again). That
// first call should come before any stream capture. All calls on a device share the arrays and
// they keep the last call's contents: the counters the GEMM relies on starting at zero are
// cleared on the caller's stream at every call that uses them, and calls whose executions
// overlap on the GPU (different streams, or different host threads without ordering) race on
// the scratch.
#include "kernels.h"
#include "../../include/tsd.h"
#include "../../include/tsd_ops.h"

#include <cstdio>
#include <mutex>

namespace tsd {
namespace {

constexpr long long kStaticWsFloats = TSD_GEMM_STATIC_WS_FLOATS;   // 8 MB of split-K partial tiles
constexpr int kStaticCounters = TSD_GEMM_STATIC_COUNTERS;          // 32 KB of tile arrival counters

static __device__ __align__(256) float g_static_ws[kStaticWsFloats];
static __device__ __align__(256) int g_static_counters[kStaticCounters];

struct DeviceScratch {
    CUcontext ctx = nullptr;     // the context the addresses belong to
    float * ws = nullptr;
    int * counters = nullptr;
};
constexpr int kMaxDevices = 64;
DeviceScratch g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

typedef CUresult (*PFN_ctxGetCurrent_t)(CUcontext *);
PFN_ctxGetCurrent_t ctx_get_current_fn() {
    static PFN_ctxGetCurrent_t fn = nullptr;
    if (!fn) {
        void * p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_ctxGetCurrent_t>(p);
    }
    return fn;
}

// Device addresses of the arrays on the current device (looked up once per device and context).
int device_scratch(DeviceScratch & out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaSetDevice(dev);   // initialises the device's primary context if needed
    if (e != cudaSuccess) {
        fprintf(stderr, "tsd_op_gemm_static: %s\n", cudaGetErrorString(e));
        return TSD_ERR_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) return TSD_ERR_ARG;
    CUcontext ctx = nullptr;
    PFN_ctxGetCurrent_t get_ctx = ctx_get_current_fn();
    if (!get_ctx || get_ctx(&ctx) != CUDA_SUCCESS || !ctx) {
        fprintf(stderr, "tsd_op_gemm_static: no current CUDA context on device %d\n", dev);
        return TSD_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    DeviceScratch & s = g_scratch[dev];
    if (!s.ws || s.ctx != ctx) {
        void * ws = nullptr, * counters = nullptr;
        e = cudaGetSymbolAddress(&ws, g_static_ws);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&counters, g_static_counters);
        if (e != cudaSuccess) {
            fprintf(stderr, "tsd_op_gemm_static: cudaGetSymbolAddress on device %d: %s\n", dev, cudaGetErrorString(e));
            return TSD_ERR_CUDA;
        }
        s.ctx = ctx;
        s.ws = static_cast<float *>(ws);
        s.counters = static_cast<int *>(counters);
    }
    out = s;
    return TSD_OK;
}

}  // namespace
}  // namespace tsd

using namespace tsd;

extern "C" int tsd_op_gemm_static(const void * W, int M, int K_in, int taps, int pad, const void * X, int nbatch, int S,
                                  int64_t x_row_stride, int64_t x_batch_stride, int mode, int act, const float * bias,
                                  int m_valid, void * out, int out_bf16, int64_t ldo, float * resid, int64_t ldr,
                                  const float * gate, int64_t ldg, int gate_div, int max_splits, int * err,
                                  void * stream) {
    if (!W || !X || mode < 0 || mode > 2 || (mode == EPI_GATE_RESID && (!resid || !gate || gate_div < 1)) ||
        (mode != EPI_GATE_RESID && !out) || M <= 0 || nbatch <= 0 || S <= 0)
        return TSD_ERR_ARG;
    const int swiglu = mode == EPI_SWIGLU;
    const int mv = m_valid > 0 ? m_valid : (swiglu ? M / 2 : M);
    DeviceScratch sc;
    int rc = device_scratch(sc);
    if (rc) return rc;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    GemmLaunch L;
    // the tiling tsd_op_gemm chooses with scratch of the arrays' size
    if (!gemm_plan(L, W, M, K_in, taps, pad, swiglu, X, nbatch, S, x_row_stride, x_batch_stride, sms, max_splits,
                   kStaticWsFloats, kStaticCounters, /*allow_cluster=*/true))
        return TSD_ERR_ARG;
    const long long need_ws = gemm_ws_floats(L);
    const long long need_cnt = need_ws ? (long long)L.p.mblocks * L.p.groups * L.p.n_tiles : 0;
    if (need_ws > kStaticWsFloats || need_cnt > kStaticCounters) {   // the planner keeps plans within the limits
        fprintf(stderr,
                "tsd_op_gemm_static: the plan needs %lld partial floats and %lld counters, beyond the static scratch "
                "of %lld floats and %d counters; use tsd_op_gemm with caller-provided scratch\n",
                need_ws, need_cnt, kStaticWsFloats, kStaticCounters);
        return TSD_ERR_ARG;
    }
    GemmParams & p = L.p;
    p.mode = mode; p.act = act;
    p.m_valid = mv;
    p.bias = bias;
    p.out = out; p.out_bf16 = out_bf16; p.ldo = ldo;
    p.resid = resid; p.ldr = ldr; p.gate = gate; p.ldg = ldg; p.gate_div = gate_div > 0 ? gate_div : 1;
    p.ws = sc.ws; p.counters = sc.counters;
    p.err = err;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (need_cnt) {
        // the arrays keep the previous call's contents: restart the arrival counts at zero
        cudaError_t e = cudaMemsetAsync(sc.counters, 0, (size_t)need_cnt * sizeof(int), st);
        if (e != cudaSuccess) {
            fprintf(stderr, "tsd_op_gemm_static: %s\n", cudaGetErrorString(e));
            return TSD_ERR_CUDA;
        }
    }
    cudaError_t e = gemm_launch(L, st);
    if (e != cudaSuccess) {
        fprintf(stderr, "tsd_op_gemm_static: launch: %s\n", cudaGetErrorString(e));
        return TSD_ERR_CUDA;
    }
    return TSD_OK;
}
