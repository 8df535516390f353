// gemm_static.cu — tsd_op_gemm_static: the projection GEMM (gemm_tc.cu) for callers that
// cannot allocate device memory.
//
// The GEMM splits K across CTAs for few-token, long-K shapes and then needs scratch: partial
// tiles plus per-tile arrival counters. tsd_op_gemm takes that scratch from the caller; this
// variant takes it from two file-scope __device__ arrays of fixed size instead, so it calls
// no cudaMalloc / cudaFree and no allocating library routine. Every GPU that loads the
// library holds the arrays (8 MB + 32 KB) until the process exits.
//
// Host code cannot use the array names as device addresses (in host code they name host-side
// stand-ins), so the first call on each device looks the addresses up with
// cudaGetSymbolAddress while that device is current, and later calls reuse them. That first
// call should come before any stream capture. All calls on a device share the arrays and
// they keep the last call's contents: the counters the GEMM relies on starting at zero are
// cleared on the caller's stream at every call, and calls whose executions overlap on the GPU
// (different streams, or different host threads without ordering) race on the scratch.
#include "kernels.h"
#include "../../include/tsd.h"
#include "../../include/tsd_ops.h"

#include <cstdio>
#include <mutex>

namespace tsd {
namespace {

constexpr long long kStaticWsFloats = 2ll << 20;                 // 8 MB of split-K partial tiles
constexpr int kStaticCounters = 8192;                            // 32 KB of tile arrival counters
constexpr long long kStaticMaxOutputs = kStaticWsFloats / 2;     // limit on m_valid * nbatch * S

static __device__ __align__(256) float g_static_ws[kStaticWsFloats];
static __device__ __align__(256) int g_static_counters[kStaticCounters];

struct DeviceScratch {
    float * ws = nullptr;
    int * counters = nullptr;
};
constexpr int kMaxDevices = 64;
DeviceScratch g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

// Device addresses of the arrays on the current device (looked up once per device).
int device_scratch(DeviceScratch & out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        fprintf(stderr, "tsd_op_gemm_static: cudaGetDevice: %s\n", cudaGetErrorString(e));
        return TSD_ERR_CUDA;
    }
    if (dev < 0 || dev >= kMaxDevices) return TSD_ERR_ARG;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    DeviceScratch & s = g_scratch[dev];
    if (!s.ws) {
        void * ws = nullptr, * counters = nullptr;
        e = cudaGetSymbolAddress(&ws, g_static_ws);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&counters, g_static_counters);
        if (e != cudaSuccess) {
            fprintf(stderr, "tsd_op_gemm_static: cudaGetSymbolAddress on device %d: %s\n", dev, cudaGetErrorString(e));
            return TSD_ERR_CUDA;
        }
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
    if ((long long)mv * nbatch * S > kStaticMaxOutputs) {
        fprintf(stderr,
                "tsd_op_gemm_static: output of %d features x %d items x %d tokens = %lld values exceeds the static "
                "scratch limit of %lld values; use tsd_op_gemm with caller-provided scratch\n",
                mv, nbatch, S, (long long)mv * nbatch * S, kStaticMaxOutputs);
        return TSD_ERR_ARG;
    }
    DeviceScratch sc;
    int rc = device_scratch(sc);
    if (rc) return rc;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    GemmLaunch L;
    // split-K always reduces through the static workspace here (no cluster reduction)
    if (!gemm_plan(L, W, M, K_in, taps, pad, swiglu, X, nbatch, S, x_row_stride, x_batch_stride, sms, max_splits,
                   kStaticWsFloats, kStaticCounters, /*allow_cluster=*/false))
        return TSD_ERR_ARG;
    GemmParams & p = L.p;
    p.mode = mode; p.act = act;
    p.m_valid = mv;
    p.bias = bias;
    p.out = out; p.out_bf16 = out_bf16; p.ldo = ldo;
    p.resid = resid; p.ldr = ldr; p.gate = gate; p.ldg = ldg; p.gate_div = gate_div > 0 ? gate_div : 1;
    p.ws = sc.ws; p.counters = sc.counters;
    p.err = err;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (p.splits > 1) {
        // the arrays keep the previous call's contents: restart the arrival counts at zero
        const size_t otiles = (size_t)p.mblocks * p.nbatch * p.n_tiles;
        cudaError_t e = cudaMemsetAsync(sc.counters, 0, otiles * sizeof(int), st);
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
