// hp.cu — head-parallel forward across the GPUs of one node (one process per GPU).
//
// The optional 30 s mode of the MM-DiT path: each of `world` ranks owns nh / world of the
// attention heads of every joint and fused block. A rank computes the QKV projection rows of its
// heads only (the reference's Wqkv, src/mmdit.cpp:219, sliced per head) and attention for those
// heads (:85-94) into its exchange buffer; a copy kernel then pushes this rank's column block of
// every row (nl * 128 contiguous bytes) into the same place in every other rank's buffer over
// NVLink and counts its arrival on each peer. Before the out-projection (:229-230) a one-warp
// kernel waits until every peer's push CTAs of that layer have arrived. Everything else (adaLN,
// LN-modulate, out-projection, FFN, pre-processing, final layer) runs replicated on every rank,
// so every rank ends with the full flow. There is no library collective: the exchange is plain
// peer stores. (Storing the rows from the attention epilogue itself was measured slower: its
// warp stores are 16-byte pieces of 32 different rows, which NVLink carries poorly.)
//
// Exchange arena (one cudaMalloc per rank, its IPC handle shared with the peers at set-up):
//   [0, kFlagBytes)           arrival counters u32 [slot][rank], monotonic
//   [kFlagBytes, +256)        forward epochs u32 [plan]
//   [kHeadBytes, end)         per-layer exchange buffers bf16 [B][S][H], bump-allocated by the
//                             plan builder in the same order on every rank (same shapes)
// A layer's counters grow by its CTA count per forward, so the wait for forward e checks
// count >= e * ctas: no reset, and a peer that is one layer ahead is harmless. Each layer of each
// plan has its own exchange buffer and counter slot (never reused), so a rank can overwrite a
// buffer a peer still reads only after passing that peer's later arrivals, which stream order
// on the peer rules out.
#include "common.cuh"
#include "runtime.h"

#include <cstring>

namespace tsd {

namespace {

constexpr size_t kFlagBytes = 64 * 1024;
constexpr size_t kHeadBytes = kFlagBytes + 4096;
constexpr int kMaxSlots = (int)(kFlagBytes / 4 / kMaxHpRanks);
constexpr int kMaxPlans = 64;

__global__ void hp_epoch_kernel(unsigned * epoch) {
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x == 0) *epoch += 1u;
}

// Waits until counter[r] >= epoch * ctas for every rank r != rank (bounded: ~2 s, then the
// device error word is set and the kernel returns).
__global__ void hp_wait_kernel(const unsigned * counters, const unsigned * epoch, int rank, int world, unsigned ctas,
                               int * err) {
    pdl_wait();
    pdl_launch_dependents();
    const int r = threadIdx.x;
    if (r < world && r != rank) {
        const unsigned want = *epoch * ctas;
        const unsigned long long t0 = globaltimer();
        unsigned v;
        for (;;) {
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(counters + r) : "memory");
            if ((int)(v - want) >= 0) break;
            if (globaltimer() - t0 > wait_ns()) {
                if (err) atomicExch(err, DEV_TIMEOUT_HP);
                break;
            }
            __nanosleep(200);
        }
    }
    __threadfence_system();
    asm volatile("fence.proxy.async.global;" ::: "memory");   // the peers' rows are next read by TMA
}

// Copies this rank's column block [col0, col0 + ncols) of every row of X ([rows][H] bf16) to the
// same place in every peer's buffer (a warp per row: the block is nl * 128 contiguous bytes, so a
// warp instruction moves 512 contiguous bytes over NVLink), then counts this CTA's arrival on
// every peer.
struct HpPeers {
    __nv_bfloat16 * dst[kMaxHpRanks];
    unsigned * flag[kMaxHpRanks];
};
__global__ void __launch_bounds__(256) hp_push_kernel(const __nv_bfloat16 * __restrict__ X, const HpPeers peers,
                                                      int n_peers, int rows, int H, int col0, int ncols) {
    pdl_wait();
    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nv = ncols >> 3;                       // 16-byte words of a row's block
    for (int r = blockIdx.x * 8 + warp; r < rows; r += gridDim.x * 8) {
        const long long base = (long long)r * H + col0;
        const uint4 * s = reinterpret_cast<const uint4 *>(X + base);
        for (int i = lane; i < nv; i += 32) {
            const uint4 v = s[i];
            for (int p = 0; p < n_peers; ++p) reinterpret_cast<uint4 *>(peers.dst[p] + base)[i] = v;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int p = 0; p < n_peers; ++p) atomicAdd_system(peers.flag[p], 1u);
    }
}

}  // namespace

int hp_push_ctas(int rows) { return rows < 1 ? 1 : (rows + 7) / 8 < 296 ? (rows + 7) / 8 : 296; }

cudaError_t hp_push_launch(const __nv_bfloat16 * X, __nv_bfloat16 * const * dst, unsigned * const * flag, int n_peers,
                           int rows, int H, int col0, int ncols, cudaStream_t st) {
    HpPeers pe{};
    for (int p = 0; p < n_peers && p < kMaxHpRanks; ++p) { pe.dst[p] = dst[p]; pe.flag[p] = flag[p]; }
    launch_pdl(hp_push_kernel, dim3(hp_push_ctas(rows)), dim3(256), 0, st, X, pe, n_peers, rows, H, col0, ncols);
    return cudaGetLastError();
}

bool hp_layout(int H, int nh, int world, int rank, int & h0, int & nl, int & sec) {
    if (world < 1 || world > kMaxHpRanks || rank < 0 || rank >= world || nh < 1 || nh % world || H != nh * 64)
        return false;
    nl = nh / world;
    h0 = rank * nl;
    sec = (nl * 64 + 127) / 128 * 128;   // rows per Q / K / V section: QKV GEMM tiles never straddle two
    return true;
}

int hp_init(Model & m, int rank, int world, size_t arena_bytes, void * handle_out) {
    if (!m.finalized) return TSD_ERR_STATE;
    int h0, nl, sec;
    if (!hp_layout(m.H, m.nh, world, rank, h0, nl, sec) || arena_bytes < kHeadBytes + (1 << 20) || !handle_out)
        return TSD_ERR_ARG;
    if (m.hpar.arena) return TSD_ERR_STATE;
    TSD_CUDA_TRY(cudaSetDevice(m.device));
    HeadParallel & hp = m.hpar;
    hp.rank = rank; hp.world = world; hp.h0 = h0; hp.nl = nl; hp.sec = sec;
    TSD_CUDA_TRY(cudaMalloc(&hp.arena, arena_bytes));
    hp.arena_bytes = arena_bytes;
    TSD_CUDA_TRY(cudaMemset(hp.arena, 0, kHeadBytes));
    cudaIpcMemHandle_t h;
    TSD_CUDA_TRY(cudaIpcGetMemHandle(&h, hp.arena));
    memcpy(handle_out, &h, sizeof(h));
    // Q / K / V rows of this rank's heads, each section padded with zero rows to `sec`
    auto slice = [&](const GW & w, GW & out) -> int {
        if (!w.w || w.q || w.taps != 1 || w.M != 3 * m.H) return TSD_ERR_UNSUPPORTED;
        out = w;
        out.M = 3 * sec;
        out.m_valid = 3 * sec;
        TSD_CUDA_TRY(cudaMalloc(&out.w, (size_t)out.M * w.K_in * 2));
        hp.allocs.push_back(out.w);
        TSD_CUDA_TRY(cudaMemset(out.w, 0, (size_t)out.M * w.K_in * 2));
        if (w.bias) {
            TSD_CUDA_TRY(cudaMalloc(&out.bias, (size_t)out.M * 4));
            hp.allocs.push_back(out.bias);
            TSD_CUDA_TRY(cudaMemset(out.bias, 0, (size_t)out.M * 4));
        }
        for (int j = 0; j < 3; ++j) {
            const size_t src_row = (size_t)j * m.H + (size_t)h0 * 64, dst_row = (size_t)j * sec;
            TSD_CUDA_TRY(cudaMemcpy(out.w + dst_row * w.K_in, w.w + src_row * w.K_in, (size_t)nl * 64 * w.K_in * 2,
                                    cudaMemcpyDeviceToDevice));
            if (w.bias)
                TSD_CUDA_TRY(cudaMemcpy(out.bias + dst_row, w.bias + src_row, (size_t)nl * 64 * 4, cudaMemcpyDeviceToDevice));
        }
        return TSD_OK;
    };
    hp.joint_qkv.assign(m.joint.size(), {});
    for (size_t i = 0; i < m.joint.size(); ++i)
        for (int s = 0; s < 3; ++s) {
            if (!m.joint[i][s].present) continue;
            const int rc = slice(m.joint[i][s].qkv, hp.joint_qkv[i][s]);
            if (rc) return rc;
        }
    hp.fused_qkv.assign(m.fused.size(), {});
    for (size_t i = 0; i < m.fused.size(); ++i) {
        const int rc = slice(m.fused[i].qkv, hp.fused_qkv[i]);
        if (rc) return rc;
    }
    m.plan.reset();
    return TSD_OK;
}

int hp_connect(Model & m, const void * handles) {
    HeadParallel & hp = m.hpar;
    if (!hp.arena || hp.connected) return TSD_ERR_STATE;
    if (!handles) return TSD_ERR_ARG;
    TSD_CUDA_TRY(cudaSetDevice(m.device));
    for (int r = 0; r < hp.world; ++r) {
        if (r == hp.rank) { hp.peer[r] = hp.arena; continue; }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t *>(handles) + (size_t)r * sizeof(h), sizeof(h));
        void * p = nullptr;
        TSD_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        hp.peer[r] = static_cast<uint8_t *>(p);
    }
    hp.connected = true;
    m.plan.reset();   // plans built from now on are head-parallel
    return TSD_OK;
}

void hp_release(Model & m) {
    HeadParallel & hp = m.hpar;
    for (int r = 0; r < kMaxHpRanks; ++r)
        if (hp.peer[r] && r != hp.rank) cudaIpcCloseMemHandle(hp.peer[r]);
    for (void * p : hp.allocs) cudaFree(p);
    if (hp.arena) cudaFree(hp.arena);
    hp = HeadParallel{};
}

// Plan-time carving, in the same order on every rank (never reused).
int hp_next_plan(Model & m) { return m.hpar.next_plan < kMaxPlans ? m.hpar.next_plan++ : -1; }
int hp_next_slot(Model & m) { return m.hpar.next_slot < kMaxSlots ? m.hpar.next_slot++ : -1; }
long long hp_carve(Model & m, size_t bytes) {
    HeadParallel & hp = m.hpar;
    const size_t off = kHeadBytes + (hp.used + 255) / 256 * 256;
    if (off + bytes > hp.arena_bytes) return -1;
    hp.used = off + bytes - kHeadBytes;
    return (long long)off;
}
unsigned * hp_counter(Model & m, int on_rank, int slot, int from_rank) {
    return reinterpret_cast<unsigned *>(m.hpar.peer[on_rank]) + (size_t)slot * kMaxHpRanks + from_rank;
}
unsigned * hp_epoch(Model & m, int plan) { return reinterpret_cast<unsigned *>(m.hpar.arena + kFlagBytes) + plan; }

cudaError_t hp_epoch_launch(unsigned * epoch, cudaStream_t st) {
    launch_pdl(hp_epoch_kernel, dim3(1), dim3(32), 0, st, epoch);
    return cudaGetLastError();
}
cudaError_t hp_wait_launch(const unsigned * counters, const unsigned * epoch, int rank, int world, unsigned ctas,
                           int * err, cudaStream_t st) {
    launch_pdl(hp_wait_kernel, dim3(1), dim3(32), 0, st, counters, epoch, rank, world, ctas, err);
    return cudaGetLastError();
}

}  // namespace tsd
