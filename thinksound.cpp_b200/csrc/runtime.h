// runtime.h — host runtime of libtsd_b200: device weight store and forward plans.
#pragma once
#include "kernels.h"
#include "../../include/tsd.h"

#include <array>
#include <cstdio>
#include <functional>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

namespace tsd {

#define TSD_CUDA_TRY(expr)                                                                                  \
    do {                                                                                                    \
        cudaError_t e_ = (expr);                                                                            \
        if (e_ != cudaSuccess) {                                                                            \
            fprintf(stderr, "tsd: CUDA error %s at %s:%d: %s\n", cudaGetErrorName(e_), __FILE__, __LINE__,     \
                    cudaGetErrorString(e_));                                                                \
            return TSD_ERR_CUDA;                                                                            \
        }                                                                                                   \
    } while (0)

enum : int { GT_F32 = 0, GT_F16 = 1, GT_Q8_0 = 8, GT_BF16 = 30 };
size_t ggml_nbytes(int type, int64_t n);

// A tensor as stored (ggml type and layout) in device memory; small tensors keep a host copy.
struct RawTensor {
    int type = GT_F32;
    int64_t ne[4] = {1, 1, 1, 1};
    void * d = nullptr;
    size_t nbytes = 0;
    std::vector<uint8_t> host;
    int64_t n() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
};

// A projection weight repacked for the tcgen05 GEMM: bf16 [M][taps*K_in], tap-major columns; or,
// for a Q8_0 source (single tap), planar Q8_0 that the GEMM dequantises in shared memory:
// q [M][K_in] int8 and qs [K_in/32][M] f16 scales (transposed so a tile's scales are one TMA box).
struct GW {
    __nv_bfloat16 * w = nullptr;
    int8_t * q = nullptr;
    __half * qs = nullptr;
    int M = 0, K_in = 0, taps = 1, pad = 0, m_valid = 0;
    float * bias = nullptr;
};
// A weight used by the few-token GEMV in its stored type.
struct VW {
    const void * w = nullptr, * w2 = nullptr;
    int type = GT_F32, M = 0, K = 0;
    const float * bias = nullptr;
};
struct StreamW {
    bool present = false, pre_only = false, conv = false;
    GW qkv, l1, w13, w2;
    const float * qg = nullptr, * kg = nullptr;
    long long ada_off = 0;   // latent-style: first row in the batched adaLN weight
    int ada_rows = 0;
    VW ada;                  // global-conditioned (clip / text): GEMV weight
    long long ada_ct_off = -1;   // clip / text: first row in the stacked clip / text adaLN (Model::ada_ct)
};

struct Plan;

// Head-parallel state (hp.cu): this rank's heads, its exchange arena and the peers' mappings.
struct HeadParallel {
    int rank = 0, world = 1;
    int h0 = 0, nl = 0, sec = 0;          // heads [h0, h0 + nl); rows per sliced Q / K / V section
    uint8_t * arena = nullptr;
    size_t arena_bytes = 0, used = 0;
    uint8_t * peer[kMaxHpRanks] = {};     // every rank's arena as mapped in this process
    bool connected = false;
    int next_plan = 0, next_slot = 0;
    std::vector<std::array<GW, 3>> joint_qkv;   // QKV rows of this rank's heads
    std::vector<GW> fused_qkv;
    std::vector<void *> allocs;
};

struct Model {
    tsd_hparams hp{};
    int device = 0, num_sms = 148;
    int H = 0, nh = 0, F = 0, L = 64;
    int clip_dim = 1024, sync_dim = 768, text_dim = 1024, t5_dim = 2048;
    bool finalized = false;
    std::unordered_map<std::string, RawTensor> raw;
    std::vector<void *> allocs;

    GW ap0, ap13, ap2, cp0, cp13, cp2, sp0, sp13, sp2, tp0, tp13, tp2, fconv;
    VW te0, te2, tcp, ccp, gc13, gc2;
    const float * sync_pe = nullptr;
    GW ada_lat;                // all latent-style adaLN weights stacked (joint latent, fused, final)
    VW ada_ct;                 // every clip / text adaLN weight stacked in its stored type (one GEMV)
    long long final_ada_off = 0;
    std::vector<std::array<StreamW, 3>> joint;
    std::vector<StreamW> fused;
    int * d_err = nullptr;
    int * h_err = nullptr;     // pinned host copy of *d_err, read after each synchronous call
    std::unique_ptr<Plan> plan;
    HeadParallel hpar;

    ~Model();
    void * dalloc(size_t bytes);
    const RawTensor * get(const std::string & n) const {
        auto it = raw.find(n);
        return it == raw.end() ? nullptr : &it->second;
    }
};

int model_set_tensor(Model & m, const char * name, int type, const int64_t ne[4], const void * data, size_t nbytes);
int model_finalize(Model & m);
int model_load_gguf(const char * path, int device, Model ** out);

// Debug snapshot of a device buffer after an op of the forward.
struct Snap {
    std::string name;
    const void * ptr;
    long long n;
    int kind;          // 0 f32, 1 bf16, 2 fp16 head-major [B][nh][S][64] (S = rows) -> [B][S][H]
    int B, nh, S;
    bool inject = false;   // teacher forcing: offered to the inject callback, which may replace it (f32 only)
    std::function<cudaError_t(cudaStream_t)> after_inject;   // rebuilds what the op derived from it, if replaced
};
enum OpKind : int { OP_GEMM = 0, OP_GEMV = 1, OP_ATTN = 2, OP_ELEM = 3, OP_COPY = 4 };
struct Op {
    std::function<cudaError_t(cudaStream_t)> fn;
    std::vector<Snap> snaps;
    std::string label;        // e.g. "f3 gemm M=8192 N=388 K=4608 grid=32x4x1"
    int kind = OP_ELEM;
    int launches = 1;          // kernel launches the op issues
    double flops = 0, bytes = 0;   // algorithmic work of the op
    // Graph replay only: the op's lane (0 = the caller's stream, 1..kSideLanes = side streams).
    // Marker ops (fn empty): sync 1 = fork (side lanes wait for lane 0), 2 = join (lane 0 waits
    // for the side lanes), 3 = this lane waits for input group `input` (Plan::in_ev) to land.
    // Op-by-op execution runs everything in order on one stream.
    int lane = 0;
    int sync = 0;
    int input = 0;
    // Conditioning-only: the op reads only the staged clip / sync / text / global inputs (or
    // other conditioning-only ops' outputs) and writes buffers nothing else writes, so a replay
    // with unchanged conditioning inputs may skip it (the sampler's steps after the first).
    bool invariant = false;
};
constexpr int kSideLanes = 2;
// Input groups of a forward, in the order the plan's first ops consume them: each has its own
// copy-completion event, so that a graph replay starts each input chain as soon as its inputs
// have landed instead of after all of them.
enum InputGroup : int { IN_LAT = 0, IN_SYNC = 1, IN_CLIP = 2, IN_TEXT = 3, IN_GTEXT = 4, kInputGroups = 5 };

struct Shape {
    int B, T, clip_S, sync_S, text_S, t5_S;
    bool operator==(const Shape & o) const {
        return B == o.B && T == o.T && clip_S == o.clip_S && sync_S == o.sync_S && text_S == o.text_S && t5_S == o.t5_S;
    }
};

struct Plan {
    Shape sh{};
    int St = 0, Sj = 0, maxS = 0;
    // inputs / output (device)
    float * lat_in = nullptr, * clip_in = nullptr, * sync_in = nullptr, * text_in = nullptr, * t5_in = nullptr;
    float * gtext_in = nullptr, * t_in = nullptr, * flow = nullptr;
    int * counters = nullptr;   // split-K arrival counters (re-zeroed after a device error)
    int n_counters = 0;
    std::vector<Op> ops;
    std::vector<void *> allocs;
    // [0] every op; [1] without the conditioning-only ops (Op::invariant)
    cudaGraphExec_t graph[2] = {};
    cudaStream_t graph_stream[2] = {};
    cudaStream_t side[kSideLanes] = {};        // side lanes of the captured graph
    std::vector<cudaEvent_t> events;           // fork / join events (capture only)
    // Overlapped input staging (stage_inputs with a host-synchronised caller): the copies run on
    // copy_st, each group recording in_ev[group]; the captured graph's lanes wait on those events
    // (external event waits), so the first kernels start under the later groups' copies.
    cudaStream_t copy_st = nullptr;
    cudaEvent_t in_ev[kInputGroups] = {};
    cudaEvent_t prev_done = nullptr;           // the caller's stream before the copies
    ~Plan();
};

int plan_build(Model & m, const Shape & sh, std::unique_ptr<Plan> & out);

// Head-parallel mode (hp.cu).
bool hp_layout(int H, int nh, int world, int rank, int & h0, int & nl, int & sec);
int hp_init(Model & m, int rank, int world, size_t arena_bytes, void * handle_out);
int hp_connect(Model & m, const void * handles);
void hp_release(Model & m);
int hp_next_plan(Model & m);
int hp_next_slot(Model & m);
long long hp_carve(Model & m, size_t bytes);            // arena offset, or -1 when exhausted
unsigned * hp_counter(Model & m, int on_rank, int slot, int from_rank);
unsigned * hp_epoch(Model & m, int plan);
cudaError_t hp_epoch_launch(unsigned * epoch, cudaStream_t st);
int hp_push_ctas(int rows);
cudaError_t hp_push_launch(const __nv_bfloat16 * X, __nv_bfloat16 * const * dst, unsigned * const * flag, int n_peers,
                           int rows, int H, int col0, int ncols, cudaStream_t st);
cudaError_t hp_wait_launch(const unsigned * counters, const unsigned * epoch, int rank, int world, unsigned ctas,
                           int * err, cudaStream_t st);
// Enqueue the forward (inputs already in the plan's buffers). reuse_cond: the conditioning
// inputs (clip_in, sync_in, text_in, t5_in, gtext_in) are unchanged since the last full run of
// this plan, whose conditioning-only results are reused instead of recomputed.
// inject (op-by-op runs only): offered the residual streams at block boundaries (Snap::inject);
// a non-zero return writes the callback's data back before the next op.
int plan_run(Model & m, Plan & p, cudaStream_t st, tsd_dbg_fn dbg, void * ud, bool reuse_cond = false,
             tsd_inject_fn inject = nullptr);
// Run the forward op by op with CUDA events around each op; per-op milliseconds.
int plan_profile(Model & m, Plan & p, cudaStream_t st, std::vector<float> & ms);

}  // namespace tsd
