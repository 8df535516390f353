// capi.cu — extern "C" entry points of libtsd_b200 (include/tsd.h, include/tsd_ops.h).
#include "runtime.h"
#include "../../include/tsd_ops.h"

#include <cstring>
#include <vector>

using namespace tsd;

namespace tsd {
// Setters of every translation unit's copy of the device wait limit (common.cuh).
static std::vector<WaitLimitSetter> & wait_limit_setters() {
    static std::vector<WaitLimitSetter> v;
    return v;
}
int register_wait_limit_setter(WaitLimitSetter fn) {
    wait_limit_setters().push_back(fn);
    return 1;
}
}  // namespace tsd

struct tsd_model {
    Model * m = nullptr;
    cudaStream_t stream = nullptr;
};

namespace {

int make_stream(tsd_model * h) {
    TSD_CUDA_TRY(cudaSetDevice(h->m->device));
    TSD_CUDA_TRY(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking));
    return TSD_OK;
}

// Reads and clears the device error word; maps it to a status.
int check_device(Model & m, cudaStream_t st) {
    int e = 0;
    if (m.h_err) {     // the error word travels with the call's last copy: one synchronisation
        TSD_CUDA_TRY(cudaMemcpyAsync(m.h_err, m.d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
        TSD_CUDA_TRY(cudaStreamSynchronize(st));
        e = *m.h_err;
    } else {
        TSD_CUDA_TRY(cudaStreamSynchronize(st));
        TSD_CUDA_TRY(cudaMemcpy(&e, m.d_err, sizeof(int), cudaMemcpyDeviceToHost));
    }
    if (e) {
        fprintf(stderr, "tsd: device error word %d (a bounded wait expired)\n", e);
        cudaMemset(m.d_err, 0, sizeof(int));
        // an interrupted split-K GEMM may have left arrival counts behind
        if (m.plan && m.plan->counters) cudaMemset(m.plan->counters, 0, sizeof(int) * m.plan->n_counters);
        return TSD_ERR_DEVICE;
    }
    return TSD_OK;
}

int get_plan(Model & m, const Shape & sh, Plan ** out) {
    if (!m.finalized) return TSD_ERR_STATE;
    if (!m.plan || !(m.plan->sh == sh)) {
        m.plan.reset();
        const int rc = plan_build(m, sh, m.plan);
        if (rc) return rc;
    }
    *out = m.plan.get();
    return TSD_OK;
}

struct Inputs {
    const float * latent, * t, * clip_f, * sync_f, * text_f, * t5, * gtext;
};

// Copies the inputs into the plan's buffers in the order the forward consumes them (input groups
// of runtime.h). overlap: the caller waits for the whole forward before it returns (so no later
// call can record the group events while a graph still waits on them): the copies run on the
// plan's copy stream after everything already queued on st, and each group records its event,
// on which the captured graph's lanes wait. Otherwise the copies are ordered on st and the group
// events are left as they are (completed, or never recorded: waits on them pass).
int stage_inputs(Model & m, Plan & p, const Inputs & in, cudaStream_t st, bool overlap = false) {
    const Shape & s = p.sh;
    const size_t B = (size_t)s.B;
    overlap = overlap && st && p.copy_st;
    cudaStream_t cs = st;
    if (overlap) {
        TSD_CUDA_TRY(cudaEventRecord(p.prev_done, st));
        TSD_CUDA_TRY(cudaStreamWaitEvent(p.copy_st, p.prev_done, 0));
        cs = p.copy_st;
    }
    const auto group_done = [&](int g) { return overlap ? cudaEventRecord(p.in_ev[g], cs) : cudaSuccess; };
    TSD_CUDA_TRY(cudaMemcpyAsync(p.lat_in, in.latent, B * m.L * s.T * 4, cudaMemcpyDefault, cs));
    TSD_CUDA_TRY(cudaMemcpyAsync(p.t_in, in.t, B * 4, cudaMemcpyDefault, cs));
    TSD_CUDA_TRY(group_done(IN_LAT));
    TSD_CUDA_TRY(cudaMemcpyAsync(p.sync_in, in.sync_f, B * s.sync_S * m.sync_dim * 4, cudaMemcpyDefault, cs));
    TSD_CUDA_TRY(group_done(IN_SYNC));
    TSD_CUDA_TRY(cudaMemcpyAsync(p.clip_in, in.clip_f, B * s.clip_S * m.clip_dim * 4, cudaMemcpyDefault, cs));
    TSD_CUDA_TRY(group_done(IN_CLIP));
    if (s.text_S) TSD_CUDA_TRY(cudaMemcpyAsync(p.text_in, in.text_f, B * s.text_S * m.text_dim * 4, cudaMemcpyDefault, cs));
    if (s.t5_S) TSD_CUDA_TRY(cudaMemcpyAsync(p.t5_in, in.t5, B * s.t5_S * m.t5_dim * 4, cudaMemcpyDefault, cs));
    TSD_CUDA_TRY(group_done(IN_TEXT));
    TSD_CUDA_TRY(cudaMemcpyAsync(p.gtext_in, in.gtext, B * m.text_dim * 4, cudaMemcpyDefault, cs));
    TSD_CUDA_TRY(group_done(IN_GTEXT));
    return TSD_OK;
}

bool shape_ok(int B, int64_t T, int64_t clip_S, int64_t sync_S, int64_t text_S, int64_t t5_S) {
    return B >= 1 && T >= 1 && T <= (1 << 20) && clip_S >= 1 && clip_S <= (1 << 20) && sync_S >= 8 && sync_S % 8 == 0 &&
           sync_S <= (1 << 20) && text_S >= 0 && t5_S >= 0 && text_S + t5_S >= 1 && text_S + t5_S <= (1 << 20);
}

std::vector<float> host_f32(const RawTensor & t) {
    std::vector<float> out((size_t)t.n());
    const uint8_t * h = t.host.data();
    for (int64_t i = 0; i < t.n(); ++i) {
        if (t.type == GT_F32) memcpy(&out[i], h + 4 * i, 4);
        else if (t.type == GT_BF16) { uint32_t u = (uint32_t)(*(const uint16_t *)(h + 2 * i)) << 16; memcpy(&out[i], &u, 4); }
        else if (t.type == GT_F16) { __half hv; memcpy(&hv, h + 2 * i, 2); out[i] = __half2float(hv); }
        else {
            const uint8_t * blk = h + (i / 32) * 34;
            __half d; memcpy(&d, blk, 2);
            out[i] = (float)(int8_t)blk[2 + i % 32] * __half2float(d);
        }
    }
    return out;
}

}  // namespace

extern "C" {

const char * tsd_version(void) { return "tsd_b200 0.1 (sm_100a)"; }

int tsd_set_wait_limit(int device, uint64_t ns) {
    if (ns < 1000000ull || ns > 60000000000ull) return TSD_ERR_ARG;
    int prev = 0;
    TSD_CUDA_TRY(cudaGetDevice(&prev));
    TSD_CUDA_TRY(cudaSetDevice(device));
    cudaError_t e = cudaSuccess;
    for (WaitLimitSetter fn : wait_limit_setters())
        if (e == cudaSuccess) e = fn((unsigned long long)ns);
    cudaSetDevice(prev);
    TSD_CUDA_TRY(e);
    return TSD_OK;
}

int tsd_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

int tsd_load_gguf(const char * path, int device, tsd_model ** out) {
    if (!path || !out) return TSD_ERR_ARG;
    Model * m = nullptr;
    const int rc = model_load_gguf(path, device, &m);
    if (rc) return rc;
    tsd_model * h = new tsd_model();
    h->m = m;
    const int rs = make_stream(h);
    if (rs) { delete m; delete h; return rs; }
    *out = h;
    return TSD_OK;
}

int tsd_model_create(const tsd_hparams * hp, int device, tsd_model ** out) {
    if (!hp || !out) return TSD_ERR_ARG;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return TSD_ERR_CUDA;
    tsd_model * h = new tsd_model();
    h->m = new Model();
    h->m->hp = *hp;
    h->m->device = device;
    cudaDeviceGetAttribute(&h->m->num_sms, cudaDevAttrMultiProcessorCount, device);
    const int rs = make_stream(h);
    if (rs) { delete h->m; delete h; return rs; }
    *out = h;
    return TSD_OK;
}

int tsd_model_set_tensor(tsd_model * h, const char * name, int ggml_type, const int64_t ne[4], const void * data,
                         size_t nbytes) {
    if (!h || !ne) return TSD_ERR_ARG;
    return model_set_tensor(*h->m, name, ggml_type, ne, data, nbytes);
}

int tsd_model_finalize(tsd_model * h) {
    if (!h) return TSD_ERR_ARG;
    return model_finalize(*h->m);
}

void tsd_model_free(tsd_model * h) {
    if (!h) return;
    if (h->m) cudaSetDevice(h->m->device);
    if (h->stream) cudaStreamDestroy(h->stream);
    delete h->m;
    delete h;
}

int tsd_hp_layout(int hidden, int n_head, int world, int rank, int32_t out[3]) {
    int h0, nl, sec;
    if (!out || !hp_layout(hidden, n_head, world, rank, h0, nl, sec)) return TSD_ERR_ARG;
    out[0] = h0; out[1] = nl; out[2] = sec;
    return TSD_OK;
}

int tsd_hp_init(tsd_model * h, int rank, int world, size_t arena_bytes, void * handle_out) {
    if (!h || !h->m) return TSD_ERR_ARG;
    TSD_CUDA_TRY(cudaStreamSynchronize(h->stream));
    return hp_init(*h->m, rank, world, arena_bytes, handle_out);
}

int tsd_hp_connect(tsd_model * h, const void * handles) {
    if (!h || !h->m) return TSD_ERR_ARG;
    return hp_connect(*h->m, handles);
}

int tsd_model_get_hparams(const tsd_model * h, tsd_hparams * out) {
    if (!h || !out) return TSD_ERR_ARG;
    *out = h->m->hp;
    return TSD_OK;
}

int tsd_get_tensor_f32(const tsd_model * h, const char * name, float * dst, int64_t n_dst, int64_t ne_out[4]) {
    if (!h || !name) return TSD_ERR_ARG;
    const RawTensor * t = h->m->get(name);
    if (!t) {
        fprintf(stderr, "tsd: tensor missing: '%s'\n", name);
        return TSD_ERR_MISSING;
    }
    if (ne_out) for (int i = 0; i < 4; ++i) ne_out[i] = t->ne[i];
    if (!dst) return TSD_OK;
    if (n_dst < t->n()) return TSD_ERR_ARG;
    if (!t->host.empty()) {
        const std::vector<float> v = host_f32(*t);
        memcpy(dst, v.data(), v.size() * 4);
        return TSD_OK;
    }
    if (!t->d) return TSD_ERR_UNSUPPORTED;   // repacked projection weight: raw copy released
    RawTensor tmp = *t;
    tmp.host.resize(t->nbytes);
    TSD_CUDA_TRY(cudaSetDevice(h->m->device));
    TSD_CUDA_TRY(cudaMemcpy(tmp.host.data(), t->d, t->nbytes, cudaMemcpyDeviceToHost));
    const std::vector<float> v = host_f32(tmp);
    memcpy(dst, v.data(), v.size() * 4);
    return TSD_OK;
}

int tsd_forward_batched(tsd_model * h, int B, const float * latent, int64_t T, const float * t, const float * clip_f,
                        int64_t clip_S, const float * sync_f, int64_t sync_S, const float * text_f, int64_t text_S,
                        const float * t5, int64_t t5_S, const float * global_text, float * flow_out, tsd_dbg_fn dbg,
                        void * ud) {
    if (!h || !latent || !t || !clip_f || !sync_f || (text_S && !text_f) || (t5_S && !t5) || !global_text || !flow_out)
        return TSD_ERR_ARG;
    if (!shape_ok(B, T, clip_S, sync_S, text_S, t5_S)) return TSD_ERR_ARG;
    Model & m = *h->m;
    TSD_CUDA_TRY(cudaSetDevice(m.device));
    Plan * p = nullptr;
    int rc = get_plan(m, Shape{B, (int)T, (int)clip_S, (int)sync_S, (int)text_S, (int)t5_S}, &p);
    if (rc) return rc;
    // this call returns only after the forward (check_device): the copies may overlap it
    rc = stage_inputs(m, *p, Inputs{latent, t, clip_f, sync_f, text_f, t5, global_text}, h->stream, !dbg);
    if (rc) return rc;
    rc = plan_run(m, *p, h->stream, dbg, ud);
    if (rc) return rc;
    TSD_CUDA_TRY(cudaMemcpyAsync(flow_out, p->flow, (size_t)B * T * m.L * 4, cudaMemcpyDefault, h->stream));
    return check_device(m, h->stream);
}

int tsd_forward_inject(tsd_model * h, int B, const float * latent, int64_t T, const float * t, const float * clip_f,
                       int64_t clip_S, const float * sync_f, int64_t sync_S, const float * text_f, int64_t text_S,
                       const float * t5, int64_t t5_S, const float * global_text, float * flow_out, tsd_dbg_fn dbg,
                       tsd_inject_fn inject, void * ud) {
    if (!h || !latent || !t || !clip_f || !sync_f || (text_S && !text_f) || (t5_S && !t5) || !global_text || !flow_out)
        return TSD_ERR_ARG;
    if (!shape_ok(B, T, clip_S, sync_S, text_S, t5_S)) return TSD_ERR_ARG;
    if (h->m->hpar.connected) return TSD_ERR_UNSUPPORTED;   // head-parallel peers run graphs in lock step
    Model & m = *h->m;
    TSD_CUDA_TRY(cudaSetDevice(m.device));
    Plan * p = nullptr;
    int rc = get_plan(m, Shape{B, (int)T, (int)clip_S, (int)sync_S, (int)text_S, (int)t5_S}, &p);
    if (rc) return rc;
    rc = stage_inputs(m, *p, Inputs{latent, t, clip_f, sync_f, text_f, t5, global_text}, h->stream);
    if (rc) return rc;
    rc = plan_run(m, *p, h->stream, dbg, ud, false, inject);
    if (rc) return rc;
    TSD_CUDA_TRY(cudaMemcpyAsync(flow_out, p->flow, (size_t)B * T * m.L * 4, cudaMemcpyDefault, h->stream));
    return check_device(m, h->stream);
}

int tsd_forward(tsd_model * h, const float * latent, int64_t T, float t, const float * clip_f, int64_t clip_S,
                const float * sync_f, int64_t sync_S, const float * text_f, int64_t text_S, const float * t5, int64_t t5_S,
                const float * global_text, float * flow_out) {
    return tsd_forward_batched(h, 1, latent, T, &t, clip_f, clip_S, sync_f, sync_S, text_f, text_S, t5, t5_S, global_text,
                               flow_out, nullptr, nullptr);
}

int tsd_forward_device(tsd_model * h, int B, const float * latent, int64_t T, const float * t, const float * clip_f,
                       int64_t clip_S, const float * sync_f, int64_t sync_S, const float * text_f, int64_t text_S,
                       const float * t5, int64_t t5_S, const float * global_text, float * flow_out, void * stream) {
    if (!h || !latent || !t || !clip_f || !sync_f || (text_S && !text_f) || (t5_S && !t5) || !global_text || !flow_out)
        return TSD_ERR_ARG;
    if (!shape_ok(B, T, clip_S, sync_S, text_S, t5_S)) return TSD_ERR_ARG;
    Model & m = *h->m;
    TSD_CUDA_TRY(cudaSetDevice(m.device));
    cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
    Plan * p = nullptr;
    int rc = get_plan(m, Shape{B, (int)T, (int)clip_S, (int)sync_S, (int)text_S, (int)t5_S}, &p);
    if (rc) return rc;
    rc = stage_inputs(m, *p, Inputs{latent, t, clip_f, sync_f, text_f, t5, global_text}, st);
    if (rc) return rc;
    rc = plan_run(m, *p, st, nullptr, nullptr);
    if (rc) return rc;
    TSD_CUDA_TRY(cudaMemcpyAsync(flow_out, p->flow, (size_t)B * T * m.L * 4, cudaMemcpyDeviceToDevice, st));
    return TSD_OK;
}

int tsd_forward_profile(tsd_model * h, int B, const float * latent, int64_t T, const float * t, const float * clip_f,
                        int64_t clip_S, const float * sync_f, int64_t sync_S, const float * text_f, int64_t text_S,
                        const float * t5, int64_t t5_S, const float * global_text, float * flow_out, void * stream,
                        int max_ops, int * n_ops, int * kind, int * launches, float * ms, double * flops, double * bytes) {
    if (!h || !n_ops || !latent || !t || !clip_f || !sync_f || !global_text || !flow_out) return TSD_ERR_ARG;
    if (!shape_ok(B, T, clip_S, sync_S, text_S, t5_S)) return TSD_ERR_ARG;
    Model & m = *h->m;
    TSD_CUDA_TRY(cudaSetDevice(m.device));
    cudaStream_t st = stream ? (cudaStream_t)stream : h->stream;
    Plan * p = nullptr;
    int rc = get_plan(m, Shape{B, (int)T, (int)clip_S, (int)sync_S, (int)text_S, (int)t5_S}, &p);
    if (rc) return rc;
    rc = stage_inputs(m, *p, Inputs{latent, t, clip_f, sync_f, text_f, t5, global_text}, st);
    if (rc) return rc;
    std::vector<float> t_ms;
    rc = plan_profile(m, *p, st, t_ms);
    if (rc) return rc;
    TSD_CUDA_TRY(cudaMemcpyAsync(flow_out, p->flow, (size_t)B * T * m.L * 4, cudaMemcpyDeviceToDevice, st));
    *n_ops = (int)p->ops.size();
    for (int i = 0; i < (int)p->ops.size() && i < max_ops; ++i) {
        const Op & o = p->ops[i];
        if (kind) kind[i] = o.kind;
        if (launches) launches[i] = o.launches;
        if (ms) ms[i] = t_ms[i];
        if (flops) flops[i] = o.flops;
        if (bytes) bytes[i] = o.bytes;
    }
    return check_device(m, st);
}

const char * tsd_plan_op_label(tsd_model * h, int i) {
    if (!h || !h->m->plan || i < 0 || i >= (int)h->m->plan->ops.size()) return nullptr;
    return h->m->plan->ops[i].label.c_str();
}

int tsd_sync_check(tsd_model * h, void * stream) {
    if (!h) return TSD_ERR_ARG;
    TSD_CUDA_TRY(cudaSetDevice(h->m->device));
    return check_device(*h->m, stream ? (cudaStream_t)stream : h->stream);
}

int tsd_sample_batched(tsd_model * h, int P, const float * noise, int64_t T, const float * clip_f, int64_t clip_S,
                       const float * sync_f, int64_t sync_S, const float * text_f, int64_t text_S, const float * t5,
                       int64_t t5_S, const float * global_text, int steps, float cfg, float * out, float * flow0) {
    if (!h || P < 1 || !noise || !clip_f || !sync_f || (text_S && !text_f) || (t5_S && !t5) || !global_text || !out || steps < 1)
        return TSD_ERR_ARG;
    const int B = 2 * P;
    if (!shape_ok(B, T, clip_S, sync_S, text_S, t5_S)) return TSD_ERR_ARG;
    Model & m = *h->m;
    TSD_CUDA_TRY(cudaSetDevice(m.device));
    // uncond conditioning: learned empties + zero global vector (mmdit.cpp:350-356, 364)
    const RawTensor * es = m.get("empty_string_feat");
    const RawTensor * et = m.get("empty_t5_feat");
    if (!es || !et) return TSD_ERR_MISSING;
    if (es->host.empty() || et->host.empty()) return TSD_ERR_UNSUPPORTED;
    if (es->ne[0] != m.text_dim || es->ne[1] < text_S || et->ne[0] != m.t5_dim || et->ne[1] < t5_S) {
        fprintf(stderr, "tsd: learned empties [%lld x %lld], [%lld x %lld] do not cover text_S %lld / t5_S %lld\n",
                (long long)es->ne[0], (long long)es->ne[1], (long long)et->ne[0], (long long)et->ne[1], (long long)text_S,
                (long long)t5_S);
        return TSD_ERR_ARG;
    }
    const std::vector<float> es_h = host_f32(*es), et_h = host_f32(*et);
    Plan * p = nullptr;
    int rc = get_plan(m, Shape{B, (int)T, (int)clip_S, (int)sync_S, (int)text_S, (int)t5_S}, &p);
    if (rc) return rc;
    cudaStream_t st = h->stream;
    const size_t L = (size_t)m.L;
    // Stage the 2P conditioning items once: item 2p = cond, 2p+1 = uncond.
    {
        const size_t cn = (size_t)clip_S * m.clip_dim, yn = (size_t)sync_S * m.sync_dim;
        const size_t tn = (size_t)text_S * m.text_dim, fn = (size_t)t5_S * m.t5_dim, gn = (size_t)m.text_dim;
        std::vector<float> c2(2 * P * cn), y2(2 * P * yn), x2(2 * P * tn), f2(2 * P * fn), g2(2 * P * gn, 0.f);
        for (int q = 0; q < P; ++q)
            for (int k = 0; k < 2; ++k) {
                const size_t i = 2 * q + k;
                memcpy(&c2[i * cn], clip_f + q * cn, cn * 4);
                memcpy(&y2[i * yn], sync_f + q * yn, yn * 4);
                if (k == 0) {
                    if (tn) memcpy(&x2[i * tn], text_f + q * tn, tn * 4);
                    if (fn) memcpy(&f2[i * fn], t5 + q * fn, fn * 4);
                    memcpy(&g2[i * gn], global_text + q * gn, gn * 4);
                } else {
                    if (tn) memcpy(&x2[i * tn], es_h.data(), tn * 4);
                    if (fn) memcpy(&f2[i * fn], et_h.data(), fn * 4);
                }
            }
        TSD_CUDA_TRY(cudaMemcpyAsync(p->clip_in, c2.data(), c2.size() * 4, cudaMemcpyHostToDevice, st));
        TSD_CUDA_TRY(cudaMemcpyAsync(p->sync_in, y2.data(), y2.size() * 4, cudaMemcpyHostToDevice, st));
        if (tn) TSD_CUDA_TRY(cudaMemcpyAsync(p->text_in, x2.data(), x2.size() * 4, cudaMemcpyHostToDevice, st));
        if (fn) TSD_CUDA_TRY(cudaMemcpyAsync(p->t5_in, f2.data(), f2.size() * 4, cudaMemcpyHostToDevice, st));
        TSD_CUDA_TRY(cudaMemcpyAsync(p->gtext_in, g2.data(), g2.size() * 4, cudaMemcpyHostToDevice, st));
        TSD_CUDA_TRY(cudaStreamSynchronize(st));
    }
    // Every step's timestep vector is staged up front, so the step loop only enqueues work.
    std::vector<float> t_host((size_t)steps * B);
    for (int s = 0; s < steps; ++s)
        for (int i = 0; i < B; ++i) t_host[(size_t)s * B + i] = 1.0f - (float)s / steps;
    float * x = nullptr, * f0 = nullptr, * t_all = nullptr;
    TSD_CUDA_TRY(cudaMalloc(&x, (size_t)P * L * T * 4));
    if (cudaMalloc(&t_all, t_host.size() * 4) != cudaSuccess) { cudaFree(x); return TSD_ERR_CUDA; }
    if (flow0) cudaMalloc(&f0, (size_t)P * L * T * 4);
    rc = TSD_OK;
    cudaError_t e = cudaMemcpyAsync(x, noise, (size_t)P * L * T * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(t_all, t_host.data(), t_host.size() * 4, cudaMemcpyHostToDevice, st);
    for (int s = 0; s < steps && e == cudaSuccess && rc == TSD_OK; ++s) {
        const float t_curr = 1.0f - (float)s / steps, t_prev = 1.0f - (float)(s + 1) / steps;
        e = cudaMemcpyAsync(p->t_in, t_all + (size_t)s * B, (size_t)B * 4, cudaMemcpyDeviceToDevice, st);
        if (e == cudaSuccess) e = dup_latent(x, P, (int)L, (int)T, p->lat_in, st);
        if (e != cudaSuccess) break;
        // the conditioning inputs were staged once above: steps after the first reuse the
        // conditioning-only results (clip / sync / text projections, global MLP) of step 0
        rc = plan_run(m, *p, st, nullptr, nullptr, s > 0);
        if (rc) break;
        e = cfg_euler(p->flow, P, (int)T, (int)L, cfg, t_prev - t_curr, x, (s == 0) ? f0 : nullptr, st);
    }
    if (e == cudaSuccess && rc == TSD_OK) e = cudaMemcpyAsync(out, x, (size_t)P * L * T * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && rc == TSD_OK && flow0 && f0) e = cudaMemcpyAsync(flow0, f0, (size_t)P * L * T * 4, cudaMemcpyDeviceToHost, st);
    if (rc == TSD_OK) rc = (e == cudaSuccess) ? check_device(m, st) : TSD_ERR_CUDA;
    if (e != cudaSuccess) fprintf(stderr, "tsd: sample: %s\n", cudaGetErrorString(e));
    cudaStreamSynchronize(st);
    cudaFree(x);
    cudaFree(t_all);
    if (f0) cudaFree(f0);
    return rc;
}

int tsd_sample(tsd_model * h, const float * noise, int64_t T, const float * clip_f, int64_t clip_S, const float * sync_f,
               int64_t sync_S, const float * text_f, int64_t text_S, const float * t5, int64_t t5_S,
               const float * global_text, int steps, float cfg, float * out, float * flow0) {
    return tsd_sample_batched(h, 1, noise, T, clip_f, clip_S, sync_f, sync_S, text_f, text_S, t5, t5_S, global_text, steps,
                              cfg, out, flow0);
}

// ------------------------------- operator-level entry points -------------------------------

int tsd_op_gemm(const void * W, int M, int K_in, int taps, int pad, const void * X, int nbatch, int S,
                int64_t x_row_stride, int64_t x_batch_stride, int mode, int act, const float * bias, int m_valid,
                void * out, int out_bf16, int64_t ldo, float * resid, int64_t ldr, const float * gate, int64_t ldg,
                int gate_div, int max_splits, float * ws, int64_t ws_floats, int * counters, int n_counters,
                int * err, void * stream) {
    if (!W || !X || mode < 0 || mode > 2 || (mode == EPI_GATE_RESID && (!resid || !gate || gate_div < 1)) ||
        (mode != EPI_GATE_RESID && !out) || (ws && !counters))
        return TSD_ERR_ARG;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    GemmLaunch L;
    const int swiglu = mode == EPI_SWIGLU;
    if (!gemm_plan(L, W, M, K_in, taps, pad, swiglu, X, nbatch, S, x_row_stride, x_batch_stride, sms,
                   max_splits, ws ? ws_floats : 0, ws ? n_counters : 0))
        return TSD_ERR_ARG;
    GemmParams & p = L.p;
    p.mode = mode; p.act = act;
    p.m_valid = m_valid > 0 ? m_valid : (swiglu ? M / 2 : M);
    p.bias = bias;
    p.out = out; p.out_bf16 = out_bf16; p.ldo = ldo;
    p.resid = resid; p.ldr = ldr; p.gate = gate; p.ldg = ldg; p.gate_div = gate_div > 0 ? gate_div : 1;
    p.ws = ws; p.counters = counters;
    p.err = err;
    TSD_CUDA_TRY(gemm_launch(L, (cudaStream_t)stream));
    return TSD_OK;
}

int tsd_op_gemm_plan(int M, int K_in, int taps, int nbatch, int S, int max_splits, int64_t ws_floats, int n_counters,
                     int64_t out[6]) {
    if (!out) return TSD_ERR_ARG;
    int dev = 0, sms = 148;
    TSD_CUDA_TRY(cudaGetDevice(&dev));
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // the tensor maps are encoded but never used: any 256-byte-aligned address serves
    const void * dummy = reinterpret_cast<const void *>(uintptr_t(1) << 20);
    GemmLaunch L;
    if (!gemm_plan(L, dummy, M, K_in, taps, 0, 0, dummy, nbatch, S, K_in, (long long)S * K_in, sms, max_splits,
                   ws_floats, n_counters, true))
        return TSD_ERR_ARG;
    out[0] = L.p.BN; out[1] = L.p.splits; out[2] = L.p.pair; out[3] = L.p.csplit; out[4] = gemm_ws_floats(L);
    out[5] = L.p.gather;
    return TSD_OK;
}

int tsd_op_peer_wait(const uint32_t * counters, const uint32_t * epoch, int rank, int world, uint32_t ctas, int * err,
                     void * stream) {
    if (!counters || !epoch || world < 1 || world > kMaxHpRanks || rank < 0 || rank >= world) return TSD_ERR_ARG;
    TSD_CUDA_TRY(hp_wait_launch(counters, epoch, rank, world, ctas, err, (cudaStream_t)stream));
    return TSD_OK;
}

int tsd_op_gemv(const void * W, int ggml_type, const void * W2, int M, int K, const float * x, int64_t ldx, int N,
                const float * bias, int act, int round_bf16, void * y, int y_bf16, int64_t ldy, void * stream) {
    if (!W || !x || !y) return TSD_ERR_ARG;
    cudaError_t e = gemv_launch(W, ggml_type, W2, M, K, x, ldx, N, bias, act, round_bf16, y, y_bf16, ldy, (cudaStream_t)stream);
    if (e == cudaErrorInvalidValue) return TSD_ERR_ARG;
    TSD_CUDA_TRY(e);
    return TSD_OK;
}

int tsd_op_attention(const void * Q, const void * K, const void * V, int B, int nh, int S, void * out, int64_t ldo, int * err,
                     void * stream) {
    if (!Q || !K || !V || !out) return TSD_ERR_ARG;
    AttnLaunch L;
    if (!attn_plan(L, Q, K, V, B, nh, S, out, ldo, err)) return TSD_ERR_ARG;
    TSD_CUDA_TRY(attn_launch(L, (cudaStream_t)stream));
    return TSD_OK;
}

int tsd_op_attention_f32(const void * Q, const void * K, const void * V, int B, int nh, int S, float * out, int64_t ldo,
                         int * err, void * stream) {
    if (!Q || !K || !V || !out) return TSD_ERR_ARG;
    AttnLaunch L;
    if (!attn_plan(L, Q, K, V, B, nh, S, out, ldo, err, true)) return TSD_ERR_ARG;
    TSD_CUDA_TRY(attn_launch(L, (cudaStream_t)stream));
    return TSD_OK;
}

int tsd_op_ln_modulate(const float * x, int rows, int H, const float * shift, const float * scale, int64_t ld_mod,
                       int per_token, int rows_per_item, void * y, void * stream) {
    if (!x || !shift || !scale || !y || rows < 1 || rows_per_item < 1) return TSD_ERR_ARG;
    cudaError_t e = ln_modulate(x, rows, H, shift, scale, ld_mod, per_token, rows_per_item, (__nv_bfloat16 *)y, (cudaStream_t)stream);
    if (e == cudaErrorInvalidValue) return TSD_ERR_ARG;
    TSD_CUDA_TRY(e);
    return TSD_OK;
}

int tsd_op_qk_norm_rope(const float * qkv, int B, int S, int H, int nh, const float * q_gain, const float * k_gain, int rope,
                        float freq_scale, float theta, void * Q, void * K, void * V, int Sj, int s_off, void * stream) {
    if (!qkv || !q_gain || !k_gain || !Q || !K || !V || s_off + S > Sj) return TSD_ERR_ARG;
    cudaError_t e = qk_norm_rope(qkv, B, S, H, nh, q_gain, k_gain, rope, freq_scale, theta, (__half *)Q, (__half *)K,
                                 (__half *)V, Sj, s_off, (cudaStream_t)stream);
    if (e == cudaErrorInvalidValue) return TSD_ERR_ARG;
    TSD_CUDA_TRY(e);
    return TSD_OK;
}

}  // extern "C"
