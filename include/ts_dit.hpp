// ts_dit.hpp — header-only C++ drop-in for the reference's `ts_dit` (src/mmdit.h:9-42),
// implemented over the C-ABI of libtsd_b200 (tsd.h).
//
// Keeps the member functions the reference's callers use with the same signatures:
//   bool load(path)                                  mmdit.h:17   (ts-generate, ts-server, dit tools)
//   std::vector<float> forward(latent, T, t, ...)    mmdit.h:23-29 (ts-dit_test, with the dbg map)
//   std::vector<float> sample(noise, T, ..., flow0)  mmdit.h:34-41 (ts-generate, ts-server, ts-dit_sample)
//   model.need(name) / model.get_data(t, dst)        ts_model.h:24-27 (generate.cpp:83-84,
//                                                    ts-server.cpp:75-79 read the learned empties)
// `model.need` returns an opaque `ggml_tensor *` handle that only get_data() interprets, so
// callers that pass it straight to get_data() compile unchanged with or without ggml.h.
// As in the reference, forward()/sample() take text and T5 features of text_seq (77) rows
// each; forward_ex()/sample_ex() take the T5 length separately.
#pragma once

#include "tsd.h"

#include <cstdio>
#include <cstdlib>
#include <map>
#include <memory>
#include <string>
#include <vector>

struct ggml_tensor;

struct ts_dit_model {
    tsd_model * h = nullptr;

    ggml_tensor * get(const std::string & name) const {
        int64_t ne[4];
        if (!h || tsd_get_tensor_f32(h, name.c_str(), nullptr, 0, ne) != TSD_OK) return nullptr;
        auto & slot = handles_[name];
        if (!slot) slot.reset(new std::string(name));
        return reinterpret_cast<ggml_tensor *>(slot.get());
    }
    // Aborts on a missing tensor, as ts_model::need (ts_model.cpp:106-113).
    ggml_tensor * need(const std::string & name) const {
        ggml_tensor * t = get(name);
        if (!t) {
            fprintf(stderr, "ts_model: required tensor missing: '%s'\n", name.c_str());
            abort();
        }
        return t;
    }
    // Copies the tensor to host as f32 (the learned empties are F32 in every DiT GGUF).
    void get_data(ggml_tensor * t, void * dst) const {
        const std::string & name = *reinterpret_cast<const std::string *>(t);
        int64_t ne[4];
        tsd_get_tensor_f32(h, name.c_str(), nullptr, 0, ne);
        const int64_t n = ne[0] * ne[1] * ne[2] * ne[3];
        if (tsd_get_tensor_f32(h, name.c_str(), static_cast<float *>(dst), n, nullptr) != TSD_OK) {
            fprintf(stderr, "ts_model: cannot read tensor '%s'\n", name.c_str());
            abort();
        }
    }

  private:
    mutable std::map<std::string, std::unique_ptr<std::string>> handles_;
};

struct ts_dit {
    ts_dit_model model;
    int device = 0;    // GPU ordinal (the reference picks the largest-memory GPU, ts_backend.h:24-35)
    int hidden = 1024, n_head = 16, head_dim = 64, depth = 21, fused_depth = 14;
    int latent_dim = 64, text_seq = 77;
    float rope_theta = 10000.f, t_max_period = 1.f;

    ts_dit() = default;
    ts_dit(const ts_dit &) = delete;
    ts_dit & operator=(const ts_dit &) = delete;
    ~ts_dit() { if (model.h) tsd_model_free(model.h); }

    bool load(const std::string & gguf_path) {
        if (const char * d = getenv("TSD_DEVICE")) device = atoi(d);
        if (tsd_load_gguf(gguf_path.c_str(), device, &model.h) != TSD_OK) return false;
        tsd_hparams hp;
        tsd_model_get_hparams(model.h, &hp);
        hidden = hp.hidden; n_head = hp.n_head; head_dim = hidden / n_head;
        depth = hp.depth; fused_depth = hp.fused_depth; latent_dim = hp.latent_dim;
        rope_theta = hp.rope_theta; t_max_period = hp.t_max_period;
        return true;
    }

    std::vector<float> forward(const float * latent, int64_t T, float t, const float * clip_f, int64_t clip_S,
                               const float * sync_f, int64_t sync_S, const float * text_f, const float * t5,
                               const float * global_text, std::map<std::string, std::vector<float>> * dbg = nullptr) {
        return forward_ex(latent, T, t, clip_f, clip_S, sync_f, sync_S, text_f, text_seq, t5, text_seq, global_text, dbg);
    }

    std::vector<float> forward_ex(const float * latent, int64_t T, float t, const float * clip_f, int64_t clip_S,
                                  const float * sync_f, int64_t sync_S, const float * text_f, int64_t text_S,
                                  const float * t5, int64_t t5_S, const float * global_text,
                                  std::map<std::string, std::vector<float>> * dbg = nullptr) {
        std::vector<float> flow((size_t)T * latent_dim);
        const int rc = tsd_forward_batched(model.h, 1, latent, T, &t, clip_f, clip_S, sync_f, sync_S, text_f, text_S, t5,
                                           t5_S, global_text, flow.data(), dbg ? &ts_dit::collect : nullptr, dbg);
        if (rc != TSD_OK) {
            fprintf(stderr, "dit: forward failed (%d)\n", rc);
            return {};
        }
        return flow;
    }

    std::vector<float> sample(const float * noise, int64_t T, const float * clip_f, int64_t clip_S, const float * sync_f,
                              int64_t sync_S, const float * text_f, const float * t5, const float * global_text, int steps,
                              float cfg_scale, std::vector<float> * flow0 = nullptr) {
        return sample_ex(noise, T, clip_f, clip_S, sync_f, sync_S, text_f, text_seq, t5, text_seq, global_text, steps,
                         cfg_scale, flow0);
    }

    std::vector<float> sample_ex(const float * noise, int64_t T, const float * clip_f, int64_t clip_S,
                                 const float * sync_f, int64_t sync_S, const float * text_f, int64_t text_S,
                                 const float * t5, int64_t t5_S, const float * global_text, int steps, float cfg_scale,
                                 std::vector<float> * flow0 = nullptr) {
        std::vector<float> out((size_t)T * latent_dim);
        if (flow0) flow0->resize((size_t)T * latent_dim);
        const int rc = tsd_sample(model.h, noise, T, clip_f, clip_S, sync_f, sync_S, text_f, text_S, t5, t5_S,
                                  global_text, steps, cfg_scale, out.data(), flow0 ? flow0->data() : nullptr);
        if (rc != TSD_OK) {
            fprintf(stderr, "dit: sample failed (%d)\n", rc);
            return {};
        }
        return out;
    }

  private:
    static void collect(void * ud, const char * name, const float * data, int64_t n) {
        (*static_cast<std::map<std::string, std::vector<float>> *>(ud))[name].assign(data, data + n);
    }
};
