// ts_server_demo.cpp — the DiT part of the reference's HTTP server request path
// (src/tools/ts-server.cpp:48-100, generate_wav) with the DiT kept resident: the reference
// constructs a ts_dit and calls load() inside every request (ts-server.cpp:74); here the first
// request loads it into a process-wide slot and every later request reuses it (requests are
// serialised by one mutex, as ts-server's gen_mu, :124,158). Each request samples one prompt;
// the plan of an input shape is built on its first request and reused.
//   ts_server_demo <dit.gguf> <steps> <out.bin> <T:seed> [<T:seed> ...]
// Inputs of a request are deterministic in its seed: noise[i] = sin(0.37 i + seed),
// text[i] = cos(0.11 i + seed), t5[i] = sin(0.05 i + 1 + seed), global[i] = cos(0.7 i + seed);
// clip / sync rows are the learned empties (generate.cpp:83-87). Writes every request's latent
// [64][T] (f32) to out.bin in order and prints the number of loads and each request's time.
#include "ts_dit.hpp"

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace {

std::mutex g_gen_mu;                   // one request at a time (ts-server.cpp:124)
std::unique_ptr<ts_dit> g_dit;         // the resident model
int g_loads = 0;

ts_dit * resident_dit(const std::string & path) {
    if (!g_dit) {
        std::unique_ptr<ts_dit> d(new ts_dit());
        if (!d->load(path)) return nullptr;
        g_dit = std::move(d);
        ++g_loads;
    }
    return g_dit.get();
}

// One request: returns the latent [latent_dim][T], or an empty vector on failure (the server
// answers HTTP 500 then, ts-server.cpp:163-166).
std::vector<float> handle_request(const std::string & path, int64_t T, double seed, int steps) {
    std::lock_guard<std::mutex> lock(g_gen_mu);
    ts_dit * dit = resident_dit(path);
    if (!dit) return {};
    const int64_t clip_S = 8 * ((T + 19) / 20), sync_S = 24 * ((T + 19) / 20);
    std::vector<float> ecv(1024), esv(768);
    dit->model.get_data(dit->model.need("empty_clip_feat"), ecv.data());
    dit->model.get_data(dit->model.need("empty_sync_feat"), esv.data());
    std::vector<float> clip_f((size_t)1024 * clip_S), sync_f((size_t)768 * sync_S);
    for (int64_t s = 0; s < clip_S; ++s) for (int i = 0; i < 1024; ++i) clip_f[(size_t)s * 1024 + i] = ecv[i];
    for (int64_t s = 0; s < sync_S; ++s) for (int i = 0; i < 768; ++i) sync_f[(size_t)s * 768 + i] = esv[i];
    std::vector<float> noise((size_t)T * dit->latent_dim), text((size_t)77 * 1024), t5((size_t)77 * 2048), gt(1024);
    for (size_t i = 0; i < noise.size(); ++i) noise[i] = (float)std::sin(0.37 * (double)i + seed);
    for (size_t i = 0; i < text.size(); ++i) text[i] = (float)std::cos(0.11 * (double)i + seed);
    for (size_t i = 0; i < t5.size(); ++i) t5[i] = (float)std::sin(0.05 * (double)i + 1.0 + seed);
    for (size_t i = 0; i < gt.size(); ++i) gt[i] = (float)std::cos(0.7 * (double)i + seed);
    return dit->sample(noise.data(), T, clip_f.data(), clip_S, sync_f.data(), sync_S, text.data(), t5.data(),
                       gt.data(), steps, 5.0f);
}

}  // namespace

int main(int argc, char ** argv) {
    if (argc < 5) {
        fprintf(stderr, "usage: ts_server_demo <dit.gguf> <steps> <out.bin> <T:seed> [<T:seed> ...]\n");
        return 2;
    }
    const int steps = atoi(argv[2]);
    FILE * fo = fopen(argv[3], "wb");
    if (!fo) return 4;
    for (int a = 4; a < argc; ++a) {
        const std::string spec = argv[a];
        const size_t c = spec.find(':');
        if (c == std::string::npos) { fclose(fo); return 2; }
        const int64_t T = atoll(spec.substr(0, c).c_str());
        const double seed = atof(spec.substr(c + 1).c_str());
        const auto t0 = std::chrono::steady_clock::now();
        const std::vector<float> lat = handle_request(argv[1], T, seed, steps);
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        if (lat.empty()) { fprintf(stderr, "request %d failed\n", a - 4); fclose(fo); return 3; }
        fwrite(lat.data(), 4, lat.size(), fo);
        printf("request %d T=%lld ms=%.2f\n", a - 4, (long long)T, ms);
    }
    fclose(fo);
    printf("loads=%d\n", g_loads);
    return 0;
}
