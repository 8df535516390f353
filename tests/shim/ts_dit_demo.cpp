// ts_dit_demo.cpp — exercises include/ts_dit.hpp the way the reference's tools use ts_dit
// (src/tools/generate.cpp:81-89, dit_test.cpp:38-44): load, read the learned empties through
// model.need + model.get_data, one forward with the dbg stage map, and a short sample.
//   ts_dit_demo <dit.gguf> <T> <clip_S> <sync_S> <steps> [out.bin]
// Inputs are deterministic: noise[i] = sin(0.37 i), text[i] = cos(0.11 i), t5[i] = sin(0.05 i + 1),
// global[i] = cos(0.7 i); clip/sync rows are the learned empties. Prints the dbg names and
// writes flow [T][64] then latent [64][T] (f32) to out.bin; exit 1 if load fails.
#include "ts_dit.hpp"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

int main(int argc, char ** argv) {
    if (argc < 6) { fprintf(stderr, "usage: ts_dit_demo <dit.gguf> <T> <clip_S> <sync_S> <steps>\n"); return 2; }
    const int64_t T = atoi(argv[2]), clip_S = atoi(argv[3]), sync_S = atoi(argv[4]);
    const int steps = atoi(argv[5]);
    ts_dit dit;
    if (!dit.load(argv[1])) { fprintf(stderr, "load failed\n"); return 1; }
    ggml_tensor * ec = dit.model.need("empty_clip_feat");
    ggml_tensor * es = dit.model.need("empty_sync_feat");
    std::vector<float> ecv(1024), esv(768);
    dit.model.get_data(ec, ecv.data());
    dit.model.get_data(es, esv.data());
    std::vector<float> clip_f((size_t)1024 * clip_S), sync_f((size_t)768 * sync_S);
    for (int s = 0; s < clip_S; ++s) for (int i = 0; i < 1024; ++i) clip_f[(size_t)s * 1024 + i] = ecv[i];
    for (int s = 0; s < sync_S; ++s) for (int i = 0; i < 768; ++i) sync_f[(size_t)s * 768 + i] = esv[i];
    std::vector<float> noise((size_t)T * dit.latent_dim), text((size_t)77 * 1024), t5((size_t)77 * 2048), gt(1024);
    for (size_t i = 0; i < noise.size(); ++i) noise[i] = std::sin(0.37 * (double)i);
    for (size_t i = 0; i < text.size(); ++i) text[i] = std::cos(0.11 * (double)i);
    for (size_t i = 0; i < t5.size(); ++i) t5[i] = std::sin(0.05 * (double)i + 1.0);
    for (size_t i = 0; i < gt.size(); ++i) gt[i] = std::cos(0.7 * (double)i);
    std::map<std::string, std::vector<float>> dbg;
    std::vector<float> flow = dit.forward(noise.data(), T, 1.0f, clip_f.data(), clip_S, sync_f.data(), sync_S,
                                          text.data(), t5.data(), gt.data(), &dbg);
    std::vector<float> latent = dit.sample(noise.data(), T, clip_f.data(), clip_S, sync_f.data(), sync_S, text.data(),
                                           t5.data(), gt.data(), steps, 5.0f);
    if (flow.empty() || latent.empty()) return 3;
    if (argc > 6) {
        FILE * fo = fopen(argv[6], "wb");
        if (!fo) return 4;
        fwrite(flow.data(), 4, flow.size(), fo);
        fwrite(latent.data(), 4, latent.size(), fo);
        fclose(fo);
    }
    printf("dbg");
    for (auto & kv : dbg) printf(" %s", kv.first.c_str());
    printf("\n");
    return 0;
}
