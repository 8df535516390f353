/* tsd.h — C-ABI of libtsd_b200: the B200-native (sm_100a) MM-DiT hot path of thinksound.cpp.
 *
 * Drop-in boundary for the reference's `ts_dit` (src/mmdit.h:9-42 in pwilkin/thinksound.cpp):
 * load a DiT GGUF, run one velocity evaluation (forward) or the full CFG rectified-flow sampler
 * (sample). Plain pointers and sizes only; every call returns a status code (never aborts).
 * Host layouts are the reference's (mmdit.h:19-40):
 *   latent / noise / sample output  [latent_dim][T]      (t fastest)
 *   clip_f [clip_S][1024], sync_f [sync_S][768], text_f [text_S][1024], t5 [t5_S][2048],
 *   global_text [1024]
 *   forward output (flow)           [T][latent_dim]      (channel fastest)
 * text_S and t5_S are separate (the reference hard-wires both to 77, mmdit.cpp:130,141-142);
 * the joint text stream is [text_f padded to 2048 | t5] of text_S + t5_S tokens.
 * Threading: a model is not re-entrant; serialise calls per model (as ts-server does).
 */
#ifndef TSD_H
#define TSD_H

#include <stddef.h>
#include <stdint.h>

#ifndef TSD_API
#if defined(__GNUC__)
#define TSD_API __attribute__((visibility("default")))
#else
#define TSD_API
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define TSD_OK 0
#define TSD_ERR_ARG (-1)          /* bad argument / unsupported shape */
#define TSD_ERR_CUDA (-2)         /* CUDA runtime error (message on stderr) */
#define TSD_ERR_IO (-3)           /* file cannot be read / is not a valid GGUF */
#define TSD_ERR_MISSING (-4)      /* a required tensor is missing (name on stderr) */
#define TSD_ERR_DEVICE (-5)       /* a kernel's bounded wait expired (device error word set) */
#define TSD_ERR_UNSUPPORTED (-6)  /* tensor type or configuration not supported */
#define TSD_ERR_STATE (-7)        /* call out of order (e.g. model not finalised) */

typedef struct tsd_model tsd_model;

/* Model hyper-parameters (GGUF keys dit.*, read as in mmdit.cpp:108-115). */
typedef struct tsd_hparams {
    int32_t hidden;        /* dit.hidden_dim        (default 1024) */
    int32_t n_head;        /* dit.num_heads         (default 16); head_dim = hidden / n_head = 64 */
    int32_t depth;         /* dit.depth             (default 21) */
    int32_t fused_depth;   /* dit.fused_depth       (default 14) */
    int32_t latent_dim;    /* dit.latent_dim        (default 64) */
    float rope_theta;      /* dit.rope_theta        (default 10000) */
    float t_max_period;    /* dit.t_embed_max_period (default 1) */
} tsd_hparams;

/* Replaces ts_dit::load (mmdit.cpp:105-117) + ts_model::load_backend (ts_model.cpp:13-41):
 * reads the GGUF, uploads every tensor to `device`, repacks the projection weights. */
TSD_API int tsd_load_gguf(const char * path, int device, tsd_model ** out);

/* Programmatic construction: the same per-tensor path the GGUF loader takes
 * (ts_model.cpp:65-77). `ggml_type` is the ggml type id (0 F32, 1 F16, 8 Q8_0, 30 BF16),
 * `ne` the ggml shape (ne[0] fastest; unused dims 1). `data` may be host or device memory. */
TSD_API int tsd_model_create(const tsd_hparams * hp, int device, tsd_model ** out);
TSD_API int tsd_model_set_tensor(tsd_model * m, const char * name, int ggml_type, const int64_t ne[4],
                         const void * data, size_t nbytes);
TSD_API int tsd_model_finalize(tsd_model * m);
TSD_API void tsd_model_free(tsd_model * m);
TSD_API int tsd_model_get_hparams(const tsd_model * m, tsd_hparams * out);

/* ts_model::need + get_data facade (ts_model.h:24-27): copy a stored tensor to host as f32
 * (dequantised). `ne_out` may be NULL. Returns TSD_ERR_MISSING for an unknown name. */
TSD_API int tsd_get_tensor_f32(const tsd_model * m, const char * name, float * dst, int64_t n_dst, int64_t ne_out[4]);

/* ts_dit::forward (mmdit.cpp:119-342) for one item; flow_out [T][latent_dim]. */
TSD_API int tsd_forward(tsd_model * m, const float * latent, int64_t T, float t, const float * clip_f, int64_t clip_S,
                const float * sync_f, int64_t sync_S, const float * text_f, int64_t text_S, const float * t5,
                int64_t t5_S, const float * global_text, float * flow_out);

/* Batched forward: B items, every input stacked along a leading batch dimension, per-item t.
 * Optional stage capture: dbg(ud, name, data, n) is called for the named intermediates of
 * mmdit.cpp:333-337 (x_in, t_emb, clip_pp, text_pp, clip_fc, text_fc, gcmlp, global_c,
 * extended_c, text_xn, a0_q, a0_k, a0_v, a0_out, jb0_lat, jb0_clip, jb0_text, after_joint,
 * after_fused, flow_cl) with host f32 data of all B items ([B][...] token-major). */
typedef void (*tsd_dbg_fn)(void * ud, const char * name, const float * data, int64_t n);
TSD_API int tsd_forward_batched(tsd_model * m, int B, const float * latent, int64_t T, const float * t,
                        const float * clip_f, int64_t clip_S, const float * sync_f, int64_t sync_S,
                        const float * text_f, int64_t text_S, const float * t5, int64_t t5_S,
                        const float * global_text, float * flow_out, tsd_dbg_fn dbg, void * ud);

/* Stage capture with teacher forcing, for parity tests (the reference's dit_test compares the
 * stages of one free-running forward, src/tools/dit_test.cpp:38-59; this also lets a test start
 * every block from the same input as the reference). Like tsd_forward_batched with `dbg`, which
 * additionally receives every block's output ("blk<i>_lat", "blk<i>_clip", "blk<i>_text"; i
 * counts the joint blocks, then the fused blocks) and the residual stream after the attention
 * half of each block ("blk<i>_attn_lat" ...). Before block i runs, inject(ud, name, data, n) is
 * offered each residual stream the block reads ("blk<i>_in_lat", "blk<i>_in_clip",
 * "blk<i>_in_text"; before the final layer "final_in_lat"), host f32 [B][S][hidden]; if it
 * returns non-zero, its (modified) data replace the stream; "blk<i>_mid_<stream>" is offered
 * between a block's attention half and its FFN half. The conditioning the blocks'
 * adaLN projections read is offered the same way ("global_c" [B][hidden], "extended_c"
 * [B][T][hidden]). Runs op by op, without a graph. */
typedef int (*tsd_inject_fn)(void * ud, const char * name, float * data, int64_t n);
TSD_API int tsd_forward_inject(tsd_model * m, int B, const float * latent, int64_t T, const float * t,
                               const float * clip_f, int64_t clip_S, const float * sync_f, int64_t sync_S,
                               const float * text_f, int64_t text_S, const float * t5, int64_t t5_S,
                               const float * global_text, float * flow_out, tsd_dbg_fn dbg, tsd_inject_fn inject,
                               void * ud);

/* Device-resident forward: same layouts, all pointers in device memory of the model's GPU,
 * enqueued on `stream` (cudaStream_t; NULL = default stream) without host synchronisation.
 * Inputs are read and flow_out written in stream order. Call tsd_sync_check afterwards to
 * synchronise and collect device-side errors. */
TSD_API int tsd_forward_device(tsd_model * m, int B, const float * latent, int64_t T, const float * t,
                       const float * clip_f, int64_t clip_S, const float * sync_f, int64_t sync_S,
                       const float * text_f, int64_t text_S, const float * t5, int64_t t5_S,
                       const float * global_text, float * flow_out, void * stream);
TSD_API int tsd_sync_check(tsd_model * m, void * stream);

/* ts_dit::sample (mmdit.cpp:344-376): `steps` Euler steps t = 1 - s/steps with CFG
 * v = u + (c - u) * cfg; uncond uses empty_string_feat, empty_t5_feat and a zero global
 * vector. noise / out / flow0 are [latent_dim][T]; flow0 may be NULL. */
TSD_API int tsd_sample(tsd_model * m, const float * noise, int64_t T, const float * clip_f, int64_t clip_S,
               const float * sync_f, int64_t sync_S, const float * text_f, int64_t text_S, const float * t5,
               int64_t t5_S, const float * global_text, int steps, float cfg, float * out, float * flow0);

/* Batched sampler over P independent prompts (inputs stacked along a leading P dimension);
 * cond and uncond of every prompt run as one batch of 2P, CFG + Euler update on the device. */
TSD_API int tsd_sample_batched(tsd_model * m, int P, const float * noise, int64_t T, const float * clip_f, int64_t clip_S,
                       const float * sync_f, int64_t sync_S, const float * text_f, int64_t text_S,
                       const float * t5, int64_t t5_S, const float * global_text, int steps, float cfg,
                       float * out, float * flow0);

/* Head-parallel mode (optional; for long inputs such as 30 s). No counterpart API exists in the
 * reference, which runs one GGML backend per process; this splits the attention heads of
 * mmdit.cpp:85-94,219 across the GPUs of one node, one process per GPU, each with its own model
 * loaded from the same weights. Rank r computes heads [h0, h0 + n_head / world) of every joint
 * and fused block (QKV rows and attention) and writes their attention rows into every rank's
 * exchange buffer over NVLink; all other work is replicated, so every rank returns the full
 * result. Call tsd_hp_init on every rank, exchange the TSD_IPC_HANDLE_BYTES handles (rank
 * order), then call tsd_hp_connect on every rank before the first forward. All ranks must then
 * issue the same forwards (same shapes, same order); a forward completes only after its peers'
 * rows of every layer arrived (bounded wait: a missing peer ends in TSD_ERR_DEVICE, after which
 * the group must be set up again with new models). `arena_bytes` bounds the exchange buffers
 * of all plans built in this mode (B * S * hidden * 2 bytes per layer and input shape; never
 * reused). Needs bf16 QKV weights (not TSD_Q8_IN_KERNEL). Free the models only after every
 * rank's last forward has returned. */
#define TSD_IPC_HANDLE_BYTES 64
TSD_API int tsd_hp_layout(int hidden, int n_head, int world, int rank, int32_t out[3]); /* h0, heads, rows per Q/K/V section */
TSD_API int tsd_hp_init(tsd_model * m, int rank, int world, size_t arena_bytes, void * handle_out);
TSD_API int tsd_hp_connect(tsd_model * m, const void * handles);

/* Deadline of every bounded device-side wait of the library's kernels on `device` (mbarrier
 * waits of the GEMM and attention pipelines, the cluster split-K handshakes, the head-parallel
 * arrival wait), in nanoseconds, 1 ms to 60 s; 2 s by default. A wait that runs out records an
 * error in the model's device error word and its kernel returns; the call then reports
 * TSD_ERR_DEVICE. No counterpart in the reference, whose GGML kernels have no device-side
 * waits. Call it while no kernel of the library runs on the device. */
TSD_API int tsd_set_wait_limit(int device, uint64_t ns);

/* Library / device information. */
TSD_API const char * tsd_version(void);
TSD_API int tsd_device_count(void);

#ifdef __cplusplus
}
#endif

#endif /* TSD_H */
