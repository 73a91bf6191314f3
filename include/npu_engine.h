/*
 * npu_engine.h -- the reference's public C ABI, exported unchanged by the B200 backend
 * (libxdna_b200.so).  Same names, signatures, ownership and error rules as
 * rust/npu-capi/include/npu_engine.h:28-103 (implementation rust/npu-capi/src/lib.rs:22-214),
 * so an embedder written against the reference links against this library instead.
 *
 * Conventions: opaque handles freed only by their *_free / *_stop; strings returned by the
 * library are malloc'd and freed by npu_string_free; failures return NULL or -1 and leave a
 * thread-local message for npu_last_error (valid until the next call on that thread); no C++
 * exception crosses the boundary.  A model handle must not be driven by two threads at once.
 */
#ifndef NPU_ENGINE_H
#define NPU_ENGINE_H

#include <stdint.h>

typedef struct NpuModel NpuModel;
typedef struct NpuRuntime NpuRuntime;

#ifdef __cplusplus
extern "C" {
#endif

/* 1 if a usable device is present (here: an sm_100 GPU), else 0.  (lib.rs:22-25) */
int npu_available(void);
/* Load a model from a scenario TOML path (scenario / model / artifacts / embeddings tables,
 * artifacts relative to the current directory).  NULL on error.  (lib.rs:27-43) */
NpuModel *npu_model_load(const char *scenario_path);
/* 0 = asr, 1 = embed, -1 = error.  (lib.rs:45-52) */
int npu_model_kind(const NpuModel *m);
/* ASR: 16 kHz mono PCM -> malloc'd UTF-8 text (free with npu_string_free); NULL on error.
 * (lib.rs:54-71) */
char *npu_transcribe(NpuModel *m, const int16_t *pcm, uintptr_t n, uint32_t sample_rate);
/* Embedding: with out == NULL or out_cap == 0 returns the dimension; otherwise copies
 * min(dim, out_cap) floats and returns the full dimension; -1 on error.  (lib.rs:73-98) */
int npu_embed(NpuModel *m, const char *text, float *out, uintptr_t out_cap);
/* Free a string returned by this library (NULL is ignored).  (lib.rs:100-105) */
void npu_string_free(char *s);
/* Free a model handle (NULL is ignored).  (lib.rs:107-112) */
void npu_model_free(NpuModel *m);
/* Thread-local last error ("" if none).  (lib.rs:114-119) */
const char *npu_last_error(void);

/* Control plane (rust/npu-capi/src/lib.rs:125-214 over rust/npu-runtime): one worker thread per
 * GPU, each holding a replica of every configured model; requests go to the least-busy worker.
 * Config TOML as npu-runtime's config.rs ([server], [defaults], [[model]] name / scenario) plus
 * `[server] gpus = N`; a missing file is the empty config.  All calls are thread safe. */
/* Start from a config path (loads its models on every GPU).  NULL on error.  (lib.rs:129-144) */
NpuRuntime *npu_runtime_start(const char *config_path);
/* ASR through the control plane (model name or NULL for the default).  Caller frees.
 * (lib.rs:146-160) */
char *npu_runtime_transcribe(NpuRuntime *rt, const char *model, const int16_t *pcm, uintptr_t n,
                             uint32_t sample_rate);
/* Embedding through the control plane: copies min(dim, out_cap) floats, returns dim; -1 on
 * error.  (lib.rs:162-182) */
int npu_runtime_embed(NpuRuntime *rt, const char *model, const char *text, float *out,
                      uintptr_t out_cap);
/* Re-read the config file and reconcile every GPU.  0 / -1.  (lib.rs:184-192) */
int npu_runtime_reload(NpuRuntime *rt);
/* Model statuses as JSON (http.rs:55-66 plus "replicas" and "devices"); free with
 * npu_string_free.  (lib.rs:194-203) */
char *npu_runtime_models_json(NpuRuntime *rt);
/* Stop the workers (their models are freed on their GPUs) and free the handle.  (lib.rs:205-214) */
void npu_runtime_stop(NpuRuntime *rt);

#ifdef __cplusplus
}
#endif

#endif /* NPU_ENGINE_H */
