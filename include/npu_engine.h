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

/* Control plane (rust/npu-capi/src/lib.rs:129-214).  Exported for link compatibility; the
 * control plane itself is not part of this backend, so these report an error. */
NpuRuntime *npu_runtime_start(const char *config_path);
char *npu_runtime_transcribe(NpuRuntime *rt, const char *model, const int16_t *pcm, uintptr_t n,
                             uint32_t sample_rate);
int npu_runtime_embed(NpuRuntime *rt, const char *model, const char *text, float *out,
                      uintptr_t out_cap);
int npu_runtime_reload(NpuRuntime *rt);
char *npu_runtime_models_json(NpuRuntime *rt);
void npu_runtime_stop(NpuRuntime *rt);

#ifdef __cplusplus
}
#endif

#endif /* NPU_ENGINE_H */
