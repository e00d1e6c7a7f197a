/*
 * forge_oracle.h — CPU restatement of ForgeLM's reference decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker and the timed
 * CPU baseline; it is never linked into, called by, or shipped with the B200
 * product library.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load it.
 *
 * Every function restates the C# reference (TitanUranus67/forge-lm, paths
 * relative to that project) and cites the file:line it follows.
 *
 * Parity status:
 *   - Forward numerics, sampler and repetition controls: restated from the
 *     reference source and pinned against the known-answer tests of
 *     tests/LLM.Core.Tests/{InferenceTests,CpuBackendTests,ModelTests}.cs
 *     (restated in tests/golden/known_answers.json).
 *   - System.Random (.NET BCL, not part of the reference tree): restated from
 *     its published algorithm (Knuth subtractive generator, TAOCP vol. 2
 *     3.2.2, in the .NET "compat" seeding variant).  No reference test pins
 *     its output and no .NET runtime exists here: RNG-stream parity with real
 *     .NET is "parity unpinned".
 */
#ifndef FORGE_ORACLE_H
#define FORGE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- System.Random (compat seeded generator) ------------------------------ */
typedef struct {
    int32_t seed_array[56];
    int32_t inext, inextp;
} orc_dotnet_random;

void   orc_random_init(orc_dotnet_random* r, int32_t seed);
int32_t orc_random_internal_sample(orc_dotnet_random* r);
double orc_random_next_double(orc_dotnet_random* r);
/* Fills out[0..n) with successive NextDouble() values. */
void   orc_random_next_doubles(orc_dotnet_random* r, double* out, int64_t n);

/* ---- Model config / parameters ------------------------------------------- */
typedef struct {
    int32_t vocab_size, context_length, d_model, n_layers, n_heads;
} orc_config;

/* Number of parameter tensors: 2 + 12*L + 2 (registration order). */
int32_t orc_param_count(const orc_config* c);
/* Element count of parameter tensor `index` in registration order. */
int64_t orc_param_numel(const orc_config* c, int32_t index);
/* Total scalar parameters. */
int64_t orc_total_params(const orc_config* c);
/* Writes the registry name of tensor `index` into buf (NUL-terminated). */
int32_t orc_param_name(const orc_config* c, int32_t index, char* buf, int32_t buflen);

/* GptModel constructor init: fills params[i] (caller-allocated, numel each)
 * in registration order from `new Random(seed)`. */
void orc_model_init(const orc_config* c, int32_t seed, float* const* params);

/* ---- Forward ---------------------------------------------------------------- */
/* Full forward over T tokens (GptModel.ForwardCore, batch 1): logits [T, V].
 * Returns 0, or -1 on invalid arguments. */
int32_t orc_forward(const orc_config* c, const float* const* params,
                    const int32_t* tokens, int32_t T, float* logits);
/* ForwardLast: logits of the last position [V]. */
int32_t orc_forward_last(const orc_config* c, const float* const* params,
                         const int32_t* tokens, int32_t T, float* logits_last);

/* ---- Sampler ------------------------------------------------------------------ */
int32_t orc_greedy(const float* logits, int32_t v);
/* Sampler.Sample with an explicit NextDouble() draw `u` (ignored when
 * temperature <= 0).  Returns the id, or -1 for invalid arguments. */
int32_t orc_sample(const float* logits, int32_t v, float temperature, int32_t top_k, double u);
/* Sampler.ApplyRepetitionControls, in place.  Returns 0 or -1 (invalid options). */
int32_t orc_apply_repetition_controls(float* logits, int32_t v, const int32_t* history,
                                      int32_t history_len, float repetition_penalty,
                                      int32_t no_repeat_ngram);
/* Sampling step used by Generate: copies logits, applies controls when
 * enabled, samples.  Consumes one NextDouble from rng iff temperature > 0. */
int32_t orc_sample_step(const float* logits, int32_t v, const int32_t* window, int32_t window_len,
                        float temperature, int32_t top_k, float repetition_penalty,
                        int32_t no_repeat_ngram, orc_dotnet_random* rng);

/* Sampler.Generate with the reference algorithm (full re-forward of the
 * window for every token, no KV cache).  eos_id < 0 means none.
 * Writes up to max_new ids into out_tokens; returns the count, or -1.
 * If out_logits is non-NULL it receives the [count, V] last-row logits that
 * each step sampled from (before repetition controls). */
int32_t orc_generate(const orc_config* c, const float* const* params,
                     const int32_t* prompt, int32_t prompt_len, int32_t max_new,
                     float temperature, int32_t top_k, orc_dotnet_random* rng, int32_t eos_id,
                     float repetition_penalty, int32_t no_repeat_ngram,
                     int32_t* out_tokens, float* out_logits);

/* Same loop driven by caller-supplied uniforms (one per sampled token) in
 * place of a System.Random stream. */
int32_t orc_generate_uniforms(const orc_config* c, const float* const* params,
                              const int32_t* prompt, int32_t prompt_len, int32_t max_new,
                              float temperature, int32_t top_k, const double* uniforms,
                              int32_t eos_id, float repetition_penalty, int32_t no_repeat_ngram,
                              int32_t* out_tokens, float* out_logits);

/* Single reference kernels, exposed for the known-answer tests. */
void orc_gelu_array(const float* x, float* y, int64_t n);                 /* CpuBackend.cs:485-514 */
void orc_layer_norm_rows(const float* x, const float* w, const float* b, float* out,
                         int32_t rows, int32_t cols);                      /* CpuBackend.cs:377-398 */
void orc_softmax_rows(float* x, int32_t rows, int32_t cols);             /* CpuBackend.cs:446-458 */

/* Threads used by the parallel matmul path (0 = all available). */
void orc_set_threads(int32_t n);
int32_t orc_get_threads(void);

/* Host libm expf, exposed so tests can compare device exponentials against it. */
void orc_expf_array(const float* x, float* y, int64_t n);
/* Scans every float bit pattern in [lo_bits, hi_bits] (as uint32 ranges of
 * non-negative or negative floats) and counts inputs where expf(x) differs
 * from (float)exp((double)x); up to max_out such inputs are written. */
int64_t orc_expf_vs_double_scan(uint32_t lo_bits, uint32_t hi_bits, uint32_t* out_bits, int64_t max_out);

/* Host twin of the library's fb2_test_expf_hash: per chunk of 2^20
 * consecutive float bit patterns, the same order-independent 64-bit hash of
 * expf's output bits (NaN inputs hash as output 0). */
void orc_expf_hash(uint32_t lo_bits, int32_t nchunks, uint64_t* hashes);

#ifdef __cplusplus
}
#endif
#endif
