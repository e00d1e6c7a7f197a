/*
 * forge_b200.h — C ABI of libforge_b200.so, the B200 (sm_100a) decode library
 * behind ForgeLM's `--backend b200`.
 *
 * The library replaces everything below Sampler.Generate for the
 * autoregressive token loop of TitanUranus67/forge-lm:
 *   - src/LLM.Core/Inference/Sampler.cs:78-109   Sampler.Generate (token loop)
 *   - src/LLM.Core/Model/GptModel.cs:202-222     ForwardLast / ForwardCore
 *   - src/LLM.Core/Inference/Sampler.cs:14-165   Greedy, Sample, ApplyRepetitionControls
 * The C# side keeps checkpoint loading, the tokenizer and the CLI; it hands
 * the fp32 weights (Parameters.Names order, GptModel.cs:14-18) to
 * fb2_model_create and calls fb2_generate from a B200Backend that the
 * reference's BackendSelection (src/LLM.Core/Tensor/BackendSelection.cs:17-18)
 * selects by the name "b200".
 *
 * Conventions
 *   - Every entry point returns FB2_OK (0) or a negative fb2_status; nothing
 *     aborts or throws across the ABI.  fb2_last_error() gives a message for
 *     the calling thread's last failure.
 *   - Plain pointers and sizes only.  Host pointers unless a name says
 *     "device".  The library copies what it keeps; callers keep ownership.
 *   - A model is read-only after creation and may be shared by sessions.
 *     A session is used by one host thread at a time (the reference's CUDA
 *     backend serialises every call the same way, CudaBackend.cs:36,125).
 *   - Token ids are int32 in [0, vocab_size).  Arithmetic is fp32, or bf16
 *     weights with fp32 accumulation when weight_dtype = FB2_WEIGHTS_BF16.
 */
#ifndef FORGE_B200_H
#define FORGE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FB2_ABI_VERSION 1

/* Status codes.  The C# shim maps INVALID_ARG to ArgumentException /
 * ArgumentOutOfRangeException (Sampler.cs:85-89, GptModel.cs:279-299) and
 * the device errors to InvalidOperationException (CudaBackend.cs:213). */
typedef enum {
    FB2_OK = 0,
    FB2_INVALID_ARG = -1,
    FB2_OUT_OF_MEMORY = -2,
    FB2_CUDA_ERROR = -3,
    FB2_TIMEOUT = -4,      /* a bounded device wait gave up; the context stays usable */
    FB2_UNSUPPORTED = -5,  /* shape or option this build does not handle */
    FB2_NO_DEVICE = -6,
    FB2_INVALID_DATA = -7  /* a checkpoint file breaks the FORGEMODEL1 rules (InvalidDataException) */
} fb2_status;

/* FB2_WEIGHTS_BF16: the caller still passes fp32 arrays; the library rounds
 * tok_emb and the four projection matrices of every layer to the nearest
 * bf16 (ties to even) and computes with those values (fp32 accumulation,
 * fp32 LayerNorm, softmax, biases and position table).  The HBM-bound decode
 * kernels read 2-byte weights.  No reference counterpart: the reference
 * stores fp32 (Parameters, GptModel.cs:14-18). */
typedef enum { FB2_WEIGHTS_FP32 = 0, FB2_WEIGHTS_BF16 = 1 } fb2_weight_dtype;

/* ModelConfig (src/LLM.Core/Model/ModelConfig.cs:8-26): MlpHidden = 4*d_model,
 * HeadDim = d_model / n_heads. */
typedef struct {
    int32_t vocab_size;
    int32_t context_length;
    int32_t d_model;
    int32_t n_layers;
    int32_t n_heads;
    int32_t weight_dtype; /* fb2_weight_dtype */
} fb2_model_desc;

/* Arguments of Sampler.Generate (Sampler.cs:78-80). */
typedef struct {
    float temperature;        /* <= 0: greedy argmax, no RNG draw (Sampler.cs:35) */
    int32_t top_k;            /* <= 0 or >= vocab: no filtering (Sampler.cs:42) */
    float repetition_penalty; /* finite, >= 1 (Sampler.cs:167-175) */
    int32_t no_repeat_ngram;  /* >= 0; 0 disables */
    int32_t eos_id;           /* < 0: no EOS stop; else in [0, vocab) (Sampler.cs:87-88,107) */
    int32_t max_new_tokens;   /* >= 0 (Sampler.cs:86) */
} fb2_sampling;

/* Where the uniforms of categorical sampling (Sampler.cs:61) come from. */
typedef enum {
    /* seeds[i]: a fresh `new Random(seeds[i])` stream per sequence for this
     * call (Program.cs:664 creates one per generate). */
    FB2_RNG_SEEDS = 0,
    /* The stream kept in the session slot of each sequence, seeded by
     * fb2_session_seed and carried across calls (chat, Program.cs:730). */
    FB2_RNG_SESSION = 1,
    /* uniforms[i * max_new + n]: the caller's NextDouble() values. */
    FB2_RNG_UNIFORMS = 2,
    /* The uniform source set with fb2_session_set_uniform_source: the
     * library pulls one value per sampled token, so a caller that forwards
     * its own Random.NextDouble() (the `rng` Sampler.Generate receives,
     * Sampler.cs:78-80, 61) advances it by exactly the draws the reference
     * makes.  fb2_generate only. */
    FB2_RNG_CALLBACK = 3
} fb2_rng_mode;

/* Uniform source of FB2_RNG_CALLBACK: returns the next NextDouble() value of
 * sequence `seq`'s stream (in [0, 1)).  The library calls it once per
 * sampled token (temperature > 0), in step order, on the thread that called
 * fb2_generate or on one of the library's device threads, never two calls at
 * once.  A sequence draws for step n only after its tokens of steps < n are
 * known and it is still running: with eos_id >= 0 or a token callback the
 * draw for step n comes after the token callback of step n-1 returned, so a
 * sequence that sampled EOS, or a callback that asked to stop, draws no
 * more (as Sampler.Generate, a lazy iterator, draws no more).  Without EOS
 * and without a token callback every sequence emits max_new_tokens tokens,
 * and the library draws all of them (step by step, sequences in order)
 * before the first decode step. */
typedef double (*fb2_uniform_cb)(void* user, int32_t seq);

/* Per-token streaming callback (Program.cs:671-677 prints each id as it is
 * yielded).  Called on the thread that called fb2_generate, in step order,
 * once per emitted token.  Return nonzero to stop generation early. */
typedef int32_t (*fb2_token_cb)(void* user, int32_t seq, int32_t step, int32_t token);

typedef struct fb2_model fb2_model;
typedef struct fb2_session fb2_session;

typedef struct {
    int64_t tokens_generated;   /* ids emitted since the last reset */
    int64_t decode_steps;       /* KV-cached single-row steps run */
    int64_t prefill_rows;       /* rows pushed through full-window prefill */
    int64_t reprefills;         /* sliding-window re-prefills (Sampler.cs:93-94) */
    double prefill_ms;          /* device time (CUDA events) per phase */
    double decode_ms;
    double sample_ms;
    int64_t kernel_launches;    /* kernels the library launched (graph nodes counted) */
    int32_t device_count;
    int32_t reserved;
    int64_t persistent_steps;   /* decode steps run inside the persistent decode kernel */
    int64_t reused_prefix_rows; /* prompt positions whose K/V a previous generate left in the cache */
} fb2_stats_t;

/* ---- library ------------------------------------------------------------- */
int32_t fb2_version(void);
const char* fb2_last_error(void);
int32_t fb2_device_count(int32_t* n);

/* ---- model ----------------------------------------------------------------
 * Replaces GptModel construction + Checkpoint.LoadCore's upload
 * (Checkpoint.cs:207-227).  params[i] points to the fp32 host data of
 * parameter i in registration order (GptModel.cs:14-18, 47-98):
 *   tok_emb [V,D], pos_emb [ctx,D],
 *   blocks.{l}.{ln1.w, ln1.b, attn.qkv.w [D,3D], attn.qkv.b, attn.proj.w [D,D],
 *               attn.proj.b, ln2.w, ln2.b, mlp.fc.w [D,4D], mlp.fc.b,
 *               mlp.proj.w [4D,D], mlp.proj.b},
 *   ln_f.w, ln_f.b.
 * n_params must be 4 + 12*n_layers.  The weights are copied to every listed
 * device (devices == NULL: device 0 only). */
int32_t fb2_model_create(const fb2_model_desc* desc, const float* const* params, int32_t n_params,
                         const int32_t* devices, int32_t n_devices, fb2_model** out);
void fb2_model_destroy(fb2_model* m);

/* ---- session --------------------------------------------------------------
 * Owns per-sequence KV caches, token histories, RNG streams and the captured
 * decode-step graphs.  max_seqs sequences are split into contiguous blocks
 * over the model's devices. */
int32_t fb2_session_create(fb2_model* m, int32_t max_seqs, fb2_session** out);
void fb2_session_destroy(fb2_session* s);
/* Seeds the FB2_RNG_SESSION stream of slot `seq` as `new Random(seed)`. */
int32_t fb2_session_seed(fb2_session* s, int32_t seq, int32_t seed);
/* Sets the uniform source used by fb2_generate with FB2_RNG_CALLBACK (cb may
 * be NULL to clear it).  No reference counterpart as a function: it carries
 * Sampler.Generate's `Random rng` argument (Sampler.cs:78-80) across the ABI. */
int32_t fb2_session_set_uniform_source(fb2_session* s, fb2_uniform_cb cb, void* user);
/* Runs the session's work for device slot `device_slot` on the caller's
 * CUDA stream (a cudaStream_t passed as void*; NULL restores the library's
 * own stream). */
int32_t fb2_session_set_stream(fb2_session* s, int32_t device_slot, void* cuda_stream);

/* ---- the token loop -------------------------------------------------------
 * Sampler.Generate (Sampler.cs:78-109) for n_seqs independent sequences.
 * prompt_tokens holds the prompts back to back; prompt_lens[i] >= 1 each.
 * out_tokens is [n_seqs * max_new_tokens]; sequence i writes its ids at
 * out_tokens[i * max_new_tokens ...] and its count to out_counts[i] (fewer
 * than max_new_tokens only when EOS was sampled; the EOS id is included).
 * Results equal the reference loop: the window is truncated to the context
 * length before each forward (a longer window is re-prefilled in full),
 * repetition controls see the truncated window, one uniform is drawn per
 * sampled token when temperature > 0. */
int32_t fb2_generate(fb2_session* s, int32_t n_seqs, const int32_t* prompt_tokens,
                     const int32_t* prompt_lens, const fb2_sampling* sp, int32_t rng_mode,
                     const int32_t* seeds, const double* uniforms, int32_t* out_tokens,
                     int32_t* out_counts, fb2_token_cb cb, void* user);

/* The same loop with device-resident inputs and outputs (single-device
 * sessions): device_prompt_tokens/device_prompt_lens/device_uniforms and
 * device_out_tokens/device_out_counts are device pointers on the session's
 * device.  No host<->device copy is made and the call returns once the work
 * is enqueued on the session stream (no callback). */
int32_t fb2_generate_device(fb2_session* s, int32_t n_seqs, const int32_t* device_prompt_tokens,
                            const int32_t* device_prompt_lens, const int32_t* host_prompt_lens,
                            const fb2_sampling* sp, int32_t rng_mode, const int32_t* seeds,
                            const double* device_uniforms, int32_t* device_out_tokens,
                            int32_t* device_out_counts);

/* ---- parity hooks -----------------------------------------------------------
 * GptModel.ForwardLast (GptModel.cs:202-209) for n_seqs windows through the
 * library's prefill path: out_logits is [n_seqs * V]. */
int32_t fb2_forward_last_logits(fb2_session* s, int32_t n_seqs, const int32_t* tokens,
                                const int32_t* lens, float* out_logits);

/* Teacher-forced decode: for each sequence, prefill tokens[0..prompt_len)
 * and then feed tokens[prompt_len..len) one at a time through the KV-cached
 * decode step.  out_logits receives, per sequence, the last-row logits after
 * each prefix of length prompt_len..len: [n_seqs * (len - prompt_len + 1) * V].
 * All sequences share len and prompt_len; len <= context_length. */
int32_t fb2_teacher_forced_logits(fb2_session* s, int32_t n_seqs, const int32_t* tokens, int32_t len,
                                  int32_t prompt_len, float* out_logits);

/* Sampler.ApplyRepetitionControls + Sampler.Sample (Sampler.cs:29-69,
 * 96-104, 111-165) on the device for n logit rows of length V:
 * windows holds the windows back to back, window_lens[i] each;
 * uniforms[i] is the NextDouble() value for row i (ignored when
 * temperature <= 0).  out_ids[n]. */
int32_t fb2_sample_logits(fb2_session* s, int32_t n, const float* logits, const int32_t* windows,
                          const int32_t* window_lens, const fb2_sampling* sp, const double* uniforms,
                          int32_t* out_ids);

/* ---- forward_last without device allocation -----------------------------------
 * No counterpart in the reference: an addition for callers that cannot call
 * cudaMalloc — a host runtime that already owns the device's memory budget
 * through its own allocator (a cudaMalloc beside it fails or breaks its
 * accounting), or a latency-critical path where cudaMalloc's implicit device
 * synchronisation is not acceptable.
 *
 * Computes what fb2_forward_last_logits computes for ONE window of n_tokens
 * (1 <= n_tokens <= 16, and <= context_length) on the model copy of
 * device_slot: device_tokens (n_tokens int32) and device_logits (vocab_size
 * floats) are the caller's device buffers on that device.  All intermediate
 * data lives in a fixed 8 MiB device array inside the library (reserved on
 * every GPU that loads it, until the process exits); the call allocates
 * nothing, enqueues its kernels on cuda_stream (a cudaStream_t as void*) and
 * returns without waiting.  Models whose intermediates exceed the 8 MiB
 * (roughly d_model > 1024 or many layers), or whose split-K partial sums
 * for this window exceed its region, are rejected with FB2_UNSUPPORTED
 * before anything is enqueued; longer windows with FB2_INVALID_ARG.  Token ids are not range-checked on
 * the host (they stay on the device); ids outside [0, vocab) read as id 0.
 * The first call on a device looks up the array's device address; make that
 * first call before any stream capture begins.  Every call shares the one
 * array: calls whose work overlaps on the GPU (different streams, or other
 * host threads) race and corrupt each other's results. */
int32_t fb2_forward_last_logits_noalloc(fb2_model* m, int32_t device_slot, int32_t n_tokens,
                                        const int32_t* device_tokens, float* device_logits, void* cuda_stream);

/* ---- synthetic weights -------------------------------------------------------
 * Host-only: fills params[i] (caller-allocated fp32 arrays of the sizes listed
 * at fb2_model_create) with the weights `new GptModel(config, backend,
 * new Random(seed))` creates (GptModel.cs:47-98; Box-Muller in double,
 * Tensor.cs:79-91): tok_emb, pos_emb, qkv.w, fc.w ~ N(0, 0.02); attn.proj.w,
 * mlp.proj.w ~ N(0, 0.02/sqrt(2L)); LayerNorm weights 1; biases 0. */
int32_t fb2_init_params(const fb2_model_desc* desc, int32_t seed, float* const* params, int32_t n_params);

/* ---- statistics -------------------------------------------------------------- */
int32_t fb2_stats(fb2_session* s, fb2_stats_t* out);
int32_t fb2_stats_reset(fb2_session* s);

/* ---- FORGEMODEL1 checkpoints (src/LLM.Core/Checkpoint/Checkpoint.cs) ----------
 * File: "FORGEMODEL1", int32 LE header length, UTF-8 JSON header, fp32 LE
 * parameters in registry order (+ Adam moments when the header says so),
 * SHA-256 of everything before the 32-byte trailer.  Every rule
 * Checkpoint.LoadCore (Checkpoint.cs:174-264) enforces returns
 * FB2_INVALID_DATA with its message; the checksum is verified before any
 * weight is used. */

/* Validates the whole file and returns its model configuration (weight_dtype
 * FB2_WEIGHTS_FP32) and ModelName (NUL-terminated, truncated to
 * name_capacity - 1 bytes; name may be NULL).  No device needed.  Replaces
 * Checkpoint.LoadWithMetadata's header half (Checkpoint.cs:124-125). */
int32_t fb2_forgemodel_read_header(const char* path, fb2_model_desc* out_desc, char* name, int32_t name_capacity);

/* Checkpoint.Load (Checkpoint.cs:121-122) straight into device memory: the
 * validated file's weights go to fb2_model_create (weight_dtype as there).
 * out_desc (may be NULL) receives the configuration. */
int32_t fb2_model_load_forgemodel(const char* path, int32_t weight_dtype, const int32_t* devices, int32_t n_devices,
                                  fb2_model_desc* out_desc, fb2_model** out);

/* Writes params (registry order, fp32) as a FORGEMODEL1 model checkpoint in
 * the layout Checkpoint.SaveTraining writes (Checkpoint.cs:63-119, 143-166),
 * with a Training header that records no optimizer state. */
int32_t fb2_forgemodel_write(const char* path, const fb2_model_desc* desc, const char* model_name,
                             const float* const* params, int32_t n_params);

/* ---- Byte-level BPE tokenizer (src/LLM.Core/Tokenizer/BpeTokenizer.cs) --------
 * Host only (no device).  fb2_tokenizer_load reads the JSON BpeTokenizer.Save
 * writes and applies BpeTokenizer.Load's checks (BpeTokenizer.cs:353-389):
 * FB2_INVALID_DATA where it throws InvalidDataException. */
typedef struct fb2_tokenizer fb2_tokenizer;
int32_t fb2_tokenizer_load(const char* path, fb2_tokenizer** out);
void fb2_tokenizer_destroy(fb2_tokenizer* t);
/* VocabSize (bytes + merges + EOS) and EosTokenId. */
int32_t fb2_tokenizer_info(const fb2_tokenizer* t, int32_t* vocab_size, int32_t* eos_id);
/* BpeTokenizer.Encode(ReadOnlySpan<byte>) (BpeTokenizer.cs:259-318): *n_ids
 * receives the count; FB2_INVALID_ARG when it exceeds capacity (ids then
 * untouched). */
int32_t fb2_tokenizer_encode(const fb2_tokenizer* t, const uint8_t* bytes, int64_t n_bytes, int32_t* ids,
                             int64_t capacity, int64_t* n_ids);
/* The bytes BpeTokenizer.Decode concatenates before its UTF-8 conversion
 * (BpeTokenizer.cs:320-339; the EOS token adds none).  An id outside the
 * vocabulary is FB2_INVALID_ARG (ArgumentOutOfRangeException); *n_bytes as
 * in fb2_tokenizer_encode. */
int32_t fb2_tokenizer_decode(const fb2_tokenizer* t, const int32_t* ids, int64_t n_ids, uint8_t* bytes,
                             int64_t capacity, int64_t* n_bytes);

#ifdef __cplusplus
}
#endif
#endif /* FORGE_B200_H */
