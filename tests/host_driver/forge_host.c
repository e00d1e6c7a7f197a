/*
 * forge_host.c — a C host that drives libforge_b200.so through
 * include/forge_b200.h exactly as the C# `B200Backend` shim does
 * (P/Invoke): create a model from host weights, open a session, and run
 * Sampler.Generate's loop (src/LLM.Core/Inference/Sampler.cs:78-109) with
 * the caller's own random stream pulled through FB2_RNG_CALLBACK and every
 * token streamed through the token callback (Program.cs:668-677 prints each
 * id as it is yielded).  Test infrastructure: tests/test_host_driver.py
 * builds and runs it and checks its output against the CPU oracle.
 *
 * Usage:  forge_host nodevice <garbage-checkpoint-path>
 *         forge_host run <uniforms-file> <n-uniforms>
 * The uniforms file holds the caller's NextDouble() stream as binary
 * doubles (`new Random(5)`'s values, written by the test).  Output: one JSON
 * object per line.
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "forge_b200.h"

/* The shim's Check(): status -> the exception type the reference throws. */
static const char* exception_of(int32_t st) {
    switch (st) {
        case FB2_OK: return "none";
        case FB2_INVALID_ARG: return "ArgumentException";
        case FB2_OUT_OF_MEMORY: return "OutOfMemoryException";
        case FB2_INVALID_DATA: return "InvalidDataException";
        case FB2_TIMEOUT: return "TimeoutException";
        default: return "InvalidOperationException";
    }
}

static void report(const char* what, int32_t st) {
    const char* msg = st ? fb2_last_error() : "";
    printf("{\"case\": \"%s\", \"status\": %d, \"exception\": \"%s\", \"message_len\": %d}\n", what, st,
           exception_of(st), (int)strlen(msg));
}

/* The caller's Random: a cursor over the pre-computed stream. */
typedef struct {
    const double* values;
    int n, next;
} Stream;

static double next_double(void* user, int32_t seq) {
    (void)seq;
    Stream* s = (Stream*)user;
    if (s->next >= s->n) return 0.0;  /* the test gives more values than any case draws */
    return s->values[s->next++];
}

typedef struct {
    int32_t tokens[256];
    int n, stop_after;
} Sink;

static int32_t on_token(void* user, int32_t seq, int32_t step, int32_t token) {
    (void)seq;
    Sink* k = (Sink*)user;
    if (k->n < 256) k->tokens[k->n++] = token;
    return (k->stop_after >= 0 && step >= k->stop_after) ? 1 : 0;
}

static void print_tokens(const char* what, const Sink* k, int draws) {
    printf("{\"case\": \"%s\", \"tokens\": [", what);
    for (int i = 0; i < k->n; i++) printf("%s%d", i ? ", " : "", k->tokens[i]);
    printf("], \"draws\": %d}\n", draws);
}

static int nodevice(const char* garbage_path) {
    /* What the shim can check without a GPU: version, symbols, and the
     * checkpoint rules (InvalidDataException, Checkpoint.cs:174-264). */
    printf("{\"case\": \"version\", \"abi\": %d}\n", fb2_version());
    fb2_model_desc d;
    report("garbage_checkpoint", fb2_forgemodel_read_header(garbage_path, &d, NULL, 0));
    report("null_session_seed", fb2_session_seed(NULL, 0, 1));
    return 0;
}

static int run(const char* upath, int nu) {
    double* uni = (double*)calloc((size_t)nu, sizeof(double));
    FILE* f = fopen(upath, "rb");
    if (!f || fread(uni, sizeof(double), (size_t)nu, f) != (size_t)nu) {
        fprintf(stderr, "cannot read %s\n", upath);
        return 2;
    }
    fclose(f);
    /* the model: GptModel(cfg, backend, new Random(11)) weights */
    fb2_model_desc desc = {96, 32, 64, 2, 4, FB2_WEIGHTS_FP32};
    const int np = 4 + 12 * desc.n_layers;
    const long long D = desc.d_model, F = 4 * D;
    long long numel[64];
    numel[0] = (long long)desc.vocab_size * D;
    numel[1] = (long long)desc.context_length * D;
    for (int l = 0; l < desc.n_layers; l++) {
        long long* q = numel + 2 + 12 * l;
        q[0] = D; q[1] = D; q[2] = D * 3 * D; q[3] = 3 * D; q[4] = D * D; q[5] = D;
        q[6] = D; q[7] = D; q[8] = D * F; q[9] = F; q[10] = F * D; q[11] = D;
    }
    numel[np - 2] = D;
    numel[np - 1] = D;
    float* params[64];
    for (int i = 0; i < np; i++) params[i] = (float*)malloc((size_t)numel[i] * sizeof(float));
    int32_t st = fb2_init_params(&desc, 11, params, np);
    report("init_params", st);
    fb2_model* model = NULL;
    st = fb2_model_create(&desc, (const float* const*)params, np, NULL, 0, &model);
    report("model_create", st);
    if (st) return 1;
    fb2_session* s = NULL;
    st = fb2_session_create(model, 1, &s);
    report("session_create", st);
    if (st) return 1;

    Stream rng = {uni, nu, 0};
    fb2_session_set_uniform_source(s, next_double, &rng);
    fb2_sampling sp = {0.8f, 10, 1.1f, 3, -1, 20};
    const int32_t prompt[5] = {5, 17, 3, 42, 8};
    int32_t plen = 5, out[64], count = 0;

    /* generate (Program.cs:664-677): streamed tokens, caller's stream */
    Sink k1 = {{0}, 0, -1};
    st = fb2_generate(s, 1, prompt, &plen, &sp, FB2_RNG_CALLBACK, NULL, NULL, out, &count, on_token, &k1);
    report("generate", st);
    print_tokens("generate", &k1, rng.next);

    /* chat (Program.cs:730-765): the same Random across turns, the whole
     * history resubmitted each turn */
    int32_t hist[128], hl = 0;
    memcpy(hist, prompt, sizeof prompt);
    hl = 5;
    for (int i = 0; i < k1.n; i++) hist[hl++] = k1.tokens[i];
    hist[hl++] = 7;
    hist[hl++] = 9;
    Sink k2 = {{0}, 0, -1};
    const int before = rng.next;
    sp.max_new_tokens = 6;
    st = fb2_generate(s, 1, hist, &hl, &sp, FB2_RNG_CALLBACK, NULL, NULL, out, &count, on_token, &k2);
    report("chat_turn2", st);
    print_tokens("chat_turn2", &k2, rng.next - before);

    /* the consumer stops early (the token callback returns nonzero): no
     * draw for tokens never asked for */
    Sink k3 = {{0}, 0, 3};
    const int before3 = rng.next;
    sp.max_new_tokens = 20;
    st = fb2_generate(s, 1, prompt, &plen, &sp, FB2_RNG_CALLBACK, NULL, NULL, out, &count, on_token, &k3);
    report("early_stop", st);
    print_tokens("early_stop", &k3, rng.next - before3);

    /* EOS (Sampler.cs:107): stops at the first sampled EOS, no later draw */
    Sink k4 = {{0}, 0, -1};
    const int before4 = rng.next;
    sp.eos_id = k1.tokens[2];
    st = fb2_generate(s, 1, prompt, &plen, &sp, FB2_RNG_CALLBACK, NULL, NULL, out, &count, NULL, NULL);
    report("eos", st);
    k4.n = count;
    for (int i = 0; i < count; i++) k4.tokens[i] = out[i];
    print_tokens("eos", &k4, rng.next - before4);
    sp.eos_id = -1;

    /* argument errors map to ArgumentException (Sampler.cs:85-89, 167-175;
     * GptModel.cs:288-299) */
    fb2_sampling bad = sp;
    bad.repetition_penalty = 0.9f;
    report("bad_penalty", fb2_generate(s, 1, prompt, &plen, &bad, FB2_RNG_CALLBACK, NULL, NULL, out, &count, NULL, NULL));
    const int32_t badtok[2] = {1, 96};
    int32_t two = 2;
    report("token_out_of_range", fb2_generate(s, 1, badtok, &two, &sp, FB2_RNG_CALLBACK, NULL, NULL, out, &count, NULL, NULL));
    bad = sp;
    bad.eos_id = 96;
    report("eos_out_of_vocab", fb2_generate(s, 1, prompt, &plen, &bad, FB2_RNG_CALLBACK, NULL, NULL, out, &count, NULL, NULL));
    fb2_session_set_uniform_source(s, NULL, NULL);
    report("no_rng", fb2_generate(s, 1, prompt, &plen, &sp, FB2_RNG_CALLBACK, NULL, NULL, out, &count, NULL, NULL));

    fb2_session_destroy(s);
    fb2_model_destroy(model);
    for (int i = 0; i < np; i++) free(params[i]);
    free(uni);
    return 0;
}

int main(int argc, char** argv) {
    if (argc >= 3 && !strcmp(argv[1], "nodevice")) return nodevice(argv[2]);
    if (argc >= 4 && !strcmp(argv[1], "run")) return run(argv[2], atoi(argv[3]));
    fprintf(stderr, "usage: forge_host nodevice <file> | run <uniforms-file> <n>\n");
    return 2;
}
