/*
 * forge_b200_testing.h — test hooks exported by libforge_b200.so.
 *
 * Not part of the reference-facing surface (no counterpart in
 * TitanUranus67/forge-lm).  The GPU tests use them to prove that the device
 * exponential of the sampler equals the host C runtime's expf, which the
 * reference sampler calls as MathF.Exp (src/LLM.Core/Inference/Sampler.cs:57).
 */
#ifndef FORGE_B200_TESTING_H
#define FORGE_B200_TESTING_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* y[i] = device exponential of x[i] (host arrays, n > 0). */
int32_t fb2_test_expf(const float* x, float* y, int64_t n);

/* For each chunk c < nchunks of 2^20 consecutive float bit patterns starting
 * at lo_bits + c * 2^20: an order-independent 64-bit hash of the device
 * exponential's output bits (NaN inputs hash as output 0). */
int32_t fb2_test_expf_hash(uint32_t lo_bits, int32_t nchunks, uint64_t* hashes);

/* n successive NextDouble() values of `new Random(seed)` as the library's
 * FB2_RNG_SEEDS mode draws them (host only; no device needed). */
int32_t fb2_test_dotnet_random(int32_t seed, int32_t n, double* out);

struct fb2_session;
/* The persistent decode kernel's per-phase %globaltimer stamps of the first
 * steps of its last launch, when the session was created with
 * FORGE_B200_MK_TRACE=<steps>: out is [CTAs][steps][64] uint64. */
int32_t fb2_test_mk_trace(struct fb2_session* s, uint64_t* out, int64_t capacity, int32_t* n_ctas,
                          int32_t* n_steps);

/* Failure detection without a GPU fault.  The next persistent-kernel launch
 * of the session's first device: CTA `cta` does not publish its q words of
 * that launch's first step (layer 0), and every bounded wait of the launch
 * gives up after wait_ns (<= 2 s) instead of 2 s.  The waiting CTAs record a
 * timeout, leave together, and the call returns FB2_TIMEOUT; the session
 * stays usable. */
int32_t fb2_test_mk_withhold(struct fb2_session* s, int32_t cta, int64_t wait_ns);

/* Geometry of the session's persistent decode kernel on its first device:
 * CTAs, cluster size and attention CTAs of the head-cluster layout (0 when
 * it uses column strips), and ring stages at one row. */
int32_t fb2_test_mk_geometry(struct fb2_session* s, int32_t* n_ctas, int32_t* cluster, int32_t* attn_ctas,
                             int32_t* stages);

/* Host-side allocation failure: the nth device allocation the library makes
 * from now on (counted over the process) fails as cudaMalloc's
 * out-of-memory would (FB2_OUT_OF_MEMORY); nth = 0 turns the hook off.
 * allocs_so_far (may be NULL) receives the allocations made so far. */
int32_t fb2_test_fail_alloc(int64_t nth, int64_t* allocs_so_far);

/* SHA-256 of n bytes (the checkpoint trailer's hash; host only). */
int32_t fb2_test_sha256(const void* data, int64_t n, uint8_t* out32);

/* out[M][N] = A[M][K] * W[K][N] through the tensor-core 3xTF32 GEMM on the
 * current device (host arrays; M, N, K > 0, N and K multiples of 4).
 * FB2_UNSUPPORTED when the tensor-core path is unavailable. */
int32_t fb2_test_gemm_tc(int32_t M, int32_t N, int32_t K, const float* A, const float* W, float* out);

#ifdef __cplusplus
}
#endif
#endif
