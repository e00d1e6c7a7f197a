// decode_mega.cuh — persistent decode kernel for up to 8 sequences (sm_100a).
//
// One launch runs `nsteps` KV-cached decode steps of the reference token loop
// (Sampler.Generate, src/LLM.Core/Inference/Sampler.cs:91-108) for MR rows:
// embed -> L x [LN1 -> QKV -> attention -> proj+res -> LN2 -> fc+GELU ->
// proj+res] -> LN_f -> tied head -> repetition controls -> Sample.
//
// Structure (grid = one CTA per SM, 288 threads):
//   thread 256      producer: streams every weight tile of this CTA and the
//                   K/V chunks of its attention units, in consumption order,
//                   with cp.async.bulk (TMA, no multicast) into a ring of
//                   16 KB shared-memory stages guarded by mbarriers.  It
//                   never waits for activations, so HBM stays busy across
//                   phase and step boundaries.
//   threads 0-255   consumers: compute on the staged tiles.
// Work split: every projection W[K][N] is split by output columns over the
// CTAs (column strip [K][w] per CTA, re-laid contiguously at model load);
// the head splits the vocabulary rows; attention splits (row, head, key
// chunk) units over the CTAs.
// Cross-CTA data (q, current K/V, attention partials, x2, h, x, candidate
// counts) is published as 64-bit (tag << 32 | value) words: a reader spins
// on the word itself, so the poll is the data load.  Tags are unique per
// (global step, layer).  Every wait is bounded (2 s); on expiry the kernel
// records an error and all threads leave together at the next check point.
// Sampling is distributed: each CTA applies the repetition controls to its
// vocabulary slice and publishes its local top-k with ties (every entry >=
// the global k-th largest is in some CTA's list), then every CTA computes
// the same token from the union; CTA 0 writes the bookkeeping.
#pragma once
#include "common.cuh"
#include "expf_libm.cuh"
#include "sampler.cuh"

namespace fb2 {

constexpr int MK_THREADS = 288;
constexpr int MK_CONS = 256;
constexpr int MK_STAGE = 16384;     // bytes per ring stage (column-strip path)
constexpr int MK_STAGE_HC = 32768;  // bytes per ring stage on the head-cluster path
constexpr int MK_MAX_ROWS = 8;
constexpr int MK_SLICE_MAX = 256;
constexpr int MK_SURV_MAX = 512;
constexpr int MK_MAX_TOPK = 64;
constexpr unsigned long long MK_TIMEOUT_NS = 2000000000ull;  // default limit of every bounded wait
// The launch's wait limit (MkArgs::timeout_ns), set by thread 0 before the
// first barrier; every bounded wait of the kernel reads it.
__shared__ unsigned long long mk_wait_ns;
// The launch's ring stage size in bytes (MkArgs::stage_bytes; MK_STAGE on
// the column-strip path), set with mk_wait_ns.
__shared__ int mk_sbytes;

// Traced runs: thread 0's time spent waiting for ring stages (reset per phase).
__shared__ unsigned long long mk_ring_wait;
// Traced runs: thread 0's stamps inside the last column GEMV (start, after
// the stages, after the reduction).
__shared__ unsigned long long mk_gemv_t[3];
#ifdef FB2_MK_PHASE_TRACE
#define MK_GEMV_STAMP(i) \
    if (threadIdx.x == 0) mk_gemv_t[i] = gtimer()
#else
#define MK_GEMV_STAMP(i) \
    do {                 \
    } while (0)
#endif

enum MkPhase { MK_QKV = 0, MK_PROJ = 1, MK_FC = 2, MK_PROJ2 = 3 };

struct MkLayer {
    const float* w[4];  // re-laid column strips
    const float* b[4];
    const float *ln1w, *ln1b, *ln2w, *ln2b;
    // head-cluster path: LayerNorm folded into the next projection.  The
    // re-laid qkv / fc weights are g_k W[k][c]; fold[0] / fold[1] hold per
    // qkv / fc column c the pair (S_c = sum_k g_k W[k][c],
    // B_c = sum_k beta_k W[k][c] + bias_c), so that
    // LN(x) W + bias = rstd (x (gW) - mu S) + B.
    const float* fold[2];
};

struct MkArgs {
    int V, ctx, D, L, H, hd, F, nW, nstage, slice_max;
    const MkLayer* layers;
    const float *tok_emb, *pos_emb, *lnf_w, *lnf_b;
    float* kv;
    long long kv_slot_stride, kv_layer_stride, v_offset;
    int* hist;
    int hist_stride;
    int* len;
    int* count;
    int* done;
    const double* uniforms;
    int uni_stride;
    int* out_tokens;
    int out_stride;
    float* logits_out;  // [MR][V] raw logits of the last step
    SampleParams sp;
    int n_rows;
    const int* row_slot;  // [n_rows]
    int bookkeep;         // 0: teacher forcing (no history / output writes)
    unsigned long long *xq, *xkv, *xx2, *xh, *xx, *xpart, *cand_hdr;
    float* xacc;  // [units][hd] attention partial sums (published by xpart's release)
    int maxc;     // max key chunks per (row, head)
    float* cand_val;
    int* cand_idx;
    unsigned int* stepdone;
    int* err;
    unsigned int gstep0;
    int nsteps;
    unsigned long long* trace;  // optional: [nW][trace_steps][MK_TRACE_POINTS] %globaltimer stamps
    int trace_steps;
    unsigned long long timeout_ns;  // limit of every bounded wait (MK_TIMEOUT_NS unless a test shortens it)
    int withhold_cta;               // test hook: this CTA never publishes its q words of step 0, layer 0 (-1: none)
    // head-cluster layer path (hc = 1): clusters of `cs` CTAs; CTAs [0, nhead)
    // = head h's cluster h (h = cta / cs) run LN1, the head's QKV columns,
    // attention and the head's rows of the attention projection; CTAs
    // [nhead, nW) run LN2, fc and mlp.proj over their hidden units.  Both
    // residual sums go through the counted fixed-point accumulators `acc`
    // ([2 step parity][L][2: x2, x][MK_MAX_ROWS][D]).
    int hc, cs, nhead;
    unsigned long long* acc;
    unsigned int prod_sleep_ns;  // the producer's back-off while the ring is full
    int stage_bytes;             // ring stage size: MK_STAGE, or MK_STAGE_HC on the head-cluster path
};

// Trace points per step: 12 per layer for layers 0 and 1 (level A start, after
// LN1, after QKV, after attention units, after combine weights, after ctx,
// after proj, after x2 gather, after LN2, after fc, after h gather, after
// proj2), 24 step start, 25 head input, 26 after LN_f, 27 head logits,
// 28 candidates, 29 first head stage ready, 30 published, 31 token known,
// 32 step end, 33 + l end of layer l, 45 middle head stage, 46 (a duration,
// not a stamp) thread 0's time in the head's ring waits, 57-62 sampler.
constexpr int MK_TRACE_POINTS = 64;
constexpr int MK_ERR_LAYOUT = 16;  // error code: a shared-memory region would be misaligned

// ---- small PTX helpers ------------------------------------------------------
FB2_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
FB2_DEV unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
FB2_DEV void mbar_init(uint64_t* b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
FB2_DEV void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
FB2_DEV void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
FB2_DEV bool mbar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
FB2_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// The same copy with an L2 cache policy (createpolicy).
FB2_DEV void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// L2 policy that evicts these lines before any others.
FB2_DEV uint64_t l2_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
FB2_DEV void cons_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// Barrier of the 256 consumer threads that also ORs `pred` over them.
FB2_DEV int cons_sync_or(int pred) {
    int r;
    asm volatile(
        "{ .reg .pred p, q; setp.ne.s32 p, %1, 0; bar.red.or.pred q, 1, 256, p; selp.s32 %0, 1, 0, q; }"
        : "=r"(r)
        : "r"(pred)
        : "memory");
    return r;
}
FB2_DEV void st_pair(unsigned long long* p, float v, uint32_t tag) {
    unsigned long long w = ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
FB2_DEV unsigned long long ld_pair(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
FB2_DEV unsigned int ld_acquire_u32(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
FB2_DEV void fence_acq_rel() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

FB2_DEV uint32_t mk_tag(unsigned int gs, int layer, int L) { return gs * (unsigned)(L + 1) + (unsigned)layer + 1u; }

// ---- cluster (distributed shared memory) helpers ---------------------------
// Shared::cluster address of the same shared variable in cluster CTA `rank`.
FB2_DEV uint32_t dsmem_addr(const void* local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
    return r;
}
FB2_DEV void dsmem_st(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// Arrives on an mbarrier of a cluster CTA, releasing this CTA's earlier
// writes (a CTA barrier before it makes the other threads' writes earlier).
FB2_DEV void mbar_arrive_cluster(uint32_t addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
FB2_DEV bool mbar_try_cluster(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
FB2_DEV void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
FB2_DEV int ld_relaxed_i32(const int* p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Bounded wait for phase `parity` of a local mbarrier that cluster CTAs
// arrive on.  Gives up on this CTA's abort, on a kernel error raised by any
// CTA (checked every 64 polls), or after the launch's wait limit.
FB2_DEV void wait_cluster_bar(uint64_t* b, uint32_t parity, int* err, volatile int* abort_flag) {
    if (mbar_try_cluster(b, parity)) return;
    const unsigned long long t0 = gtimer();
    for (int n = 1;; n++) {
        if (mbar_try_cluster(b, parity) || *abort_flag) return;
        if ((n & 63) == 0 && ld_relaxed_i32(err) != 0) {
            *abort_flag = 1;
            return;
        }
        if (gtimer() - t0 > mk_wait_ns) {
            atomicExch(err, 5);
            *abort_flag = 1;
            return;
        }
    }
}

FB2_DEV void dsmem_st_pair(uint32_t addr, float v, uint32_t tag) {
    const unsigned long long w = ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
    asm volatile("st.shared::cluster.u64 [%0], %1;" ::"r"(addr), "l"(w) : "memory");
}
// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) of
// this CTA's shared memory to shared::cluster address `dst` of a cluster CTA,
// completing on that CTA's mbarrier (shared::cluster address `mbar`).  The
// writers of `src` fence their generic-proxy writes (fence_async_smem) and
// pass a barrier before the copy is issued.
FB2_DEV void bulk_s2c(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
    asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     dst),
                 "r"(smem_u32(src)), "r"(bytes), "r"(mbar)
                 : "memory");
}
FB2_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Waits until words buf[0..n) of this CTA's shared memory (pushed by cluster
// CTAs) carry `tag`; bounded like every other wait.
FB2_DEV void wait_tags_smem(const unsigned long long* buf, int n, uint32_t tag, int* err, volatile int* abort_flag) {
    for (int i = threadIdx.x; i < n; i += MK_CONS) {
        const volatile unsigned long long* p = buf + i;
        if ((uint32_t)(*p >> 32) == tag) continue;
        const unsigned long long t0 = gtimer();
        for (int k = 1;; k++) {
            if ((uint32_t)(*p >> 32) == tag) break;
            if (*abort_flag) return;
            if ((k & 63) == 0 && ld_relaxed_i32(err) != 0) {
                *abort_flag = 1;
                return;
            }
            if (gtimer() - t0 > mk_wait_ns) {
                atomicExch(err, 5);
                *abort_flag = 1;
                return;
            }
        }
    }
}

// ---- counted fixed-point accumulators ----------------------------------------
// A residual sum over many CTAs: word = (sum of round(v * 2^32)) << 8 | count.
// Every contributor adds (round(v * 2^32) << 8) + 1 with one 64-bit atomic,
// so the word is complete when its count reaches the number of contributors
// and its value does not depend on the order of the additions (deterministic).
// Range: |sum| < 2^23; resolution 2^-32.
FB2_DEV unsigned long long acc_term(float v) {
    const long long q = __float2ll_rn(v * 4294967296.0f);
    return ((unsigned long long)q << 8) + 1ull;
}
FB2_DEV float acc_value(unsigned long long w) { return (float)((double)((long long)w >> 8) * 0x1p-32); }
FB2_DEV void acc_add(unsigned long long* p, unsigned long long term) {
    asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(term) : "memory");
}
// out[i] = value of words src[i], i < n, once each word's count is `count`.
__device__ __noinline__ void acc_gather(const unsigned long long* src, float* out, int n, uint32_t count, int* err,
                                        volatile int* abort_flag) {
    for (int base = 0; base < n; base += 8 * MK_CONS) {
        unsigned long long w[8];
        uint32_t pend = 0;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int i = base + k * MK_CONS + (int)threadIdx.x;
            w[k] = 0ull;
            if (i < n) {
                w[k] = ld_pair(src + i);
                pend |= 1u << k;
            }
        }
        unsigned long long t0 = 0;
        for (int n_poll = 0;; n_poll++) {
            uint32_t still = 0;
#pragma unroll
            for (int k = 0; k < 8; k++)
                if (((pend >> k) & 1u) && (uint32_t)(w[k] & 255ull) != count) still |= 1u << k;
            if (!still || *abort_flag) break;
            const unsigned long long now = gtimer();
            if (!t0) t0 = now;
            else if (now - t0 > mk_wait_ns) {
                atomicExch(err, 6);
                *abort_flag = 1;
                break;
            }
            if ((n_poll & 63) == 63 && ld_relaxed_i32(err) != 0) {
                *abort_flag = 1;
                break;
            }
#pragma unroll
            for (int k = 0; k < 8; k++)
                if ((still >> k) & 1u) w[k] = ld_pair(src + base + k * MK_CONS + (int)threadIdx.x);
        }
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int i = base + k * MK_CONS + (int)threadIdx.x;
            if (i < n) out[i] = acc_value(w[k]);
        }
    }
}

// Residual add at a fixed-point exchange: out[m][n] = base[m][n] + (value of
// src[m * D + n] + bias of column n), n = tid + 256 k (bias k in b0..b3, D <=
// 1024), once each word's count is `count`; also the per-warp moments of the
// out rows into mslots (the layout and summation order of mk_row_moments).
// Bounded like acc_gather.  No trailing barrier.
template <int MR>
__device__ __noinline__ void acc_gather_res(const unsigned long long* src, float* out, const float* base, int D,
                                            float b0, float b1, float b2, float b3, uint32_t count, float* mslots,
                                            int* err, volatile int* abort_flag) {
    constexpr int NM = MR < 2 ? MR : 2;  // rows in flight
    const int tid = threadIdx.x;
    const float bk[4] = {b0, b1, b2, b3};
    for (int m0 = 0; m0 < MR; m0 += NM) {
        unsigned long long w[NM][4];
        uint32_t pend = 0;
#pragma unroll
        for (int mm = 0; mm < NM; mm++)
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int n = tid + k * MK_CONS;
                w[mm][k] = 0ull;
                if (n < D) {
                    w[mm][k] = ld_pair(src + (size_t)(m0 + mm) * D + n);
                    pend |= 1u << (mm * 4 + k);
                }
            }
        unsigned long long t0 = 0;
        for (int n_poll = 0;; n_poll++) {
            uint32_t still = 0;
#pragma unroll
            for (int mm = 0; mm < NM; mm++)
#pragma unroll
                for (int k = 0; k < 4; k++)
                    if (((pend >> (mm * 4 + k)) & 1u) && (uint32_t)(w[mm][k] & 255ull) != count)
                        still |= 1u << (mm * 4 + k);
            if (!still || *abort_flag) break;
            const unsigned long long now = gtimer();
            if (!t0) t0 = now;
            else if (now - t0 > mk_wait_ns) {
                atomicExch(err, 6);
                *abort_flag = 1;
                break;
            }
            if ((n_poll & 63) == 63 && ld_relaxed_i32(err) != 0) {
                *abort_flag = 1;
                break;
            }
#pragma unroll
            for (int mm = 0; mm < NM; mm++)
#pragma unroll
                for (int k = 0; k < 4; k++)
                    if ((still >> (mm * 4 + k)) & 1u)
                        w[mm][k] = ld_pair(src + (size_t)(m0 + mm) * D + tid + k * MK_CONS);
        }
#pragma unroll
        for (int mm = 0; mm < NM; mm++) {
            const int m = m0 + mm;
            float s1 = 0.f, s2 = 0.f;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int n = tid + k * MK_CONS;
                if (n < D) {
                    const float v = base[m * D + n] + (acc_value(w[mm][k]) + bk[k]);
                    out[m * D + n] = v;
                    s1 += v;
                    s2 += v * v;
                }
            }
            s1 = warp_sum(s1);
            s2 = warp_sum(s2);
            if ((tid & 31) == 0) {
                mslots[m * 16 + (tid >> 5)] = s1;
                mslots[m * 16 + 8 + (tid >> 5)] = s2;
            }
        }
    }
}

// Column strip of CTA c for an N-column projection (balanced split).
FB2_DEV void strip(int N, int nW, int c, int& n0, int& w) {
    n0 = (int)(((long long)c * N) / nW);
    w = (int)(((long long)(c + 1) * N) / nW) - n0;
}
// Rows of a [K][w] strip per 16 KB stage (a multiple of 4 so every chunk is a
// multiple of 16 bytes).
FB2_DEV int strip_rows(int w, int K) {
    if (w <= 0) return 0;
    int R = mk_sbytes / 4 / w;
    if (w & 3) R &= ~3;  // a row of w floats is not a 16-byte multiple: whole groups of 4 rows
    return R < K ? R : K;
}

// Spins until word p carries `tag` and returns its value.  On timeout sets
// the error and the CTA's abort flag; after an abort it stops waiting.
FB2_DEV float wait_pair(const unsigned long long* p, uint32_t tag, int* err, volatile int* abort_flag) {
    unsigned long long w = ld_pair(p);
    if ((uint32_t)(w >> 32) == tag) return __uint_as_float((uint32_t)w);
    const unsigned long long t0 = gtimer();
    while (true) {
        __nanosleep(40);  // back off: waiting threads must not crowd L2 out for the weight stream
        w = ld_pair(p);
        if ((uint32_t)(w >> 32) == tag) return __uint_as_float((uint32_t)w);
        if (*abort_flag) return 0.f;
        if (gtimer() - t0 > mk_wait_ns) {
            atomicExch(err, 1);
            *abort_flag = 1;
            return 0.f;
        }
    }
}
// Resolves a word already loaded: returns its value if the tag matches, else
// keeps polling the address.
FB2_DEV float resolve_pair(unsigned long long w, const unsigned long long* p, uint32_t tag, int* err,
                           volatile int* abort_flag) {
    if ((uint32_t)(w >> 32) == tag) return __uint_as_float((uint32_t)w);
    return wait_pair(p, tag, err, abort_flag);
}
// Waits until every word k with bit k of `pend` set carries `tag`.  w[k]
// holds a first load of word addr(k); each retry reloads every word still
// pending, so a late batch costs its arrival time plus one round trip (not
// one round trip per word).
template <int N, class Addr>
FB2_DEV void resolve_batch(unsigned long long* w, uint32_t pend, Addr addr, uint32_t tag, int* err,
                           volatile int* abort_flag) {
    unsigned long long t0 = 0;
    while (true) {
        uint32_t still = 0;
#pragma unroll
        for (int k = 0; k < N; k++)
            if (((pend >> k) & 1u) && (uint32_t)(w[k] >> 32) != tag) still |= 1u << k;
        if (!still || *abort_flag) return;
        const unsigned long long now = gtimer();
        if (!t0) t0 = now;
        else if (now - t0 > mk_wait_ns) {
            atomicExch(err, 1);
            *abort_flag = 1;
            return;
        }
        __nanosleep(32);
#pragma unroll
        for (int k = 0; k < N; k++)
            if ((still >> k) & 1u) w[k] = ld_pair(addr(k));
        pend = still;
    }
}
FB2_DEV float pair_value(unsigned long long w) { return __uint_as_float((uint32_t)w); }

// dst[i] = value of src[i] for i < n once every word carries `tag`: each
// thread loads up to 16 words, then waits on them together.
__device__ __noinline__ void gather_tagged(const unsigned long long* src, float* dst, int n, uint32_t tag, int* err,
                           volatile int* abort_flag) {
    for (int base = 0; base < n; base += 16 * MK_CONS) {
        unsigned long long w[16];
        uint32_t pend = 0;
#pragma unroll
        for (int k = 0; k < 16; k++) {
            const int i = base + k * MK_CONS + (int)threadIdx.x;
            w[k] = 0ull;
            if (i < n) {
                w[k] = ld_pair(src + i);
                pend |= 1u << k;
            }
        }
        resolve_batch<16>(w, pend, [&](int k) { return src + base + k * MK_CONS + (int)threadIdx.x; }, tag, err,
                          abort_flag);
#pragma unroll
        for (int k = 0; k < 16; k++)
            if ((pend >> k) & 1u) dst[base + k * MK_CONS + threadIdx.x] = pair_value(w[k]);
    }
}
FB2_DEV void st_pair_release(unsigned long long* p, float v, uint32_t tag) {
    unsigned long long w = ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
FB2_DEV unsigned long long ld_pair_acquire(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// Acquire-polls a header word until it carries `tag`.
FB2_DEV float wait_pair_acquire(const unsigned long long* p, uint32_t tag, int* err, volatile int* abort_flag) {
    const unsigned long long t0 = gtimer();
    for (int n = 0;; n++) {
        if (n) __nanosleep(40);
        const unsigned long long w = ld_pair_acquire(p);
        if ((uint32_t)(w >> 32) == tag) return __uint_as_float((uint32_t)w);
        if (*abort_flag) return 0.f;
        if (gtimer() - t0 > mk_wait_ns) {
            atomicExch(err, 1);
            *abort_flag = 1;
            return 0.f;
        }
    }
}
// Exclusive prefix sum over the 256 consumer threads (wsum: 8 ints of shared scratch).
FB2_DEV int cons_excl_scan(int v, int* wsum, int& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += t;
    }
    if (lane == 31) wsum[warp] = x;
    cons_sync();
    int base = 0, tot = 0;
#pragma unroll
    for (int w8 = 0; w8 < 8; w8++) {
        const int t = wsum[w8];
        if (w8 < warp) base += t;
        tot += t;
    }
    cons_sync();
    total = tot;
    return base + x - v;
}
// The k-th largest (in float_key order) of the slices' top values tops[ns][4]
// (ns <= 256 slices, 1 <= k <= 4 ns), with ties counted: the key with fewer
// than k keys above it and at least k at or above it.  When k <= ns the k-th
// largest of the slices' first entries bounds it from below (a subset's k-th
// largest), so only the entries at or above that bound are ranked.
// kbuf: 256 + 4 * ns words; st: 10 ints.  Ends behind a barrier.
__device__ __noinline__ float cons_kth_tops(const float* tops, int ns, int k, uint32_t* kbuf, int* st) {
    const int tid = threadIdx.x;
    uint32_t* k1 = kbuf;        // [256] keys of the first entries
    uint32_t* cand = kbuf + 256;  // [4 ns] candidate keys
    uint32_t bound = 0u;          // the smallest key: everything is a candidate
    if (k <= ns) {
        const uint32_t mine = tid < ns ? float_key(tops[tid * 4]) : 0u;
        k1[tid] = mine;
        cons_sync();
        if (tid < ns) {
            int gt = 0, ge = 0;
            for (int j = 0; j < ns; j++) {
                const uint32_t kj = k1[j];
                gt += kj > mine;
                ge += kj >= mine;
            }
            if (gt < k && ge >= k) st[0] = (int)mine;  // every such thread writes the same key
        }
        cons_sync();
        bound = (uint32_t)st[0];
    }
    uint32_t ck[4];
    int c = 0;
    if (tid < ns)
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const uint32_t key = float_key(tops[tid * 4 + q]);
            ck[q] = key;
            c += key >= bound;
        }
    int C;
    const int off = cons_excl_scan(c, st + 2, C);
    if (tid < ns) {
        int o = off;
#pragma unroll
        for (int q = 0; q < 4; q++)
            if (ck[q] >= bound) cand[o++] = ck[q];
    }
    cons_sync();
    for (int i = tid; i < C; i += MK_CONS) {
        const uint32_t mine = cand[i];
        int gt = 0, ge = 0;
        for (int j = 0; j < C; j++) {
            const uint32_t kj = cand[j];
            gt += kj > mine;
            ge += kj >= mine;
        }
        if (gt < k && ge >= k) st[1] = (int)mine;
    }
    cons_sync();
    return key_float((uint32_t)st[1]);
}
// Warp 0: the bin (counted from the top of a 256-bin histogram) that holds the
// k-th largest key, and the count in the bins above it.
FB2_DEV void radix_pick(const uint32_t* hist, int kk, int& bin, int& above_out) {
    const int lane = threadIdx.x & 31;
    uint32_t c[8], local = 0;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        c[j] = hist[lane * 8 + j];
        local += c[j];
    }
    uint32_t incl = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_down_sync(0xffffffffu, incl, o);
        if (lane + o < 32) incl += t;
    }
    const uint32_t above = incl - local;
    int found = -1;
    uint32_t na = 0;
    if ((int)above < kk && (int)incl >= kk) {
        uint32_t acc = above;
#pragma unroll
        for (int j = 7; j >= 0; j--)
            if (found < 0) {
                if ((int)(acc + c[j]) >= kk) {
                    found = lane * 8 + j;
                    na = acc;
                } else acc += c[j];
            }
    }
    const unsigned bal = __ballot_sync(0xffffffffu, found >= 0);
    const int src = bal ? __ffs(bal) - 1 : 0;
    bin = __shfl_sync(0xffffffffu, found, src);
    above_out = (int)__shfl_sync(0xffffffffu, na, src);
    if (bin < 0) bin = 0;
}


// A consumer's ring position: stage index in the low 16 bits, the stage's
// phase parity in bit 16 (advanced without a division).
FB2_DEV uint32_t rp_stage(uint32_t it) { return it & 0xFFFFu; }
FB2_DEV uint32_t rp_next(uint32_t it, int nstage) {
    const uint32_t st = (it & 0xFFFFu) + 1u;
    return st == (uint32_t)nstage ? ((it ^ 0x10000u) & 0x10000u) : ((it & 0x10000u) | st);
}
FB2_DEV void wait_full(uint64_t* full, uint32_t it, int nstage, int* err, volatile int* abort_flag) {
    (void)nstage;
    uint64_t* b = &full[it & 0xFFFFu];
    const uint32_t par = (it >> 16) & 1u;
    if (mbar_try(b, par)) return;
    const unsigned long long t0 = gtimer();
    while (!mbar_try(b, par)) {
        if (*abort_flag) return;
        if (gtimer() - t0 > mk_wait_ns) {
            atomicExch(err, 2);
            *abort_flag = 1;
            return;
        }
    }
    if (threadIdx.x == 0) mk_ring_wait += gtimer() - t0;
}

FB2_DEV void release_stage(uint64_t* empty, uint32_t it, int nstage) {
    (void)nstage;
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[it & 0xFFFFu]);
}

// Sum over the 256 consumer threads through shared scratch `scr` (8 floats).
FB2_DEV float cons_sum(float v, float* scr) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) scr[threadIdx.x >> 5] = v;
    cons_sync();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) t += scr[i];
    cons_sync();
    return t;
}

// LayerNorm parameters of this thread's columns (tid + 256*k), loaded ahead
// of use so their latency hides behind the wait for the input vector.
struct LnRegs {
    float w[8], b[8];
};
FB2_DEV LnRegs ln_prefetch(const float* w, const float* b, int D) {
    LnRegs r;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int i = threadIdx.x + k * MK_CONS;
        r.w[k] = i < D ? __ldg(w + i) : 0.f;
        r.b[k] = i < D ? __ldg(b + i) : 0.f;
    }
    return r;
}
// Sum over the 256 consumer threads into a dedicated 8-float slot (no
// trailing barrier: each call site uses its own slot).
FB2_DEV float cons_sum_slot(float v, float* slot) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) slot[threadIdx.x >> 5] = v;
    cons_sync();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < 8; i++) t += slot[i];
    return t;
}
// Per-warp partial moments of MR rows of x [MR][D] (sum and sum of squares)
// into slots[m * 16 + warp] and slots[m * 16 + 8 + warp]; no barrier (a
// later one orders them before mk_row_stats reads them).
template <int MR>
FB2_DEV void mk_row_moments(const float* x, int D, float* slots) {
#pragma unroll
    for (int m = 0; m < MR; m++) {
        float s1 = 0.f, s2 = 0.f;
        for (int i = threadIdx.x; i < D; i += MK_CONS) {
            const float v = x[m * D + i];
            s1 += v;
            s2 += v * v;
        }
        s1 = warp_sum(s1);
        s2 = warp_sum(s2);
        if ((threadIdx.x & 31) == 0) {
            slots[m * 16 + (threadIdx.x >> 5)] = s1;
            slots[m * 16 + 8 + (threadIdx.x >> 5)] = s2;
        }
    }
}
// Mean and 1/sqrt(biased variance + eps) of row m from the partial moments
// (LayerNorm statistics, CpuBackend.cs:377-398; variance as E[x^2] - mean^2,
// in float like the per-warp partial sums it combines, tree-summed: this runs
// on the critical path between a GEMV's partial sums and its epilogue).
FB2_DEV void mk_row_stats(const float* slots, int m, int D, float& mu, float& rstd) {
    const float* a = slots + m * 16;
    const float s1 = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
    const float s2 = ((a[8] + a[9]) + (a[10] + a[11])) + ((a[12] + a[13]) + (a[14] + a[15]));
    const float mean = s1 / (float)D, var = s2 / (float)D - mean * mean;
    mu = mean;
    rstd = 1.0f / sqrtf(fmaxf(var, 0.f) + kLnEps);
}

// Two-pass LayerNorm of MR rows of length D <= 2048 from src into dst
// (shared), CpuBackend.cs:377-398.  `slots` = 16*MR floats of scratch that
// stay untouched until the next barrier-separated phase.
template <int MR>
__device__ __noinline__ void mk_layernorm(const float* src, float* dst, int D, const LnRegs p, float* slots) {
#pragma unroll 1
    for (int m = 0; m < MR; m++) {
        const float* x = src + m * D;
        float xv[8];
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int i = threadIdx.x + k * MK_CONS;
            xv[k] = i < D ? x[i] : 0.f;
            s += xv[k];
        }
        const float mu = cons_sum_slot(s, slots + 16 * m) / (float)D;
        float q = 0.f;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int i = threadIdx.x + k * MK_CONS;
            const float d = i < D ? xv[k] - mu : 0.f;
            q += d * d;
        }
        const float rs = 1.0f / sqrtf(cons_sum_slot(q, slots + 16 * m + 8) / (float)D + kLnEps);
#pragma unroll
        for (int k = 0; k < 8; k++) {
            const int i = threadIdx.x + k * MK_CONS;
            if (i < D) dst[m * D + i] = (xv[k] - mu) * rs * p.w[k] + p.b[k];
        }
    }
    cons_sync();
}

// Shared memory of the head-cluster layer path (offsets in floats from a
// 16-byte aligned base; every part a multiple of 4 floats):
//   qkv_in [cs][MR][q3]      q/k/v parts pushed by each cluster CTA (q3 = 3 hd / cs),
//                            64-bit words (round tag << 32 | value bits)
//   part_in[cs][MR][ps]      attention partials (max, sum, acc[hd], padding) of each
//                            cluster CTA, floats, by bulk copy (completion on mbar[0])
//   red_in [cs][MR][D / cs]  (MR <= 2) MLP partials of this CTA's column block
//                            from each cluster CTA, floats, by bulk copy (mbar[1])
// One buffer each suffices: a round's words are read before any CTA can
// reach the next round (that needs the layer's global sum, to which every
// reader contributes after reading).
//   part_out[MR][ps]         this CTA's attention partials, the bulk copies' source
//   ctxs   [MR][hd]          the head's combined context
//   att_p  [np]              scores / probabilities of this CTA's keys of one row
//   pvred  [256]             p.V partial sums per thread group
//   ys     [MR][ymax]        outputs of a column slice
//   hscr   [64]              q of one row, scratch
//   mbar   [8] (u64)         [0] partials received, [1] MLP partials received, [4] exit
//   lay    [L] MkLayer        the layer table (pointers), copied once per launch
struct MkHcLayout {
    int q3, ps, np, ymax;
    int qkv_in, part_in, red_in, part_out, ctxs, att_p, pvred, ys, hscr, mbar, lay;
    int total_floats;
};
__host__ __device__ inline int mk_r4(int v) { return (v + 3) & ~3; }
__host__ __device__ inline MkHcLayout mk_hc_layout(int MR, int D, int F, int hd, int ctx, int cs, int nW, int nlayers) {
    MkHcLayout L{};
    const int jmax = (F + nW - 1) / nW;  // every CTA takes a share of the MLP
    L.q3 = 3 * (hd / cs);
    L.ps = mk_r4(hd + 2);
    L.np = mk_r4((ctx + cs - 1) / cs);
    int ym = L.q3 > D / cs ? L.q3 : D / cs;
    L.ymax = mk_r4(ym > jmax ? ym : jmax);
    int o = 0;
    L.qkv_in = o; o += 2 * mk_r4(cs * MR * L.q3);  // u64 words
    L.part_in = o; o += 2 * (cs * MR * L.ps);
    L.red_in = o; o += MR <= 2 ? 2 * mk_r4(cs * MR * (D / cs)) : 0;
    L.part_out = o; o += MR * L.ps;
    L.ctxs = o; o += mk_r4(MR * hd);
    L.att_p = o; o += L.np;
    L.pvred = o; o += 256;
    L.ys = o; o += MR * L.ymax;
    L.hscr = o; o += 64;
    L.mbar = o; o += 16;  // 8 x u64; then 5 x 8 u32: cluster addresses of qkv_in, part_in,
    o += 40;              // red_in, mbar[0] and mbar[1] of each rank
    L.lay = o; o += nlayers * (int)(sizeof(MkLayer) / 4);
    L.total_floats = o;
    return L;
}

// Shared-memory bytes the kernel needs besides the ring.
inline size_t mk_aux_bytes(int MR, int D, int F, int H, int ctx, int slice_max, int maxc, int nstage) {
    size_t floats = (size_t)MR * F + 2 * (size_t)MR * D + (size_t)MR * 256 + (size_t)MR * slice_max + 512 + 512 + 2048;
    size_t ints = 2048 + (size_t)MR * ctx;
    size_t wts = 2 * (size_t)MR * H * maxc;
    return 2 * (size_t)nstage * 8 + floats * 4 + ints * 4 + MK_SURV_MAX * 8 + wts * 4;
}
// ... plus the head-cluster region (and its 16-byte alignment) when used.
inline size_t mk_hc_bytes(int MR, int D, int F, int hd, int ctx, int cs, int nW, int nlayers) {
    return (size_t)mk_hc_layout(MR, D, F, hd, ctx, cs, nW, nlayers).total_floats * 4 + 16;
}

// y[m][c] = sum_k act[m][k] * W[k][n0 + c] over this CTA's strip, with the
// strip's weights arriving through the ring.  Row groups g (of G) keep four
// independent partial sums; the G partials of an output are reduced by one
// warp (shuffles) when G is large, else serially.  Results land in ys[MR*w]
// behind a barrier.  Returns the ring position after the strip.
template <int MR>
__device__ __noinline__ uint32_t mk_gemv_strip(const float* actv, int K, int N, int cta, int nW, unsigned char* ring,
                                               uint64_t* full, uint64_t* empty, int nstage, uint32_t it, float* red,
                                               float* ys, int* err, volatile int* abort_flag) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int n0, w;
    strip(N, nW, cta, n0, w);
    const int R = strip_rows(w, K);
    const int G = MK_CONS / w, g = tid / w, c = tid - g * w;
    const bool valid = tid < G * w;
    float acc[MR][4];
#pragma unroll
    for (int m = 0; m < MR; m++) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
    for (int r0 = 0; r0 < K; r0 += R) {
        const int rows = min(R, K - r0);
        wait_full(full, it, nstage, err, abort_flag);
        const float* st = reinterpret_cast<const float*>(ring + (size_t)rp_stage(it) * mk_sbytes);
        if (valid) {
            const float* av = actv + r0;
            int r = g;
            for (; r + 3 * G < rows; r += 4 * G) {
                const float v0 = st[r * w + c], v1 = st[(r + G) * w + c];
                const float v2 = st[(r + 2 * G) * w + c], v3 = st[(r + 3 * G) * w + c];
#pragma unroll
                for (int m = 0; m < MR; m++) {
                    acc[m][0] += av[m * K + r] * v0;
                    acc[m][1] += av[m * K + r + G] * v1;
                    acc[m][2] += av[m * K + r + 2 * G] * v2;
                    acc[m][3] += av[m * K + r + 3 * G] * v3;
                }
            }
            for (; r < rows; r += G) {
                const float v = st[r * w + c];
#pragma unroll
                for (int m = 0; m < MR; m++) acc[m][0] += av[m * K + r] * v;
            }
        }
        release_stage(empty, it, nstage);
        it = rp_next(it, nstage);
    }
#pragma unroll
    for (int m = 0; m < MR; m++) red[m * 256 + tid] = valid ? (acc[m][0] + acc[m][1]) + (acc[m][2] + acc[m][3]) : 0.f;
    cons_sync();
    const int np = MR * w;
    if (G >= 24 && np <= 32) {
        for (int p = warp; p < np; p += 8) {
            const int m = p / w, cc = p - m * w;
            float t = 0.f;
            for (int gg = lane; gg < G; gg += 32) t += red[m * 256 + gg * w + cc];
            t = warp_sum(t);
            if (lane == 0) ys[p] = t;
        }
    } else if (tid < np) {
        const int m = tid / w, cc = tid - m * w;
        const float* rp = red + m * 256 + cc;
        float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
        int gg = 0;
        for (; gg + 3 < G; gg += 4) {
            t0 += rp[gg * w];
            t1 += rp[(gg + 1) * w];
            t2 += rp[(gg + 2) * w];
            t3 += rp[(gg + 3) * w];
        }
        for (; gg < G; gg++) t0 += rp[gg * w];
        ys[tid] = (t0 + t1) + (t2 + t3);
    }
    cons_sync();
    return it;
}

// y[m][c] = sum_k act[m][k] * W[k][c] for a [K][w] slice (w <= 256) whose
// rows arrive through the ring in stages of strip_rows(w, K) rows.  Row
// groups g (of G = 256 / w) keep four partial sums each; the G partials of
// an output are summed in a fixed order.  ys[MR*w] holds the results behind
// a barrier.  Returns the ring position after the slice.
template <int MR>
__device__ __noinline__ uint32_t mk_gemv_cols(const float* actv, int K, int w, unsigned char* ring, uint64_t* full,
                                              uint64_t* empty, int nstage, uint32_t it, float* red, float* ys, int* err,
                                              volatile int* abort_flag) {
    const int tid = threadIdx.x;
    const int R = strip_rows(w, K);
    const int G = MK_CONS / w, g = tid / w, c = tid - g * w;
    const bool valid = tid < G * w;
    float acc[MR][4];
#pragma unroll
    for (int m = 0; m < MR; m++) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
    for (int r0 = 0; r0 < K; r0 += R) {
        const int rows = min(R, K - r0);
        wait_full(full, it, nstage, err, abort_flag);
        const float* st = reinterpret_cast<const float*>(ring + (size_t)rp_stage(it) * mk_sbytes);
        if (valid) {
            const float* av = actv + r0;
            int r = g;
            for (; r + 3 * G < rows; r += 4 * G) {
                const float v0 = st[r * w + c], v1 = st[(r + G) * w + c];
                const float v2 = st[(r + 2 * G) * w + c], v3 = st[(r + 3 * G) * w + c];
#pragma unroll
                for (int m = 0; m < MR; m++) {
                    acc[m][0] += av[m * K + r] * v0;
                    acc[m][1] += av[m * K + r + G] * v1;
                    acc[m][2] += av[m * K + r + 2 * G] * v2;
                    acc[m][3] += av[m * K + r + 3 * G] * v3;
                }
            }
            for (; r < rows; r += G) {
                const float v = st[r * w + c];
#pragma unroll
                for (int m = 0; m < MR; m++) acc[m][0] += av[m * K + r] * v;
            }
        }
        release_stage(empty, it, nstage);
        it = rp_next(it, nstage);
    }
#pragma unroll
    for (int m = 0; m < MR; m++) red[m * 256 + tid] = valid ? (acc[m][0] + acc[m][1]) + (acc[m][2] + acc[m][3]) : 0.f;
    cons_sync();
    for (int p = tid; p < MR * w; p += MK_CONS) {
        const int m = p / w, cc = p - m * w;
        const float* rp = red + m * 256 + cc;
        float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
        int gg = 0;
        for (; gg + 3 < G; gg += 4) {
            t0 += rp[gg * w];
            t1 += rp[(gg + 1) * w];
            t2 += rp[(gg + 2) * w];
            t3 += rp[(gg + 3) * w];
        }
        for (; gg < G; gg++) t0 += rp[gg * w];
        ys[p] = (t0 + t1) + (t2 + t3);
    }
    cons_sync();
    return it;
}

// y[m][c] = sum_k act[m][k] * W[k][c] for a [K][w] slice, w % 4 == 0: thread
// (g, q) reads column quad q of rows g, g + G, ... as float4 (consecutive
// threads read consecutive 16-byte words of a stage), two row chains each;
// the G partials of an output go through scr (4096 floats) and are summed in
// a fixed order into ys[MR*w] behind a barrier.
// Geometry of a [K][w] column-quad slice (w % 4 == 0), computed once per
// launch: R rows per ring stage; thread (g, q) = (tid >> lgp, tid & (2^lgp - 1))
// reads quad q of rows g, g + G, ... (threads with q >= w / 4 or g >= G idle).
struct MkGeo {
    int R, G, lgp, mc;  // mc: rows of partials per pass through the 4096-float scratch
};
FB2_DEV MkGeo mk_geo(int w, int K, int MR) {
    MkGeo g{0, 1, 0, 1};
    if (w <= 0) return g;
    g.R = strip_rows(w, K);
    const int nq = w >> 2;
    while ((1 << g.lgp) < nq) g.lgp++;
    g.G = MK_CONS >> g.lgp;  // lgp <= 8: w <= 1024
    const int P = g.lgp <= 5 ? 8 : g.G;
    g.mc = 4096 / (P * w);
    if (g.mc > MR) g.mc = MR;
    if (g.mc < 1) g.mc = 1;
    return g;
}

// y[m][c] = sum_k act[m][k] * W[k][c] for a [K][w] slice, w % 4 == 0: thread
// (g, q) reads column quad q of rows g, g + G, ... as float4 (consecutive
// threads read consecutive 16-byte words of a stage row), U rows in flight
// per pass (the loop is bound by shared-memory latency, not bandwidth).
// Partials: for w <= 128 the groups of a warp are summed with shuffles and the
// 8 warp partials of an output go through scr; wider slices put their G
// (<= 4) group partials there.  Rows go through scr (4096 floats) in chunks;
// the summation order is fixed.  ys[MR*w] holds the results behind a barrier.
// With `mslots` set, warp 7 also turns the per-warp moments mslots (see
// mk_row_moments, rows of length K) into stats[2m] = mean, stats[2m+1] =
// 1/sqrt(var + eps) while the partials are summed.  No division in the
// loops: the geometry comes precomputed.  Loops stay rolled: the persistent
// kernel runs this once per phase, so code size costs instruction fetches.
template <int MR>
__device__ __noinline__ uint32_t mk_gemv_q4(const float* actv, int K, int w, MkGeo geo, unsigned char* ring,
                                            uint64_t* full, uint64_t* empty, int nstage, uint32_t it, float* scr4k,
                                            float* ys, int* err, volatile int* abort_flag,
                                            const float* mslots = nullptr, float* stats = nullptr) {
    constexpr int U = MR <= 2 ? 4 : 2;  // 4 in flight measured fastest (2 and 8 slower)
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int R = geo.R, G = geo.G, nq = w >> 2;
    const int q = tid & ((1 << geo.lgp) - 1), g = tid >> geo.lgp;
    const bool valid = g < G && q < nq;
    MK_GEMV_STAMP(0);
    float4 a0[MR], a1[MR];
#pragma unroll
    for (int m = 0; m < MR; m++) a0[m] = a1[m] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
    for (int r0 = 0; r0 < K; r0 += R) {
        const int rows = min(R, K - r0);
        wait_full(full, it, nstage, err, abort_flag);
        const float4* st = reinterpret_cast<const float4*>(ring + (size_t)rp_stage(it) * mk_sbytes);
        if (valid) {
            const float* av = actv + r0;
#pragma unroll 1
            for (int r = g; r < rows; r += U * G) {
                float4 wv[U];
#pragma unroll
                for (int u = 0; u < U; u++)
                    wv[u] = r + u * G < rows ? st[(r + u * G) * nq + q] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int m = 0; m < MR; m++) {
                    float xv[U];
#pragma unroll
                    for (int u = 0; u < U; u++) xv[u] = r + u * G < rows ? av[m * K + r + u * G] : 0.f;
#pragma unroll
                    for (int u = 0; u < U; u += 2) {
                        a0[m].x += xv[u] * wv[u].x; a0[m].y += xv[u] * wv[u].y;
                        a0[m].z += xv[u] * wv[u].z; a0[m].w += xv[u] * wv[u].w;
                        a1[m].x += xv[u + 1] * wv[u + 1].x; a1[m].y += xv[u + 1] * wv[u + 1].y;
                        a1[m].z += xv[u + 1] * wv[u + 1].z; a1[m].w += xv[u + 1] * wv[u + 1].w;
                    }
                }
            }
        }
        release_stage(empty, it, nstage);
        it = rp_next(it, nstage);
    }
    MK_GEMV_STAMP(1);
    float4 p[MR];
#pragma unroll
    for (int m = 0; m < MR; m++)
        p[m] = make_float4(a0[m].x + a1[m].x, a0[m].y + a1[m].y, a0[m].z + a1[m].z, a0[m].w + a1[m].w);
    int P, pidx;  // partials per output; this thread's partial index
    bool writer;
    if (geo.lgp <= 5) {
        // the 32 >> lgp groups of this warp (lanes differing in bits lgp..4)
#pragma unroll 1
        for (int o = 16; o >= (1 << geo.lgp); o >>= 1)
#pragma unroll
            for (int m = 0; m < MR; m++) {
                p[m].x += __shfl_xor_sync(0xffffffffu, p[m].x, o);
                p[m].y += __shfl_xor_sync(0xffffffffu, p[m].y, o);
                p[m].z += __shfl_xor_sync(0xffffffffu, p[m].z, o);
                p[m].w += __shfl_xor_sync(0xffffffffu, p[m].w, o);
            }
        P = 8;
        pidx = warp;
        writer = lane < (1 << geo.lgp) && q < nq;
    } else {
        P = G;
        pidx = g;
        writer = valid;
    }
    const int mc = geo.mc;
#pragma unroll 1
    for (int m0 = 0; m0 < MR; m0 += mc) {
        if (writer)
#pragma unroll
            for (int m = 0; m < MR; m++)
                if (m >= m0 && m < m0 + mc)
                    reinterpret_cast<float4*>(scr4k)[(((m - m0) * P + pidx) * w >> 2) + q] = p[m];
        cons_sync();
#pragma unroll 1
        for (int mm = 0; mm < mc && m0 + mm < MR; mm++)
#pragma unroll 1
            for (int c = tid; c < w; c += MK_CONS) {
                const float* rp = scr4k + (mm * P) * w + c;
                float t0 = 0.f, t1 = 0.f, t2 = 0.f, t3 = 0.f;
                int gg = 0;
#pragma unroll 1
                for (; gg + 3 < P; gg += 4) {
                    t0 += rp[gg * w];
                    t1 += rp[(gg + 1) * w];
                    t2 += rp[(gg + 2) * w];
                    t3 += rp[(gg + 3) * w];
                }
                for (; gg < P; gg++) t0 += rp[gg * w];
                ys[(m0 + mm) * w + c] = (t0 + t1) + (t2 + t3);
            }
        if (m0 + mc < MR) cons_sync();  // scr is rewritten by the next pass
    }
    if (mslots && warp == 7 && lane < MR) mk_row_stats(mslots, lane, K, stats[2 * lane], stats[2 * lane + 1]);
    cons_sync();
    MK_GEMV_STAMP(2);
    return it;
}

// Wide [K][w] slice, w % 4 == 0, w <= 1024: thread t sums column quad t over
// the K rows (float4 loads) and adds each output to the fixed-point
// accumulator out[m * w + c] (one count), or, with out null, stores it to
// red_out[own][m][blk] (own = c / blk).  Returns the ring position.
template <int MR>
__device__ __noinline__ uint32_t mk_gemv_wide_q4(const float* actv, int K, int w, int R, unsigned char* ring,
                                                 uint64_t* full, uint64_t* empty, int nstage, uint32_t it,
                                                 unsigned long long* out, float* red_out, int blk, int* err,
                                                 volatile int* abort_flag) {
    constexpr int U = MR <= 2 ? 4 : 2;  // rows in flight per pass
    const int tid = threadIdx.x;
    const int nq = w >> 2;
    float4 acc[MR];
#pragma unroll
    for (int m = 0; m < MR; m++) acc[m] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r0 = 0; r0 < K; r0 += R) {
        const int rows = min(R, K - r0);
        wait_full(full, it, nstage, err, abort_flag);
        const float4* st = reinterpret_cast<const float4*>(ring + (size_t)rp_stage(it) * mk_sbytes);
        if (tid < nq)
            for (int r = 0; r < rows; r += U) {
                float4 v[U];
#pragma unroll
                for (int u = 0; u < U; u++) v[u] = r + u < rows ? st[(r + u) * nq + tid] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int m = 0; m < MR; m++) {
                    float x[U];
#pragma unroll
                    for (int u = 0; u < U; u++) x[u] = r + u < rows ? actv[m * K + r0 + r + u] : 0.f;
#pragma unroll
                    for (int u = 0; u < U; u++) {
                        acc[m].x += x[u] * v[u].x; acc[m].y += x[u] * v[u].y;
                        acc[m].z += x[u] * v[u].z; acc[m].w += x[u] * v[u].w;
                    }
                }
            }
        release_stage(empty, it, nstage);
        it = rp_next(it, nstage);
    }
    if (tid < nq) {
        if (out) {
            // straight to the global accumulators (one count each)
#pragma unroll
            for (int m = 0; m < MR; m++) {
                unsigned long long* o = out + (size_t)m * w + 4 * tid;
                acc_add(o, acc_term(acc[m].x));
                acc_add(o + 1, acc_term(acc[m].y));
                acc_add(o + 2, acc_term(acc[m].z));
                acc_add(o + 3, acc_term(acc[m].w));
            }
        } else {
            // into red_out[own][m][blk] for the cluster CTA `own` that owns columns
            // 4 tid .. 4 tid + 3 (blocks of blk, blk % 4 == 0)
            const int c = 4 * tid, own = c / blk, oc = c - own * blk;
#pragma unroll
            for (int m = 0; m < MR; m++) reinterpret_cast<float4*>(red_out + (own * MR + m) * blk + oc)[0] = acc[m];
        }
    }
    return it;
}

// Wide slice (256 < w <= 1024 columns): thread t sums columns t + 256 i over
// the K rows, and adds each output to the fixed-point accumulator
// out[m * w + c] (one count).  Returns the ring position after the slice.
template <int MR>
__device__ __noinline__ uint32_t mk_gemv_wide_acc(const float* actv, int K, int w, unsigned char* ring,
                                                  uint64_t* full, uint64_t* empty, int nstage, uint32_t it,
                                                  unsigned long long* out, int* err, volatile int* abort_flag) {
    const int tid = threadIdx.x;
    const int R = strip_rows(w, K);
    float acc[MR][4];
#pragma unroll
    for (int m = 0; m < MR; m++) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
    for (int r0 = 0; r0 < K; r0 += R) {
        const int rows = min(R, K - r0);
        wait_full(full, it, nstage, err, abort_flag);
        const float* st = reinterpret_cast<const float*>(ring + (size_t)rp_stage(it) * mk_sbytes);
        for (int r = 0; r < rows; r++) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int c = tid + i * MK_CONS;
                if (c < w) {
                    const float v = st[r * w + c];
#pragma unroll
                    for (int m = 0; m < MR; m++) acc[m][i] += actv[m * K + r0 + r] * v;
                }
            }
        }
        release_stage(empty, it, nstage);
        it = rp_next(it, nstage);
    }
#pragma unroll
    for (int m = 0; m < MR; m++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int c = tid + i * MK_CONS;
            if (c < w) acc_add(out + (size_t)m * w + c, acc_term(acc[m][i]));
        }
    return it;
}

#define MK_TRACE(pt)                                                                                 \
    do {                                                                                             \
        if (a.trace && tid == 0 && s < a.trace_steps && (pt) < MK_TRACE_POINTS)                     \
            a.trace[((size_t)cta * a.trace_steps + s) * MK_TRACE_POINTS + (pt)] = gtimer();          \
    } while (0)
#define MK_TRACE_ANY(pt)                                                                             \
    do {                                                                                             \
        if (a.trace && s < a.trace_steps && (pt) < MK_TRACE_POINTS)                                  \
            a.trace[((size_t)cta * a.trace_steps + s) * MK_TRACE_POINTS + (pt)] = gtimer();          \
    } while (0)
// Phase-level stamps inside a layer (layer 0 only) and GEMV timings: built
// only with FB2_MK_PHASE_TRACE (FORGE_B200_PHASE_TRACE=1 at build time).  The
// persistent kernel runs each layer's code once per layer, so every extra
// instruction there costs instruction-cache misses in the production build.
#ifdef FB2_MK_PHASE_TRACE
#define MK_TRACE_DUR(pt, v)                                                                         \
    do {                                                                                            \
        if (a.trace && tid == 0 && s < a.trace_steps && (pt) < MK_TRACE_POINTS)                    \
            a.trace[((size_t)cta * a.trace_steps + s) * MK_TRACE_POINTS + (pt)] = (v);              \
    } while (0)
#define MK_TRACE_L(off)                  \
    do {                                 \
        if (l < 1) MK_TRACE(l * 12 + (off)); \
    } while (0)
#else
#define MK_TRACE_DUR(pt, v) \
    do {                    \
    } while (0)
#define MK_TRACE_L(off) \
    do {                \
    } while (0)
#endif

// ---- the kernel ---------------------------------------------------------------
// HC: the head-cluster layer path (a separate instantiation, so each path
// gets the registers of its own code; MkArgs::hc must match).
template <int MR, bool HC>
__global__ void __launch_bounds__(MK_THREADS, 1) k_decode_mega(const MkArgs a) {
    extern __shared__ __align__(128) unsigned char mk_smem_raw[];
    const int tid = threadIdx.x;
    const int cta = blockIdx.x, nW = a.nW;
    const int D = a.D, F = a.F, L = a.L, H = a.H, hd = a.hd, V = a.V;
    const int KC = MK_STAGE / (hd * 4);  // keys per attention chunk
    unsigned char* ring = mk_smem_raw;
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + (size_t)a.nstage * a.stage_bytes);
    uint64_t* empty = full + a.nstage;
    float* act = reinterpret_cast<float*>(empty + a.nstage);  // [MR][F]
    float* xres = act + MR * F;                                // [MR][D]
    float* x2res = xres + MR * D;                              // [MR][D]
    float* red = x2res + MR * D;                               // [MR][256]
    float* slice = red + MR * 256;                             // [MR][slice_max]
    float* scr = slice + MR * a.slice_max;                     // [512]
    float* uacc = scr + 512;                                   // [8][64] attention unit: per-warp p.V
    float* hstage = uacc + 512;                                // [2][4][256] sampler: slices' top 4 (value, id)
    int* iscr = reinterpret_cast<int*>(hstage + 2048);         // [2048]
    int* win = iscr + 2048;                                    // [MR][ctx]
    float* surv_v = reinterpret_cast<float*>(win + MR * a.ctx);  // [MK_SURV_MAX]
    int* surv_i = reinterpret_cast<int*>(surv_v + MK_SURV_MAX);  // [MK_SURV_MAX]
    float* wts_m = reinterpret_cast<float*>(surv_i + MK_SURV_MAX);  // [MR*H][maxc] chunk weights
    // head-cluster region (hc launches only)
    const MkHcLayout hcl = mk_hc_layout(MR, D, F, hd, a.ctx, HC ? a.cs : 1, nW, L);
    float* hcb = reinterpret_cast<float*>(
        (reinterpret_cast<uintptr_t>(wts_m + 2 * MR * H * a.maxc) + 15) & ~(uintptr_t)15);
    unsigned long long* qkv_in = reinterpret_cast<unsigned long long*>(hcb + hcl.qkv_in);
    float* part_in = hcb + hcl.part_in;
    float* part_out = hcb + hcl.part_out;
    float* ctxs = hcb + hcl.ctxs;
    float* att_p = hcb + hcl.att_p;
    float* pvred = hcb + hcl.pvred;
    float* hc_ys = hcb + hcl.ys;
    float* hscr = hcb + hcl.hscr;
    uint64_t* hc_mbar = reinterpret_cast<uint64_t*>(hcb + hcl.mbar);  // [0] partials, [1] MLP partials, [4] exit
    float* red_in = hcb + hcl.red_in;
    MkLayer* hc_lay = reinterpret_cast<MkLayer*>(hcb + hcl.lay);
    uint32_t* hc_rb = reinterpret_cast<uint32_t*>(hcb + hcl.mbar + 16);  // [5][8] cluster addresses
    // iscr regions
    uint32_t* seen = reinterpret_cast<uint32_t*>(iscr);  // [8] bits of the slice
    uint32_t* ban = seen + 8;                            // [8]
    int* wbi = iscr + 16;                                // [8] per-warp argmax index
    int* rcnt = iscr + 32;                               // [8] candidates per row
    int* rtok = iscr + 48;                               // [8] token per row
    int* misc = iscr + 64;                               // [64]
    int* flag = iscr + 256;                              // [256]
    int* cnts = iscr + 512;                              // [256]

    __shared__ int s_slot[MK_MAX_ROWS], s_pos0[MK_MAX_ROWS], s_tok[MK_MAX_ROWS], s_cnt0[MK_MAX_ROWS];
    __shared__ double s_ud[MK_MAX_ROWS];  // this step's uniform draw per row
    __shared__ int s_len0[MK_MAX_ROWS], s_dead[MK_MAX_ROWS], s_dummy[MK_MAX_ROWS], s_ubase[MK_MAX_ROWS + 1];
    __shared__ volatile int s_abort;
    __shared__ MkGeo s_geo[3];  // head-cluster slices: qkv, proj, fc (column quads)
    __shared__ int s_hci[8];    // log2 cs, log2 hq, log2 hd, j0, J, proj2 stage rows

    // float4 accesses to the scratch regions need slice_max % 4 == 0
    if ((a.slice_max & 3) != 0) {
        if (tid == 0) atomicExch(a.err, MK_ERR_LAYOUT);
        return;
    }
    if (tid < MR) {
        const int m = tid;
        const bool dummy = m >= a.n_rows;
        const int slot = a.row_slot[dummy ? 0 : m];
        const int len = a.len[slot];
        s_slot[m] = slot;
        s_dummy[m] = dummy;
        s_len0[m] = dummy ? 1 : len;
        s_pos0[m] = dummy ? 0 : len - 1;
        s_tok[m] = dummy ? 0 : a.hist[(size_t)slot * a.hist_stride + len - 1];
        s_cnt0[m] = dummy ? 0 : a.count[slot];
        s_dead[m] = dummy ? 1 : a.done[slot];
    }
    if (tid == 0) {
        s_abort = 0;
        mk_wait_ns = a.timeout_ns;
        mk_sbytes = a.stage_bytes;

        for (int i = 0; i < a.nstage; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 8);
        }
        if (HC) {
            mbar_init(&hc_mbar[0], 1);     // partials: this CTA's expect_tx arrival + the copies' bytes
            mbar_init(&hc_mbar[1], 1);     // MLP partials: the same
            mbar_init(&hc_mbar[4], a.cs);  // exit handshake: one arrival per cluster CTA
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if constexpr (HC) {
        for (int i = tid; i < L * (int)(sizeof(MkLayer) / 8); i += MK_THREADS)
            reinterpret_cast<const float**>(hc_lay)[i] = reinterpret_cast<const float* const*>(a.layers)[i];
        {
            // the exchange words start untagged in every launch (no word of an
            // earlier launch can carry a tag of this one)
            const int nq = a.cs * MR * hcl.q3;
            for (int i = tid; i < nq; i += MK_THREADS) qkv_in[i] = 0ull;
            if (tid < a.cs) {
                hc_rb[tid] = dsmem_addr(qkv_in, tid);
                hc_rb[8 + tid] = dsmem_addr(part_in, tid);
                hc_rb[16 + tid] = dsmem_addr(red_in, tid);
                hc_rb[24 + tid] = dsmem_addr(&hc_mbar[0], tid);
                hc_rb[32 + tid] = dsmem_addr(&hc_mbar[1], tid);
            }
        }
    }
    __syncthreads();
    // the cluster's mbarriers are initialised before any CTA arrives on them
    if constexpr (HC) cluster_sync_all();

    // positions at step s (dummy rows stay at 0); attention units (m, h, c)
    // cover the cached keys [0, pos-1) in chunks of KC
    auto pos_of = [&](int m, int s) { return s_dummy[m] ? 0 : s_pos0[m] + s; };
    auto nch_of = [&](int m, int s) {
        const int old = pos_of(m, s) - 1;
        return old > 0 ? (old + KC - 1) / KC : 0;
    };

    // =========================== producer ===================================
    if (tid >= MK_CONS) {
        if (tid != MK_CONS) return;
        uint32_t it = 0;
        bool ok = true;
        // Weights and the head's embedding rows are read once per step (391 MB
        // for Forge-98M, beyond L2): they go through L2 evict-first, so the
        // kernel's code, the small per-layer parameters, the exchange words
        // and the sequence's K/V (normal priority) stay resident across steps.
        const uint64_t stream_policy = l2_evict_first();
        auto issue = [&](const void* src, uint32_t bytes, bool streamed) {
            if (!ok) return;
            const int st = it % a.nstage;
            if (it >= (uint32_t)a.nstage) {
                const uint32_t par = ((it / a.nstage) - 1) & 1u;
                if (!mbar_try(&empty[st], par)) {
                    const unsigned long long t0 = gtimer();
                    while (!mbar_try(&empty[st], par)) {
                        // the producer's warp shares a scheduler with consumer warps 0
                        // and 4: back off instead of competing with them for issue slots
                        __nanosleep(a.prod_sleep_ns);
                        if (s_abort || gtimer() - t0 > mk_wait_ns) {
                            if (!s_abort) atomicExch(a.err, 3);
                            s_abort = 1;
                            ok = false;
                            return;
                        }
                    }
                }
            }
            mbar_expect_tx(&full[st], bytes);
            if (streamed) bulk_g2s_hint(ring + (size_t)st * mk_sbytes, src, bytes, &full[st], stream_policy);
            else bulk_g2s(ring + (size_t)st * mk_sbytes, src, bytes, &full[st]);
            it++;
        };
        auto issue_strip = [&](const float* Wt, int K, int N) {
            int n0, w;
            strip(N, nW, cta, n0, w);
            const int R = strip_rows(w, K);
            if (R == 0) return;
            const float* base = Wt + (size_t)K * n0;
            for (int r0 = 0; r0 < K && ok; r0 += R) issue(base + (size_t)r0 * w, (uint32_t)(min(R, K - r0) * w * 4), true);
        };
        auto issue_cols = [&](const float* W, int K, int w) {
            const int R = strip_rows(w, K);
            if (R == 0) return;
            for (int r0 = 0; r0 < K && ok; r0 += R) issue(W + (size_t)r0 * w, (uint32_t)(min(R, K - r0) * w * 4), true);
        };
        for (int s = 0; s < a.nsteps && ok; s++) {
            const unsigned int gs = a.gstep0 + s;
            if constexpr (HC) {
                // this CTA's slices of every layer, in the order the consumers use them
                const int q3 = hcl.q3, wp = D / a.cs;
                const int j0 = 4 * (int)((long long)cta * (F / 4) / nW), j1 = 4 * (int)((long long)(cta + 1) * (F / 4) / nW);
                for (int l = 0; l < L && ok; l++) {
                    const MkLayer& ly = hc_lay[l];
                    if (cta < a.nhead) {
                        issue_cols(ly.w[MK_QKV] + (size_t)cta * D * q3, D, q3);
                        issue_cols(ly.w[MK_PROJ] + (size_t)cta * hd * wp, hd, wp);
                    }
                    if (j1 > j0) {
                        issue_cols(ly.w[MK_FC] + (size_t)D * j0, D, j1 - j0);
                        issue_cols(ly.w[MK_PROJ2] + (size_t)j0 * D, j1 - j0, D);
                    }
                }
            }
            for (int l = 0; l < L && ok && !HC; l++) {
                const MkLayer& ly = a.layers[l];
                issue_strip(ly.w[MK_QKV], D, 3 * D);
                if (l == 0 && gs >= 2 && ok) {
                    // The K/V rows read below were written by steps <= gs-2:
                    // wait until those steps finished on every CTA, then order
                    // the async-proxy reads after them.
                    const unsigned int target = (gs - 1) * (unsigned)nW;
                    const unsigned long long t0 = gtimer();
                    while (ld_acquire_u32(a.stepdone) < target) {
                        __nanosleep(200);
                        if (s_abort || gtimer() - t0 > mk_wait_ns) {
                            if (!s_abort) atomicExch(a.err, 4);
                            s_abort = 1;
                            ok = false;
                            break;
                        }
                    }
                    asm volatile("fence.proxy.async.global;" ::: "memory");
                }
                // units u = (m, h, c) in row-major order; this CTA owns u = cta (mod nW)
                int ubase = 0;
                for (int m = 0; m < MR && ok; m++) {
                    const int nc = nch_of(m, s), old = pos_of(m, s) - 1, nu = H * nc;
                    for (int u = ubase + ((cta - ubase) % nW + nW) % nW; u < ubase + nu && ok; u += nW) {
                        const int h = (u - ubase) / nc, c = (u - ubase) - h * nc;
                        if (l == 1 && u == cta) MK_TRACE_ANY(63);
                        const int nk = min(KC, old - c * KC);
                        const float* kb = a.kv + (size_t)s_slot[m] * a.kv_slot_stride + (size_t)l * a.kv_layer_stride +
                                          ((size_t)h * a.ctx + c * KC) * hd;
                        issue(kb, (uint32_t)(nk * hd * 4), false);
                        issue(kb + a.v_offset, (uint32_t)(nk * hd * 4), false);
                    }
                    ubase += nu;
                }
                issue_strip(ly.w[MK_PROJ], D, D);
                issue_strip(ly.w[MK_FC], D, F);
                issue_strip(ly.w[MK_PROJ2], F, D);
            }
            const int v0 = (int)(((long long)cta * V) / nW), v1 = (int)(((long long)(cta + 1) * V) / nW);
            const int Rh = max(1, mk_sbytes / (D * 4));
            for (int r0 = v0; r0 < v1 && ok; r0 += Rh)
                issue(a.tok_emb + (size_t)r0 * D, (uint32_t)(min(Rh, v1 - r0) * D * 4), true);
        }
        // wait (bounded) for copies still landing in this CTA's ring
        for (uint32_t j = (it > (uint32_t)a.nstage ? it - a.nstage : 0); j < it; j++) {
            const unsigned long long t0 = gtimer();
            while (!mbar_try(&full[j % a.nstage], (j / a.nstage) & 1u))
                if (gtimer() - t0 > mk_wait_ns) break;
        }
        return;
    }

    // =========================== consumers ==================================
    // (a lambda: every early exit of the consumers returns here, so that the
    // head clusters' exit handshake below always runs)
    auto consumers = [&]() {
    const int lane = tid & 31, warp = tid >> 5;
    const float scale = 1.0f / sqrtf((float)hd);  // Layers.cs:174
    const SampleParams sp = a.sp;
    const bool controls = sp.penalty != 1.0f || sp.ngram > 0;
    const bool sampled = sp.temperature > 0.0f;
    uint32_t it = 0;
    if (controls)
        for (int m = 0; m < MR; m++)
            for (int i = tid; i < s_len0[m] && i < a.ctx; i += MK_CONS)
                win[m * a.ctx + i] = s_dummy[m] ? 0 : a.hist[(size_t)s_slot[m] * a.hist_stride + i];
    cons_sync();

    // This CTA's column strip of y = act * W (+ epilogue(m, n, sum)).
    // This CTA's column strip of y = act * W, then epilogue(m, n, sum) once
    // per output (one shared, out-of-line copy of the strip code).
    auto gemv = [&](const float* actv, int K, int N, auto&& epilogue) {
        int n0, w;
        strip(N, nW, cta, n0, w);
        if (w <= 0) return;
        it = mk_gemv_strip<MR>(actv, K, N, cta, nW, ring, full, empty, a.nstage, it, red, uacc, a.err, &s_abort);
        for (int p = tid; p < MR * w; p += MK_CONS) epilogue(p / w, n0 + p % w, uacc[p]);
    };

    if (HC && tid == 0) {
        // the head-cluster geometry, with the launch's only divisions
        int lcs = 0, lhd = 0;
        while ((1 << lcs) < a.cs) lcs++;
        while ((1 << lhd) < hd) lhd++;
        const int j0 = 4 * (int)((long long)cta * (F / 4) / nW);
        const int J = 4 * (int)((long long)(cta + 1) * (F / 4) / nW) - j0;
        s_hci[0] = lcs;
        s_hci[1] = lhd - lcs;
        s_hci[2] = lhd;
        s_hci[3] = j0;
        s_hci[4] = J;
        s_hci[5] = J > 0 ? strip_rows(D, J) : 0;
        s_geo[0] = mk_geo(hcl.q3, D, MR);
        s_geo[1] = mk_geo(D >> lcs, hd, MR);
        s_geo[2] = mk_geo(J, D, MR);
    }
    cons_sync();
    for (int s = 0; s < a.nsteps; s++) {
        const unsigned int gs = a.gstep0 + s;
        if (tid == 0) {
            int acc = 0;
            for (int m = 0; m < MR; m++) {
                s_ubase[m] = acc;
                acc += H * nch_of(m, s);
            }
            s_ubase[MR] = acc;
        }
        cons_sync();
        MK_TRACE(24);
        if constexpr (HC) {
            // ======== head-cluster layers ========
            // Per layer two exchanges through global memory: the attention
            // projection's head partials -> x2, every CTA's MLP partials -> x
            // (counted fixed-point accumulators).  q/k/v parts and attention
            // partials move inside a head's cluster (DSMEM).  Parameters a
            // phase needs are loaded before the wait that precedes it.
            const int cs = a.cs, nhead = a.nhead;
            const bool is_head = cta < nhead;
            const int lcs = s_hci[0], lhq = s_hci[1], lhd = s_hci[2];
            const int hh = cta >> lcs, rk = cta & (cs - 1);
            const int hq = 1 << lhq, q3 = hcl.q3, wp = D >> lcs, ps = hcl.ps;
            // hidden units in groups of 4 (every slice a whole number of float4 columns)
            const int j0 = s_hci[3], J = s_hci[4];
            // this thread's q / k / v column of head hh (threads < q3)
            const int qpart = tid >> lhq, qi = tid & (hq - 1);
            const int qcol = qpart * D + hh * hd + rk * hq + qi;
            float* gscr = hstage;  // 4096 floats (hstage + iscr), free while the layers run
            const unsigned int par = gs & 1u;
            // per-thread columns n = tid + 256 k (D <= 1024)
            auto load_cols = [&](const float* b, float (&r)[4]) {
#pragma unroll
                for (int k = 0; k < 4; k++) r[k] = tid + k * MK_CONS < D ? __ldg(b + tid + k * MK_CONS) : 0.f;
            };
            float fqS = 0.f, fqB = 0.f;  // this thread's qkv column: folded LN1 sum and bias
            if (is_head && tid < q3) {
                fqS = __ldg(hc_lay[0].fold[0] + 2 * qcol);
                fqB = __ldg(hc_lay[0].fold[0] + 2 * qcol + 1);
            }
            for (int l = 0; l < L; l++) {
                const MkLayer& ly = hc_lay[l];
                unsigned long long* accx2 = a.acc + (((size_t)par * L + l) * 2) * MK_MAX_ROWS * D;
                unsigned long long* accx = accx2 + (size_t)MK_MAX_ROWS * D;
                // the cluster mbarriers start at phase 0 in every launch: rounds count
                // from the launch's first step
                const unsigned int rnd = (unsigned)s * (unsigned)L + (unsigned)l;
                const int buf = 0;  // one buffer per exchange (see the layout)
                MK_TRACE_L(0);
                if (l == 0) {
                    for (int m = 0; m < MR; m++) {
                        const float* te = a.tok_emb + (size_t)s_tok[m] * D;
                        const float* pe = a.pos_emb + (size_t)pos_of(m, s) * D;
                        for (int i = tid; i < D; i += MK_CONS) xres[m * D + i] = __ldg(te + i) + __ldg(pe + i);
                    }
                    cons_sync();
                }
                float bproj[4];
                load_cols(ly.b[MK_PROJ], bproj);
                if (is_head) {
                    // the cached K and V rows of this CTA's keys (written by earlier
                    // steps), pulled into L1 while the q/k/v GEMV runs (4 lines of
                    // 128 bytes per key at head_dim 64; read below with L1-cached loads)
                    for (int m = 0; m < MR; m++) {
                        const int pos = pos_of(m, s), T = pos + 1;
                        const int k0 = (rk * T) >> lcs;
                        const int kend = min(((rk + 1) * T) >> lcs, pos);
                        const int lpr = hd >> 5;  // 128-byte lines per row
                        const char* kb = reinterpret_cast<const char*>(
                            a.kv + (size_t)s_slot[m] * a.kv_slot_stride + (size_t)l * a.kv_layer_stride +
                            (size_t)hh * a.ctx * hd);
                        for (int i = tid; i < 2 * lpr * (kend - k0); i += MK_CONS) {
                            const int key = k0 + (i >> (lhd - 4)), part = i & (2 * lpr - 1);
                            const char* ln = kb + (part >= lpr ? (size_t)a.v_offset * 4 : 0) +
                                             ((size_t)key * hd) * 4 + (size_t)(part % lpr) * 128;
                            asm volatile("prefetch.global.L1 [%0];" ::"l"(ln));
                        }
                    }
                    // ---- LN1 folded into this CTA's q, k, v columns of head hh -------
                    // (row moments: the previous layer's x gather, or here at layer 0)
                    if (l == 0) mk_row_moments<MR>(xres, D, scr + 384);
                    MK_TRACE_L(1);
                    if (tid == 0) mk_ring_wait = 0;
                    it = mk_gemv_q4<MR>(xres, D, q3, s_geo[0], ring, full, empty, a.nstage, it, gscr, hc_ys, a.err,
                                        &s_abort, scr + 384, scr + 320);
                    MK_TRACE_L(2);
                    if (l == 0) {
                        MK_TRACE_DUR(22, mk_gemv_t[0]);
                        MK_TRACE_DUR(23, mk_gemv_t[1]);
                        MK_TRACE_DUR(47, mk_gemv_t[2]);
                    }
                    if (l == 0) MK_TRACE_DUR(14, mk_ring_wait);
                    const bool withhold = cta == a.withhold_cta && s == 0 && l == 0;
                    const uint32_t xtag = rnd + 1u;  // exchange words of this round
                    if (tid < q3)  // q3 <= 256
                        for (int m = 0; m < MR; m++) {
                            const float mu = scr[320 + 2 * m], rstd = scr[321 + 2 * m];
                            const float v = rstd * (hc_ys[m * q3 + tid] - mu * fqS) + fqB;
                            if (qpart > 0 && !s_dummy[m])
                                a.kv[(size_t)s_slot[m] * a.kv_slot_stride + (size_t)l * a.kv_layer_stride +
                                     (qpart == 2 ? a.v_offset : 0) + ((size_t)hh * a.ctx + pos_of(m, s)) * hd + rk * hq +
                                     qi] = v;
                            const uint32_t off = (uint32_t)(((buf * cs + rk) * MR + m) * q3 + tid) * 8u;
                            if (!withhold)
                                for (int q = 0; q < cs; q++) dsmem_st_pair(hc_rb[q] + off, v, xtag);
                        }
                    MK_TRACE_L(19);
                    wait_tags_smem(qkv_in + buf * cs * MR * q3, cs * MR * q3, xtag, a.err, &s_abort);
                    MK_TRACE_L(3);
                    if (cons_sync_or(s_abort)) return;
                    // ---- attention of head hh over this CTA's share of the keys -----
                    for (int m = 0; m < MR; m++) {
                        const int pos = pos_of(m, s), T = pos + 1;
                        const int k0 = (rk * T) >> lcs, k1 = ((rk + 1) * T) >> lcs;
                        const int nk = k1 - k0;
                        const unsigned long long* qin = qkv_in + (buf * cs * MR + m) * q3;  // rank q at + q * MR * q3
                        auto qkv_at = [&](int part, int d) {  // element d of q / k / v of row m
                            return __uint_as_float((uint32_t)qin[(d >> lhq) * MR * q3 + part * hq + (d & (hq - 1))]);
                        };
                        if (tid < hd) hscr[tid] = qkv_at(0, tid);
                        cons_sync();
                        const float* kbase = a.kv + (size_t)s_slot[m] * a.kv_slot_stride +
                                             (size_t)l * a.kv_layer_stride + (size_t)hh * a.ctx * hd;
                        const float* vbase = kbase + a.v_offset;
                        float mloc = -INFINITY;
                        for (int t = tid; t < nk; t += MK_CONS) {
                            const int j = k0 + t;
                            float d = 0.f;
                            if (j < pos) {
                                const float4* q4 = reinterpret_cast<const float4*>(hscr);
                                const float4* kr = reinterpret_cast<const float4*>(kbase + (size_t)j * hd);
                                int e0 = 0;
                                for (; e0 + 8 <= hd / 4; e0 += 8) {  // 8 loads in flight (one L2 trip on a miss)
                                    float4 kv4[8];
#pragma unroll
                                    for (int e = 0; e < 8; e++) kv4[e] = __ldca(kr + e0 + e);
#pragma unroll
                                    for (int e = 0; e < 8; e++) {
                                        const float4 qv = q4[e0 + e];
                                        d += qv.x * kv4[e].x + qv.y * kv4[e].y + qv.z * kv4[e].z + qv.w * kv4[e].w;
                                    }
                                }
                                for (; e0 < hd / 4; e0 += 4) {
                                    float4 kv4[4];
#pragma unroll
                                    for (int e = 0; e < 4; e++) kv4[e] = __ldca(kr + e0 + e);
#pragma unroll
                                    for (int e = 0; e < 4; e++) {
                                        const float4 qv = q4[e0 + e];
                                        d += qv.x * kv4[e].x + qv.y * kv4[e].y + qv.z * kv4[e].z + qv.w * kv4[e].w;
                                    }
                                }
                            } else {
                                for (int e = 0; e < hd; e++) d += hscr[e] * qkv_at(1, e);
                            }
                            const float sc = d * scale;
                            att_p[t] = sc;
                            mloc = fmaxf(mloc, sc);
                        }
                        // this thread's V values (dimension d, keys g, g + ng, ...),
                        // loaded before the softmax reductions
                        const int ng = MK_CONS >> lhd, d = tid & (hd - 1), g = tid >> lhd;
                        float vv[8];
                        const int nv = (nk - g + ng - 1) >> (8 - lhd);
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const int j = k0 + g + i * ng;
                            vv[i] = 0.f;
                            if (i < nv) vv[i] = j < pos ? __ldca(vbase + (size_t)j * hd + d) : qkv_at(2, d);
                        }
                        mloc = warp_max(mloc);
                        if (lane == 0) scr[256 + warp] = mloc;
                        cons_sync();
                        float M = -INFINITY;
#pragma unroll
                        for (int w8 = 0; w8 < 8; w8++) M = fmaxf(M, scr[256 + w8]);
                        float lsum = 0.f;
                        for (int t = tid; t < nk; t += MK_CONS) {
                            const float pr = __expf(att_p[t] - M);
                            att_p[t] = pr;
                            lsum += pr;
                        }
                        const float S = cons_sum_slot(lsum, scr + 272);  // barrier: att_p complete
                        if (m == 0) MK_TRACE_L(20);
                        float av0 = 0.f, av1 = 0.f;
#pragma unroll
                        for (int i = 0; i < 8; i += 2) {
                            if (i < nv) av0 += att_p[g + i * ng] * vv[i];
                            if (i + 1 < nv) av1 += att_p[g + (i + 1) * ng] * vv[i + 1];
                        }
                        for (int i = 8; i < nv; i++) {
                            const int j = k0 + g + i * ng;
                            av0 += att_p[g + i * ng] * (j < pos ? __ldcg(vbase + (size_t)j * hd + d) : qkv_at(2, d));
                        }
                        pvred[g * hd + d] = av0 + av1;
                        cons_sync();
                        if (m == 0) MK_TRACE_L(21);
                        // this row's partial (max, sum, p.V) into the copies' source
                        if (tid < hd) {
                            float A = 0.f;
                            for (int gg = 0; gg < ng; gg++) A += pvred[gg * hd + tid];
                            part_out[m * ps + 2 + tid] = A;
                        } else if (tid == hd) {
                            part_out[m * ps] = nk > 0 ? M : -INFINITY;
                            part_out[m * ps + 1] = nk > 0 ? S : 0.f;
                        }
                        fence_async_smem();
                        cons_sync();
                    }
                    // this CTA's partials to every cluster CTA: one bulk copy each,
                    // completing on the receiver's mbar[0] (one phase per round)
                    if (tid < cs)
                        bulk_s2c(hc_rb[8 + tid] + (uint32_t)(rk * MR * ps) * 4u, part_out, (uint32_t)(MR * ps) * 4u,
                                 hc_rb[24 + tid]);
                    MK_TRACE_L(4);
                    if (tid == 0) mbar_expect_tx(&hc_mbar[0], (uint32_t)(cs * MR * ps) * 4u);
                    wait_cluster_bar(&hc_mbar[0], rnd & 1u, a.err, &s_abort);
                    MK_TRACE_L(5);
                    if (cons_sync_or(s_abort)) return;
                    // ---- combine the cluster's partials -> ctx of head hh -------------
                    for (int p = tid; p < MR * hd; p += MK_CONS) {
                        const int m = p >> lhd, dd = p & (hd - 1);
                        const float* pr = part_in + m * ps;  // rank q's row m at pr + q * MR * ps
                        float Ms = -INFINITY;
                        for (int q = 0; q < cs; q++) Ms = fmaxf(Ms, pr[q * MR * ps]);
                        float ls = 0.f, A = 0.f;
                        for (int q = 0; q < cs; q++) {
                            const float* pq = pr + q * MR * ps;
                            const float mq = pq[0];
                            const float w = mq == -INFINITY ? 0.f : __expf(mq - Ms);
                            ls += pq[1] * w;
                            A += pq[2 + dd] * w;
                        }
                        ctxs[p] = A / ls;
                    }
                    cons_sync();
                    MK_TRACE_L(18);
                    // ---- this CTA's columns of ctx_hh * Wproj[hh rows] -> x2 partials --
                    if (tid == 0) mk_ring_wait = 0;
                    it = mk_gemv_q4<MR>(ctxs, hd, wp, s_geo[1], ring, full, empty, a.nstage, it, gscr, hc_ys, a.err,
                                        &s_abort);
                    MK_TRACE_L(6);
                    if (l == 0) MK_TRACE_DUR(15, mk_ring_wait);
                    for (int m = 0; m < MR; m++)
                        for (int c = tid; c < wp; c += MK_CONS)
                            acc_add(accx2 + (size_t)m * D + rk * wp + c, acc_term(hc_ys[m * wp + c]));
                    MK_TRACE_L(7);
                }
                // ---- x2 = x + attention projection; LN2 -> fc -> GELU -> proj2 ------
                const float ffS = tid < J ? __ldg(ly.fold[1] + 2 * (j0 + tid)) : 0.f;  // folded LN2 of fc column
                const float ffB = tid < J ? __ldg(ly.fold[1] + 2 * (j0 + tid) + 1) : 0.f;
                // x2 = x + (projection + bias), with LN2's row moments (LN2 itself is
                // folded into fc)
                acc_gather_res<MR>(accx2, x2res, xres, D, bproj[0], bproj[1], bproj[2], bproj[3],
                                   (uint32_t)(nhead / cs), scr + 384, a.err, &s_abort);
                MK_TRACE_L(8);
                if (cons_sync_or(s_abort)) return;
                float bproj2[4];
                load_cols(ly.b[MK_PROJ2], bproj2);
                MK_TRACE_L(11);
                float* red_out = act;  // [cs][MR][wp] (MR <= 2): this CTA's proj2 partials by owner rank
                if (J > 0) {
                    float* hb = act + MR * D;  // [MR][J]
                    if (tid == 0) mk_ring_wait = 0;
                    it = mk_gemv_q4<MR>(x2res, D, J, s_geo[2], ring, full, empty, a.nstage, it, gscr, hc_ys, a.err,
                                        &s_abort, scr + 384, scr + 320);
                    MK_TRACE_L(12);
                    if (l == 0) MK_TRACE_DUR(16, mk_ring_wait);
                    if (tid < J)  // J <= 256
                        for (int m = 0; m < MR; m++) {
                            const float mu = scr[320 + 2 * m], rstd = scr[321 + 2 * m];
                            hb[m * J + tid] = gelu_tanh(rstd * (hc_ys[m * J + tid] - mu * ffS) + ffB);
                        }
                    cons_sync();
                    MK_TRACE_L(13);
                    if (tid == 0) mk_ring_wait = 0;
                    it = mk_gemv_wide_q4<MR>(hb, J, D, s_hci[5], ring, full, empty, a.nstage, it,
                                             MR <= 2 ? nullptr : accx, red_out, wp, a.err, &s_abort);
                    if (l == 0) MK_TRACE_DUR(17, mk_ring_wait);
                } else if (MR > 2) {
                    for (int p = tid; p < MR * D; p += MK_CONS) acc_add(accx + p, acc_term(0.f));
                } else {
                    for (int p = tid; p < MR * D; p += MK_CONS) red_out[p] = 0.f;  // no hidden units here
                }
                if (MR <= 2) {
                    // each column block to its owner (one bulk copy per cluster CTA,
                    // completing on the owner's mbar[1]); this CTA's block: the
                    // cluster's partials summed in rank order, one fixed-point term
                    // per cluster and column
                    fence_async_smem();
                    cons_sync();
                    if (tid < cs)
                        bulk_s2c(hc_rb[16 + tid] + (uint32_t)(rk * MR * wp) * 4u, red_out + tid * MR * wp,
                                 (uint32_t)(MR * wp) * 4u, hc_rb[32 + tid]);
                    if (tid == 0) mbar_expect_tx(&hc_mbar[1], (uint32_t)(cs * MR * wp) * 4u);
                    wait_cluster_bar(&hc_mbar[1], rnd & 1u, a.err, &s_abort);
                    if (cons_sync_or(s_abort)) return;
                    for (int m = 0; m < MR; m++)
                        for (int c = tid; c < wp; c += MK_CONS) {
                            float sum = 0.f;
                            for (int q = 0; q < cs; q++) sum += red_in[(q * MR + m) * wp + c];
                            acc_add(accx + (size_t)m * D + rk * wp + c, acc_term(sum));
                        }
                }
                MK_TRACE_L(9);
                // next layer's LN1 parameters and qkv bias, loaded during the wait
                if (is_head && l + 1 < L && tid < q3) {
                    fqS = __ldg(hc_lay[l + 1].fold[0] + 2 * qcol);
                    fqB = __ldg(hc_lay[l + 1].fold[0] + 2 * qcol + 1);
                }
                // ---- x of the next layer (every CTA) --------------------------------
                // x = x2 + (MLP output + bias), with the next layer's LN1 row moments
                acc_gather_res<MR>(accx, xres, x2res, D, bproj2[0], bproj2[1], bproj2[2], bproj2[3],
                                   (uint32_t)(MR <= 2 ? nW / cs : nW), scr + 384, a.err, &s_abort);
                if (cons_sync_or(s_abort)) return;
                MK_TRACE_L(10);
                if (l < 24) MK_TRACE(33 + l);
            }
        }
        for (int l = 0; l < L && !HC; l++) {
            const MkLayer& ly = a.layers[l];
            const uint32_t tg = mk_tag(gs, l, L);
            MK_TRACE_L(0);
            // small parameters of this layer, loaded ahead of their use
            const LnRegs ln1 = ln_prefetch(ly.ln1w, ly.ln1b, D);
            const LnRegs ln2 = ln_prefetch(ly.ln2w, ly.ln2b, D);
            float pb[4];
            {
                const int Ns[4] = {3 * D, D, F, D};
#pragma unroll
                for (int ph = 0; ph < 4; ph++) {
                    int n0, w;
                    strip(Ns[ph], nW, cta, n0, w);
                    pb[ph] = (w > 0 && tid < w * MR) ? __ldg(ly.b[ph] + n0 + tid % w) : 0.f;
                }
            }
            // ---- level A: x -> LN1 -> QKV (q, K/V to the cache) ----------------
            if (l == 0) {
                for (int m = 0; m < MR; m++) {
                    const float* te = a.tok_emb + (size_t)s_tok[m] * D;
                    const float* pe = a.pos_emb + (size_t)pos_of(m, s) * D;
                    for (int i = tid; i < D; i += MK_CONS) xres[m * D + i] = __ldg(te + i) + __ldg(pe + i);
                }
            } else {
                gather_tagged(a.xx, xres, MR * D, mk_tag(gs, l - 1, L), a.err, &s_abort);
            }
            if (cons_sync_or(s_abort)) return;
            mk_layernorm<MR>(xres, act, D, ln1, scr + 384);
            MK_TRACE_L(1);
            {
                const bool withhold = cta == a.withhold_cta && s == 0 && l == 0;
                auto epi = [&](int m, int n, float v) {
                    v += pb[MK_QKV];
                    if (n < D) {
                        if (!withhold) st_pair(a.xq + m * D + n, v, tg);
                        return;
                    }
                    const int which = n < 2 * D ? 0 : 1;
                    const int cc = n - D - which * D, h = cc / hd, d = cc - h * hd;
                    if (!s_dummy[m])
                        a.kv[(size_t)s_slot[m] * a.kv_slot_stride + (size_t)l * a.kv_layer_stride + (which ? a.v_offset : 0) +
                             ((size_t)h * a.ctx + pos_of(m, s)) * hd + d] = v;
                    st_pair(a.xkv + (size_t)m * 2 * D + (n - D), v, tg);
                };
                gemv(act, D, 3 * D, epi);
                MK_TRACE_L(2);
            }
            // ---- level B: attention units over the cached keys [0, pos-1) -----
            // Unit (m, h, c) = keys [c*KC, c*KC + nk) of head h.  Warp w takes
            // KC/8 keys (lpk lanes per key, 16 dims a lane), keeps its own
            // max / sum / p.V, and the 8 warps merge once at the end.
            {
                float* qs = scr;                  // [hd]
                float* wm = scr + 128;            // [8] warp max
                float* wl = scr + 136;            // [8] warp sum
                float* wacc = uacc;               // [8][hd] warp p.V
                const int kpw = KC / 8, lpk = 32 / kpw;  // keys per warp, lanes per key (16 dims a lane)
                const int kw = lane / lpk, part = lane - kw * lpk;
                for (int m = 0; m < MR; m++) {
                    const int nc = nch_of(m, s), old = pos_of(m, s) - 1, ubase = s_ubase[m];
                    for (int u = ubase + ((cta - ubase) % nW + nW) % nW; u < ubase + H * nc; u += nW) {
                        const int h = (u - ubase) / nc, c = (u - ubase) - h * nc;
                        const int nk = min(KC, old - c * KC);
                        if (tid < hd) qs[tid] = wait_pair(a.xq + m * D + h * hd + tid, tg, a.err, &s_abort);
                        cons_sync();
                        wait_full(full, it, a.nstage, a.err, &s_abort);
                        const float* Kt = reinterpret_cast<const float*>(ring + (size_t)rp_stage(it) * mk_sbytes);
                        const int j = warp * kpw + kw;  // this lane's key
                        float d = 0.f;
                        if (j < nk) {
                            const float4* kr = reinterpret_cast<const float4*>(Kt + j * hd) + part;
                            const float4* qr = reinterpret_cast<const float4*>(qs) + part;
#pragma unroll
                            for (int e4 = 0; e4 < 4; e4++) {  // dims 4*(part + lpk*e4) .. +3
                                const float4 k4 = kr[lpk * e4], q4 = qr[lpk * e4];
                                d += q4.x * k4.x + q4.y * k4.y + q4.z * k4.z + q4.w * k4.w;
                            }
                        }
                        for (int o = 1; o < lpk; o <<= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                        const float sc = j < nk ? d * scale : -INFINITY;
                        release_stage(empty, it, a.nstage);
                        it = rp_next(it, a.nstage);
                        const float mw = warp_max(sc);
                        const float p = j < nk ? __expf(sc - mw) : 0.f;
                        const float lw = warp_sum(part == 0 ? p : 0.f);
                        wait_full(full, it, a.nstage, a.err, &s_abort);
                        const float* Vt = reinterpret_cast<const float*>(ring + (size_t)rp_stage(it) * mk_sbytes);
                        float a0 = 0.f, a1 = 0.f;
                        for (int kk = 0; kk < kpw; kk++) {
                            const float pk = __shfl_sync(0xffffffffu, p, kk * lpk);
                            const int jj = warp * kpw + kk;
                            if (jj < nk) {
                                a0 += pk * Vt[jj * hd + lane];
                                if (hd > 32) a1 += pk * Vt[jj * hd + lane + 32];
                            }
                        }
                        release_stage(empty, it, a.nstage);
                        it = rp_next(it, a.nstage);
                        wacc[warp * hd + lane] = a0;
                        if (hd > 32) wacc[warp * hd + lane + 32] = a1;
                        if (lane == 0) {
                            wm[warp] = mw;
                            wl[warp] = lw;
                        }
                        cons_sync();
                        // partial record [max, sum, acc[hd]], every word tagged
                        if (tid < hd) {
                            float M = -INFINITY;
#pragma unroll
                            for (int w8 = 0; w8 < 8; w8++) M = fmaxf(M, wm[w8]);
                            float L = 0.f, A = 0.f;
#pragma unroll
                            for (int w8 = 0; w8 < 8; w8++) {
                                const float f = wm[w8] == -INFINITY ? 0.f : __expf(wm[w8] - M);
                                L += wl[w8] * f;
                                A += wacc[w8 * hd + tid] * f;
                            }
                            unsigned long long* pr = a.xpart + (size_t)u * (hd + 2);
                            st_pair(pr + 2 + tid, A, tg);
                            if (tid == 0) {
                                st_pair(pr, M, tg);
                                st_pair(pr + 1, L, tg);
                            }
                        }
                    }
                }
            }
            MK_TRACE_L(3);
            // ---- level C: combine partials + keys pos-1, pos -> ctx -> proj ---
            // phase 1, an 8-lane group per (row, head): log-sum-exp weights of
            // the key chunks and of the two directly read keys; ctx starts as
            // the direct keys' share.  Every load is issued before any is used.
            {
                const int grp = tid >> 3, l8 = tid & 7, dpl = hd >> 3;  // hd <= 64
                for (int p0 = 0; p0 < MR * H; p0 += 32) {
                    const int p = p0 + grp;
                    const bool on = p < MR * H;
                    const int m = on ? p / H : 0, h = on ? p - (p / H) * H : 0;
                    const int pos = pos_of(m, s), nc = on ? nch_of(m, s) : 0;
                    const int ub = s_ubase[m] + h * nc;
                    const int dq = m * D + h * hd + l8 * dpl;           // q / ctx column
                    const size_t dk = (size_t)m * 2 * D + h * hd + l8 * dpl;  // current K (V at +D)
                    unsigned long long wq[8], wk[8], wv[8], wmc[4], wlc[4];
                    float kp[8], vp[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        wq[e] = wk[e] = wv[e] = 0ull;
                        kp[e] = vp[e] = 0.f;
                    }
                    if (on) {
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            if (e >= dpl) break;
                            wq[e] = ld_pair(a.xq + dq + e);
                            wk[e] = ld_pair(a.xkv + dk + e);
                            wv[e] = ld_pair(a.xkv + dk + D + e);
                        }
                        if (pos >= 1) {
                            const float* kb = a.kv + (size_t)s_slot[m] * a.kv_slot_stride + (size_t)l * a.kv_layer_stride +
                                              ((size_t)h * a.ctx + pos - 1) * hd + l8 * dpl;
#pragma unroll
                            for (int e = 0; e < 8; e++) {
                                if (e >= dpl) break;
                                kp[e] = __ldcg(kb + e);
                                vp[e] = __ldcg(kb + a.v_offset + e);
                            }
                        }
                    }
#pragma unroll
                    for (int c4 = 0; c4 < 4; c4++) {
                        const int c = l8 + 8 * c4;
                        wmc[c4] = wlc[c4] = 0ull;
                        if (on && c < nc) {
                            const unsigned long long* pr = a.xpart + (size_t)(ub + c) * (hd + 2);
                            wmc[c4] = ld_pair(pr);
                            wlc[c4] = ld_pair(pr + 1);
                        }
                    }
                    {
                        // one wait over all 32 words: q, K, V (8 each), chunk (max, sum) x4
                        unsigned long long wall[32];
                        uint32_t pend = 0;
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            wall[e] = wq[e];
                            wall[8 + e] = wk[e];
                            wall[16 + e] = wv[e];
                            if (on && e < dpl) pend |= (1u << e) | (1u << (8 + e)) | (1u << (16 + e));
                        }
#pragma unroll
                        for (int c4 = 0; c4 < 4; c4++) {
                            wall[24 + c4] = wmc[c4];
                            wall[28 + c4] = wlc[c4];
                            if (on && l8 + 8 * c4 < nc) pend |= (1u << (24 + c4)) | (1u << (28 + c4));
                        }
                        auto addr = [&](int k) -> const unsigned long long* {
                            if (k < 8) return a.xq + dq + k;
                            if (k < 16) return a.xkv + dk + (k - 8);
                            if (k < 24) return a.xkv + dk + D + (k - 16);
                            const int c4 = (k - 24) & 3;
                            return a.xpart + (size_t)(ub + l8 + 8 * c4) * (hd + 2) + (k < 28 ? 0 : 1);
                        };
                        resolve_batch<32>(wall, pend, addr, tg, a.err, &s_abort);
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            wq[e] = wall[e];
                            wk[e] = wall[8 + e];
                            wv[e] = wall[16 + e];
                        }
#pragma unroll
                        for (int c4 = 0; c4 < 4; c4++) {
                            wmc[c4] = wall[24 + c4];
                            wlc[c4] = wall[28 + c4];
                        }
                    }
                    float dcur = 0.f, dprev = 0.f, vc[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        vc[e] = 0.f;
                        if (on && e < dpl) {
                            const float q = pair_value(wq[e]);
                            vc[e] = pair_value(wv[e]);
                            dcur += q * pair_value(wk[e]);
                            dprev += q * kp[e];
                        }
                    }
                    float mc[4], lc[4], mloc = -INFINITY;
#pragma unroll
                    for (int c4 = 0; c4 < 4; c4++) {
                        const int c = l8 + 8 * c4;
                        mc[c4] = -INFINITY;
                        lc[c4] = 0.f;
                        if (on && c < nc) {
                            mc[c4] = pair_value(wmc[c4]);
                            lc[c4] = pair_value(wlc[c4]);
                            mloc = fmaxf(mloc, mc[c4]);
                        }
                    }
#pragma unroll
                    for (int o = 1; o < 8; o <<= 1) {
                        dcur += __shfl_xor_sync(0xffffffffu, dcur, o);
                        dprev += __shfl_xor_sync(0xffffffffu, dprev, o);
                        mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, o));
                    }
                    dcur *= scale;
                    dprev *= scale;
                    float M = fmaxf(mloc, dcur);
                    if (pos >= 1) M = fmaxf(M, dprev);
                    float ls = 0.f;
#pragma unroll
                    for (int c4 = 0; c4 < 4; c4++) {
                        const int c = l8 + 8 * c4;
                        if (on && c < nc) {
                            mc[c4] = __expf(mc[c4] - M);
                            ls += lc[c4] * mc[c4];
                        }
                    }
#pragma unroll
                    for (int o = 1; o < 8; o <<= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
                    const float wcur = __expf(dcur - M), wprev = pos >= 1 ? __expf(dprev - M) : 0.f;
                    const float inv = 1.0f / (ls + wcur + wprev);
                    if (on) {
#pragma unroll
                        for (int c4 = 0; c4 < 4; c4++) {
                            const int c = l8 + 8 * c4;
                            if (c < nc) wts_m[(size_t)p * a.maxc + c] = mc[c4] * inv;
                        }
#pragma unroll
                        for (int e = 0; e < 8; e++)
                            if (e < dpl) act[dq + e] = (wcur * vc[e] + wprev * vp[e]) * inv;
                    }
                }
            }
            cons_sync();
            MK_TRACE_L(4);
            // phase 2, all threads: ctx += sum_c w_c * partial_c (tagged words,
            // eight loads in flight per thread)
            for (int e = tid; e < MR * D; e += MK_CONS) {
                const int m = e / D, col = e - m * D, h = col / hd, d = col - h * hd;
                const int nc = nch_of(m, s), ub = s_ubase[m] + h * nc;
                const float* wrow = wts_m + (size_t)(m * H + h) * a.maxc;
                float accc = 0.f;
                for (int c0 = 0; c0 < nc; c0 += 8) {
                    unsigned long long w8[8];
                    uint32_t pend = 0;
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        w8[j] = 0ull;
                        if (c0 + j < nc) {
                            w8[j] = ld_pair(a.xpart + (size_t)(ub + c0 + j) * (hd + 2) + 2 + d);
                            pend |= 1u << j;
                        }
                    }
                    resolve_batch<8>(w8, pend, [&](int j) { return a.xpart + (size_t)(ub + c0 + j) * (hd + 2) + 2 + d; },
                                     tg, a.err, &s_abort);
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        if (c0 + j < nc) accc += wrow[c0 + j] * pair_value(w8[j]);
                }
                act[e] += accc;
            }
            if (cons_sync_or(s_abort)) return;
            {
                auto epi = [&](int m, int n, float v) {
                    st_pair(a.xx2 + m * D + n, (v + pb[MK_PROJ]) + xres[m * D + n], tg);
                };
                MK_TRACE_L(5);
                gemv(act, D, D, epi);
                MK_TRACE_L(6);
            }
            // ---- level D: LN2 -> fc + GELU ---------------------------------------
            gather_tagged(a.xx2, x2res, MR * D, tg, a.err, &s_abort);
            if (cons_sync_or(s_abort)) return;
            MK_TRACE_L(7);
            mk_layernorm<MR>(x2res, act, D, ln2, scr + 384);
            {
                auto epi = [&](int m, int n, float v) {
                    st_pair(a.xh + (size_t)m * F + n, gelu_tanh(v + pb[MK_FC]), tg);
                };
                MK_TRACE_L(8);
                gemv(act, D, F, epi);
                MK_TRACE_L(9);
            }
            // ---- level E: proj2 + residual ----------------------------------------
            gather_tagged(a.xh, act, MR * F, tg, a.err, &s_abort);
            if (cons_sync_or(s_abort)) return;
            {
                auto epi = [&](int m, int n, float v) {
                    st_pair(a.xx + m * D + n, (v + pb[MK_PROJ2]) + x2res[m * D + n], tg);
                };
                MK_TRACE_L(10);
                gemv(act, F, D, epi);
                MK_TRACE_L(11);
                if (l < 24) MK_TRACE(33 + l);
            }
        }
        // ---- head: LN_f -> logits of this CTA's vocabulary slice ----------------
        const uint32_t th = mk_tag(gs, L, L);
        const LnRegs lnf = ln_prefetch(a.lnf_w, a.lnf_b, D);
        if constexpr (!HC) {
            gather_tagged(a.xx, xres, MR * D, mk_tag(gs, L - 1, L), a.err, &s_abort);
            if (cons_sync_or(s_abort)) return;
        } else {
            // zero the accumulator set the next step uses (the previous step's,
            // read by every CTA before this step began); the fence before this
            // step's header publish orders the zeros before the next step's adds
            const size_t W = (size_t)L * 2 * MK_MAX_ROWS * D;
            unsigned long long* z = a.acc + (size_t)((gs & 1u) ^ 1u) * W;
            const size_t z0 = (size_t)cta * W / nW, z1 = (size_t)(cta + 1) * W / nW;
            for (size_t i = z0 + tid; i < z1; i += MK_CONS) z[i] = 0ull;
        }
        MK_TRACE(25);
        // this step's uniform for row tid, loaded before the head (a cold
        // global load) and parked in shared memory before the sampler
        double ud_next = 0.0;
        if (sampled && tid < MR)
            ud_next = a.uniforms[(size_t)s_slot[tid] * a.uni_stride + min(s_cnt0[tid] + s, max(sp.max_new - 1, 0))];
        mk_layernorm<MR>(xres, act, D, lnf, scr + 384);
        MK_TRACE(26);
        const int v0 = (int)(((long long)cta * V) / nW), v1 = (int)(((long long)(cta + 1) * V) / nW);
        const int nsl = v1 - v0;
        {
            const int Rh = max(1, mk_sbytes / (D * 4));
            unsigned long long head_wait = 0;  // thread 0's time inside the ring waits (traced runs)
            for (int r0 = v0; r0 < v1; r0 += Rh) {
                const int rows = min(Rh, v1 - r0);
                if (a.trace && tid == 0) {
                    const unsigned long long t0 = gtimer();
                    wait_full(full, it, a.nstage, a.err, &s_abort);
                    head_wait += gtimer() - t0;
                } else {
                    wait_full(full, it, a.nstage, a.err, &s_abort);
                }
                if (r0 == v0) MK_TRACE(29);
                if (r0 - v0 == ((nsl / Rh) / 2) * Rh) MK_TRACE(45);
                const float* E = reinterpret_cast<const float*>(ring + (size_t)rp_stage(it) * mk_sbytes);
                // slice row idx = r0 - v0 + r goes to warp idx % 8: a warp with no
                // row here moves on to the next stage while the others finish
                // (every warp still waits for each stage before releasing it)
                for (int r = ((warp - (r0 - v0)) % 8 + 8) % 8; r < rows; r += 8) {
                    float acc0[MR], acc1[MR];
#pragma unroll
                    for (int m = 0; m < MR; m++) acc0[m] = acc1[m] = 0.f;
                    const float4* er = reinterpret_cast<const float4*>(E + (size_t)r * D);
                    const int n4 = D / 4;
                    int i = lane;
                    // six float4 of the row per lane issued before their FMAs
                    for (; i + 160 < n4; i += 192) {
                        float4 e[6];
#pragma unroll
                        for (int u = 0; u < 6; u++) e[u] = er[i + 32 * u];
#pragma unroll
                        for (int m = 0; m < MR; m++) {
                            float4 x[6];
#pragma unroll
                            for (int u = 0; u < 6; u++) x[u] = *reinterpret_cast<const float4*>(act + m * D + (i + 32 * u) * 4);
#pragma unroll
                            for (int u = 0; u < 6; u += 2) {
                                acc0[m] += x[u].x * e[u].x + x[u].y * e[u].y + x[u].z * e[u].z + x[u].w * e[u].w;
                                acc1[m] += x[u + 1].x * e[u + 1].x + x[u + 1].y * e[u + 1].y + x[u + 1].z * e[u + 1].z +
                                           x[u + 1].w * e[u + 1].w;
                            }
                        }
                    }
                    for (; i + 32 < n4; i += 64) {
                        const float4 e0 = er[i], e1 = er[i + 32];
#pragma unroll
                        for (int m = 0; m < MR; m++) {
                            const float4 x0 = *reinterpret_cast<const float4*>(act + m * D + i * 4);
                            const float4 x1 = *reinterpret_cast<const float4*>(act + m * D + (i + 32) * 4);
                            acc0[m] += x0.x * e0.x + x0.y * e0.y + x0.z * e0.z + x0.w * e0.w;
                            acc1[m] += x1.x * e1.x + x1.y * e1.y + x1.z * e1.z + x1.w * e1.w;
                        }
                    }
                    if (i < n4) {
                        const float4 e0 = er[i];
#pragma unroll
                        for (int m = 0; m < MR; m++) {
                            const float4 x0 = *reinterpret_cast<const float4*>(act + m * D + i * 4);
                            acc0[m] += x0.x * e0.x + x0.y * e0.y + x0.z * e0.z + x0.w * e0.w;
                        }
                    }
#pragma unroll
                    for (int m = 0; m < MR; m++) {
                        const float t = warp_sum(acc0[m] + acc1[m]);
                        if (lane == 0) slice[m * a.slice_max + (r0 - v0) + r] = t;
                    }
                }
                release_stage(empty, it, a.nstage);
                it = rp_next(it, a.nstage);
            }
            if (a.trace && tid == 0 && s < a.trace_steps)
                a.trace[((size_t)cta * a.trace_steps + s) * MK_TRACE_POINTS + 46] = head_wait;
        }
        cons_sync();
        MK_TRACE(27);
        // ---- candidates of this slice (repetition controls applied here) -------
        for (int m = 0; m < MR; m++) {
            float* sl = slice + m * a.slice_max;
            for (int i = tid; i < nsl; i += MK_CONS) a.logits_out[(size_t)m * V + v0 + i] = sl[i];
            const int wl = min(s_len0[m] + s, a.ctx);
            const int* wv = win + m * a.ctx + (s_len0[m] + s - wl);
            if (controls) {
                if (tid < 16) seen[tid] = 0u;  // clears seen[] and ban[]
                cons_sync();
                if (sp.penalty != 1.0f)  // once per distinct window token (Sampler.cs:117-127)
                    for (int i = tid; i < wl; i += MK_CONS) {
                        const int t = wv[i] - v0;
                        if (t >= 0 && t < nsl) atomicOr(&seen[t >> 5], 1u << (t & 31));
                    }
                if (sp.ngram > 0 && wl >= sp.ngram - 1) {  // Sampler.cs:129-154
                    const int n = sp.ngram;
                    if (n == 1) {
                        for (int i = tid; i < wl; i += MK_CONS) {
                            const int t = wv[i] - v0;
                            if (t >= 0 && t < nsl) atomicOr(&ban[t >> 5], 1u << (t & 31));
                        }
                    } else {
                        const int pre = n - 1, suf = wl - pre;
                        for (int st0 = tid; st0 + n <= wl; st0 += MK_CONS) {
                            bool match = true;
                            for (int j = 0; j < pre; j++)
                                if (wv[st0 + j] != wv[suf + j]) {
                                    match = false;
                                    break;
                                }
                            if (!match) continue;
                            const int t = wv[st0 + pre] - v0;
                            if (t >= 0 && t < nsl) atomicOr(&ban[t >> 5], 1u << (t & 31));
                        }
                    }
                }
                cons_sync();
                for (int i = tid; i < nsl; i += MK_CONS) {
                    float l = sl[i];
                    if ((seen[i >> 5] >> (i & 31)) & 1u) l = l < 0.0f ? l * sp.penalty : l / sp.penalty;
                    if ((ban[i >> 5] >> (i & 31)) & 1u) l = -INFINITY;
                    sl[i] = l;
                }
                cons_sync();
            }
            float* cv = a.cand_val + ((size_t)m * nW + cta) * a.slice_max;
            int* ci = a.cand_idx + ((size_t)m * nW + cta) * a.slice_max;
            if (!sampled) {  // local first argmax (Sampler.cs:14-20)
                float bv = -INFINITY;
                int bi = -1;
                for (int i = tid; i < nsl; i += MK_CONS) {
                    const float v = sl[i];
                    if (v != v) continue;
                    if (bi < 0 || v > bv) {
                        bv = v;
                        bi = i;
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
                        bv = ov;
                        bi = oi;
                    }
                }
                if (lane == 0) {
                    scr[warp] = bv;
                    wbi[warp] = bi;
                }
                cons_sync();
                if (tid == 0) {
                    float b = -INFINITY;
                    int ix = -1;
                    for (int w8 = 0; w8 < 8; w8++) {
                        const int oi = wbi[w8];
                        const float ov = scr[w8];
                        if (oi >= 0 && (ix < 0 || ov > b || (ov == b && oi < ix))) {
                            b = ov;
                            ix = oi;
                        }
                    }
                    int cnt = 0;
                    if (ix >= 0) {
                        cv[0] = b;
                        ci[0] = v0 + ix;
                        cnt = 1;
                    }
                    rcnt[m] = cnt;
                }
                cons_sync();
            } else {
                for (int i = tid; i < nsl; i += MK_CONS) sl[i] = sl[i] / sp.temperature;  // Sampler.cs:40
                cons_sync();
                // keep entries with fewer than k strictly larger ones (ties kept);
                // the slice's 4 largest entries (ties by lower index) go to the header
                float* top4 = reinterpret_cast<float*>(misc) + 48 + 4 * m;
                int* top4i = iscr + 160 + 4 * m;
                if (tid < 4) {
                    top4[tid] = -INFINITY;
                    top4i[tid] = -1;
                }
                cons_sync();
                int f = 0;
                if (tid < nsl) {
                    const float v = sl[tid];
                    int rank = 0, tie = 0;
                    for (int j = 0; j < nsl; j++) {
                        const float u = sl[j];
                        rank += u > v;
                        tie += (u == v) & (j < tid);
                    }
                    f = rank < sp.top_k;
                    if (rank + tie < 4) {
                        top4[rank + tie] = v;
                        top4i[rank + tie] = v0 + tid;
                    }
                }
                flag[tid] = f;
                // the local k-th largest (smallest kept value) is a lower bound
                // of the row's k-th largest; -inf when the slice has < k entries
                float lk = f ? sl[tid] : INFINITY;
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) lk = fminf(lk, __shfl_xor_sync(0xffffffffu, lk, o));
                if (lane == 0) scr[256 + warp] = lk;
                // exclusive scan of the flags -> candidate order = index order
                int x = f;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, x, o);
                    if (lane >= o) x += t;
                }
                if (lane == 31) misc[warp] = x;
                cons_sync();
                int base = 0;
                for (int w8 = 0; w8 < warp; w8++) base += misc[w8];
                if (f) {
                    cv[base + x - 1] = sl[tid];
                    ci[base + x - 1] = v0 + tid;
                }
                if (tid == 0) {
                    int tot = 0;
                    float mn = INFINITY;
                    for (int w8 = 0; w8 < 8; w8++) {
                        tot += misc[w8];
                        mn = fminf(mn, scr[256 + w8]);
                    }
                    rcnt[m] = tot;
                    (void)mn;
                }
                cons_sync();
            }
        }
        MK_TRACE(28);
        // publish: release every plain write of this step (K/V cache, logits,
        // candidates), then per (row, slice) the tagged count and local k-th
        if (tid < MR) s_ud[tid] = ud_next;
        __threadfence();
        cons_sync();
        if (tid < MR) {
            unsigned long long* hp = a.cand_hdr + ((size_t)tid * nW + cta) * 9;
            const float* top4 = reinterpret_cast<float*>(misc) + 48 + 4 * tid;
            const int* top4i = iscr + 160 + 4 * tid;
            st_pair(hp, __int_as_float(rcnt[tid]), th);
            for (int q4 = 0; q4 < 4; q4++) {
                st_pair(hp + 1 + 2 * q4, sampled ? top4[q4] : -INFINITY, th);
                st_pair(hp + 2 + 2 * q4, __int_as_float(sampled ? top4i[q4] : -1), th);
            }
        }
        MK_TRACE(30);
        // ---- finalize: every CTA computes the same token for each row ----------
        for (int m = 0; m < MR; m++) {
            float* tops = hstage;                                    // [nW][4] slices' largest values
            int* topi = reinterpret_cast<int*>(hstage + 4 * 256);  // [nW][4] their vocabulary ids
            if (tid < nW) {  // nW <= 256: one slice header per thread
                const unsigned long long* hp = a.cand_hdr + ((size_t)m * nW + tid) * 9;
                unsigned long long w[9];
#pragma unroll
                for (int q4 = 0; q4 < 9; q4++) w[q4] = ld_pair(hp + q4);
                resolve_batch<9>(w, 0x1ffu, [&](int k) { return hp + k; }, th, a.err, &s_abort);
                if (m == 0) MK_TRACE(55);
                cnts[tid] = __float_as_int(pair_value(w[0]));
#pragma unroll
                for (int q4 = 0; q4 < 4; q4++) {
                    tops[tid * 4 + q4] = pair_value(w[1 + 2 * q4]);
                    topi[tid * 4 + q4] = __float_as_int(pair_value(w[2 + 2 * q4]));
                }
            }
            if (cons_sync_or(s_abort)) return;
            if (m == 0) MK_TRACE(56);
            fence_acq_rel();
            if (m == 0) MK_TRACE(57);
            if (!sampled) {
                // one candidate (the slice's first argmax) per slice
                float bv = -INFINITY;
                int bi = -1;
                if (tid < nW && cnts[tid] > 0) {
                    const size_t at = ((size_t)m * nW + tid) * a.slice_max;
                    bv = __ldcg(a.cand_val + at);
                    bi = __ldcg(a.cand_idx + at);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) {
                        bv = ov;
                        bi = oi;
                    }
                }
                if (lane == 0) {
                    scr[warp] = bv;
                    wbi[warp] = bi;
                }
                cons_sync();
                if (tid == 0) {
                    float b = -INFINITY;
                    int ix = -1;
                    for (int w8 = 0; w8 < 8; w8++) {
                        const int oi = wbi[w8];
                        const float ov = scr[w8];
                        if (oi >= 0 && (ix < 0 || ov > b || (ov == b && oi < ix))) {
                            b = ov;
                            ix = oi;
                        }
                    }
                    rtok[m] = ix < 0 ? 0 : ix;
                }
                cons_sync();
            } else {
                // lower bound of the row's k-th largest: the k-th largest of the
                // slices' top values (a subset of the row)
                const int ntops = 4 * nW;
                const float tlo =
                    cons_kth_tops(tops, nW, min(sp.top_k, ntops), reinterpret_cast<uint32_t*>(iscr + 768), misc + 24);
                if (m == 0) MK_TRACE(58);
                // stage every candidate >= the bound: from the header when the
                // slice's 4th largest is below the bound (then every such entry
                // is among its top 4), else from the slice's list
                int q = 0;
                const float* cvs = a.cand_val + ((size_t)m * nW + tid) * a.slice_max;
                const int* cis = a.cand_idx + ((size_t)m * nW + tid) * a.slice_max;
                const int mycnt = tid < nW ? cnts[tid] : 0;
                const bool from_list = tid < nW && !(tops[tid * 4 + 3] < tlo);
                if (tid < nW) {
                    if (from_list) {
                        for (int i = 0; i < mycnt; i++) q += !(__ldcg(cvs + i) < tlo);
                    } else {
#pragma unroll
                        for (int q4 = 0; q4 < 4; q4++) q += topi[tid * 4 + q4] >= 0 && !(tops[tid * 4 + q4] < tlo);
                    }
                }
                // when no slice needed its list, every entry >= the bound is
                // among the tops, so the bound is the row's exact k-th largest
                const int any_list = cons_sync_or(from_list ? 1 : 0);
                int Q;
                const int off = cons_excl_scan(q, misc + 16, Q);
                if (m == 0) MK_TRACE(59);
                if (Q <= MK_SURV_MAX && tid < nW) {
                    int o = off;
                    if (from_list) {
                        for (int i = 0; i < mycnt; i++) {
                            const float v = __ldcg(cvs + i);
                            if (v < tlo) continue;
                            surv_v[o] = v;
                            surv_i[o] = __ldcg(cis + i);
                            o++;
                        }
                    } else {
#pragma unroll
                        for (int q4 = 0; q4 < 4; q4++)
                            if (topi[tid * 4 + q4] >= 0 && !(tops[tid * 4 + q4] < tlo)) {
                                surv_v[o] = tops[tid * 4 + q4];
                                surv_i[o] = topi[tid * 4 + q4];
                                o++;
                            }
                    }
                }
                cons_sync();
                if (Q <= MK_SURV_MAX) {
                    // index order (the serial sums follow it): rank by vocabulary id
                    float rv[2];
                    int ri[2], rr[2];
#pragma unroll
                    for (int j2 = 0; j2 < 2; j2++) {
                        const int i = tid + j2 * MK_CONS;
                        rr[j2] = -1;
                        if (i < Q) {
                            rv[j2] = surv_v[i];
                            ri[j2] = surv_i[i];
                            int r = 0;
                            for (int j = 0; j < Q; j++) r += surv_i[j] < ri[j2];
                            rr[j2] = r;
                        }
                    }
                    cons_sync();
#pragma unroll
                    for (int j2 = 0; j2 < 2; j2++)
                        if (rr[j2] >= 0) {
                            surv_v[rr[j2]] = rv[j2];
                            surv_i[rr[j2]] = ri[j2];
                        }
                    cons_sync();
                }
                if (Q <= MK_SURV_MAX) {
                    // exact threshold: smallest staged value with < k larger ones
                    if (m == 0) MK_TRACE(60);
                    float thr = INFINITY, mx = -INFINITY;
                    for (int i = tid; i < Q; i += MK_CONS) {
                        const float v = surv_v[i];
                        mx = fmaxf(mx, v);
                        if (any_list) {
                            int rank = 0;
                            for (int j = 0; j < Q; j++) rank += surv_v[j] > v;
                            if (rank < sp.top_k) thr = fminf(thr, v);
                        }
                    }
                    if (!any_list) thr = tlo;
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        thr = fminf(thr, __shfl_xor_sync(0xffffffffu, thr, o));
                        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                    }
                    if (lane == 0) {
                        scr[256 + warp] = thr;
                        scr[264 + warp] = mx;
                    }
                    cons_sync();
                    float T = INFINITY, M = -INFINITY;
                    for (int w8 = 0; w8 < 8; w8++) {
                        T = fminf(T, scr[256 + w8]);
                        M = fmaxf(M, scr[264 + w8]);
                    }
                    // exponentials of the survivors in parallel (Sampler.cs:57),
                    if (m == 0) MK_TRACE(61);
                    // zero for the entries below the threshold
                    for (int i = tid; i < Q; i += MK_CONS) {
                        const float v = surv_v[i];
                        surv_v[i] = (v < T) ? 0.0f : expf_libm(v - M);
                    }
                    cons_sync();
                    if (tid == 0) {
                        const double ud = s_ud[m];
                        float sum = 0.0f;  // index order (Sampler.cs:54-59)
                        for (int i = 0; i < Q; i++) sum += surv_v[i];
                        const float uu = (float)ud * sum;  // Sampler.cs:61
                        float accp = 0.0f;
                        int pick = V - 1;  // rounding fallback (Sampler.cs:68)
                        for (int i = 0; i < Q; i++) {
                            accp += surv_v[i];
                            if (uu < accp) {
                                pick = surv_i[i];
                                break;
                            }
                        }
                        if (sum != sum) pick = V - 1;
                        rtok[m] = pick;
                    }
                    cons_sync();
                    if (m == 0) MK_TRACE(62);
                } else {
                    // more candidates above the bound than shared memory stages
                    // (massive ties): radix-select the threshold over memory,
                    // each thread scanning its slice's list
                    uint32_t* hist = reinterpret_cast<uint32_t*>(scr);
                    if (tid == 0) {
                        misc[0] = 0;
                        misc[1] = 0;
                        misc[2] = sp.top_k;
                    }
                    cons_sync();
                    for (int shift = 24; shift >= 0; shift -= 8) {
                        hist[tid] = 0u;
                        const uint32_t prefix = (uint32_t)misc[0], mask = (uint32_t)misc[1];
                        cons_sync();
                        for (int i = 0; i < mycnt; i++) {
                            const float v = __ldcg(cvs + i);
                            if (v < tlo) continue;
                            const uint32_t key = float_key(v);
                            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
                        }
                        cons_sync();
                        if (warp == 0) {
                            const int kk = misc[2];
                            int bin, above;
                            radix_pick(hist, kk, bin, above);
                            if (lane == 0) {
                                misc[0] = (int)(prefix | ((uint32_t)bin << shift));
                                misc[1] = (int)(mask | (255u << shift));
                                misc[2] = kk - above;
                            }
                        }
                        cons_sync();
                    }
                    const float T = key_float((uint32_t)misc[0]);
                    // survivors (>= T), in index order
                    int ns = 0;
                    float mx = -INFINITY;
                    for (int i = 0; i < mycnt; i++) {
                        const float v = __ldcg(cvs + i);
                        if (v < T) continue;
                        ns++;
                        mx = fmaxf(mx, v);
                    }
                    mx = warp_max(mx);
                    if (lane == 0) scr[264 + warp] = mx;
                    int S;
                    const int so = cons_excl_scan(ns, misc + 16, S);
                    float M = -INFINITY;
                    for (int w8 = 0; w8 < 8; w8++) M = fmaxf(M, scr[264 + w8]);
                    if (S <= MK_SURV_MAX) {
                        int o = so;
                        for (int i = 0; i < mycnt; i++) {
                            const float v = __ldcg(cvs + i);
                            if (v < T) continue;
                            surv_v[o] = expf_libm(v - M);  // Sampler.cs:57
                            surv_i[o] = __ldcg(cis + i);
                            o++;
                        }
                    }
                    cons_sync();
                    if (tid == 0) {
                        const double ud = s_ud[m];
                        float sum = 0.0f;
                        int pick = V - 1;
                        if (S <= MK_SURV_MAX) {
                            for (int i = 0; i < S; i++) sum += surv_v[i];
                            const float uu = (float)ud * sum;
                            float accp = 0.0f;
                            for (int i = 0; i < S; i++) {
                                accp += surv_v[i];
                                if (uu < accp) {
                                    pick = surv_i[i];
                                    break;
                                }
                            }
                        } else {  // serial over the lists, one pass each for sum and draw
                            for (int c = 0; c < nW; c++)
                                for (int i = 0; i < cnts[c]; i++) {
                                    const float v = __ldcg(a.cand_val + ((size_t)m * nW + c) * a.slice_max + i);
                                    if (!(v < T)) sum += expf_libm(v - M);
                                }
                            const float uu = (float)ud * sum;
                            float accp = 0.0f;
                            for (int c = 0; c < nW && pick == V - 1; c++)
                                for (int i = 0; i < cnts[c]; i++) {
                                    const size_t at = ((size_t)m * nW + c) * a.slice_max + i;
                                    const float v = __ldcg(a.cand_val + at);
                                    if (v < T) continue;
                                    accp += expf_libm(v - M);
                                    if (uu < accp) {
                                        pick = __ldcg(a.cand_idx + at);
                                        break;
                                    }
                                }
                        }
                        if (sum != sum) pick = V - 1;
                        rtok[m] = pick;
                    }
                    cons_sync();
                }
            }
            // bookkeeping (CTA 0) and this CTA's state for the next step
            if (tid == 0) {
                const int tok = rtok[m];
                if (!s_dead[m]) {
                    const int c = s_cnt0[m] + s;
                    const bool fin = (sp.eos >= 0 && tok == sp.eos) || c + 1 >= sp.max_new;
                    if (a.bookkeep && cta == 0) {
                        const int slot = s_slot[m];
                        a.out_tokens[(size_t)slot * a.out_stride + c] = tok;
                        a.hist[(size_t)slot * a.hist_stride + s_len0[m] + s] = tok;
                        a.len[slot] = s_len0[m] + s + 1;
                        a.count[slot] = c + 1;
                        if (fin) a.done[slot] = 1;
                    }
                    if (fin) s_dead[m] = 1;
                }
                s_tok[m] = tok;
                if (controls && s_len0[m] + s < a.ctx) win[m * a.ctx + s_len0[m] + s] = tok;
            }
            cons_sync();
        }
        MK_TRACE(31);
        if (tid == 0) {
            __threadfence();
            atomicAdd(a.stepdone, 1u);
        }
        MK_TRACE(32);
    }
    };
    consumers();
    if constexpr (HC) {
        // no CTA of a cluster leaves while a cluster CTA may still write
        // into its shared memory: each arrives on every CTA's exit barrier after
        // its last push, then waits (bounded) for all of them
        cons_sync();
        if (tid == 0)
            for (int q = 0; q < a.cs; q++) mbar_arrive_cluster(dsmem_addr(&hc_mbar[4], q));
        const unsigned long long t0 = gtimer();
        while (!mbar_try_cluster(&hc_mbar[4], 0))
            if (gtimer() - t0 > 4 * mk_wait_ns) break;
        // after an abort a cluster CTA's last bulk copy into this CTA's shared
        // memory may not have been waited for: let it land before leaving
        if (s_abort) {
            const unsigned long long t1 = gtimer();
            while (gtimer() - t1 < 50000ull) __nanosleep(1000);
        }
    }
}

}  // namespace fb2
