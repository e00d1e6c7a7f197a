// sampler.cuh — on-device restatement of the reference sampler
// (src/LLM.Core/Inference/Sampler.cs), bit-exact given the same logits,
// window and uniform:
//   ApplyRepetitionControls (Sampler.cs:111-165): penalty once per distinct
//     window token (l<0 ? l*p : l/p); no-repeat-ngram ban; if the ban would
//     leave every logit at -inf, the pre-ban values stand.
//   Sample (Sampler.cs:29-69): temperature <= 0 -> first argmax (no draw);
//     else l / T (true division), top-k threshold = k-th largest (ties kept),
//     exp(l - max) with the host libm expf, sum in index order, then the
//     first index whose running sum exceeds (float)u * sum, else V-1.
// One CTA of 1024 threads per row; the logits row lives in shared memory.
#pragma once
#include "common.cuh"
#include "expf_libm.cuh"

namespace fb2 {

constexpr int kSampleThreads = 1024;

struct SampleParams {
    float temperature;
    int top_k;
    float penalty;
    int ngram;
    int eos;
    int max_new;
};

// Shared memory needed for vocabulary V.
inline size_t sampler_smem_bytes(int V) {
    size_t words = (size_t)(V + 31) / 32;
    return (size_t)V * 4 /*vals*/ + (size_t)V * 4 /*list*/ + 2 * words * 4 + 256 * 4 + 64;
}

struct SampleSmem {
    float* vals;
    int* list;
    uint32_t* seen;
    uint32_t* ban;
    uint32_t* hist;
};

FB2_DEV SampleSmem carve(void* base, int V) {
    SampleSmem s;
    size_t words = (size_t)(V + 31) / 32;
    s.vals = reinterpret_cast<float*>(base);
    s.list = reinterpret_cast<int*>(s.vals + V);
    s.seen = reinterpret_cast<uint32_t*>(s.list + V);
    s.ban = s.seen + words;
    s.hist = s.ban + words;
    return s;
}

// Block-wide argmax with the reference tie rule (first index of the max;
// NaN at index 0 wins because nothing compares greater than it).
FB2_DEV int block_argmax(const float* vals, int V) {
    __shared__ float bv[32];
    __shared__ int bi[32];
    __shared__ int result;
    float best = -INFINITY;
    int bidx = -1;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        float v = vals[i];
        if (v != v) continue;
        if (bidx < 0 || v > best) { best = v; bidx = i; }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float ov = __shfl_xor_sync(0xffffffffu, best, o);
        int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
        if (oi >= 0 && (bidx < 0 || ov > best || (ov == best && oi < bidx))) { best = ov; bidx = oi; }
    }
    if (lane == 0) { bv[warp] = best; bi[warp] = bidx; }
    __syncthreads();
    if (warp == 0) {
        int nw = blockDim.x >> 5;
        best = lane < nw ? bv[lane] : -INFINITY;
        bidx = lane < nw ? bi[lane] : -1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ov = __shfl_xor_sync(0xffffffffu, best, o);
            int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
            if (oi >= 0 && (bidx < 0 || ov > best || (ov == best && oi < bidx))) { best = ov; bidx = oi; }
        }
        if (lane == 0) {
            float v0 = vals[0];
            result = (v0 != v0 || bidx < 0) ? 0 : bidx;
        }
    }
    __syncthreads();
    return result;
}

// k-th largest value of vals[0..V) in Array.Sort order (4-pass radix select).
FB2_DEV float block_kth_largest(const float* vals, int V, int k, uint32_t* hist) {
    __shared__ uint32_t s_prefix, s_mask;
    __shared__ int s_k;
    if (threadIdx.x == 0) { s_prefix = 0; s_mask = 0; s_k = k; }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        const uint32_t prefix = s_prefix, mask = s_mask;
        // warp-aggregated histogram: logits cluster in few bins, so lanes with
        // the same digit add once (every lane runs the same trip count)
        for (int base = 0; base < V; base += blockDim.x) {
            const int i = base + threadIdx.x;
            uint32_t digit = 256u;
            if (i < V) {
                uint32_t key = float_key(vals[i]);
                if ((key & mask) == prefix) digit = (key >> shift) & 255u;
            }
            const unsigned grp = __match_any_sync(0xffffffffu, digit);
            if (digit < 256u && (threadIdx.x & 31) == __ffs(grp) - 1) atomicAdd(&hist[digit], (uint32_t)__popc(grp));
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            const int lane = threadIdx.x;
            // lane owns bins [lane*8, lane*8+8)
            uint32_t c[8], local = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) { c[j] = hist[lane * 8 + j]; local += c[j]; }
            // exclusive suffix sum over lanes (count in bins above this lane's range)
            uint32_t incl = local;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                uint32_t t = __shfl_down_sync(0xffffffffu, incl, o);
                if (lane + o < 32) incl += t;
            }
            uint32_t above = incl - local;
            int kk = s_k;
            int found = -1;
            uint32_t new_above = 0;
            if ((int)above < kk && (int)incl >= kk) {
                uint32_t acc = above;
#pragma unroll
                for (int j = 7; j >= 0; j--) {
                    if (found < 0) {
                        if ((int)(acc + c[j]) >= kk) { found = lane * 8 + j; new_above = acc; }
                        else acc += c[j];
                    }
                }
            }
            unsigned bal = __ballot_sync(0xffffffffu, found >= 0);
            int src = __ffs(bal) - 1;
            int bin = __shfl_sync(0xffffffffu, found, src < 0 ? 0 : src);
            uint32_t na = __shfl_sync(0xffffffffu, new_above, src < 0 ? 0 : src);
            if (lane == 0) {
                if (src < 0) bin = 0;  // cannot happen for 1 <= k <= V
                s_prefix = prefix | ((uint32_t)bin << shift);
                s_mask = mask | (255u << shift);
                s_k = kk - (int)na;
            }
        }
        __syncthreads();
    }
    return key_float(s_prefix);
}

// Samples one id from `logits` (global, V floats) with the window `win`.
// Returns the id (same value in every thread).
FB2_DEV int sample_row(const float* __restrict__ logits, const int* __restrict__ win, int wlen, const SampleParams& sp,
                       double u, int V, SampleSmem S) {
    const int tid = threadIdx.x, nt = blockDim.x;
    const int words = (V + 31) / 32;
    for (int i = tid; i < V; i += nt) S.vals[i] = logits[i];
    const bool controls = sp.penalty != 1.0f || sp.ngram > 0;  // Sampler.cs:98
    if (controls && sp.penalty != 1.0f) {
        for (int i = tid; i < words; i += nt) S.seen[i] = 0u;
        __syncthreads();
        for (int i = tid; i < wlen; i += nt) {
            int t = win[i];
            if ((unsigned)t >= (unsigned)V) continue;
            uint32_t bit = 1u << (t & 31);
            uint32_t old = atomicOr(&S.seen[t >> 5], bit);
            if (!(old & bit)) {
                float l = S.vals[t];
                S.vals[t] = l < 0.0f ? l * sp.penalty : l / sp.penalty;
            }
        }
    }
    __syncthreads();
    if (controls && sp.ngram > 0 && wlen >= sp.ngram - 1) {
        for (int i = tid; i < words; i += nt) S.ban[i] = 0u;
        __syncthreads();
        const int n = sp.ngram;
        if (n == 1) {
            for (int i = tid; i < wlen; i += nt) {
                int t = win[i];
                if ((unsigned)t < (unsigned)V) atomicOr(&S.ban[t >> 5], 1u << (t & 31));
            }
        } else {
            const int prefix = n - 1, suffix = wlen - prefix;
            for (int start = tid; start + n <= wlen; start += nt) {
                bool match = true;
                for (int j = 0; j < prefix; j++)
                    if (win[start + j] != win[suffix + j]) { match = false; break; }
                if (!match) continue;
                int t = win[start + prefix];
                if ((unsigned)t < (unsigned)V) atomicOr(&S.ban[t >> 5], 1u << (t & 31));
            }
        }
        __syncthreads();
        // Would any logit stay finite-or-+inf (not -inf) after the ban?
        int avail = 0;
        for (int i = tid; i < V; i += nt) {
            bool banned = (S.ban[i >> 5] >> (i & 31)) & 1u;
            float l = S.vals[i];
            if (!banned && !(l == -INFINITY)) avail = 1;
        }
        avail = __syncthreads_or(avail);
        if (avail) {
            for (int i = tid; i < V; i += nt)
                if ((S.ban[i >> 5] >> (i & 31)) & 1u) S.vals[i] = -INFINITY;
        }
        __syncthreads();
    }
    if (!(sp.temperature > 0.0f)) return block_argmax(S.vals, V);  // Sampler.cs:35

    for (int i = tid; i < V; i += nt) S.vals[i] = S.vals[i] / sp.temperature;  // Sampler.cs:40
    __syncthreads();
    if (sp.top_k > 0 && sp.top_k < V) {  // Sampler.cs:42-50
        float thr = block_kth_largest(S.vals, V, sp.top_k, S.hist);
        for (int i = tid; i < V; i += nt)
            if (S.vals[i] < thr) S.vals[i] = -INFINITY;
        __syncthreads();
    }
    // max (Sampler.cs:52-53): NaN never compares greater, start at -inf
    __shared__ float wm[32];
    float mx = -INFINITY;
    for (int i = tid; i < V; i += nt) {
        float v = S.vals[i];
        if (v > mx) mx = v;
    }
    mx = warp_max(mx);
    if ((tid & 31) == 0) wm[tid >> 5] = mx;
    __syncthreads();
    if (tid < 32) {
        float v = tid < (nt >> 5) ? wm[tid] : -INFINITY;
        v = warp_max(v);
        if (tid == 0) wm[0] = v;
    }
    __syncthreads();
    mx = wm[0];
    // exponentials; contiguous ranges per thread so the compaction keeps index order
    const int per = (V + nt - 1) / nt;
    const int b0 = min(V, tid * per), b1 = min(V, b0 + per);
    int cnt = 0, has_nan = 0;
    for (int i = b0; i < b1; i++) {
        float e = expf_libm(S.vals[i] - mx);
        S.vals[i] = e;
        if (e != e) has_nan = 1;
        else if (e != 0.0f) cnt++;
    }
    has_nan = __syncthreads_or(has_nan);
    if (has_nan) return V - 1;  // NaN poisons the sum: every `u < acc` test fails
    // exclusive scan of cnt over the block
    __shared__ int wsum[32];
    int lane = tid & 31, warp = tid >> 5;
    int x = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += t;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int y = lane < (nt >> 5) ? wsum[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int t = __shfl_up_sync(0xffffffffu, y, o);
            if (lane >= o) y += t;
        }
        wsum[lane] = y;  // inclusive
    }
    __syncthreads();
    int off = x - cnt + (warp > 0 ? wsum[warp - 1] : 0);
    const int total = wsum[(nt >> 5) - 1];
    for (int i = b0; i < b1; i++)
        if (S.vals[i] != 0.0f) S.list[off++] = i;
    __syncthreads();
    __shared__ int s_pick;
    if (tid == 0) {
        float sum = 0.0f;  // sequential, index order (Sampler.cs:54-59)
        for (int j = 0; j < total; j++) sum += S.vals[S.list[j]];
        float uu = (float)u * sum;  // Sampler.cs:61
        float acc = 0.0f;
        int pick = V - 1;
        for (int j = 0; j < total; j++) {
            int i = S.list[j];
            acc += S.vals[i];
            if (uu < acc) { pick = i; break; }
        }
        s_pick = pick;
    }
    __syncthreads();
    return s_pick;
}

// Generate-mode sampling step: one CTA per session slot.  Appends the id to
// the slot's history and output row; marks the slot done on EOS.
__global__ void __launch_bounds__(kSampleThreads) k_sample_step(
    int n, const float* __restrict__ logits, int V, int ctx, int* __restrict__ hist, int hist_stride,
    int* __restrict__ len, int* __restrict__ count, int* __restrict__ done, const double* __restrict__ uniforms,
    int uni_stride, SampleParams sp, int* __restrict__ out_tokens, int out_stride) {
    pdl_wait();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int s = blockIdx.x;
    if (s >= n) return;
    if (done[s] || count[s] >= sp.max_new) return;
    const int L = len[s];
    const int wlen = min(L, ctx);
    const int* win = hist + (size_t)s * hist_stride + (L - wlen);
    const int c = count[s];
    double u = (sp.temperature > 0.0f) ? uniforms[(size_t)s * uni_stride + c] : 0.0;
    SampleSmem S = carve(smem_raw, V);
    int id = sample_row(logits + (size_t)s * V, win, wlen, sp, u, V, S);
    if (threadIdx.x == 0) {
        out_tokens[(size_t)s * out_stride + c] = id;
        hist[(size_t)s * hist_stride + L] = id;
        len[s] = L + 1;
        count[s] = c + 1;
        if ((sp.eos >= 0 && id == sp.eos) || c + 1 >= sp.max_new) done[s] = 1;
    }
}

// Standalone sampling of n given rows (parity hook fb2_sample_logits).
__global__ void __launch_bounds__(kSampleThreads) k_sample_rows(int n, const float* __restrict__ logits, int V,
                                                                const int* __restrict__ windows,
                                                                const int* __restrict__ win_off,
                                                                const int* __restrict__ win_len,
                                                                const double* __restrict__ uniforms, SampleParams sp,
                                                                int* __restrict__ out_ids) {
    pdl_wait();
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int r = blockIdx.x;
    if (r >= n) return;
    SampleSmem S = carve(smem_raw, V);
    int id = sample_row(logits + (size_t)r * V, windows + win_off[r], win_len[r], sp, uniforms ? uniforms[r] : 0.0, V, S);
    if (threadIdx.x == 0) out_ids[r] = id;
}

// Test hook: device expf_libm over an array (compared with the host libm).
__global__ void k_expf_libm(const float* __restrict__ x, float* __restrict__ y, long long n) {
    pdl_wait();
    long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) y[i] = expf_libm(x[i]);
}

// Test hook: exhaustive range check.  For each chunk of 2^20 consecutive
// float bit patterns starting at lo_bits, a 64-bit hash of the outputs.
__global__ void k_expf_libm_hash(uint32_t lo_bits, int nchunks, unsigned long long* __restrict__ hashes) {
    pdl_wait();
    const int chunk = blockIdx.x;
    if (chunk >= nchunks) return;
    unsigned long long h = 0;
    for (uint32_t j = threadIdx.x; j < (1u << 20); j += blockDim.x) {
        uint32_t bits = lo_bits + (uint32_t)chunk * (1u << 20) + j;
        float x = __uint_as_float(bits);
        uint32_t o = (x != x) ? 0u : __float_as_uint(expf_libm(x));
        unsigned long long v = ((unsigned long long)o * 0x9E3779B97F4A7C15ull) ^ ((unsigned long long)bits << 17);
        h += v * 0xBF58476D1CE4E5B9ull + (v >> 29);
    }
    // order-independent combine across threads
    atomicAdd(&hashes[chunk], h);
}

}  // namespace fb2
