// kernels.cuh — decode/prefill kernels of libforge_b200 (sm_100a, fp32).
//
// Row model: every kernel works on "rows".  A row is one token position of one
// sequence: row_seq[r] (session slot), row_pos[r] (position in the window),
// row_hidx[r] (index into that slot's token history), row_active[r].
// Prefill pushes all window rows of a set of sequences; a decode step pushes
// one row per sequence.
//
// KV cache layout (fp32): [slot][layer][K|V][head][ctx][head_dim], so one
// head's keys are a contiguous [ctx][head_dim] block that attention streams.
#pragma once
#include "common.cuh"
#include "expf_libm.cuh"

namespace fb2 {

// ---------------------------------------------------------------------------
// Row bookkeeping
// ---------------------------------------------------------------------------
struct Rows {
    const int* seq;     // [rows] session slot
    const int* pos;     // [rows] position in the window (0-based)
    const int* hidx;    // [rows] index into the slot's history
    const int* active;  // [rows] 0: skip (finished / handled elsewhere)
};

// Decode-step rows: one per slot, position = current length - 1.
// A slot whose window would exceed the context (len > ctx) is re-prefilled by
// the host instead (Sampler.cs:93-94), so it is inactive here.
__global__ void k_step_prepare(int n, const int* __restrict__ len, const int* __restrict__ done, int ctx,
                               int* row_seq, int* row_pos, int* row_hidx, int* row_active) {
    pdl_wait();
    int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;
    int L = len[r];
    int act = (!done[r]) && L >= 1 && L <= ctx;
    row_seq[r] = r;
    row_pos[r] = act ? L - 1 : 0;
    row_hidx[r] = act ? L - 1 : 0;
    row_active[r] = act;
}

// x[r] = tok_emb[token] + pos_emb[pos]  (Layers.cs:347-353; GptModel.cs:217-218).
__global__ void k_embed(int rows, Rows R, const int* __restrict__ hist, int hist_stride,
                        const float* __restrict__ tok_emb, const float* __restrict__ pos_emb, int D, int V,
                        float* __restrict__ x) {
    pdl_wait();
    int r = blockIdx.x;
    if (r >= rows) return;
    int s = R.seq[r];
    int tok = hist[(size_t)s * hist_stride + R.hidx[r]];
    if (tok < 0 || tok >= V || !R.active[r]) tok = 0;  // inactive rows compute harmless values
    int p = R.active[r] ? R.pos[r] : 0;
    const float4* te = reinterpret_cast<const float4*>(tok_emb + (size_t)tok * D);
    const float4* pe = reinterpret_cast<const float4*>(pos_emb + (size_t)p * D);
    float4* xo = reinterpret_cast<float4*>(x + (size_t)r * D);
    for (int i = threadIdx.x; i < D / 4; i += blockDim.x) {
        float4 a = te[i], b = pe[i];
        xo[i] = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
    }
}

// ---------------------------------------------------------------------------
// LayerNorm: one warp per row, two-pass mean / biased variance
// (CpuBackend.cs:377-398).  D <= 32 * 64.
// ---------------------------------------------------------------------------
// y_lo != null: y and y_lo receive the TF32 halves of the result (the
// operand of a tensor-core GEMM, as k_split_tf32 would make it).
template <int PER_LANE>
__global__ void k_layernorm(int rows, int D, const float* __restrict__ x, const float* __restrict__ w,
                            const float* __restrict__ b, float* __restrict__ y, const int* __restrict__ row_map,
                            float* __restrict__ y_lo) {
    int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    int lane = threadIdx.x & 31;
    // gain and bias (weights, written only when the model is created) are
    // loaded before the grid-dependency wait, so their round trip overlaps
    // the predecessor's tail instead of following the statistics
    constexpr bool kPre = PER_LANE <= 32;
    float wv[kPre ? PER_LANE : 1], bv[kPre ? PER_LANE : 1];
    if constexpr (kPre) {
#pragma unroll
        for (int i = 0; i < PER_LANE; i++) {
            const int c = lane + i * 32;
            wv[i] = c < D ? w[c] : 0.f;
            bv[i] = c < D ? b[c] : 0.f;
        }
    }
    pdl_wait();
    if (warp >= rows) return;
    int src = row_map ? row_map[warp] : warp;
    const float* xr = x + (size_t)src * D;
    float v[PER_LANE];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < PER_LANE; i++) {
        int c = lane + i * 32;
        v[i] = c < D ? xr[c] : 0.f;
        s += v[i];
    }
    s = warp_sum(s);
    float mu = s / (float)D;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < PER_LANE; i++) {
        int c = lane + i * 32;
        float d = c < D ? v[i] - mu : 0.f;
        q += d * d;
    }
    q = warp_sum(q);
    float rs = 1.0f / sqrtf(q / (float)D + kLnEps);
    float* yr = y + (size_t)warp * D;
    if (y_lo) {
        float* yl = y_lo + (size_t)warp * D;
#pragma unroll
        for (int i = 0; i < PER_LANE; i++) {
            int c = lane + i * 32;
            if (c < D) {
                const float g = kPre ? wv[kPre ? i : 0] : w[c], be = kPre ? bv[kPre ? i : 0] : b[c];
                tf32_split((v[i] - mu) * rs * g + be, yr[c], yl[c]);
            }
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < PER_LANE; i++) {
        int c = lane + i * 32;
        if (c < D) {
            const float g = kPre ? wv[kPre ? i : 0] : w[c], be = kPre ? bv[kPre ? i : 0] : b[c];
            yr[c] = (v[i] - mu) * rs * g + be;
        }
    }
}

// ---------------------------------------------------------------------------
// GEMM epilogues: y = acc + bias (Linear.Forward, Layers.cs:29-37), then
//   EPI_RESID: + residual (TransformerBlock, Layers.cs:387, 390)
//   EPI_GELU : GELU (Mlp.Forward, Layers.cs:306-313)
//   EPI_QKV  : Q to q_out, K/V appended to the cache at the row's position.
// ---------------------------------------------------------------------------
enum EpiKind { EPI_BIAS = 0, EPI_RESID = 1, EPI_GELU = 2, EPI_QKV = 3, EPI_GELU_SPLIT = 4 };

struct Epi {
    int kind;
    const float* bias;
    const float* resid;  // [M][N] for EPI_RESID
    float* out;          // [M][N] (or q [M][D] for EPI_QKV; the TF32 hi half for EPI_GELU_SPLIT)
    float* out_lo;       // [M][N] the TF32 lo half (EPI_GELU_SPLIT)
    // EPI_QKV
    float* kv_layer;     // cache + layer offset (slot 0)
    long long kv_slot_stride;
    long long v_offset;  // elements from K block to V block of one layer
    int D, hd, ctx;
    Rows R;
};

// One output element through the same epilogue as epi_store4.
FB2_DEV void epi_store1(const Epi& e, int m, int n, int N, float a) {
    a += e.bias[n];
    if (e.kind == EPI_RESID) {
        a += e.resid[(size_t)m * N + n];
    } else if (e.kind == EPI_GELU) {
        a = gelu_tanh(a);
    } else if (e.kind == EPI_GELU_SPLIT) {
        float h, l;
        tf32_split(gelu_tanh(a), h, l);
        e.out[(size_t)m * N + n] = h;
        e.out_lo[(size_t)m * N + n] = l;
        return;
    } else if (e.kind == EPI_QKV) {
        const int D = e.D;
        if (n < D) {
            e.out[(size_t)m * D + n] = a;
            return;
        }
        if (!e.R.active[m]) return;
        const int pos = e.R.pos[m];
        if (pos < 0 || pos >= e.ctx) return;
        const int which = n < 2 * D ? 0 : 1;
        const int c = n - D - which * D;
        const int h = c / e.hd, d = c - h * e.hd;
        e.kv_layer[(size_t)e.R.seq[m] * e.kv_slot_stride + (which ? e.v_offset : 0) + ((size_t)h * e.ctx + pos) * e.hd + d] = a;
        return;
    }
    e.out[(size_t)m * N + n] = a;
}

// The epilogue's operands of output quad (m, n..n+3): the bias, and the
// residual for EPI_RESID (zeros otherwise).
FB2_DEV void epi_operands4(const Epi& e, int m, int n, int N, float4& bb, float4& rr) {
    bb = *reinterpret_cast<const float4*>(e.bias + n);
    rr = e.kind == EPI_RESID ? *reinterpret_cast<const float4*>(e.resid + (size_t)m * N + n)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
}
// epi_store4 with its operands already loaded (epi_operands4).
FB2_DEV void epi_store4_with(const Epi& e, int m, int n, int N, float4 a, float4 bb, float4 r) {
    a.x += bb.x; a.y += bb.y; a.z += bb.z; a.w += bb.w;
    if (e.kind == EPI_RESID) {
        a.x += r.x; a.y += r.y; a.z += r.z; a.w += r.w;
    } else if (e.kind == EPI_GELU) {
        a.x = gelu_tanh(a.x); a.y = gelu_tanh(a.y); a.z = gelu_tanh(a.z); a.w = gelu_tanh(a.w);
    } else if (e.kind == EPI_GELU_SPLIT) {  // the next GEMM's operand, as k_split_tf32 would make it
        a.x = gelu_tanh(a.x); a.y = gelu_tanh(a.y); a.z = gelu_tanh(a.z); a.w = gelu_tanh(a.w);
        float4 h, l;
        tf32_split(a.x, h.x, l.x);
        tf32_split(a.y, h.y, l.y);
        tf32_split(a.z, h.z, l.z);
        tf32_split(a.w, h.w, l.w);
        *reinterpret_cast<float4*>(e.out + (size_t)m * N + n) = h;
        *reinterpret_cast<float4*>(e.out_lo + (size_t)m * N + n) = l;
        return;
    } else if (e.kind == EPI_QKV) {
        int D = e.D;
        if (n < D) {
            *reinterpret_cast<float4*>(e.out + (size_t)m * D + n) = a;
            return;
        }
        if (!e.R.active[m]) return;
        int pos = e.R.pos[m];
        if (pos < 0 || pos >= e.ctx) return;
        int which = n < 2 * D ? 0 : 1;
        int c = n - D - which * D;
        int h = c / e.hd, d = c - h * e.hd;
        float* base = e.kv_layer + (size_t)e.R.seq[m] * e.kv_slot_stride + (which ? e.v_offset : 0) +
                      ((size_t)h * e.ctx + pos) * e.hd + d;
        *reinterpret_cast<float4*>(base) = a;
        return;
    }
    *reinterpret_cast<float4*>(e.out + (size_t)m * N + n) = a;
}

FB2_DEV void epi_store4(const Epi& e, int m, int n, int N, float4 a) {
    float4 bb, rr;
    epi_operands4(e, m, n, N, bb, rr);
    epi_store4_with(e, m, n, N, a, bb, rr);
}

// ---------------------------------------------------------------------------
// Skinny GEMM for decode (M <= MR rows): y[M,N] = A[M,K] * W[K,N].
// W is streamed once from HBM with 16-byte non-allocating loads.  Grid:
// (N/64 column blocks, S k-splits).  256 threads = 16 column quads x 16 k
// lanes.  With S > 1 each CTA writes a partial tile to `partial` and the last
// CTA of a column block (atomic ticket) sums the S partials in split order,
// so the result is deterministic.
// ---------------------------------------------------------------------------
template <int MR, class WL = WF32>
__global__ void __launch_bounds__(256) k_gemv(int M, int K, int N, int kchunk, const float* __restrict__ A,
                                              const typename WL::T* __restrict__ W, float* __restrict__ partial,
                                              unsigned int* __restrict__ tickets, Epi e) {
    pdl_wait();
    extern __shared__ float smem[];
    float* As = smem;                     // [MR][kchunk]
    float* red = smem + MR * kchunk;      // [16][MR][64]
    const int tid = threadIdx.x;
    const int cq = tid & 15, kl = tid >> 4;
    const int col0 = blockIdx.x * 64;
    const int S = gridDim.y, sidx = blockIdx.y;
    const int k0 = sidx * kchunk;
    const int k1 = min(K, k0 + kchunk);
    const int kn = k1 - k0;
    for (int i = tid; i < MR * kchunk; i += 256) {
        int m = i / kchunk, kk = i - m * kchunk;
        As[i] = (m < M && kk < kn) ? A[(size_t)m * K + k0 + kk] : 0.f;
    }
    __syncthreads();
    float acc[MR][4];
#pragma unroll
    for (int m = 0; m < MR; m++) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0.f;
    const int col = col0 + cq * 4;
    const bool col_ok = col < N;
    const size_t w4 = ((size_t)k0 * N + col) / 4;  // this thread's first weight quad
    const size_t n4 = (size_t)N / 4;               // quads per k row
    int kk = kl;
    constexpr int U = 4;
    for (; kk + 16 * (U - 1) < kn; kk += 16 * U) {
        float4 w[U];
#pragma unroll
        for (int u = 0; u < U; u++)
            w[u] = col_ok ? WL::load4(W, w4 + (size_t)(kk + 16 * u) * n4) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int u = 0; u < U; u++) {
#pragma unroll
            for (int m = 0; m < MR; m++) {
                float a = As[m * kchunk + kk + 16 * u];
                acc[m][0] += a * w[u].x;
                acc[m][1] += a * w[u].y;
                acc[m][2] += a * w[u].z;
                acc[m][3] += a * w[u].w;
            }
        }
    }
    for (; kk < kn; kk += 16) {
        float4 w = col_ok ? WL::load4(W, w4 + (size_t)kk * n4) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int m = 0; m < MR; m++) {
            float a = As[m * kchunk + kk];
            acc[m][0] += a * w.x;
            acc[m][1] += a * w.y;
            acc[m][2] += a * w.z;
            acc[m][3] += a * w.w;
        }
    }
    // reduce the 16 k lanes
#pragma unroll
    for (int m = 0; m < MR; m++)
        *reinterpret_cast<float4*>(&red[(kl * MR + m) * 64 + cq * 4]) =
            make_float4(acc[m][0], acc[m][1], acc[m][2], acc[m][3]);
    __syncthreads();
    // 256 threads finalize MR*64 outputs (one float4 each for MR*16 threads)
    __shared__ unsigned int s_last;
    const int nout4 = MR * 16;
    float4 tot = make_float4(0.f, 0.f, 0.f, 0.f);
    int om = 0, oc = 0;
    if (tid < nout4) {
        om = tid / 16;
        oc = (tid & 15) * 4;
#pragma unroll 4
        for (int l = 0; l < 16; l++) {
            float4 v = *reinterpret_cast<float4*>(&red[(l * MR + om) * 64 + oc]);
            tot.x += v.x; tot.y += v.y; tot.z += v.z; tot.w += v.w;
        }
    }
    if (S == 1) {
        if (tid < nout4 && om < M && col0 + oc < N) epi_store4(e, om, col0 + oc, N, tot);
        return;
    }
    if (tid < nout4 && om < M && col0 + oc < N)
        *reinterpret_cast<float4*>(partial + ((size_t)sidx * M + om) * N + col0 + oc) = tot;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned int t = atomicAdd(&tickets[blockIdx.x], 1u);
        s_last = (t == (unsigned)(S - 1));
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (tid < nout4 && om < M && col0 + oc < N) {
        float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s = 0; s < S; s++) {
            float4 v = ld_cg4(reinterpret_cast<const float4*>(partial + ((size_t)s * M + om) * N + col0 + oc));
            sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
        }
        epi_store4(e, om, col0 + oc, N, sum);
    }
    if (tid == 0) tickets[blockIdx.x] = 0u;  // ready for the next launch
}

// ---------------------------------------------------------------------------
// Tiled SIMT GEMM for prefill / larger batches: y[M,N] = A[M,K] * W[K,N].
// Tile BM x 128 x 16, 256 threads, (BM/16) x 8 outputs per thread.
// Requires K % 4 == 0 and N % 4 == 0.
// ---------------------------------------------------------------------------
template <int BM>
__global__ void __launch_bounds__(256) k_gemm_tiled(int M, int K, int N, const float* __restrict__ A,
                                                    const float* __restrict__ W, Epi e) {
    pdl_wait();
    constexpr int BN = 128, BK = 16, TM = BM / 16;
    __shared__ __align__(16) float As[BK][BM + 4];
    __shared__ __align__(16) float Bs[BK][BN + 4];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    float acc[TM][8];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.f;

    constexpr int A_F4 = BM * BK / 4 / 256;  // float4 per thread for A
    for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
        for (int i = 0; i < A_F4; i++) {
            int idx = tid + i * 256;
            int row = idx / (BK / 4), kq = (idx % (BK / 4)) * 4;
            int gm = m0 + row, gk = k0 + kq;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (gm < M && gk < K) v = *reinterpret_cast<const float4*>(A + (size_t)gm * K + gk);
            As[kq + 0][row] = v.x; As[kq + 1][row] = v.y; As[kq + 2][row] = v.z; As[kq + 3][row] = v.w;
        }
#pragma unroll
        for (int i = 0; i < 2; i++) {
            int idx = tid + i * 256;
            int kr = idx / (BN / 4), nq = (idx % (BN / 4)) * 4;
            int gk = k0 + kr, gn = n0 + nq;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (gk < K && gn < N) v = *reinterpret_cast<const float4*>(W + (size_t)gk * N + gn);
            *reinterpret_cast<float4*>(&Bs[kr][nq]) = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float a[TM], b[8];
#pragma unroll
            for (int i = 0; i < TM / 4; i++) {
                float4 v = *reinterpret_cast<const float4*>(&As[kk][ty * 4 + i * 64]);
                a[i * 4 + 0] = v.x; a[i * 4 + 1] = v.y; a[i * 4 + 2] = v.z; a[i * 4 + 3] = v.w;
            }
#pragma unroll
            for (int j = 0; j < 2; j++) {
                float4 v = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4 + j * 64]);
                b[j * 4 + 0] = v.x; b[j * 4 + 1] = v.y; b[j * 4 + 2] = v.z; b[j * 4 + 3] = v.w;
            }
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] += a[i] * b[j];
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < TM; i++) {
        int gm = m0 + ty * 4 + (i / 4) * 64 + (i % 4);
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < 2; j++) {
            int gn = n0 + tx * 4 + j * 64;
            if (gn >= N) continue;
            epi_store4(e, gm, gn, N, make_float4(acc[i][j * 4], acc[i][j * 4 + 1], acc[i][j * 4 + 2], acc[i][j * 4 + 3]));
        }
    }
}

// ---------------------------------------------------------------------------
// Decode attention over the KV cache (MultiHeadAttention.Forward,
// Layers.cs:191-229, for the last row only): split-KV partials + combine.
// Scores are (q . k) * (1/sqrt(hd)) (Layers.cs:174; ITensorBackend.cs:117-122).
// ---------------------------------------------------------------------------
constexpr int kAttnChunk = 64;

template <int HD>
__global__ void __launch_bounds__(128) k_attn_decode_partial(const float* __restrict__ q, const float* __restrict__ kv_layer,
                                                             long long kv_slot_stride, long long v_offset, int H, int ctx,
                                                             float scale, Rows R, float* __restrict__ part, int nsplit) {
    pdl_wait();
    constexpr int LPK = HD / 4;        // lanes per key
    constexpr int KPW = 32 / LPK;      // keys per warp iteration
    const int r = blockIdx.x, h = blockIdx.y, sp = blockIdx.z;
    if (!R.active[r]) return;
    const int T = R.pos[r] + 1;
    const int k0 = sp * kAttnChunk;
    if (k0 >= T) return;
    const int k1 = min(T, k0 + kAttnChunk);
    const int D = H * HD;
    __shared__ float sc[kAttnChunk];
    __shared__ float red[4][HD];
    __shared__ float wmax[4], wsum[4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane % LPK, grp = lane / LPK;
    const float4 qv = *reinterpret_cast<const float4*>(q + (size_t)r * D + h * HD + sub * 4);
    const float* Kb = kv_layer + (size_t)R.seq[r] * kv_slot_stride + (size_t)h * ctx * HD;
    const float* Vb = Kb + v_offset;
    // this lane group's keys j = k0 + (4i + warp) KPW + grp: every K and V
    // load of the chunk is issued before the first is used (one round trip)
    constexpr int ROUNDS = (kAttnChunk + 4 * KPW - 1) / (4 * KPW);
    float4 kk[ROUNDS], vv[ROUNDS];
#pragma unroll
    for (int i = 0; i < ROUNDS; i++) {
        const int j = k0 + (4 * i + warp) * KPW + grp;
        const bool in = j < k1;
        kk[i] = in ? ld_cg4(reinterpret_cast<const float4*>(Kb + (size_t)j * HD + sub * 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
        vv[i] = in ? ld_cg4(reinterpret_cast<const float4*>(Vb + (size_t)j * HD + sub * 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    // scores
#pragma unroll
    for (int i = 0; i < ROUNDS; i++) {
        const int j = k0 + (4 * i + warp) * KPW + grp;
        float d = qv.x * kk[i].x + qv.y * kk[i].y + qv.z * kk[i].z + qv.w * kk[i].w;
#pragma unroll
        for (int o = LPK / 2; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (j < k1 && sub == 0) sc[j - k0] = d * scale;
    }
    __syncthreads();
    const int n = k1 - k0;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += 128) m = fmaxf(m, sc[i]);
    m = warp_max(m);
    if (lane == 0) wmax[warp] = m;
    __syncthreads();
    m = fmaxf(fmaxf(wmax[0], wmax[1]), fmaxf(wmax[2], wmax[3]));
    float l = 0.f;
    for (int i = threadIdx.x; i < n; i += 128) {
        float p = __expf(sc[i] - m);
        sc[i] = p;
        l += p;
    }
    l = warp_sum(l);
    if (lane == 0) wsum[warp] = l;
    __syncthreads();
    // P.V: lane group accumulates its keys over 4 dims
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int i = 0; i < ROUNDS; i++) {
        const int j = k0 + (4 * i + warp) * KPW + grp;
        if (j >= k1) break;
        const float p = sc[j - k0];
        acc.x += p * vv[i].x; acc.y += p * vv[i].y; acc.z += p * vv[i].z; acc.w += p * vv[i].w;
    }
#pragma unroll
    for (int o = LPK; o < 32; o <<= 1) {
        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
        acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
        acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
    }
    if (grp == 0) *reinterpret_cast<float4*>(&red[warp][sub * 4]) = acc;
    __syncthreads();
    float* out = part + (((size_t)r * H + h) * nsplit + sp) * (HD + 2);
    for (int d = threadIdx.x; d < HD; d += 128) out[2 + d] = red[0][d] + red[1][d] + red[2][d] + red[3][d];
    if (threadIdx.x == 0) {
        out[0] = m;
        out[1] = wsum[0] + wsum[1] + wsum[2] + wsum[3];
    }
}

template <int HD>
__global__ void k_attn_decode_combine(const float* __restrict__ part, int H, int nsplit, Rows R,
                                      float* __restrict__ ctx_out) {
    pdl_wait();
    const int r = blockIdx.x, h = blockIdx.y;
    const int D = H * HD;
    float* o = ctx_out + (size_t)r * D + h * HD;
    if (!R.active[r]) {
        for (int d = threadIdx.x; d < HD; d += blockDim.x) o[d] = 0.f;
        return;
    }
    const int T = R.pos[r] + 1;
    const int ns = (T + kAttnChunk - 1) / kAttnChunk;
    const float* p = part + ((size_t)r * H + h) * nsplit * (HD + 2);
    // loads eight chunks at a time ahead of their use; sums in chunk order
    float M = -INFINITY;
    for (int s0 = 0; s0 < ns; s0 += 8) {
        float mv[8];
#pragma unroll
        for (int j = 0; j < 8; j++) mv[j] = s0 + j < ns ? p[(s0 + j) * (HD + 2)] : -INFINITY;
#pragma unroll
        for (int j = 0; j < 8; j++) M = fmaxf(M, mv[j]);
    }
    float L = 0.f;
    for (int s0 = 0; s0 < ns; s0 += 8) {
        float mv[8], lv[8];
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (s0 + j < ns) {
                mv[j] = p[(s0 + j) * (HD + 2)];
                lv[j] = p[(s0 + j) * (HD + 2) + 1];
            }
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (s0 + j < ns) L += lv[j] * __expf(mv[j] - M);
    }
    float inv = 1.0f / L;
    for (int d = threadIdx.x; d < HD; d += blockDim.x) {
        float a = 0.f;
        for (int s0 = 0; s0 < ns; s0 += 8) {
            float mv[8], xv[8];
#pragma unroll
            for (int j = 0; j < 8; j++)
                if (s0 + j < ns) {
                    mv[j] = p[(s0 + j) * (HD + 2)];
                    xv[j] = p[(s0 + j) * (HD + 2) + 2 + d];
                }
#pragma unroll
            for (int j = 0; j < 8; j++)
                if (s0 + j < ns) a += xv[j] * __expf(mv[j] - M);
        }
        o[d] = a * inv;
    }
}

// ---------------------------------------------------------------------------
// Prefill attention: causal, flash-style online softmax, fp32 SIMT.
// One CTA = one query block (<= 64 consecutive positions of one sequence)
// x one head.  256 threads: 4 per query row, each owning HD/4 output dims.
// qblk[b] = {first row, count, seq, first position}.
// ---------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(256) k_attn_prefill(const float* __restrict__ q, const float* __restrict__ kv_layer,
                                                      long long kv_slot_stride, long long v_offset, int H, int ctx,
                                                      float scale, const int4* __restrict__ qblk,
                                                      float* __restrict__ ctx_out) {
    pdl_wait();
    constexpr int BQ = 64, BK = 64, DPT = (HD + 3) / 4;  // dims per thread
    extern __shared__ float sm[];
    float* Qs = sm;                          // [BQ][HD+1]
    float* Ks = Qs + BQ * (HD + 1);          // [BK][HD+1]
    float* Vs = Ks + BK * (HD + 1);          // [BK][HD]
    float* Ps = Vs + BK * HD;                // [BQ][BK+1]
    const int4 blk = qblk[blockIdx.x];
    const int h = blockIdx.y;
    const int row0 = blk.x, nq = blk.y, seq = blk.z, p0 = blk.w;
    const int D = H * HD;
    const int tid = threadIdx.x, qi = tid >> 2, sub = tid & 3;
    for (int i = tid; i < BQ * HD; i += 256) {
        int rr = i / HD, d = i - rr * HD;
        Qs[rr * (HD + 1) + d] = rr < nq ? q[(size_t)(row0 + rr) * D + h * HD + d] : 0.f;
    }
    const float* Kb = kv_layer + (size_t)seq * kv_slot_stride + (size_t)h * ctx * HD;
    const float* Vb = Kb + v_offset;
    float o[DPT];
#pragma unroll
    for (int i = 0; i < DPT; i++) o[i] = 0.f;
    float m = -INFINITY, l = 0.f;
    const int myp = p0 + qi;  // position of this query row
    const int last_key = p0 + nq - 1;
    for (int kt = 0; kt <= last_key; kt += BK) {
        __syncthreads();
        for (int i = tid; i < BK * HD; i += 256) {
            int j = i / HD, d = i - j * HD;
            bool ok = kt + j <= last_key;
            Ks[j * (HD + 1) + d] = ok ? Kb[(size_t)(kt + j) * HD + d] : 0.f;
            Vs[j * HD + d] = ok ? Vb[(size_t)(kt + j) * HD + d] : 0.f;
        }
        __syncthreads();
        float s[BK / 4];
        float tmax = -INFINITY;
#pragma unroll
        for (int jj = 0; jj < BK / 4; jj++) {
            int j = sub + 4 * jj;
            float d = 0.f;
#pragma unroll 8
            for (int dd = 0; dd < HD; dd++) d += Qs[qi * (HD + 1) + dd] * Ks[j * (HD + 1) + dd];
            d *= scale;
            if (kt + j > myp || qi >= nq) d = -INFINITY;  // causal mask (CpuBackend.cs:547-553)
            s[jj] = d;
            tmax = fmaxf(tmax, d);
        }
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 1));
        tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
        float mnew = fmaxf(m, tmax);
        float corr = (mnew == -INFINITY) ? 1.f : __expf(m - mnew);
        float psum = 0.f;
#pragma unroll
        for (int jj = 0; jj < BK / 4; jj++) {
            float p = (s[jj] == -INFINITY) ? 0.f : __expf(s[jj] - mnew);
            Ps[qi * (BK + 1) + sub + 4 * jj] = p;
            psum += p;
        }
        psum += __shfl_xor_sync(0xffffffffu, psum, 1);
        psum += __shfl_xor_sync(0xffffffffu, psum, 2);
        l = l * corr + psum;
        m = mnew;
        __syncwarp();
#pragma unroll
        for (int i = 0; i < DPT; i++) o[i] *= corr;
        for (int j = 0; j < BK; j++) {
            float p = Ps[qi * (BK + 1) + j];
#pragma unroll
            for (int i = 0; i < DPT; i++) {
                int d = sub * DPT + i;
                if (d < HD) o[i] += p * Vs[j * HD + d];
            }
        }
    }
    if (qi < nq) {
        float inv = 1.0f / l;
        float* out = ctx_out + (size_t)(row0 + qi) * D + h * HD;
#pragma unroll
        for (int i = 0; i < DPT; i++) {
            int d = sub * DPT + i;
            if (d < HD) out[d] = o[i] * inv;
        }
    }
}

// ---------------------------------------------------------------------------
// Prefill attention, register-tiled (HD in {32, 64, 128}): the same causal
// flash-style online softmax as k_attn_prefill, with thread (tq, tk) of the
// 16 x 16 grid computing scores of queries 4tq..4tq+3 against keys tk + 16j
// (float4 loads along the head dimension), and then the 4 queries' context
// for dims tk*HD/16 .. +HD/16.  qblk[b] = {first row, count, seq, first
// position}; one CTA per (query block of <= 64 rows, head).
// ---------------------------------------------------------------------------
template <int HD>
__global__ void __launch_bounds__(256) k_attn_prefill_rt(const float* __restrict__ q, const float* __restrict__ kv_layer,
                                                         long long kv_slot_stride, long long v_offset, int H, int ctx,
                                                         float scale, const int4* __restrict__ qblk,
                                                         float* __restrict__ ctx_out) {
    pdl_wait();
    constexpr int BQ = 64, BK = 64, LD = HD + 4, LP = BK + 4, DPT = HD / 16;
    static_assert(HD % 16 == 0 && HD <= 128, "head dim");
    extern __shared__ __align__(16) float sm[];
    float* Qs = sm;               // [BQ][LD]
    float* Ks = Qs + BQ * LD;     // [BK][LD]
    float* Vs = Ks + BK * LD;     // [BK][HD]
    float* Ps = Vs + BK * HD;     // [BQ][LP]
    const int4 blk = qblk[blockIdx.x];
    const int h = blockIdx.y;
    const int row0 = blk.x, nq = blk.y, seq = blk.z, p0 = blk.w;
    const int D = H * HD;
    const int tid = threadIdx.x, tq = tid >> 4, tk = tid & 15;
    for (int i = tid; i < BQ * (HD / 4); i += 256) {
        const int r = i / (HD / 4), d4 = i - r * (HD / 4);
        const float4 v = r < nq ? *reinterpret_cast<const float4*>(q + (size_t)(row0 + r) * D + h * HD + 4 * d4)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(Qs + r * LD + 4 * d4) = v;
    }
    const float* Kb = kv_layer + (size_t)seq * kv_slot_stride + (size_t)h * ctx * HD;
    const float* Vb = Kb + v_offset;
    float o[4][DPT];
    float m[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int e = 0; e < DPT; e++) o[i][e] = 0.f;
    }
    const int last_key = p0 + nq - 1;
    for (int kt = 0; kt <= last_key; kt += BK) {
        __syncthreads();
        for (int i = tid; i < BK * (HD / 4); i += 256) {
            const int j = i / (HD / 4), d4 = i - j * (HD / 4);
            const bool ok = kt + j <= last_key;
            const float4 kk = ok ? *reinterpret_cast<const float4*>(Kb + (size_t)(kt + j) * HD + 4 * d4)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 vv = ok ? *reinterpret_cast<const float4*>(Vb + (size_t)(kt + j) * HD + 4 * d4)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4*>(Ks + j * LD + 4 * d4) = kk;
            *reinterpret_cast<float4*>(Vs + j * HD + 4 * d4) = vv;
        }
        __syncthreads();
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) sc[i][j] = 0.f;
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            float4 qa[4], ka[4];
#pragma unroll
            for (int i = 0; i < 4; i++) qa[i] = *reinterpret_cast<const float4*>(Qs + (4 * tq + i) * LD + d);
#pragma unroll
            for (int j = 0; j < 4; j++) ka[j] = *reinterpret_cast<const float4*>(Ks + (tk + 16 * j) * LD + d);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    sc[i][j] += qa[i].x * ka[j].x + qa[i].y * ka[j].y + qa[i].z * ka[j].z + qa[i].w * ka[j].w;
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int qr = 4 * tq + i, qpos = p0 + qr;
            float tmax = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float d = sc[i][j] * scale;
                if (kt + tk + 16 * j > qpos || qr >= nq) d = -INFINITY;  // causal mask (CpuBackend.cs:547-553)
                sc[i][j] = d;
                tmax = fmaxf(tmax, d);
            }
#pragma unroll
            for (int o2 = 1; o2 < 16; o2 <<= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o2));
            const float mnew = fmaxf(m[i], tmax);
            const float corr = (mnew == -INFINITY) ? 1.f : __expf(m[i] - mnew);
            float psum = 0.f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float pv = (sc[i][j] == -INFINITY) ? 0.f : __expf(sc[i][j] - mnew);
                Ps[qr * LP + tk + 16 * j] = pv;
                psum += pv;
            }
#pragma unroll
            for (int o2 = 1; o2 < 16; o2 <<= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o2);
            l[i] = l[i] * corr + psum;
            m[i] = mnew;
#pragma unroll
            for (int e = 0; e < DPT; e++) o[i][e] *= corr;
        }
        __syncthreads();
#pragma unroll 4
        for (int j = 0; j < BK; j++) {
            float pv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) pv[i] = Ps[(4 * tq + i) * LP + j];
            float vv[DPT];
#pragma unroll
            for (int e = 0; e < DPT; e += 4) {
                const float4 v4 = *reinterpret_cast<const float4*>(Vs + j * HD + tk * DPT + e);
                vv[e] = v4.x;
                if (e + 1 < DPT) vv[e + 1] = v4.y;
                if (e + 2 < DPT) vv[e + 2] = v4.z;
                if (e + 3 < DPT) vv[e + 3] = v4.w;
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int e = 0; e < DPT; e++) o[i][e] += pv[i] * vv[e];
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int qr = 4 * tq + i;
        if (qr >= nq) continue;
        const float inv = 1.0f / l[i];
        float* out = ctx_out + (size_t)(row0 + qr) * D + h * HD + tk * DPT;
#pragma unroll
        for (int e = 0; e < DPT; e++) out[e] = o[i][e] * inv;
    }
}

// ---------------------------------------------------------------------------
// LM head on selected rows (TiedOutputProjection.Forward, Layers.cs:80-86,
// last row only): logits[m][v] = dot(xln[m], tok_emb[v]).  One warp per
// vocab row, MR rows at a time, xln staged in shared memory.
// ---------------------------------------------------------------------------
template <int MR, class WL = WF32>
__global__ void __launch_bounds__(256) k_head(int M, int D, int V, const float* __restrict__ xln,
                                              const typename WL::T* __restrict__ E, float* __restrict__ logits,
                                              int logits_stride) {
    pdl_wait();
    extern __shared__ float xs[];  // [MR][D]
    for (int i = threadIdx.x; i < MR * D; i += blockDim.x) {
        int m = i / D;
        xs[i] = m < M ? xln[i] : 0.f;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    for (int v = blockIdx.x * warps + (threadIdx.x >> 5); v < V; v += gridDim.x * warps) {
        const size_t e4 = (size_t)v * D / 4;
        float acc[MR];
#pragma unroll
        for (int m = 0; m < MR; m++) acc[m] = 0.f;
        for (int i = lane; i < D / 4; i += 32) {
            float4 w = WL::load4(E, e4 + i);
#pragma unroll
            for (int m = 0; m < MR; m++) {
                float4 x = *reinterpret_cast<const float4*>(&xs[m * D + i * 4]);
                acc[m] += x.x * w.x + x.y * w.y + x.z * w.z + x.w * w.w;
            }
        }
#pragma unroll
        for (int m = 0; m < MR; m++) {
            float a = warp_sum(acc[m]);
            if (lane == 0 && m < M) logits[(size_t)m * logits_stride + v] = a;
        }
    }
}

}  // namespace fb2
