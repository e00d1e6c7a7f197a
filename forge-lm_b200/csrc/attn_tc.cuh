// attn_tc.cuh — causal prefill attention on the tensor cores (sm_100a),
// head_dim 64.
//
// The same computation as k_attn_prefill_rt (softmax(q k^T * scale, causal)
// v per head, CpuBackend.cs:540-575: scale, mask, softmax, weighted sum),
// with both products on the 5th-generation tensor cores in TF32 and the
// 3xTF32 compensation of gemm_tc.cuh (x = hi + lo, hi*hi + hi*lo + lo*hi).
//
// One CTA of 256 threads per (query block of <= 128 rows, head).  Query row
// r is TMEM lane r; warps w and w + 4 both read lane quarter w % 4, warp w
// taking columns 0..31 and warp w + 4 columns 32..63 of the S and O tiles,
// and combine a row's max and sum through shared memory.
// K and V tiles (64 keys) are split into TF32 halves and written as K-major,
// 128-byte swizzled operands, K [64 keys][64 dims] and V^T [64 dims][64
// keys], from registers loaded one tile ahead.  Thread 0 issues the MMAs
// (M128 N64, 8 k-steps x 3) and commits them to mbarriers.  The two products
// are software-pipelined against the threads' work; iteration t:
//   1. wait for S(t) = Q K(t)^T (TMEM columns 64 (t % 2) ..);
//   2. write K(t+1) (its buffer is free) and issue S(t+1), which runs on the
//      tensor cores during the rest of the iteration;
//   3. load the half score row (tcgen05.ld), apply scale and the causal mask,
//      update the row's running max m and sum l (online softmax); wait for
//      O(t-1) = P(t-1) V(t-1) (TMEM columns 128..191) and fold it into the
//      registers, o = o * alpha(t-1) + O(t-1); write p = exp(s - m) as P's
//      TF32 halves;
//   4. write V(t) and issue O(t), which runs during the next iteration's
//      steps 1-2.
// The last O is folded after the loop.
// Rows past the block and keys past the last query are zero operands (the
// cache beyond them may hold anything); masked scores are -inf.
// Every mbarrier wait is bounded (kTcTimeoutNs); on expiry the CTA records
// TC_ERR_TIMEOUT, drains its MMAs (bounded), frees TMEM and returns.
#pragma once
#include "gemm_tc.cuh"

namespace fb2 {

constexpr int ATC_THREADS = 256;
constexpr int ATC_BQ = 128, ATC_BK = 64, ATC_HD = 64;
constexpr int ATC_QB = ATC_BQ * ATC_HD * 4;   // one TF32 half of Q (or P): 32 KB
constexpr int ATC_KB = ATC_BK * ATC_HD * 4;   // one TF32 half of K (or V^T): 16 KB
constexpr int ATC_SMEM = 4 * ATC_QB + 4 * ATC_KB + 1024;  // Q, P, K, V^T halves + alignment slack
constexpr uint32_t ATC_TMEM_COLS = 256;       // S: columns 0..63 and 64..127 (double), O tile: 128..191

namespace atc {
// Byte offset of fp32 element (row, col) in a K-major operand of `rows` rows
// and 64 columns, stored as two 128-byte-wide blocks (columns 0..31, 32..63),
// each rows x 128 B with the 128-byte swizzle (16-byte chunk c of row r at
// c ^ (r % 8)) that the tensor cores' SWIZZLE_128B descriptor reads.
FB2_DEV uint32_t swz(int row, int col, int rows) {
    const int blk = col >> 5, c = col & 31;
    return (uint32_t)(blk * rows * 128 + row * 128 + ((((c >> 2) ^ (row & 7)) << 4) | ((c & 3) << 2)));
}
// Descriptor of k-step kk (8 TF32 columns) of such an operand at `base`.
FB2_DEV uint64_t kdesc(uint32_t base, int kk, int rows) {
    return tc::sw128_desc(base + (uint32_t)((kk >> 2) * rows * 128 + (kk & 3) * 32), 16, 1024);
}
FB2_DEV void st_shared_v4(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}
FB2_DEV void st_shared_f32(uint32_t addr, float v) { asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory"); }
// x = hi + lo with hi, lo TF32 (tf32_split_rn of gemm_tc.cuh).
FB2_DEV void split4(float4 v, float4& hi, float4& lo) {
    tf32_split_rn(v.x, hi.x, lo.x);
    tf32_split_rn(v.y, hi.y, lo.y);
    tf32_split_rn(v.z, hi.z, lo.z);
    tf32_split_rn(v.w, hi.w, lo.w);
}
// Shared memory written by the threads -> visible to the tensor cores.
FB2_DEV void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 3 x 8 MMAs of one M128 N64 K64 product (A, B: K-major TF32 halves).
FB2_DEV void mma_3x(uint32_t d, uint32_t a_hi, uint32_t a_lo, int a_rows, uint32_t b_hi, uint32_t b_lo, int b_rows) {
    constexpr uint32_t idesc = tc::idesc_tf32(ATC_BQ, 64);
#pragma unroll
    for (int kk = 0; kk < ATC_HD / 8; kk++) {
        const uint64_t ah = kdesc(a_hi, kk, a_rows), al = kdesc(a_lo, kk, a_rows);
        const uint64_t bh = kdesc(b_hi, kk, b_rows), bl = kdesc(b_lo, kk, b_rows);
        tc::mma_tf32(d, ah, bh, idesc, kk != 0);
        tc::mma_tf32(d, ah, bl, idesc, 1u);
        tc::mma_tf32(d, al, bh, idesc, 1u);
    }
}
}  // namespace atc

// qblk[b] = {first row, count (<= 128), sequence slot, first position}; the
// block's rows are that sequence's consecutive positions.  ctx_lo != null:
// ctx_out and ctx_lo receive the TF32 halves of the result (the operand of
// the next tensor-core GEMM, as k_split_tf32 would make it).
__global__ void __launch_bounds__(ATC_THREADS, 1)
    k_attn_prefill_tc(const float* __restrict__ q, const float* __restrict__ kv_layer, long long kv_slot_stride,
                      long long v_offset, int H, int ctx, float scale, const int4* __restrict__ qblk,
                      float* __restrict__ ctx_out, int* err, float* __restrict__ ctx_lo) {
    extern __shared__ unsigned char atc_smem_raw[];
    __shared__ __align__(8) uint64_t bar_s, bar_o, drain;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int s_abort;
    __shared__ float s_red[2][2][ATC_BQ];  // [max | sum][column half][row]
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(atc_smem_raw) + 1023) & ~(uintptr_t)1023);
    const uint32_t Qh = tc::smem_addr(sm), Ql = Qh + ATC_QB, Ph = Ql + ATC_QB, Pl = Ph + ATC_QB;
    const uint32_t Kh = Pl + ATC_QB, Kl = Kh + ATC_KB, Vh = Kl + ATC_KB, Vl = Vh + ATC_KB;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int quarter = warp & 3, half = warp >> 2;

    if (tid == 0) {
        s_abort = 0;
        tc::bar_init(&bar_s, 1);
        tc::bar_init(&bar_o, 1);
        tc::bar_init(&drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_addr(&tmem_base)),
                     "r"(ATC_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = tmem_base;
    // this warp's lane quarter and column half of a 64-column TMEM tile
    const uint32_t t_mine = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(32 * half);
    constexpr uint32_t kO = 128;  // TMEM column of the O tile
    pdl_wait();  // barriers and tensor memory set up; global memory from here on

    const int4 blk = qblk[blockIdx.x];
    const int h = blockIdx.y;
    const int row0 = blk.x, nq = blk.y, seq = blk.z, p0 = blk.w;
    const int D = H * ATC_HD;
    // Q block -> TF32 halves (16 threads per row: coalesced loads)
    for (int i = tid; i < ATC_BQ * 16; i += ATC_THREADS) {
        const int r = i >> 4, c4 = i & 15;
        const float4 v = r < nq ? __ldg(reinterpret_cast<const float4*>(q + (size_t)(row0 + r) * D + h * ATC_HD) + c4)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
        float4 hi, lo;
        atc::split4(v, hi, lo);
        const uint32_t o = atc::swz(r, 4 * c4, ATC_BQ);
        atc::st_shared_v4(Qh + o, hi);
        atc::st_shared_v4(Ql + o, lo);
    }
    const float* Kb = kv_layer + (size_t)seq * kv_slot_stride + (size_t)h * ctx * ATC_HD;
    const float* Vb = Kb + v_offset;
    const int last_key = p0 + nq - 1, ntiles = last_key / ATC_BK + 1;
    // K as 4 float4 per thread (16 threads per key row); V as 4 float4 per
    // thread, a warp's lanes on 32 consecutive keys and 16 dims (the
    // transposed stores are then conflict-free)
    const int vkey = 32 * (warp & 1) + lane, vd0 = 16 * (warp >> 1);
    float4 kr[4], vr[4];
    auto load_k = [&](int kt) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = tid + ATC_THREADS * j, key = kt + (i >> 4), c4 = i & 15;
            kr[j] = key <= last_key ? __ldcg(reinterpret_cast<const float4*>(Kb + (size_t)key * ATC_HD) + c4)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto load_v = [&](int kt) {
        const int vk = kt + vkey;
#pragma unroll
        for (int j = 0; j < 4; j++)
            vr[j] = vk <= last_key ? __ldcg(reinterpret_cast<const float4*>(Vb + (size_t)vk * ATC_HD + vd0) + j)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    auto store_k = [&]() {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int i = tid + ATC_THREADS * j, key = i >> 4, c4 = i & 15;
            float4 hi, lo;
            atc::split4(kr[j], hi, lo);
            const uint32_t ko = atc::swz(key, 4 * c4, ATC_BK);
            atc::st_shared_v4(Kh + ko, hi);
            atc::st_shared_v4(Kl + ko, lo);
        }
    };
    auto store_v = [&]() {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float4 vh, vl;
            atc::split4(vr[j], vh, vl);
            const int d = vd0 + 4 * j;
            atc::st_shared_f32(Vh + atc::swz(d, vkey, ATC_HD), vh.x);
            atc::st_shared_f32(Vl + atc::swz(d, vkey, ATC_HD), vl.x);
            atc::st_shared_f32(Vh + atc::swz(d + 1, vkey, ATC_HD), vh.y);
            atc::st_shared_f32(Vl + atc::swz(d + 1, vkey, ATC_HD), vl.y);
            atc::st_shared_f32(Vh + atc::swz(d + 2, vkey, ATC_HD), vh.z);
            atc::st_shared_f32(Vl + atc::swz(d + 2, vkey, ATC_HD), vl.z);
            atc::st_shared_f32(Vh + atc::swz(d + 3, vkey, ATC_HD), vh.w);
            atc::st_shared_f32(Vl + atc::swz(d + 3, vkey, ATC_HD), vl.w);
        }
    };
    // shared-memory operands written by the threads -> one thread issues
    auto publish = [&]() {
        atc::fence_async_shared();
        tc::fence_before();
        __syncthreads();
    };
    auto issue_s = [&](int t) {
        if (tid == 0) {
            tc::fence_after();
            atc::mma_3x(tmem + 64u * (uint32_t)(t & 1), Qh, Ql, ATC_BQ, Kh, Kl, ATC_BK);
            tc::mma_commit(&bar_s);
        }
    };

    // prologue: S(0) in flight, K(1) and V(0) in registers
    load_k(0);
    load_v(0);
    store_k();
    publish();
    issue_s(0);
    if (ntiles > 1) load_k(ATC_BK);

    const int r = 32 * quarter + lane, qpos = p0 + r;
    float o[32];
#pragma unroll
    for (int d = 0; d < 32; d++) o[d] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 1.f;
    auto fold_o = [&](float a) {
#pragma unroll
        for (int c = 0; c < 2; c++) {
            float ot[16];
            tc::tmem_ld16(t_mine + kO + 16 * c, ot);
#pragma unroll
            for (int i = 0; i < 16; i++) o[16 * c + i] = o[16 * c + i] * a + ot[i];
        }
    };
    bool ok = true;
    for (int t = 0; t < ntiles; t++) {
        const int kt = t * ATC_BK;
        // 1. S(t) complete: the K buffer is free
        ok = tc::bar_wait(&bar_s, (uint32_t)(t & 1), &s_abort);
        if (!__syncthreads_and(ok)) break;
        tc::fence_after();
        // 2. K(t+1) and S(t+1)
        if (t + 1 < ntiles) {
            store_k();
            publish();
            issue_s(t + 1);
            if (t + 2 < ntiles) load_k(kt + 2 * ATC_BK);
        }
        // 3. softmax of this tile's half row
        float s[32];
        tc::tmem_ld16(t_mine + 64u * (uint32_t)(t & 1), s);
        tc::tmem_ld16(t_mine + 64u * (uint32_t)(t & 1) + 16, s + 16);
        const int k0 = kt + 32 * half;
        float tmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const float v = k0 + j > qpos ? -INFINITY : s[j] * scale;
            s[j] = v;
            tmax = fmaxf(tmax, v);
        }
        s_red[0][half][r] = tmax;
        if (t > 0) {  // O(t-1) complete: P, V and the O tile are free
            ok = tc::bar_wait(&bar_o, (uint32_t)((t - 1) & 1), &s_abort);
        }
        if (!__syncthreads_and(ok)) break;
        tc::fence_after();
        if (t > 0) fold_o(alpha_prev);
        const float mnew = fmaxf(m, fmaxf(s_red[0][0][r], s_red[0][1][r]));
        const float alpha = mnew == -INFINITY ? 1.f : __expf(m - mnew);
        float psum = 0.f;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const float p = s[j] == -INFINITY ? 0.f : __expf(s[j] - mnew);
            s[j] = p;
            psum += p;
        }
        s_red[1][half][r] = psum;
        m = mnew;
#pragma unroll
        for (int c4 = 0; c4 < 8; c4++) {
            float4 hi, lo;
            atc::split4(make_float4(s[4 * c4], s[4 * c4 + 1], s[4 * c4 + 2], s[4 * c4 + 3]), hi, lo);
            const uint32_t po = atc::swz(r, 32 * half + 4 * c4, ATC_BQ);
            atc::st_shared_v4(Ph + po, hi);
            atc::st_shared_v4(Pl + po, lo);
        }
        // 4. V(t) and O(t) = P(t) V(t)
        store_v();
        publish();
        l = l * alpha + (s_red[1][0][r] + s_red[1][1][r]);
        alpha_prev = alpha;
        if (tid == 0) {
            tc::fence_after();
            atc::mma_3x(tmem + kO, Ph, Pl, ATC_BQ, Vh, Vl, ATC_HD);
            tc::mma_commit(&bar_o);
        }
        if (t + 1 < ntiles) load_v(kt + ATC_BK);
    }
    if (!s_abort && ok) {  // the last O tile
        ok = tc::bar_wait(&bar_o, (uint32_t)((ntiles - 1) & 1), &s_abort);
        if (__syncthreads_and(ok)) {
            tc::fence_after();
            fold_o(alpha_prev);
        }
    }
    if (!s_abort && r < nq) {
        const float inv = 1.0f / l;
        const size_t at = (size_t)(row0 + r) * D + h * ATC_HD + 32 * half;
        float4* out = reinterpret_cast<float4*>(ctx_out + at);
#pragma unroll
        for (int d4 = 0; d4 < 8; d4++) {
            const float4 v = make_float4(o[4 * d4] * inv, o[4 * d4 + 1] * inv, o[4 * d4 + 2] * inv, o[4 * d4 + 3] * inv);
            if (ctx_lo) {
                float4 hi, lo;
                tf32_split(v.x, hi.x, lo.x);
                tf32_split(v.y, hi.y, lo.y);
                tf32_split(v.z, hi.z, lo.z);
                tf32_split(v.w, hi.w, lo.w);
                out[d4] = hi;
                reinterpret_cast<float4*>(ctx_lo + at)[d4] = lo;
            } else {
                out[d4] = v;
            }
        }
    }
    if (s_abort && tid == 0) {
        atomicExch(err, TC_ERR_TIMEOUT);
        // every MMA issued completes before tensor memory is freed
        tc::mma_commit(&drain);
        const unsigned long long t0 = tc::now_ns();
        while (!tc::bar_try(&drain, 0) && tc::now_ns() - t0 < kTcTimeoutNs) {
        }
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ATC_TMEM_COLS) : "memory");
    }
}

}  // namespace fb2
