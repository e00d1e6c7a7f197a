// Tensor-core GEMM for the prefill / batched projections (sm_100a).
//
// y[M,N] = A[M,K] * W[K,N] (+ the Epi epilogue of kernels.cuh), fp32 in and
// out, computed on the 5th-generation tensor cores in TF32 with the 3xTF32
// error compensation: every fp32 operand x is carried as hi = x rounded to
// the nearest TF32 value and lo = x - hi, itself rounded to TF32 (both exact
// for the tensor cores, which read the top 19 bits), and
//   A*W ~= A_hi*W_hi + A_hi*W_lo + A_lo*W_hi
// accumulates in fp32 in tensor memory (each operand is carried to ~2^-22
// relative, unbiased; the dropped lo*lo term is ~2^-22), which keeps the
// result within the fp32 parity tolerance of the reference's
// CpuBackend.MatMulNN (CpuBackend.cs:118-164).
//
// The weight halves are stored transposed, W^T [N][K], so both operands are
// K-major tiles (rows of 32 fp32 = 128 bytes, 128-byte swizzled).
//
// One CTA computes a 128 x 128 output tile:
//   warp 0 / lane 0  TMA producer: per 32-deep k block, A_hi and A_lo tiles
//                    (128 rows of A) and W_hi, W_lo tiles (128 rows of W^T)
//                    into a 3-stage ring guarded by full/empty mbarriers;
//   warp 1 / lane 0  MMA issuer: 4 k-steps x 3 tcgen05.mma (M128 N128 K8)
//                    per stage into one TMEM accumulator, tcgen05.commit
//                    frees the stage; a final commit signals the epilogue;
//   warps 0-3        epilogue: tcgen05.ld of the thread's accumulator row
//                    (TMEM lane = row), 16 columns at a time, into epi_store4.
// Every mbarrier wait is bounded (kTcTimeoutNs); on expiry the CTA records
// an error, stops issuing, waits (bounded) for work in flight, frees its TMEM
// and returns.
#pragma once
#include <cuda.h>
#include <stdint.h>

#include "common.cuh"
#include "kernels.cuh"

namespace fb2 {

constexpr int TC_BM = 128, TC_BK = 32;
constexpr int TC_TILE_A = TC_BM * TC_BK * 4;  // 16 KB: 128 rows x 32 fp32

// Tile shape and ring of the prefill GEMM.
template <int BN>
struct TcCfg {
    static constexpr int TILE_B = BN * TC_BK * 4;
    static constexpr int STAGE = 2 * TC_TILE_A + 2 * TILE_B;
    static constexpr int STAGES = (200 * 1024) / STAGE > 8 ? 8 : (200 * 1024) / STAGE;
    static constexpr int SMEM = STAGES * STAGE + 1024;  // + alignment slack
    static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
};
constexpr unsigned long long kTcTimeoutNs = 2000000000ull;
constexpr int TC_ERR_TIMEOUT = 1;

struct TcMaps {
    CUtensorMap a_hi, a_lo, b_hi, b_lo;
};

namespace tc {

FB2_DEV uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
FB2_DEV unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
FB2_DEV void bar_init(uint64_t* b, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(b)), "r"(count) : "memory");
}
FB2_DEV void bar_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(b)), "r"(bytes) : "memory");
}
FB2_DEV bool bar_try(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(ok)
        : "r"(smem_addr(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for phase `parity` of barrier b; false on expiry or abort.
FB2_DEV bool bar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag) {
    if (bar_try(b, parity)) return true;
    const unsigned long long t0 = now_ns();
    while (!bar_try(b, parity)) {
        if (*abort_flag) return false;
        if (now_ns() - t0 > kTcTimeoutNs) {
            *abort_flag = 1;
            return false;
        }
    }
    return true;
}
FB2_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}
// Shared-memory matrix descriptor (sm_100 format, version 1) for a
// 128-byte-swizzled tile whose 1024-byte swizzle atoms start 1024-aligned.
FB2_DEV uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version for sm_100
    d |= (uint64_t)2 << 61;  // SWIZZLE_128B
    return d;
}
// Instruction descriptor: A, B TF32, both K-major, D F32, M x N.
constexpr uint32_t idesc_tf32(int M, int N) {
    return (1u << 4)                    // D format F32
           | (2u << 7) | (2u << 10)     // A, B format TF32
           | (0u << 15) | (0u << 16)    // A, B K-major
           | ((uint32_t)(N >> 3) << 17)  // N / 8
           | ((uint32_t)(M >> 4) << 24);  // M / 16
}
FB2_DEV void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p; }" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}
FB2_DEV void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
FB2_DEV void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
FB2_DEV void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 32 lanes x 16 consecutive 32-bit columns of TMEM into registers.
FB2_DEV void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

}  // namespace tc

// W [K][N] -> W^T halves hiT, loT [N][K] (32 x 32 tiles through shared
// memory), and W^T itself into rawT when it is not null.
__global__ void k_split_tf32_transpose(const float* __restrict__ W, int K, int N, float* __restrict__ hiT,
                                       float* __restrict__ loT, float* __restrict__ rawT) {
    pdl_wait();
    __shared__ float t[32][33];
    const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int k = k0 + r, n = n0 + threadIdx.x;
        t[r][threadIdx.x] = (k < K && n < N) ? W[(size_t)k * N + n] : 0.f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int n = n0 + r, k = k0 + threadIdx.x;
        if (n < N && k < K) {
            float h, l;
            const float v = t[threadIdx.x][r];
            tf32_split(v, h, l);
            hiT[(size_t)n * K + k] = h;
            loT[(size_t)n * K + k] = l;
            if (rawT) rawT[(size_t)n * K + k] = v;
        }
    }
}

// x -> (hi, lo) TF32 halves.
__global__ void k_split_tf32(const float4* __restrict__ x, size_t n4, float4* __restrict__ hi, float4* __restrict__ lo) {
    pdl_wait();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = x[i];
        float4 h, l;
        tf32_split(v.x, h.x, l.x);
        tf32_split(v.y, h.y, l.y);
        tf32_split(v.z, h.z, l.z);
        tf32_split(v.w, h.w, l.w);
        hi[i] = h;
        lo[i] = l;
    }
}

// Persistent, warp-specialized: one CTA per SM walks the 128 x BN output
// tiles t = blockIdx.x, += gridDim.x (row-major over N, so neighbouring CTAs
// share A rows in L2).  Warp 0 lane 0 feeds the smem ring with TMA for tile
// after tile; warp 1 lane 0 issues the MMAs into one of two TMEM
// accumulators (2 x BN columns), so warps 2-5 can drain tile i (tcgen05.ld
// of their TMEM lane quarter, the fused epilogue) while tile i+1 accumulates.
// Barriers: full/empty per ring stage; tfull[a] (MMA commit: accumulator a
// holds a finished tile) and tempty[a] (the 4 epilogue warps drained it).
constexpr int TCP_THREADS = 192;

template <int BN>
__global__ void __launch_bounds__(TCP_THREADS, 1) k_gemm_tc(const __grid_constant__ TcMaps maps, int M, int N, int K,
                                                            Epi e, int* err) {
    using Cfg = TcCfg<BN>;
    constexpr int STAGES = Cfg::STAGES, STAGE = Cfg::STAGE, TILE_B = Cfg::TILE_B;
    constexpr uint32_t TCOLS = 2 * BN;  // two accumulators
    extern __shared__ unsigned char tc_smem_raw[];
    __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2], drain;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int s_abort;
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tiles_n = (N + BN - 1) / BN, tiles_m = (M + TC_BM - 1) / TC_BM, ntiles = tiles_n * tiles_m;
    const int nk = (K + TC_BK - 1) / TC_BK;

    if (tid == 0) {
        s_abort = 0;
        for (int i = 0; i < STAGES; i++) {
            tc::bar_init(&full[i], 1);
            tc::bar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            tc::bar_init(&tfull[i], 1);
            tc::bar_init(&tempty[i], 4);
        }
        tc::bar_init(&drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_addr(&tmem_base)),
                     "r"(TCOLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = tmem_base;
    pdl_wait();  // barriers and tensor memory set up; global memory from here on

    if (warp == 0 && lane == 0) {
        // ---- TMA producer ----
        uint32_t it = 0;
        for (int t = blockIdx.x; t < ntiles && !s_abort; t += gridDim.x) {
            const int m0 = (t / tiles_n) * TC_BM, n0 = (t % tiles_n) * BN;
            for (int kb = 0; kb < nk; kb++, it++) {
                const int st = it % STAGES;
                if (it >= (uint32_t)STAGES && !tc::bar_wait(&empty[st], ((it / STAGES) - 1) & 1, &s_abort)) break;
                unsigned char* sb = sm + (size_t)st * STAGE;
                tc::bar_expect_tx(&full[st], STAGE);
                const int k0 = kb * TC_BK;
                tc::tma_load_2d(sb, &maps.a_hi, k0, m0, &full[st]);
                tc::tma_load_2d(sb + TC_TILE_A, &maps.a_lo, k0, m0, &full[st]);
                tc::tma_load_2d(sb + 2 * TC_TILE_A, &maps.b_hi, k0, n0, &full[st]);
                tc::tma_load_2d(sb + 2 * TC_TILE_A + TILE_B, &maps.b_lo, k0, n0, &full[st]);
            }
        }
        // copies still landing (after an abort): wait for each stage's latest fill
        if (s_abort)
            for (uint32_t j = it > (uint32_t)STAGES ? it - STAGES : 0; j < it; j++) {
                const unsigned long long t0 = tc::now_ns();
                while (!tc::bar_try(&full[j % STAGES], (j / STAGES) & 1) && tc::now_ns() - t0 < kTcTimeoutNs / 4) {
                }
            }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        constexpr uint32_t idesc = tc::idesc_tf32(TC_BM, BN);
        uint32_t it = 0, local = 0;
        for (int t = blockIdx.x; t < ntiles && !s_abort; t += gridDim.x, local++) {
            const uint32_t acc = local & 1;
            if (local >= 2 && !tc::bar_wait(&tempty[acc], ((local / 2) - 1) & 1, &s_abort)) break;
            tc::fence_after();
            const uint32_t d = tmem + acc * BN;
            bool ok = true;
            for (int kb = 0; kb < nk; kb++, it++) {
                const int st = it % STAGES;
                if (!tc::bar_wait(&full[st], (it / STAGES) & 1, &s_abort)) {
                    ok = false;
                    break;
                }
                tc::fence_after();
                const uint32_t sa = tc::smem_addr(sm + (size_t)st * STAGE);
                const uint32_t a_hi = sa, a_lo = sa + TC_TILE_A, b_hi = sa + 2 * TC_TILE_A, b_lo = b_hi + TILE_B;
#pragma unroll
                for (int ks = 0; ks < TC_BK / 8; ks++) {
                    const uint64_t dah = tc::sw128_desc(a_hi + ks * 32, 16, 1024);
                    const uint64_t dal = tc::sw128_desc(a_lo + ks * 32, 16, 1024);
                    const uint64_t dbh = tc::sw128_desc(b_hi + ks * 32, 16, 1024);
                    const uint64_t dbl = tc::sw128_desc(b_lo + ks * 32, 16, 1024);
                    tc::mma_tf32(d, dah, dbh, idesc, (kb | ks) != 0);
                    tc::mma_tf32(d, dah, dbl, idesc, 1u);
                    tc::mma_tf32(d, dal, dbh, idesc, 1u);
                }
                tc::mma_commit(&empty[st]);
            }
            if (!ok) break;
            tc::mma_commit(&tfull[acc]);
        }
        // every MMA issued above completes before the accumulators are freed
        tc::mma_commit(&drain);
        const unsigned long long t0 = tc::now_ns();
        while (!tc::bar_try(&drain, 0) && tc::now_ns() - t0 < kTcTimeoutNs) {
        }
    } else if (warp >= 2) {
        // ---- epilogue: TMEM lane quarter q = warp % 4 (rows 32q .. 32q+31 of the tile) ----
        const int q = warp & 3;
        uint32_t local = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, local++) {
            // warp-uniform decisions: tcgen05.ld below needs the whole warp
            if (__any_sync(0xffffffffu, s_abort != 0)) break;
            const uint32_t acc = local & 1;
            const bool ok = tc::bar_wait(&tfull[acc], (local / 2) & 1, &s_abort);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc::fence_after();
            const int m0 = (t / tiles_n) * TC_BM, n0 = (t % tiles_n) * BN;
            const int row = m0 + q * 32 + lane;
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 16) {
                float v[16];
                tc::tmem_ld16(tmem + acc * BN + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
                if (row < M) {
#pragma unroll
                    for (int k4 = 0; k4 < 4; k4++) {
                        const int n = n0 + c0 + 4 * k4;
                        if (n < N) epi_store4(e, row, n, N, make_float4(v[4 * k4], v[4 * k4 + 1], v[4 * k4 + 2], v[4 * k4 + 3]));
                    }
                }
            }
            tc::fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_addr(&tempty[acc])) : "memory");
        }
    }
    __syncwarp();
    if (s_abort && tid == 0) atomicExch(err, TC_ERR_TIMEOUT);
    tc::fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS) : "memory");
    }
}

// ---------------------------------------------------------------------------
// Decode batches (17..128 rows): the same 3xTF32 tensor-core product with the
// operands swapped, y^T = W^T * A^T.  The weights (W^T [N][K], K-major) are
// the 128-row MMA operand, read exactly once per step across the grid; the
// batch rows (A [M][K]) are the BNB-column operand.  TMEM lane = output
// column n, TMEM column = batch row m.  gridDim = (ceil(N/128),
// ceil(M/BNB), S): with S > 1 each CTA writes partial[z][M][N] and
// k_splitk_reduce sums the splits in order and applies the epilogue.
//
// Both operands arrive as they are stored, so each weight element crosses
// HBM once: maps.b_hi describes W^T itself (fp32, or bf16 when WB16) and
// maps.a_hi the fp32 batch rows.  Per stage, warps 2-7 turn the landed tiles
// into TF32 halves in shared memory and release the stage to the MMA warp
// through split[stage]:
//   fp32 W^T and A: in place (x_hi) plus x_lo at the same swizzled offset
//                   (the 128-byte swizzle places hi, lo and the source alike);
//   bf16 W^T:       the 64-byte rows land unswizzled in the w_lo slot and are
//                   widened into the swizzled w_hi tile; a bf16 value is exact
//                   in TF32, so w_lo is zero and its MMA is skipped.
// The halves equal the ones k_split_tf32_transpose makes for the prefill GEMM
// (both round to nearest, ties to even).
constexpr int TCS_THREADS = 256;
constexpr int TCS_SPLIT_WARPS = 6;  // warps 2..7

template <int BNB>
struct TcSwabCfg {
    static constexpr int TILE_B = BNB * TC_BK * 4;
    static constexpr int STAGE = 2 * TC_TILE_A + 2 * TILE_B;
    static constexpr int STAGES = (200 * 1024) / STAGE > 8 ? 8 : (200 * 1024) / STAGE;
    static constexpr int SMEM = STAGES * STAGE + 1024;
};

template <int BNB, bool WB16>
__global__ void __launch_bounds__(TCS_THREADS, 1) k_gemm_tc_swab(const __grid_constant__ TcMaps maps, int M, int N,
                                                                 int K, Epi e, int* err, float* __restrict__ partial) {
    using Cfg = TcSwabCfg<BNB>;
    constexpr int STAGES = Cfg::STAGES, STAGE = Cfg::STAGE, TILE_B = Cfg::TILE_B;
    constexpr int W_BYTES = WB16 ? TC_TILE_A / 2 : TC_TILE_A;  // one weight tile as stored
    extern __shared__ unsigned char tc_smem_raw[];
    __shared__ __align__(8) uint64_t full[STAGES], split[STAGES], empty[STAGES], accb;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int s_abort;
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * 128, m0 = blockIdx.y * BNB;
    const int S = gridDim.z, z = blockIdx.z;
    const int nk_all = (K + TC_BK - 1) / TC_BK;
    const int kb0 = (int)(((long long)z * nk_all) / S), kb1 = (int)(((long long)(z + 1) * nk_all) / S);
    const int nk = kb1 - kb0;

    if (tid == 0) {
        s_abort = 0;
        for (int i = 0; i < STAGES; i++) {
            tc::bar_init(&full[i], 1);
            tc::bar_init(&split[i], TCS_SPLIT_WARPS);  // one arrival per splitting warp
            tc::bar_init(&empty[i], 1);
        }
        tc::bar_init(&accb, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_addr(&tmem_base)),
                     "r"((uint32_t)BNB)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = tmem_base;
    pdl_wait();  // barriers and tensor memory set up; global memory from here on

    if (warp == 0 && lane == 0) {
        for (int i = 0; i < nk; i++) {
            const int st = i % STAGES;
            if (i >= STAGES && !tc::bar_wait(&empty[st], ((i / STAGES) - 1) & 1, &s_abort)) break;
            unsigned char* sb = sm + (size_t)st * STAGE;
            tc::bar_expect_tx(&full[st], W_BYTES + TILE_B);
            const int k0 = (kb0 + i) * TC_BK;
            // weights W^T (128-row boxes): fp32 into w_hi, bf16 into the w_lo slot
            tc::tma_load_2d(sb + (WB16 ? TC_TILE_A : 0), &maps.b_hi, k0, n0, &full[st]);
            tc::tma_load_2d(sb + 2 * TC_TILE_A, &maps.a_hi, k0, m0, &full[st]);
        }
    } else if (warp >= 2) {
        const int t = tid - 64;
        constexpr int NT = TCS_SPLIT_WARPS * 32;
        for (int i = 0; i < nk; i++) {
            const int st = i % STAGES;
            const bool ok = tc::bar_wait(&full[st], (i / STAGES) & 1, &s_abort);
            if (!__all_sync(0xffffffffu, ok)) break;
            unsigned char* sb = sm + (size_t)st * STAGE;
            float4* xh = reinterpret_cast<float4*>(sb + 2 * TC_TILE_A);
            float4* xl = reinterpret_cast<float4*>(sb + 2 * TC_TILE_A + TILE_B);
#pragma unroll 2
            for (int j = t; j < TILE_B / 16; j += NT) {
                const float4 v = xh[j];
                float4 h, l;
                tf32_split_rn(v.x, h.x, l.x);
                tf32_split_rn(v.y, h.y, l.y);
                tf32_split_rn(v.z, h.z, l.z);
                tf32_split_rn(v.w, h.w, l.w);
                xh[j] = h;
                xl[j] = l;
            }
            if constexpr (WB16) {
                // 128 rows x 32 bf16 (64 bytes) -> the swizzled fp32 tile:
                // element k of row r sits in 16-byte chunk (k / 4) ^ (r % 8)
                const uint4* src = reinterpret_cast<const uint4*>(sb + TC_TILE_A);
#pragma unroll 2
                for (int j = t; j < TC_TILE_A / 2 / 16; j += NT) {
                    const uint4 u = src[j];
                    const int r = j >> 2, c = (j & 3) * 2;
                    float4 a, b;
                    a.x = __uint_as_float(u.x << 16);
                    a.y = __uint_as_float(u.x & 0xFFFF0000u);
                    a.z = __uint_as_float(u.y << 16);
                    a.w = __uint_as_float(u.y & 0xFFFF0000u);
                    b.x = __uint_as_float(u.z << 16);
                    b.y = __uint_as_float(u.z & 0xFFFF0000u);
                    b.z = __uint_as_float(u.w << 16);
                    b.w = __uint_as_float(u.w & 0xFFFF0000u);
                    unsigned char* row = sb + r * 128;
                    *reinterpret_cast<float4*>(row + ((c ^ (r & 7)) << 4)) = a;
                    *reinterpret_cast<float4*>(row + (((c + 1) ^ (r & 7)) << 4)) = b;
                }
            } else {
                float4* wh = reinterpret_cast<float4*>(sb);
                float4* wl = reinterpret_cast<float4*>(sb + TC_TILE_A);
#pragma unroll 2
                for (int j = t; j < TC_TILE_A / 16; j += NT) {
                    const float4 v = wh[j];
                    float4 h, l;
                    tf32_split_rn(v.x, h.x, l.x);
                    tf32_split_rn(v.y, h.y, l.y);
                    tf32_split_rn(v.z, h.z, l.z);
                    tf32_split_rn(v.w, h.w, l.w);
                    wh[j] = h;
                    wl[j] = l;
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc::smem_addr(&split[st])) : "memory");
        }
    } else if (warp == 1 && lane == 0) {
        constexpr uint32_t idesc = tc::idesc_tf32(128, BNB);
        for (int i = 0; i < nk; i++) {
            const int st = i % STAGES;
            if (!tc::bar_wait(&split[st], (i / STAGES) & 1, &s_abort)) break;
            tc::fence_after();
            const uint32_t sa = tc::smem_addr(sm + (size_t)st * STAGE);
            const uint32_t w_hi = sa, w_lo = sa + TC_TILE_A, x_hi = sa + 2 * TC_TILE_A, x_lo = x_hi + TILE_B;
#pragma unroll
            for (int ks = 0; ks < TC_BK / 8; ks++) {
                const uint64_t dwh = tc::sw128_desc(w_hi + ks * 32, 16, 1024);
                const uint64_t dxh = tc::sw128_desc(x_hi + ks * 32, 16, 1024);
                const uint64_t dxl = tc::sw128_desc(x_lo + ks * 32, 16, 1024);
                tc::mma_tf32(tmem, dwh, dxh, idesc, (i | ks) != 0);
                tc::mma_tf32(tmem, dwh, dxl, idesc, 1u);
                if constexpr (!WB16) tc::mma_tf32(tmem, tc::sw128_desc(w_lo + ks * 32, 16, 1024), dxh, idesc, 1u);
            }
            tc::mma_commit(&empty[st]);
        }
        tc::mma_commit(&accb);
    }
    __syncwarp();

    bool ok = tc::bar_try(&accb, 0);
    if (!ok) {
        const unsigned long long t0 = tc::now_ns();
        while (!(ok = tc::bar_try(&accb, 0)) && tc::now_ns() - t0 < kTcTimeoutNs) {
        }
        if (!ok) s_abort = 1;
    }
    __syncwarp();
    tc::fence_after();
    // epilogue, warps 0-3 (TMEM lane quarter = warp; TMEM lane = output
    // column, TMEM column = batch row): the accumulator goes through shared
    // memory (the ring is free: every MMA, and so every read of the ring, has
    // completed) as a [BNB rows][128 columns] tile, then each warp writes
    // whole rows, one float4 per lane (512 contiguous bytes a store), through
    // the quad epilogue or into the split's partial rows.  Per-column stores
    // straight from the TMEM registers (128 bytes a store, a row apart)
    // measured 1.3-1.5 us slower a launch.
    const bool epi = ok && !s_abort && nk > 0;
    float* stg = reinterpret_cast<float*>(sm);
    if (warp < 4 && epi) {
#pragma unroll 1
        for (int c0 = 0; c0 < BNB; c0 += 16) {
            float v[16];
            tc::tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c0, v);
#pragma unroll
            for (int i = 0; i < 16; i++) stg[(c0 + i) * 128 + warp * 32 + lane] = v[i];
        }
    }
    if (warp < 4) asm volatile("bar.sync 1, 128;" ::: "memory");
    if (warp < 4 && epi) {
        const int nq = n0 + 4 * lane;
#pragma unroll 1
        for (int ml = warp; ml < BNB; ml += 4) {
            const int m = m0 + ml;
            if (m >= M) break;
            if (nq < N) {
                const float4 v = *reinterpret_cast<const float4*>(stg + ml * 128 + 4 * lane);
                if (S == 1) epi_store4(e, m, nq, N, v);
                else *reinterpret_cast<float4*>(partial + ((size_t)z * M + m) * N + nq) = v;
            }
        }
    }
    if (s_abort && tid == 0) {
        atomicExch(err, TC_ERR_TIMEOUT);
        for (int st = 0; st < STAGES && st < nk; st++) {
            const int last = st + ((nk - 1 - st) / STAGES) * STAGES;
            const unsigned long long t0 = tc::now_ns();
            while (!tc::bar_try(&full[st], (last / STAGES) & 1) && tc::now_ns() - t0 < kTcTimeoutNs / 4) {
            }
        }
    }
    tc::fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)BNB) : "memory");
    }
}

// y[m][n..n+3] = epilogue(sum over z = 0..S-1 of partial[z][m][n..n+3]).
__global__ void k_splitk_reduce(const float* __restrict__ partial, int S, int M, int N, Epi e) {
    pdl_wait();
    const int n4 = N / 4;
    const size_t total = (size_t)M * n4;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int m = (int)(i / n4), n = (int)(i - (size_t)m * n4) * 4;
        float4 bb, rr;
        epi_operands4(e, m, n, N, bb, rr);  // in flight with the partials
        float4 acc = __ldcg(reinterpret_cast<const float4*>(partial + (size_t)m * N + n));
        // eight splits' loads in flight before their adds (one L2 round trip
        // per eight); the adds keep the order z = 1, 2, ...
        for (int z0 = 1; z0 < S; z0 += 8) {
            float4 p[8];
#pragma unroll
            for (int j = 0; j < 8; j++)
                if (z0 + j < S) p[j] = __ldcg(reinterpret_cast<const float4*>(partial + ((size_t)(z0 + j) * M + m) * N + n));
#pragma unroll
            for (int j = 0; j < 8; j++)
                if (z0 + j < S) {
                    acc.x += p[j].x;
                    acc.y += p[j].y;
                    acc.z += p[j].z;
                    acc.w += p[j].w;
                }
        }
        epi_store4_with(e, m, n, N, acc, bb, rr);
    }
}

}  // namespace fb2
