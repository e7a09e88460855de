// gather_gemm.cuh -- a memory layer's read-out: the latest-k gather fused into the
// `fuse` Linear (ravel_lm/model.py:367-388), on the 5th-generation tensor cores.
//
// The reference materialises the read rows A = [latest-k values | segmented sums]
// ([B*T, C*k*D + C*D], ravel_lm/model.py:383-385), then runs `fuse` on them
// (fast_linear, a TF32 GEMM on CUDA) and the gate residual (model.py:388).  Here
// one kernel computes out = A * W^T (+ the gate residual) without A ever being
// written: every A tile is gathered from the payload rows named by the latest-k
// source table (and from the sums) straight into shared memory.
//
//   k_lk_sources     the source table: src[r, j] = flat payload row of read r's
//                    j-th latest earlier write, -1 for an invalid slot (whose
//                    reference value candidate*0 contributes zero to A * W^T).
//   k_gather_gemm    one CTA per 128 tokens x BN outputs.  Warps 0-7 gather A
//                    tiles (128 rows x 32 floats) with cp.async into the 128-byte
//                    swizzled K-major layout; warp 9 lane 0 loads the W tiles
//                    (BN rows x 32 floats) by TMA (this GPU's own memory, no
//                    multicast); warp 8 lane 0 issues tcgen05.mma kind::tf32
//                    (M 128, N BN, K 8 per instruction) into a TMEM accumulator;
//                    a 4-stage mbarrier ring connects them.  Warps 0-7 then read
//                    the accumulator with tcgen05.ld (warps w and w+4 share the
//                    TMEM lanes of rows 32(w%4).., half the columns each) and
//                    store it, optionally as x + sigmoid(gate) * acc.  Every wait is bounded: on a
//                    timeout the kernel sets RAVEL_DEVERR_SPIN, drains its own
//                    copies, frees its TMEM and returns.
//   k_gather_rows    the same gather written out as A (the backward's GEMMs).
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "latestk.cuh"

namespace ravel {

// ------------------------------------------------------------------ latest-k source table
// Aliased tapes: one thread per sorted position of a stream (the read at the
// same time t sees the writes before it in its address segment).
template <typename KeyT>
__global__ void k_lk_sources_aliased(const KeyT* __restrict__ keys, int64_t S, int64_t T, int64_t C, int tbits,
                                     int k, int32_t* __restrict__ src) {
    const KeyT tmask = (static_cast<KeyT>(1) << tbits) - 1;
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < S * T;
         g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t s = g / T, i = g - s * T;
        const KeyT* ks = keys + s * T;
        const KeyT ki = ks[i];
        const int64_t b = s / C, c = s - b * C;
        const int64_t row = (b * T + static_cast<int64_t>(ki & tmask)) * C + c;
        for (int j = 0; j < k; ++j) {
            const int64_t q = i - 1 - j;
            int32_t v = -1;
            if (q >= 0) {
                const KeyT kq = ks[q];
                if ((kq >> tbits) == (ki >> tbits))
                    v = static_cast<int32_t>((b * T + static_cast<int64_t>(kq & tmask)) * C + c);
            }
            src[row * k + j] = v;
        }
    }
}

// General tapes (reads apart from writes, or a write mask): one thread per
// (read, slot), the candidate rule of the general latest-k forward.
template <typename KeyT>
__global__ void k_lk_sources_general(LkArgs a, int32_t* __restrict__ src) {
    const int64_t n = a.B * a.T * a.C * a.k;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < n;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t row;
        bool valid;
        general_candidate<KeyT>(a, e / a.k, static_cast<int>(e % a.k), row, valid);
        src[e] = valid ? static_cast<int32_t>(row) : -1;
    }
}

// ------------------------------------------------------------------ PTX helpers (sm_100a)
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait on an mbarrier phase; false when the bound ran out (or abort is set).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
    const uint32_t limit = 4u * *const_cast<volatile unsigned int*>(&g_wait_limit);
    for (uint32_t it = 0; it < limit; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 1023u) == 1023u && *abort) return false;
        if (it > 4096u) __nanosleep(64);
    }
    return false;
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
// Four rows (y0..y3) of a 2-D tensor map, `x` elements into each, one box width
// each, into four consecutive 128-byte rows of shared memory (this GPU's memory,
// one CTA: no multicast).  A row index past the tensor reads zeros.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* map, int x, int y0, int y1, int y2,
                                            int y3, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand in the 128-byte swizzle layout: rows of 128 bytes, 8-row groups
// 1024 bytes apart (SBO), LBO unused (1), descriptor version 1, swizzle mode 2.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(1) << 16;               // leading byte offset (unused for this layout)
    d |= static_cast<uint64_t>(1024 >> 4) << 32;       // stride byte offset: 8 rows x 128 B
    d |= static_cast<uint64_t>(1) << 46;               // descriptor version
    d |= static_cast<uint64_t>(2) << 61;               // 128-byte swizzle
    return d;
}

// kind::tf32, D float32, A and B TF32, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ------------------------------------------------------------------ the read rows (A)
// Element kidx of read row n: latest-k slot s = kidx / D (value of slot (c, j) =
// (c*k + j)) from the payload row src[n, s] (zero when -1), then the sums of head
// c = s - C*k.  A 16-byte piece never straddles slots (D % 4 == 0).
struct GatherArgs {
    const float* payload;  // [B*T*C, D]
    const int32_t* src;    // [B*T, C*k] flat payload rows, -1 = invalid
    const float* sums;     // [B*T, C, D] or null (no sum read)
    int64_t M;             // tokens B*T
    int C, k, D, K;        // K = C*k*D (+ C*D with sums)
};

__device__ __forceinline__ const float* gather_piece(const GatherArgs& g, int64_t n, int kidx, bool& valid) {
    valid = false;
    if (n >= g.M || kidx >= g.K) return g.payload;
    const int s = kidx / g.D, d = kidx - s * g.D;
    const int ck = g.C * g.k;
    if (s < ck) {
        const int32_t row = g.src[n * ck + s];
        if (row < 0) return g.payload;
        valid = true;
        return g.payload + static_cast<int64_t>(row) * g.D + d;
    }
    valid = true;
    return g.sums + (n * g.C + (s - ck)) * static_cast<int64_t>(g.D) + d;
}

__global__ void k_gather_rows(GatherArgs g, float* __restrict__ A) {
    const int64_t pieces = g.M * (g.K / 4);
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < pieces;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t n = i / (g.K / 4);
        const int kidx = static_cast<int>(i - n * (g.K / 4)) * 4;
        bool valid;
        const float* p = gather_piece(g, n, kidx, valid);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (valid) v = *reinterpret_cast<const float4*>(p);
        *reinterpret_cast<float4*>(A + n * g.K + kidx) = v;
    }
}

// ------------------------------------------------------------------ the fused GEMM
constexpr int GG_BM = 128;         // tokens per CTA (UMMA M)
constexpr int GG_BK = 32;          // floats per K chunk: one 128-byte swizzle row
// pipeline depth per column tile: as many stages as fit in shared memory
// (64 columns: 8 x 24 KB, 128: 6 x 32 KB, 256: 4 x 48 KB)
template <int BN>
__host__ __device__ constexpr int gg_stages() { return BN <= 64 ? 8 : (BN <= 128 ? 6 : 4); }
constexpr int GG_PWARPS = 8;       // warps 0-7 gather A, then run the epilogue
constexpr int GG_PRODUCERS = GG_PWARPS * 32;
constexpr int GG_MMA_WARP = GG_PWARPS;      // lane 0 issues the MMAs
constexpr int GG_TMA_WARP = GG_PWARPS + 1;  // lane 0 loads the W tiles
constexpr int GG_THREADS = GG_PRODUCERS + 64;

struct GemmArgs {
    GatherArgs g;
    int N;                 // outputs (weight rows)
    float* out;            // [M, N]
    float* pre;            // [M, N] the GEMM result before the gate, or null
    const float* x;        // gate residual: out = x + sigmoid(gate) * acc (both [M, N]) or null
    const float* gate;
    int ck_smem;           // > 0: the source table of a tile is staged in shared memory
};

// Dynamic shared memory: the stage ring, barriers, and (when it fits, ck_smem > 0)
// the tile's source-row table [128][ck] int32.
template <int BN>
constexpr size_t gather_gemm_smem(int ck_smem) {
    return 1024 /* alignment slack */ + static_cast<size_t>(gg_stages<BN>()) * (GG_BM + BN) * GG_BK * 4 + 256 +
           static_cast<size_t>(ck_smem) * GG_BM * 4;
}

// sigmoid for the TF32 epilogue: 1 / (1 + e^-x) with the fast exponential
__device__ __forceinline__ float gg_sigmoid(float x) { return __frcp_rn(1.0f + __expf(-x)); }

// Epilogue of one 32-column slice of the accumulator: TMEM lanes 32*(warp % 4) ..
// +31 are this warp's rows.
template <int BN>
__device__ __forceinline__ void gg_epilogue_slice(const GemmArgs& a, uint32_t tmem, int warp, int lane, int64_t m0,
                                                  int n0, int c0) {
    uint32_t r[32];
    tmem_ld32(tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + static_cast<uint32_t>(c0), r);
    const int64_t gm = m0 + (warp & 3) * 32 + lane;
    if (gm >= a.g.M || n0 + c0 >= a.N) return;
    const bool vec = (a.N & 3) == 0;  // rows start 16-byte aligned: 4-float stores
#pragma unroll
    for (int c = 0; c < 32; c += 4) {
        const int col = n0 + c0 + c;
        if (col >= a.N) break;
        const int64_t o = gm * a.N + col;
        float v[4] = {__uint_as_float(r[c]), __uint_as_float(r[c + 1]), __uint_as_float(r[c + 2]),
                      __uint_as_float(r[c + 3])};
        const int nv = (a.N - col) < 4 ? (a.N - col) : 4;
        if (vec) {
            if (a.pre) *reinterpret_cast<float4*>(a.pre + o) = make_float4(v[0], v[1], v[2], v[3]);
            if (a.x) {
                const float4 xv = *reinterpret_cast<const float4*>(a.x + o);
                const float4 gv = *reinterpret_cast<const float4*>(a.gate + o);
                const float xs[4] = {xv.x, xv.y, xv.z, xv.w}, gs[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) v[e] = xs[e] + gg_sigmoid(gs[e]) * v[e];
            }
            *reinterpret_cast<float4*>(a.out + o) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
            for (int e = 0; e < nv; ++e) {
                if (a.pre) a.pre[o + e] = v[e];
                float y = v[e];
                if (a.x) y = a.x[o + e] + gg_sigmoid(a.gate[o + e]) * y;
                a.out[o + e] = y;
            }
        }
    }
}

// GATHER4: A tiles come from TMA gather4 loads of the payload and sums rows (D a
// multiple of 32: a K chunk lies in one slot), issued by the TMA warp; otherwise the
// producer warps gather 16-byte pieces with cp.async.
template <int BN, bool GATHER4>
__global__ void __launch_bounds__(GG_THREADS, 1) k_gather_gemm(const __grid_constant__ CUtensorMap wmap,
                                                              const __grid_constant__ CUtensorMap pmap,
                                                              const __grid_constant__ CUtensorMap smap,
                                                              GemmArgs a) {
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "UMMA N for M = 128; two column halves of 32k");
    constexpr int GG_STAGES = gg_stages<BN>();
    constexpr uint32_t A_BYTES = GG_BM * GG_BK * 4, B_BYTES = BN * GG_BK * 4;
    constexpr uint32_t TMEM_COLS = BN <= 64 ? 64 : (BN <= 128 ? 128 : 256);
    constexpr int ROWS_PER_THREAD = GG_BM * 8 / GG_PRODUCERS;  // 8 pieces of 16 bytes per row
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // swizzled tiles need 1024-byte alignment
    const uint32_t sA = base, sB = base + GG_STAGES * A_BYTES;
    const uint32_t sbar = sB + GG_STAGES * B_BYTES;  // full[S], empty[S], done
    unsigned char* gen = smem_raw + (sbar + 8 * (2 * GG_STAGES + 1) - raw);
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(gen);
    volatile int* abort = reinterpret_cast<volatile int*>(gen + 4);
    int32_t* ssrc = reinterpret_cast<int32_t*>(gen + 16);  // [128][ck] when a.ck_smem
    const uint32_t bar_full = sbar, bar_empty = sbar + 8 * GG_STAGES, bar_done = sbar + 16 * GG_STAGES;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t m0 = static_cast<int64_t>(blockIdx.x) * GG_BM;
    const int n0 = blockIdx.y * BN;
    const int nk = (a.g.K + GG_BK - 1) / GG_BK;
    const int ck = a.g.C * a.g.k;
    if (a.ck_smem && warp < GG_PWARPS) {  // the tile's rows of the source table are contiguous
        const int64_t rows = (a.g.M - m0) < GG_BM ? (a.g.M - m0) : GG_BM;
        for (int i = tid; i < GG_BM * ck; i += GG_PRODUCERS)
            ssrc[i] = i < rows * ck ? __ldg(a.g.src + m0 * ck + i) : -1;
    }

    if (tid == 0) {
        for (int s = 0; s < GG_STAGES; ++s) {
            mbar_init(bar_full + 8 * s, GATHER4 ? 1 : GG_PRODUCERS + 1);
            mbar_init(bar_empty + 8 * s, 1);
        }
        mbar_init(bar_done, 1);
        *abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {  // one warp allocates the accumulator's TMEM columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(gen)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < GG_PWARPS) {
        // ---------------- A producers.  Thread t owns 16-byte piece pc = t % 8 of rows
        // t / 8 + 32 i: the piece's slot and offset are worked out once per chunk, and
        // its rows' source rows are independent loads issued back to back.
        const int pc = tid & 7, r0 = tid >> 3;
        for (int kc = 0; kc < (GATHER4 ? 0 : nk); ++kc) {
            const int s = kc % GG_STAGES;
            if (kc >= GG_STAGES && !mbar_wait(bar_empty + 8 * s, ((kc / GG_STAGES) - 1) & 1, abort)) {
                *abort = 1;
                break;
            }
            const int kidx = kc * GG_BK + pc * 4;
            const bool in_k = kidx < a.g.K;
            const int slot = in_k ? kidx / a.g.D : 0;
            const int d = kidx - slot * a.g.D;
            const bool lk = slot < ck;
            int32_t srow[ROWS_PER_THREAD];
#pragma unroll
            for (int i = 0; i < ROWS_PER_THREAD; ++i) {
                const int64_t n = m0 + r0 + 32 * i;
                srow[i] = (in_k && lk && n < a.g.M)
                              ? (a.ck_smem ? ssrc[(r0 + 32 * i) * ck + slot] : __ldg(a.g.src + n * ck + slot))
                              : -1;
            }
            const uint32_t stage = sA + s * A_BYTES;
#pragma unroll
            for (int i = 0; i < ROWS_PER_THREAD; ++i) {
                const int r = r0 + 32 * i;
                const int64_t n = m0 + r;
                const float* src = a.g.payload;
                bool valid = false;
                if (in_k && n < a.g.M) {
                    if (lk) {
                        valid = srow[i] >= 0;
                        if (valid) src = a.g.payload + static_cast<int64_t>(srow[i]) * a.g.D + d;
                    } else {
                        valid = true;
                        src = a.g.sums + (n * a.g.C + (slot - ck)) * static_cast<int64_t>(a.g.D) + d;
                    }
                }
                cp_async16_zfill(stage + r * 128 + ((pc ^ (r & 7)) << 4), src, valid);
            }
            cp_async_commit();
            if (kc >= GG_STAGES - 1) {  // the chunk issued STAGES-1 iterations ago has landed
                cp_async_wait<GG_STAGES - 1>();
                fence_proxy_async_smem();
                mbar_arrive(bar_full + 8 * ((kc - (GG_STAGES - 1)) % GG_STAGES));
            }
        }
        if (!GATHER4) {
            cp_async_wait<0>();
            fence_proxy_async_smem();
            if (!*abort) {
                for (int kc = nk - (GG_STAGES - 1) < 0 ? 0 : nk - (GG_STAGES - 1); kc < nk; ++kc)
                    mbar_arrive(bar_full + 8 * (kc % GG_STAGES));
            }
        }
        // ---------------- epilogue: warps w and w + 4 share TMEM lanes 32*(w%4), each
        // takes half of the columns.  The wait for the last MMA sleeps between polls,
        // leaving the issue slots to the TMA and MMA warps.
        bool ok = !*abort;
        if (ok) {
            ok = false;
            const uint32_t limit = 4u * *const_cast<volatile unsigned int*>(&g_wait_limit);
            for (uint32_t it = 0; it < limit; ++it) {
                if (mbar_try_wait(bar_done, 0)) { ok = true; break; }
                if ((it & 255u) == 255u && *abort) break;
                __nanosleep(256);
            }
        }
        tc_fence_after();
        if (!ok) {
            *abort = 1;
        } else {
            const int half = warp >> 2;
            for (int c0 = half * (BN / 2); c0 < (half + 1) * (BN / 2); c0 += 32)
                gg_epilogue_slice<BN>(a, tmem, warp, lane, m0, n0, c0);
        }
    } else if (warp == GG_MMA_WARP && lane == 0) {
        // ---------------- the MMAs of each chunk, as soon as its A and W tiles landed
        constexpr uint32_t IDESC = idesc_tf32(GG_BM, BN);
        for (int kc = 0; kc < nk; ++kc) {
            const int s = kc % GG_STAGES;
            if (!mbar_wait(bar_full + 8 * s, (kc / GG_STAGES) & 1, abort)) {
                *abort = 1;
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < GG_BK / 8; ++kk) {  // K = 8 per tf32 MMA: 32 bytes along the row
                const uint64_t da = smem_desc_sw128(sA + s * A_BYTES + kk * 32);
                const uint64_t db = smem_desc_sw128(sB + s * B_BYTES + kk * 32);
                umma_tf32(tmem, da, db, IDESC, (kc > 0 || kk > 0) ? 1u : 0u);
            }
            umma_commit(bar_empty + 8 * s);  // frees the stage when these MMAs have read it
        }
        umma_commit(bar_done);  // arrives when every MMA issued above has completed
    } else if (warp == GG_TMA_WARP && (GATHER4 || lane == 0)) {
        // ---------------- W tiles by TMA (this GPU's memory, no multicast), STAGES ahead;
        // with GATHER4 the warp's lanes also fetch the A tile, 4 rows per gather4
        const int64_t rows_p = a.g.M * a.g.C;  // payload / sums rows: past them reads zeros
        for (int kc = 0; kc < nk; ++kc) {
            const int s = kc % GG_STAGES;
            bool go = true;
            if (lane == 0) {
                if (kc >= GG_STAGES && !mbar_wait(bar_empty + 8 * s, ((kc / GG_STAGES) - 1) & 1, abort)) {
                    *abort = 1;
                    go = false;
                } else {
                    mbar_arrive_expect_tx(bar_full + 8 * s, B_BYTES + (GATHER4 ? A_BYTES : 0u));
                    tma_load_2d(sB + s * B_BYTES, &wmap, kc * GG_BK, n0, bar_full + 8 * s);
                }
            }
            if (GATHER4) {
                go = __shfl_sync(0xffffffffu, go, 0);
                if (!go) break;
                // chunk kc: slot and column offset (a chunk lies in one slot: D % 32 == 0)
                const int kidx = kc * GG_BK;
                const int slot = kidx / a.g.D, d = kidx - slot * a.g.D;
                const bool lk = slot < ck;
                int y[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int r = lane * 4 + i;
                    const int64_t n = m0 + r;
                    int64_t row = rows_p;  // out of range: zero fill
                    if (n < a.g.M) {
                        if (lk) {
                            const int32_t v = a.ck_smem ? ssrc[r * ck + slot] : __ldg(a.g.src + n * ck + slot);
                            if (v >= 0) row = v;
                        } else {
                            row = n * a.g.C + (slot - ck);
                        }
                    }
                    y[i] = static_cast<int>(row);
                }
                tma_gather4(sA + s * A_BYTES + lane * 512, lk ? &pmap : &smap, d, y[0], y[1], y[2], y[3],
                            bar_full + 8 * s);
            } else if (!go) {
                break;
            }
        }
        if (*abort) {
            // tile loads still in flight land within microseconds; give them a bounded
            // while before the CTA's shared memory is released
            for (int i = 0; i < 256; ++i) __nanosleep(4000);
        }
    }
    // ---------------- teardown: the MMAs are complete (done barrier) before TMEM is freed
    if (warp == GG_MMA_WARP && lane == 0 && *abort) (void)mbar_wait(bar_done, 0, abort);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (*abort && tid == 0) flag_error(RAVEL_DEVERR_SPIN);
    if (warp == 0) {
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS)
                     : "memory");
    }
}

}  // namespace ravel
