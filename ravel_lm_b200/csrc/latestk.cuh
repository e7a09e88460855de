// latestk.cuh -- causal latest-k lookup over the sorted event tape.
//
// Reference: ravel_lm/ravel_memory.py:153-176.  For a read at time t the
// reference searches its key (base, t-1) in the sorted write keys, takes the k
// sorted positions idx, idx-1, ..., idx-k+1, marks a slot valid when that key is
// in the same (stream, address) group, and returns payload[order[safe]] * valid.
// An invalid slot therefore holds candidate*0 (+-0 with the candidate's sign);
// these kernels reproduce that bit for bit, including candidates that fall in
// an earlier stream of the reference's global sorted order.
//
// Aliased reads, no mask ("fast" path): the read at sorted position p has its
// latest earlier writes at p-1, p-2, ... (its own key is (addr, t) and every
// key below it is <= (addr, t-1)), so one CTA handles a chunk of P sorted
// positions with a window of P+k payload rows staged in shared memory by
// cp.async.  Every row is read from HBM once; each output block of k*D
// elements is one contiguous streaming store.
//
// General reads or a write mask: each read's latest index comes from
// k_merge_ranks; the forward takes reads in their original order so the output
// is written sequentially, and gathers the candidate rows directly; the backward
// gathers over the read tape (k_lk_bwd_gather).
#pragma once

#include "common.cuh"

namespace ravel {

struct LkArgs {
    const void* keys;       // [S][T] sorted per stream
    const int* nvalid;      // general: [S]
    const int64_t* soff;    // general: [S+1] exclusive prefix of nvalid
    const int32_t* ridx;    // general: [N]
    const void* raddr;      // general: [N]
    int addr_i64, key32;
    const void* payload;    // [N, D]
    const void* grad;       // backward: grad of values [N, k, D]
    void* out;              // forward: values [N, k, D]; backward: grad payload [N, D] / fp32 accum
    uint8_t* out_mask;      // forward: [N, k]
    int64_t B, T, C, D, A, k;
    int tbits;
    int64_t row_bytes;      // D * element bytes
    int P;                  // sorted positions per CTA (fast path)
    int64_t nchunks;        // chunks per stream (fast path)
    FastDiv fd_rv, fd_bv, fd_k;  // divisions by vectors-per-row, vectors-per-block, k
    FastDiv fd_C, fd_T;          // flat row -> (b, t, c)
    int accumulate;         // backward: add to grad payload instead of overwriting it
};

// Flat payload row of (stream s, time t) = ((s / C) * T + t) * C + s % C,
// computed as base + t*C with the stream's base precomputed once (rows are
// below 2^31: the entry points reject larger B*T*C).
struct RowMap {
    uint32_t base, C;
    __device__ __forceinline__ RowMap(int64_t s, int64_t T, int64_t Cn) {
        const int64_t b = s / Cn, c = s - (s / Cn) * Cn;
        base = static_cast<uint32_t>(b * T * Cn + c);
        C = static_cast<uint32_t>(Cn);
    }
    __device__ __forceinline__ uint32_t operator()(uint64_t t) const {
        return base + static_cast<uint32_t>(t) * C;
    }
};

// Row of (stream s, time t) for a stream that is not the thread's own (rare paths).
__device__ __forceinline__ int64_t flat_row(int64_t s, int64_t t, int64_t T, int64_t C) {
    return ((s / C) * T + t) * C + (s % C);
}

// ------------------------------------------------------------------ fast forward
template <typename KeyT, int DT, int VB>
__global__ void __launch_bounds__(256) k_lk_fwd_fast(LkArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int k = static_cast<int>(a.k);
    const int W = a.P + k;
    int64_t* wrow = reinterpret_cast<int64_t*>(smem);
    uint64_t* wadr = reinterpret_cast<uint64_t*>(wrow + W);
    unsigned char* rows = reinterpret_cast<unsigned char*>(wadr + W);
    rows += (16 - (reinterpret_cast<uintptr_t>(rows) & 15)) & 15;

    const int tid = threadIdx.x;
    const int64_t T = a.T, C = a.C;
    const int64_t s = blockIdx.x / a.nchunks;
    const int64_t p0 = (blockIdx.x % a.nchunks) * a.P;
    const int np = static_cast<int>((T - p0) < a.P ? (T - p0) : a.P);
    const int nw = np + k;
    const KeyT* keys = static_cast<const KeyT*>(a.keys);
    const KeyT tmask = (static_cast<KeyT>(1) << a.tbits) - 1;

    const RowMap rows_of(s, T, C);
    for (int i = tid; i < nw; i += 256) {
        const int64_t p = p0 - k + i;
        if (p >= 0) {
            const KeyT key = keys[s * T + p];
            wrow[i] = rows_of(key & tmask);
            wadr[i] = static_cast<uint64_t>(key >> a.tbits);
        } else {
            // candidate in an earlier stream of the reference's global order:
            // never valid, only its sign bits are used (ravel_memory.py:163 clamp)
            int64_t g = s * T + p;
            if (g < 0) g = 0;
            const KeyT key = keys[g];
            wrow[i] = flat_row(g / T, static_cast<int64_t>(key & tmask), T, C);
            wadr[i] = ~0ull;
        }
    }
    __syncthreads();

    const uint32_t rv = static_cast<uint32_t>(a.row_bytes / VB);
    const char* pay = static_cast<const char*>(a.payload);
    for (uint32_t e = tid; e < static_cast<uint32_t>(nw) * rv; e += 256) {
        uint32_t i, v;
        a.fd_rv.divmod(e, i, v);
        const char* src = pay + wrow[i] * a.row_bytes + v * VB;
        unsigned char* dst = rows + static_cast<int64_t>(i) * a.row_bytes + v * VB;
        if constexpr (VB == 16) cp_async16(dst, src);
        else if constexpr (VB == 8) cp_async8(dst, src);
        else if constexpr (VB == 4) cp_async4(dst, src);
        else st_vec<2>(dst, ld_vec<2>(src));
    }
    cp_async_wait_all();
    __syncthreads();

    // Output: warp w walks positions w, w+8, ...; within a position the block of
    // k*rv vectors is covered by the 32 lanes in passes.  Each lane's (position
    // offset, slot, vector) decomposition is computed once, not per element.
    char* outv = static_cast<char*>(a.out);
    const int lane = tid & 31, warp = tid >> 5;
    const uint32_t bv = rv * static_cast<uint32_t>(k);  // vectors per output block
    if (bv == 0) {
        for (int e = tid; e < np * k; e += 256) {
            const int i = e / k, j = e % k;
            a.out_mask[wrow[i + k] * k + j] = wadr[i + k - 1 - j] == wadr[i + k] ? 1 : 0;
        }
        return;
    }
    if (bv <= 32) {
        // several positions per warp pass
        const int gp = static_cast<int>(32 / bv);
        uint32_t dp, v, j, o;
        a.fd_bv.divmod(static_cast<uint32_t>(lane), dp, v);
        a.fd_rv.divmod(v, j, o);
        const bool lane_on = static_cast<int>(dp) < gp;
        for (int i0 = warp * gp; i0 < np; i0 += 8 * gp) {
            const int i = i0 + static_cast<int>(dp);
            if (!lane_on || i >= np) continue;
            const int wi = i + k;
            const int src = wi - 1 - static_cast<int>(j);
            const bool valid = wadr[src] == wadr[wi];
            uint4 x = ld_vec<VB>(rows + static_cast<int64_t>(src) * a.row_bytes + o * VB);
            if (!valid) x = VecZero<DT, VB>::apply(x);
            const int64_t blk = wrow[wi] * k + j;
            st_vec_stream<VB>(outv + blk * a.row_bytes + o * VB, x);
            if (o == 0) a.out_mask[blk] = valid ? 1 : 0;
        }
    } else if (32 % rv == 0 && DT != RAVEL_F64) {
        // one position per warp; lane = (slot offset j0, vector o) fixed for the
        // kernel, slots j0, j0 + 32/rv, ... in successive passes
        const uint32_t jstep = 32 / rv;
        const uint32_t o = static_cast<uint32_t>(lane) % rv, j0 = static_cast<uint32_t>(lane) / rv;
        const uint32_t rows_s = smem_u32(rows) + o * VB;
        const uint32_t rb32 = static_cast<uint32_t>(a.row_bytes);
        const uint64_t blk_bytes = static_cast<uint64_t>(a.row_bytes) * static_cast<uint64_t>(k);
        for (int i = warp; i < np; i += 8) {
            const int wi = i + k;
            const uint32_t my = static_cast<uint32_t>(wadr[wi]);
            const uint32_t orow = static_cast<uint32_t>(wrow[wi]);
            char* ob = outv + orow * blk_bytes + o * VB;
            uint8_t* mb = a.out_mask + static_cast<uint64_t>(orow) * static_cast<uint64_t>(k);
            for (uint32_t j = j0; j < static_cast<uint32_t>(k); j += jstep) {
                const int src = wi - 1 - static_cast<int>(j);
                const bool valid = static_cast<uint32_t>(wadr[src]) == my;
                uint4 x;
                asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                             : "=r"(x.x), "=r"(x.y), "=r"(x.z), "=r"(x.w)
                             : "r"(rows_s + static_cast<uint32_t>(src) * rb32));
                if (!valid) {
                    x.x = zero_word_packed<DT>(x.x);
                    if constexpr (VB >= 8) x.y = zero_word_packed<DT>(x.y);
                    if constexpr (VB == 16) { x.z = zero_word_packed<DT>(x.z); x.w = zero_word_packed<DT>(x.w); }
                }
                st_vec_stream<VB>(ob + j * rb32, x);
                if (o == 0) mb[j] = valid ? 1 : 0;
            }
        }
    } else {
        // one position per warp, ceil(bv/32) passes
        for (int i = warp; i < np; i += 8) {
            const int wi = i + k;
            const uint64_t my = wadr[wi];
            const int64_t base = wrow[wi] * k;
            for (uint32_t v = lane; v < bv; v += 32) {
                uint32_t j, o;
                a.fd_rv.divmod(v, j, o);
                const int src = wi - 1 - static_cast<int>(j);
                const bool valid = wadr[src] == my;
                uint4 x = ld_vec<VB>(rows + static_cast<int64_t>(src) * a.row_bytes + o * VB);
                if (!valid) x = VecZero<DT, VB>::apply(x);
                st_vec_stream<VB>(outv + (base + j) * a.row_bytes + o * VB, x);
                if (o == 0) a.out_mask[base + j] = valid ? 1 : 0;
            }
        }
    }
}

inline size_t lk_fast_smem(int P, int64_t k, int64_t row_bytes) {
    return static_cast<size_t>(P + k) * 16 + 16 + static_cast<size_t>(P + k) * row_bytes;
}

// ------------------------------------------------------------------ fast backward
// grad[q] = sum_j [addr(q+1+j) == addr(q)] * grad_vals[read at q+1+j, slot j]:
// every valid (read, slot) feeds exactly one write, so the sum is a gather and
// needs no atomics.  Accumulates in float (double for float64).
template <typename KeyT, int DT, int VB>
__global__ void __launch_bounds__(256) k_lk_bwd_fast(LkArgs a) {
    using E = Elem<DT>;
    using Acc = typename E::Acc;
    using V = typename E::T;
    constexpr int EPV = VB / sizeof(V);  // elements per vector
    extern __shared__ __align__(16) unsigned char smem[];
    const int k = static_cast<int>(a.k);
    const int W = a.P + k;
    int64_t* wrow = reinterpret_cast<int64_t*>(smem);
    uint64_t* wadr = reinterpret_cast<uint64_t*>(wrow + W);

    const int tid = threadIdx.x;
    const int64_t T = a.T, C = a.C;
    const int64_t s = blockIdx.x / a.nchunks;
    const int64_t q0 = (blockIdx.x % a.nchunks) * a.P;
    const int np = static_cast<int>((T - q0) < a.P ? (T - q0) : a.P);
    const int64_t avail = T - q0;  // positions of this stream from q0 on
    const int nw = static_cast<int>((np + k) < avail ? (np + k) : avail);
    const KeyT* keys = static_cast<const KeyT*>(a.keys) + s * T;
    const KeyT tmask = (static_cast<KeyT>(1) << a.tbits) - 1;
    const RowMap rows_of(s, T, C);
    for (int i = tid; i < nw; i += 256) {
        const KeyT key = keys[q0 + i];
        wrow[i] = rows_of(key & tmask);
        wadr[i] = static_cast<uint64_t>(key >> a.tbits);
    }
    __syncthreads();

    const uint32_t rv = static_cast<uint32_t>(a.row_bytes / VB);
    const char* g = static_cast<const char*>(a.grad);
    char* outp = static_cast<char*>(a.out);
    for (uint32_t e = tid; e < static_cast<uint32_t>(np) * rv; e += 256) {
        uint32_t i, v;
        a.fd_rv.divmod(e, i, v);
        Acc acc[EPV];
#pragma unroll
        for (int x = 0; x < EPV; ++x) acc[x] = Acc(0);
        if (a.accumulate) {
            const uint4 prev = ld_vec<VB>(outp + wrow[i] * a.row_bytes + v * VB);
            const V* pv0 = reinterpret_cast<const V*>(&prev);
#pragma unroll
            for (int x = 0; x < EPV; ++x) acc[x] = E::to_acc(pv0[x]);
        }
        const uint64_t my = wadr[i];
        for (int j = 0; j < k; ++j) {
            const int wi = static_cast<int>(i) + 1 + j;
            if (wi >= nw || wadr[wi] != my) break;  // segments are contiguous
            const uint4 raw = ldg_vec<VB>(g + (wrow[wi] * k + j) * a.row_bytes + v * VB);
            const V* vals = reinterpret_cast<const V*>(&raw);
#pragma unroll
            for (int x = 0; x < EPV; ++x) acc[x] += E::to_acc(vals[x]);
        }
        uint4 packed = make_uint4(0u, 0u, 0u, 0u);
        V* pv = reinterpret_cast<V*>(&packed);
#pragma unroll
        for (int x = 0; x < EPV; ++x) pv[x] = E::from_acc(acc[x]);
        st_vec<VB>(outp + wrow[i] * a.row_bytes + v * VB, packed);
    }
}

inline size_t lk_bwd_fast_smem(int P, int64_t k) { return static_cast<size_t>(P + k) * 16; }

// ------------------------------------------------------------------ general forward
// One thread per (read, slot, vector); reads in their original order.
template <typename KeyT>
__device__ __forceinline__ void general_candidate(const LkArgs& a, int64_t r, int j, int64_t& row, bool& valid) {
    const int64_t T = a.T, C = a.C;
    uint32_t bt, c32, b32, t32;
    a.fd_C.divmod(static_cast<uint32_t>(r), bt, c32);  // r = (b*T + t)*C + c
    a.fd_T.divmod(bt, b32, t32);
    const int64_t s = static_cast<int64_t>(b32) * C + c32;
    const KeyT* keys = static_cast<const KeyT*>(a.keys);
    const KeyT tmask = (static_cast<KeyT>(1) << a.tbits) - 1;
    const int64_t S = a.B * C;
    if (a.soff[S] == 0) { row = -1; valid = false; return; }  // ravel_memory.py:146-149
    const int64_t q = static_cast<int64_t>(a.ridx[r]) - j;
    if (q >= 0) {
        const KeyT key = keys[s * T + q];
        const uint64_t ra = fold_addr(load_addr(a.raddr, r, a.addr_i64), a.A, a.key32);
        valid = static_cast<uint64_t>(key >> a.tbits) == ra;
        row = r + (static_cast<int64_t>(key & tmask) - static_cast<int64_t>(t32)) * C;  // same (b, c), time t'
        return;
    }
    // Candidate before this stream in the global sorted order (always invalid):
    // the stream s2 with soff[s2] <= gpos < soff[s2+1] (non-empty by construction).
    int64_t gpos = a.soff[s] + q;
    if (gpos < 0) gpos = 0;
    int64_t lo = 0, hi = S - 1;
    while (lo < hi) {  // last s2 with soff[s2] <= gpos
        const int64_t mid = (lo + hi + 1) >> 1;
        if (a.soff[mid] <= gpos) lo = mid; else hi = mid - 1;
    }
    const int64_t s2 = lo;
    const KeyT key = keys[s2 * T + (gpos - a.soff[s2])];
    row = flat_row(s2, static_cast<int64_t>(key & tmask), T, C);
    valid = false;
}

template <typename KeyT, int DT, int VB>
__global__ void __launch_bounds__(256) k_lk_fwd_general(LkArgs a, int64_t reads_per_cta) {
    __shared__ int64_t srow[512];
    __shared__ uint8_t sval[512];
    const int k = static_cast<int>(a.k);
    const int64_t N = a.B * a.T * a.C;
    const int64_t r0 = blockIdx.x * reads_per_cta;
    const int nr = static_cast<int>((N - r0) < reads_per_cta ? (N - r0) : reads_per_cta);
    const int ns = nr * k;  // <= 512
    for (int e = threadIdx.x; e < ns; e += 256) {
        int64_t row; bool valid;
        general_candidate<KeyT>(a, r0 + e / k, e % k, row, valid);
        srow[e] = row;
        sval[e] = valid;
        a.out_mask[r0 * k + e] = valid ? 1 : 0;
    }
    __syncthreads();
    const uint32_t rv = static_cast<uint32_t>(a.row_bytes / VB);
    const char* pay = static_cast<const char*>(a.payload);
    char* outv = static_cast<char*>(a.out) + r0 * k * a.row_bytes;
    for (uint32_t e = threadIdx.x; e < static_cast<uint32_t>(ns) * rv; e += 256) {
        uint32_t sl, v;
        a.fd_rv.divmod(e, sl, v);
        const int64_t row = srow[sl];
        uint4 x = make_uint4(0u, 0u, 0u, 0u);
        if (row >= 0) {
            x = ldg_vec<VB>(pay + row * a.row_bytes + v * VB);
            if (!sval[sl]) x = VecZero<DT, VB>::apply(x);
        }
        st_vec_stream<VB>(outv + static_cast<int64_t>(sl) * a.row_bytes + v * VB, x);
    }
}

// General latest-k backward as a gather (no atomics, deterministic): the gradient
// of the write at sorted position q of stream s is the sum, over slots j < k whose
// write q+j lies in q's segment, of grad_vals[r, j] over the reads r of q's address
// whose latest earlier write is q+j (bucket q+j of the read tape).  Every write row is stored
// once, zeros for masked writes.  A group of 2^lshift lanes takes one write, a
// lane one VB-byte vector of the row (row_bytes / VB = 2^lshift).
template <typename KeyT, int DT, int VB>
__global__ void __launch_bounds__(256) k_lk_bwd_gather(LkArgs a, const KeyT* rkeys, const int32_t* rridx,
                                                       const int32_t* bstart, int lshift) {
    using E = Elem<DT>;
    using Acc = typename E::Acc;
    using V = typename E::T;
    constexpr int EPV = VB / static_cast<int>(sizeof(V));
    const int lane = threadIdx.x & 31;
    const uint32_t L = 1u << lshift;
    const uint32_t grp = static_cast<uint32_t>(lane) >> lshift, lig = static_cast<uint32_t>(lane) & (L - 1);
    const int64_t gpw = 32 >> lshift;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t T = a.T, S = a.B * a.C, D = a.D;
    const int k = static_cast<int>(a.k);
    const KeyT tmask = (static_cast<KeyT>(1) << a.tbits) - 1;
    const V* grad = static_cast<const V*>(a.grad);
    V* out = static_cast<V*>(a.out);
    for (int64_t gi = warp0 * gpw + grp; gi < S * T; gi += nwarps * gpw) {
        const int64_t s = gi / T, q = gi - s * T;
        const int64_t n_s = a.nvalid ? a.nvalid[s] : T;
        const KeyT* wk = static_cast<const KeyT*>(a.keys) + s * T;
        const KeyT kq = wk[q];
        const RowMap rows_of(s, T, a.C);
        const uint64_t orow = static_cast<uint64_t>(rows_of(kq & tmask));
        Acc acc[EPV];
#pragma unroll
        for (int e = 0; e < EPV; ++e) acc[e] = Acc(0);
        if (a.accumulate) {
            const uint4 prev = ld_vec<VB>(out + orow * D + lig * EPV);
            const V* pv0 = reinterpret_cast<const V*>(&prev);
#pragma unroll
            for (int e = 0; e < EPV; ++e) acc[e] = E::to_acc(pv0[e]);
        }
        if (q < n_s) {
            // slots j < jmax keep write q+j in q's segment: k write keys loaded 8 at a
            // time, independently
            const KeyT aq = kq >> a.tbits;
            int jmax = 0;
            for (int j0 = 0; j0 < k && jmax == j0; j0 += 8) {
                bool m[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int64_t qq = q + j0 + u;
                    m[u] = j0 + u < k && qq < n_s && (wk[qq < n_s ? qq : q] >> a.tbits) == aq;
                }
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    if (jmax == j0 + u && m[u]) ++jmax;
            }
            // the reads whose latest write is q .. q+jmax-1 are one contiguous run of
            // the read tape; a read of q's address takes slot (its latest write - q),
            // reads of other addresses in the run see no write of their own address
            const int32_t* bs = bstart + s * (T + 2);
            const KeyT* rk = rkeys + s * T;
            const int32_t* rr = rridx + s * T;
            const int32_t i0 = bs[q + 1], i1 = bs[q + 1 + jmax];
            for (int32_t i = i0; i < i1; i += 4) {
                uint32_t rrow[4];
                int jj[4];
                bool use[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const KeyT key = i + u < i1 ? rk[i + u] : KeyT(0);
                    rrow[u] = rows_of(key & tmask);
                    jj[u] = static_cast<int>((i + u < i1 ? rr[i + u] : 0) - q);
                    use[u] = i + u < i1 && (key >> a.tbits) == aq;
                }
                uint4 x[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    x[u] = use[u] ? ldg_vec<VB>(grad + (static_cast<uint64_t>(rrow[u]) * k + jj[u]) * D + lig * EPV)
                                  : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const V* xv = reinterpret_cast<const V*>(&x[u]);
#pragma unroll
                    for (int e = 0; e < EPV; ++e) acc[e] += E::to_acc(xv[e]);
                }
            }
        }
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        V* ov = reinterpret_cast<V*>(&o);
#pragma unroll
        for (int e = 0; e < EPV; ++e) ov[e] = E::from_acc(acc[e]);
        st_vec<VB>(out + orow * D + lig * EPV, o);
    }
}

// The same backward over chunks of the write tape: a CTA owns P consecutive
// sorted writes of one stream and first stages, with coalesced loads, their
// keys and the k after them, their bucket starts, and -- when the run of the
// read tape their buckets cover holds at most rcap reads -- those reads' keys
// and latest writes.  Each lane group then sums one write's gradient rows as
// k_lk_bwd_gather does, with no dependent global load before the gradient
// gathers (a chunk with a longer read run reads its read keys from global
// memory).  Same sums in the same order as k_lk_bwd_gather.
template <typename KeyT, int DT, int VB>
__global__ void __launch_bounds__(256) k_lk_bwd_chunk(LkArgs a, const KeyT* rkeys, const int32_t* rridx,
                                                      const int32_t* bstart, int lshift, int rcap) {
    using E = Elem<DT>;
    using Acc = typename E::Acc;
    using V = typename E::T;
    constexpr int EPV = VB / static_cast<int>(sizeof(V));
    extern __shared__ __align__(16) unsigned char smem[];
    const int P = a.P, k = static_cast<int>(a.k);
    const int64_t T = a.T, D = a.D;
    const int64_t s = blockIdx.x / a.nchunks;
    const int64_t q0 = (blockIdx.x % a.nchunks) * P;
    const int np = static_cast<int>((T - q0) < P ? (T - q0) : P);
    const int64_t n_s = a.nvalid ? a.nvalid[s] : T;
    KeyT* sk = reinterpret_cast<KeyT*>(smem);                              // [P + k] keys q0 ..
    int32_t* sb = reinterpret_cast<int32_t*>(sk + P + k);                  // [P + k + 1] bstart[q0 + 1 + m]
    KeyT* srk = reinterpret_cast<KeyT*>(sb + ((P + k + 2) & ~1));          // [rcap] read keys of the run
    int32_t* srr = reinterpret_cast<int32_t*>(srk + rcap);                 // [rcap] their latest writes
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const KeyT* wk = static_cast<const KeyT*>(a.keys) + s * T;
    const int32_t* bs = bstart + s * (T + 2);
    const KeyT* rk = rkeys + s * T;
    const int32_t* rr = rridx + s * T;
    for (int m = tid; m < np + k; m += 256) sk[m] = q0 + m < T ? wk[q0 + m] : KeyT(0);
    for (int m = tid; m <= np + k; m += 256) {
        const int64_t idx = q0 + 1 + m;
        sb[m] = bs[idx < T + 1 ? idx : T + 1];
    }
    __syncthreads();
    const int32_t ilo = sb[0], ihi = sb[np - 1 + k];  // the reads whose latest write is q0 .. q0+np-1+k-1
    const bool staged = ihi - ilo <= rcap;
    if (staged) {
        for (int e = tid; e < ihi - ilo; e += 256) {
            srk[e] = rk[ilo + e];
            srr[e] = rr[ilo + e];
        }
    }
    __syncthreads();
    const uint32_t L = 1u << lshift;
    const uint32_t grp = static_cast<uint32_t>(lane) >> lshift, lig = static_cast<uint32_t>(lane) & (L - 1);
    const int gpb = 8 * (32 >> lshift);
    const KeyT tmask = (static_cast<KeyT>(1) << a.tbits) - 1;
    const V* grad = static_cast<const V*>(a.grad);
    V* out = static_cast<V*>(a.out);
    const RowMap rows_of(s, T, a.C);
    for (int qq = warp * (32 >> lshift) + static_cast<int>(grp); qq < np; qq += gpb) {
        const int64_t q = q0 + qq;
        const KeyT kq = sk[qq];
        const uint64_t orow = static_cast<uint64_t>(rows_of(kq & tmask));
        Acc acc[EPV];
#pragma unroll
        for (int e = 0; e < EPV; ++e) acc[e] = Acc(0);
        if (a.accumulate) {
            const uint4 prev = ld_vec<VB>(out + orow * D + lig * EPV);
            const V* pv0 = reinterpret_cast<const V*>(&prev);
#pragma unroll
            for (int e = 0; e < EPV; ++e) acc[e] = E::to_acc(pv0[e]);
        }
        if (q < n_s) {
            // slots j < jmax keep write q+j in q's segment
            const KeyT aq = kq >> a.tbits;
            int jmax = 0;
            while (jmax < k && q + jmax < n_s && (sk[qq + jmax] >> a.tbits) == aq) ++jmax;
            const int32_t i0 = sb[qq], i1 = sb[qq + jmax];
            for (int32_t i = i0; i < i1; i += 4) {
                uint32_t rrow[4];
                int jj[4];
                bool use[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const bool in = i + u < i1;
                    const KeyT key = !in ? KeyT(0) : (staged ? srk[i + u - ilo] : rk[i + u]);
                    const int32_t rank = !in ? 0 : (staged ? srr[i + u - ilo] : rr[i + u]);
                    rrow[u] = rows_of(key & tmask);
                    jj[u] = static_cast<int>(rank - q);
                    use[u] = in && (key >> a.tbits) == aq;
                }
                uint4 x[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    x[u] = use[u] ? ldg_vec<VB>(grad + (static_cast<uint64_t>(rrow[u]) * k + jj[u]) * D + lig * EPV)
                                  : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const V* xv = reinterpret_cast<const V*>(&x[u]);
#pragma unroll
                    for (int e = 0; e < EPV; ++e) acc[e] += E::to_acc(xv[e]);
                }
            }
        }
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        V* ov = reinterpret_cast<V*>(&o);
#pragma unroll
        for (int e = 0; e < EPV; ++e) ov[e] = E::from_acc(acc[e]);
        st_vec<VB>(out + orow * D + lig * EPV, o);
    }
}

inline size_t lk_bwd_chunk_smem(int P, int64_t k, int rcap, size_t key_bytes) {
    return (static_cast<size_t>(P) + static_cast<size_t>(k)) * key_bytes +
           (static_cast<size_t>(P) + static_cast<size_t>(k) + 2) * 4 + static_cast<size_t>(rcap) * (key_bytes + 4) + 16;
}

// The same gather for rows that do not split into 2^m <= 32 vectors (odd
// widths, rows beyond 512 bytes): one warp per write, its lanes over the row's
// elements 32 apart.  Each element sums the same reads in the same order as
// k_lk_bwd_gather, so every row shape is deterministic (no atomics).
template <typename KeyT, int DT>
__global__ void __launch_bounds__(256) k_lk_bwd_gather_rows(LkArgs a, const KeyT* rkeys, const int32_t* rridx,
                                                            const int32_t* bstart) {
    using E = Elem<DT>;
    using Acc = typename E::Acc;
    using V = typename E::T;
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t T = a.T, S = a.B * a.C, D = a.D;
    const int k = static_cast<int>(a.k);
    const KeyT tmask = (static_cast<KeyT>(1) << a.tbits) - 1;
    const V* grad = static_cast<const V*>(a.grad);
    V* out = static_cast<V*>(a.out);
    for (int64_t gi = warp0; gi < S * T; gi += nwarps) {
        const int64_t s = gi / T, q = gi - s * T;
        const int64_t n_s = a.nvalid ? a.nvalid[s] : T;
        const KeyT* wk = static_cast<const KeyT*>(a.keys) + s * T;
        const KeyT kq = wk[q];
        const RowMap rows_of(s, T, a.C);
        const uint64_t orow = static_cast<uint64_t>(rows_of(kq & tmask));
        int32_t i0 = 0, i1 = 0;
        const KeyT aq = kq >> a.tbits;
        if (q < n_s) {
            int jmax = 0;  // slots j < jmax keep write q+j in q's segment
            while (jmax < k && q + jmax < n_s && (wk[q + jmax] >> a.tbits) == aq) ++jmax;
            const int32_t* bs = bstart + s * (T + 2);
            i0 = bs[q + 1];
            i1 = bs[q + 1 + jmax];
        }
        const KeyT* rk = rkeys + s * T;
        const int32_t* rr = rridx + s * T;
        for (int64_t d = lane; d < D; d += 32) {
            Acc acc = a.accumulate ? E::to_acc(out[orow * D + d]) : Acc(0);
            for (int32_t i = i0; i < i1; ++i) {
                const KeyT key = rk[i];
                if ((key >> a.tbits) != aq) continue;
                const int jj = static_cast<int>(rr[i] - q);
                acc += E::to_acc(grad[(static_cast<uint64_t>(rows_of(key & tmask)) * k + jj) * D + d]);
            }
            out[orow * D + d] = E::from_acc(acc);
        }
    }
}


}  // namespace ravel
