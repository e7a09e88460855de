// segsum.cuh -- causal segmented sum over the sorted event tape.
//
// Reference: ravel_lm/ravel_memory.py:216-241 sorts the payloads into tape
// order, takes a global cumsum, subtracts the cumsum before each segment start
// and gathers it at every read's latest write.  Here the tape is scanned once
// as a segmented scan (a segment = one (stream, address) group) with
// decoupled look-back between chunks:
//
//   * CTAs take chunk tickets from an atomic counter, so every chunk a CTA
//     waits on already belongs to a running CTA (forward progress);
//   * a chunk publishes its aggregate (flag 1) or, once known, its inclusive
//     prefix (flag 2); a chunk containing a segment start publishes its
//     inclusive value at once, so look-back stops at the nearest segment start;
//   * every wait is bounded: after SPIN_LIMIT polls the kernel flags
//     RAVEL_DEVERR_SPIN in the device error word and continues with a zero
//     carry instead of hanging.
//
// One kernel serves four uses (reverse = scan from the end of each stream):
//   forward, aliased reads:  exclusive, gather payload rows by time, scatter
//                            sums by time, write the mask
//   backward, aliased reads: exclusive + reverse over grad_sums rows
//   general forward:         inclusive into a float tape buffer (then gather)
//   general backward:        inclusive + reverse over the tape buffer that
//                            read gradients were added into
#pragma once

#include <type_traits>

#include "common.cuh"
#include "latestk.cuh"

namespace ravel {

constexpr int SCAN_THREADS = 256;
constexpr unsigned SPIN_LIMIT = 1u << 22;

template <typename Acc>
struct ScanArgs {
    const void* keys;        // [S][T]
    const int* nvalid;       // [S] or null (all T)
    int64_t B, T, C, D;
    int tbits;
    const void* in;          // in_sorted ? Acc [S*T, D] : dtype [N, D]
    void* out;               // out_sorted ? Acc [S*T, D] : dtype [N, D]
    uint8_t* out_mask;       // optional [N]: 1 unless the position starts its segment
    int in_sorted, out_sorted, inclusive, reverse;
    int P;                   // positions per chunk
    int parts;               // sequential parts per chunk (threads per column)
    int64_t nchunks;         // chunks per stream
    unsigned* flags;         // [S*nchunks], zeroed before launch
    unsigned* ticket;        // zeroed before launch
    Acc* agg;                // [S*nchunks, D]
    Acc* incl;               // [S*nchunks, D]
    FastDiv fd_d;
    FastDiv fd_vpr;          // 16-byte vectors per staged row
};

template <typename KeyT, int DT, bool VEC>
__global__ void __launch_bounds__(SCAN_THREADS) k_segscan(ScanArgs<typename Elem<DT>::Acc> a) {
    using E = Elem<DT>;
    using Acc = typename E::Acc;
    using V = typename E::T;
    extern __shared__ __align__(16) unsigned char smem[];
    const int P = a.P;
    const int D = static_cast<int>(a.D);
    Acc* rows = reinterpret_cast<Acc*>(smem);                      // [P][D]
    Acc* pagg = rows + static_cast<int64_t>(P) * D;                // [parts][D]
    Acc* carry = pagg + static_cast<int64_t>(a.parts) * D;         // [D]
    uintptr_t tail = reinterpret_cast<uintptr_t>(carry + D);
    tail = (tail + 15) & ~static_cast<uintptr_t>(15);
    int64_t* srow = reinterpret_cast<int64_t*>(tail);              // [P] flat row or (flat row, tape index)
    uint64_t* sadr = reinterpret_cast<uint64_t*>(srow + P);        // [P]
    uint8_t* sstart = reinterpret_cast<uint8_t*>(sadr + P);        // [P]
    __shared__ unsigned s_ticket;
    __shared__ int s_phs[SCAN_THREADS];
    __shared__ int s_first_start;

    const int tid = threadIdx.x;
    if (tid == 0) s_ticket = atomicAdd(a.ticket, 1u);
    if (tid == 0) s_first_start = P;
    __syncthreads();
    const int64_t L = s_ticket;
    const int64_t s = L / a.nchunks;
    const int64_t ch = L % a.nchunks;
    const int64_t T = a.T, C = a.C;
    const int64_t n_s = a.nvalid ? a.nvalid[s] : T;
    const int64_t i0 = ch * P;
    if (i0 >= n_s) return;  // nothing here; later chunks of this stream are empty too
    const int np = static_cast<int>((n_s - i0) < P ? (n_s - i0) : P);
    const KeyT* keys = static_cast<const KeyT*>(a.keys) + s * T;
    const KeyT tmask = (static_cast<KeyT>(1) << a.tbits) - 1;

    const RowMap rows_of(s, T, C);
    // tape positions in scan order
    for (int i = tid; i < np; i += SCAN_THREADS) {
        const int64_t si = i0 + i;
        const int64_t p = a.reverse ? (n_s - 1 - si) : si;
        const KeyT key = keys[p];
        sadr[i] = static_cast<uint64_t>(key >> a.tbits);
        srow[i] = rows_of(key & tmask);
        if (a.in_sorted || a.out_sorted) srow[i] = (srow[i] << 32) | p;  // pack (flat row, tape index)
    }
    __syncthreads();
    for (int i = tid; i < np; i += SCAN_THREADS) {
        uint64_t prev;
        bool has_prev = true;
        if (i > 0) prev = sadr[i - 1];
        else if (i0 > 0) {
            const int64_t si = i0 - 1;
            const int64_t p = a.reverse ? (n_s - 1 - si) : si;
            prev = static_cast<uint64_t>(keys[p] >> a.tbits);
        } else { prev = 0; has_prev = false; }
        const bool st = !has_prev || prev != sadr[i];
        sstart[i] = st;
        if (st) atomicMin(&s_first_start, i);
    }
    // stage rows as Acc
    const bool packed = a.in_sorted || a.out_sorted;
    if (a.in_sorted) {
        const Acc* in = static_cast<const Acc*>(a.in) + s * T * D;
        for (uint32_t e = tid; e < static_cast<uint32_t>(np * D); e += SCAN_THREADS) {
            uint32_t i, d;
            a.fd_d.divmod(e, i, d);
            const int64_t p = srow[i] & 0xffffffffll;
            rows[e] = in[p * D + d];
        }
    } else {
        const V* in = static_cast<const V*>(a.in);
        if constexpr (VEC) {
            constexpr int EPV = 16 / sizeof(V);
            const uint32_t dv = static_cast<uint32_t>(D / EPV);
            for (uint32_t e = tid; e < static_cast<uint32_t>(np) * dv; e += SCAN_THREADS) {
                const uint32_t i = e / dv, v = e % dv;
                const int64_t fr = packed ? (srow[i] >> 32) : srow[i];
                const uint4 raw = ld_nc_v4(in + fr * D + v * EPV);
                const V* x = reinterpret_cast<const V*>(&raw);
#pragma unroll
                for (int q = 0; q < EPV; ++q) rows[i * D + v * EPV + q] = E::to_acc(x[q]);
            }
        } else {
            for (uint32_t e = tid; e < static_cast<uint32_t>(np * D); e += SCAN_THREADS) {
                uint32_t i, d;
                a.fd_d.divmod(e, i, d);
                const int64_t fr = packed ? (srow[i] >> 32) : srow[i];
                rows[e] = E::to_acc(in[fr * D + d]);
            }
        }
    }
    __syncthreads();

    // sequential scan of each (part, column)
    const int ncol = D < 1 ? 1 : (D < SCAN_THREADS ? D : SCAN_THREADS);
    const int parts = a.parts;
    const int PP = (np + parts - 1) / parts;
    const int part = tid / ncol;
    if (part < parts) {
        const int b0 = part * PP;
        const int b1 = (b0 + PP) < np ? (b0 + PP) : np;
        int phs = 0;
        for (int col = tid % ncol; col < D; col += ncol) {
            Acc run = Acc(0);
            for (int i = b0; i < b1; ++i) {
                if (sstart[i]) { run = Acc(0); phs = 1; }
                const Acc v = rows[i * D + col];
                if (a.inclusive) { run += v; rows[i * D + col] = run; }
                else { rows[i * D + col] = run; run += v; }
            }
            pagg[part * D + col] = run;
        }
        if (tid % ncol == 0) s_phs[part] = phs;
    }
    __syncthreads();
    // carry between parts, and the chunk aggregate
    if (part < parts) {
        for (int col = tid % ncol; col < D; col += ncol) {
            Acc cin = Acc(0);
            for (int q = 0; q < part; ++q) cin = s_phs[q] ? pagg[q * D + col] : cin + pagg[q * D + col];
            const int b0 = part * PP;
            const int b1 = (b0 + PP) < np ? (b0 + PP) : np;
            for (int i = b0; i < b1 && !sstart[i]; ++i) rows[i * D + col] += cin;
            if (part == parts - 1) carry[col] = s_phs[part] ? pagg[part * D + col] : cin + pagg[part * D + col];
        }
    }
    __syncthreads();
    // carry[] now holds the chunk aggregate (trailing segment sum)
    const int first_start = s_first_start;
    const bool chunk_has_start = first_start < np;
    if (chunk_has_start) {
        // inclusive prefix == aggregate: publish it at once
        for (int col = tid; col < D; col += SCAN_THREADS) a.incl[L * D + col] = carry[col];
        __threadfence();
        __syncthreads();
        if (tid == 0) st_release(a.flags + L, 2u);
    } else {
        for (int col = tid; col < D; col += SCAN_THREADS) a.agg[L * D + col] = carry[col];
        __threadfence();
        __syncthreads();
        if (tid == 0) st_release(a.flags + L, 1u);
    }
    if (first_start > 0) {
        // look back (chunk 0 of a stream always starts a segment, so ch >= 1 here)
        if (tid < 32) {
            // pagg (free after the part carries) accumulates the look-back carry;
            // lane l owns columns l, l+32, ...
            const int lane = tid;
            for (int col = lane; col < D; col += 32) pagg[col] = Acc(0);
            int64_t j = L - 1;
            while (true) {
                unsigned f;
                unsigned spins = 0;
                bool bail = false;
                while ((f = ld_acquire(a.flags + j)) == 0u) {
                    if (++spins > SPIN_LIMIT) { bail = true; break; }
                    __nanosleep(64);
                }
                if (bail) {
                    if (lane == 0) flag_error(RAVEL_DEVERR_SPIN);
                    break;
                }
                const Acc* src = (f == 2u) ? a.incl + j * D : a.agg + j * D;
                for (int col = lane; col < D; col += 32) pagg[col] += src[col];
                if (f == 2u) break;
                --j;
            }
        }
        __syncthreads();
        if (!chunk_has_start) {
            for (int col = tid; col < D; col += SCAN_THREADS) a.incl[L * D + col] = pagg[col] + carry[col];
            __threadfence();
            __syncthreads();
            if (tid == 0) st_release(a.flags + L, 2u);
        }
        // apply the look-back carry to positions before the first segment start
        for (uint32_t e = tid; e < static_cast<uint32_t>(first_start * D); e += SCAN_THREADS) {
            uint32_t i, d;
            a.fd_d.divmod(e, i, d);
            rows[e] += pagg[d];
        }
        __syncthreads();
    }

    // write out
    if (a.out_sorted) {
        Acc* out = static_cast<Acc*>(a.out) + s * T * D;
        for (uint32_t e = tid; e < static_cast<uint32_t>(np * D); e += SCAN_THREADS) {
            uint32_t i, d;
            a.fd_d.divmod(e, i, d);
            out[(srow[i] & 0xffffffffll) * D + d] = rows[e];
        }
    } else {
        V* out = static_cast<V*>(a.out);
        if constexpr (VEC) {
            constexpr int EPV = 16 / sizeof(V);
            const uint32_t dv = static_cast<uint32_t>(D / EPV);
            for (uint32_t e = tid; e < static_cast<uint32_t>(np) * dv; e += SCAN_THREADS) {
                const uint32_t i = e / dv, v = e % dv;
                const int64_t fr = packed ? (srow[i] >> 32) : srow[i];
                uint4 raw;
                V* x = reinterpret_cast<V*>(&raw);
#pragma unroll
                for (int q = 0; q < EPV; ++q) x[q] = E::from_acc(rows[i * D + v * EPV + q]);
                *reinterpret_cast<uint4*>(out + fr * D + v * EPV) = raw;
            }
        } else {
            for (uint32_t e = tid; e < static_cast<uint32_t>(np * D); e += SCAN_THREADS) {
                uint32_t i, d;
                a.fd_d.divmod(e, i, d);
                const int64_t fr = packed ? (srow[i] >> 32) : srow[i];
                out[fr * D + d] = E::from_acc(rows[e]);
            }
        }
        if (a.out_mask) {
            for (int i = tid; i < np; i += SCAN_THREADS) {
                const int64_t fr = packed ? (srow[i] >> 32) : srow[i];
                a.out_mask[fr] = sstart[i] ? 0 : 1;
            }
        }
    }
}

// ------------------------------------------------------------------ warp-register scan
// The main scan kernel.  A CTA of 8 warps takes a chunk of 8*R tape positions
// (one ticket); warp w owns R consecutive positions and lane l owns columns
// [l*EL, l*EL+EL) of every row, so each row moves as one coalesced warp access.
// A warp issues all R row loads at once into registers and scans them with a
// zero carry (pass 1): every position from the warp's first segment start on
// is final and is stored at once, and the scan ends with the warp's trailing
// segment sum.  Warp 0 folds the warp sums into the chunk aggregate, publishes
// it and, if the chunk's first position continues a segment, looks back for
// the chunk carry.  Only warps whose head positions (before their first start)
// need a carry rescan them (pass 2); of those, only warps 0..m (m = first warp
// with a start) wait for the look-back, on a named barrier.  Many small CTAs per
// SM keep loads, look-backs and stores of different chunks overlapped.
constexpr int SCANW_WARPS = 8;

template <int N> struct RawWords { uint32_t w[(N + 3) / 4]; };

// Load / store EL elements of type X at p (element-aligned to EL*sizeof(X)).
template <typename X, int EL>
__device__ __forceinline__ RawWords<EL * sizeof(X)> ld_frag(const X* p) {
    RawWords<EL * sizeof(X)> r;
    constexpr int B = EL * sizeof(X);
    if constexpr (B == 2) r.w[0] = *reinterpret_cast<const uint16_t*>(p);
    else if constexpr (B == 4) r.w[0] = *reinterpret_cast<const uint32_t*>(p);
    else if constexpr (B == 8) { const uint2 v = *reinterpret_cast<const uint2*>(p); r.w[0] = v.x; r.w[1] = v.y; }
    else {
#pragma unroll
        for (int q = 0; q < B / 16; ++q) {
            const uint4 v = ld_nc_v4(reinterpret_cast<const char*>(p) + 16 * q);
            r.w[4 * q] = v.x; r.w[4 * q + 1] = v.y; r.w[4 * q + 2] = v.z; r.w[4 * q + 3] = v.w;
        }
    }
    return r;
}

template <typename X, int EL>
__device__ __forceinline__ RawWords<EL * sizeof(X)> ld_frag_smem(const X* p) {
    RawWords<EL * sizeof(X)> r;
    constexpr int B = EL * sizeof(X);
    if constexpr (B == 2) r.w[0] = *reinterpret_cast<const uint16_t*>(p);
    else if constexpr (B == 4) r.w[0] = *reinterpret_cast<const uint32_t*>(p);
    else if constexpr (B == 8) { const uint2 v = *reinterpret_cast<const uint2*>(p); r.w[0] = v.x; r.w[1] = v.y; }
    else {
#pragma unroll
        for (int q = 0; q < B / 16; ++q) {
            const uint4 v = *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(p) + 16 * q);
            r.w[4 * q] = v.x; r.w[4 * q + 1] = v.y; r.w[4 * q + 2] = v.z; r.w[4 * q + 3] = v.w;
        }
    }
    return r;
}

template <typename X, int EL>
__device__ __forceinline__ void st_frag(X* p, const RawWords<EL * sizeof(X)>& r) {
    constexpr int B = EL * sizeof(X);
    if constexpr (B == 2) *reinterpret_cast<uint16_t*>(p) = static_cast<uint16_t>(r.w[0]);
    else if constexpr (B == 4) *reinterpret_cast<uint32_t*>(p) = r.w[0];
    else if constexpr (B == 8) *reinterpret_cast<uint2*>(p) = make_uint2(r.w[0], r.w[1]);
    else {
#pragma unroll
        for (int q = 0; q < B / 16; ++q)
            *reinterpret_cast<uint4*>(reinterpret_cast<char*>(p) + 16 * q) =
                make_uint4(r.w[4 * q], r.w[4 * q + 1], r.w[4 * q + 2], r.w[4 * q + 3]);
    }
}

template <typename X, typename Acc, int EL>
__device__ __forceinline__ Acc frag_get(const RawWords<EL * sizeof(X)>& r, int q) {
    const X* x = reinterpret_cast<const X*>(&r.w[0]);
    if constexpr (sizeof(X) == sizeof(Acc) && std::is_same<X, Acc>::value) return x[q];
    else return static_cast<Acc>(Elem<sizeof(X) == 2 ? (std::is_same<X, __half>::value ? RAVEL_F16 : RAVEL_BF16)
                                                     : RAVEL_F32>::to_acc(x[q]));
}

template <typename X, typename Acc>
__device__ __forceinline__ X acc_to(Acc v) {
    if constexpr (std::is_same<X, Acc>::value) return v;
    else if constexpr (std::is_same<X, float>::value) return static_cast<float>(v);
    else if constexpr (std::is_same<X, __half>::value) return __float2half_rn(static_cast<float>(v));
    else return __float2bfloat16_rn(static_cast<float>(v));
}

// Decoupled look-back over a window of 32 predecessors at a time: lane i polls
// the flag of chunk j-i (bounded wait), the nearest chunk with an inclusive
// prefix (flag 2) ends the walk, and the warp then adds the published vectors
// of chunks j .. that chunk, lanes over columns.  A chain of n aggregate-only
// predecessors (a long segment) costs n/32 flag round trips instead of n.
// `jmin` is the first chunk of the stream, which always publishes flag 2.
template <typename Acc, int EL>
__device__ __forceinline__ void windowed_lookback(unsigned* flags, const Acc* agg, const Acc* incl, int64_t j,
                                                  int64_t jmin, uint32_t D, int lane, bool active, uint32_t col,
                                                  Acc (&cin)[EL]) {
    while (true) {
        const int64_t idx = j - lane;
        unsigned f = 2u;  // slots before the stream start are never reached
        if (idx >= jmin) {
            unsigned spins = 0;
            while ((f = ld_acquire(flags + idx)) == 0u) {
                if (++spins > SPIN_LIMIT) { f = 3u; break; }
                __nanosleep(32);
            }
            if (f == 3u) flag_error(RAVEL_DEVERR_SPIN);
        }
        const unsigned term = __ballot_sync(0xffffffffu, f >= 2u);
        int stop = term ? __ffs(term) - 1 : 31;
        // never step past the stream's first chunk or a timed-out slot
        const unsigned bad = __ballot_sync(0xffffffffu, (j - lane) < jmin || f == 3u);
        if (bad) {
            const int b = __ffs(bad) - 1;
            if (b <= stop) stop = b - 1 + ((j - b) >= jmin && __shfl_sync(0xffffffffu, f, b) == 2u ? 1 : 0);
        }
        // add the published vectors of chunks j .. j-stop, eight loads in flight
        for (int c0 = 0; c0 <= stop; c0 += 8) {
            Acc tmp[8][EL];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = c0 + u;
                const unsigned fc = __shfl_sync(0xffffffffu, f, c & 31);
                const Acc* src = (fc == 2u) ? incl + (j - c) * D : agg + (j - c) * D;
#pragma unroll
                for (int q = 0; q < EL; ++q) tmp[u][q] = (c <= stop && active) ? src[col + q] : Acc(0);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
#pragma unroll
                for (int q = 0; q < EL; ++q) cin[q] += tmp[u][q];
            }
        }
        if (term || bad) return;
        j -= 32;
    }
}

// Named barrier over the first `threads` threads of the CTA (ID 1; ID 0 is
// __syncthreads).
__device__ __forceinline__ void named_barrier(int threads) {
    asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

template <typename KeyT, int DT, int EL, bool IN_SORTED, bool OUT_SORTED, int R>
__global__ void __launch_bounds__(SCANW_WARPS * 32) k_segscan_w(ScanArgs<typename Elem<DT>::Acc> a) {
    using E = Elem<DT>;
    using Acc = typename E::Acc;
    using V = typename E::T;
    using InT = typename std::conditional<IN_SORTED, Acc, V>::type;
    using OutT = typename std::conditional<OUT_SORTED, Acc, V>::type;
    constexpr int NW = SCANW_WARPS;
    constexpr int P = NW * R;
    extern __shared__ __align__(16) unsigned char smem[];
    const uint32_t D = static_cast<uint32_t>(a.D);
    Acc* wagg = reinterpret_cast<Acc*>(smem);  // [NW][D] trailing-segment sums of the warps
    Acc* carry = wagg + NW * D;                // [D] chunk carry-in
    __shared__ unsigned s_ticket;
    __shared__ unsigned s_startmask[NW];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) s_ticket = atomicAdd(a.ticket, 1u);
    __syncthreads();
    const int64_t L = s_ticket;
    const int64_t s = L / a.nchunks;
    const int64_t ch = L % a.nchunks;
    const int64_t T = a.T, C = a.C;
    const int64_t n_s = a.nvalid ? a.nvalid[s] : T;
    const int64_t i0 = ch * P;
    if (i0 >= n_s) return;  // beyond this stream's tape; no later chunk waits on it
    const KeyT* keys = static_cast<const KeyT*>(a.keys) + s * T;
    const KeyT tmask = (static_cast<KeyT>(1) << a.tbits) - 1;
    const int64_t w0 = i0 + warp * R;
    const int nv = static_cast<int>(n_s - w0 < 0 ? 0 : (n_s - w0 < R ? n_s - w0 : R));

    // keys -> flat payload row, tape index, segment start
    uint32_t my_flat = 0, my_tix = 0;
    bool my_start = false;
    if (lane < nv) {
        const int64_t si = w0 + lane;
        const int64_t p = a.reverse ? (n_s - 1 - si) : si;
        const KeyT key = keys[p];
        my_flat = RowMap(s, T, C)(key & tmask);
        my_tix = static_cast<uint32_t>(s * T + p);
        if (si == 0) {
            my_start = true;
        } else {
            const int64_t pp = a.reverse ? (n_s - si) : (si - 1);
            my_start = (keys[pp] >> a.tbits) != (key >> a.tbits);
        }
    }
    const unsigned startmask = __ballot_sync(0xffffffffu, my_start);
    const int first = startmask ? __ffs(startmask) - 1 : R;  // positions [0, first) continue a segment
    const uint32_t my_in = IN_SORTED ? my_tix : my_flat;
    const uint32_t my_out = OUT_SORTED ? my_tix : my_flat;
    const bool active = static_cast<uint32_t>(lane * EL) < D;
    const uint32_t col = static_cast<uint32_t>(lane * EL);
    const InT* in = static_cast<const InT*>(a.in);
    OutT* out = static_cast<OutT*>(a.out);

    RawWords<EL * sizeof(InT)> x[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const uint32_t row = __shfl_sync(0xffffffffu, my_in, i);
        if (i < nv && active) x[i] = ld_frag<InT, EL>(in + static_cast<uint64_t>(row) * D + col);
    }

    // Pass 1: scan with zero carry.  Positions from the warp's first segment
    // start on are final and stored now; `run` ends as the warp's trailing
    // segment sum.
    Acc run[EL];
#pragma unroll
    for (int q = 0; q < EL; ++q) run[q] = Acc(0);
#pragma unroll
    for (int i = 0; i < R; ++i) {
        if (i < nv) {
            const bool st = (startmask >> i) & 1u;
            const uint32_t row = __shfl_sync(0xffffffffu, my_out, i);
            RawWords<EL * sizeof(OutT)> o;
            OutT* ov = reinterpret_cast<OutT*>(&o.w[0]);
#pragma unroll
            for (int q = 0; q < EL; ++q) {
                if (st) run[q] = Acc(0);
                const Acc v = frag_get<InT, Acc, EL>(x[i], q);
                if (a.inclusive) { run[q] += v; ov[q] = acc_to<OutT, Acc>(run[q]); }
                else { ov[q] = acc_to<OutT, Acc>(run[q]); run[q] += v; }
            }
            if (i >= first && active) st_frag<OutT, EL>(out + static_cast<uint64_t>(row) * D + col, o);
        }
    }
    if (active) {
#pragma unroll
        for (int q = 0; q < EL; ++q) wagg[warp * D + col + q] = run[q];
    }
    if (lane == 0) s_startmask[warp] = startmask;
    if (a.out_mask != nullptr && lane < nv) a.out_mask[my_flat] = my_start ? 0 : 1;
    __syncthreads();

    // m = first warp of the chunk that starts a segment (NW if none)
    int m = NW;
#pragma unroll
    for (int w = NW - 1; w >= 0; --w) if (s_startmask[w] != 0u) m = w;
    const bool head_continues = (s_startmask[0] & 1u) == 0u;  // chunk head continues a segment
    const int waiters = (m < NW ? m : NW - 1) + 1;          // warps 0..m need the chunk carry

    if (warp == 0) {
        // chunk aggregate: fold the warps' trailing sums in order
        Acc cagg[EL];
#pragma unroll
        for (int q = 0; q < EL; ++q) cagg[q] = Acc(0);
        for (int w = 0; w < NW; ++w) {
            const bool hs = s_startmask[w] != 0u;
            if (active) {
#pragma unroll
                for (int q = 0; q < EL; ++q) {
                    const Acc v = wagg[w * D + col + q];
                    cagg[q] = hs ? v : cagg[q] + v;
                }
            }
        }
        const bool chunk_hs = m < NW;
        Acc* dst = chunk_hs ? a.incl : a.agg;
        if (active) {
#pragma unroll
            for (int q = 0; q < EL; ++q) dst[L * D + col + q] = cagg[q];
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release(a.flags + L, chunk_hs ? 2u : 1u);
        if (head_continues) {
            Acc cin[EL];
#pragma unroll
            for (int q = 0; q < EL; ++q) cin[q] = Acc(0);
            windowed_lookback<Acc, EL>(a.flags, a.agg, a.incl, L - 1, L - ch, D, lane, active, col, cin);
            if (!chunk_hs) {
                if (active) {
#pragma unroll
                    for (int q = 0; q < EL; ++q) a.incl[L * D + col + q] = cin[q] + cagg[q];
                }
                __threadfence();
                __syncwarp();
                if (lane == 0) st_release(a.flags + L, 2u);
            }
            if (active) {
#pragma unroll
                for (int q = 0; q < EL; ++q) carry[col + q] = cin[q];
            }
        }
    }
    // warps 0..m wait for the chunk carry (only when the chunk head continues)
    if (head_continues && warp < waiters && waiters > 1) named_barrier(waiters * 32);

    // Pass 2: the warp's head positions [0, first) with their carry-in.
    if (first > 0 && nv > 0) {
        Acc cin[EL];
#pragma unroll
        for (int q = 0; q < EL; ++q) cin[q] = Acc(0);
        bool any_start = false;
        for (int w = 0; w < warp; ++w) {
            const bool hs = s_startmask[w] != 0u;
            any_start |= hs;
            if (active) {
#pragma unroll
                for (int q = 0; q < EL; ++q) {
                    const Acc v = wagg[w * D + col + q];
                    cin[q] = hs ? v : cin[q] + v;
                }
            }
        }
        if (!any_start && head_continues && active) {
#pragma unroll
            for (int q = 0; q < EL; ++q) cin[q] += carry[col + q];
        }
#pragma unroll
        for (int q = 0; q < EL; ++q) run[q] = cin[q];
#pragma unroll
        for (int i = 0; i < R; ++i) {
            if (i < first && i < nv) {
                const uint32_t row = __shfl_sync(0xffffffffu, my_out, i);
                RawWords<EL * sizeof(OutT)> o;
                OutT* ov = reinterpret_cast<OutT*>(&o.w[0]);
#pragma unroll
                for (int q = 0; q < EL; ++q) {
                    const Acc v = frag_get<InT, Acc, EL>(x[i], q);
                    if (a.inclusive) { run[q] += v; ov[q] = acc_to<OutT, Acc>(run[q]); }
                    else { ov[q] = acc_to<OutT, Acc>(run[q]); run[q] += v; }
                }
                if (active) st_frag<OutT, EL>(out + static_cast<uint64_t>(row) * D + col, o);
            }
        }
    }
}

template <typename X, int EL>
__device__ __forceinline__ void st_frag_smem(X* p, const RawWords<EL * sizeof(X)>& r) {
    constexpr int B = EL * sizeof(X);
    if constexpr (B == 2) *reinterpret_cast<uint16_t*>(p) = static_cast<uint16_t>(r.w[0]);
    else if constexpr (B == 4) *reinterpret_cast<uint32_t*>(p) = r.w[0];
    else if constexpr (B == 8) *reinterpret_cast<uint2*>(p) = make_uint2(r.w[0], r.w[1]);
    else {
#pragma unroll
        for (int q = 0; q < B / 16; ++q)
            *reinterpret_cast<uint4*>(reinterpret_cast<char*>(p) + 16 * q) =
                make_uint4(r.w[4 * q], r.w[4 * q + 1], r.w[4 * q + 2], r.w[4 * q + 3]);
    }
}

// Copy staged result rows [r0, r1) of the chunk to their output rows, 16 bytes
// per lane (rows are whole multiples of 16 bytes).
template <typename AccT, typename X>
__device__ __forceinline__ void store_rows(const ScanArgs<AccT>& a, const X* rows, const uint32_t* s_out, int r0,
                                           int r1, uint32_t rb, X* out, int lane) {
    const uint32_t vpr = rb / 16;
    const uint32_t n = static_cast<uint32_t>(r1 > r0 ? r1 - r0 : 0) * vpr;
    for (uint32_t e = lane; e < n; e += 32) {
        uint32_t r, v;
        a.fd_vpr.divmod(e, r, v);
        const uint4 val = *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(rows) +
                                                          static_cast<size_t>(r0 + r) * rb + v * 16);
        *reinterpret_cast<uint4*>(reinterpret_cast<char*>(out) + static_cast<uint64_t>(s_out[r0 + r]) * rb + v * 16) =
            val;
    }
}

// ------------------------------------------------------------------ lane fragments in shared memory
// 32-bit shared-memory addressing and paired 16-bit conversions for the scan's
// inner loop (one tape position per iteration, lanes over columns).
template <int B>
__device__ __forceinline__ RawWords<B> lds_words(uint32_t addr) {
    RawWords<B> r;
    if constexpr (B == 2) {
        unsigned short h;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(addr));
        r.w[0] = h;
    } else if constexpr (B == 4) {
        asm volatile("ld.shared.b32 %0, [%1];" : "=r"(r.w[0]) : "r"(addr));
    } else if constexpr (B == 8) {
        asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(r.w[0]), "=r"(r.w[1]) : "r"(addr));
    } else {
#pragma unroll
        for (int q = 0; q < B / 16; ++q)
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(r.w[4 * q]), "=r"(r.w[4 * q + 1]), "=r"(r.w[4 * q + 2]), "=r"(r.w[4 * q + 3])
                         : "r"(addr + 16 * q));
    }
    return r;
}

template <int B>
__device__ __forceinline__ void sts_words(uint32_t addr, const RawWords<B>& r) {
    if constexpr (B == 2) {
        const unsigned short h = static_cast<unsigned short>(r.w[0]);
        asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(h) : "memory");
    } else if constexpr (B == 4) {
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(r.w[0]) : "memory");
    } else if constexpr (B == 8) {
        asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(addr), "r"(r.w[0]), "r"(r.w[1]) : "memory");
    } else {
#pragma unroll
        for (int q = 0; q < B / 16; ++q)
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr + 16 * q), "r"(r.w[4 * q]),
                         "r"(r.w[4 * q + 1]), "r"(r.w[4 * q + 2]), "r"(r.w[4 * q + 3])
                         : "memory");
    }
}

// Unpack EL elements of X held in raw words into accumulators.
template <typename X, typename Acc, int EL>
__device__ __forceinline__ void unpack(const RawWords<EL * sizeof(X)>& r, Acc (&v)[EL]) {
    if constexpr (std::is_same<X, __nv_bfloat16>::value && EL % 2 == 0) {
#pragma unroll
        for (int q = 0; q < EL / 2; ++q) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.w[q]));
            v[2 * q] = f.x; v[2 * q + 1] = f.y;
        }
    } else if constexpr (std::is_same<X, __half>::value && EL % 2 == 0) {
#pragma unroll
        for (int q = 0; q < EL / 2; ++q) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&r.w[q]));
            v[2 * q] = f.x; v[2 * q + 1] = f.y;
        }
    } else {
#pragma unroll
        for (int q = 0; q < EL; ++q) v[q] = frag_get<X, Acc, EL>(r, q);
    }
}

// Pack EL accumulators into raw words of X (round to nearest even).
template <typename X, typename Acc, int EL>
__device__ __forceinline__ RawWords<EL * sizeof(X)> pack(const Acc (&v)[EL]) {
    RawWords<EL * sizeof(X)> r;
    if constexpr (std::is_same<X, __nv_bfloat16>::value && EL % 2 == 0) {
#pragma unroll
        for (int q = 0; q < EL / 2; ++q) {
            const __nv_bfloat162 h = __float22bfloat162_rn(make_float2(v[2 * q], v[2 * q + 1]));
            r.w[q] = *reinterpret_cast<const uint32_t*>(&h);
        }
    } else if constexpr (std::is_same<X, __half>::value && EL % 2 == 0) {
#pragma unroll
        for (int q = 0; q < EL / 2; ++q) {
            const __half2 h = __float22half2_rn(make_float2(v[2 * q], v[2 * q + 1]));
            r.w[q] = *reinterpret_cast<const uint32_t*>(&h);
        }
    } else {
        X* x = reinterpret_cast<X*>(&r.w[0]);
#pragma unroll
        for (int q = 0; q < EL; ++q) x[q] = acc_to<X, Acc>(v[q]);
    }
    return r;
}

// ------------------------------------------------------------------ range scan (two kernels)
// The scan used for rows that are whole multiples of 16 bytes.  Each stream's
// tape (in scan order) is cut into R ranges of RL positions, and no CTA ever
// waits on another:
//   k_range_tail  one CTA per range: finds the range's last segment start from
//                 the keys and sums the rows after it (its trailing segment),
//                 i.e. the carry it hands to later ranges; has_start says
//                 whether the range contains a segment start at all;
//   k_range_scan  one CTA per range: folds the tails of the earlier ranges of
//                 its stream into its carry-in, then streams its chunks of 256
//                 positions: warp w owns 32 rows per chunk, stages them with
//                 cp.async into a double-buffered tile (keys prefetched two
//                 chunks ahead), scans them with lanes over columns, writes the
//                 results in place and stores whole rows 16 bytes per lane.
// The tails cost one extra read of the rows after each range's last segment
// start (a few percent of the tape for Zipf addresses).
constexpr int RS_WARPS = 8;
constexpr int RS_CHUNK = RS_WARPS * 32;

struct RangeArgs {
    int64_t S;             // streams
    const void* keys;      // [S][T]
    const int* nvalid;     // [S] or null
    int64_t T, C;
    uint32_t D;
    int tbits;
    int reverse, inclusive;
    int64_t R, RL;         // ranges per stream, positions per range (multiple of RS_CHUNK)
    const void* in;        // dtype [N, D] gathered by flat row, or Acc [S*T, D] by tape index
    void* out;             // dtype [N, D] scattered by flat row, or Acc [S*T, D] by tape index
    uint8_t* out_mask;     // optional [N]
    void* tail;            // Acc [S*R, D]
    uint32_t* tail_hs;     // [S*R]
    int64_t* bounds;       // [S*(R+1)] range boundaries in scan order
    FastDiv fd_vpr;        // 16-byte vectors per input row
};

template <typename KeyT>
__device__ __forceinline__ bool range_is_start(const KeyT* keys, int64_t si, int64_t n_s, int reverse, int tbits) {
    if (si == 0) return true;
    const int64_t p = reverse ? (n_s - 1 - si) : si;
    const int64_t pp = reverse ? (n_s - si) : (si - 1);
    return (keys[p] >> tbits) != (keys[pp] >> tbits);
}

template <typename KeyT>
__device__ __forceinline__ uint32_t range_row(const KeyT* keys, const RowMap& rows_of, int64_t s, int64_t si,
                                              int64_t n_s, int reverse, int tbits, int64_t T, bool sorted) {
    const int64_t p = reverse ? (n_s - 1 - si) : si;
    if (sorted) return static_cast<uint32_t>(s * T + p);
    const KeyT tmask = (static_cast<KeyT>(1) << tbits) - 1;
    return rows_of(keys[p] & tmask);
}

// First segment start in [x, end) of the scan order, or -1 (block-wide).
template <typename KeyT>
__device__ int64_t first_start_from(const KeyT* keys, int64_t x, int64_t end, int64_t n_s, int reverse, int tbits,
                                    int* s_tmp) {
    for (int64_t b0 = x; b0 < end; b0 += RS_CHUNK) {
        if (threadIdx.x == 0) *s_tmp = RS_CHUNK;
        __syncthreads();
        const int64_t si = b0 + threadIdx.x;
        if (si < end && range_is_start(keys, si, n_s, reverse, tbits)) atomicMin(s_tmp, static_cast<int>(threadIdx.x));
        __syncthreads();
        const int f = *s_tmp;
        __syncthreads();
        if (f < RS_CHUNK) return b0 + f;
    }
    return -1;
}

// Last segment start in [x, end) of the scan order, or -1 (block-wide).
template <typename KeyT>
__device__ int64_t last_start_before(const KeyT* keys, int64_t x, int64_t end, int64_t n_s, int reverse, int tbits,
                                     int* s_tmp) {
    for (int64_t e0 = end; e0 > x; e0 -= RS_CHUNK) {
        if (threadIdx.x == 0) *s_tmp = -1;
        __syncthreads();
        const int64_t si = e0 - 1 - threadIdx.x;
        if (si >= x && range_is_start(keys, si, n_s, reverse, tbits)) atomicMax(s_tmp, static_cast<int>(si - x));
        __syncthreads();
        const int f = *s_tmp;
        __syncthreads();
        if (f >= 0) return x + f;
    }
    return -1;
}

// Range boundaries: the nominal boundary r*RL moves forward to the next segment
// start within one range length, so that the range needs no carry.  Only when
// a segment is longer than a range does a boundary stay unsnapped; then the
// range before it publishes its tail (sum of its rows after its last segment
// start, or of all its rows when it has none) for the next range to fold.
template <typename KeyT, int DT, int EL, bool IN_SORTED>
__global__ void __launch_bounds__(RS_WARPS * 32) k_range_tail(RangeArgs a) {
    using Acc = typename Elem<DT>::Acc;
    using InT = typename std::conditional<IN_SORTED, Acc, typename Elem<DT>::T>::type;
    __shared__ int s_tmp;
    __shared__ uint32_t s_rows[RS_CHUNK];
    __shared__ Acc s_red[RS_WARPS][32 * EL];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t s = blockIdx.x / a.R, r = blockIdx.x % a.R;
    const int64_t n_s = a.nvalid ? a.nvalid[s] : a.T;
    const KeyT* keys = static_cast<const KeyT*>(a.keys) + s * a.T;
    const uint32_t D = a.D;
    Acc* tail = static_cast<Acc*>(a.tail) + (s * a.R + r) * D;
    auto snap = [&](int64_t x) -> int64_t {  // boundary at nominal position x
        if (x >= n_s) return n_s;
        if (x == 0) return 0;
        const int64_t f = first_start_from(keys, x, x + a.RL < n_s ? x + a.RL : n_s, n_s, a.reverse, a.tbits, &s_tmp);
        return f >= 0 ? f : x;
    };
    const int64_t lo = snap(r * a.RL);
    const int64_t hi = snap((r + 1) * a.RL);
    if (tid == 0) {
        a.bounds[s * (a.R + 1) + r] = lo;
        if (r == a.R - 1) a.bounds[s * (a.R + 1) + a.R] = n_s;
    }
    const bool hi_unsnapped = hi < n_s && !range_is_start(keys, hi, n_s, a.reverse, a.tbits);
    if (!hi_unsnapped || lo >= hi) {
        if (tid == 0) a.tail_hs[s * a.R + r] = 1u;  // never folded past
        return;
    }
    const int64_t ls = last_start_before(keys, lo, hi, n_s, a.reverse, a.tbits, &s_tmp);
    const RowMap rows_of(s, a.T, a.C);
    const int64_t t0 = ls >= 0 ? ls : lo;
    const bool active = static_cast<uint32_t>(lane * EL) < D;
    const uint32_t col = static_cast<uint32_t>(lane * EL);
    const InT* in = static_cast<const InT*>(a.in);
    Acc acc[EL];
#pragma unroll
    for (int q = 0; q < EL; ++q) acc[q] = Acc(0);
    for (int64_t b0 = t0; b0 < hi; b0 += RS_CHUNK) {  // 256 rows at a time, all loads in flight
        const int64_t si = b0 + tid;
        if (si < hi) s_rows[tid] = range_row(keys, rows_of, s, si, n_s, a.reverse, a.tbits, a.T, IN_SORTED);
        __syncthreads();
        const int nb = static_cast<int>(hi - b0 < RS_CHUNK ? hi - b0 : RS_CHUNK);
#pragma unroll 8
        for (int i = warp; i < nb; i += RS_WARPS) {
            if (active) {
                const RawWords<EL * sizeof(InT)> x = ld_frag<InT, EL>(in + static_cast<uint64_t>(s_rows[i]) * D + col);
#pragma unroll
                for (int q = 0; q < EL; ++q) acc[q] += frag_get<InT, Acc, EL>(x, q);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int q = 0; q < EL; ++q) s_red[warp][lane * EL + q] = acc[q];
    __syncthreads();
    if (warp == 0 && active) {
#pragma unroll
        for (int q = 0; q < EL; ++q) {
            Acc v = Acc(0);
            for (int w = 0; w < RS_WARPS; ++w) v += s_red[w][lane * EL + q];
            tail[col + q] = v;
        }
    }
    if (tid == 0) a.tail_hs[s * a.R + r] = ls >= 0 ? 1u : 0u;
}

template <typename KeyT, int DT, int EL, bool IN_SORTED, bool OUT_SORTED, bool INCL>
__global__ void __launch_bounds__(RS_WARPS * 32) k_range_scan(RangeArgs a) {
    using E = Elem<DT>;
    using Acc = typename E::Acc;
    using V = typename E::T;
    using InT = typename std::conditional<IN_SORTED, Acc, V>::type;
    using OutT = typename std::conditional<OUT_SORTED, Acc, V>::type;
    constexpr bool INPLACE = std::is_same<InT, OutT>::value;
    extern __shared__ __align__(16) unsigned char smem[];
    const uint32_t D = a.D;
    const uint32_t rb = D * static_cast<uint32_t>(sizeof(InT));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // each warp owns one range and a double-buffered tile of 2 x 32 rows
    unsigned char* wbuf = smem + static_cast<size_t>(warp) * 2 * 32 * rb;
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * RS_WARPS + warp;
    const int64_t S = a.S;
    if (gw >= S * a.R) return;
    const int64_t s = gw / a.R, r = gw % a.R;
    const int64_t n_s = a.nvalid ? a.nvalid[s] : a.T;
    const int64_t lo = a.bounds[s * (a.R + 1) + r];
    const int64_t hi = a.bounds[s * (a.R + 1) + r + 1];
    if (lo >= hi) return;
    const KeyT* keys = static_cast<const KeyT*>(a.keys) + s * a.T;
    const bool active = static_cast<uint32_t>(lane * EL) < D;
    const uint32_t col = static_cast<uint32_t>(lane * EL);
    const InT* in = static_cast<const InT*>(a.in);
    OutT* out = static_cast<OutT*>(a.out);
    const int nch = static_cast<int>((hi - lo + 31) / 32);
    const KeyT tmask = (static_cast<KeyT>(1) << a.tbits) - 1;
    const RowMap rows_of(s, a.T, a.C);

    // carry-in: zero when the range starts a segment (snapped boundary), else
    // the tails of the earlier ranges back to the one holding the segment start
    Acc run[EL];
#pragma unroll
    for (int q = 0; q < EL; ++q) run[q] = Acc(0);
    if (!range_is_start(keys, lo, n_s, a.reverse, a.tbits) && active) {
        const Acc* tails = static_cast<const Acc*>(a.tail) + s * a.R * D;
        for (int64_t rr = r - 1; rr >= 0; --rr) {
#pragma unroll
            for (int q = 0; q < EL; ++q) run[q] += tails[rr * D + col + q];
            if (a.tail_hs[s * a.R + rr] != 0u) break;
        }
    }

    struct KeyPair { KeyT k, kp; };
    auto load_keys = [&](int c) -> KeyPair {
        KeyPair kk{KeyT(0), KeyT(0)};
        const int64_t si = lo + static_cast<int64_t>(c) * 32 + lane;
        if (c < nch && si < hi) {
            kk.k = keys[a.reverse ? (n_s - 1 - si) : si];
            if (si > 0) kk.kp = keys[a.reverse ? (n_s - si) : (si - 1)];
        }
        return kk;
    };
    // row indices (input, output) and segment start of this lane's position in chunk c
    auto derive = [&](int c, const KeyPair& kk, uint32_t& my_in, uint32_t& my_out, bool& st) {
        const int64_t si = lo + static_cast<int64_t>(c) * 32 + lane;
        my_in = 0; my_out = 0; st = false;
        if (c < nch && si < hi) {
            const int64_t p = a.reverse ? (n_s - 1 - si) : si;
            const uint32_t tix = static_cast<uint32_t>(s * a.T + p);
            const uint32_t flat = rows_of(kk.k & tmask);
            my_in = IN_SORTED ? tix : flat;
            my_out = OUT_SORTED ? tix : flat;
            st = si == 0 || (kk.k >> a.tbits) != (kk.kp >> a.tbits);
        }
    };
    const uint32_t vpr = rb / 16;
    // lane -> (row offset, 16-byte vector) once, when a row's vectors divide 32
    const bool lane_split = vpr <= 32 && (32 % vpr) == 0;
    uint32_t l_rr = 0, l_v = 0;
    a.fd_vpr.divmod(static_cast<uint32_t>(lane), l_rr, l_v);
    const uint32_t rows_per_pass = lane_split ? 32 / vpr : 0;
    auto stage = [&](int c, uint32_t my_in) {
        unsigned char* tile = wbuf + static_cast<size_t>(c & 1) * 32 * rb;
        const int64_t base = lo + static_cast<int64_t>(c) * 32;
        const int nvw = static_cast<int>(hi - base < 32 ? hi - base : 32);
        if (lane_split) {
            for (uint32_t rr = l_rr; rr < 32; rr += rows_per_pass) {  // uniform trip count
                const uint32_t row = __shfl_sync(0xffffffffu, my_in, static_cast<int>(rr));
                if (static_cast<int>(rr) < nvw)
                    cp_async16(tile + rr * rb + l_v * 16,
                               reinterpret_cast<const char*>(in + static_cast<uint64_t>(row) * D) + l_v * 16);
            }
        } else {
            const uint32_t total = static_cast<uint32_t>(nvw) * vpr;
            for (uint32_t e0 = 0; e0 < total; e0 += 32) {  // uniform trip count: full-warp shuffles
                const uint32_t e = e0 + lane;
                uint32_t rr, v;
                a.fd_vpr.divmod(e, rr, v);
                const uint32_t row = __shfl_sync(0xffffffffu, my_in, static_cast<int>(rr & 31u));
                if (e < total)
                    cp_async16(tile + rr * rb + v * 16,
                               reinterpret_cast<const char*>(in + static_cast<uint64_t>(row) * D) + v * 16);
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    uint32_t in_cur, out_cur;
    bool st_cur;
    derive(0, load_keys(0), in_cur, out_cur, st_cur);
    stage(0, in_cur);
    KeyPair k_next = load_keys(1);

    for (int c = 0; c < nch; ++c) {
        uint32_t in_nx = 0, out_nx = 0;
        bool st_nx = false;
        if (c + 1 < nch) {
            derive(c + 1, k_next, in_nx, out_nx, st_nx);
            stage(c + 1, in_nx);
            k_next = load_keys(c + 2);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncwarp();
        const unsigned sm = __ballot_sync(0xffffffffu, st_cur);
        const int64_t base = lo + static_cast<int64_t>(c) * 32;
        const int nv = static_cast<int>(hi - base < 32 ? hi - base : 32);
        if (a.out_mask != nullptr && lane < nv) a.out_mask[out_cur] = st_cur ? 0 : 1;
        unsigned char* tile = wbuf + static_cast<size_t>(c & 1) * 32 * rb;
        const uint32_t tile_s = smem_u32(tile) + col * static_cast<uint32_t>(sizeof(InT));
        // one pass with the running carry
        if (INPLACE && nv == 32) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const uint32_t addr = tile_s + static_cast<uint32_t>(i) * rb;
                // lanes past the row's columns (lane*EL >= D) must not touch shared
                // memory: their addresses run past the row and, on the last row of
                // the last tile, past the allocation
                RawWords<EL * sizeof(InT)> x{};
                if (active) x = lds_words<EL * sizeof(InT)>(addr);
                Acc v[EL];
                unpack<InT, Acc, EL>(x, v);
                const bool stt = (sm >> i) & 1u;
                Acc o[EL];
#pragma unroll
                for (int q = 0; q < EL; ++q) {
                    run[q] = stt ? Acc(0) : run[q];
                    if (INCL) { run[q] += v[q]; o[q] = run[q]; }
                    else { o[q] = run[q]; run[q] += v[q]; }
                }
                if (active) sts_words<EL * sizeof(OutT)>(addr, pack<OutT, Acc, EL>(o));
            }
        } else {
            for (int i = 0; i < nv; ++i) {
                const uint32_t addr = tile_s + static_cast<uint32_t>(i) * rb;
                RawWords<EL * sizeof(InT)> x{};
                if (active) x = lds_words<EL * sizeof(InT)>(addr);  // see the guard above
                Acc v[EL];
                unpack<InT, Acc, EL>(x, v);
                const uint32_t orow = INPLACE ? 0u : __shfl_sync(0xffffffffu, out_cur, i);
                const bool stt = (sm >> i) & 1u;
                Acc o[EL];
#pragma unroll
                for (int q = 0; q < EL; ++q) {
                    run[q] = stt ? Acc(0) : run[q];
                    if (INCL) { run[q] += v[q]; o[q] = run[q]; }
                    else { o[q] = run[q]; run[q] += v[q]; }
                }
                if (active) {
                    if constexpr (INPLACE) sts_words<EL * sizeof(OutT)>(addr, pack<OutT, Acc, EL>(o));
                    else st_frag<OutT, EL>(out + static_cast<uint64_t>(orow) * D + col, pack<OutT, Acc, EL>(o));
                }
            }
        }
        if constexpr (INPLACE) {
            __syncwarp();
            if (lane_split) {
                for (uint32_t rr = l_rr; rr < 32; rr += rows_per_pass) {
                    const uint32_t orow = __shfl_sync(0xffffffffu, out_cur, static_cast<int>(rr));
                    if (static_cast<int>(rr) < nv) {
                        const uint4 val = *reinterpret_cast<const uint4*>(tile + rr * rb + l_v * 16);
                        *reinterpret_cast<uint4*>(reinterpret_cast<char*>(out) + static_cast<uint64_t>(orow) * rb +
                                                  l_v * 16) = val;
                    }
                }
            } else {
                const uint32_t total = static_cast<uint32_t>(nv) * vpr;
                for (uint32_t e0 = 0; e0 < total; e0 += 32) {
                    const uint32_t e = e0 + lane;
                    uint32_t rr, v;
                    a.fd_vpr.divmod(e, rr, v);
                    const uint32_t orow = __shfl_sync(0xffffffffu, out_cur, static_cast<int>(rr & 31u));
                    if (e < total) {
                        const uint4 val = *reinterpret_cast<const uint4*>(tile + rr * rb + v * 16);
                        *reinterpret_cast<uint4*>(reinterpret_cast<char*>(out) + static_cast<uint64_t>(orow) * rb +
                                                  v * 16) = val;
                    }
                }
            }
        }
        __syncwarp();
        in_cur = in_nx;
        out_cur = out_nx;
        st_cur = st_nx;
    }
}

template <typename Acc>
inline size_t range_scan_smem(int64_t D, size_t in_elem) {
    return static_cast<size_t>(RS_WARPS) * 2 * 32 * D * in_elem;
}

// Rows a warp holds in registers: at most 64 bytes of input per lane (16 rows
// of 4 bytes).
constexpr int scanw_rows(int el, int bytes) {
    return (64 / (el * bytes)) > 16 ? 16 : ((64 / (el * bytes)) < 1 ? 1 : 64 / (el * bytes));
}

template <typename Acc>
inline size_t segscan_w_smem(int64_t D) {
    return static_cast<size_t>(SCANW_WARPS + 1) * D * sizeof(Acc);
}

template <typename Acc>
inline size_t segscan_smem(int P, int parts, int64_t D) {
    return static_cast<size_t>(P) * D * sizeof(Acc) + static_cast<size_t>(parts) * D * sizeof(Acc) +
           D * sizeof(Acc) + static_cast<size_t>(P) * (8 + 8 + 1) + 16;
}

// ------------------------------------------------------------------ general sum helpers
struct SsGenArgs {
    const void* keys;
    const int64_t* soff;
    const int32_t* ridx;
    const void* raddr;
    int addr_i64, key32;
    int64_t B, T, C, D, A;
    int tbits;
    const void* tapebuf;   // Acc [S*T, D] (forward: inclusive segmented sums)
    void* accbuf;          // Acc [S*T, D] (backward: read gradients added at their latest write)
    const void* grad;      // backward: grad_sums [N, D]
    void* out;             // forward: sums [N, D]
    uint8_t* out_mask;     // forward: [N]
    FastDiv fd_C, fd_T;    // flat row -> (b, t, c)
};

template <typename KeyT>
__device__ __forceinline__ bool ss_valid(const SsGenArgs& a, int64_t r, int64_t& tape_index) {
    const int64_t T = a.T, C = a.C;
    uint32_t bt, c32, b32, t32;
    a.fd_C.divmod(static_cast<uint32_t>(r), bt, c32);
    a.fd_T.divmod(bt, b32, t32);
    const int64_t s = static_cast<int64_t>(b32) * C + c32;
    const int32_t idx = a.ridx[r];
    if (idx < 0) return false;
    const KeyT key = static_cast<const KeyT*>(a.keys)[s * T + idx];
    const uint64_t ra = fold_addr(load_addr(a.raddr, r, a.addr_i64), a.A, a.key32);
    tape_index = s * T + idx;
    return static_cast<uint64_t>(key >> a.tbits) == ra;
}

// sums[r] = valid ? tape[latest(r)] : 0 (ravel_memory.py:235-240)
template <typename KeyT, int DT>
__global__ void __launch_bounds__(256) k_ss_gather(SsGenArgs a) {
    using E = Elem<DT>;
    using Acc = typename E::Acc;
    using V = typename E::T;
    const int64_t N = a.B * a.T * a.C, D = a.D;
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t r = warp0; r < N; r += nwarps) {
        int64_t ti = 0;
        const bool valid = ss_valid<KeyT>(a, r, ti);
        const Acc* src = static_cast<const Acc*>(a.tapebuf) + ti * D;
        V* dst = static_cast<V*>(a.out) + r * D;
        for (int64_t d = lane; d < D; d += 32) dst[d] = E::from_acc(valid ? src[d] : Acc(0));
        if (lane == 0) a.out_mask[r] = valid ? 1 : 0;
    }
}

// accbuf[latest(r)] += grad_sums[r] for every valid read (transpose of the gather)
template <typename KeyT, int DT>
__global__ void __launch_bounds__(256) k_ss_scatter(SsGenArgs a) {
    using E = Elem<DT>;
    using Acc = typename E::Acc;
    using V = typename E::T;
    const int64_t N = a.B * a.T * a.C, D = a.D;
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t r = warp0; r < N; r += nwarps) {
        int64_t ti = 0;
        if (!ss_valid<KeyT>(a, r, ti)) continue;
        Acc* dst = static_cast<Acc*>(a.accbuf) + ti * D;
        const V* g = static_cast<const V*>(a.grad) + r * D;
        for (int64_t d = lane; d < D; d += 32) atomicAdd(dst + d, E::to_acc(g[d]));
    }
}

}  // namespace ravel
