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
//   * a chunk containing a segment start publishes its inclusive value (flag 2),
//     any other chunk only its aggregate (flag 1); look-back adds aggregates back
//     to the nearest chunk with a segment start (chunk 0 of every stream is one).
//     Every successor thus adds the same values in the same order, and the sums
//     are the same bits from run to run;
//   * every wait is bounded: after g_wait_limit polls the kernel flags
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

template <typename Acc>
struct ScanArgs {
    const void* keys;        // [S][T]
    const int* nvalid;       // [S] or null (all T)
    int64_t B, T, C, D;
    int tbits;
    const void* in;          // in_sorted ? Acc [S*T, D] : dtype [N, D]
    void* out;               // dtype: [S*T, D] by tape index when out_sorted, else [N, D] by flat row
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
                const unsigned f = wait_flag(a.flags + j, 64);
                if (f == 0u) break;  // gave up: RAVEL_DEVERR_SPIN is set
                const Acc* src = (f == 2u) ? a.incl + j * D : a.agg + j * D;
                for (int col = lane; col < D; col += 32) pagg[col] += src[col];
                if (f == 2u) break;
                --j;
            }
        }
        __syncthreads();
        // (a chunk without a segment start never publishes an inclusive value: its
        // successors always add the same aggregates in the same order, so sums are
        // the same bits from run to run)
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
        V* out = static_cast<V*>(a.out) + s * T * D;
        for (uint32_t e = tid; e < static_cast<uint32_t>(np * D); e += SCAN_THREADS) {
            uint32_t i, d;
            a.fd_d.divmod(e, i, d);
            out[(srow[i] & 0xffffffffll) * D + d] = E::from_acc(rows[e]);
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
            f = wait_flag(flags + idx, 32);
            if (f == 0u) f = 3u;  // gave up: RAVEL_DEVERR_SPIN is set
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
    using OutT = V;  // sorted outputs too are stored in the payload dtype
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
            // no inclusive value for a chunk without a segment start: a fixed set of
            // aggregates in a fixed order reaches every successor (reproducible sums)
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


// Copy staged result rows [r0, r1) of the chunk to their output rows, 16 bytes
// per lane (rows are whole multiples of 16 bytes).

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

// ------------------------------------------------------------------ group scan
// The scan used for rows that are whole multiples of 16 bytes, up to 1 KB.
// Each stream's tape (in scan order) is cut into R ranges of about RL
// positions; a nominal boundary r*RL moves forward to a segment start when one
// lies within `snap` positions, so every range stays within RL + snap.  A
// range's *piece* is the sum of its rows from its last segment start (from its
// lower boundary lo when it holds none) to its upper boundary hi, when hi falls
// inside a segment: the carry it hands to the next range.
//
// k_range_scan: a block owns GPB = GS_WARPS * 32 / L consecutive ranges of one
// stream, one range per lane group of L = row_bytes / (16 VPL) lanes (each lane
// owns VPL 16-byte column slices of every row).  Blocks take tickets, so every
// block one waits on is already running.
//   1. segment-start bitmap of the block's span from one coalesced pass over
//      its keys; each range's bounds, its last segment start and whether hi
//      falls inside a segment;
//   2. each lane group sums its range's piece;
//   3. warp 0 publishes the block's outgoing carry (the pieces back to the last
//      range with a segment start: final at once when there is one, else an
//      aggregate until the incoming carry is known), looks back over the
//      blocks before for the incoming carry when the block's first position
//      does not start a segment, and turns the pieces into every range's
//      incoming carry;
//   4. each lane group scans its range through a lane-private cp.async ring
//      of GS_Q blocks of GS_U rows in shared memory, so no lane waits on
//      another: the piece rows first (just read, still in L2), then lo .. rot-1
//      with the carry entering at lo.  The running sum resets at segment starts.
// Rows are read and written in tape order, i.e. at random row addresses, so
// the kernel is bounded by random 16-byte-sliced row traffic rather than by
// streaming bandwidth.  Look-back waits are bounded (RAVEL_DEVERR_SPIN, the
// carry taken as found).
// Tuning constants (overridable at build time for sweeps).
#ifndef RAVEL_GS_WARPS
#define RAVEL_GS_WARPS 4
#endif
#ifndef RAVEL_GS_U
#define RAVEL_GS_U 4
#endif
#ifndef RAVEL_GS_Q
#define RAVEL_GS_Q 3
#endif
#ifndef RAVEL_GS_SNAP
#define RAVEL_GS_SNAP 32
#endif
constexpr int GS_WARPS = RAVEL_GS_WARPS;  // warps per block
constexpr int GS_U = RAVEL_GS_U;          // rows per ring block
constexpr int GS_Q = RAVEL_GS_Q;          // ring blocks (GS_Q - 1 blocks in flight)
constexpr int GS_SNAP = RAVEL_GS_SNAP;    // boundary snap window, <= 32
static_assert(GS_SNAP >= 0 && GS_SNAP <= 32, "snap window is one warp ballot");

struct GsArgs {
    int64_t S;             // streams
    const void* keys;      // [S][T]
    const int* nvalid;     // [S] or null
    int64_t T, C;
    uint32_t D;
    int tbits;
    int reverse;
    int lshift;            // log2 of lanes per row group (L)
    int snap;              // boundary snap window, <= 32
    int64_t R, RL;         // ranges per stream, nominal positions per range
    const void* in;        // dtype [N, D] by flat row, or Acc [S*T, D] by tape index
    void* out;             // dtype [N, D] by flat row, or Acc [S*T, D] by tape index
    uint8_t* out_mask;     // optional [N]: 1 where an earlier write of the segment exists
    int64_t CB;            // blocks per stream
    int bmw;               // segment-start bitmap words per block
    unsigned* bflags;      // [S*CB] look-back states, then the ticket counter; zeroed before launch
    void* bval;            // Acc [S*CB][2][D]: block aggregate, block inclusive carry
    // merged scans (general tapes): the stream's valid writes and all its reads in one
    // sequence; only positions of role `load_role` read a row, only the others store one
    const uint8_t* role;   // [S][Ts]: bit 0 a write, bit 1 a read with an earlier write of its address
    int64_t Ts;            // keys (and roles) per stream in `keys`
    int load_role;
};

inline size_t range_scan_smem(int vpl, int64_t gpb, int64_t D, size_t acc_bytes, int64_t bmw) {
    size_t b = static_cast<size_t>(GS_WARPS) * GS_Q * GS_U * 32 * (16 * vpl + 4);
    b += static_cast<size_t>(gpb) * D * acc_bytes;
    b += static_cast<size_t>(bmw) * 4 + static_cast<size_t>(gpb + 1) * 4 + static_cast<size_t>(gpb) * 8;
    return b;
}

template <typename KeyT, int DT, bool IN_SORTED, bool OUT_SORTED, bool INCL, int VPL, bool MERGED>
// Build-time knob: RAVEL_GS_MINB = resident blocks per SM the register allocation
// must allow.  Measured at config 3 (sum forward / backward, us): none 168 / 160,
// 6 blocks (80 registers) 166 / 158, 8 blocks (64 registers) 168 / 161, 1 block
// 194 / 185; a 2-block ring 179 / 170, 8 warps per block 206 / 196.
#ifdef RAVEL_GS_MINB
#define RAVEL_GS_BOUNDS __launch_bounds__(GS_WARPS * 32, RAVEL_GS_MINB)
#else
#define RAVEL_GS_BOUNDS __launch_bounds__(GS_WARPS * 32)
#endif
__global__ void RAVEL_GS_BOUNDS k_range_scan(GsArgs a) {
    using E = Elem<DT>;
    using Acc = typename E::Acc;
    using V = typename E::T;
    using InT = typename std::conditional<IN_SORTED, Acc, V>::type;
    using OutT = V;
    constexpr int EL = 16 / static_cast<int>(sizeof(InT));
    constexpr int NE = VPL * EL;
    constexpr int SLOTS = GS_Q * GS_U;
    constexpr int PU = 8 / VPL;  // piece rows per lane in flight
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t L = 1u << a.lshift;
    const int gpw = 32 >> a.lshift, GPB = GS_WARPS * gpw;
    const uint32_t grp = static_cast<uint32_t>(lane) >> a.lshift, lig = static_cast<uint32_t>(lane) & (L - 1);
    const int gib = warp * gpw + static_cast<int>(grp);
    const uint32_t D = a.D;
    const int tb = a.tbits;
    const uint32_t ring = smem_u32(smem) + static_cast<uint32_t>(warp) * SLOTS * 32 * (16 * VPL + 4);
    const uint32_t meta = ring + SLOTS * 32 * 16 * VPL;
    Acc* cpc = reinterpret_cast<Acc*>(smem + static_cast<size_t>(GS_WARPS) * SLOTS * 32 * (16 * VPL + 4));
    uint32_t* bm = reinterpret_cast<uint32_t*>(cpc + static_cast<size_t>(GPB) * D);
    int32_t* glo = reinterpret_cast<int32_t*>(bm + a.bmw);  // [GPB + 1] range bounds
    int32_t* grot = glo + GPB + 1;                           // [GPB] first piece position
    int32_t* gfl = grot + GPB;                               // [GPB] bit 0 start inside, bit 1 hi open, bit 2 lo starts
    __shared__ unsigned s_tk;
    if (tid == 0) s_tk = atomicAdd(a.bflags + a.S * a.CB, 1u);
    __syncthreads();
    const int64_t tk = s_tk;
    const int64_t s = tk / a.CB, cb = tk - s * a.CB;
    // merged: the stream's valid writes and its T reads
    const int32_t n_s = (a.nvalid ? a.nvalid[s] : static_cast<int32_t>(a.T)) + (MERGED ? static_cast<int32_t>(a.T) : 0);
    const int64_t Ts = MERGED ? a.Ts : a.T;
    const int64_t r0 = cb * GPB;
    const int nr = static_cast<int>(a.R - r0 < GPB ? a.R - r0 : GPB);
    const int32_t RL = static_cast<int32_t>(a.RL);
    const int32_t X0 = static_cast<int32_t>(r0 * a.RL);
    if (nr <= 0 || X0 >= n_s) return;  // whole block: the empty tail of the stream

    const int32_t dir = a.reverse ? -1 : 1;
    const KeyT* kbase = static_cast<const KeyT*>(a.keys) + s * Ts + (a.reverse ? n_s - 1 : 0);
    const uint8_t* rbase = MERGED ? a.role + s * Ts + (a.reverse ? n_s - 1 : 0) : nullptr;
    const uint8_t lrole = static_cast<uint8_t>(a.load_role);
    const uint32_t tix0 = static_cast<uint32_t>(s * a.T) + static_cast<uint32_t>(a.reverse ? n_s - 1 : 0);
    // 1. segment starts of scan positions [X0, X0 + 32 bmw)
    for (int w = warp; w < a.bmw; w += GS_WARPS) {
        const int32_t si = X0 + 32 * w + lane;
        const bool live = si < n_s;
        const KeyT k = live ? kbase[dir * si] : KeyT(0);
        KeyT kp = __shfl_up_sync(0xffffffffu, k, 1);
        if (lane == 0 && live && si > 0) kp = kbase[dir * (si - 1)];
        const unsigned b = __ballot_sync(0xffffffffu, live && (si == 0 || ((k ^ kp) >> tb) != 0));
        if (lane == 0) bm[w] = b;
    }
    __syncthreads();
    auto bit = [&](int32_t x) -> bool {
        if (x >= n_s) return false;
        const int32_t o = x - X0;
        return (bm[o >> 5] >> (o & 31)) & 1u;
    };
    if (warp == 0) {
        const unsigned smask = a.snap >= 32 ? 0xffffffffu : ((1u << a.snap) - 1u);
        for (int j = lane; j <= nr; j += 32) {
            const int32_t x = X0 + j * RL;
            int32_t lo;
            if (x >= n_s) lo = n_s;
            else if (x == 0) lo = 0;
            else {
                const int32_t o = x - X0;
                const uint64_t w2 = static_cast<uint64_t>(bm[o >> 5]) | (static_cast<uint64_t>(bm[(o >> 5) + 1]) << 32);
                const unsigned win = static_cast<unsigned>(w2 >> (o & 31)) & smask;
                lo = win ? x + __ffs(win) - 1 : x;
            }
            glo[j] = lo;
        }
        __syncwarp();
        for (int j = lane; j < nr; j += 32) {
            const int32_t l = glo[j], h = glo[j + 1];
            int32_t ls = -1;
            for (int32_t e = h; e > l && ls < 0;) {  // last start in [l, h), a word at a time
                const int32_t o = e - 1 - X0;
                const int w = o >> 5;
                unsigned m = bm[w] & (0xffffffffu >> (31 - (o & 31)));
                const int32_t wb = X0 + 32 * w;
                if (wb < l) m &= ~((1u << (l - wb)) - 1u);
                if (m) ls = wb + 31 - __clz(m);
                e = wb;
            }
            grot[j] = ls >= 0 ? ls : l;
            gfl[j] = (ls >= 0 ? 1 : 0) | ((h < n_s && l < h && !bit(h)) ? 2 : 0) | (bit(l) ? 4 : 0);
        }
    }
    __syncthreads();

    const RowMap rows_of(s, a.T, a.C);
    const KeyT tmask = (static_cast<KeyT>(1) << tb) - 1;
    const char* in = static_cast<const char*>(a.in) + lig * 16u;
    const uint32_t rbi = D * static_cast<uint32_t>(sizeof(InT));
    auto row_in = [&](int32_t si, KeyT k) -> uint32_t {
        return IN_SORTED ? tix0 + static_cast<uint32_t>(dir * si) : rows_of(k & tmask);
    };
    // 2. pieces
    {
        int32_t p0 = 0, n = 0;
        if (gib < nr && (gfl[gib] & 2)) {
            p0 = grot[gib];
            n = glo[gib + 1] - p0;
        }
        int32_t nmax = n;
        for (uint32_t off = L; off < 32u; off <<= 1) {
            const int32_t o = __shfl_xor_sync(0xffffffffu, nmax, static_cast<int>(off));
            nmax = o > nmax ? o : nmax;
        }
        Acc acc[NE];
#pragma unroll
        for (int q = 0; q < NE; ++q) acc[q] = Acc(0);
        KeyT kn[PU];
        bool ld[PU];  // the position reads a row (merged: only positions of the loading role)
#pragma unroll
        for (int u = 0; u < PU; ++u) {
            kn[u] = u < n ? kbase[dir * (p0 + u)] : KeyT(0);
            ld[u] = u < n && (!MERGED || (rbase[dir * (p0 + u)] & 1) == lrole);
        }
        for (int32_t i0 = 0; i0 < nmax; i0 += PU) {
            uint4 w[PU][VPL];
#pragma unroll
            for (int u = 0; u < PU; ++u) {
                const int32_t i = i0 + u;
                const uint32_t row = row_in(p0 + i, kn[u]);
#pragma unroll
                for (int v = 0; v < VPL; ++v)
                    w[u][v] = ld[u] ? ld_nc_v4(in + static_cast<uint64_t>(row) * rbi + v * L * 16u)
                                    : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < PU; ++u) {
                const int32_t i = i0 + PU + u;
                kn[u] = i < n ? kbase[dir * (p0 + i)] : KeyT(0);
                ld[u] = i < n && (!MERGED || (rbase[dir * (p0 + i)] & 1) == lrole);
            }
#pragma unroll
            for (int u = 0; u < PU; ++u)
#pragma unroll
                for (int v = 0; v < VPL; ++v) {
                    RawWords<16> x;
                    x.w[0] = w[u][v].x; x.w[1] = w[u][v].y; x.w[2] = w[u][v].z; x.w[3] = w[u][v].w;
                    Acc f[EL];
                    unpack<InT, Acc, EL>(x, f);
#pragma unroll
                    for (int e = 0; e < EL; ++e) acc[v * EL + e] += f[e];
                }
        }
#pragma unroll
        for (int v = 0; v < VPL; ++v)
#pragma unroll
            for (int e = 0; e < EL; ++e) cpc[static_cast<uint32_t>(gib) * D + (lig + v * L) * EL + e] = acc[v * EL + e];
    }
    __syncthreads();
    // 3. block carry: publish, look back, per-range carries (warp 0, lane owns columns lane + 32 q)
    if (warp == 0) {
        Acc* bv = static_cast<Acc*>(a.bval);
        int jstar = -1;
        for (int j = 0; j < nr; ++j)
            if (gfl[j] & 1) jstar = j;
        const bool closed = jstar >= 0;
        for (uint32_t col = lane; col < D; col += 32) {
            Acc o = Acc(0);
            for (int j = closed ? jstar : 0; j < nr; ++j) o += cpc[static_cast<uint32_t>(j) * D + col];
            bv[(tk * 2 + (closed ? 1 : 0)) * D + col] = o;
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) st_release(a.bflags + tk, closed ? 2u : 1u);
        const bool need = cb > 0 && !(gfl[0] & 4);
        // incoming carry of the block, per owned column
        constexpr int MAXC = (1024 / static_cast<int>(sizeof(V)) + 31) / 32;  // rows up to 1 KB
        Acc cin[MAXC];
#pragma unroll
        for (int q = 0; q < MAXC; ++q) cin[q] = Acc(0);
        if (need) {
            for (int64_t j = tk - 1;; --j) {
                const unsigned f = wait_flag(a.bflags + j, 64);
                if (f == 0u) break;  // gave up: RAVEL_DEVERR_SPIN is set
                const Acc* src = bv + (j * 2 + (f == 2u ? 1 : 0)) * D;
#pragma unroll
                for (int q = 0; q < MAXC; ++q) {
                    const uint32_t col = lane + 32u * q;
                    if (col < D) cin[q] += __ldcg(src + col);
                }
                if (f == 2u || j == tk - cb) break;
            }
        }
        // A block without a segment start publishes only its aggregate (never an
        // inclusive value once its own look-back is done): every successor then adds
        // the same aggregates in the same order back to the nearest block holding a
        // segment start, so the sums are the same bits from run to run.
        // carries: c_0 = cin; c_{j+1} = 0 if lo_{j+1} starts a segment, else piece_j (+ c_j when range j holds no start)
#pragma unroll
        for (int q = 0; q < MAXC; ++q) {
            const uint32_t col = lane + 32u * q;
            if (col >= D) continue;
            Acc c = cin[q];
            for (int j = 0; j < nr; ++j) {
                const Acc p = cpc[static_cast<uint32_t>(j) * D + col];
                cpc[static_cast<uint32_t>(j) * D + col] = c;
                const int fl = gfl[j];
                c = (j + 1 < nr && (gfl[j + 1] & 4)) ? Acc(0) : ((fl & 1) ? p : c + p);
            }
        }
    }
    __syncthreads();
    // 4. scan of the range, the carry entering at lo
    if (gib >= nr) return;  // this group only: nothing below synchronises lanes
    const int32_t lo = glo[gib], hi = glo[gib + 1];
    if (lo >= hi) return;
    Acc carry[NE];
#pragma unroll
    for (int v = 0; v < VPL; ++v)
#pragma unroll
        for (int e = 0; e < EL; ++e) carry[v * EL + e] = cpc[static_cast<uint32_t>(gib) * D + (lig + v * L) * EL + e];
    // rows rot .. hi-1 first (the piece rows just read), then lo .. rot-1
    const int32_t rot = grot[gib];
    const int32_t len = hi - lo, nA = hi - rot;
    const int32_t offA = rot, offB = lo - nA;  // scan position of sequence index i: i + (i < nA ? offA : offB)
    const int32_t inj = nA == len ? 0 : nA;    // sequence index of position lo
    const KeyT kbr0 = rot > 0 ? kbase[dir * (rot - 1)] : ~kbase[dir * rot];
    const KeyT kbrA = (nA < len && lo > 0) ? kbase[dir * (lo - 1)] : ~kbase[dir * lo];
    char* out = static_cast<char*>(a.out) + lig * static_cast<uint32_t>(EL * sizeof(OutT));
    uint8_t* omask = (a.out_mask != nullptr && lig == 0) ? a.out_mask : nullptr;
    const uint32_t rbo = D * static_cast<uint32_t>(sizeof(OutT));
    const int32_t nb = (len + GS_U - 1) / GS_U;
    const uint32_t lane_slot = static_cast<uint32_t>(lane);

    // merged scans: each position's role byte beside its key
    auto load_keys = [&](int32_t b, KeyT (&k)[GS_U], uint8_t (&r)[GS_U]) {
#pragma unroll
        for (int u = 0; u < GS_U; ++u) {
            const int32_t i = b * GS_U + u;
            if (i < len) {
                const int32_t sp = i + (i < nA ? offA : offB);
                k[u] = kbase[dir * sp];
                if (MERGED) r[u] = rbase[dir * sp];
            }
        }
    };
    KeyT klast = KeyT(0);  // key of the row staged last
    auto stage = [&](int32_t b, const KeyT (&kb)[GS_U], const uint8_t (&rb)[GS_U]) {
        if (b < nb) {
            const uint32_t slot0 = static_cast<uint32_t>(b % GS_Q) * GS_U;
#pragma unroll
            for (int u = 0; u < GS_U; ++u) {
                const int32_t i = b * GS_U + u;
                if (i < len) {
                    const KeyT k = kb[u];
                    const KeyT kp = i == 0 ? kbr0 : (i == nA ? kbrA : (u > 0 ? kb[u - 1] : klast));
                    const bool st = ((k ^ kp) >> tb) != 0;
                    uint32_t rin, rout;
                    if (IN_SORTED || OUT_SORTED) {
                        const uint32_t tix = tix0 + static_cast<uint32_t>(dir * (i + (i < nA ? offA : offB)));
                        const uint32_t flat = rows_of(k & tmask);
                        rin = IN_SORTED ? tix : flat;
                        rout = OUT_SORTED ? tix : flat;
                    } else {
                        rin = rout = rows_of(k & tmask);
                    }
                    const uint32_t slot = (slot0 + u) * 32 + lane_slot;
                    // merged: a loading position stores nothing (bit 30), the others read nothing;
                    // bit 29 carries a storing read's mask
                    const bool loads = !MERGED || (rb[u] & 1) == lrole;
                    if (loads) {
#pragma unroll
                        for (int v = 0; v < VPL; ++v)
                            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(ring + (slot * VPL + v) * 16),
                                         "l"(in + static_cast<uint64_t>(rin) * rbi + v * L * 16u)
                                         : "memory");
                    } else {
#pragma unroll
                        for (int v = 0; v < VPL; ++v)
                            asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(ring + (slot * VPL + v) * 16),
                                         "r"(0u)
                                         : "memory");
                    }
                    const uint32_t mflags = MERGED ? ((loads ? 0x40000000u : 0u) | ((rb[u] & 2) ? 0x20000000u : 0u)) : 0u;
                    asm volatile("st.shared.u32 [%0], %1;" ::"r"(meta + slot * 4),
                                 "r"(rout | mflags | (st ? 0x80000000u : 0u))
                                 : "memory");
                }
            }
            klast = kb[GS_U - 1];
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    Acc acc[NE];
#pragma unroll
    for (int q = 0; q < NE; ++q) acc[q] = Acc(0);
    auto process = [&](int32_t b) {
        asm volatile("cp.async.wait_group %0;" ::"n"(GS_Q - 1) : "memory");
        const uint32_t slot0 = static_cast<uint32_t>(b % GS_Q) * GS_U;
#pragma unroll
        for (int u = 0; u < GS_U; ++u) {
            const int32_t i = b * GS_U + u;
            if (i < len) {
                if (i == inj) {
#pragma unroll
                    for (int q = 0; q < NE; ++q) acc[q] = carry[q];
                }
                const uint32_t slot = (slot0 + u) * 32 + lane_slot;
                uint32_t mw;
                asm volatile("ld.shared.u32 %0, [%1];" : "=r"(mw) : "r"(meta + slot * 4));
                const bool st = static_cast<int32_t>(mw) < 0;
                const bool store = !MERGED || (mw & 0x40000000u) == 0u;
                const uint32_t orow = mw & (MERGED ? 0x1fffffffu : 0x7fffffffu);
#pragma unroll
                for (int v = 0; v < VPL; ++v) {
                    const RawWords<16> x = lds_words<16>(ring + (slot * VPL + v) * 16);
                    Acc f[EL], o[EL];
                    unpack<InT, Acc, EL>(x, f);
#pragma unroll
                    for (int e = 0; e < EL; ++e) {
                        Acc& c = acc[v * EL + e];
                        c = st ? Acc(0) : c;
                        if (INCL) { c += f[e]; o[e] = c; }
                        else { o[e] = c; c += f[e]; }
                    }
                    if (store)
                        st_frag<OutT, EL>(reinterpret_cast<OutT*>(out + static_cast<uint64_t>(orow) * rbo +
                                                                  v * L * static_cast<uint32_t>(EL * sizeof(OutT))),
                                          pack<OutT, Acc, EL>(o));
                }
                if (MERGED) {
                    if (omask != nullptr && store) omask[orow] = (mw & 0x20000000u) ? 1 : 0;
                } else if (omask != nullptr) {
                    omask[orow] = st ? 0 : 1;
                }
            }
        }
    };
    KeyT k0[GS_U], k1[GS_U];
    uint8_t r0v[GS_U], r1v[GS_U];
#pragma unroll
    for (int u = 0; u < GS_U; ++u) r0v[u] = r1v[u] = 0;
#pragma unroll
    for (int b = 0; b < GS_Q - 1; ++b) {
        load_keys(b, k0, r0v);
        stage(b, k0, r0v);
    }
    load_keys(GS_Q - 1, k0, r0v);
    load_keys(GS_Q, k1, r1v);
    for (int32_t b = 0; b < nb; b += 2) {
        stage(b + GS_Q - 1, k0, r0v);
        load_keys(b + GS_Q + 1, k0, r0v);
        process(b);
        if (b + 1 < nb) {
            stage(b + GS_Q, k1, r1v);
            load_keys(b + GS_Q + 2, k1, r1v);
            process(b + 1);
        }
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
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
    const void* tapebuf;   // dtype [S*T, D] (forward: inclusive segmented sums, rounded once)
    void* accbuf;          // Acc [S*T, D] (backward: read gradients added at their latest write)
    const void* grad;      // backward: grad_sums [N, D]
    void* out;             // forward: sums [N, D]
    uint8_t* out_mask;     // forward: [N]
    FastDiv fd_C, fd_T;    // flat row -> (b, t, c)
    int vshift;            // 16-bit payloads: log2(D/8) when rows split into 2^vshift 8-element
                           // chunks (D/8 a power of two <= 32, 16-byte aligned), else -1
};

// 8 elements of a 16-bit payload type packed in a uint4, as floats.
template <typename V>
__device__ __forceinline__ void unpack8(const uint4& w, float (&f)[8]) {
    RawWords<16> x;
    x.w[0] = w.x; x.w[1] = w.y; x.w[2] = w.z; x.w[3] = w.w;
    unpack<V, float, 8>(x, f);
}

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
    if constexpr (sizeof(V) == 2) {
        if (a.vshift >= 0) {  // 2^vshift lanes per read, 8 elements (16 bytes out) per lane
            const int sh = a.vshift;
            const int sub = lane >> sh, c = lane & ((1 << sh) - 1);
            const int64_t per = 32 >> sh;
            for (int64_t r0 = warp0 * per; r0 < N; r0 += nwarps * per) {
                const int64_t r = r0 + sub;
                if (r >= N) continue;
                int64_t ti = 0;
                const bool valid = ss_valid<KeyT>(a, r, ti);
                const uint4 w = valid ? ld_nc_v4(static_cast<const V*>(a.tapebuf) + ti * D + c * 8)
                                      : make_uint4(0u, 0u, 0u, 0u);
                *reinterpret_cast<uint4*>(static_cast<V*>(a.out) + r * D + c * 8) = w;
                if (c == 0) a.out_mask[r] = valid ? 1 : 0;
            }
            return;
        }
    }
    for (int64_t r = warp0; r < N; r += nwarps) {
        int64_t ti = 0;
        const bool valid = ss_valid<KeyT>(a, r, ti);
        const V* src = static_cast<const V*>(a.tapebuf) + ti * D;
        V* dst = static_cast<V*>(a.out) + r * D;
        for (int64_t d = lane; d < D; d += 32) dst[d] = valid ? src[d] : E::from_acc(Acc(0));
        if (lane == 0) a.out_mask[r] = valid ? 1 : 0;
    }
}


// General sum backward, second half.  The first half is a reverse inclusive
// segmented scan over the *read* tape (reads sorted by (address, t)), which
// leaves at each sorted read the sum of the gradients of itself and of every
// later read of its address, in the payload dtype.  The reads whose latest
// valid write is at or after write q are, among the reads of q's address,
// exactly those from the first read ranked >= q to the end of that address:
// grad_payload[write q] = suffix[bs[q + 1]] when that read has q's address,
// else zero (ravel_memory.py:223-240 through autograd).  One lane group per
// write; a row copy.
template <typename KeyT, int DT, int VB>
__global__ void __launch_bounds__(256) k_ss_bwd_suffix(const KeyT* wkeys, const KeyT* rkeys, const int32_t* bstart,
                                                       const int* nvalid, const void* suffix, void* grad, int64_t S,
                                                       int64_t T, int64_t C, int64_t D, int tbits, int lshift) {
    using V = typename Elem<DT>::T;
    constexpr int EPV = VB / static_cast<int>(sizeof(V));
    const int lane = threadIdx.x & 31;
    const uint32_t L = 1u << lshift;
    const uint32_t grp = static_cast<uint32_t>(lane) >> lshift, lig = static_cast<uint32_t>(lane) & (L - 1);
    const int64_t gpw = 32 >> lshift;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const KeyT tmask = (static_cast<KeyT>(1) << tbits) - 1;
    for (int64_t gi = warp0 * gpw + grp; gi < S * T; gi += nwarps * gpw) {
        const int64_t s = gi / T, q = gi - s * T;
        const int64_t n_s = nvalid ? nvalid[s] : T;
        if (q >= n_s) continue;  // masked writes: their rows were zeroed before
        const KeyT wk = wkeys[gi];
        const int32_t i = bstart[s * (T + 2) + q + 1];
        const bool valid = i < T && (rkeys[s * T + i] >> tbits) == (wk >> tbits);
        uint4 x = make_uint4(0u, 0u, 0u, 0u);
        if (valid) x = ldg_vec<VB>(static_cast<const V*>(suffix) + (s * T + i) * D + lig * EPV);
        const RowMap rows_of(s, T, C);
        st_vec<VB>(static_cast<V*>(grad) + static_cast<uint64_t>(rows_of(wk & tmask)) * D + lig * EPV, x);
    }
}

// k_ss_bwd_suffix for rows that do not split into 2^m <= 32 vectors: one warp per
// write, its lanes over the row's elements 32 apart (a copy, so deterministic).
template <typename KeyT, int DT>
__global__ void __launch_bounds__(256) k_ss_bwd_suffix_rows(const KeyT* wkeys, const KeyT* rkeys,
                                                            const int32_t* bstart, const int* nvalid,
                                                            const void* suffix, void* grad, int64_t S, int64_t T,
                                                            int64_t C, int64_t D, int tbits) {
    using V = typename Elem<DT>::T;
    const int lane = threadIdx.x & 31;
    const int64_t warp0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const KeyT tmask = (static_cast<KeyT>(1) << tbits) - 1;
    for (int64_t gi = warp0; gi < S * T; gi += nwarps) {
        const int64_t s = gi / T, q = gi - s * T;
        const int64_t n_s = nvalid ? nvalid[s] : T;
        if (q >= n_s) continue;  // masked writes: their rows were zeroed before
        const KeyT wk = wkeys[gi];
        const int32_t i = bstart[s * (T + 2) + q + 1];
        const bool valid = i < T && (rkeys[s * T + i] >> tbits) == (wk >> tbits);
        const RowMap rows_of(s, T, C);
        V* dst = static_cast<V*>(grad) + static_cast<uint64_t>(rows_of(wk & tmask)) * D;
        const V* src = static_cast<const V*>(suffix) + (s * T + i) * D;
        for (int64_t d = lane; d < D; d += 32) dst[d] = valid ? src[d] : Elem<DT>::from_acc(typename Elem<DT>::Acc(0));
    }
}

}  // namespace ravel
