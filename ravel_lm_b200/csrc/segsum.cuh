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

    // tape positions in scan order
    for (int i = tid; i < np; i += SCAN_THREADS) {
        const int64_t si = i0 + i;
        const int64_t p = a.reverse ? (n_s - 1 - si) : si;
        const KeyT key = keys[p];
        sadr[i] = static_cast<uint64_t>(key >> a.tbits);
        srow[i] = flat_row(s, static_cast<int64_t>(key & tmask), T, C);
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
        const int stop = term ? __ffs(term) - 1 : 31;
        for (int c = 0; c <= stop; ++c) {
            const unsigned fc = __shfl_sync(0xffffffffu, f, c);
            const int64_t jc = j - c;
            if (jc < jmin || fc == 3u) break;
            const Acc* src = (fc == 2u) ? incl + jc * D : agg + jc * D;
            if (active) {
#pragma unroll
                for (int q = 0; q < EL; ++q) cin[q] += src[col + q];
            }
        }
        if (term) return;
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
        my_flat = static_cast<uint32_t>(flat_row(s, static_cast<int64_t>(key & tmask), T, C));
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

// ------------------------------------------------------------------ TMA-staged scan
// The scan kernel for rows that are whole multiples of 16 bytes.  A CTA of 8
// warps takes a chunk of 256 tape positions (one ticket).  Warp 0 issues one
// TMA bulk copy (cp.async.bulk, no multicast) per row into shared memory on an
// mbarrier; the rows then sit in shared memory, not registers, so ~7 CTAs per
// SM keep ~200 KB of loads in flight and hide the look-back latency of their
// neighbours.  Warp w scans positions [32w, 32w+32) with lanes over columns
// (pass 1 stores every position from the warp's first segment start on),
// warp 0 folds the warp sums, publishes the chunk and looks back (windowed),
// and warps whose head continues a segment rescan it with their carry (pass 2).
constexpr int SCANT_WARPS = 8;
constexpr int SCANT_P = SCANT_WARPS * 32;
constexpr uint32_t TMA_WAIT_LIMIT = 1u << 24;

template <typename KeyT, int DT, int EL, bool IN_SORTED, bool OUT_SORTED>
__global__ void __launch_bounds__(SCANT_WARPS * 32) k_segscan_t(ScanArgs<typename Elem<DT>::Acc> a) {
    using E = Elem<DT>;
    using Acc = typename E::Acc;
    using V = typename E::T;
    using InT = typename std::conditional<IN_SORTED, Acc, V>::type;
    using OutT = typename std::conditional<OUT_SORTED, Acc, V>::type;
    constexpr int NW = SCANT_WARPS;
    constexpr int P = SCANT_P;
    extern __shared__ __align__(16) unsigned char smem[];
    const uint32_t D = static_cast<uint32_t>(a.D);
    const uint32_t rb = D * static_cast<uint32_t>(sizeof(InT));  // input row bytes (multiple of 16)
    InT* rows = reinterpret_cast<InT*>(smem);                     // [P][D]
    Acc* wagg = reinterpret_cast<Acc*>(smem + static_cast<size_t>(P) * rb);  // [NW][D]
    Acc* carry = wagg + NW * D;                                   // [D]
    __shared__ __align__(8) uint64_t s_bar;
    __shared__ unsigned s_ticket;
    __shared__ unsigned s_startmask[NW];
    __shared__ uint32_t s_in[P];
    __shared__ uint32_t s_out[P];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        s_ticket = atomicAdd(a.ticket, 1u);
        mbar_init(&s_bar, 1);
    }
    __syncthreads();
    const int64_t L = s_ticket;
    const int64_t s = L / a.nchunks;
    const int64_t ch = L % a.nchunks;
    const int64_t T = a.T, C = a.C;
    const int64_t n_s = a.nvalid ? a.nvalid[s] : T;
    const int64_t i0 = ch * P;
    if (i0 >= n_s) return;  // beyond this stream's tape; no later chunk waits on it
    const int np = static_cast<int>(n_s - i0 < P ? n_s - i0 : P);
    const KeyT* keys = static_cast<const KeyT*>(a.keys) + s * T;
    const KeyT tmask = (static_cast<KeyT>(1) << a.tbits) - 1;

    // keys -> row indices and segment starts (position i = tid)
    bool my_start = false;
    uint32_t my_flat = 0;
    if (tid < np) {
        const int64_t si = i0 + tid;
        const int64_t p = a.reverse ? (n_s - 1 - si) : si;
        const KeyT key = keys[p];
        my_flat = static_cast<uint32_t>(flat_row(s, static_cast<int64_t>(key & tmask), T, C));
        const uint32_t tix = static_cast<uint32_t>(s * T + p);
        s_in[tid] = IN_SORTED ? tix : my_flat;
        s_out[tid] = OUT_SORTED ? tix : my_flat;
        if (si == 0) {
            my_start = true;
        } else {
            const int64_t pp = a.reverse ? (n_s - si) : (si - 1);
            my_start = (keys[pp] >> a.tbits) != (key >> a.tbits);
        }
    }
    const unsigned startmask = __ballot_sync(0xffffffffu, my_start);
    if (a.out_mask != nullptr && tid < np) a.out_mask[my_flat] = my_start ? 0 : 1;
    __syncthreads();

    // TMA: one bulk copy per row, all on one mbarrier
    const InT* in = static_cast<const InT*>(a.in);
    if (warp == 0) {
        if (lane == 0) mbar_arrive_expect_tx(&s_bar, static_cast<uint32_t>(np) * rb);
        __syncwarp();
        for (int r = lane; r < np; r += 32)
            tma_load_1d(rows + static_cast<size_t>(r) * D, in + static_cast<uint64_t>(s_in[r]) * D, rb, &s_bar);
    }
    bool loaded = mbar_wait_bounded(&s_bar, 0, TMA_WAIT_LIMIT);
    if (!loaded) mbar_wait_bounded(&s_bar, 0, TMA_WAIT_LIMIT);  // let copies in flight land before exit

    const int w0 = warp * 32;
    const int nv = np - w0 < 0 ? 0 : (np - w0 < 32 ? np - w0 : 32);
    const int first = startmask ? __ffs(startmask) - 1 : 32;
    const bool active = static_cast<uint32_t>(lane * EL) < D;
    const uint32_t col = static_cast<uint32_t>(lane * EL);
    OutT* out = static_cast<OutT*>(a.out);

    // pass 1
    Acc run[EL];
#pragma unroll
    for (int q = 0; q < EL; ++q) run[q] = Acc(0);
    if (loaded) {
        for (int i = 0; i < nv; ++i) {
            const bool st = (startmask >> i) & 1u;
            const RawWords<EL * sizeof(InT)> x = ld_frag_smem<InT, EL>(rows + static_cast<size_t>(w0 + i) * D + col);
            RawWords<EL * sizeof(OutT)> o;
            OutT* ov = reinterpret_cast<OutT*>(&o.w[0]);
#pragma unroll
            for (int q = 0; q < EL; ++q) {
                if (st) run[q] = Acc(0);
                const Acc v = active ? frag_get<InT, Acc, EL>(x, q) : Acc(0);
                if (a.inclusive) { run[q] += v; ov[q] = acc_to<OutT, Acc>(run[q]); }
                else { ov[q] = acc_to<OutT, Acc>(run[q]); run[q] += v; }
            }
            if (i >= first && active) st_frag<OutT, EL>(out + static_cast<uint64_t>(s_out[w0 + i]) * D + col, o);
        }
    }
    if (active) {
#pragma unroll
        for (int q = 0; q < EL; ++q) wagg[warp * D + col + q] = run[q];
    }
    if (lane == 0) s_startmask[warp] = nv > 0 ? startmask : 0u;
    __syncthreads();

    int m = NW;
#pragma unroll
    for (int w = NW - 1; w >= 0; --w) if (s_startmask[w] != 0u) m = w;
    const bool head_continues = (s_startmask[0] & 1u) == 0u;
    const int waiters = (m < NW ? m : NW - 1) + 1;

    if (warp == 0) {
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
    if (head_continues && warp < waiters && waiters > 1) named_barrier(waiters * 32);

    // pass 2: head positions [0, first) of the warp with their carry-in
    if (first > 0 && nv > 0 && loaded) {
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
        const int hn = first < nv ? first : nv;
        for (int i = 0; i < hn; ++i) {
            const RawWords<EL * sizeof(InT)> x = ld_frag_smem<InT, EL>(rows + static_cast<size_t>(w0 + i) * D + col);
            RawWords<EL * sizeof(OutT)> o;
            OutT* ov = reinterpret_cast<OutT*>(&o.w[0]);
#pragma unroll
            for (int q = 0; q < EL; ++q) {
                const Acc v = active ? frag_get<InT, Acc, EL>(x, q) : Acc(0);
                if (a.inclusive) { cin[q] += v; ov[q] = acc_to<OutT, Acc>(cin[q]); }
                else { ov[q] = acc_to<OutT, Acc>(cin[q]); cin[q] += v; }
            }
            if (active) st_frag<OutT, EL>(out + static_cast<uint64_t>(s_out[w0 + i]) * D + col, o);
        }
    }
}

template <typename Acc>
inline size_t segscan_t_smem(int64_t D, size_t in_elem) {
    return static_cast<size_t>(SCANT_P) * D * in_elem + static_cast<size_t>(SCANT_WARPS + 1) * D * sizeof(Acc);
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
};

template <typename KeyT>
__device__ __forceinline__ bool ss_valid(const SsGenArgs& a, int64_t r, int64_t& tape_index) {
    const int64_t T = a.T, C = a.C;
    const int64_t c = r % C, b = r / (C * T);
    const int64_t s = b * C + c;
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
