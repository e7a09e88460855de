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
