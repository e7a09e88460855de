// cache.cuh -- decode-time latest-value cache (RavelLayerCache).
//
// Reference: ravel_lm/ravel_memory.py:244-292.  values [B, C, A, D] and
// filled [B, C, A]; read gathers the row at the clamped address and multiplies
// it by the filled bit, write scatters the new row and sets the bit.  One
// decode step of a memory layer reads then writes (ravel_lm/model.py:421-424);
// k_cache_step does both in one launch with the read ordered before the write
// for every (b, c) pair.  Rows move as VB-byte vectors; each CTA owns whole
// pairs so the read-then-write order needs only a block barrier.
#pragma once

#include "common.cuh"

namespace ravel {

struct CacheArgs {
    void* values;            // [B*C, A, D]
    uint8_t* filled;         // [B*C, A]
    const void* raddr;       // [B*C] or null
    const void* waddr;       // [B*C] or null
    int addr_i64;
    const void* payload;     // [B*C, D] (write)
    void* out_vals;          // [B*C, D] (read)
    uint8_t* out_mask;       // [B*C]    (read)
    int64_t pairs, A, row_bytes;
    int pairs_per_cta;
    FastDiv fd_rv;
};

template <int DT, int VB>
__global__ void __launch_bounds__(256) k_cache_step(CacheArgs a) {
    const uint32_t rv = static_cast<uint32_t>(a.row_bytes / VB);
    const int64_t pr0 = static_cast<int64_t>(blockIdx.x) * a.pairs_per_cta;
    const int64_t npr = (a.pairs - pr0) < a.pairs_per_cta ? (a.pairs - pr0) : a.pairs_per_cta;
    char* vals = static_cast<char*>(a.values);
    // read phase
    if (a.raddr != nullptr) {
        for (uint32_t e = threadIdx.x; e < static_cast<uint32_t>(npr) * rv; e += blockDim.x) {
            uint32_t i, v;
            a.fd_rv.divmod(e, i, v);
            const int64_t pr = pr0 + i;
            const int64_t idx = clamp_addr(load_addr(a.raddr, pr, a.addr_i64), a.A);
            const bool f = a.filled[pr * a.A + idx] != 0;
            uint4 x = ld_vec<VB>(vals + (pr * a.A + idx) * a.row_bytes + v * VB);
            if (!f) x = VecZero<DT, VB>::apply(x);
            st_vec<VB>(static_cast<char*>(a.out_vals) + pr * a.row_bytes + v * VB, x);
        }
        for (int64_t i = threadIdx.x; i < npr; i += blockDim.x) {
            const int64_t pr = pr0 + i;
            const int64_t idx = clamp_addr(load_addr(a.raddr, pr, a.addr_i64), a.A);
            a.out_mask[pr] = a.filled[pr * a.A + idx] != 0 ? 1 : 0;
        }
    }
    if (a.waddr == nullptr) return;
    if (a.raddr != nullptr) __syncthreads();
    // write phase
    for (uint32_t e = threadIdx.x; e < static_cast<uint32_t>(npr) * rv; e += blockDim.x) {
        uint32_t i, v;
        a.fd_rv.divmod(e, i, v);
        const int64_t pr = pr0 + i;
        const int64_t idx = clamp_addr(load_addr(a.waddr, pr, a.addr_i64), a.A);
        const uint4 x = ld_vec<VB>(static_cast<const char*>(a.payload) + pr * a.row_bytes + v * VB);
        st_vec<VB>(vals + (pr * a.A + idx) * a.row_bytes + v * VB, x);
    }
    for (int64_t i = threadIdx.x; i < npr; i += blockDim.x) {
        const int64_t pr = pr0 + i;
        const int64_t idx = clamp_addr(load_addr(a.waddr, pr, a.addr_i64), a.A);
        a.filled[pr * a.A + idx] = 1;
    }
}

// Bulk prefill: every stream's writes are sorted by (clamped address, t); the
// last write of each address segment is the one a token-by-token prefill leaves
// in the cache.  One thread per sorted position copies that write's payload row
// into values[b, c, address] (VB bytes at a time) and sets filled.  Each cache
// entry has at most one writer, so there are no races.
template <typename KeyT, int VB>
__global__ void __launch_bounds__(256) k_cache_prefill(const KeyT* keys, int64_t S, int64_t T, int64_t C, int64_t A,
                                                       int tbits, const void* payload, int64_t row_bytes,
                                                       void* values, uint8_t* filled) {
    const KeyT tmask = (static_cast<KeyT>(1) << tbits) - 1;
    for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; e < S * T;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t s = e / T, p = e - s * T;
        const KeyT key = keys[e];
        if (p + 1 < T && (keys[e + 1] >> tbits) == (key >> tbits)) continue;  // a later write of this address
        const int64_t b = s / C, c = s - b * C;
        const int64_t t = static_cast<int64_t>(key & tmask);
        const int64_t addr = static_cast<int64_t>(key >> tbits);
        const char* src = static_cast<const char*>(payload) + ((b * T + t) * C + c) * row_bytes;
        char* dst = static_cast<char*>(values) + (s * A + addr) * row_bytes;
        for (int64_t o = 0; o < row_bytes; o += VB) st_vec<VB>(dst + o, ldg_vec<VB>(src + o));
        filled[s * A + addr] = 1;
    }
}

}  // namespace ravel
