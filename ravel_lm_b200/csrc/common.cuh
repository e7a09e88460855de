// common.cuh -- shared device helpers of the RAVEL event-memory kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/ravel_b200.h"

namespace ravel {

// ----------------------------------------------------------------- device error word
// One word per device; kernels OR RAVEL_DEVERR_* bits into it.  Never traps.
__device__ unsigned int g_error_word = 0u;

__device__ __forceinline__ void flag_error(unsigned int bits) { atomicOr(&g_error_word, bits); }

// Polls a wait on another block's flag may take before it gives up (sets
// RAVEL_DEVERR_SPIN and returns); one per device, set by ravel_set_wait_limit.
__device__ unsigned int g_wait_limit = 1u << 22;

// ----------------------------------------------------------------- memory-order helpers
__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release(unsigned int* p, unsigned int v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until *p (published by another block with st_release) is nonzero and
// return it; after g_wait_limit polls give up, flag RAVEL_DEVERR_SPIN and
// return 0.  Every look-back wait of the scans goes through here.
__device__ __forceinline__ unsigned int wait_flag(const unsigned int* p, unsigned int sleep_ns) {
    const unsigned int limit = *const_cast<volatile unsigned int*>(&g_wait_limit);
    unsigned int f, spins = 0;
    while ((f = ld_acquire(p)) == 0u) {
        if (++spins > limit) {
            flag_error(RAVEL_DEVERR_SPIN);
            return 0u;
        }
        __nanosleep(sleep_ns);
    }
    return f;
}

// Streaming (evict-first) 16-byte store: the latest-k outputs are written once
// and never re-read by the producing kernel.
__device__ __forceinline__ void st_cs_v4(void* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
                 "r"(v.z), "r"(v.w)
                 : "memory");
}

// Read-only 16-byte load through the non-coherent path.
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Asynchronous global->shared copies (16 / 8 / 4 bytes), committed as one group.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
    unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
    unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// 32-bit shared-memory address of a generic pointer into shared memory.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// One warp waits on a flag with the scans' own bounded wait (ravel_wait_selftest):
// given a word nothing sets, the wait gives up and RAVEL_DEVERR_SPIN comes back.
__global__ void k_wait_selftest(const unsigned int* flag) { (void)wait_flag(flag, 32); }

// ----------------------------------------------------------------- address folding
// ravel_lm/ravel_memory.py:127-128: .to(key_dtype).remainder(A).  With int32 keys
// (B*C*A*(T+1) <= 2^31-1) an int64 address is first truncated to 32 bits.
__device__ __forceinline__ int64_t load_addr(const void* base, int64_t i, int addr_i64) {
    return addr_i64 ? static_cast<const int64_t*>(base)[i]
                    : static_cast<int64_t>(static_cast<const int32_t*>(base)[i]);
}

__device__ __forceinline__ uint64_t fold_addr(int64_t a, int64_t A, int key32) {
    if (key32) a = static_cast<int64_t>(static_cast<int32_t>(static_cast<uint32_t>(a)));
    // in-range addresses (the usual case) and power-of-two spaces need no division
    if (a >= 0 && a < A) return static_cast<uint64_t>(a);
    if ((A & (A - 1)) == 0) return static_cast<uint64_t>(a & (A - 1));
    int64_t r = a % A;
    if (r < 0) r += A;
    return static_cast<uint64_t>(r);
}

// torch's remainder of an int64 by a positive A (floor modulo).
__device__ __forceinline__ int64_t floor_mod(int64_t x, int64_t A) {
    const int64_t r = x % A;
    return r < 0 ? r + A : r;
}

// Literal address family j of token t in batch row b (ravel_lm/model.py:195-231):
//   0: tok;  1: prev1*257 + tok*131 + 17;  2: prev2*65537 + prev1*257 + tok*131 + 31;
//   j >= 3: tok*(1009 + 2j) + t*(9176 + j) + 97j;  all mod A (floor), with the
// previous tokens taken as bos before the sequence starts.  The products wrap in
// 64 bits, as torch's int64 arithmetic does.
__device__ __forceinline__ int64_t literal_addr(const int64_t* tokens, int64_t T, int64_t b, int64_t t, int j,
                                                int64_t bos, int64_t A) {
    const int64_t* row = tokens + b * T;
    const uint64_t x = static_cast<uint64_t>(row[t]);
    if (j == 0) return floor_mod(static_cast<int64_t>(x), A);
    const uint64_t p1 = static_cast<uint64_t>(t >= 1 ? row[t - 1] : bos);
    if (j == 1) return floor_mod(static_cast<int64_t>(p1 * 257u + x * 131u + 17u), A);
    const uint64_t p2 = static_cast<uint64_t>(t >= 2 ? row[t - 2] : bos);
    if (j == 2) return floor_mod(static_cast<int64_t>(p2 * 65537u + p1 * 257u + x * 131u + 31u), A);
    const uint64_t uj = static_cast<uint64_t>(j);
    return floor_mod(static_cast<int64_t>(x * (1009u + 2u * uj) + static_cast<uint64_t>(t) * (9176u + uj) + uj * 97u),
                     A);
}

// Where the address of event (b, t, c) comes from: a [B, T, C] integer tensor, or
// (token mode, tokens != null) the literal families of the token ids for the
// first `lit` heads and a [B, T, C - lit] tensor of learned addresses for the rest
// -- the concatenation of ravel_lm/model.py:347-349, never materialised.
struct AddrSrc {
    const void* addr;       // plain: [B, T, C]; token mode: [B, T, C - lit] (null when C == lit)
    int i64;                // addr holds int64 (else int32)
    const int64_t* tokens;  // token mode: [B, T] token ids
    int lit;
    int64_t bos;
};

__device__ __forceinline__ int64_t src_addr(const AddrSrc& s, int64_t b, int64_t t, int64_t c, int64_t T,
                                            int64_t C, int64_t A) {
    if (s.tokens == nullptr) return load_addr(s.addr, (b * T + t) * C + c, s.i64);
    if (c < s.lit) return literal_addr(s.tokens, T, b, t, static_cast<int>(c), s.bos, A);
    const int64_t Cl = C - s.lit;
    return load_addr(s.addr, (b * T + t) * Cl + (c - s.lit), s.i64);
}

// Decode-cache addresses are clamped, not wrapped (ravel_memory.py:276, :289).
__device__ __forceinline__ int64_t clamp_addr(int64_t a, int64_t A) {
    return a < 0 ? 0 : (a > A - 1 ? A - 1 : a);
}

// ----------------------------------------------------------------- payload dtypes
// Element traits: storage type, accumulation type and conversions.
template <int DT> struct Elem;
template <> struct Elem<RAVEL_F32> {
    using T = float; using Acc = float;
    static __device__ __forceinline__ Acc to_acc(T v) { return v; }
    static __device__ __forceinline__ T from_acc(Acc v) { return v; }
};
template <> struct Elem<RAVEL_BF16> {
    using T = __nv_bfloat16; using Acc = float;
    static __device__ __forceinline__ Acc to_acc(T v) { return __bfloat162float(v); }
    static __device__ __forceinline__ T from_acc(Acc v) { return __float2bfloat16_rn(v); }
};
template <> struct Elem<RAVEL_F16> {
    using T = __half; using Acc = float;
    static __device__ __forceinline__ Acc to_acc(T v) { return __half2float(v); }
    static __device__ __forceinline__ T from_acc(Acc v) { return __float2half_rn(v); }
};
template <> struct Elem<RAVEL_F64> {
    using T = double; using Acc = double;
    static __device__ __forceinline__ Acc to_acc(T v) { return v; }
    static __device__ __forceinline__ T from_acc(Acc v) { return v; }
};

inline int elem_bytes(int dt) { return dt == RAVEL_F32 ? 4 : (dt == RAVEL_F64 ? 8 : 2); }

// Two packed 16-bit elements (low half first) to floats.
template <typename V> __device__ __forceinline__ float2 pair_to_float2(uint32_t w);
template <> __device__ __forceinline__ float2 pair_to_float2<__nv_bfloat16>(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
}
template <> __device__ __forceinline__ float2 pair_to_float2<__half>(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// candidate * 0 on raw bits (ravel_memory.py:175, :280): a finite value keeps only
// its sign bit (+-0); Inf/NaN become the dtype's canonical quiet NaN.
template <int DT> __device__ __forceinline__ uint32_t zero_word(uint32_t w);
template <> __device__ __forceinline__ uint32_t zero_word<RAVEL_F32>(uint32_t w) {
    return ((w & 0x7f800000u) == 0x7f800000u) ? 0x7fc00000u : (w & 0x80000000u);
}
__device__ __forceinline__ uint32_t zero_half_pair(uint32_t w, uint32_t expmask, uint32_t qnan) {
    uint32_t lo = w & 0xffffu, hi = w >> 16;
    lo = ((lo & expmask) == expmask) ? qnan : (lo & 0x8000u);
    hi = ((hi & expmask) == expmask) ? qnan : (hi & 0x8000u);
    return lo | (hi << 16);
}
template <> __device__ __forceinline__ uint32_t zero_word<RAVEL_BF16>(uint32_t w) {
    return zero_half_pair(w, 0x7f80u, 0x7fc0u);
}
template <> __device__ __forceinline__ uint32_t zero_word<RAVEL_F16>(uint32_t w) {
    return zero_half_pair(w, 0x7c00u, 0x7e00u);
}
// float64 is handled on 32-bit word pairs: the high word carries sign and exponent.
__device__ __forceinline__ void zero_f64_pair(uint32_t& lo, uint32_t& hi) {
    if ((hi & 0x7ff00000u) == 0x7ff00000u) { hi = 0x7ff80000u; lo = 0u; }
    else { hi &= 0x80000000u; lo = 0u; }
}

// candidate * 0 on a whole 32-bit word at once (two 16-bit elements, or one
// float): a half's exponent field is all ones exactly when adding one unit to
// it carries into bit 15, so the non-finite halves are found without branches.
template <int DT> __device__ __forceinline__ uint32_t zero_word_packed(uint32_t w) {
    if constexpr (DT == RAVEL_F32) {
        const uint32_t nf = ((w & 0x7f800000u) + 0x00800000u) & 0x80000000u;
        return nf ? 0x7fc00000u : (w & 0x80000000u);
    } else {
        constexpr uint32_t EXP = DT == RAVEL_BF16 ? 0x7f807f80u : 0x7c007c00u;
        constexpr uint32_t ONE = DT == RAVEL_BF16 ? 0x00800080u : 0x04000400u;
        constexpr uint32_t QNAN = DT == RAVEL_BF16 ? 0x7fc07fc0u : 0x7e007e00u;
        const uint32_t nf = ((w & EXP) + ONE) & 0x80008000u;
        const uint32_t mm = (nf >> 15) * 0xffffu;  // all ones over each non-finite half
        return (mm & QNAN) | (w & 0x80008000u & ~mm);
    }
}

// Zero a vector of VB bytes (VB in {2, 4, 8, 16}) held as 32-bit words.
template <int DT, int VB> struct VecZero {
    static __device__ __forceinline__ uint4 apply(uint4 v) {
        if constexpr (DT == RAVEL_F64) {
            zero_f64_pair(v.x, v.y);
            if constexpr (VB == 16) zero_f64_pair(v.z, v.w);
        } else {
            v.x = zero_word<DT>(v.x);
            if constexpr (VB >= 8) v.y = zero_word<DT>(v.y);
            if constexpr (VB == 16) { v.z = zero_word<DT>(v.z); v.w = zero_word<DT>(v.w); }
        }
        return v;
    }
};
template <int DT> struct VecZero<DT, 2> {
    static __device__ __forceinline__ uint4 apply(uint4 v) {
        // one 16-bit element in the low half
        if constexpr (DT == RAVEL_BF16) {
            v.x = ((v.x & 0x7f80u) == 0x7f80u) ? 0x7fc0u : (v.x & 0x8000u);
        } else {
            v.x = ((v.x & 0x7c00u) == 0x7c00u) ? 0x7e00u : (v.x & 0x8000u);
        }
        return v;
    }
};

// Load / store VB bytes as a uint4 (unused words are zero).
template <int VB> __device__ __forceinline__ uint4 ld_vec(const void* p) {
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if constexpr (VB == 16) v = *static_cast<const uint4*>(p);
    else if constexpr (VB == 8) { uint2 t = *static_cast<const uint2*>(p); v.x = t.x; v.y = t.y; }
    else if constexpr (VB == 4) v.x = *static_cast<const uint32_t*>(p);
    else v.x = *static_cast<const uint16_t*>(p);
    return v;
}
template <int VB> __device__ __forceinline__ uint4 ldg_vec(const void* p) {
    if constexpr (VB == 16) return ld_nc_v4(p);
    else return ld_vec<VB>(p);
}
template <int VB> __device__ __forceinline__ void st_vec(void* p, uint4 v) {
    if constexpr (VB == 16) *static_cast<uint4*>(p) = v;
    else if constexpr (VB == 8) *static_cast<uint2*>(p) = make_uint2(v.x, v.y);
    else if constexpr (VB == 4) *static_cast<uint32_t*>(p) = v.x;
    else *static_cast<uint16_t*>(p) = static_cast<uint16_t>(v.x);
}
template <int VB> __device__ __forceinline__ void st_vec_stream(void* p, uint4 v) {
    if constexpr (VB == 16) st_cs_v4(p, v);
    else st_vec<VB>(p, v);
}

// Widest vector width (bytes) that divides a row of `row_bytes` and the base
// alignment of every pointer involved.
inline int pick_vec_bytes(int64_t row_bytes, uintptr_t align_bits) {
    for (int vb = 16; vb >= 2; vb >>= 1) {
        if (row_bytes % vb == 0 && (align_bits % vb) == 0) return vb;
    }
    return 2;
}

// ----------------------------------------------------------------- key layout
// Per-stream event key: [invalid bit][address bits][time bits].  Keys are unique
// within a stream because the time field is unique; sorting them is a stable
// sort by address of a time-ordered sequence.
struct KeyLayout {
    int tbits;   // bits of the time field
    int abits;   // bits of the address field
    int mbit;    // 1 when a write mask is present (invalid bit above the address)
    int key64;   // keys need 64 bits
};

inline int bits_for(uint64_t n) {  // bits to hold values 0..n-1 (n >= 1)
    int b = 0;
    while (b < 64 && (uint64_t(1) << b) < n) ++b;
    return b;
}

inline KeyLayout key_layout(int64_t T, int64_t A, int has_mask) {
    KeyLayout L;
    L.tbits = bits_for(static_cast<uint64_t>(T > 1 ? T : 1));
    if (L.tbits == 0) L.tbits = 1;
    L.abits = bits_for(static_cast<uint64_t>(A));
    L.mbit = has_mask ? 1 : 0;
    L.key64 = (L.tbits + L.abits + L.mbit) > 32 ? 1 : 0;
    return L;
}

inline size_t align_up(size_t x, size_t a = 256) { return (x + a - 1) / a * a; }

// Unsigned division by a run-time constant through a multiply-high and a shift
// (the round-up reciprocal method of Granlund & Montgomery, PLDI 1994).  Exact
// for numerators below 2^31, which every in-kernel index it is used on is.
struct FastDiv {
    uint32_t d, m, s;
    FastDiv() : d(1), m(0), s(0) {}
    explicit FastDiv(uint32_t div) : d(div) {
        s = 0;
        while ((uint64_t(1) << s) < div) ++s;
        m = static_cast<uint32_t>(((uint64_t(1) << 32) * ((uint64_t(1) << s) - div)) / div + 1);
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        return static_cast<uint32_t>((static_cast<uint64_t>(__umulhi(n, m)) + n) >> s);
    }
    __device__ __forceinline__ void divmod(uint32_t n, uint32_t& q, uint32_t& r) const {
        q = div(n);
        r = n - q * d;
    }
};

}  // namespace ravel
