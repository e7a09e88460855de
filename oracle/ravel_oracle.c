/*
 * ravel_oracle.c -- CPU restatement of RAVEL's exact event-memory operator.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library in
 * ravel_lm_b200/csrc.  Only tests/, __graft_entry__.smoke() and bench.py's
 * reference ("cpu_baseline") leg may load it.  The product path never calls
 * it and has no CPU fallback.
 *
 * It follows the steps of the reference operator (file:line relative to the
 * ravel-lm project):
 *   ravel_lm/ravel_memory.py:45-49   key dtype: int32 iff B*C*A*(T+1) <= 2^31-1
 *   ravel_lm/ravel_memory.py:127-128 addresses .to(key_dtype).remainder(A)
 *   ravel_lm/ravel_memory.py:26-38   composite base (b*C + c)*A + addr
 *   ravel_lm/ravel_memory.py:133-135 write key = base*(T+1) + t
 *   ravel_lm/ravel_memory.py:139-144 write_mask compaction (broadcast over C)
 *   ravel_lm/ravel_memory.py:146-149 no writes left -> zeros + false
 *   ravel_lm/ravel_memory.py:151     sort of the write keys
 *   ravel_lm/ravel_memory.py:153-159 read key = base*(T+1) + (t-1);
 *                                    latest = searchsorted(right=True) - 1
 *   ravel_lm/ravel_memory.py:160-168 k candidates latest-j, valid if >= 0 and
 *                                    same composite base
 *   ravel_lm/ravel_memory.py:173-176 gather order[safe] * valid
 *   ravel_lm/ravel_memory.py:216-229 segmented cumulative sum over the sorted tape
 *   ravel_lm/ravel_memory.py:235-241 sum lookup = segcum[safe] * valid
 * Backward passes restate the autograd of those expressions:
 *   latest-k: index_select backward = index_add of grad_out*valid into order[safe]
 *   sum:      index_add into the sorted tape, reverse segmented cumsum, unpermute.
 *
 * Deliberate differences (documented, none changes a value that is compared
 * bit-for-bit):
 *   - The global sort is done per stream (b, c) and concatenated in stream
 *     order.  The stream id is the most significant part of every key
 *     (ravel_memory.py:26-38), so the concatenation IS the global sorted order.
 *   - Sums and all gradients are accumulated in double, i.e. this is the
 *     reference evaluated on payloads.double().  The segmented sum is a running
 *     sum reset at each segment start instead of "global cumsum minus the
 *     cumsum before the segment start" (same value up to rounding; the running
 *     form is the more accurate of the two and is the better checker).
 *   - Keys are always held in int64.  When the reference uses int32 keys every
 *     key fits in int32, so the order is identical.  The one visible effect of
 *     the int32 key dtype -- int64 addresses are truncated to 32 bits before the
 *     remainder (ravel_memory.py:127) -- is reproduced by oracle_fold_address().
 *
 * Payload element codes: 0 = float32, 1 = bfloat16, 2 = float16, 3 = float64.
 * Latest-k values are copied as raw element bits.  An invalid slot holds
 * candidate*0 (ravel_memory.py:175): +-0 with the candidate's sign bit for a
 * finite candidate, a quiet NaN otherwise.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static int64_t floor_mod(int64_t a, int64_t m) {
    int64_t r = a % m;
    if (r < 0) r += m;
    return r;
}

/* ravel_memory.py:127-128: .to(key_dtype).remainder(A).  With int32 keys an
 * int64 address is first truncated to its low 32 bits (two's complement). */
int64_t oracle_fold_address(int64_t a, int64_t A, int key32) {
    if (key32) a = (int64_t)(int32_t)(uint32_t)(uint64_t)a;
    return floor_mod(a, A);
}

/* ravel_memory.py:45-49 */
int oracle_key_is_int32(int64_t B, int64_t T, int64_t C, int64_t A) {
    /* the product can exceed int64 only for absurd sizes; use long double */
    long double bound = (long double)B * (long double)C * (long double)A * (long double)(T + 1);
    return bound <= 2147483647.0L ? 1 : 0;
}

static int cmp_i64(const void* x, const void* y) {
    int64_t a = *(const int64_t*)x, b = *(const int64_t*)y;
    return (a > b) - (a < b);
}

/*
 * Build the sorted write tape and the per-read search result.
 *
 *   sorted_keys[0..nw)  composite keys in ascending order (ravel_memory.py:151)
 *   order[0..nw)        flat row (b*T + t)*C + c of each sorted write
 *   latest[r]           searchsorted(sorted_keys, read_key[r], right=True) - 1
 *   read_base[r]        composite base of read r (ravel_memory.py:153,157)
 * Returns nw, the number of unmasked writes.
 */
int64_t oracle_tape(const int64_t* waddr, const int64_t* raddr, const uint8_t* wmask,
                    int64_t B, int64_t T, int64_t C, int64_t A, int key32,
                    int64_t* sorted_keys, int64_t* order, int64_t* latest,
                    int64_t* read_base) {
    const int64_t S = B * C;
    const int64_t N = B * T * C;
    int64_t* counts = (int64_t*)calloc((size_t)(S + 1), sizeof(int64_t));
    /* per-stream write counts (mask broadcast over heads, :142) */
    for (int64_t b = 0; b < B; ++b) {
        int64_t n = 0;
        for (int64_t t = 0; t < T; ++t) n += wmask ? (wmask[b * T + t] != 0) : 1;
        for (int64_t c = 0; c < C; ++c) counts[b * C + c + 1] = n;
    }
    for (int64_t s = 0; s < S; ++s) counts[s + 1] += counts[s];
    const int64_t nw = counts[S];

#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t s = 0; s < S; ++s) {
        const int64_t b = s / C, c = s % C;
        int64_t* kk = sorted_keys + counts[s];
        int64_t n = 0;
        for (int64_t t = 0; t < T; ++t) {
            if (wmask && !wmask[b * T + t]) continue;
            const int64_t a = oracle_fold_address(waddr[(b * T + t) * C + c], A, key32);
            const int64_t base = (b * C + c) * A + a;            /* :26-38 */
            kk[n++] = base * (T + 1) + t;                         /* :133-135 */
        }
        qsort(kk, (size_t)n, sizeof(int64_t), cmp_i64);           /* :151 */
        for (int64_t i = 0; i < n; ++i) {
            const int64_t key = kk[i];
            const int64_t t = key % (T + 1);
            order[counts[s] + i] = (b * T + t) * C + c;
        }
    }

#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < N; ++r) {
        const int64_t c = r % C, t = (r / C) % T, b = r / (C * T);
        const int64_t a = oracle_fold_address(raddr[r], A, key32);
        const int64_t base = (b * C + c) * A + a;
        const int64_t key = base * (T + 1) + (t - 1);                /* :155 */
        /* searchsorted(right=True): first index with sorted_keys[i] > key */
        int64_t lo = 0, hi = nw;
        while (lo < hi) {
            const int64_t mid = lo + (hi - lo) / 2;
            if (sorted_keys[mid] <= key) lo = mid + 1; else hi = mid;
        }
        latest[r] = lo - 1;                                          /* :159 */
        read_base[r] = base;
    }
    free(counts);
    return nw;
}

/* candidate * 0 for one element of the given dtype (ravel_memory.py:175) */
static void zero_like(const unsigned char* src, unsigned char* dst, int dtype) {
    switch (dtype) {
    case 0: { uint32_t v; memcpy(&v, src, 4);
              uint32_t o = ((v & 0x7f800000u) == 0x7f800000u) ? 0x7fc00000u : (v & 0x80000000u);
              memcpy(dst, &o, 4); break; }
    case 1: { uint16_t v; memcpy(&v, src, 2);
              uint16_t o = ((v & 0x7f80u) == 0x7f80u) ? 0x7fc0u : (uint16_t)(v & 0x8000u);
              memcpy(dst, &o, 2); break; }
    case 2: { uint16_t v; memcpy(&v, src, 2);
              uint16_t o = ((v & 0x7c00u) == 0x7c00u) ? 0x7e00u : (uint16_t)(v & 0x8000u);
              memcpy(dst, &o, 2); break; }
    default: { uint64_t v; memcpy(&v, src, 8);
               uint64_t o = ((v & 0x7ff0000000000000ull) == 0x7ff0000000000000ull)
                                ? 0x7ff8000000000000ull : (v & 0x8000000000000000ull);
               memcpy(dst, &o, 8); break; }
    }
}

static int dtype_size(int dtype) {
    return dtype == 0 ? 4 : (dtype == 3 ? 8 : 2);
}

/*
 * Latest-k forward (ravel_memory.py:146-176).
 *   out_vals [N, k, D] (payload dtype), out_mask [N, k], out_src [N, k]:
 *   the flat payload row each slot was gathered from (the clamped candidate,
 *   also for invalid slots), or -1 when there are no writes at all.
 */
int oracle_latestk_fwd(const int64_t* sorted_keys, const int64_t* order,
                       const int64_t* latest, const int64_t* read_base, int64_t nw,
                       const void* payload, int dtype, int64_t N, int64_t T, int64_t D,
                       int64_t k, void* out_vals, uint8_t* out_mask, int64_t* out_src) {
    const int es = dtype_size(dtype);
    const size_t row = (size_t)D * (size_t)es;
    const unsigned char* p = (const unsigned char*)payload;
    unsigned char* o = (unsigned char*)out_vals;
    if (nw == 0) {                                                   /* :146-149 */
        memset(out_vals, 0, (size_t)N * (size_t)k * row);
        memset(out_mask, 0, (size_t)N * (size_t)k);
        for (int64_t i = 0; i < N * k; ++i) out_src[i] = -1;
        return 0;
    }
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < N; ++r) {
        for (int64_t j = 0; j < k; ++j) {
            const int64_t cand = latest[r] - j;                       /* :161 */
            const int64_t safe = cand < 0 ? 0 : cand;                 /* :163 */
            const int valid = cand >= 0 && (sorted_keys[safe] / (T + 1)) == read_base[r]; /* :162-168 */
            const int64_t src = order[safe];                          /* :173 */
            const unsigned char* srow = p + (size_t)src * row;
            unsigned char* orow = o + ((size_t)r * (size_t)k + (size_t)j) * row;
            if (valid) {
                memcpy(orow, srow, row);                              /* :174 */
            } else {
                for (int64_t d = 0; d < D; ++d) zero_like(srow + d * es, orow + d * es, dtype); /* :175 */
            }
            out_mask[r * k + j] = (uint8_t)valid;
            out_src[r * k + j] = src;
        }
    }
    return 0;
}

/*
 * Latest-k backward: autograd of index_select(order[safe]) * valid.
 * grad_payload[src] += grad_out[r, j] for every valid slot; double precision.
 * grad_payload must be zeroed by the caller.  Sequential in r (deterministic).
 */
int oracle_latestk_bwd(const uint8_t* mask, const int64_t* src, const double* grad_out,
                       int64_t N, int64_t D, int64_t k, double* grad_payload) {
    for (int64_t r = 0; r < N; ++r)
        for (int64_t j = 0; j < k; ++j) {
            if (!mask[r * k + j]) continue;
            const double* g = grad_out + ((size_t)r * k + j) * D;
            double* dst = grad_payload + (size_t)src[r * k + j] * D;
            for (int64_t d = 0; d < D; ++d) dst[d] += g[d];
        }
    return 0;
}

/* start index of each segment: first sorted position of its composite base */
static int is_seg_start(const int64_t* sorted_keys, int64_t q, int64_t T) {
    return q == 0 || (sorted_keys[q] / (T + 1)) != (sorted_keys[q - 1] / (T + 1));
}

/*
 * Sum forward (ravel_memory.py:179-241) on double payloads.
 *   out_sums [N, D], out_mask [N].  segcum is caller scratch of nw*D doubles.
 */
int oracle_segsum_fwd(const int64_t* sorted_keys, const int64_t* order,
                      const int64_t* latest, const int64_t* read_base, int64_t nw,
                      const double* payload, int64_t N, int64_t T, int64_t D,
                      double* segcum, double* out_sums, uint8_t* out_mask) {
    if (nw == 0) {                                                   /* :213-214 */
        memset(out_sums, 0, (size_t)N * (size_t)D * sizeof(double));
        memset(out_mask, 0, (size_t)N);
        return 0;
    }
    /* :216-229, one running sum per segment; segments never span streams so
     * the scan is split at stream-aligned segment starts for threading. */
    const int64_t nchunks = 256;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t ch = 0; ch < nchunks; ++ch) {
        int64_t q0 = nw * ch / nchunks, q1 = nw * (ch + 1) / nchunks;
        /* move both bounds forward to the next segment start */
        while (q0 < nw && q0 > 0 && !is_seg_start(sorted_keys, q0, T)) ++q0;
        while (q1 < nw && !is_seg_start(sorted_keys, q1, T)) ++q1;
        for (int64_t q = q0; q < q1; ++q) {
            const double* src = payload + (size_t)order[q] * D;      /* :217 */
            double* dst = segcum + (size_t)q * D;
            if (is_seg_start(sorted_keys, q, T)) {
                for (int64_t d = 0; d < D; ++d) dst[d] = src[d];
            } else {
                const double* prev = dst - D;
                for (int64_t d = 0; d < D; ++d) dst[d] = prev[d] + src[d];
            }
        }
    }
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < N; ++r) {
        const int64_t idx = latest[r];
        const int64_t safe = idx < 0 ? 0 : idx;                       /* :237 */
        const int valid = idx >= 0 && (sorted_keys[safe] / (T + 1)) == read_base[r]; /* :236-239 */
        const double* srow = segcum + (size_t)safe * D;
        double* orow = out_sums + (size_t)r * D;
        for (int64_t d = 0; d < D; ++d) orow[d] = srow[d] * (valid ? 1.0 : 0.0); /* :240 */
        out_mask[r] = (uint8_t)valid;
    }
    return 0;
}

/*
 * Sum backward: autograd of :240 (index_add of grad*valid into the sorted
 * tape at latest[r]), :223-229 (reverse segmented cumsum) and :217
 * (scatter back through order).  G is caller scratch of nw*D doubles.
 * grad_payload must be zeroed by the caller (rows of masked writes stay 0).
 */
int oracle_segsum_bwd(const int64_t* sorted_keys, const int64_t* order,
                      const int64_t* latest, const uint8_t* mask, int64_t nw,
                      const double* grad_sums, int64_t N, int64_t T, int64_t D,
                      double* G, double* grad_payload) {
    if (nw == 0) return 0;
    memset(G, 0, (size_t)nw * (size_t)D * sizeof(double));
    for (int64_t r = 0; r < N; ++r) {
        if (!mask[r]) continue;
        double* dst = G + (size_t)latest[r] * D;
        const double* g = grad_sums + (size_t)r * D;
        for (int64_t d = 0; d < D; ++d) dst[d] += g[d];
    }
    const int64_t nchunks = 256;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t ch = 0; ch < nchunks; ++ch) {
        int64_t q0 = nw * ch / nchunks, q1 = nw * (ch + 1) / nchunks;
        while (q0 < nw && q0 > 0 && !is_seg_start(sorted_keys, q0, T)) ++q0;
        while (q1 < nw && !is_seg_start(sorted_keys, q1, T)) ++q1;
        for (int64_t q = q1 - 1; q >= q0; --q) {
            double* cur = G + (size_t)q * D;
            const int last = (q == nw - 1) || is_seg_start(sorted_keys, q + 1, T);
            if (!last) {
                const double* nxt = cur + D;
                for (int64_t d = 0; d < D; ++d) cur[d] += nxt[d];
            }
            double* dst = grad_payload + (size_t)order[q] * D;
            for (int64_t d = 0; d < D; ++d) dst[d] = cur[d];
        }
    }
    return 0;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
