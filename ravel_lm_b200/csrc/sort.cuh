// sort.cuh -- per-stream event sort: the "tape" of RAVEL's event memory.
//
// The reference builds composite keys ((b*C + c)*A + addr)*(T+1) + t and calls
// torch.sort on all B*T*C of them (ravel_lm/ravel_memory.py:126-151).  The stream
// id (b, c) is the key's most significant part, so that global sort is the
// concatenation of independent per-stream sorts.  Here every stream's events are
// sorted on their own, as 32-bit keys (addr << tbits | t) when they fit (64-bit
// otherwise), which needs far fewer radix digits than a global 64-bit key.
//
//   k_tile_sort   one CTA per (stream, tile of up to 8192 steps): loads and folds
//                 the addresses, builds keys, and runs an LSD radix sort on the
//                 address bits only (the input is time-ordered and the sort is
//                 stable) in shared memory.  Ranking uses __match_any_sync per
//                 warp, warp-private digit histograms and a block-wide scan.
//   k_merge       merge-path merge of sorted runs for streams longer than a
//                 tile (log2(tiles) passes, global memory ping-pong).
//   k_merge_ranks general tapes: the reads sorted like the writes (in the
//                 writes' launch), then merged with the sorted writes; each
//                 read's rank = searchsorted(right=True)-1 of
//                 ravel_memory.py:159, restricted to the stream, and each
//                 write's first read ranked at or after it; block 0 also writes
//                 the per-stream offsets of the valid writes.
#pragma once

#include <cooperative_groups.h>

#include "common.cuh"

namespace ravel {

struct SortArgs {
    AddrSrc src;           // where the events' addresses come from
    int32_t* addr_out;     // [B, T, C]: the folded addresses are stored here too, or null
    const uint8_t* wmask;  // [B, T] or null
    int key32;             // reference key dtype is int32 (address truncation)
    int64_t B, T, C, A;
    int tbits, abits, mbit;
    int64_t tiles;         // tiles per stream
    void* keys_out;        // [S][T]
    int* nvalid;           // [S], pre-zeroed, or null when there is no mask
    int clamp;             // addresses clamped to [0, A-1] (decode cache) instead of wrapped
};

// Two sorts in one launch: the blocks (tile sort) or clusters (cluster sort)
// below `first` sort a[0], the rest a[1] -- a general tape's writes and reads,
// which are independent.  A single sort sets `first` to the whole grid.
struct SortPair {
    SortArgs a[2];
    int64_t first;
};

// Sort key of event (b, c, t) (stream s = b*C + c): (invalid bit | address)
// above t, the address folded as the reference does (or clamped for the decode
// cache); a masked write sorts after every valid one.
template <typename KeyT>
__device__ __forceinline__ KeyT sort_key(const SortArgs& a, int64_t b, int64_t c, int64_t s, int64_t t,
                                         int& nvalid_local) {
    (void)s;
    const int64_t raw = src_addr(a.src, b, t, c, a.T, a.C, a.A);
    const uint64_t ad = a.clamp ? static_cast<uint64_t>(clamp_addr(raw, a.A)) : fold_addr(raw, a.A, a.key32);
    if (a.addr_out != nullptr) a.addr_out[(b * a.T + t) * a.C + c] = static_cast<int32_t>(ad);
    const bool valid = a.wmask == nullptr || a.wmask[b * a.T + t] != 0;
    if (valid) {
        ++nvalid_local;
        return (static_cast<KeyT>(ad) << a.tbits) | static_cast<KeyT>(t);
    }
    // masked write: invalid bit above the address field, sorts last
    return (static_cast<KeyT>(1) << (a.tbits + a.abits)) | static_cast<KeyT>(t);
}

template <typename KeyT, int THREADS, int ITEMS>
__global__ void __launch_bounds__(THREADS) k_tile_sort(const __grid_constant__ SortPair p) {
    constexpr int TILE = THREADS * ITEMS;
    constexpr int NW = THREADS / 32;
    extern __shared__ __align__(16) unsigned char smem[];
    KeyT* ka = reinterpret_cast<KeyT*>(smem);
    KeyT* kb = ka + TILE;
    uint16_t* whist = reinterpret_cast<uint16_t*>(kb + TILE);
    uint32_t* dbase = reinterpret_cast<uint32_t*>(whist + NW * 256);

    const int which = static_cast<int64_t>(blockIdx.x) >= p.first ? 1 : 0;
    const SortArgs& a = p.a[which];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t C = a.C, T = a.T;
    int64_t blk = static_cast<int64_t>(blockIdx.x) - (which ? p.first : 0);
    // c varies fastest so that the C streams of one (b, tile) read the same
    // address sectors back to back (addresses are [B, T, C]).
    const int64_t c = blk % C;
    blk /= C;
    const int64_t tile = blk % a.tiles;
    const int64_t b = blk / a.tiles;
    const int64_t s = b * C + c;
    const int64_t t0 = tile * TILE;

    int nvalid_local = 0;
    for (int i = tid; i < TILE; i += THREADS) {
        const int64_t t = t0 + i;
        // tile padding sorts after everything
        const KeyT key = t < T ? sort_key<KeyT>(a, b, c, s, t, nvalid_local) : ~static_cast<KeyT>(0);
        ka[i] = key;
    }
    if (a.nvalid != nullptr) {
        const int w = __reduce_add_sync(0xffffffffu, static_cast<unsigned>(nvalid_local));
        if (lane == 0 && w) atomicAdd(a.nvalid + s, w);
    }
    __syncthreads();

    const int top = a.tbits + a.abits + a.mbit;
    for (int shift = a.tbits; shift < top; shift += 8) {
        const int nb = (top - shift) < 8 ? (top - shift) : 8;
        const unsigned dmask = (1u << nb) - 1u;
        for (int d = lane; d < 256; d += 32) whist[warp * 256 + d] = 0;
        __syncwarp();
        KeyT kv[ITEMS];
        uint16_t loc[ITEMS];
        uint16_t dig[ITEMS];
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) {
            const int idx = warp * (32 * ITEMS) + it * 32 + lane;
            const KeyT key = ka[idx];
            const unsigned d = static_cast<unsigned>(key >> shift) & dmask;
            const unsigned peers = __match_any_sync(0xffffffffu, d);
            const unsigned rank = __popc(peers & lanemask_lt());
            const unsigned before = whist[warp * 256 + d];
            __syncwarp();
            if (rank == 0) whist[warp * 256 + d] = static_cast<uint16_t>(before + __popc(peers));
            __syncwarp();
            kv[it] = key;
            loc[it] = static_cast<uint16_t>(before + rank);
            dig[it] = static_cast<uint16_t>(d);
        }
        __syncthreads();
        // per digit: exclusive prefix over warps (warp order == time order)
        for (int d = tid; d < 256; d += THREADS) {
            uint32_t run = 0;
#pragma unroll 4
            for (int w = 0; w < NW; ++w) {
                const uint32_t v = whist[w * 256 + d];
                whist[w * 256 + d] = static_cast<uint16_t>(run);
                run += v;
            }
            dbase[d] = run;
        }
        __syncthreads();
        if (warp == 0) {  // exclusive scan of the 256 digit totals
            uint32_t v[8];
            uint32_t sum = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) { v[i] = dbase[lane * 8 + i]; sum += v[i]; }
            uint32_t incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += n;
            }
            uint32_t run = incl - sum;
#pragma unroll
            for (int i = 0; i < 8; ++i) { dbase[lane * 8 + i] = run; run += v[i]; }
        }
        __syncthreads();
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) {
            const uint32_t dst = dbase[dig[it]] + whist[warp * 256 + dig[it]] + loc[it];
            kb[dst] = kv[it];
        }
        __syncthreads();
        KeyT* tmp = ka; ka = kb; kb = tmp;
    }

    const int64_t cnt = (T - t0) < TILE ? (T - t0) : TILE;
    KeyT* out = static_cast<KeyT*>(a.keys_out) + s * T + t0;
    for (int i = tid; i < cnt; i += THREADS) out[i] = ka[i];
}

// One stream per thread-block cluster: CTA r of the cluster loads tile r of the
// stream (8192 steps), and every LSD pass ranks locally, exchanges the 256
// digit totals of all CTAs through distributed shared memory, and scatters each
// key straight into the shared memory of the CTA that owns its destination
// (st.shared::cluster).  After the last pass CTA r holds sorted positions
// [r*8192, (r+1)*8192) of the stream: no global round trips, no merge passes.
// Used for streams of 2..8 tiles (T <= 65536); cluster size = tiles.
template <typename KeyT, int THREADS, int ITEMS>
__global__ void __launch_bounds__(THREADS) k_cluster_sort(const __grid_constant__ SortPair p) {
    namespace cg = cooperative_groups;
    constexpr int TILE = THREADS * ITEMS;
    constexpr int NW = THREADS / 32;
    extern __shared__ __align__(16) unsigned char smem[];
    KeyT* ka = reinterpret_cast<KeyT*>(smem);
    KeyT* kb = ka + TILE;
    uint16_t* whist = reinterpret_cast<uint16_t*>(kb + TILE);
    uint32_t* tot = reinterpret_cast<uint32_t*>(whist + NW * 256);  // this CTA's digit totals
    uint32_t* dbase = tot + 256;                                    // destination base per digit
    uint32_t* before = dbase + 256;                                 // keys of the digit in lower CTAs

    cg::cluster_group cluster = cg::this_cluster();
    const int crank = static_cast<int>(cluster.block_rank());
    const int csize = static_cast<int>(cluster.num_blocks());
    const int64_t cl = blockIdx.x / csize;  // cluster = stream of one of the two sorts
    const int which = cl >= p.first ? 1 : 0;
    const SortArgs& a = p.a[which];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t C = a.C, T = a.T;
    const int64_t s = cl - (which ? p.first : 0);
    const int64_t b = s / C, c = s % C;
    const int64_t t0 = static_cast<int64_t>(crank) * TILE;

    int nvalid_local = 0;
    for (int i = tid; i < TILE; i += THREADS) {
        const int64_t t = t0 + i;
        const KeyT key = t < T ? sort_key<KeyT>(a, b, c, s, t, nvalid_local) : ~static_cast<KeyT>(0);
        ka[i] = key;
    }
    if (a.nvalid != nullptr) {
        const int w = __reduce_add_sync(0xffffffffu, static_cast<unsigned>(nvalid_local));
        if (lane == 0 && w) atomicAdd(a.nvalid + s, w);
    }
    __syncthreads();

    const int top = a.tbits + a.abits + a.mbit;
    for (int shift = a.tbits; shift < top; shift += 8) {
        const int nb = (top - shift) < 8 ? (top - shift) : 8;
        const unsigned dmask = (1u << nb) - 1u;
        for (int d = lane; d < 256; d += 32) whist[warp * 256 + d] = 0;
        __syncwarp();
        KeyT kv[ITEMS];
        uint16_t loc[ITEMS];
        uint16_t dig[ITEMS];
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) {
            const int idx = warp * (32 * ITEMS) + it * 32 + lane;
            const KeyT key = ka[idx];
            const unsigned d = static_cast<unsigned>(key >> shift) & dmask;
            const unsigned peers = __match_any_sync(0xffffffffu, d);
            const unsigned rank = __popc(peers & lanemask_lt());
            const unsigned before = whist[warp * 256 + d];
            __syncwarp();
            if (rank == 0) whist[warp * 256 + d] = static_cast<uint16_t>(before + __popc(peers));
            __syncwarp();
            kv[it] = key;
            loc[it] = static_cast<uint16_t>(before + rank);
            dig[it] = static_cast<uint16_t>(d);
        }
        __syncthreads();
        for (int d = tid; d < 256; d += THREADS) {
            uint32_t run = 0;
#pragma unroll 4
            for (int w = 0; w < NW; ++w) {
                const uint32_t v = whist[w * 256 + d];
                whist[w * 256 + d] = static_cast<uint16_t>(run);
                run += v;
            }
            tot[d] = run;
        }
        cluster.sync();  // every CTA's totals are visible cluster-wide
        // per digit: keys of this digit in lower-ranked CTAs, and over the cluster
        for (int d = tid; d < 256; d += THREADS) {
            uint32_t lower = 0, all = 0;
            for (int r = 0; r < csize; ++r) {
                const uint32_t v = *cluster.map_shared_rank(tot + d, r);
                if (r < crank) lower += v;
                all += v;
            }
            dbase[d] = all;
            before[d] = lower;
        }
        __syncthreads();
        if (warp == 0) {  // exclusive scan of the cluster-wide digit totals
            uint32_t v[8];
            uint32_t sum = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) { v[i] = dbase[lane * 8 + i]; sum += v[i]; }
            uint32_t incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += n;
            }
            uint32_t run = incl - sum;
#pragma unroll
            for (int i = 0; i < 8; ++i) { dbase[lane * 8 + i] = run + before[lane * 8 + i]; run += v[i]; }
        }
        __syncthreads();
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) {
            const uint32_t dst = dbase[dig[it]] + whist[warp * 256 + dig[it]] + loc[it];
            KeyT* remote = cluster.map_shared_rank(kb, static_cast<int>(dst / TILE));
            remote[dst % TILE] = kv[it];
        }
        cluster.sync();  // all keys have landed before anyone reads them or reuses tot
        KeyT* tmp = ka; ka = kb; kb = tmp;
    }

    const int64_t cnt = (T - t0) < TILE ? (T - t0) : TILE;
    KeyT* out = static_cast<KeyT*>(a.keys_out) + s * T + t0;
    for (int i = tid; i < cnt; i += THREADS) out[i] = ka[i];
}

template <int THREADS, int ITEMS, typename KeyT>
inline size_t cluster_sort_smem() {
    return 2 * sizeof(KeyT) * THREADS * ITEMS + sizeof(uint16_t) * (THREADS / 32) * 256 + 4 * 768;
}

template <int THREADS, int ITEMS, typename KeyT>
inline size_t tile_sort_smem() {
    return 2 * sizeof(KeyT) * THREADS * ITEMS + sizeof(uint16_t) * (THREADS / 32) * 256 + 4 * 256;
}

// Number of elements of A among the first d outputs of merge(A, B) (unique keys).
template <typename KeyT>
__device__ __forceinline__ int64_t co_rank(const KeyT* A, int64_t la, const KeyT* Bk, int64_t lb, int64_t d) {
    int64_t lo = d - lb > 0 ? d - lb : 0;
    int64_t hi = d < la ? d : la;
    while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (A[mid] < Bk[d - mid - 1]) lo = mid + 1; else hi = mid;
    }
    return lo;
}

constexpr int MERGE_THREADS = 256;
constexpr int MERGE_ITEMS = 8;
constexpr int MERGE_OUT = MERGE_THREADS * MERGE_ITEMS;  // divides every run length (>= 2048)

// Merge pairs of sorted runs of length `run` within each stream.
template <typename KeyT>
__global__ void __launch_bounds__(MERGE_THREADS) k_merge(const KeyT* __restrict__ in, KeyT* __restrict__ out,
                                                         int64_t T, int64_t run, int64_t ctas_per_stream) {
    __shared__ KeyT sm[MERGE_OUT];
    __shared__ KeyT so[MERGE_OUT];
    __shared__ int64_t cr[2];
    const int tid = threadIdx.x;
    const int64_t s = blockIdx.x / ctas_per_stream;
    const int64_t o0 = (blockIdx.x % ctas_per_stream) * MERGE_OUT;
    if (o0 >= T) return;
    const int64_t o1 = (o0 + MERGE_OUT) < T ? (o0 + MERGE_OUT) : T;
    const int64_t ps = (o0 / (2 * run)) * (2 * run);
    const int64_t a0 = ps, a1 = (ps + run) < T ? (ps + run) : T;
    const int64_t b1 = (ps + 2 * run) < T ? (ps + 2 * run) : T;
    const int64_t la = a1 - a0, lb = b1 - a1;
    const KeyT* Ap = in + s * T + a0;
    const KeyT* Bp = in + s * T + a1;
    const int64_t d0 = o0 - ps, d1 = o1 - ps;
    if (tid < 2) cr[tid] = co_rank(Ap, la, Bp, lb, tid ? d1 : d0);
    __syncthreads();
    const int64_t i0 = cr[0], i1 = cr[1];
    const int64_t j0 = d0 - i0, j1 = d1 - i1;
    const int na = static_cast<int>(i1 - i0), nb = static_cast<int>(j1 - j0);
    for (int i = tid; i < na; i += MERGE_THREADS) sm[i] = Ap[i0 + i];
    for (int i = tid; i < nb; i += MERGE_THREADS) sm[na + i] = Bp[j0 + i];
    __syncthreads();
    const int n = na + nb;
    const int dd = tid * MERGE_ITEMS;
    if (dd < n) {
        int i = static_cast<int>(co_rank(sm, na, sm + na, nb, dd));
        int j = dd - i;
#pragma unroll
        for (int e = 0; e < MERGE_ITEMS; ++e) {
            if (dd + e >= n) break;
            const bool takeA = (j >= nb) || (i < na && sm[i] < sm[na + j]);
            so[dd + e] = takeA ? sm[i] : sm[na + j];
            if (takeA) ++i; else ++j;
        }
    }
    __syncthreads();
    KeyT* dst = out + s * T + o0;
    for (int i = tid; i < n; i += MERGE_THREADS) dst[i] = so[i];
}

// Exclusive prefix of the per-stream valid-write counts: soff[s] = writes of the
// streams before s in the reference's global sorted order; soff[S] = total.
// Run by one whole block (any multiple of 32 threads).
__device__ void stream_offsets_block(const int* __restrict__ nvalid, int64_t* __restrict__ soff, int64_t S,
                                     int64_t T) {
    __shared__ int64_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __shared__ int64_t wsum[32];
    for (int64_t base = 0; base < S; base += blockDim.x) {
        const int64_t s = base + threadIdx.x;
        const int64_t v = s < S ? (nvalid ? nvalid[s] : T) : 0;
        int64_t incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int64_t n = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += n;
        }
        if (lane == 31) wsum[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            const int nw = blockDim.x / 32;
            int64_t x = lane < nw ? wsum[lane] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int64_t n = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += n;
            }
            if (lane < nw) wsum[lane] = x;  // inclusive over warps
        }
        __syncthreads();
        const int64_t before = carry + (warp ? wsum[warp - 1] : 0) + incl - v;
        if (s < S) soff[s] = before;
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) carry = before + v;
        __syncthreads();
    }
    if (threadIdx.x == 0) soff[S] = carry;
}

// Read ranks and bucket starts in one pass: the merge of a stream's sorted
// writes W (its valid ones, n) and sorted reads R, a read placed before a write
// of equal key.  A read's rank is then the number of writes merged before it,
// minus one (searchsorted(right=True)-1 of ravel_memory.py:159, restricted to
// the stream: the latest valid write strictly below it), and bstart[j + 1] for
// write j is the number of reads merged before it.
//
// Merge path in two levels: a CTA owns MergeTile::TILE consecutive positions of
// one stream's merged order; two threads find the tile's co-ranks on its two
// diagonals (binary searches in global memory), the CTA loads the tile's reads
// and writes (plus the write before them) into shared memory with coalesced
// loads, and each thread finds its own co-rank in shared memory and merges
// MergeTile::E positions from there.  The merged order itself is staged and
// stored in coalesced runs (mkeys, and mrole: bit 0 a write, bit 1 a read whose
// latest earlier write has its address) for the sum lookup's scans.  CTAs past
// the tiles fill bstart[0] = 0 and bstart[n + 1 .. T + 1] = T, 4 entries a
// thread, so a heavy write mask (n << T) leaves no thread with T stores.  CTA 0
// first writes the stream offsets (stream_offsets_block), which this launch's
// merges do not read.
template <typename KeyT> struct MergeTile {
    static constexpr int E = sizeof(KeyT) == 4 ? 8 : 4;  // merged positions per thread
    static constexpr int TILE = 256 * E;                  // per CTA (static shared memory < 48 KB)
};
constexpr int MR_TAIL = 1024;  // bstart entries per tail CTA
__host__ __device__ inline int64_t mr_tiles(int64_t T, int tile) { return (2 * T + tile - 1) / tile; }
__host__ __device__ inline int64_t mr_tail_blocks(int64_t T) { return (T + 2 + MR_TAIL - 1) / MR_TAIL; }

template <typename KeyT>
__global__ void __launch_bounds__(256) k_merge_ranks(const KeyT* wkeys, const int* nvalid, const KeyT* rkeys,
                                                   int64_t S, int64_t T, int64_t C, int tbits, int32_t* rridx,
                                                   int32_t* ridx, int32_t* bstart, int64_t* soff, KeyT* mkeys,
                                                   uint8_t* mrole) {
    constexpr int E = MergeTile<KeyT>::E, TILE = MergeTile<KeyT>::TILE;
    __shared__ KeyT sR[TILE];      // the tile's reads
    __shared__ KeyT sW[TILE + 1];  // the write before the tile's writes, then its writes
    __shared__ KeyT sk[TILE];      // merged keys of the tile
    __shared__ uint8_t sr[TILE];   // their roles
    __shared__ int64_t s_co[2];
    if (blockIdx.x == 0) stream_offsets_block(nvalid, soff, S, T);
    const int tid = threadIdx.x;
    const int64_t tiles = mr_tiles(T, TILE);
    const int64_t bid = blockIdx.x;
    if (bid >= S * tiles) {  // bstart[0] and the entries past the last valid write
        const int64_t b2 = bid - S * tiles, tb = mr_tail_blocks(T);
        const int64_t s = b2 / tb, jb = (b2 - s * tb) * MR_TAIL;
        if (s >= S) return;
        const int64_t n = nvalid ? nvalid[s] : T;
        int32_t* bs = bstart + s * (T + 2);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int64_t j = jb + tid * 4 + u;
            if (j > T + 1) break;
            if (j == 0) bs[0] = 0;
            else if (j > n) bs[j] = static_cast<int32_t>(T);
        }
        return;
    }
    const int64_t s = bid / tiles, tile = bid - s * tiles;
    const int64_t n = nvalid ? nvalid[s] : T;
    const int64_t M = n + T;
    const int64_t d0 = tile * TILE;
    if (d0 >= M) return;
    const int64_t d1 = d0 + TILE < M ? d0 + TILE : M;
    const KeyT* W = wkeys + s * T;
    const KeyT* R = rkeys + s * T;
    if (tid < 64) {
        // co-rank: the largest i (reads among the first d merged) with R[i-1] <= W[d-i]
        // (true for every i up to it, false after), warp 0 for d0 and warp 1 for d1, each
        // lane probing one of 32 points of the remaining interval per round
        const int lane = tid & 31;
        const int64_t d = tid < 32 ? d0 : d1;
        int64_t lo = d - n > 0 ? d - n : 0, hi = d < T ? d : T;
        while (lo < hi) {
            const int64_t span = hi - lo;
            const int64_t step = (span + 31) / 32;
            const int64_t mid = lo + (lane + 1) * step < hi ? lo + (lane + 1) * step : hi;
            const int64_t j = d - mid;
            const bool ok = j >= n || R[mid - 1] <= W[j];
            const unsigned yes = __ballot_sync(0xffffffffu, ok);
            const unsigned no = __ballot_sync(0xffffffffu, !ok);
            // probes rise with the lane: the last true one and the first false one bound the answer
            const int lt = yes ? 31 - __clz(yes) : -1;
            const int lf = no ? __ffs(no) - 1 : 32;
            const int64_t nlo = lt >= 0 ? (lo + (lt + 1) * step < hi ? lo + (lt + 1) * step : hi) : lo;
            const int64_t nhi = lf < 32 ? (lo + (lf + 1) * step < hi ? lo + (lf + 1) * step : hi) - 1 : hi;
            lo = nlo;
            hi = nhi;
            if (step == 1) break;
        }
        if (lane == 0) s_co[tid >> 5] = lo;
    }
    __syncthreads();
    const int64_t i0 = s_co[0], j0 = d0 - i0;
    const int nr = static_cast<int>(s_co[1] - i0), nw = static_cast<int>((d1 - s_co[1]) - j0);
    for (int e = tid; e < nr; e += 256) sR[e] = R[i0 + e];
    for (int e = tid; e <= nw; e += 256) sW[e] = (e > 0 || j0 > 0) ? W[j0 - 1 + e] : KeyT(0);
    __syncthreads();
    const int len = static_cast<int>(d1 - d0);
    const int e0 = tid * E;
    if (e0 < len) {
        // this thread's co-rank inside the tile (a write past the tile's writes counts as +inf:
        // every read of the tile precedes it)
        int lo = e0 - nw > 0 ? e0 - nw : 0, hi = e0 < nr ? e0 : nr;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            const int jr = e0 - mid;
            if (jr >= nw || sR[mid - 1] <= sW[1 + jr]) lo = mid;
            else hi = mid - 1;
        }
        int i = lo, jr = e0 - lo;
        const int e1 = e0 + E < len ? e0 + E : len;
        const KeyT tmask = (static_cast<KeyT>(1) << tbits) - 1;
        const int64_t b = s / C, c = s - b * C;
        int32_t* bs = bstart + s * (T + 2);
        for (int e = e0; e < e1; ++e) {
            const int64_t jg = j0 + jr;
            if (i < nr && (jr >= nw || sR[i] <= sW[1 + jr])) {
                const KeyT q = sR[i];
                const int64_t ig = i0 + i;
                rridx[s * T + ig] = static_cast<int32_t>(jg - 1);
                ridx[(b * T + static_cast<int64_t>(q & tmask)) * C + c] = static_cast<int32_t>(jg - 1);
                sk[e] = q;
                // bit 1: the latest earlier write is of the read's own address (the sum lookup's mask)
                sr[e] = (jg > 0 && (sW[jr] >> tbits) == (q >> tbits)) ? 2 : 0;
                ++i;
            } else {
                bs[jg + 1] = static_cast<int32_t>(i0 + i);
                sk[e] = sW[1 + jr];
                sr[e] = 1;
                ++jr;
            }
        }
    }
    __syncthreads();
    KeyT* mk = mkeys + s * 2 * T + d0;
    uint8_t* mr = mrole + s * 2 * T + d0;
    for (int e = tid; e < len; e += 256) {
        mk[e] = sk[e];
        mr[e] = sr[e];
    }
}

// ------------------------------------------------------------------ literal addresses
// literal_addresses_from_tokens (ravel_lm/model.py:195-231): out [B, T, L] int64,
// one thread per element.
__global__ void k_literal_addresses(const int64_t* __restrict__ tokens, int64_t B, int64_t T, int L, int64_t bos,
                                    int64_t A, int64_t* __restrict__ out) {
    const int64_t n = B * T * L;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t bt = i / L;
        const int j = static_cast<int>(i - bt * L);
        const int64_t b = bt / T, t = bt - (bt / T) * T;
        out[i] = literal_addr(tokens, T, b, t, j, bos, A);
    }
}


}  // namespace ravel
