// ravel_b200.cu -- C ABI of the RAVEL event-memory operator for B200 (sm_100a).
//
// Entry points are declared (and their reference counterparts cited) in
// include/ravel_b200.h.  This file holds argument validation, the tape and
// scratch layouts, and the launch plumbing; the kernels live in the headers.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>
#include <initializer_list>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "sort.cuh"
#include "latestk.cuh"
#include "segsum.cuh"
#include "cache.cuh"
#include "glue.cuh"
#include "gather_gemm.cuh"

namespace ravel {
namespace {

// ------------------------------------------------------------------ layouts
struct TapeLayout {
    KeyLayout kl;
    int general;            // reads use the search path
    int has_mask;
    size_t key_bytes;
    size_t off_keys, off_nvalid, off_soff, off_ridx, off_rkeys, off_rridx, off_bstart, off_mkeys, off_mrole, total;
};

TapeLayout tape_layout(int64_t B, int64_t T, int64_t C, int64_t A, int flags) {
    TapeLayout t;
    t.has_mask = (flags & RAVEL_TAPE_WRITE_MASK) ? 1 : 0;
    t.general = flags != 0 ? 1 : 0;
    t.kl = key_layout(T, A, t.has_mask);
    t.key_bytes = t.kl.key64 ? 8 : 4;
    const size_t S = static_cast<size_t>(B * C), N = static_cast<size_t>(B * T * C);
    t.off_keys = 0;
    t.off_nvalid = align_up(S * static_cast<size_t>(T) * t.key_bytes);
    t.off_soff = t.off_nvalid + align_up(S * 4);
    t.off_ridx = t.off_soff + align_up((S + 1) * 8);
    t.off_rkeys = t.off_ridx + (t.general ? align_up(N * 4) : 0);
    t.off_rridx = t.off_rkeys + (t.general ? align_up(S * static_cast<size_t>(T) * t.key_bytes) : 0);
    t.off_bstart = t.off_rridx + (t.general ? align_up(S * static_cast<size_t>(T) * 4) : 0);
    t.off_mkeys = t.off_bstart + (t.general ? align_up(S * static_cast<size_t>(T + 2) * 4) : 0);
    t.off_mrole = t.off_mkeys + (t.general ? align_up(S * static_cast<size_t>(2 * T) * t.key_bytes) : 0);
    t.total = t.off_mrole + (t.general ? align_up(S * static_cast<size_t>(2 * T)) : 0);
    return t;
}

struct TapeView {
    void* keys;
    int* nvalid;       // null unless a mask is present
    int64_t* soff;
    int32_t* ridx;
    void* rkeys;       // general tapes: [S][T] read keys sorted by (address, t), write key width
    int32_t* rridx;    // general tapes: [S][T] latest valid write below each sorted read, -1 if none
    int32_t* bstart;   // general tapes: [S][T+2] first sorted read of each rridx value + 1
    void* mkeys;       // general tapes: [S][2T] the valid writes and the reads merged (a read first on equal keys)
    uint8_t* mrole;    // general tapes: [S][2T] bit 0: a write; bit 1: a read whose latest earlier
                       // valid write has its address (the sum lookup's mask)
};

TapeView tape_view(const void* tape, const TapeLayout& t) {
    char* base = static_cast<char*>(const_cast<void*>(tape));
    TapeView v;
    v.keys = base + t.off_keys;
    v.nvalid = t.has_mask ? reinterpret_cast<int*>(base + t.off_nvalid) : nullptr;
    v.soff = reinterpret_cast<int64_t*>(base + t.off_soff);
    v.ridx = t.general ? reinterpret_cast<int32_t*>(base + t.off_ridx) : nullptr;
    v.rkeys = t.general ? static_cast<void*>(base + t.off_rkeys) : nullptr;
    v.rridx = t.general ? reinterpret_cast<int32_t*>(base + t.off_rridx) : nullptr;
    v.bstart = t.general ? reinterpret_cast<int32_t*>(base + t.off_bstart) : nullptr;
    v.mkeys = t.general ? static_cast<void*>(base + t.off_mkeys) : nullptr;
    v.mrole = t.general ? reinterpret_cast<uint8_t*>(base + t.off_mrole) : nullptr;
    return v;
}

// tile sort configuration for a stream length T
struct SortPlan {
    int threads;
    int items;  // keys per thread
    int64_t tiles;
    int merge_passes;
};

// Build-time knob: keys per thread of the tile sort for streams that fit one CTA at
// that count (8 otherwise; more threads with fewer keys each shorten the ranking).
// Measured at config 5 (T = 1024, writes and reads in one launch; step replayed
// from a CUDA graph, ms): 8 keys 0.0726, 4 keys 0.0686, 2 keys 0.0685.
#ifndef RAVEL_SORT_SHORT_ITEMS
#define RAVEL_SORT_SHORT_ITEMS 4
#endif
static_assert(RAVEL_SORT_SHORT_ITEMS == 2 || RAVEL_SORT_SHORT_ITEMS == 4 || RAVEL_SORT_SHORT_ITEMS == 8,
              "keys per thread");

SortPlan sort_plan(int64_t T) {
    SortPlan p;
    const int64_t tile_cap = 8192;
    p.items = T <= 1024 * RAVEL_SORT_SHORT_ITEMS ? RAVEL_SORT_SHORT_ITEMS : 8;
    int threads = 32;
    while (threads < 1024 && static_cast<int64_t>(threads) * p.items < T) threads *= 2;
    p.threads = threads;
    const int64_t tile = static_cast<int64_t>(threads) * p.items;
    p.tiles = T <= tile ? 1 : (T + tile_cap - 1) / tile_cap;
    p.merge_passes = 0;
    while ((int64_t(1) << p.merge_passes) < p.tiles) ++p.merge_passes;
    return p;
}

int acc_bytes(int dtype) { return dtype == RAVEL_F64 ? 8 : 4; }

// 16-bit payload rows taken as 2^v chunks of 8 elements (16 bytes): v when D/8 is a
// power of two up to 32 and every pointer involved is 16-byte aligned, else -1.
int vshift16(int dtype, int64_t D, uintptr_t align_bits) {
    if (dtype != RAVEL_BF16 && dtype != RAVEL_F16) return -1;
    if (D <= 0 || D % 8 != 0 || align_bits % 16 != 0) return -1;
    const int64_t c = D / 8;
    if (c > 32 || (c & (c - 1)) != 0) return -1;
    int v = 0;
    while ((int64_t{1} << v) < c) ++v;
    return v;
}

struct ScanPlan {
    int P, parts, min_P;
    int64_t nchunks;      // chunks per stream of the fallback kernel
    int64_t max_nchunks;  // chunks per stream of the smallest chunk size in use
};

// Chunk size of the warp-register scan kernel (0 when it does not apply).
int scanw_positions(int64_t D, int elem_bytes_in) {
    for (int el = 1; el <= 8; el *= 2) {
        if (D > 0 && D % el == 0 && D / el <= 32) return SCANW_WARPS * scanw_rows(el, elem_bytes_in);
    }
    return 0;
}

// Plan of the shared-memory scan kernel (the fallback); the look-back state in
// scratch is sized for the smallest chunk either kernel may use (min_P).
ScanPlan scan_plan(int64_t T, int64_t D, int dtype) {
    ScanPlan s;
    const int64_t per = (D > 0 ? D : 1) * acc_bytes(dtype);
    int64_t P = 32768 / per;
    if (P > 256) P = 256;
    if (P < 16) P = 16;
    P -= P % 8;
    s.P = static_cast<int>(P);
    int min_p = s.P;
    for (int eb : {elem_bytes(dtype), acc_bytes(dtype)}) {
        const int pw = scanw_positions(D, eb);
        if (pw > 0 && pw < min_p) min_p = pw;
    }
    s.min_P = min_p;
    const int ncol = D < 1 ? 1 : (D < SCAN_THREADS ? static_cast<int>(D) : SCAN_THREADS);
    int parts = SCAN_THREADS / ncol;
    if (parts < 1) parts = 1;
    if (parts > s.P) parts = s.P;
    s.parts = parts;
    s.nchunks = (T + s.P - 1) / s.P;
    s.max_nchunks = (T + s.min_P - 1) / s.min_P;
    return s;
}

// Ranges per stream for the range scan: `slots` ranges over T positions, each
// range between rl_min and rl_max positions (a multiple of 8).  Scratch is
// sized for the most ranges any plan can use (max_ranges).
struct RangePlan {
    int64_t R, RL;
};

RangePlan range_plan(int64_t S, int64_t T, int64_t slots, int64_t rl_max = int64_t{1} << 40, int64_t rl_min = 64) {
    RangePlan p;
    int64_t R = S > 0 ? slots / S : 1;
    if (R < 1) R = 1;
    int64_t RL = (T + R - 1) / R;
    RL = (RL + 7) / 8 * 8;
    if (RL > rl_max) RL = rl_max;
    if (RL < rl_min) RL = rl_min;
    p.RL = RL;
    p.R = T > 0 ? (T + RL - 1) / RL : 1;
    return p;
}

// Range-scan launch shape (overridable at build time for sweeps): blocks for
// RAVEL_RS_WAVES waves of resident blocks, so that blocks at different phases
// (piece sums, look-back, scan) share an SM.  Ranges hold at least 64
// positions, or down to RAVEL_RS_RLMIN when 64-position ranges would not fill
// one wave of blocks (short streams); the snap window is at most half a range,
// so that no range is empty.
// Measured at config 3 (sum forward / backward, µs): 1 wave 197 / 183,
// 2 waves 173 / 170, 3 waves 167 / 158-166; 2-warp blocks, 48-position ranges
// and a deeper ring were no faster.
#ifndef RAVEL_RS_WAVES
#define RAVEL_RS_WAVES 3
#endif
#ifndef RAVEL_RS_RLMIN
#define RAVEL_RS_RLMIN 16
#endif
// Blocks per SM for short streams (their ranges shrink down to RAVEL_RS_RLMIN
// positions).  Measured at config 5's merged sum scans (2048 positions per
// stream, us forward / backward): 2 blocks 27.9 / 28.2, 4 blocks 24.3 / 23.7,
// 8 blocks (16-position ranges) 21.7 / 22.1.
#ifndef RAVEL_RS_SHORT_BPS
#define RAVEL_RS_SHORT_BPS 8
#endif
static_assert(RAVEL_RS_RLMIN >= 16 && RAVEL_RS_RLMIN <= 64 && RAVEL_RS_RLMIN % 8 == 0, "range length floor");
int64_t max_ranges(int64_t T) { return T > 0 ? (T + RAVEL_RS_RLMIN - 1) / RAVEL_RS_RLMIN : 1; }
// Build-time knob: rows of at least this many 16-byte vectors give each lane of the
// range scan two vectors (half the lanes per row, twice the ranges per warp).
// Measured at config 3 (128-byte rows, 8 vectors): one vector per lane 170.6 /
// 160.0 us (sum forward / backward), two 223.4 / 211.3 us.
#ifndef RAVEL_RS_VPL2_NVEC
#define RAVEL_RS_VPL2_NVEC 64
#endif
static_assert(RAVEL_RS_VPL2_NVEC >= 2 && RAVEL_RS_VPL2_NVEC <= 64, "two vectors per lane need two per row");

int sm_count() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
    }
    return n;
}

struct ScratchLayout {
    size_t off_sort, off_flags, off_ticket, off_agg, off_incl, off_bflags, off_bval, off_big, total;
};

ScratchLayout scratch_layout(int64_t B, int64_t T, int64_t C, int64_t D, int64_t A, int dtype, int flags) {
    ScratchLayout l;
    const TapeLayout t = tape_layout(B, T, C, A, flags);
    const SortPlan sp = sort_plan(T);
    const ScanPlan sc = scan_plan(T, D, dtype);
    const size_t S = static_cast<size_t>(B * C), N = static_cast<size_t>(B * T * C);
    const size_t nch = S * static_cast<size_t>(sc.max_nchunks);
    const size_t ab = static_cast<size_t>(acc_bytes(dtype));
    l.off_sort = 0;
    l.off_flags = align_up(sp.tiles > 1 ? S * static_cast<size_t>(T) * t.key_bytes : 0);
    l.off_ticket = l.off_flags + align_up(nch * 4);
    l.off_agg = l.off_ticket + 256;
    l.off_incl = l.off_agg + align_up(nch * static_cast<size_t>(D) * ab);
    // range-scan blocks hold at least GS_WARPS ranges; general tapes' merged scans walk up to 2T positions
    const int64_t Tm = t.general ? 2 * T : T;
    const size_t nb = S * static_cast<size_t>((max_ranges(Tm) + GS_WARPS - 1) / GS_WARPS);
    l.off_bflags = l.off_incl + align_up(nch * static_cast<size_t>(D) * ab);
    l.off_bval = l.off_bflags + align_up((nb + 1) * 4);
    l.off_big = l.off_bval + align_up(nb * 2 * static_cast<size_t>(D) * ab);
    l.total = l.off_big + (t.general ? align_up(N * static_cast<size_t>(D) * ab) : 0);
    return l;
}

// ------------------------------------------------------------------ dispatch helpers
template <int V> using IC = std::integral_constant<int, V>;

template <typename F>
int with_key(int key64, F&& f) {
    return key64 ? f(uint64_t(0)) : f(uint32_t(0));
}

template <typename F>
int with_dtype(int dt, F&& f) {
    switch (dt) {
        case RAVEL_F32: return f(IC<RAVEL_F32>{});
        case RAVEL_BF16: return f(IC<RAVEL_BF16>{});
        case RAVEL_F16: return f(IC<RAVEL_F16>{});
        case RAVEL_F64: return f(IC<RAVEL_F64>{});
        default: return RAVEL_ERR_INVALID_ARG;
    }
}

template <typename F>
int with_vb(int vb, F&& f) {
    switch (vb) {
        case 16: return f(IC<16>{});
        case 8: return f(IC<8>{});
        case 4: return f(IC<4>{});
        default: return f(IC<2>{});
    }
}

// Vector widths that can occur for a dtype (a row is a whole number of elements).
template <int DT, int VB>
constexpr bool vb_ok() {
    return (DT == RAVEL_F64) ? (VB >= 8) : (DT == RAVEL_F32 ? VB >= 4 : true);
}

std::atomic<uint64_t> g_launches{0};

// Called once after every kernel launch of this library.
int check_launch() {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? RAVEL_OK : RAVEL_ERR_CUDA;
}

// Per-(kernel, device) results of CUDA attribute calls, so that a launch pays for
// them once per process instead of on every call.
std::mutex g_attr_mu;
std::map<std::pair<const void*, int>, size_t> g_smem_set;            // dynamic smem limit raised to
std::map<std::tuple<const void*, int, int, size_t>, int> g_occupancy;  // blocks per SM

int current_device() {
    int dev = 0;
    return cudaGetDevice(&dev) == cudaSuccess ? dev : 0;
}

template <typename K>
int set_smem(K kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return RAVEL_OK;
    if (bytes > 227 * 1024) return RAVEL_ERR_UNSUPPORTED;
    const auto key = std::make_pair(reinterpret_cast<const void*>(kernel), current_device());
    std::lock_guard<std::mutex> lock(g_attr_mu);
    auto it = g_smem_set.find(key);
    if (it != g_smem_set.end() && it->second >= bytes) return RAVEL_OK;
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    if (e != cudaSuccess) return RAVEL_ERR_CUDA;
    g_smem_set[key] = bytes;
    return RAVEL_OK;
}

// cudaOccupancyMaxActiveBlocksPerMultiprocessor, remembered per (kernel, device, block, smem).
template <typename K>
int occupancy(K kernel, int threads, size_t smem) {
    const auto key = std::make_tuple(reinterpret_cast<const void*>(kernel), current_device(), threads, smem);
    {
        std::lock_guard<std::mutex> lock(g_attr_mu);
        auto it = g_occupancy.find(key);
        if (it != g_occupancy.end()) return it->second;
    }
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, smem) != cudaSuccess || occ < 1) occ = 1;
    std::lock_guard<std::mutex> lock(g_attr_mu);
    g_occupancy[key] = occ;
    return occ;
}

uintptr_t addr_bits(const void* p) { return reinterpret_cast<uintptr_t>(p); }

// Grid-stride kernels: at most 64 blocks per SM of the current device.
int grid_cap(int64_t blocks) {
    const int64_t cap = static_cast<int64_t>(sm_count()) * 64;
    return static_cast<int>(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

// ------------------------------------------------------------------ validation
int check_sizes(int64_t B, int64_t T, int64_t C, int64_t D, int64_t A) {
    if (B < 0 || T < 0 || C < 0 || D < 0) return RAVEL_ERR_INVALID_ARG;
    if (A <= 0) return RAVEL_ERR_INVALID_ARG;
    const KeyLayout kl = key_layout(T, A, 1);
    if (kl.tbits + kl.abits + 1 > 64 || T > (int64_t(1) << 30)) return RAVEL_ERR_UNSUPPORTED;
    const long double N = static_cast<long double>(B) * T * C;
    if (N >= 2147483647.0L) return RAVEL_ERR_UNSUPPORTED;  // flat rows are packed in 32 bits
    return RAVEL_OK;
}

int key32_of(int64_t B, int64_t T, int64_t C, int64_t A) {
    const long double bound = static_cast<long double>(B) * C * A * (T + 1);
    return bound <= 2147483647.0L ? 1 : 0;
}

// ------------------------------------------------------------------ tape build
// Sort every stream's events (the keys sort_key builds) into `out0`: one cluster
// per stream for 2-8 tiles, one CTA per stream for one tile, else tiles sorted in
// shared memory and merged through `other` (ping-pong, S*T keys).  With `a1`
// (a general tape's reads) the second sort into `out1` shares the launch of the
// first when a stream takes one cluster or one CTA; streams that need merge
// passes sort one after the other.
template <typename KeyT>
int sort_streams(const SortArgs& a0, void* out0, const SortArgs* a1, void* out1, void* other, int64_t S, int64_t T,
                 cudaStream_t st) {
    const SortPlan sp = sort_plan(T);
    const int64_t nsort = a1 != nullptr ? 2 : 1;
    SortPair p;
    p.a[0] = a0;
    p.a[0].tiles = sp.tiles;
    p.a[0].keys_out = out0;
    p.a[1] = a1 != nullptr ? *a1 : a0;
    p.a[1].tiles = sp.tiles;
    p.a[1].keys_out = a1 != nullptr ? out1 : out0;
    p.first = S;
    if (sp.tiles > 1 && sp.tiles <= 8) {
        // one cluster of CTAs per stream, straight into the output: CTAs of CT threads x 8 keys,
        // as many as the stream needs (2..8)
        auto try_cluster = [&](auto ctc) -> int {
            constexpr int CT = decltype(ctc)::value;
            const int64_t tile = static_cast<int64_t>(CT) * 8;
            const int64_t ctiles = (T + tile - 1) / tile;
            if (ctiles < 2 || ctiles > 8) return -1;
            const size_t smem = cluster_sort_smem<CT, 8, KeyT>();
            if (set_smem(k_cluster_sort<KeyT, CT, 8>, smem) != RAVEL_OK) return -1;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(static_cast<unsigned>(nsort * S * ctiles));
            cfg.blockDim = dim3(CT);
            cfg.dynamicSmemBytes = smem;
            cfg.stream = st;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = static_cast<unsigned>(ctiles);
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            if (cudaLaunchKernelEx(&cfg, k_cluster_sort<KeyT, CT, 8>, p) == cudaSuccess) return check_launch();
            (void)cudaGetLastError();  // not schedulable here
            return -1;
        };
// Build-time knob: threads of the cluster sort's CTAs for streams that fit 8 of them.
// Measured at config 3 (T = 32768, tape build, us): 1024 threads (clusters of 4)
// 71.5, 512 (clusters of 8, two CTAs per SM) 70.9, 256 73.5: the sort does not
// gain from a second resident CTA.
#ifndef RAVEL_SORT_CT
#define RAVEL_SORT_CT 1024
#endif
        int rc = T <= static_cast<int64_t>(RAVEL_SORT_CT) * 64 ? try_cluster(IC<RAVEL_SORT_CT>{}) : -1;
        if (rc < 0 && RAVEL_SORT_CT != 1024) rc = try_cluster(IC<1024>{});
        if (rc >= 0) return rc;  // otherwise: tiles + merges
    }
    if (sp.tiles > 1 && a1 != nullptr) {  // the two sorts share the merge scratch: one after the other
        if (int e = sort_streams<KeyT>(a0, out0, nullptr, nullptr, other, S, T, st)) return e;
        return sort_streams<KeyT>(*a1, out1, nullptr, nullptr, other, S, T, st);
    }
    void* first = (sp.merge_passes % 2 == 0) ? out0 : other;
    p.a[0].keys_out = first;
    p.first = S * sp.tiles;
    const int64_t grid = nsort * S * sp.tiles;
    auto launch = [&](auto th, auto it) -> int {
        constexpr int TH = decltype(th)::value;
        constexpr int IT = decltype(it)::value;
        const size_t smem = tile_sort_smem<TH, IT, KeyT>();
        if (int e = set_smem(k_tile_sort<KeyT, TH, IT>, smem)) return e;
        k_tile_sort<KeyT, TH, IT><<<static_cast<unsigned>(grid), TH, smem, st>>>(p);
        return check_launch();
    };
    auto by_threads = [&](auto it) -> int {
        switch (sp.threads) {
            case 32: return launch(IC<32>{}, it);
            case 64: return launch(IC<64>{}, it);
            case 128: return launch(IC<128>{}, it);
            case 256: return launch(IC<256>{}, it);
            case 512: return launch(IC<512>{}, it);
            default: return launch(IC<1024>{}, it);
        }
    };
    int e = RAVEL_OK;
    if (RAVEL_SORT_SHORT_ITEMS != 8 && sp.items == RAVEL_SORT_SHORT_ITEMS) e = by_threads(IC<RAVEL_SORT_SHORT_ITEMS>{});
    else e = by_threads(IC<8>{});
    if (e) return e;
    const KeyT* src = static_cast<const KeyT*>(first);
    int64_t run = static_cast<int64_t>(sp.threads) * 8;
    const int64_t cps = (T + MERGE_OUT - 1) / MERGE_OUT;
    for (int pass = 0; pass < sp.merge_passes; ++pass) {
        KeyT* dst = (src == static_cast<const KeyT*>(out0)) ? static_cast<KeyT*>(other) : static_cast<KeyT*>(out0);
        k_merge<KeyT><<<static_cast<unsigned>(S * cps), MERGE_THREADS, 0, st>>>(src, dst, T, run, cps);
        if (int e2 = check_launch()) return e2;
        src = dst;
        run *= 2;
    }
    return RAVEL_OK;
}

// Sort the writes (and for general tapes the reads) of every stream.  `wsrc` /
// `rsrc` say where addresses come from; `raddr_out`, when given, receives the
// folded read addresses as int32 [B, T, C] (the reads' own pass for general
// reads, else the writes' pass).
int tape_build_src(const AddrSrc& wsrc, const AddrSrc& rsrc, int32_t* raddr_out, const uint8_t* wmask,
                   int64_t B, int64_t T, int64_t C, int64_t A, int flags, void* tape, size_t tape_bytes,
                   void* scratch, size_t scratch_bytes, cudaStream_t st) {
    if (int e = check_sizes(B, T, C, 0, A)) return e;
    if ((flags & RAVEL_TAPE_WRITE_MASK) && wmask == nullptr) return RAVEL_ERR_INVALID_ARG;
    const int64_t S = B * C, N = B * T * C;
    if (N == 0) return RAVEL_OK;
    if (tape == nullptr) return RAVEL_ERR_INVALID_ARG;
    const TapeLayout tl = tape_layout(B, T, C, A, flags);
    const ScratchLayout sl = scratch_layout(B, T, C, 0, A, RAVEL_F32, flags);
    if (tape_bytes < tl.total) return RAVEL_ERR_WORKSPACE;
    const SortPlan sp = sort_plan(T);
    if (sp.tiles > 1 && (scratch == nullptr || scratch_bytes < sl.off_flags)) return RAVEL_ERR_WORKSPACE;
    const TapeView tv = tape_view(tape, tl);
    if (tl.has_mask && cudaMemsetAsync(tv.nvalid, 0, S * sizeof(int), st) != cudaSuccess) return RAVEL_ERR_CUDA;

    SortArgs a;
    std::memset(&a, 0, sizeof(a));
    a.src = wsrc;
    a.addr_out = (flags & RAVEL_TAPE_GENERAL_READS) ? nullptr : raddr_out;
    a.wmask = tl.has_mask ? wmask : nullptr;
    a.key32 = key32_of(B, T, C, A);
    a.B = B; a.T = T; a.C = C; a.A = A;
    a.tbits = tl.kl.tbits; a.abits = tl.kl.abits; a.mbit = tl.kl.mbit;
    a.tiles = sp.tiles;
    a.nvalid = tv.nvalid;
    a.clamp = 0;
    void* other = static_cast<char*>(scratch) + sl.off_sort;
    int rc = with_key(tl.kl.key64, [&](auto kt) -> int {
        using KeyT = decltype(kt);
        if (!tl.general) return sort_streams<KeyT>(a, tv.keys, nullptr, nullptr, other, S, T, st);
        // read tape: the reads sorted like the writes (by address, t) -- in the writes'
        // launch -- then ranked against the sorted writes (the rank is each read's
        // latest earlier write); the merge kernel also writes the stream offsets
        SortArgs ra = a;
        ra.src = (flags & RAVEL_TAPE_GENERAL_READS) ? rsrc : wsrc;
        ra.addr_out = (flags & RAVEL_TAPE_GENERAL_READS) ? raddr_out : nullptr;
        ra.wmask = nullptr;
        ra.nvalid = nullptr;
        ra.mbit = 0;
        if (int e = sort_streams<KeyT>(a, tv.keys, &ra, tv.rkeys, other, S, T, st)) return e;
        const int64_t mgrid = S * mr_tiles(T, MergeTile<KeyT>::TILE) + S * mr_tail_blocks(T);
        if (mgrid > 2147483647LL) return RAVEL_ERR_UNSUPPORTED;
        k_merge_ranks<KeyT><<<static_cast<unsigned>(mgrid), 256, 0, st>>>(
            static_cast<const KeyT*>(tv.keys), tv.nvalid, static_cast<const KeyT*>(tv.rkeys), S, T, C,
            tl.kl.tbits, tv.rridx, tv.ridx, tv.bstart, tv.soff, static_cast<KeyT*>(tv.mkeys), tv.mrole);
        return check_launch();
    });
    return rc;
}

AddrSrc plain_src(const void* addr, int addr_dtype) {
    AddrSrc s;
    std::memset(&s, 0, sizeof(s));
    s.addr = addr;
    s.i64 = addr_dtype == RAVEL_I64;
    return s;
}

int tape_build(const void* waddr, const void* raddr, int addr_dtype, const uint8_t* wmask, int64_t B,
               int64_t T, int64_t C, int64_t A, int flags, void* tape, size_t tape_bytes, void* scratch,
               size_t scratch_bytes, cudaStream_t st) {
    if (addr_dtype != RAVEL_I32 && addr_dtype != RAVEL_I64) return RAVEL_ERR_INVALID_ARG;
    if ((flags & RAVEL_TAPE_GENERAL_READS) && raddr == nullptr) return RAVEL_ERR_INVALID_ARG;
    if (B * T * C != 0 && waddr == nullptr) return RAVEL_ERR_INVALID_ARG;
    return tape_build_src(plain_src(waddr, addr_dtype), plain_src(raddr ? raddr : waddr, addr_dtype), nullptr,
                          wmask, B, T, C, A, flags, tape, tape_bytes, scratch, scratch_bytes, st);
}

// ------------------------------------------------------------------ latest-k
LkArgs lk_args(const TapeView& tv, const TapeLayout& tl, const void* raddr, int addr_dtype, int64_t B,
               int64_t T, int64_t C, int64_t D, int64_t A, int64_t k, int dtype) {
    LkArgs a;
    std::memset(&a, 0, sizeof(a));
    a.keys = tv.keys;
    a.nvalid = tv.nvalid;
    a.soff = tv.soff;
    a.ridx = tv.ridx;
    a.raddr = raddr;
    a.addr_i64 = addr_dtype == RAVEL_I64;
    a.key32 = key32_of(B, T, C, A);
    a.B = B; a.T = T; a.C = C; a.D = D; a.A = A; a.k = k;
    a.tbits = tl.kl.tbits;
    a.row_bytes = D * elem_bytes(dtype);
    a.fd_C = FastDiv(static_cast<uint32_t>(C > 0 ? C : 1));
    a.fd_T = FastDiv(static_cast<uint32_t>(T > 0 ? T : 1));
    return a;
}

// Build-time knob: (read, slot) pairs per CTA of the general latest-k forward (at most 512).
// Measured (us, general forward at config 5 / config 3 with independent reads): 512 pairs
// 14.7 / 535, 256 pairs 13.9 / 562, 128 pairs 13.5 / 650.
#ifndef RAVEL_LK_GEN_SLOTS
#define RAVEL_LK_GEN_SLOTS 512
#endif
static_assert(RAVEL_LK_GEN_SLOTS >= 1 && RAVEL_LK_GEN_SLOTS <= 512, "the kernel's slot arrays hold 512");

int lk_fwd_tape(const void* tape, int flags, const void* raddr, int addr_dtype, const void* payload, int dtype,
                int64_t B, int64_t T, int64_t C, int64_t D, int64_t A, int64_t k, void* out_vals,
                uint8_t* out_mask, cudaStream_t st) {
    if (int e = check_sizes(B, T, C, D, A)) return e;
    if (k <= 0) return RAVEL_ERR_INVALID_ARG;
    if (k > 512) return RAVEL_ERR_UNSUPPORTED;
    if (dtype < 0 || dtype > 3) return RAVEL_ERR_INVALID_ARG;
    const int64_t N = B * T * C;
    if (N == 0) return RAVEL_OK;
    if (tape == nullptr || out_mask == nullptr || (D > 0 && (payload == nullptr || out_vals == nullptr)))
        return RAVEL_ERR_INVALID_ARG;
    const TapeLayout tl = tape_layout(B, T, C, A, flags);
    if (tl.general && raddr == nullptr) return RAVEL_ERR_INVALID_ARG;
    const TapeView tv = tape_view(tape, tl);
    LkArgs a = lk_args(tv, tl, raddr, addr_dtype, B, T, C, D, A, k, dtype);
    a.payload = payload;
    a.out = out_vals;
    a.out_mask = out_mask;
    const int vb = pick_vec_bytes(a.row_bytes, addr_bits(payload) | addr_bits(out_vals));
    const int64_t rv = a.row_bytes / vb;
    a.fd_rv = FastDiv(static_cast<uint32_t>(rv > 0 ? rv : 1));
    a.fd_bv = FastDiv(static_cast<uint32_t>(rv * k > 0 ? rv * k : 1));
    a.fd_k = FastDiv(static_cast<uint32_t>(k));
    const int64_t S = B * C;
    return with_key(tl.kl.key64, [&](auto kt) -> int {
        using KeyT = decltype(kt);
        return with_dtype(dtype, [&](auto dtc) -> int {
            constexpr int DT = decltype(dtc)::value;
            return with_vb(vb, [&](auto vbc) -> int {
                constexpr int VB = decltype(vbc)::value;
                if constexpr (!vb_ok<DT, VB>()) {
                    return RAVEL_ERR_INVALID_ARG;
                } else {
                    if (!tl.general) {
                        int64_t P = 40960 / (a.row_bytes + 16) - k;
// Build-time knob: at most this many sorted positions per CTA of the aliased latest-k
// forward.  Measured at config 3 (us): 128 positions 439.8, 64 positions 435.7.
#ifndef RAVEL_LK_PMAX
#define RAVEL_LK_PMAX 64
#endif
                        if (P > RAVEL_LK_PMAX) P = RAVEL_LK_PMAX;
                        if (P < 16) P = 16;
                        a.P = static_cast<int>(P);
                        a.nchunks = (T + P - 1) / P;
                        const size_t smem = lk_fast_smem(a.P, k, a.row_bytes);
                        if (int e = set_smem(k_lk_fwd_fast<KeyT, DT, VB>, smem)) return e;
                        k_lk_fwd_fast<KeyT, DT, VB><<<static_cast<unsigned>(S * a.nchunks), 256, smem, st>>>(a);
                    } else {
                        const int64_t rpc = (RAVEL_LK_GEN_SLOTS / k) > 0 ? RAVEL_LK_GEN_SLOTS / k : 1;
                        k_lk_fwd_general<KeyT, DT, VB><<<static_cast<unsigned>((N + rpc - 1) / rpc), 256, 0, st>>>(a, rpc);
                    }
                    return check_launch();
                }
            });
        });
    });
}

// Build-time knob: sorted positions per CTA of the aliased latest-k backward.
// Measured at config 3 (us, accumulate mode): 64 positions 412.6, 128 402.1, 256 404.4.
#ifndef RAVEL_LK_BWD_P
#define RAVEL_LK_BWD_P 128
#endif
// Build-time knob: 0 keeps the general latest-k backward on the per-write gather (k_lk_bwd_gather).
#ifndef RAVEL_LK_BWD_CHUNK
#define RAVEL_LK_BWD_CHUNK 1
#endif

int lk_bwd(const void* tape, int flags, const void* raddr, int addr_dtype, const void* grad_vals, int dtype,
           int64_t B, int64_t T, int64_t C, int64_t D, int64_t A, int64_t k, void* grad_payload, void* scratch,
           size_t scratch_bytes, cudaStream_t st, int accumulate = 0) {
    if (int e = check_sizes(B, T, C, D, A)) return e;
    if (k <= 0) return RAVEL_ERR_INVALID_ARG;
    if (k > 512) return RAVEL_ERR_UNSUPPORTED;
    if (dtype < 0 || dtype > 3) return RAVEL_ERR_INVALID_ARG;
    const int64_t N = B * T * C;
    if (N == 0 || D == 0) return RAVEL_OK;
    if (tape == nullptr || grad_vals == nullptr || grad_payload == nullptr) return RAVEL_ERR_INVALID_ARG;
    const TapeLayout tl = tape_layout(B, T, C, A, flags);
    if (tl.general && raddr == nullptr) return RAVEL_ERR_INVALID_ARG;
    const TapeView tv = tape_view(tape, tl);
    LkArgs a = lk_args(tv, tl, raddr, addr_dtype, B, T, C, D, A, k, dtype);
    a.grad = grad_vals;
    a.accumulate = accumulate;
    const int64_t S = B * C;
    if (!tl.general) {
        a.out = grad_payload;
        const int vb = pick_vec_bytes(a.row_bytes, addr_bits(grad_vals) | addr_bits(grad_payload));
        const int64_t rv = a.row_bytes / vb;
        a.fd_rv = FastDiv(static_cast<uint32_t>(rv));
        a.P = RAVEL_LK_BWD_P;
        a.nchunks = (T + a.P - 1) / a.P;
        return with_key(tl.kl.key64, [&](auto kt) -> int {
            using KeyT = decltype(kt);
            return with_dtype(dtype, [&](auto dtc) -> int {
                constexpr int DT = decltype(dtc)::value;
                return with_vb(vb, [&](auto vbc) -> int {
                    constexpr int VB = decltype(vbc)::value;
                    if constexpr (!vb_ok<DT, VB>()) {
                        return RAVEL_ERR_INVALID_ARG;
                    } else {
                        const size_t smem = lk_bwd_fast_smem(a.P, k);
                        k_lk_bwd_fast<KeyT, DT, VB><<<static_cast<unsigned>(S * a.nchunks), 256, smem, st>>>(a);
                        return check_launch();
                    }
                });
            });
        });
    }
    // general: a gather over the read tape, with one lane per vector when a row
    // splits into 2^m <= 32 vectors, else one warp per write over its elements
    {
        const int gvb = pick_vec_bytes(a.row_bytes, addr_bits(grad_vals) | addr_bits(grad_payload));
        const int64_t grv = a.row_bytes / gvb;
        if (grv >= 1 && grv <= 32 && (grv & (grv - 1)) == 0) {
            int lsh = 0;
            while ((int64_t{1} << lsh) < grv) ++lsh;
            a.out = grad_payload;
            const int64_t groups = B * C * T;
            const int64_t warps = (groups + (32 >> lsh) - 1) / (32 >> lsh);
            return with_key(tl.kl.key64, [&](auto kt) -> int {
                using KeyT = decltype(kt);
                return with_dtype(dtype, [&](auto dtc) -> int {
                    constexpr int DT = decltype(dtc)::value;
                    return with_vb(gvb, [&](auto vbc) -> int {
                        constexpr int VB = decltype(vbc)::value;
                        if constexpr (!vb_ok<DT, VB>()) {
                            return RAVEL_ERR_INVALID_ARG;
                        } else if (RAVEL_LK_BWD_CHUNK && k <= 64) {
                            // chunks of the write tape with their keys, bucket starts and read run staged
                            constexpr int kRcap = 1024;
                            a.P = 4 * 8 * (32 >> lsh);
                            a.nchunks = (T + a.P - 1) / a.P;
                            const size_t smem = lk_bwd_chunk_smem(a.P, k, kRcap, sizeof(KeyT));
                            if (int e = set_smem(k_lk_bwd_chunk<KeyT, DT, VB>, smem)) return e;
                            k_lk_bwd_chunk<KeyT, DT, VB><<<static_cast<unsigned>(B * C * a.nchunks), 256, smem, st>>>(
                                a, static_cast<const KeyT*>(tv.rkeys), tv.rridx, tv.bstart, lsh, kRcap);
                            return check_launch();
                        } else {
                            k_lk_bwd_gather<KeyT, DT, VB><<<grid_cap((warps * 32 + 255) / 256), 256, 0, st>>>(
                                a, static_cast<const KeyT*>(tv.rkeys), tv.rridx, tv.bstart, lsh);
                            return check_launch();
                        }
                    });
                });
            });
        }
    }
    // other row shapes: the same gather, one warp per write over the row's elements
    a.out = grad_payload;
    return with_key(tl.kl.key64, [&](auto kt) -> int {
        using KeyT = decltype(kt);
        return with_dtype(dtype, [&](auto dtc) -> int {
            constexpr int DT = decltype(dtc)::value;
            k_lk_bwd_gather_rows<KeyT, DT><<<grid_cap((B * C * T * 32 + 255) / 256), 256, 0, st>>>(
                a, static_cast<const KeyT*>(tv.rkeys), tv.rridx, tv.bstart);
            return check_launch();
        });
    });
}

// ------------------------------------------------------------------ segmented sum
template <typename KeyT, int DT>
int launch_segscan(const TapeView& tv, const TapeLayout& tl, int64_t B, int64_t T, int64_t C, int64_t D,
                   const void* in, int in_sorted, void* out, int out_sorted, uint8_t* out_mask, int inclusive,
                   int reverse, void* scratch, const ScratchLayout& sl, cudaStream_t st, int merged = 0,
                   int load_role = 0) {
    using Acc = typename Elem<DT>::Acc;
    const ScanPlan sp = scan_plan(T, D, DT);
    ScanArgs<Acc> a;
    a.keys = tv.keys;
    a.nvalid = tv.nvalid;
    a.B = B; a.T = T; a.C = C; a.D = D;
    a.tbits = tl.kl.tbits;
    a.in = in; a.out = out; a.out_mask = out_mask;
    a.in_sorted = in_sorted; a.out_sorted = out_sorted; a.inclusive = inclusive; a.reverse = reverse;
    a.P = sp.P; a.parts = sp.parts; a.nchunks = sp.nchunks;
    char* sc = static_cast<char*>(scratch);
    a.flags = reinterpret_cast<unsigned*>(sc + sl.off_flags);
    a.ticket = reinterpret_cast<unsigned*>(sc + sl.off_ticket);
    a.agg = reinterpret_cast<Acc*>(sc + sl.off_agg);
    a.incl = reinterpret_cast<Acc*>(sc + sl.off_incl);
    a.fd_d = FastDiv(static_cast<uint32_t>(D > 0 ? D : 1));
    using V = typename Elem<DT>::T;
    const size_t in_es = in_sorted ? sizeof(Acc) : sizeof(V);
    const size_t out_es = sizeof(V);  // sorted outputs are stored in the payload dtype too
    // group scan: rows of 16-byte vectors, 1..32 lanes per row (2 vectors per lane up to 1 KB rows)
    const int64_t nvec = (D * static_cast<int64_t>(in_es)) % 16 == 0 ? D * static_cast<int64_t>(in_es) / 16 : 0;
    int vpl = 0, lshift = 0;
    if (nvec > 0 && (nvec & (nvec - 1)) == 0 && nvec <= 64) {
        vpl = nvec >= RAVEL_RS_VPL2_NVEC ? 2 : 1;
        const int64_t L = nvec / vpl;
        while ((int64_t{1} << lshift) < L) ++lshift;
    }
    const size_t ovec = (16 / in_es) * out_es;  // output bytes per 16-byte input vector
    // merged scans (a general tape's writes and reads in one sequence, see k_range_scan):
    // row indices must leave bits 29 and 30 of the scan's row word free
    if (merged && !(vpl && addr_bits(in) % 16 == 0 && addr_bits(out) % ovec == 0 && B * T * C < (int64_t{1} << 29) &&
                    tv.mkeys != nullptr && !in_sorted && !out_sorted))
        return -1;  // not this kernel's shape: the caller takes the two-pass form
    if (vpl && addr_bits(in) % 16 == 0 && addr_bits(out) % ovec == 0) {
        const int64_t Tm = merged ? 2 * T : T;  // positions per stream of the scanned sequence
        GsArgs ga;
        ga.S = B * C;
        ga.keys = merged ? tv.mkeys : tv.keys;
        ga.role = merged ? tv.mrole : nullptr;
        ga.Ts = Tm;
        ga.load_role = load_role;
        ga.nvalid = tv.nvalid;
        ga.T = T; ga.C = C;
        ga.D = static_cast<uint32_t>(D);
        ga.tbits = tl.kl.tbits;
        ga.reverse = reverse;
        ga.lshift = lshift;
        ga.snap = GS_SNAP;
        ga.in = in; ga.out = out; ga.out_mask = out_mask;
        auto go = [&](auto vplc, auto inc, auto outc) -> int {
            constexpr int VPL = decltype(vplc)::value;
            constexpr bool IS = decltype(inc)::value != 0;
            constexpr bool OS = decltype(outc)::value != 0;
            auto kern = merged ? k_range_scan<KeyT, DT, false, false, false, VPL, true>
                               : (inclusive ? k_range_scan<KeyT, DT, IS, OS, true, VPL, false>
                                            : k_range_scan<KeyT, DT, IS, OS, false, VPL, false>);
            const int64_t gpb = GS_WARPS * (int64_t{32} >> lshift);
            constexpr int64_t kRlMax = 1024;
            const int64_t bmw_max = gpb * kRlMax / 32 + 2;
            const size_t smem_max = range_scan_smem(VPL, gpb, D, sizeof(Acc), bmw_max);
            if (int e = set_smem(kern, smem_max)) return e;
            const int occ = occupancy(kern, GS_WARPS * 32, range_scan_smem(VPL, gpb, D, sizeof(Acc), 2));
            // one range per lane group; whole blocks per stream, RAVEL_RS_WAVES waves of blocks
            // Short streams (64-position ranges do not fill one wave): about
            // RAVEL_RS_SHORT_BPS blocks per SM, ranges down to RAVEL_RS_RLMIN positions.
            const int64_t S = B * C > 0 ? B * C : 1;
            const int64_t blocks64 = S * (((Tm + 63) / 64 + gpb - 1) / gpb);
            const bool short_streams = blocks64 < static_cast<int64_t>(occ) * sm_count();
            int64_t bps = short_streams ? RAVEL_RS_SHORT_BPS * sm_count() / S
                                        : static_cast<int64_t>(occ) * sm_count() * RAVEL_RS_WAVES / S;
            if (bps < 1) bps = 1;
            const RangePlan rp = range_plan(1, Tm, bps * gpb, kRlMax, short_streams ? RAVEL_RS_RLMIN : 64);
            ga.R = rp.R;
            ga.RL = rp.RL;
            ga.snap = static_cast<int>(rp.RL / 2 < GS_SNAP ? rp.RL / 2 : GS_SNAP);
            ga.CB = (rp.R + gpb - 1) / gpb;
            ga.bmw = static_cast<int>(gpb * rp.RL / 32 + 2);
            ga.bflags = reinterpret_cast<unsigned*>(sc + sl.off_bflags);
            ga.bval = sc + sl.off_bval;
            const int64_t nblocks = B * C * ga.CB;
            if (cudaMemsetAsync(ga.bflags, 0, static_cast<size_t>(nblocks + 1) * 4, st) != cudaSuccess)
                return RAVEL_ERR_CUDA;
            const size_t smem = range_scan_smem(VPL, gpb, D, sizeof(Acc), ga.bmw);
            kern<<<static_cast<unsigned>(nblocks), GS_WARPS * 32, smem, st>>>(ga);
            return check_launch();
        };
        auto by_mode = [&](auto vplc) -> int {
            if (in_sorted) return go(vplc, IC<1>{}, IC<0>{});
            if (out_sorted) return go(vplc, IC<0>{}, IC<1>{});
            return go(vplc, IC<0>{}, IC<0>{});
        };
        return vpl == 2 ? by_mode(IC<2>{}) : by_mode(IC<1>{});
    }
    // fallbacks: chunked scans with decoupled look-back (flags start at zero)
    const int64_t nch = B * C * sp.nchunks;
    if (cudaMemsetAsync(a.flags, 0, sl.off_agg - sl.off_flags, st) != cudaSuccess) return RAVEL_ERR_CUDA;
    // warp-register kernel when one warp access covers a row
    int el = 0;
    for (int cand = 1; cand <= 8; cand *= 2) {
        if (D > 0 && D % cand == 0 && D / cand <= 32) { el = cand; break; }
    }
    if (el) {
        const bool aligned = addr_bits(in) % (el * in_es) == 0 && addr_bits(out) % (el * out_es) == 0;
        const int P = scanw_positions(D, static_cast<int>(in_es));
        if (aligned && P >= sp.min_P) {
            a.P = P;
            a.nchunks = (T + P - 1) / P;
            const int64_t nchw = B * C * a.nchunks;
            const size_t smem = segscan_w_smem<Acc>(D);
            auto go = [&](auto elc, auto inc, auto outc) -> int {
                constexpr int EL = decltype(elc)::value;
                constexpr bool IS = decltype(inc)::value != 0;
                constexpr bool OS = decltype(outc)::value != 0;
                constexpr int R = scanw_rows(EL, IS ? static_cast<int>(sizeof(Acc)) : static_cast<int>(sizeof(V)));
                auto kern = k_segscan_w<KeyT, DT, EL, IS, OS, R>;
                if (int e = set_smem(kern, smem)) return e;
                kern<<<static_cast<unsigned>(nchw), SCANW_WARPS * 32, smem, st>>>(a);
                return check_launch();
            };
            auto by_mode = [&](auto elc) -> int {
                if (in_sorted) return go(elc, IC<1>{}, IC<0>{});
                if (out_sorted) return go(elc, IC<0>{}, IC<1>{});
                return go(elc, IC<0>{}, IC<0>{});
            };
            switch (el) {
                case 1: return by_mode(IC<1>{});
                case 2: return by_mode(IC<2>{});
                case 4: return by_mode(IC<4>{});
                default: return by_mode(IC<8>{});
            }
        }
    }
    const size_t smem = segscan_smem<Acc>(sp.P, sp.parts, D);
    constexpr int EPV = 16 / sizeof(typename Elem<DT>::T);
    const bool vec = !in_sorted && !out_sorted && D % EPV == 0 && (addr_bits(in) % 16 == 0) &&
                     (addr_bits(out) % 16 == 0);
    const bool vec_in_only = false;
    (void)vec_in_only;
    if (vec) {
        if (int e = set_smem(k_segscan<KeyT, DT, true>, smem)) return e;
        k_segscan<KeyT, DT, true><<<static_cast<unsigned>(nch), SCAN_THREADS, smem, st>>>(a);
    } else {
        if (int e = set_smem(k_segscan<KeyT, DT, false>, smem)) return e;
        k_segscan<KeyT, DT, false><<<static_cast<unsigned>(nch), SCAN_THREADS, smem, st>>>(a);
    }
    return check_launch();
}

int ss_fwd_tape(const void* tape, int flags, const void* raddr, int addr_dtype, const void* payload, int dtype,
                int64_t B, int64_t T, int64_t C, int64_t D, int64_t A, void* out_sums, uint8_t* out_mask,
                void* scratch, size_t scratch_bytes, cudaStream_t st) {
    if (int e = check_sizes(B, T, C, D, A)) return e;
    if (dtype < 0 || dtype > 3) return RAVEL_ERR_INVALID_ARG;
    const int64_t N = B * T * C;
    if (N == 0) return RAVEL_OK;
    if (tape == nullptr || out_mask == nullptr || (D > 0 && (payload == nullptr || out_sums == nullptr)))
        return RAVEL_ERR_INVALID_ARG;
    const TapeLayout tl = tape_layout(B, T, C, A, flags);
    if (tl.general && raddr == nullptr) return RAVEL_ERR_INVALID_ARG;
    const ScratchLayout sl = scratch_layout(B, T, C, D, A, dtype, flags);
    if (scratch == nullptr || scratch_bytes < sl.total) return RAVEL_ERR_WORKSPACE;
    const TapeView tv = tape_view(tape, tl);
    return with_key(tl.kl.key64, [&](auto kt) -> int {
        using KeyT = decltype(kt);
        return with_dtype(dtype, [&](auto dtc) -> int {
            constexpr int DT = decltype(dtc)::value;
            if (!tl.general) {
                return launch_segscan<KeyT, DT>(tv, tl, B, T, C, D, payload, 0, out_sums, 0, out_mask,
                                                /*inclusive=*/0, /*reverse=*/0, scratch, sl, st);
            }
            // one scan over the merged sequence of valid writes and reads: writes add their
            // payload rows, reads store the running sum and the mask the merge decided
            if (D > 0) {
                const int rc = launch_segscan<KeyT, DT>(tv, tl, B, T, C, D, payload, 0, out_sums, 0, out_mask, 0, 0,
                                                        scratch, sl, st, /*merged=*/1, /*load_role=*/1);
                if (rc >= 0) return rc;
            }
            // other row shapes: an inclusive scan of the writes, then a gather per read
            void* tapebuf = static_cast<char*>(scratch) + sl.off_big;
            if (int e = launch_segscan<KeyT, DT>(tv, tl, B, T, C, D, payload, 0, tapebuf, 1, nullptr, 1, 0,
                                                 scratch, sl, st))
                return e;
            SsGenArgs g;
            std::memset(&g, 0, sizeof(g));
            g.keys = tv.keys; g.soff = tv.soff; g.ridx = tv.ridx;
            g.raddr = raddr;
            g.addr_i64 = addr_dtype == RAVEL_I64;
            g.key32 = key32_of(B, T, C, A);
            g.B = B; g.T = T; g.C = C; g.D = D; g.A = A;
            g.tbits = tl.kl.tbits;
            g.fd_C = FastDiv(static_cast<uint32_t>(C));
            g.fd_T = FastDiv(static_cast<uint32_t>(T));
            g.tapebuf = tapebuf;
            g.out = out_sums;
            g.out_mask = out_mask;
            g.vshift = vshift16(DT, D, addr_bits(out_sums) | addr_bits(tapebuf));
            k_ss_gather<KeyT, DT><<<grid_cap((N * 32 + 255) / 256), 256, 0, st>>>(g);
            return check_launch();
        });
    });
}

int ss_bwd(const void* tape, int flags, const void* raddr, int addr_dtype, const void* grad_sums, int dtype,
           int64_t B, int64_t T, int64_t C, int64_t D, int64_t A, void* grad_payload, void* scratch,
           size_t scratch_bytes, cudaStream_t st) {
    if (int e = check_sizes(B, T, C, D, A)) return e;
    if (dtype < 0 || dtype > 3) return RAVEL_ERR_INVALID_ARG;
    const int64_t N = B * T * C;
    if (N == 0 || D == 0) return RAVEL_OK;
    if (tape == nullptr || grad_sums == nullptr || grad_payload == nullptr) return RAVEL_ERR_INVALID_ARG;
    const TapeLayout tl = tape_layout(B, T, C, A, flags);
    if (tl.general && raddr == nullptr) return RAVEL_ERR_INVALID_ARG;
    const ScratchLayout sl = scratch_layout(B, T, C, D, A, dtype, flags);
    if (scratch == nullptr || scratch_bytes < sl.total) return RAVEL_ERR_WORKSPACE;
    const TapeView tv = tape_view(tape, tl);
    return with_key(tl.kl.key64, [&](auto kt) -> int {
        using KeyT = decltype(kt);
        return with_dtype(dtype, [&](auto dtc) -> int {
            constexpr int DT = decltype(dtc)::value;
            if (!tl.general) {
                return launch_segscan<KeyT, DT>(tv, tl, B, T, C, D, grad_sums, 0, grad_payload, 0, nullptr,
                                                /*inclusive=*/0, /*reverse=*/1, scratch, sl, st);
            }
            void* accbuf = static_cast<char*>(scratch) + sl.off_big;
            if (tl.has_mask &&
                cudaMemsetAsync(grad_payload, 0, static_cast<size_t>(N) * D * elem_bytes(DT), st) != cudaSuccess)
                return RAVEL_ERR_CUDA;
            // the merged sequence scanned from its end: reads add their gradient rows, every
            // valid write stores the running sum of the reads after it (masked writes stay 0)
            {
                const int rc = launch_segscan<KeyT, DT>(tv, tl, B, T, C, D, grad_sums, 0, grad_payload, 0, nullptr, 0,
                                                        1, scratch, sl, st, /*merged=*/1, /*load_role=*/0);
                if (rc >= 0) return rc;
            }
            // other row shapes: a reverse inclusive scan of the read gradients over the
            // read tape (suffix sums per address, payload dtype, in accbuf), then each
            // write copies the suffix at its first read ranked at or after it (one lane
            // per vector for rows of 2^m <= 32 vectors, else a warp over its elements)
            const int gvb = pick_vec_bytes(D * elem_bytes(DT), addr_bits(grad_sums) | addr_bits(grad_payload));
            const int64_t grv = D * elem_bytes(DT) / gvb;
            {
                TapeView rv = tv;
                rv.keys = tv.rkeys;
                rv.nvalid = nullptr;  // every read is on the read tape
                if (int e = launch_segscan<KeyT, DT>(rv, tl, B, T, C, D, grad_sums, 0, accbuf, 1, nullptr,
                                                     /*inclusive=*/1, /*reverse=*/1, scratch, sl, st))
                    return e;
            }
            if (grv >= 1 && grv <= 32 && (grv & (grv - 1)) == 0) {
                int lsh = 0;
                while ((int64_t{1} << lsh) < grv) ++lsh;
                const int64_t warps = (B * C * T + (32 >> lsh) - 1) / (32 >> lsh);
                return with_vb(gvb, [&](auto vbc) -> int {
                    constexpr int VB = decltype(vbc)::value;
                    if constexpr (!vb_ok<DT, VB>()) {
                        return RAVEL_ERR_INVALID_ARG;
                    } else {
                        k_ss_bwd_suffix<KeyT, DT, VB><<<grid_cap((warps * 32 + 255) / 256), 256, 0, st>>>(
                            static_cast<const KeyT*>(tv.keys), static_cast<const KeyT*>(tv.rkeys), tv.bstart, tv.nvalid,
                            accbuf, grad_payload, B * C, T, C, D, tl.kl.tbits, lsh);
                        return check_launch();
                    }
                });
            }
            k_ss_bwd_suffix_rows<KeyT, DT><<<grid_cap((B * C * T * 32 + 255) / 256), 256, 0, st>>>(
                static_cast<const KeyT*>(tv.keys), static_cast<const KeyT*>(tv.rkeys), tv.bstart, tv.nvalid, accbuf,
                grad_payload, B * C, T, C, D, tl.kl.tbits);
            return check_launch();
        });
    });
}

// ------------------------------------------------------------------ decode cache
// ------------------------------------------------------------------ decode cache bulk prefill
struct PrefillLayout {
    KeyLayout kl;
    size_t key_bytes, off_keys, off_other, total;
};

PrefillLayout prefill_layout(int64_t B, int64_t T, int64_t C, int64_t A) {
    PrefillLayout l;
    l.kl = key_layout(T, A, 0);
    l.key_bytes = l.kl.key64 ? 8 : 4;
    const size_t n = static_cast<size_t>(B * C) * static_cast<size_t>(T) * l.key_bytes;
    l.off_keys = 0;
    l.off_other = align_up(n);
    l.total = l.off_other + (sort_plan(T).tiles > 1 ? align_up(n) : 0);
    return l;
}

int cache_prefill(void* values, uint8_t* filled, const void* addr, int addr_dtype, const void* payload, int dtype,
                  int64_t B, int64_t T, int64_t C, int64_t A, int64_t D, void* scratch, size_t scratch_bytes,
                  cudaStream_t st) {
    if (int e = check_sizes(B, T, C, D, A)) return e;
    if (addr_dtype != RAVEL_I32 && addr_dtype != RAVEL_I64) return RAVEL_ERR_INVALID_ARG;
    if (dtype < 0 || dtype > 3) return RAVEL_ERR_INVALID_ARG;
    const int64_t S = B * C;
    if (S * T == 0) return RAVEL_OK;
    if (values == nullptr || filled == nullptr || addr == nullptr || (D > 0 && payload == nullptr))
        return RAVEL_ERR_INVALID_ARG;
    const PrefillLayout pl = prefill_layout(B, T, C, A);
    if (scratch == nullptr || scratch_bytes < pl.total) return RAVEL_ERR_WORKSPACE;
    char* sc = static_cast<char*>(scratch);
    SortArgs a;
    std::memset(&a, 0, sizeof(a));
    a.src = plain_src(addr, addr_dtype);
    a.key32 = 0;
    a.B = B; a.T = T; a.C = C; a.A = A;
    a.tbits = pl.kl.tbits; a.abits = pl.kl.abits; a.mbit = 0;
    a.clamp = 1;
    const int64_t row_bytes = D * elem_bytes(dtype);
    const int vb = row_bytes > 0 ? pick_vec_bytes(row_bytes, addr_bits(values) | addr_bits(payload)) : 2;
    return with_key(pl.kl.key64, [&](auto kt) -> int {
        using KeyT = decltype(kt);
        if (int e = sort_streams<KeyT>(a, sc + pl.off_keys, nullptr, nullptr, sc + pl.off_other, S, T, st)) return e;
        return with_vb(vb, [&](auto vbc) -> int {
            constexpr int VB = decltype(vbc)::value;
            k_cache_prefill<KeyT, VB><<<grid_cap((S * T + 255) / 256), 256, 0, st>>>(
                reinterpret_cast<const KeyT*>(sc + pl.off_keys), S, T, C, A, pl.kl.tbits, payload, row_bytes, values,
                filled);
            return check_launch();
        });
    });
}

int cache_op(void* values, uint8_t* filled, const void* raddr, const void* waddr, int addr_dtype,
             const void* payload, int dtype, int64_t B, int64_t C, int64_t A, int64_t D, void* out_vals,
             uint8_t* out_mask, cudaStream_t st) {
    if (B < 0 || C < 0 || D < 0 || A <= 0) return RAVEL_ERR_INVALID_ARG;
    if (addr_dtype != RAVEL_I32 && addr_dtype != RAVEL_I64) return RAVEL_ERR_INVALID_ARG;
    if (dtype < 0 || dtype > 3) return RAVEL_ERR_INVALID_ARG;
    const int64_t pairs = B * C;
    if (pairs == 0) return RAVEL_OK;
    if (values == nullptr || filled == nullptr) return RAVEL_ERR_INVALID_ARG;
    if (raddr != nullptr && (out_mask == nullptr || (D > 0 && out_vals == nullptr))) return RAVEL_ERR_INVALID_ARG;
    if (waddr != nullptr && D > 0 && payload == nullptr) return RAVEL_ERR_INVALID_ARG;
    CacheArgs a;
    a.values = values; a.filled = filled; a.raddr = raddr; a.waddr = waddr;
    a.addr_i64 = addr_dtype == RAVEL_I64;
    a.payload = payload; a.out_vals = out_vals; a.out_mask = out_mask;
    a.pairs = pairs; a.A = A;
    a.row_bytes = D * elem_bytes(dtype);
    const int vb = pick_vec_bytes(a.row_bytes, addr_bits(values) | addr_bits(payload) | addr_bits(out_vals));
    const int64_t rv = a.row_bytes / vb;
    int64_t ppc = rv > 0 ? 256 / rv : 256;
    if (ppc < 1) ppc = 1;
    a.pairs_per_cta = static_cast<int>(ppc);
    a.fd_rv = FastDiv(static_cast<uint32_t>(rv > 0 ? rv : 1));
    const unsigned grid = static_cast<unsigned>((pairs + ppc - 1) / ppc);
    return with_dtype(dtype, [&](auto dtc) -> int {
        constexpr int DT = decltype(dtc)::value;
        return with_vb(vb, [&](auto vbc) -> int {
            constexpr int VB = decltype(vbc)::value;
            if constexpr (!vb_ok<DT, VB>()) {
                return RAVEL_ERR_INVALID_ARG;
            } else {
                k_cache_step<DT, VB><<<grid, 256, 0, st>>>(a);
                return check_launch();
            }
        });
    });
}

__global__ void k_clear_error() { g_error_word = 0u; }

}  // namespace
}  // namespace ravel

// ------------------------------------------------------------------ no-allocation variant
// Tape and scratch of ravel_segsum_fwd_noalloc.  Host code must not use the
// array's name as a device pointer; its device address is looked up once per
// device below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[RAVEL_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_base[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (set up on first use).
int noalloc_base(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return RAVEL_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return RAVEL_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_base[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return RAVEL_ERR_CUDA;
        g_noalloc_base[dev] = p;
    }
    *out = g_noalloc_base[dev];
    return RAVEL_OK;
}
// ------------------------------------------------------------------ glue (gate residual, RMSNorm)
constexpr int64_t kRmsMaxK = 4096;
constexpr int64_t kRmsBwdBlocks = 296;  // fixed cap, so dg's summation order depends on M only

int64_t rms_bwd_blocks(int64_t M) {
    const int64_t b = (M + 7) / 8;
    return b < 1 ? 1 : (b > kRmsBwdBlocks ? kRmsBwdBlocks : b);
}

template <typename F>
int with_glue_type(int dtype, F&& f) {
    if (dtype == RAVEL_F32) return f(float(0));
    if (dtype == RAVEL_BF16) return f(__nv_bfloat16());
    return RAVEL_ERR_UNSUPPORTED;
}

int elem_vec_ok(int64_t n, int esize, std::initializer_list<const void*> ptrs) {
    if ((n * esize) % 16 != 0) return 0;
    for (const void* p : ptrs)
        if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return 0;
    return 1;
}
// ------------------------------------------------------------------ fused gather + fuse Linear
// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
int encode_weight_map(CUtensorMap* map, const float* W, int64_t N, int64_t K, int box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (encode == nullptr) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || fn == nullptr)
            return RAVEL_ERR_CUDA;
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 4};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(ravel::GG_BK), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(W), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? RAVEL_OK : RAVEL_ERR_CUDA;
}

// Rows of `rows` x D floats (payload or sums) for TMA gather4: boxes of one row x 32 floats.
int encode_rows_map(CUtensorMap* map, const float* base, int64_t rows, int64_t D) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    if (encode == nullptr) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || fn == nullptr)
            return RAVEL_ERR_CUDA;
        encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(D) * 4};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(ravel::GG_BK), 1};
    cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? RAVEL_OK : RAVEL_ERR_CUDA;
}

int gather_args(ravel::GatherArgs& g, const float* payload, const int32_t* src, const float* sums, int64_t B, int64_t T,
                int64_t C, int64_t D, int64_t k) {
    if (B < 0 || T < 0 || C <= 0 || D <= 0 || k <= 0) return RAVEL_ERR_INVALID_ARG;
    if (D % 4 != 0) return RAVEL_ERR_UNSUPPORTED;  // 16-byte pieces stay inside one slot
    const int64_t K = C * k * D + (sums ? C * D : 0);
    if (K > (int64_t{1} << 30) || B * T * C >= 2147483647LL) return RAVEL_ERR_UNSUPPORTED;
    if (payload == nullptr || src == nullptr) return RAVEL_ERR_INVALID_ARG;
    if (ravel::addr_bits(payload) % 16 || (sums && ravel::addr_bits(sums) % 16)) return RAVEL_ERR_INVALID_ARG;
    g.payload = payload; g.src = src; g.sums = sums;
    g.M = B * T;
    g.C = static_cast<int>(C); g.k = static_cast<int>(k); g.D = static_cast<int>(D); g.K = static_cast<int>(K);
    return RAVEL_OK;
}
// ------------------------------------------------------------------ per-entry GPU timing
// Off by default.  ravel_timing_start(n) makes n pairs of CUDA events; while it
// is on, each timed entry point records one pair on its stream around the work
// it enqueues (nothing while that stream is being captured into a graph), and
// ravel_timing_read returns the entry's name and the milliseconds between the
// pair.  One pair per call costs two cudaEventRecord calls of host time, less
// than timing the call from the caller's language.
struct EntryTiming {
    std::atomic<bool> on{false};
    std::atomic<int64_t> next{0};
    int64_t cap = 0;
    int device = -1;
    std::vector<cudaEvent_t> ev;         // 2 per record
    std::vector<const char*> name;       // entry point of each record
    std::vector<unsigned char> closed;   // the end event was recorded
};
EntryTiming g_timing;

class EntryTimer {
  public:
    EntryTimer(const char* entry, void* stream) : st_(static_cast<cudaStream_t>(stream)) {
        if (!g_timing.on.load(std::memory_order_acquire)) return;
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(st_, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return;
        const int64_t i = g_timing.next.fetch_add(1, std::memory_order_relaxed);
        if (i >= g_timing.cap) return;
        g_timing.name[i] = entry;
        if (cudaEventRecord(g_timing.ev[2 * i], st_) == cudaSuccess) slot_ = i;
    }
    ~EntryTimer() {
        if (slot_ >= 0 && cudaEventRecord(g_timing.ev[2 * slot_ + 1], st_) == cudaSuccess) g_timing.closed[slot_] = 1;
    }
    EntryTimer(const EntryTimer&) = delete;
    EntryTimer& operator=(const EntryTimer&) = delete;

  private:
    cudaStream_t st_;
    int64_t slot_ = -1;
};

void timing_release() {
    if (g_timing.device >= 0) {
        int cur = 0;
        const bool switched = cudaGetDevice(&cur) == cudaSuccess && cur != g_timing.device &&
                              cudaSetDevice(g_timing.device) == cudaSuccess;
        for (cudaEvent_t e : g_timing.ev) cudaEventDestroy(e);
        if (switched) cudaSetDevice(cur);
    }
    g_timing.ev.clear();
    g_timing.name.clear();
    g_timing.closed.clear();
    g_timing.cap = 0;
    g_timing.device = -1;
    g_timing.next.store(0);
}
}  // namespace

// one timing record around the rest of the enclosing entry point
#define RAVEL_TIMED(entry, stream) EntryTimer ravel_entry_timer_(entry, stream)

using namespace ravel;

extern "C" {

int ravel_set_wait_limit(uint32_t polls) {
    if (polls < 1 || polls > (1u << 28)) return RAVEL_ERR_INVALID_ARG;
    return cudaMemcpyToSymbol(g_wait_limit, &polls, sizeof(polls)) == cudaSuccess ? RAVEL_OK : RAVEL_ERR_CUDA;
}

int ravel_wait_selftest(const uint32_t* flag, void* stream) {
    if (flag == nullptr) return RAVEL_ERR_INVALID_ARG;
    k_wait_selftest<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flag);
    return check_launch();
}

int ravel_latestk_sources(const void* tape, int tape_flags, const void* raddr, int addr_dtype, int64_t B, int64_t T,
                          int64_t C, int64_t A, int64_t k, int32_t* src, void* stream) {
    RAVEL_TIMED("ravel_latestk_sources", stream);
    if (int e = check_sizes(B, T, C, 0, A)) return e;
    if (k <= 0) return RAVEL_ERR_INVALID_ARG;
    if (k > 512) return RAVEL_ERR_UNSUPPORTED;
    const int64_t N = B * T * C;
    if (N == 0) return RAVEL_OK;
    if (tape == nullptr || src == nullptr) return RAVEL_ERR_INVALID_ARG;
    const TapeLayout tl = tape_layout(B, T, C, A, tape_flags);
    if (tl.general && raddr == nullptr) return RAVEL_ERR_INVALID_ARG;
    const TapeView tv = tape_view(tape, tl);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    return with_key(tl.kl.key64, [&](auto kt) -> int {
        using KeyT = decltype(kt);
        if (!tl.general) {
            k_lk_sources_aliased<KeyT><<<grid_cap((N + 255) / 256), 256, 0, st>>>(
                static_cast<const KeyT*>(tv.keys), B * C, T, C, tl.kl.tbits, static_cast<int>(k), src);
        } else {
            LkArgs a = lk_args(tv, tl, raddr, addr_dtype, B, T, C, 1, A, k, RAVEL_F32);
            k_lk_sources_general<KeyT><<<grid_cap((N * k + 255) / 256), 256, 0, st>>>(a, src);
        }
        return check_launch();
    });
}

int ravel_gather_rows(const float* payload, const int32_t* src, const float* sums, int64_t B, int64_t T, int64_t C,
                      int64_t D, int64_t k, float* rows, void* stream) {
    RAVEL_TIMED("ravel_gather_rows", stream);
    GatherArgs g;
    if (int e = gather_args(g, payload, src, sums, B, T, C, D, k)) return e;
    if (g.M == 0) return RAVEL_OK;
    if (rows == nullptr || addr_bits(rows) % 16) return RAVEL_ERR_INVALID_ARG;
    const int64_t pieces = g.M * (g.K / 4);
    k_gather_rows<<<grid_cap((pieces + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(g, rows);
    return check_launch();
}

int ravel_gather_gemm(const float* payload, const int32_t* src, const float* sums, int64_t B, int64_t T, int64_t C,
                      int64_t D, int64_t k, const float* weight, int64_t N, const float* x, const float* gate,
                      float* out, float* pre, void* stream) {
    RAVEL_TIMED("ravel_gather_gemm", stream);
    GemmArgs a;
    std::memset(&a, 0, sizeof(a));
    if (int e = gather_args(a.g, payload, src, sums, B, T, C, D, k)) return e;
    if (N <= 0 || N > (int64_t{1} << 24)) return RAVEL_ERR_INVALID_ARG;
    if (a.g.M == 0) return RAVEL_OK;
    if (weight == nullptr || out == nullptr || ((x == nullptr) != (gate == nullptr))) return RAVEL_ERR_INVALID_ARG;
    if (addr_bits(weight) % 16 || (a.g.K * 4) % 16) return RAVEL_ERR_UNSUPPORTED;  // TMA rows: 16-byte strides
    for (const void* p : {static_cast<const void*>(out), static_cast<const void*>(pre), static_cast<const void*>(x),
                          static_cast<const void*>(gate)})
        if (p != nullptr && addr_bits(p) % 16) return RAVEL_ERR_INVALID_ARG;
    a.N = static_cast<int>(N);
    a.out = out; a.pre = pre; a.x = x; a.gate = gate;
    const int64_t mtiles = (a.g.M + GG_BM - 1) / GG_BM;
    // one wave of CTAs where possible: 256-column tiles once the token tiles fill the SMs
#ifdef RAVEL_GG_FORCE_BN
    const int bn = RAVEL_GG_FORCE_BN;  // build-time tuning knob (sweeps)
#else
    const int bn = N <= 64 ? 64 : ((N <= 128 || mtiles < sm_count()) ? 128 : 256);
#endif
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    // A tiles by TMA gather4 (a K chunk of 32 floats inside one slot) or by the cp.async
    // producers.  Measured at config-5 layer shapes: gather4 68 us, cp.async 42-46 us --
    // 768 four-row gathers per CTA keep the TMA unit busy ~170 cycles each -- so
    // cp.async is the default and gather4 a build-time option.
#ifdef RAVEL_GG_GATHER4
    const bool gather4 = a.g.D % GG_BK == 0;
#else
    const bool gather4 = false;
#endif
    auto go = [&](auto bnc) -> int {
        constexpr int BN = decltype(bnc)::value;
        CUtensorMap map, pmap, smap;
        if (int e = encode_weight_map(&map, weight, N, a.g.K, BN)) return e;
        std::memset(&pmap, 0, sizeof(pmap));
        std::memset(&smap, 0, sizeof(smap));
        if (gather4) {
            if (int e = encode_rows_map(&pmap, payload, a.g.M * C, D)) return e;
            if (int e = encode_rows_map(&smap, sums ? sums : payload, a.g.M * C, D)) return e;
        }
        const int ck = a.g.C * a.g.k;
        a.ck_smem = gather_gemm_smem<BN>(ck) <= 227 * 1024 ? ck : 0;  // stage the source table if it fits
        const size_t smem = gather_gemm_smem<BN>(a.ck_smem);
        const dim3 grid(static_cast<unsigned>(mtiles), static_cast<unsigned>((N + BN - 1) / BN));
        if (gather4) {
            if (int e = set_smem(k_gather_gemm<BN, true>, smem)) return e;
            k_gather_gemm<BN, true><<<grid, GG_THREADS, smem, st>>>(map, pmap, smap, a);
        } else {
            if (int e = set_smem(k_gather_gemm<BN, false>, smem)) return e;
            k_gather_gemm<BN, false><<<grid, GG_THREADS, smem, st>>>(map, pmap, smap, a);
        }
        return check_launch();
    };
    if (bn == 64) return go(IC<64>{});
    if (bn == 128) return go(IC<128>{});
    return go(IC<256>{});
}

int ravel_tape_build_tokens(const int64_t* tokens, int n_literal, int64_t bos_token_id, const void* learned_write,
                            const void* learned_read, int learned_dtype, const uint8_t* wmask, int64_t B, int64_t T,
                            int64_t C, int64_t A, int tape_flags, int32_t* read_addr_out, void* tape,
                            size_t tape_bytes, void* scratch, size_t scratch_bytes, void* stream) {
    RAVEL_TIMED("ravel_tape_build_tokens", stream);
    if (n_literal < 0 || n_literal > C) return RAVEL_ERR_INVALID_ARG;
    if (learned_dtype != RAVEL_I32 && learned_dtype != RAVEL_I64) return RAVEL_ERR_INVALID_ARG;
    if (B * T * C == 0) return RAVEL_OK;
    if (tokens == nullptr) return RAVEL_ERR_INVALID_ARG;
    if (n_literal < C && learned_write == nullptr) return RAVEL_ERR_INVALID_ARG;
    if (n_literal < C && (tape_flags & RAVEL_TAPE_GENERAL_READS) && learned_read == nullptr)
        return RAVEL_ERR_INVALID_ARG;
    if (tape_flags != 0 && read_addr_out == nullptr) return RAVEL_ERR_INVALID_ARG;
    if (A > 2147483647) return RAVEL_ERR_UNSUPPORTED;  // folded read addresses are stored as int32
    AddrSrc w;
    std::memset(&w, 0, sizeof(w));
    w.addr = learned_write;
    w.i64 = learned_dtype == RAVEL_I64;
    w.tokens = tokens;
    w.lit = n_literal;
    w.bos = bos_token_id;
    AddrSrc r = w;
    if (tape_flags & RAVEL_TAPE_GENERAL_READS) r.addr = learned_read;
    return tape_build_src(w, r, read_addr_out, wmask, B, T, C, A, tape_flags, tape, tape_bytes, scratch,
                          scratch_bytes, static_cast<cudaStream_t>(stream));
}

int ravel_literal_addresses(const int64_t* tokens, int64_t B, int64_t T, int n_heads, int64_t bos_token_id,
                            int64_t A, int64_t* out, void* stream) {
    RAVEL_TIMED("ravel_literal_addresses", stream);
    if (B < 0 || T < 0 || n_heads < 0 || A <= 0) return RAVEL_ERR_INVALID_ARG;
    const int64_t n = B * T * n_heads;
    if (n == 0) return RAVEL_OK;
    if (tokens == nullptr || out == nullptr) return RAVEL_ERR_INVALID_ARG;
    k_literal_addresses<<<grid_cap((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        tokens, B, T, n_heads, bos_token_id, A, out);
    return check_launch();
}

int ravel_gate_residual_fwd(const void* x, const void* gate, const void* fused, void* out, int64_t n, int dtype,
                            void* stream) {
    RAVEL_TIMED("ravel_gate_residual_fwd", stream);
    if (n < 0) return RAVEL_ERR_INVALID_ARG;
    if (n == 0) return RAVEL_OK;
    if (!x || !gate || !fused || !out) return RAVEL_ERR_INVALID_ARG;
    return with_glue_type(dtype, [&](auto tv) -> int {
        using T = decltype(tv);
        const int vec = elem_vec_ok(n, sizeof(T), {x, gate, fused, out});
        const int64_t units = vec ? n / (16 / sizeof(T)) : n;
        k_gate_res_fwd<T><<<grid_cap((units + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const T*>(x), static_cast<const T*>(gate), static_cast<const T*>(fused),
            static_cast<T*>(out), n, vec);
        return check_launch();
    });
}

int ravel_gate_residual_bwd(const void* gate, const void* fused, const void* grad_out, void* grad_gate,
                            void* grad_fused, int64_t n, int dtype, void* stream) {
    RAVEL_TIMED("ravel_gate_residual_bwd", stream);
    if (n < 0) return RAVEL_ERR_INVALID_ARG;
    if (n == 0) return RAVEL_OK;
    if (!gate || !fused || !grad_out || !grad_gate || !grad_fused) return RAVEL_ERR_INVALID_ARG;
    return with_glue_type(dtype, [&](auto tv) -> int {
        using T = decltype(tv);
        const int vec = elem_vec_ok(n, sizeof(T), {gate, fused, grad_out, grad_gate, grad_fused});
        const int64_t units = vec ? n / (16 / sizeof(T)) : n;
        k_gate_res_bwd<T><<<grid_cap((units + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const T*>(gate), static_cast<const T*>(fused), static_cast<const T*>(grad_out),
            static_cast<T*>(grad_gate), static_cast<T*>(grad_fused), n, vec);
        return check_launch();
    });
}

size_t ravel_rms_norm_scratch_bytes(int64_t M, int64_t K) {
    if (M < 0 || K <= 0) return 0;
    return static_cast<size_t>(rms_bwd_blocks(M) * K) * sizeof(float);
}

int ravel_rms_norm_fwd(const void* x, const void* weight, float eps, void* y, float* rstd, int64_t M, int64_t K,
                       int dtype, void* stream) {
    RAVEL_TIMED("ravel_rms_norm_fwd", stream);
    if (M < 0 || K <= 0) return RAVEL_ERR_INVALID_ARG;
    if (K > kRmsMaxK) return RAVEL_ERR_UNSUPPORTED;
    if (M == 0) return RAVEL_OK;
    if (!x || !weight || !y || !rstd) return RAVEL_ERR_INVALID_ARG;
    return with_glue_type(dtype, [&](auto tv) -> int {
        using T = decltype(tv);
        k_rms_fwd<T><<<grid_cap((M + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
            static_cast<const T*>(x), static_cast<const T*>(weight), static_cast<T*>(y), rstd, M,
            static_cast<int>(K), eps);
        return check_launch();
    });
}

int ravel_rms_norm_bwd(const void* x, const void* weight, const void* grad_y, const float* rstd, void* grad_x,
                       void* grad_weight, int64_t M, int64_t K, int dtype, void* scratch, size_t scratch_bytes,
                       void* stream) {
    RAVEL_TIMED("ravel_rms_norm_bwd", stream);
    if (M < 0 || K <= 0) return RAVEL_ERR_INVALID_ARG;
    if (K > kRmsMaxK) return RAVEL_ERR_UNSUPPORTED;
    if (!x || !weight || !grad_y || !rstd || !grad_x || !grad_weight) return RAVEL_ERR_INVALID_ARG;
    if (scratch == nullptr || scratch_bytes < ravel_rms_norm_scratch_bytes(M, K)) return RAVEL_ERR_WORKSPACE;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    return with_glue_type(dtype, [&](auto tv) -> int {
        using T = decltype(tv);
        const int64_t nb = rms_bwd_blocks(M);
        float* part = static_cast<float*>(scratch);
        const size_t smem = static_cast<size_t>(8 * K) * sizeof(float);
        if (int e = set_smem(k_rms_bwd<T>, smem)) return e;
        k_rms_bwd<T><<<static_cast<unsigned>(nb), 256, smem, st>>>(
            static_cast<const T*>(x), static_cast<const T*>(weight), static_cast<const T*>(grad_y), rstd,
            static_cast<T*>(grad_x), part, M, static_cast<int>(K));
        if (int e = check_launch()) return e;
        k_rms_dg_reduce<T><<<static_cast<unsigned>((K + 255) / 256), 256, 0, st>>>(
            part, static_cast<int>(nb), static_cast<int>(K), static_cast<T*>(grad_weight));
        return check_launch();
    });
}


size_t ravel_tape_bytes(int64_t B, int64_t T, int64_t C, int64_t A, int tape_flags) {
    if (B < 0 || T < 0 || C < 0 || A <= 0) return 0;
    return tape_layout(B, T, C, A, tape_flags).total;
}

size_t ravel_scratch_bytes(int64_t B, int64_t T, int64_t C, int64_t D, int64_t A, int64_t k, int dtype,
                           int tape_flags) {
    (void)k;
    if (B < 0 || T < 0 || C < 0 || D < 0 || A <= 0 || dtype < 0 || dtype > 3) return 0;
    return scratch_layout(B, T, C, D, A, dtype, tape_flags).total;
}

int ravel_tape_build(const void* waddr, const void* raddr, int addr_dtype, const uint8_t* wmask, int64_t B,
                     int64_t T, int64_t C, int64_t A, int tape_flags, void* tape, size_t tape_bytes,
                     void* scratch, size_t scratch_bytes, void* stream) {
    RAVEL_TIMED("ravel_tape_build", stream);
    return tape_build(waddr, raddr, addr_dtype, wmask, B, T, C, A, tape_flags, tape, tape_bytes, scratch,
                      scratch_bytes, static_cast<cudaStream_t>(stream));
}

int ravel_latestk_fwd_tape(const void* tape, int tape_flags, const void* raddr, int addr_dtype,
                           const void* payload, int dtype, int64_t B, int64_t T, int64_t C, int64_t D,
                           int64_t A, int64_t k, void* out_vals, uint8_t* out_mask, void* stream) {
    RAVEL_TIMED("ravel_latestk_fwd_tape", stream);
    return lk_fwd_tape(tape, tape_flags, raddr, addr_dtype, payload, dtype, B, T, C, D, A, k, out_vals, out_mask,
                       static_cast<cudaStream_t>(stream));
}

int ravel_latestk_fwd(const void* waddr, const void* raddr, int addr_dtype, const uint8_t* wmask,
                      const void* payload, int dtype, int64_t B, int64_t T, int64_t C, int64_t D, int64_t A,
                      int64_t k, void* out_vals, uint8_t* out_mask, void* tape, size_t tape_bytes,
                      void* scratch, size_t scratch_bytes, void* stream) {
    RAVEL_TIMED("ravel_latestk_fwd", stream);
    if (raddr == waddr) raddr = nullptr;
    const int flags = (raddr ? RAVEL_TAPE_GENERAL_READS : 0) | (wmask ? RAVEL_TAPE_WRITE_MASK : 0);
    if (k <= 0) return RAVEL_ERR_INVALID_ARG;
    if (int e = tape_build(waddr, raddr, addr_dtype, wmask, B, T, C, A, flags, tape, tape_bytes, scratch,
                           scratch_bytes, static_cast<cudaStream_t>(stream)))
        return e;
    return lk_fwd_tape(tape, flags, raddr ? raddr : waddr, addr_dtype, payload, dtype, B, T, C, D, A, k,
                       out_vals, out_mask, static_cast<cudaStream_t>(stream));
}

int ravel_latestk_bwd(const void* tape, int tape_flags, const void* raddr, int addr_dtype, const void* grad_vals,
                      int dtype, int64_t B, int64_t T, int64_t C, int64_t D, int64_t A, int64_t k,
                      void* grad_payload, void* scratch, size_t scratch_bytes, void* stream) {
    RAVEL_TIMED("ravel_latestk_bwd", stream);
    return lk_bwd(tape, tape_flags, raddr, addr_dtype, grad_vals, dtype, B, T, C, D, A, k, grad_payload, scratch,
                  scratch_bytes, static_cast<cudaStream_t>(stream));
}

int ravel_latestk_bwd_accumulate(const void* tape, int tape_flags, const void* raddr, int addr_dtype,
                                 const void* grad_vals, int dtype, int64_t B, int64_t T, int64_t C, int64_t D,
                                 int64_t A, int64_t k, void* grad_payload, void* scratch, size_t scratch_bytes,
                                 void* stream) {
    RAVEL_TIMED("ravel_latestk_bwd_accumulate", stream);
    return lk_bwd(tape, tape_flags, raddr, addr_dtype, grad_vals, dtype, B, T, C, D, A, k, grad_payload, scratch,
                  scratch_bytes, static_cast<cudaStream_t>(stream), /*accumulate=*/1);
}

int ravel_segsum_fwd_tape(const void* tape, int tape_flags, const void* raddr, int addr_dtype,
                          const void* payload, int dtype, int64_t B, int64_t T, int64_t C, int64_t D, int64_t A,
                          void* out_sums, uint8_t* out_mask, void* scratch, size_t scratch_bytes, void* stream) {
    RAVEL_TIMED("ravel_segsum_fwd_tape", stream);
    return ss_fwd_tape(tape, tape_flags, raddr, addr_dtype, payload, dtype, B, T, C, D, A, out_sums, out_mask,
                       scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
}

int ravel_segsum_fwd(const void* waddr, const void* raddr, int addr_dtype, const uint8_t* wmask,
                     const void* payload, int dtype, int64_t B, int64_t T, int64_t C, int64_t D, int64_t A,
                     void* out_sums, uint8_t* out_mask, void* tape, size_t tape_bytes, void* scratch,
                     size_t scratch_bytes, void* stream) {
    RAVEL_TIMED("ravel_segsum_fwd", stream);
    if (raddr == waddr) raddr = nullptr;
    const int flags = (raddr ? RAVEL_TAPE_GENERAL_READS : 0) | (wmask ? RAVEL_TAPE_WRITE_MASK : 0);
    if (int e = tape_build(waddr, raddr, addr_dtype, wmask, B, T, C, A, flags, tape, tape_bytes, scratch,
                           scratch_bytes, static_cast<cudaStream_t>(stream)))
        return e;
    return ss_fwd_tape(tape, flags, raddr ? raddr : waddr, addr_dtype, payload, dtype, B, T, C, D, A, out_sums,
                       out_mask, scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
}

int ravel_segsum_fwd_noalloc(const void* waddr, const void* raddr, int addr_dtype, const uint8_t* wmask,
                             const void* payload, int dtype, int64_t B, int64_t T, int64_t C, int64_t D, int64_t A,
                             void* out_sums, uint8_t* out_mask, void* stream) {
    RAVEL_TIMED("ravel_segsum_fwd_noalloc", stream);
    if (raddr == waddr) raddr = nullptr;
    const int flags = (raddr ? RAVEL_TAPE_GENERAL_READS : 0) | (wmask ? RAVEL_TAPE_WRITE_MASK : 0);
    if (int e = check_sizes(B, T, C, D, A)) return e;
    if (dtype < 0 || dtype > 3) return RAVEL_ERR_INVALID_ARG;
    const size_t tape_sz = align_up(tape_layout(B, T, C, A, flags).total);
    const size_t scratch_sz = scratch_layout(B, T, C, D, A, dtype, flags).total;
    if (tape_sz + scratch_sz > RAVEL_NOALLOC_SCRATCH_BYTES) return RAVEL_ERR_WORKSPACE;
    void* base = nullptr;
    if (int e = noalloc_base(&base)) return e;
    void* tape = base;
    void* scratch = static_cast<char*>(base) + tape_sz;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (int e = tape_build(waddr, raddr, addr_dtype, wmask, B, T, C, A, flags, tape, tape_sz, scratch, scratch_sz, st))
        return e;
    return ss_fwd_tape(tape, flags, raddr ? raddr : waddr, addr_dtype, payload, dtype, B, T, C, D, A, out_sums,
                       out_mask, scratch, scratch_sz, st);
}

int ravel_segsum_bwd(const void* tape, int tape_flags, const void* raddr, int addr_dtype, const void* grad_sums,
                     int dtype, int64_t B, int64_t T, int64_t C, int64_t D, int64_t A, void* grad_payload,
                     void* scratch, size_t scratch_bytes, void* stream) {
    RAVEL_TIMED("ravel_segsum_bwd", stream);
    return ss_bwd(tape, tape_flags, raddr, addr_dtype, grad_sums, dtype, B, T, C, D, A, grad_payload, scratch,
                  scratch_bytes, static_cast<cudaStream_t>(stream));
}

int ravel_cache_read(const void* values, const uint8_t* filled, const void* addr, int addr_dtype, int dtype,
                     int64_t B, int64_t C, int64_t A, int64_t D, void* out_vals, uint8_t* out_mask, void* stream) {
    RAVEL_TIMED("ravel_cache_read", stream);
    if (addr == nullptr) return RAVEL_ERR_INVALID_ARG;
    return cache_op(const_cast<void*>(values), const_cast<uint8_t*>(filled), addr, nullptr, addr_dtype, nullptr,
                    dtype, B, C, A, D, out_vals, out_mask, static_cast<cudaStream_t>(stream));
}

int ravel_cache_write(void* values, uint8_t* filled, const void* addr, int addr_dtype, const void* payload,
                      int dtype, int64_t B, int64_t C, int64_t A, int64_t D, void* stream) {
    RAVEL_TIMED("ravel_cache_write", stream);
    if (addr == nullptr) return RAVEL_ERR_INVALID_ARG;
    return cache_op(values, filled, nullptr, addr, addr_dtype, payload, dtype, B, C, A, D, nullptr, nullptr,
                    static_cast<cudaStream_t>(stream));
}

int ravel_cache_step(void* values, uint8_t* filled, const void* raddr, const void* waddr, int addr_dtype,
                     const void* payload, int dtype, int64_t B, int64_t C, int64_t A, int64_t D, void* out_vals,
                     uint8_t* out_mask, void* stream) {
    RAVEL_TIMED("ravel_cache_step", stream);
    if (raddr == nullptr || waddr == nullptr) return RAVEL_ERR_INVALID_ARG;
    return cache_op(values, filled, raddr, waddr, addr_dtype, payload, dtype, B, C, A, D, out_vals, out_mask,
                    static_cast<cudaStream_t>(stream));
}

size_t ravel_cache_prefill_scratch_bytes(int64_t B, int64_t T, int64_t C, int64_t A) {
    if (B < 0 || T < 0 || C < 0 || A <= 0) return 0;
    return prefill_layout(B, T, C, A).total;
}

int ravel_cache_prefill(void* values, uint8_t* filled, const void* addr, int addr_dtype, const void* payload,
                        int dtype, int64_t B, int64_t T, int64_t C, int64_t A, int64_t D, void* scratch,
                        size_t scratch_bytes, void* stream) {
    RAVEL_TIMED("ravel_cache_prefill", stream);
    return cache_prefill(values, filled, addr, addr_dtype, payload, dtype, B, T, C, A, D, scratch, scratch_bytes,
                         static_cast<cudaStream_t>(stream));
}

int ravel_device_error(int* out, void* stream) {
    if (out == nullptr) return RAVEL_ERR_INVALID_ARG;
    unsigned int v = 0;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyFromSymbolAsync(&v, g_error_word, sizeof(v), 0, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return RAVEL_ERR_CUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return RAVEL_ERR_CUDA;
    *out = static_cast<int>(v);
    return RAVEL_OK;
}

int ravel_clear_device_error(void* stream) {
    k_clear_error<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>();
    return check_launch();
}

uint64_t ravel_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

int ravel_timing_start(int64_t max_records) {
    if (max_records <= 0 || max_records > (int64_t{1} << 20)) return RAVEL_ERR_INVALID_ARG;
    g_timing.on.store(false);
    timing_release();
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return RAVEL_ERR_CUDA;
    g_timing.device = dev;
    g_timing.ev.reserve(static_cast<size_t>(2 * max_records));
    for (int64_t i = 0; i < 2 * max_records; ++i) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) {
            timing_release();
            return RAVEL_ERR_CUDA;
        }
        g_timing.ev.push_back(e);
    }
    g_timing.name.assign(static_cast<size_t>(max_records), nullptr);
    g_timing.closed.assign(static_cast<size_t>(max_records), 0);
    g_timing.cap = max_records;
    g_timing.next.store(0);
    g_timing.on.store(true, std::memory_order_release);
    return RAVEL_OK;
}

int ravel_timing_stop(void) {
    g_timing.on.store(false, std::memory_order_release);
    return RAVEL_OK;
}

int64_t ravel_timing_count(void) {
    const int64_t n = g_timing.next.load();
    return n < g_timing.cap ? n : g_timing.cap;
}

int ravel_timing_read(int64_t i, const char** entry, float* ms) {
    if (entry == nullptr || ms == nullptr || i < 0 || i >= ravel_timing_count()) return RAVEL_ERR_INVALID_ARG;
    if (g_timing.name[i] == nullptr || !g_timing.closed[i]) return RAVEL_ERR_INVALID_ARG;
    if (cudaEventSynchronize(g_timing.ev[2 * i + 1]) != cudaSuccess) return RAVEL_ERR_CUDA;
    if (cudaEventElapsedTime(ms, g_timing.ev[2 * i], g_timing.ev[2 * i + 1]) != cudaSuccess) return RAVEL_ERR_CUDA;
    *entry = g_timing.name[i];
    return RAVEL_OK;
}

const char* ravel_status_string(int status) {
    switch (status) {
        case RAVEL_OK: return "ok";
        case RAVEL_ERR_INVALID_ARG: return "invalid argument";
        case RAVEL_ERR_WORKSPACE: return "tape or scratch buffer too small";
        case RAVEL_ERR_CUDA: return "CUDA launch or runtime error";
        case RAVEL_ERR_UNSUPPORTED: return "sizes beyond the supported range";
        case RAVEL_ERR_DEVICE: return "a kernel reported an error";
        default: return "unknown status";
    }
}

const char* ravel_version(void) { return "ravel_b200 0.1.0 (sm_100a)"; }

}  // extern "C"
