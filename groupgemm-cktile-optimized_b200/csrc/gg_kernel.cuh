// Persistent, warp-specialised grouped GEMM for sm_100a (B200):
//
//     out[rows of group g] = x[rows of group g] @ w[g]^T      (RCR, fp32 accumulate)
//
//   x   [sum(M_g), K] row-major  -- A operand, K-major
//   w   [G, N, K]     row-major  -- B operand, K-major
//   out [sum(M_g), N] row-major
//
// This replaces the reference's CK Tile GroupedGemmKernel + HandPipelineAsmS main loop +
// FastEpilogue (ck_kernel/ck_grouped_gemm.cpp:34-124, ck_kernel/hand_pipeline_asm_s.hpp:157-357,
// ck_kernel/fast_epilogue.hpp:29-118) with a Blackwell design:
//
//   * one CTA per SM (kCG = 1) or one CTA pair per two SMs (kCG = 2, tcgen05 cta_group::2),
//     persistent over a static schedule of work units that covers every group (the scheduler
//     is on the device: a unit is a tile or a contiguous K range of one -- a split-K split or a
//     stream-K piece --, a tile index is mapped to (group, m-tile, n-tile) from per-group tile
//     offsets);
//   * warp 0: TMA producer. 128-byte-swizzled A (128 x 64) and B (BN/kCG x 64) tiles into a
//     STAGES-deep shared-memory ring guarded by full/empty mbarriers (no multicast: every CTA
//     loads its own halves);
//   * warp 1: TMEM allocator and, in the pair leader, the MMA issuer. The accumulator lives in
//     Tensor Memory, double-buffered (2 x BN fp32 columns) so the epilogue of tile i overlaps
//     the main loop of tile i+1;
//   * the producer and MMA warps run their loops converged and one elected lane issues the
//     single-thread instructions (predicated), which keeps the MMA issue at the tensor pipe's
//     rate for every tile width;
//   * warps 2-5: epilogue. tcgen05.ld 32 lanes x 32 columns, fp32 -> bf16/fp16 (RNE), then
//     per warp 32-row x 64-column boxes through 128-byte-swizzled shared-memory staging and TMA
//     stores with an evict-first L2 policy (the analogue of the reference's non-temporal C
//     stores, ck_kernel/coherence_epilogue.hpp:17-30); slabs that cross a group's end, column
//     tails and split-K sums use masked 32-byte streaming stores;
//   * launched with programmatic stream serialisation: on-chip set-up overlaps the previous
//     kernel, global memory is touched only after griddepcontrol.wait.
//
// Tails: TMA zero-fills reads past the tensor ends (K tail, N tail via the 3-D weight map,
// rows past sum(M)). A tile that runs past its group's last row reads the next group's rows;
// those accumulator rows are never stored. There is no K % 64 restriction (the reference
// refuses one, ck_kernel/ck_grouped_gemm.cpp:191-193).
//
// Every wait is bounded. A wait that runs out sets a device status word (role and barrier)
// and all roles leave their loops; the kernel then frees its Tensor Memory and returns.
//
// The same kernel, instantiated per operation (kOp), computes the two backward grouped GEMMs of
// the MoE layer (the transA / non-transA calls of the reference's vendored Primus-Turbo grouped
// GEMM, third_party/primus_turbo/kernels/hipblaslt_grouped_gemm.cu:80-96,199-240):
//
//   dgrad: dx[rows of g] = dy[rows of g] @ w[g]      dy [sum(M), N] (A, K-major over N),
//                                                    w[g] [N, K] (B, MN-major), dx [sum(M), K]
//   wgrad: dw[g] = dy[rows of g]^T @ x[rows of g]    dy^T (A, MN-major), x (B, MN-major),
//                                                    dw [G, N, K]; the reduction runs over the
//                                                    group's tokens, an expert without tokens
//                                                    gets dw[g] = 0
//
// MN-major operands are loaded as 64-wide boxes (one 128-byte swizzle row each) and described to
// the tensor core with MN-major shared-memory descriptors; no transpose pass is needed. For wgrad
// the K tail of every group (tokens past the group's last row) must read zeros, so each group has
// its own pair of tensor maps, bounded by the group's rows, in global memory.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "gg_ptx.cuh"

#ifndef GG_TMA_STORE
#define GG_TMA_STORE 1
#endif

namespace gg {

constexpr int kThreads = 192;  // 6 warps: producer, MMA, 4 x epilogue
constexpr int kBM = 128;       // accumulator rows per CTA (TMEM lanes)
constexpr int kBK = 64;        // K per swizzle atom: one 128-byte row of 16-bit elements
constexpr int kUmmaK = 16;     // K per tcgen05.mma (kind::f16)
constexpr int kSmemBudget = 200 * 1024;

// Status word values (0 = ok). Timeouts encode role (bits 8-11) and barrier (bits 0-7); a failed
// check of the bounds-checked debug build (GG_DEBUG) encodes the check's site in bits 0-7.
enum : uint32_t {
    kStatusTimeout = 0x1000u,
    kStatusBounds = 0x2000u,
    kRoleProducer = 1u << 8,
    kRoleMma = 2u << 8,
    kRoleEpilogue = 3u << 8,
};

// Operation computed by one instance of the kernel.
enum : int { kOpForward = 0, kOpDgrad = 1, kOpWgrad = 2 };

struct KernelParams {
    const int32_t *tile_off;  // [G+1] first tile of each group (cluster tiles)
    const int32_t *row_off;   // [G+1] first row (token) of each group in x / dy / out / dx
    const int32_t *tile_list; // null: tiles in group order (tile_off, raster bands); else [total_tiles]
                              // pairs (group, mt << 16 | nt): a tile order planned on the host
    const int32_t *row_cnt;   // null: group g has row_off[g+1] - row_off[g] rows; else [G] the rows this
                              // launch covers from row_off[g] (a split launch: the pair kernel takes each
                              // group's whole 256-row tiles, a one-CTA launch the remainders)
    void *out;
    uint32_t *status;
    const CUtensorMap *gmaps;  // wgrad: [2G] per-group maps (A = dy rows of g, B = x rows of g)
    int32_t group_num;
    int32_t n;            // output columns: N (forward), K (dgrad, wgrad)
    int32_t k;            // reduction extent: K (forward), N (dgrad); unused by wgrad
    int32_t tile_rows;    // wgrad: output rows per group (N)
    int32_t num_kb;       // ceil(reduction / 64): K atoms (forward, dgrad)
    int32_t tiles_n;      // ceil(N / bn)
    int32_t bn;           // tile N of this launch: a multiple of 32, <= the variant's kBN
    int32_t total_tiles;  // tile_off[G]
    int32_t splits;       // K splits of each split tile (0 or 1 = none); with stream-K the most
                          // pieces any stream-K tile has (the workspace stride)
    int32_t split_tiles;  // splits > 1: tiles [0, split_tiles) are split in `splits`, the rest run whole
    int32_t sk_tiles;     // > 0: stream-K. The K atoms of tiles [0, sk_tiles) are dealt out in equal
                          // contiguous ranges to all clusters; the remaining tiles run whole
    float *ws;            // split / stream-K: fp32 partial sums, per split tile
                          // [kCG][4 warps][splits][ceil(bn/32)] 4-KB blocks
    int32_t *counters;    // split / stream-K: [split tiles][kCG][4] arrival counts, 0 between launches
    int32_t band;         // tiles per raster band (L2 reuse, see decode_tile)
    int32_t raster;       // 0: bands of `band` m-tiles, n-tiles swept; 1: bands of `band` n-tiles
    int32_t store_min_atoms;  // a tile with at least this many K atoms stores out straight from
                              // registers; shorter tiles go through staging + TMA stores
    int32_t test_stall;   // test only: 1 = the first stage of cluster 0 is never loaded, so the
                          // MMA wait on it runs out and the status word reports it
    int32_t half_tiles;   // 1: a group's last m-tile with at most 128 rows runs half height (pair
                          // variant, forward / dgrad, whole tiles; needs bn % 32 == 0)
    int32_t mn_chunks;    // wgrad: bit 0 = the A maps (dy) and bit 1 = the B maps (x) are 3-D views
                          // (64 columns, rows, 64-column chunks) whose one box covers all the 64-column
                          // chunks a CTA loads per atom (else one 2-D box per chunk)
    int32_t *tile_ctr;    // non-null: dynamic tile dispatch (whole tiles only: splits <= 1, no
                          // stream-K). Cluster c takes tile c first, then tile C + atomicAdd(tile_ctr, 1)
                          // until past the last tile; 0 between launches (the last fetch resets it)
    int32_t l2_a;         // forward: L2 eviction priority of the A loads (activations):
    int32_t l2_b;         // and of the B loads (weights): 0 no hint, 1 evict_first, 2 evict_last
    int32_t out_rows;     // rows of the output tensor (sum(M), or G * N for wgrad): debug checks
    int64_t ws_float4s;   // float4 entries of the split-K / stream-K workspace: debug checks
    int32_t ctr_entries;  // entries of the arrival-counter array: debug checks
    uint64_t timeout_ns;
};

// Bounds-checked debug build (-DGG_DEBUG, lib/libgg_b200_debug.so): GG_CHECK(cond, site) records
// kStatusBounds | site in the status word (the first failure wins) and yields false, so the guarded
// access is skipped; gg_device_status reports it. Nothing traps. In the release build it is true.
#ifdef GG_DEBUG
#define GG_CHECK(cond, site) ((cond) ? true : (atomicCAS(p.status, 0u, ::gg::kStatusBounds | uint32_t(site)), false))
#else
#define GG_CHECK(cond, site) true
#endif

template <typename T> struct Fmt;
template <> struct Fmt<__nv_bfloat16> {
    static constexpr uint32_t kUmma = 1;
};
template <> struct Fmt<__half> {
    static constexpr uint32_t kUmma = 0;
};

// A stage holds kAtoms K-atoms (64 elements each) of the A and B tiles, so one barrier wait and
// one commit of the MMA thread cover kAtoms x 4 tcgen05.mma instructions.
template <int kCG, int kBN, int kAtoms> struct TileCfg {
    static_assert(kCG == 1 || kCG == 2, "CTA group of 1 or 2");
    static_assert(kBN % 16 == 0 && kBN >= 32 && kBN <= 256, "UMMA N");
    static_assert(kAtoms >= 1 && kAtoms <= 4, "atoms per stage");
    static constexpr int kClusterM = kBM * kCG;  // rows per (cluster) tile
    static constexpr int kBRows = kBN / kCG;     // weight rows each CTA loads
    static constexpr int kAAtomBytes = kBM * kBK * 2;
    static constexpr int kBAtomBytes = kBRows * kBK * 2;
    static constexpr int kABytes = kAtoms * kAAtomBytes;
    static constexpr int kBBytes = kAtoms * kBAtomBytes;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kMaxStages = 8;
    static constexpr int kStages = (kSmemBudget / kStageBytes) > kMaxStages ? kMaxStages : (kSmemBudget / kStageBytes);
    static constexpr int kRingBytes = kStages * kStageBytes;  // sized for the widest tile (kBN)
    // A launch with a narrower tile (bn < kBN) packs its stages tighter: each stage holds the A
    // atoms and bn/kCG B rows per atom, so more of them fit in the same ring. Stage starts stay
    // 1024-byte aligned (b_rows is a multiple of 8).
    __host__ __device__ static constexpr int stage_bytes(int b_rows) { return kAtoms * (kAAtomBytes + b_rows * kBK * 2); }
    __host__ __device__ static constexpr int stages_for(int b_rows) {
        return kRingBytes / stage_bytes(b_rows) > kMaxStages ? kMaxStages : kRingBytes / stage_bytes(b_rows);
    }
    static constexpr int kTmemCols = (2 * kBN) <= 32 ? 32 : (2 * kBN) <= 64 ? 64 : (2 * kBN) <= 128 ? 128
                                     : (2 * kBN) <= 256 ? 256 : 512;
    // Epilogue staging for TMA stores: per epilogue warp two 32-row x 64-column boxes (4 KB each,
    // 128-byte swizzle), after the ring.
    static constexpr int kStageOutBytes = 32 * 64 * 2;
    static constexpr int kOutOffset = kRingBytes;
    static constexpr int kOutBytes = GG_TMA_STORE ? 4 * 2 * kStageOutBytes : 0;
    // barriers: full[S], empty[S], tmem_full[2], tmem_empty[2], sched_full[R], sched_empty[R]; then
    // 16 bytes (TMEM base, abort flag, spare) and the R tile slots of the dynamic schedule
    static constexpr int kSched = 4;  // tile slots between the dispatching producer and the other roles
    static constexpr int kBarOffset = kOutOffset + kOutBytes;
    static constexpr int kNumBars = 2 * kMaxStages + 4 + 2 * kSched;
    static constexpr int kSlotOffset = kBarOffset + kNumBars * 8;
    static constexpr int kSmemBytes = kSlotOffset + 16 + kSched * 4 + 1024;  // + align slack
    static_assert(kSmemBytes <= 232448, "over the 227 KB shared-memory limit");
    static_assert(kStages >= 2, "ring too shallow");
    static_assert(kAAtomBytes % 1024 == 0 && kBAtomBytes % 1024 == 0, "swizzle atoms 1024-byte aligned");
};

struct TileCoord {
    int g, mt, nt;
    int rows;          // output rows of the group (tokens for forward/dgrad, N for wgrad)
    int out_row0;      // first output row of the group
    int red_atoms;     // 64-wide reduction atoms of the group
    bool half;         // a half-height pair tile (see is_half_tile)
};

// Half-height pair tiles (KernelParams::half_tiles): when the last m-tile of a group holds at most
// 128 of the 256 rows a CTA pair covers, it runs as a 128-row tile (64 rows per CTA) with an
// M = 128 cta_group::2 MMA, which the tensor cores execute at the same rate per row as M = 256, so
// a small expert's remainder costs half a tile instead of a padded whole one. Forward and dgrad
// (tiles over tokens); wgrad tiles run over the weight rows and never use them.
template <int kClusterM, int kOp>
__host__ __device__ __forceinline__ bool is_half_tile(int half_tiles, int rows, int mt) {
    if (kClusterM != 256 || kOp == 2 || !half_tiles)
        return false;
    const int rem = rows & 255;
    return rem != 0 && rem <= 128 && mt == (rows - 1) / 256;
}

// Map a linear tile index to (group, m-tile, n-tile). Within a group, tiles are rastered in
// bands (the role CK's GemmSpatiallyLocalTilePartitioner<8,4> plays in the reference,
// ck_kernel/ck_grouped_gemm_config.hpp:74-77):
//   raster 0: bands of `band` m-tiles; all n-tiles of a band are visited m-fastest, so
//             concurrently running tiles share a weight panel and the band's activation rows
//             stay in L2 (each weight panel is read from DRAM once per band);
//   raster 1: bands of `band` n-tiles; all m-tiles of a band are visited n-fastest, so the band's
//             weight panels stay in L2 and each activation row block is read from DRAM once per
//             band (with one band covering every n-tile: each operand once).
// Read-only load of the group tables: through the read-only data cache on the device, a plain load
// on the host (where the CPU schedule test walks decode_tile over host arrays).
__host__ __device__ __forceinline__ int32_t ld_table(const int32_t *q) {
#ifdef __CUDA_ARCH__
    return __ldg(q);
#else
    return *q;
#endif
}

// The group a role last decoded, with its table entries. A cluster's tile indices only grow
// (static schedule, split units and dynamic dispatch alike), and consecutive tiles mostly belong to
// one group, so decode_tile reads the tables only when a tile lies past the cached group: the
// dependent global loads would otherwise stall each role for several hundred cycles per tile.
struct GroupCursor {
    int g = 0;         // group of the cached entries (the search starts here)
    int t_begin = 0;   // tile_off[g]
    int t_end = -1;    // tile_off[g + 1]; -1 = nothing cached
    int r0 = 0;        // row_off[g]
    int m = 0;         // rows of group g
};

template <int kClusterM, int kOp>
__host__ __device__ __forceinline__ TileCoord decode_tile(const KernelParams &p, int t, GroupCursor &gc) {
    TileCoord tc;
    if (p.tile_list) {
        // a planned order: the tile's coordinates come from the list (the cursor is not used)
        tc.g = ld_table(&p.tile_list[2 * int64_t(t)]);
        const int mn = ld_table(&p.tile_list[2 * int64_t(t) + 1]);
        tc.mt = mn >> 16;
        tc.nt = mn & 0xffff;
        const int r0 = ld_table(&p.row_off[tc.g]);
        const int m = p.row_cnt ? ld_table(&p.row_cnt[tc.g]) : ld_table(&p.row_off[tc.g + 1]) - r0;
        if constexpr (kOp == kOpWgrad) {
            tc.rows = p.tile_rows;
            tc.out_row0 = tc.g * p.tile_rows;
            tc.red_atoms = (m + kBK - 1) / kBK;
        } else {
            tc.rows = m;
            tc.out_row0 = r0;
            tc.red_atoms = p.num_kb;
        }
        tc.half = is_half_tile<kClusterM, kOp>(p.half_tiles, tc.rows, tc.mt);
        return tc;
    }
    if (t >= gc.t_end || t < gc.t_begin) {
        int g = t < gc.t_begin ? 0 : gc.g;
        while (ld_table(&p.tile_off[g + 1]) <= t)
            ++g;
        gc.g = g;
        gc.t_begin = ld_table(&p.tile_off[g]);
        gc.t_end = ld_table(&p.tile_off[g + 1]);
        gc.r0 = ld_table(&p.row_off[g]);
        gc.m = p.row_cnt ? ld_table(&p.row_cnt[g]) : ld_table(&p.row_off[g + 1]) - gc.r0;
    }
    tc.g = gc.g;
    const int local = t - gc.t_begin;
    const int r0 = gc.r0;
    const int m = gc.m;
    if constexpr (kOp == kOpWgrad) {
        tc.rows = p.tile_rows;
        tc.out_row0 = tc.g * p.tile_rows;
        tc.red_atoms = (m + kBK - 1) / kBK;
    } else {
        tc.rows = m;
        tc.out_row0 = r0;
        tc.red_atoms = p.num_kb;
    }
    const int tiles_m = (tc.rows + kClusterM - 1) / kClusterM;
    if (p.raster == 0) {
        const int band_tiles = p.band * p.tiles_n;
        const int b = local / band_tiles;
        const int r = local - b * band_tiles;
        const int rows = min(p.band, tiles_m - b * p.band);
        tc.nt = r / rows;
        tc.mt = b * p.band + (r - tc.nt * rows);
    } else {
        const int band_tiles = p.band * tiles_m;
        const int b = local / band_tiles;
        const int r = local - b * band_tiles;
        const int cols = min(p.band, p.tiles_n - b * p.band);
        tc.mt = r / cols;
        tc.nt = b * p.band + (r - tc.mt * cols);
    }
    tc.half = is_half_tile<kClusterM, kOp>(p.half_tiles, tc.rows, tc.mt);
    return tc;
}

// The same with a bare group cursor (host callers: the tile-order planner and the CPU tests).
template <int kClusterM, int kOp>
__host__ __device__ __forceinline__ TileCoord decode_tile(const KernelParams &p, int t, int &cursor) {
    GroupCursor gc;
    gc.g = cursor;
    gc.t_begin = 0;  // nothing cached; the search starts at the cursor (t only grows)
    const TileCoord tc = decode_tile<kClusterM, kOp>(p, t, gc);
    cursor = gc.g;
    return tc;
}

// A work unit: K atoms [atom0, atom1) of tile t, piece `piece` of the `npieces` pieces the tile
// is cut into (npieces > 1: every piece publishes an fp32 partial and the last to arrive sums them
// in piece order). Each cluster (CTA or CTA pair) walks its own list of units, in order:
//   split-K (splits > 1, sk_tiles == 0): units [0, split_tiles x splits) are the equal K splits of
//     tiles [0, split_tiles), then one unit per remaining tile; unit u goes to cluster
//     u % clusters. split_tiles = total_tiles is plain split-K; fewer split tiles is split-K for
//     what would otherwise be a partial last wave.
//   stream-K (sk_tiles > 0): the sk_tiles x num_kb atoms of tiles [0, sk_tiles), in tile-major
//     order, are cut into one contiguous range per cluster (cluster c: [c S / C, (c+1) S / C),
//     S atoms, C clusters), split at tile boundaries into pieces; then whole tiles
//     sk_tiles + c, sk_tiles + c + C, ... Every cluster gets the same number of atoms (+-1),
//     whatever the number of tiles.
// Either way the pieces of a tile come first in each cluster's list, so the fix-up runs in the
// epilogue warps while the MMA warp works on what follows. (Host-callable as well, so that a CPU
// test can walk the exact schedule: tests/test_schedule.py.)
struct Unit {
    int t, atom0, atom1, piece, npieces;
};

// Stream-K: the cluster whose range holds atom g (S = atoms in the stream-K region; S >= C).
__host__ __device__ __forceinline__ int sk_cluster_of(int64_t g, int64_t S, int C) { return int(((g + 1) * C - 1) / S); }

struct UnitList {
    int n;              // units of this cluster
    int n_sk;           // stream-K pieces among them (listed first)
    int64_t sk0, sk1;   // stream-K: this cluster's atom range
};

__host__ __device__ __forceinline__ UnitList units_of(const KernelParams &p, int c, int C) {
    UnitList l{0, 0, 0, 0};
    if (p.sk_tiles > 0) {
        const int64_t A = p.num_kb, S = int64_t(p.sk_tiles) * A;
        l.sk0 = S * c / C;
        l.sk1 = S * (c + 1) / C;
        l.n_sk = l.sk1 > l.sk0 ? int((l.sk1 - 1) / A - l.sk0 / A + 1) : 0;
        const int rest = p.total_tiles - p.sk_tiles - c;
        l.n = l.n_sk + (rest > 0 ? (rest + C - 1) / C : 0);
    } else {
        const int s = p.splits > 1 ? p.splits : 1;
        const int total = p.total_tiles + (s > 1 ? p.split_tiles * (s - 1) : 0);
        l.n = c < total ? (total - c + C - 1) / C : 0;
    }
    return l;
}

__host__ __device__ __forceinline__ Unit unit_at(const KernelParams &p, const UnitList &l, int c, int C, int i) {
    const int A = p.num_kb;
    if (p.sk_tiles > 0) {
        if (i < l.n_sk) {
            const int64_t S = int64_t(p.sk_tiles) * A;
            const int t = int(l.sk0 / A) + i;
            const int64_t t0 = int64_t(t) * A;
            const int first = sk_cluster_of(t0, S, C);
            const int last = sk_cluster_of(t0 + A - 1, S, C);
            return {t, int((l.sk0 > t0 ? l.sk0 : t0) - t0), int((l.sk1 < t0 + A ? l.sk1 : t0 + A) - t0), c - first,
                    last - first + 1};
        }
        return {p.sk_tiles + c + (i - l.n_sk) * C, 0, A, 0, 1};
    }
    const int u = c + i * C;
    const int s = p.splits > 1 ? p.splits : 1;
    if (s > 1 && u < p.split_tiles * s) {
        // split j of s covers atoms [j A / s, (j + 1) A / s): balanced, never empty while s <= A
        const int q = u / s;
        const int j = u - q * s;
        return {q, j * A / s, (j + 1) * A / s, j, s};
    }
    return {s > 1 ? u - p.split_tiles * (s - 1) : u, 0, A, 0, 1};
}

// Dynamic tile dispatch (KernelParams::tile_ctr): cluster c runs tile c first; after each tile it
// fetches a counter value v (atomicAdd) and runs tile C + v next, until that is past the last tile.
// Each cluster makes exactly one fetch past the end, so a launch makes total_tiles fetches and the
// one that returns total_tiles - 1 is the last: it resets the counter to 0 for the next launch.
// (Host-callable, so that a CPU test can play out any order of fetches.)
__host__ __device__ __forceinline__ int dispatched_tile(int fetched, int clusters, int total_tiles) {
    const int t = clusters + fetched;
    return t < total_tiles ? t : -1;
}
__host__ __device__ __forceinline__ bool is_last_fetch(int fetched, int total_tiles) {
    return fetched == total_tiles - 1;
}

struct Abort {
    uint32_t *status;         // global
    volatile uint32_t *flag;  // this CTA's shared abort flag
    uint64_t timeout_ns;
};

// Slow path of a bounded wait: spin on try_wait, and every 256 tries check the abort flags
// and the time limit. Returns false if this or another role gave up.
template <bool kClusterScope>
__device__ __noinline__ bool wait_slow(uint32_t bar, uint32_t parity, const Abort ab, uint32_t code) {
    const uint64_t t0 = ptx::globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (kClusterScope ? ptx::mbar_try_wait_cluster(bar, parity) : ptx::mbar_try_wait(bar, parity))
            return true;
        if ((it & 255u) == 0) {
            if (*ab.flag != 0u || *(volatile uint32_t *)ab.status != 0u) {
                *ab.flag = 1u;
                return false;
            }
            if (ptx::globaltimer() - t0 > ab.timeout_ns) {
                atomicCAS(ab.status, 0u, code);
                *ab.flag = 1u;
                return false;
            }
        }
    }
}

// Bounded wait in the calling thread: an inline first test, the loop out of line.
template <bool kClusterScope = false>
__device__ __forceinline__ bool wait_one(uint32_t bar, uint32_t parity, const Abort &ab, uint32_t code) {
    if (kClusterScope ? ptx::mbar_try_wait_cluster(bar, parity) : ptx::mbar_try_wait(bar, parity))
        return true;
    return wait_slow<kClusterScope>(bar, parity, ab, code);
}

// Bounded wait by one thread until a global counter, written by other CTAs, reaches `want`.
// Returns false if this or another role gave up.
__device__ __noinline__ bool wait_count(const int32_t *ctr, int want, const Abort ab, uint32_t code) {
    const uint64_t t0 = ptx::globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (*reinterpret_cast<const volatile int32_t *>(ctr) >= want)
            return true;
        __nanosleep(32);
        if ((it & 63u) == 0) {
            if (*ab.flag != 0u || *(volatile uint32_t *)ab.status != 0u) {
                *ab.flag = 1u;
                return false;
            }
            if (ptx::globaltimer() - t0 > ab.timeout_ns) {
                atomicCAS(ab.status, 0u, code);
                *ab.flag = 1u;
                return false;
            }
        }
    }
}

// Bounded wait by a whole converged warp (the producer and MMA roles): every lane tests the
// barrier and the warp agrees on the outcome (a wait that ran out in any lane ends the role in all).
template <bool kClusterScope = false>
__device__ __forceinline__ bool wait_all(uint32_t bar, uint32_t parity, const Abort &ab, uint32_t code) {
    const bool ok = wait_one<kClusterScope>(bar, parity, ab, code);
    return __all_sync(0xffffffffu, ok ? 1 : 0) != 0;
}

// Warp-uniform bounded wait: lane 0 waits, the result is broadcast.
__device__ __forceinline__ bool wait_warp(uint32_t bar, uint32_t parity, const Abort &ab, uint32_t code) {
    int ok = 1;
    if ((threadIdx.x & 31u) == 0)
        ok = wait_one(bar, parity, ab, code) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(uint32_t a, uint32_t b) {
    if constexpr (sizeof(T) == 2 && Fmt<T>::kUmma == 1) {
        __nv_bfloat162 v = __floats2bfloat162_rn(__uint_as_float(a), __uint_as_float(b));
        return *reinterpret_cast<uint32_t *>(&v);
    } else {
        __half2 v = __floats2half2_rn(__uint_as_float(a), __uint_as_float(b));
        return *reinterpret_cast<uint32_t *>(&v);
    }
}

// Issue one 2-D / 3-D TMA load into this CTA's shared memory, completing on `bar` (in a CTA pair
// the leader's barrier, through the .cta_group::2 form); only in the lane where `pred` != 0.
template <int kCG>
__device__ __forceinline__ void load_2d(uint32_t dst, const void *map, uint32_t bar, int c0, int c1, uint32_t pred) {
    if constexpr (kCG == 1)
        ptx::tma_load_2d(dst, map, bar, c0, c1, pred);
    else
        ptx::tma_load_2d_pair(dst, map, bar, c0, c1, pred);
}
template <int kCG>
__device__ __forceinline__ void load_3d(uint32_t dst, const void *map, uint32_t bar, int c0, int c1, int c2,
                                        uint32_t pred) {
    if constexpr (kCG == 1)
        ptx::tma_load_3d(dst, map, bar, c0, c1, c2, pred);
    else
        ptx::tma_load_3d_pair(dst, map, bar, c0, c1, c2, pred);
}
// The same with an L2 eviction-priority policy when `hinted` (KernelParams::l2_a / l2_b), without
// one otherwise (a uniform branch: every lane of the warp takes the same side).
template <int kCG>
__device__ __forceinline__ void load_2d(uint32_t dst, const void *map, uint32_t bar, int c0, int c1, bool hinted,
                                        uint64_t policy, uint32_t pred) {
    if (!hinted)
        load_2d<kCG>(dst, map, bar, c0, c1, pred);
    else if constexpr (kCG == 1)
        ptx::tma_load_2d_hint(dst, map, bar, c0, c1, policy, pred);
    else
        ptx::tma_load_2d_pair_hint(dst, map, bar, c0, c1, policy, pred);
}
template <int kCG>
__device__ __forceinline__ void load_3d(uint32_t dst, const void *map, uint32_t bar, int c0, int c1, int c2,
                                        bool hinted, uint64_t policy, uint32_t pred) {
    if (!hinted)
        load_3d<kCG>(dst, map, bar, c0, c1, c2, pred);
    else if constexpr (kCG == 1)
        ptx::tma_load_3d_hint(dst, map, bar, c0, c1, c2, policy, pred);
    else
        ptx::tma_load_3d_pair_hint(dst, map, bar, c0, c1, c2, policy, pred);
}

// L2 policy of an operand's loads: 1 evict_first, 2 evict_last (KernelParams::l2_a / l2_b).
__device__ __forceinline__ uint64_t l2_load_policy(int hint) {
    return hint == 2 ? ptx::l2_policy_evict_last() : ptx::l2_policy_evict_first();
}

constexpr int kMnBoxBytes = 64 * kBK * 2;  // one MN-major box: 64 MN x 64 K elements

template <typename T, int kCG, int kBN, int kAtoms, int kOp>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_sm100(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                       const __grid_constant__ CUtensorMap tmap_out,
                       const __grid_constant__ CUtensorMap tmap_a_half,  // A in 64-row boxes (half tiles)
                       const __grid_constant__ KernelParams p) {
    using C = TileCfg<kCG, kBN, kAtoms>;
    // A is MN-major for wgrad (dy^T), B is MN-major for both backward operations.
    constexpr bool kAMn = kOp == kOpWgrad;
    constexpr bool kBMn = kOp != kOpForward;
    // Tile N is a launch parameter (multiple of 32, at most kBN; for an MN-major B also a multiple
    // of 64 per CTA): the smem ring and TMEM are sized for kBN, a narrower tile uses the first
    // bn/kCG B rows (columns) of each atom and bn columns of each accumulator.
    const int bn = p.bn;
    const int b_rows = bn / kCG;
    const uint32_t idesc = ptx::f16_idesc(Fmt<T>::kUmma, kBM * kCG, bn, kAMn ? 1u : 0u, kBMn ? 1u : 0u);
    const uint32_t idesc_half = ptx::f16_idesc(Fmt<T>::kUmma, 128, bn, 0u, kBMn ? 1u : 0u);  // M = 128 pair tile

    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the 128-byte swizzle atoms.
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t smem_base = ptx::smem_addr(smem);
    const uint32_t bar_base = smem_base + C::kBarOffset;
    // Ring geometry of this launch's tile width: stage count and bytes per stage and per B atom.
    const int num_stages = C::stages_for(b_rows);
    const uint32_t stage_bytes = uint32_t(C::stage_bytes(b_rows));
    const uint32_t b_atom_bytes = uint32_t(b_rows * kBK * 2);
    auto full_bar = [&](int s) { return bar_base + 8u * s; };
    auto empty_bar = [&](int s) { return bar_base + 8u * (C::kMaxStages + s); };
    auto tfull_bar = [&](int a) { return bar_base + 8u * (2 * C::kMaxStages + a); };
    auto tempty_bar = [&](int a) { return bar_base + 8u * (2 * C::kMaxStages + 2 + a); };
    // dynamic tile dispatch: slot r holds the tile of units r, r + R, ... of this cluster
    auto sfull_bar = [&](int r) { return bar_base + 8u * (2 * C::kMaxStages + 4 + r); };
    auto sempty_bar = [&](int r) { return bar_base + 8u * (2 * C::kMaxStages + 4 + C::kSched + r); };
    uint32_t *tmem_ptr_slot = reinterpret_cast<uint32_t *>(smem + C::kSlotOffset);
    volatile uint32_t *abort_flag = tmem_ptr_slot + 1;
    const uint32_t sched_slots = smem_base + C::kSlotOffset + 16;
    const volatile int32_t *sched_slot = reinterpret_cast<const volatile int32_t *>(smem + C::kSlotOffset + 16);
    const bool dyn = p.tile_ctr != nullptr;

    const int warp = threadIdx.x / 32;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t cta_rank = kCG == 2 ? ptx::cluster_ctarank() : 0u;
    const bool leader = cta_rank == 0;
    const int cluster_id = blockIdx.x / kCG;
    const int num_clusters = gridDim.x / kCG;

    if (threadIdx.x == 0) {
        for (int s = 0; s < num_stages; ++s) {
            ptx::mbar_init(full_bar(s), 1);   // leader producer's arrive.expect_tx
            ptx::mbar_init(empty_bar(s), 1);  // one tcgen05.commit per use
        }
        for (int a = 0; a < 2; ++a) {
            ptx::mbar_init(tfull_bar(a), 1);         // one tcgen05.commit per tile
            ptx::mbar_init(tempty_bar(a), 4 * kCG);  // one arrive per epilogue warp of the pair
        }
        for (int r = 0; r < C::kSched; ++r) {
            ptx::mbar_init(sfull_bar(r), 1);  // the pair leader's producer publishes the tile
            // read by: the leader's MMA warp, every epilogue warp of the pair, the peer's producer
            ptx::mbar_init(sempty_bar(r), 1 + 4 * kCG + (kCG - 1));
        }
        *abort_flag = 0u;
        ptx::fence_mbar_init();
        ptx::fence_proxy_async_smem();
    }
    if (warp == 0 && lane == 0) {
        if constexpr (kOp != kOpWgrad) {  // wgrad loads through the per-group maps instead
            ptx::prefetch_tmap(&tmap_a);
            ptx::prefetch_tmap(&tmap_b);
        }
        if (GG_TMA_STORE)
            ptx::prefetch_tmap(&tmap_out);
        if (p.half_tiles)
            ptx::prefetch_tmap(&tmap_a_half);
    }
    if (warp == 1) {
        ptx::tmem_alloc<kCG>(ptx::smem_addr(tmem_ptr_slot), C::kTmemCols);
        ptx::tmem_relinquish<kCG>();
    }
    ptx::tc_fence_before();
    __syncthreads();
    if constexpr (kCG == 2)
        ptx::cluster_sync();  // peer barriers are initialised before any remote arrive
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_ptr_slot;
    // Everything above is on-chip set-up; with programmatic dependent launch it overlaps the
    // previous kernel's tail. The group-offset table is written by the host before the stream
    // reaches this launch (prepare synchronises its stream), or by gg_run_noalloc's publish kernel,
    // which precedes a launch made without programmatic serialisation; never by a kernel this
    // launch may overlap. So the first tile's look-up may run before the dependency wait. Every
    // other global access comes after the wait.
    const UnitList units = units_of(p, cluster_id, num_clusters);
    // The producer decodes its first unit's tile here, so that its first TMA loads can be issued
    // right after the dependency wait (decoding after it would wait on dependent global loads).
    // (Unit 0 is tile cluster_id with dynamic dispatch too: that needs whole tiles.)
    TileCoord first_tc{};
    GroupCursor first_cursor;
    if (warp <= 1 && units.n > 0)  // the producer, and the MMA warp (tile height, wgrad reduction)
        first_tc = decode_tile<C::kClusterM, kOp>(p, unit_at(p, units, cluster_id, num_clusters, 0).t, first_cursor);
    ptx::griddep_wait();
    // TMA loads and stores go through the async proxy; a proxy fence orders them after the
    // generic-proxy writes of the previous kernel that the wait made visible (a conservative
    // ordering, one fence per thread per launch).
    ptx::fence_proxy_async_global();
    ptx::griddep_launch_dependents();

    const Abort ab{p.status, abort_flag, p.timeout_ns};
    // Work units (unit_at): each covers a contiguous range of K atoms of one tile and runs the same
    // producer/MMA/epilogue pipeline over it. (wgrad runs whole tiles: its reduction length differs
    // per group.)

    if (warp == 0) {
        // ---------------- TMA producer (warp 0) ----------------
        // The warp runs the loop converged; one elected lane issues the barrier arrive and the TMA
        // loads (predicated instructions, no divergent branch around them).
        {
            const uint32_t issue = ptx::elect_one_sync();
            const uint32_t full_leader0 = kCG == 2 ? ptx::mapa(full_bar(0), 0) : full_bar(0);
            GroupCursor cursor;
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            int fenced_g = -1;  // wgrad: group whose tensor maps the warp has acquired
            const int issue_lane = __ffs(__ballot_sync(0xffffffffu, issue)) - 1;
            const uint64_t pol_a = l2_load_policy(p.l2_a), pol_b = l2_load_policy(p.l2_b);
            int fetched = 0;  // dynamic dispatch, issuing lane of the leader: the next unit's fetch
            for (int i = 0; ok; ++i) {
                Unit un;
                if (dyn) {
                    // The pair leader's producer dispatches: unit 0 is tile cluster_id, each later
                    // unit the tile its fetch (issued one unit ahead) returned; past the last tile it
                    // publishes -1 and every role stops. The fetch that returns the launch's last
                    // counter value resets the counter for the next launch.
                    const int r = i % C::kSched;
                    const uint32_t par = uint32_t(i / C::kSched) & 1u;
                    int t = 0;
                    if (leader) {
                        if (issue) {
                            t = i == 0 ? (cluster_id < p.total_tiles ? cluster_id : -1)
                                       : dispatched_tile(fetched, num_clusters, p.total_tiles);
                            if (i > 0 && is_last_fetch(fetched, p.total_tiles))
                                atomicExch(p.tile_ctr, 0);
                        }
                        t = __shfl_sync(0xffffffffu, t, issue_lane);
                        if (!wait_all(sempty_bar(r), par ^ 1u, ab, kStatusTimeout | kRoleProducer | 0x50u | uint32_t(r))) {
                            ok = false;
                            break;
                        }
                        if (issue) {
                            ptx::st_shared_u32(sched_slots + 4u * r, uint32_t(t));
                            ptx::mbar_arrive(sfull_bar(r));
                            if constexpr (kCG == 2) {
                                ptx::st_cluster_u32(ptx::mapa(sched_slots + 4u * r, 1), uint32_t(t));
                                ptx::mbar_arrive_cluster(ptx::mapa(sfull_bar(r), 1));
                            }
                            if (t >= 0)
                                fetched = atomicAdd(p.tile_ctr, 1);
                        }
                        __syncwarp();
                    } else {
                        if (!wait_all<true>(sfull_bar(r), par, ab, kStatusTimeout | kRoleProducer | 0x60u | uint32_t(r))) {
                            ok = false;
                            break;
                        }
                        t = sched_slot[r];
                        if (issue)
                            ptx::mbar_arrive_cluster(ptx::mapa(sempty_bar(r), 0));
                        __syncwarp();
                    }
                    if (t < 0)
                        break;
                    un = Unit{t, 0, p.num_kb, 0, 1};
                } else {
                    if (i >= units.n)
                        break;
                    un = unit_at(p, units, cluster_id, num_clusters, i);
                }
                TileCoord tc;
                if (i == 0) {  // decoded before the dependency wait
                    tc = first_tc;
                    cursor = first_cursor;
                } else {
                    tc = decode_tile<C::kClusterM, kOp>(p, un.t, cursor);
                }
                GG_CHECK(tc.g >= 0 && tc.g < p.group_num && tc.mt >= 0 && tc.nt >= 0 && tc.nt < p.tiles_n &&
                             tc.mt * C::kClusterM < max(tc.rows, 1), 1);
                const int atom0 = kOp == kOpWgrad ? 0 : un.atom0;
                const int atom1 = kOp == kOpWgrad ? tc.red_atoms : un.atom1;
                const int num_ks = (atom1 - atom0 + kAtoms - 1) / kAtoms;
                // A: first row (forward/dgrad: token row; wgrad: row of dw[g], a column of dy); a
                // half tile gives each CTA 64 rows, loaded through the 64-row map
                const bool half = tc.half;
                const int a_row = (kOp == kOpWgrad ? 0 : tc.out_row0) + tc.mt * C::kClusterM + int(cta_rank) * (half ? 64 : kBM);
                const uint32_t a_atom_load = half ? uint32_t(C::kAAtomBytes / 2) : uint32_t(C::kAAtomBytes);
                // B: first weight row (forward) / first output column (backward) of this CTA
                const int b_row = tc.nt * bn + int(cta_rank) * b_rows;
                const void *map_a = &tmap_a;
                const void *map_b = &tmap_b;
                if constexpr (kOp == kOpWgrad) {
                    map_a = p.gmaps + 2 * tc.g;
                    map_b = p.gmaps + 2 * tc.g + 1;
                    if (tc.g != fenced_g && num_ks > 0) {
                        ptx::fence_tensormap_acquire(map_a);
                        ptx::fence_tensormap_acquire(map_b);
                        fenced_g = tc.g;
                    }
                }
                for (int ks = 0; ks < num_ks; ++ks) {
                    if (!wait_all(empty_bar(s), ph ^ 1u, ab, kStatusTimeout | kRoleProducer | uint32_t(s))) {
                        ok = false;
                        break;
                    }
                    // K atoms of this stage that lie inside the unit's range (the rest would be zero fill)
                    const int na = min(kAtoms, atom1 - (atom0 + ks * kAtoms));
                    const uint32_t a_dst = smem_base + uint32_t(s) * stage_bytes;
                    const uint32_t b_dst = a_dst + C::kABytes;
                    const uint32_t fb = full_leader0 + 8u * s;
                    // test hook: the leader skips its arrive and loads of cluster 0's first stage
                    const bool skip = p.test_stall != 0 && cluster_id == 0 && leader && ks == 0 && i == 0;
                    ptx::mbar_arrive_expect_tx(full_bar(s), uint32_t(kCG * na) * (a_atom_load + b_atom_bytes),
                                               leader && !skip ? issue : 0u);
#pragma unroll
                    for (int a = 0; a < kAtoms; ++a) {
                        if (a < na && !skip) {
                            const int k0 = (atom0 + ks * kAtoms + a) * kBK;
                            const uint32_t ad = a_dst + a * C::kAAtomBytes;
                            const uint32_t bd = b_dst + a * b_atom_bytes;
                            if constexpr (kAMn) {
                                // wgrad A = dy^T: the CTA's two 64-column chunks of the group's dy
                                // rows, one box of the 3-D chunk view or two 2-D boxes
                                if (p.mn_chunks & 1) {
                                    load_3d<kCG>(ad, map_a, fb, 0, k0, a_row / 64, issue);
                                } else {
                                    load_2d<kCG>(ad, map_a, fb, a_row, k0, issue);
                                    load_2d<kCG>(ad + kMnBoxBytes, map_a, fb, a_row + 64, k0, issue);
                                }
                            } else {
                                // the L2 policy form only in the forward op: in the dgrad producer the
                                // hinted form cost more than any hint saved (dgrad L -10%)
                                if constexpr (kOp == kOpForward)
                                    load_2d<kCG>(ad, half ? static_cast<const void *>(&tmap_a_half) : map_a, fb, k0, a_row,
                                                 p.l2_a != 0, pol_a, issue);
                                else
                                    load_2d<kCG>(ad, half ? static_cast<const void *>(&tmap_a_half) : map_a, fb, k0, a_row, issue);
                            }
                            if constexpr (kOp == kOpForward) {
                                load_3d<kCG>(bd, map_b, fb, k0, b_row, tc.g, p.l2_b != 0, pol_b, issue);
                            } else if (kOp == kOpWgrad && (p.mn_chunks & 2)) {
                                // x rows (tokens) k0.. of the group, all b_rows / 64 chunks at once
                                load_3d<kCG>(bd, map_b, fb, 0, k0, b_row / 64, issue);
                            } else {
                                for (int j = 0; j < b_rows / 64; ++j) {
                                    if constexpr (kOp == kOpDgrad)  // w[g] rows k0.., columns b_row + 64j..
                                        load_3d<kCG>(bd + j * kMnBoxBytes, map_b, fb, b_row + 64 * j, k0, tc.g, issue);
                                    else  // x rows (tokens) k0.. of the group, columns b_row + 64j..
                                        load_2d<kCG>(bd + j * kMnBoxBytes, map_b, fb, b_row + 64 * j, k0, issue);
                                }
                            }
                        }
                    }
                    if (++s == num_stages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            // Tail: every stage released, so no tcgen05.commit is still in flight to this CTA.
            for (int i = 0; ok && i < num_stages; ++i) {
                ok = wait_all(empty_bar(s), ph ^ 1u, ab, kStatusTimeout | kRoleProducer | 0x80u);
                if (++s == num_stages) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (warp 1 of the pair leader) ----------------
        // The warp runs the loop converged; one elected lane issues the tcgen05.mma and
        // tcgen05.commit instructions (predicated), which keeps the issue at the tensor pipe's rate.
        if (leader) {
            const uint32_t issue = ptx::elect_one_sync();
            uint32_t tl = 0;
            int s = 0;
            uint32_t ph = 0;
            bool ok = true;
            GroupCursor cursor;
            for (int i = 0; ok; ++i, ++tl) {
                Unit un;
                if (dyn) {
                    const int r = i % C::kSched;
                    if (!wait_all<kCG == 2>(sfull_bar(r), uint32_t(i / C::kSched) & 1u, ab,
                                            kStatusTimeout | kRoleMma | 0x60u | uint32_t(r))) {
                        ok = false;
                        break;
                    }
                    const int t = sched_slot[r];
                    if (issue)
                        ptx::mbar_arrive(sempty_bar(r));
                    __syncwarp();
                    if (t < 0)
                        break;
                    un = Unit{t, 0, p.num_kb, 0, 1};
                } else {
                    if (i >= units.n)
                        break;
                    un = unit_at(p, units, cluster_id, num_clusters, i);
                }
                int atom0 = un.atom0, atom1 = un.atom1;
                bool half = false;
                if (kOp == kOpWgrad || p.half_tiles) {
                    TileCoord tcm;
                    if (i == 0) {  // decoded before the dependency wait
                        tcm = first_tc;
                        cursor = first_cursor;
                    } else {
                        tcm = decode_tile<C::kClusterM, kOp>(p, un.t, cursor);
                    }
                    if constexpr (kOp == kOpWgrad) {
                        atom0 = 0;
                        atom1 = tcm.red_atoms;  // 0 for an empty group
                    }
                    half = tcm.half;
                }
                const uint32_t idesc_t = half ? idesc_half : idesc;
                const int num_ks = (atom1 - atom0 + kAtoms - 1) / kAtoms;
                const int acc = int(tl & 1u);
                const uint32_t acc_ph = (tl >> 1) & 1u;
                // The epilogue warps (also the peer's) arrive after tcgen05.wait::ld, so their reads of
                // this accumulator are complete; a CTA-scope wait is enough before overwriting it.
                if (!wait_all(tempty_bar(acc), acc_ph ^ 1u, ab, kStatusTimeout | kRoleMma | 0x40u | uint32_t(acc))) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + uint32_t(acc * kBN);
                for (int ks = 0; ks < num_ks; ++ks) {
                    if (!wait_all(full_bar(s), ph, ab, kStatusTimeout | kRoleMma | uint32_t(s))) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const int na = min(kAtoms, atom1 - (atom0 + ks * kAtoms));
                    const uint32_t a_addr = smem_base + uint32_t(s) * stage_bytes;
                    const uint64_t adesc = kAMn ? ptx::sw128_mnmajor_desc(a_addr) : ptx::sw128_kmajor_desc(a_addr);
                    const uint64_t bdesc = kBMn ? ptx::sw128_mnmajor_desc(a_addr + C::kABytes)
                                                : ptx::sw128_kmajor_desc(a_addr + C::kABytes);
                    // 16 K elements: 32 bytes along a K-major row, or 16 rows of 128 bytes MN-major
                    constexpr int kStepA = kAMn ? 16 * 128 : 32;
                    constexpr int kStepB = kBMn ? 16 * 128 : 32;
#pragma unroll
                    for (int a = 0; a < kAtoms; ++a) {
                        if (a < na) {
#pragma unroll
                            for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
                                // atom a, then the kk-th 16-element K step inside the atom
                                const uint64_t da = uint64_t((a * C::kAAtomBytes + kk * kStepA) >> 4);
                                const uint64_t db = uint64_t((a * b_atom_bytes + kk * kStepB) >> 4);
                                ptx::umma_f16<kCG>(d_tmem, adesc + da, bdesc + db, idesc_t,
                                                   (ks | a | kk) != 0 ? 1u : 0u, issue);
                            }
                        }
                    }
                    ptx::umma_commit<kCG>(empty_bar(s), issue);
                    if constexpr (kCG == 2)
                        ptx::umma_commit<kCG>(ptx::mapa(empty_bar(s), 1), issue);
                    if (++s == num_stages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok)
                    break;
                ptx::umma_commit<kCG>(tfull_bar(acc), issue);
                if constexpr (kCG == 2)
                    ptx::umma_commit<kCG>(ptx::mapa(tfull_bar(acc), 1), issue);
            }
            // Tail: both accumulators released by every epilogue warp of the pair.
            for (uint32_t i = tl; ok && i < tl + 2; ++i)
                ok = wait_all(tempty_bar(int(i & 1u)), ((i >> 1) & 1u) ^ 1u, ab, kStatusTimeout | kRoleMma | 0x80u);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (4 warps) ----------------
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int row_in_cta = q * 32 + int(lane);
        const uint32_t tempty_leader0 = kCG == 2 ? ptx::mapa(tempty_bar(0), 0) : tempty_bar(0);
        T *out = static_cast<T *>(p.out);
        // this warp's two staging buffers
        const uint32_t out_stage = smem_base + C::kOutOffset + uint32_t(q) * 2u * C::kStageOutBytes;
        const uint64_t store_policy = ptx::l2_policy_evict_first();  // out is never re-read here
        int out_buf = 0;
        GroupCursor cursor;
        uint32_t tl = 0;
        for (int i = 0;; ++i, ++tl) {
            Unit un;
            if (dyn) {
                const int r = i % C::kSched;
                int t = -1;
                if (lane == 0) {
                    if (wait_one<kCG == 2>(sfull_bar(r), uint32_t(i / C::kSched) & 1u, ab,
                                           kStatusTimeout | kRoleEpilogue | 0x60u | uint32_t(r))) {
                        t = sched_slot[r];
                        if constexpr (kCG == 2)
                            ptx::mbar_arrive_cluster(ptx::mapa(sempty_bar(r), 0));
                        else
                            ptx::mbar_arrive(sempty_bar(r));
                    }
                }
                t = __shfl_sync(0xffffffffu, t, 0);
                if (t < 0)
                    break;
                un = Unit{t, 0, p.num_kb, 0, 1};
            } else {
                if (i >= units.n)
                    break;
                un = unit_at(p, units, cluster_id, num_clusters, i);
            }
            const int t = un.t;
            const int split = un.piece;
            const int nsplit = un.npieces;
            const TileCoord tc = decode_tile<C::kClusterM, kOp>(p, t, cursor);
            GG_CHECK(tc.g >= 0 && tc.g < p.group_num && tc.mt >= 0 && tc.nt >= 0 && tc.nt < p.tiles_n &&
                         t >= 0 && t < p.total_tiles, 1);
            const int acc = int(tl & 1u);
            const uint32_t acc_ph = (tl >> 1) & 1u;
            if (!wait_warp(tfull_bar(acc), acc_ph, ab, kStatusTimeout | kRoleEpilogue | uint32_t(acc)))
                break;
            ptx::tc_fence_after();
            const int g_row0 = tc.out_row0;
            const int m = tc.rows;
            // wgrad of an expert without tokens: no MMA ran, the tile is written as zeros
            const bool zero_tile = kOp == kOpWgrad && tc.red_atoms == 0;
            // A half tile's accumulator (M = 128 pair MMA): CTA r holds its 64 rows in TMEM lanes
            // 0-63 for output columns [0, bn/2) and again in lanes 64-127 for [bn/2, bn), in
            // bn/2 TMEM columns. So warp quarter q stores rows (q & 1) * 32 + lane of the CTA's 64,
            // columns from (q >> 1) * bn/2; a whole tile's quarter stores rows q * 32 + lane, all bn.
            const bool half = tc.half;
            const int local_row = half ? tc.mt * C::kClusterM + int(cta_rank) * 64 + (q & 1) * 32 + int(lane)
                                       : tc.mt * C::kClusterM + int(cta_rank) * kBM + row_in_cta;
            const int tile_w = half ? bn / 2 : bn;                      // output columns of this warp
            const int col0 = tc.nt * bn + (half && q >= 2 ? bn / 2 : 0);  // its first output column
            const bool row_ok = local_row < m;
            const int64_t grow = int64_t(g_row0) + local_row;
            T *orow = out + grow * p.n;
            const uint32_t t_row = tmem_base + (uint32_t(q * 32) << 16) + uint32_t(acc * kBN);
            bool store_out = true;
            // 32-column chunks of the tile (a tile width of 16 mod 32 ends in a half chunk: it is read
            // whole from TMEM, inside the accumulator buffer, and its upper 16 columns are dropped)
            const int nch = (tile_w + 31) / 32;
            // split-K: first float4 of this warp's workspace region (p.splits x nch blocks of 4 KB)
            const int64_t ws_warp = ((int64_t(t) * kCG + int(cta_rank)) * 4 + q) * int64_t(p.splits) * nch * 256;
            if (nsplit > 1) {
                // A tile in pieces. Each piece but the one that sums publishes its fp32 partial and
                // counts itself in (per tile, CTA and warp). Split-K: the splits of a tile run side
                // by side, so whichever arrives last sums them. Stream-K: piece 0 is the end of its
                // cluster's range, processed after the other pieces (the starts of theirs), so it
                // is the fixed summer: it writes no partial and waits (bounded) for the others'.
                // This warp's workspace blocks of the tile: [piece][chunk], each block the 32 x 32
                // fp32 fragment of one tcgen05.ld in lane order (float4 j of lane l at j * 32 + l),
                // so every warp access is 512 contiguous bytes.
                int32_t *ctr = p.counters + (int64_t(t) * kCG + int(cta_rank)) * 4 + q;
                if (!GG_CHECK((int64_t(t) * kCG + int(cta_rank)) * 4 + q < p.ctr_entries, 5))
                    break;
                const bool fixed_summer = p.sk_tiles > 0 && split == 0;
                if (!fixed_summer) {
                    float4 *wsw = reinterpret_cast<float4 *>(p.ws) + ws_warp + (int64_t(split) * nch) * 256 + lane;
#pragma unroll 1
                    for (int c = 0; c < nch; ++c) {
                        uint32_t r[32];
                        ptx::tmem_ld_32x32b_x32(t_row + uint32_t(c * 32), r);
                        ptx::tmem_wait_ld(r);
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            if (GG_CHECK(ws_warp + (int64_t(split) * nch + c) * 256 + lane + j * 32 < p.ws_float4s, 4))
                            __stcg(wsw + c * 256 + j * 32,
                                   make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                               __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
                    }
                    __threadfence();
                    __syncwarp();
                    int prev = 0;
                    if (lane == 0)
                        prev = atomicAdd(ctr, 1);
                    prev = __shfl_sync(0xffffffffu, prev, 0);
                    store_out = p.sk_tiles == 0 && prev == nsplit - 1;
                } else {
                    int ok = 1;
                    if (lane == 0)
                        ok = wait_count(ctr, nsplit - 1, ab, kStatusTimeout | kRoleEpilogue | 0x30u | uint32_t(q)) ? 1 : 0;
                    if (__shfl_sync(0xffffffffu, ok, 0) == 0)
                        break;
                }
                if (store_out) {
                    __threadfence();
                    if (lane == 0)
                        *ctr = 0;  // ready for the next launch
                }
            }
            // TMA-store path: the warp's 32 rows all inside the group, no split-K sums, and a short
            // reduction (the epilogue is then the bottleneck and the asynchronous bulk stores keep
            // the warp free); each pair of 32-column chunks goes out as one 64 x 32 box through a
            // staging buffer. Tiles with a long reduction store straight from registers: their
            // epilogue is hidden behind the next main loop, and skipping the staging spares the
            // shared-memory bandwidth the main loop uses (measured: +2-5% on configs D, E, P).
            const int slab_rows_ok = m - (tc.mt * C::kClusterM + int(cta_rank) * kBM + q * 32);
            const int c_tma = (GG_TMA_STORE && !half && nsplit == 1 && slab_rows_ok >= 32 && tc.red_atoms < p.store_min_atoms)
                                  ? (bn / 64) * 2 : 0;
#pragma unroll 1
            for (int c = 0; c < c_tma; c += 2) {
                const uint32_t buf = out_stage + uint32_t(out_buf) * C::kStageOutBytes;
                if (lane == 0)
                    ptx::bulk_wait_group_read<1>();  // this buffer's previous store has read it
                __syncwarp();
                // both 32-column halves of the box in flight before one wait
                uint32_t rr[2][32];
                ptx::tmem_ld_32x32b_x32(t_row + uint32_t(c * 32), rr[0]);
                ptx::tmem_ld_32x32b_x32(t_row + uint32_t((c + 1) * 32), rr[1]);
                ptx::tmem_wait_ld(rr[0]);
                ptx::tmem_tie(rr[1]);
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t (&r)[32] = rr[hh];
                    if (zero_tile) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            r[j] = 0u;
                    }
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        const int j = hh * 4 + jj;  // 16-byte chunk of the 128-byte row
                        const uint32_t dst = buf + uint32_t(lane) * 128u + uint32_t(((j ^ int(lane & 7u)) * 16));
                        ptx::st_shared_v4(dst, pack2<T>(r[8 * jj + 0], r[8 * jj + 1]), pack2<T>(r[8 * jj + 2], r[8 * jj + 3]),
                                          pack2<T>(r[8 * jj + 4], r[8 * jj + 5]), pack2<T>(r[8 * jj + 6], r[8 * jj + 7]));
                    }
                }
                ptx::fence_proxy_async_smem();  // generic-proxy writes -> visible to the TMA engine
                __syncwarp();
                if (lane == 0) {
                    // a box that starts past the last column (the N tail of a tile) holds nothing to store
                    const int sx = tc.nt * bn + c * 32, sy = g_row0 + tc.mt * C::kClusterM + int(cta_rank) * kBM + q * 32;
                    if (sx < p.n && GG_CHECK(sx >= 0 && (sx & 7) == 0 && sy >= 0 && sy + 32 <= p.out_rows, 3))
                        ptx::tma_store_2d(&tmap_out, buf, sx, sy, store_policy);
                    ptx::bulk_commit_group();
                }
                out_buf ^= 1;
            }
            const int col_end = min(p.n, col0 + tile_w);  // this warp's last column + 1
            // Store 32 accumulator columns (fp32 bits) of this lane's row: whole 32-byte sectors
            // where the row allows (N % 16 == 0 keeps rows 32-byte aligned), else 16-byte pieces;
            // columns past the tile or past N are skipped in 8s.
            auto store_chunk = [&](int c, const uint32_t (&r)[32]) {
                if (!row_ok)
                    return;
                const int col = col0 + c * 32;
                if (!GG_CHECK(grow >= 0 && grow < p.out_rows && col >= 0 && (col & 7) == 0, 2))
                    return;
                uint32_t h[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    h[j] = pack2<T>(r[2 * j], r[2 * j + 1]);
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    T *dst = orow + col + hh * 16;
                    if (col + hh * 16 + 16 <= col_end && (reinterpret_cast<uintptr_t>(dst) & 31u) == 0 &&
                        GG_CHECK(col + hh * 16 + 16 <= p.n, 2)) {
                        ptx::st_cs_v8(dst, h[8 * hh], h[8 * hh + 1], h[8 * hh + 2], h[8 * hh + 3], h[8 * hh + 4],
                                      h[8 * hh + 5], h[8 * hh + 6], h[8 * hh + 7]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 2; ++j)
                            if (col + hh * 16 + j * 8 < col_end && GG_CHECK(col + hh * 16 + j * 8 + 8 <= p.n, 2))
                                __stcs(reinterpret_cast<uint4 *>(dst + j * 8),
                                       make_uint4(h[8 * hh + 4 * j], h[8 * hh + 4 * j + 1], h[8 * hh + 4 * j + 2],
                                                  h[8 * hh + 4 * j + 3]));
                    }
                }
            };
            if (store_out && nsplit > 1) {
                // Sum of the tile's pieces 0..nsplit-1 in that order (this unit's own from TMEM),
                // chunk by chunk. The other pieces' blocks stream in (chunk, piece) order through a
                // ring of kPrefetch register buffers, so that many L2 reads are in flight at once;
                // the ring is indexed at compile time (block b sits in buffer b % kPrefetch).
                constexpr int kPrefetch = 2;
                const int others = nsplit - 1;
                const int nb = nch * others;
                auto load_blk = [&](int b, float4 (&dst)[8]) {
                    const int c = b / others;
                    const int o = b - c * others;
                    const int s2 = o + (o >= split ? 1 : 0);
                    const float4 *src = reinterpret_cast<const float4 *>(p.ws) + ws_warp + (int64_t(s2) * nch + c) * 256 + lane;
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        dst[j] = GG_CHECK(ws_warp + (int64_t(s2) * nch + c) * 256 + lane + j * 32 < p.ws_float4s, 4)
                                     ? __ldcg(src + j * 32) : make_float4(0.f, 0.f, 0.f, 0.f);
                };
                float4 pf[kPrefetch][8];
#pragma unroll
                for (int i = 0; i < kPrefetch; ++i)
                    if (i < nb)
                        load_blk(i, pf[i]);
                uint32_t r[32];
                float sum[32];
#pragma unroll 1
                for (int b0 = 0; b0 < nb; b0 += kPrefetch) {
#pragma unroll
                    for (int i = 0; i < kPrefetch; ++i) {
                        const int b = b0 + i;
                        if (b < nb) {
                            const int c = b / others;
                            const int o = b - c * others;
                            if (o == 0) {
                                ptx::tmem_ld_32x32b_x32(t_row + uint32_t(c * 32), r);
                                ptx::tmem_wait_ld(r);
#pragma unroll
                                for (int j = 0; j < 32; ++j)
                                    sum[j] = 0.f;
                            }
                            if (o == split) {
#pragma unroll
                                for (int j = 0; j < 32; ++j)
                                    sum[j] += __uint_as_float(r[j]);
                            }
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                sum[4 * j] += pf[i][j].x;
                                sum[4 * j + 1] += pf[i][j].y;
                                sum[4 * j + 2] += pf[i][j].z;
                                sum[4 * j + 3] += pf[i][j].w;
                            }
                            if (b + kPrefetch < nb)
                                load_blk(b + kPrefetch, pf[i]);
                            if (o == others - 1) {
                                if (split == others) {
#pragma unroll
                                    for (int j = 0; j < 32; ++j)
                                        sum[j] += __uint_as_float(r[j]);
                                }
#pragma unroll
                                for (int j = 0; j < 32; ++j)
                                    r[j] = __float_as_uint(sum[j]);
                                store_chunk(c, r);
                            }
                        }
                    }
                }
            } else {
#pragma unroll 1
                for (int c = c_tma; store_out && c < nch; ++c) {
                    uint32_t r[32];
                    ptx::tmem_ld_32x32b_x32(t_row + uint32_t(c * 32), r);
                    ptx::tmem_wait_ld(r);
                    if (zero_tile) {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            r[j] = 0u;
                    }
                    store_chunk(c, r);
                }
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (kCG == 2)
                    ptx::mbar_arrive_cluster_cta(tempty_leader0 + 8u * acc);
                else
                    ptx::mbar_arrive(tempty_bar(acc));
            }
        }
        if (GG_TMA_STORE && lane == 0)
            ptx::bulk_wait_group_all();  // stores complete before the CTA (and its smem) goes away
        __syncwarp();
    }

    // ---------------- teardown ----------------
    if (*abort_flag != 0u) {
        // Let copies and MMAs already issued drain before the memory they target goes away.
        const uint64_t t0 = ptx::globaltimer();
        while (ptx::globaltimer() - t0 < 200000ull)
            __nanosleep(1000);
    }
    ptx::tc_fence_before();
    __syncthreads();
    if constexpr (kCG == 2)
        ptx::cluster_sync();  // no remote arrive or MMA still targets either CTA
    ptx::tc_fence_after();
    if (warp == 1)
        ptx::tmem_dealloc<kCG>(tmem_base, C::kTmemCols);
}

}  // namespace gg
