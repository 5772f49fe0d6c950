// gg_sched.h -- host side of the launch schedule: the cost model that picks the tile shape, tile
// width and split-K / stream-K form of a launch (choose_tiling), and the stream-K arithmetic that
// sizes its fp32 workspace. Shared by the library (gg_capi.cu) and the CPU tests
// (tests/sched_check.cu, tests/test_schedule.py). The device side of the same schedule (each
// cluster's unit list, the tile decode) is units_of / unit_at / decode_tile in gg_kernel.cuh.
#pragma once

#include <algorithm>
#include <cstdint>
#include <vector>

#include "gg_b200.h"
#include "gg_kernel.cuh"

namespace gg {

// Stream-K region of a launch: the first `sk_tiles` tiles, whose K atoms are dealt out evenly to
// the `clusters` clusters. kind 1: the tiles that would form a partial last wave (tiles % clusters);
// kind 2: those plus one full wave, so that each cluster's range spans at least one tile. Returns 0
// when the kind does not apply (no partial wave, too few tiles, or fewer atoms than clusters).
inline int64_t sk_tiles_for(int64_t tiles, int64_t clusters, int64_t atoms, int kind) {
    const int64_t rem = tiles % clusters;
    const int64_t sk = kind == 1 ? rem : kind == 2 && rem > 0 && tiles >= rem + clusters ? rem + clusters : 0;
    return sk > 0 && sk * atoms >= clusters ? sk : 0;
}

// Most pieces any stream-K tile is cut into (cluster c's range is [c S / C, (c+1) S / C)); the
// kernel's workspace stride and the length of its longest fix-up.
inline int sk_max_pieces(int64_t sk_tiles, int64_t clusters, int64_t atoms) {
    const int64_t S = sk_tiles * atoms;
    auto cluster_of = [&](int64_t g) { return ((g + 1) * clusters - 1) / S; };
    int64_t most = 1;
    for (int64_t t = 0; t < sk_tiles; ++t)
        most = std::max(most, cluster_of((t + 1) * atoms - 1) - cluster_of(t * atoms) + 1);
    return int(most);
}

// The shape of one compiled kernel variant, as the cost model sees it.
struct TileShape {
    int cg;         // CTAs per tile (1 or 2)
    int bn;         // widest tile N of the variant
    int cluster_m;  // tile M
    int atoms;      // 64-element K atoms per pipeline stage
};

inline int64_t tiles_for(const gg_problem *p, const TileShape &v, int bn) {
    const int64_t tn = (p->n + bn - 1) / bn;
    int64_t t = 0;
    for (int g = 0; g < p->group_num; ++g)
        t += (p->group_m[g] + v.cluster_m - 1) / v.cluster_m * tn;
    return t;
}

struct Choice {
    int variant;
    int bn;
    int splits;
    bool hybrid;  // splits > 1: only tiles % slots tiles are split (what would be a partial last wave)
    int sk;       // stream-K: 0 none, 1 over the tiles of the partial last wave, 2 over those and
                  // one full wave more
};

// Cycles per MMA of one CTA (pair) for a tile width, fitted to B200 measurements in two regimes.
// Few waves: the MMA issue keeps pace with the tensor pipe, so an MMA of width bn costs about bn/2
// cycles plus a small constant (one-wave runs with K = 16384, every width; the one-atom-stage
// variant a little more). That holds for the pair variant up to three waves of tiles whatever the
// K; the one-CTA variants keep it only for a short launch (one wave of at most 64 K-atoms per SM,
// burst clocks): over longer ones they run power-capped and measured 1.5-2x slower per flop than
// a pair (each SM loads its own B tile). Many waves: the launch runs power-capped and narrow tiles
// pay for their extra operand traffic per flop; the costs there are the older multi-wave fit, which
// picks the measured best widths on those shapes (240 over 192 on N = 2880, 256 on L, D, E).
// `atoms` is the K atoms one cluster works through in the launch.
inline double cycles_per_mma(const TileShape &v, int bn, int64_t tiles, int slots, double atoms) {
    const bool few_waves = v.cg == 2 ? tiles <= 3 * int64_t(slots) : tiles <= slots && atoms <= 64.0;
    if (few_waves)
        return 0.4 * bn + (v.cg == 1 && v.atoms < 2 ? 26.0 : 24.0);
    if (v.cg == 2)
        return std::max(0.344 * bn + 60.0, 130.0);
    return v.atoms >= 2 ? 0.344 * bn + 63.0 : std::max(0.396 * bn + 70.0, 150.0);
}

// Model of one launch in cycles per SM: waves x K-atoms x 4 MMAs x cycles per MMA. Waves count
// whole, so the model trades tile width against wave quantisation and M/N tail waste. With
// splits > 1 every tile (hybrid = false), or only tiles % slots of them (hybrid = true: the
// tiles that would form a partial last wave), is cut into `splits` K ranges whose fp32
// partials the last arriving split sums. Split units run first; in the hybrid form the whole
// tiles that follow hide that fix-up, in the plain form it ends the launch.
inline double model_cycles(const gg_problem *p, const TileShape &v, int bn, int slots, int splits, bool hybrid, int sk = 0) {
    const int64_t tiles = tiles_for(p, v, bn);
    const int64_t atoms = (p->k + kBK - 1) / kBK;
    // A CTA pair pays a fixed start-up cost (cluster barrier, cross-CTA pipeline fill) that only
    // matters for launches of a few microseconds.
    double fixed = v.cg == 2 ? 1500.0 : 0.0;
    double unit_atoms;
    if (sk > 0) {
        // stream-K: whole waves, then an equal share of the stream-K region's atoms. Every cluster
        // writes an fp32 partial and reads one back at about the same time, so the fix-up runs at
        // the GPU-wide store rate: timestamps inside the kernel show ~3.5-5 us per 128 x 240 fp32
        // partial per CTA (~16 bytes per cycle per SM) plus ~2 us of fence and arrival latency.
        const int64_t skt = sk_tiles_for(tiles, slots, atoms, sk);
        const int64_t S = skt * atoms;
        unit_atoms = double((tiles - skt) / slots) * double(atoms) + double((S + slots - 1) / slots);
        fixed += 4000.0 + double(sk_max_pieces(skt, slots, atoms) - 1) * double(bn) * 64.0;
    } else if (splits <= 1) {
        unit_atoms = double((tiles + slots - 1) / slots) * double(atoms);
    } else {
        const int64_t whole = hybrid ? tiles / slots * slots : 0;
        const int64_t split_units = (tiles - whole) * splits;
        unit_atoms = double(whole / slots) * double(atoms) +
                     double((split_units + slots - 1) / slots) * double((atoms + splits - 1) / splits);
        // fix-up: each split writes its fp32 partial (128 x bn per CTA), the last arriver reads
        // the others back and stores out with direct stores
        fixed += hybrid ? 1000.0 + double(splits - 1) * double(bn) * 12.0 : 2500.0 + double(splits) * double(bn) * 10.0;
    }
    return unit_atoms * 4.0 * cycles_per_mma(v, bn, tiles, slots, unit_atoms) + fixed;
}

// Pick the variant, tile width and split-K / stream-K form with the smallest modelled time.
// `forced_variant` >= 0 and `forced_bn` > 0 restrict the search; `min_splits`..`max_splits` is
// the range of split counts tried; `forced_hybrid` is -1 (either form), 0 or 1; `stream_k` is -1
// (automatic), 0 (never) or the stream-K kind to use. `pairs` is the number of co-resident CTA
// pairs of the 2-CTA variant.
inline Choice choose_tiling(const TileShape *shapes, int nshapes, const gg_problem *p, int num_sms, int pairs,
                            int forced_variant, int forced_bn,
                     int max_splits = 1, bool mn_major_b = false, int min_splits = 1, int forced_hybrid = -1,
                     int stream_k = 0) {
    Choice best{-1, 0, 1, false, 0};
    double best_t = 0;
    const int64_t atoms = (p->k + kBK - 1) / kBK;
    for (int vi = 0; vi < nshapes; ++vi) {
        if (forced_variant >= 0 && vi != forced_variant)
            continue;
        const TileShape &v = shapes[vi];
        const int slots = v.cg == 2 ? pairs : num_sms;
        if (slots < 1)
            continue;
        for (int bn = v.bn; bn >= 16; bn -= 16) {
            if (forced_bn > 0 && bn != forced_bn)
                continue;
            if (forced_bn <= 0 && bn < 96)
                continue;  // narrower tiles only on request
            if (forced_bn <= 0 && bn < 128 && tiles_for(p, v, bn) > slots)
                continue;  // below 128 columns only for a one-wave tiling (it fills more SMs)
            // A width in steps of 16 (not 32) only where it tiles N exactly (N = 2880 = 12 x 240
            // against 256's 6.7% padding: +2-9% measured), or where a width of at least 160 fits
            // the launch in one wave (one tile per CTA or pair: 1 x 512 x 6144 x 16384 as 70 pairs
            // of 256 x 176 +5.5% over 3-way split-K, 240-wide one-CTA and pair tilings of four more
            // single-wave suite shapes +0.6-2.4%); with a ragged N tail over several waves it
            // measured between -5% and +3% against the widths in steps of 32.
            if (forced_bn <= 0 && bn % 32 != 0 && p->n % bn != 0 && !(bn >= 160 && tiles_for(p, v, bn) <= slots))
                continue;
            if (mn_major_b && (bn / v.cg) % 64 != 0)
                continue;  // MN-major B is loaded in 64-column boxes
            const int64_t tiles = tiles_for(p, v, bn);
            // stream-K candidates (kinds 1 and 2), unless split-K is forced
            for (int kind = 1; kind <= 2 && min_splits == 1 && stream_k != 0; ++kind) {
                if (stream_k > 0 && kind != stream_k)
                    continue;
                const int64_t skt = sk_tiles_for(tiles, slots, atoms, kind);
                if (skt == 0)
                    continue;
                const int pieces = sk_max_pieces(skt, slots, atoms);
                // automatic: at most 4 pieces per tile and >= 4 atoms per cluster
                if (stream_k < 0 && (pieces > 4 || skt * atoms < 4 * int64_t(slots)))
                    continue;
                const double t = model_cycles(p, v, bn, slots, 1, false, kind);
                if (best.variant < 0 || t < best_t * 0.999) {
                    best = {vi, bn, pieces, false, kind};
                    best_t = t;
                }
            }
            if (stream_k > 0)
                continue;  // a forced stream-K kind is the only form tried
            for (int s = min_splits; s <= max_splits; ++s) {
                for (int hy = 0; hy < 2; ++hy) {
                    if ((s == 1 && hy == 1) || (forced_hybrid >= 0 && s > 1 && hy != forced_hybrid))
                        continue;
                    const bool forced = min_splits > 1;
                    if (s > 1 && !forced) {
                        // automatic split-K: >= 8 K atoms per split, and the split units of the
                        // pure form fill at most 4 waves, those of the hybrid form 2
                        const int64_t rem = hy ? tiles % slots : tiles;
                        if (atoms < 8 * s || rem == 0 || (hy && tiles < slots) || (!hy && tiles >= slots) ||
                            rem * s > (hy ? 2 : 4) * int64_t(slots))
                            continue;
                    }
                    if (s > 1 && hy && tiles % slots == 0)
                        continue;  // no partial wave to split
                    const double t = model_cycles(p, v, bn, slots, s, hy == 1);
                    if (best.variant < 0 || t < best_t * 0.999) {
                        best = {vi, bn, s, hy == 1, 0};
                        best_t = t;
                    }
                }
            }
        }
    }
    return best;
}

// Planned tile order for launches whose tiles cost very different amounts (wgrad under skewed
// routing: an expert with few tokens has a short reduction, so its tiles are bound by their stores
// -- a whole tile of output each -- while a large expert's tiles are bound by the tensor pipe). In
// group order the two kinds run as separate phases, first one resource idle, then the other.
// `natural` holds the tiles in group order as pairs (group, mt << 16 | nt); `cost[g]` estimates
// a tile's cycles and `store_bound[g]` its kind. The two kinds are merged so that each has
// dispatched the same fraction of its total estimated work at every point (ties to the
// tensor-bound kind); within a kind the group order is kept. With dynamic dispatch, each cluster
// then takes the next tile of the merged list as it finishes one, so stores and MMAs overlap.
inline void interleave_tiles(const std::vector<int32_t> &natural, const std::vector<double> &cost,
                             const std::vector<char> &store_bound, std::vector<int32_t> &out) {
    const size_t n = natural.size() / 2;
    double total[2] = {0, 0};
    std::vector<size_t> idx[2];
    for (size_t i = 0; i < n; ++i) {
        const int g = natural[2 * i];
        const int k = store_bound[size_t(g)] ? 1 : 0;
        idx[k].push_back(i);
        total[k] += cost[size_t(g)];
    }
    out.clear();
    out.reserve(natural.size());
    size_t pos[2] = {0, 0};
    double done[2] = {0, 0};
    while (pos[0] < idx[0].size() || pos[1] < idx[1].size()) {
        int k;
        if (pos[0] >= idx[0].size())
            k = 1;
        else if (pos[1] >= idx[1].size())
            k = 0;
        else
            k = done[0] / total[0] <= done[1] / total[1] ? 0 : 1;
        const size_t i = idx[k][pos[k]++];
        out.push_back(natural[2 * i]);
        out.push_back(natural[2 * i + 1]);
        done[k] += cost[size_t(natural[2 * i])];
    }
}

}  // namespace gg
