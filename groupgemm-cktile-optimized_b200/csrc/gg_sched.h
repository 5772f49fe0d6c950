// gg_sched.h -- host-side arithmetic of the stream-K schedule, shared by the library (which
// sizes the launch and the fp32 workspace with it) and the CPU schedule test. The device side of
// the same schedule (each cluster's unit list) is units_of / unit_at in gg_kernel.cuh.
#pragma once

#include <algorithm>
#include <cstdint>

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

}  // namespace gg
