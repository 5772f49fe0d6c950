// CPU check of the kernel's work-unit schedule (built and run by tests/test_schedule.py).
//
// It calls the same units_of / unit_at the kernel runs on the device (gg_kernel.cuh, host-callable)
// and the host-side stream-K arithmetic the library sizes the launch with (gg_sched.h), for every
// cluster of random launches of each schedule form the library produces: whole tiles, plain
// split-K, split-K of the partial last wave, and stream-K of kind 1 and 2. For each launch:
//   * every (tile, K atom) is covered by exactly one unit, and every unit is non-empty;
//   * the pieces of a tile are numbered 0..n-1 in K order and agree on n (the fixed summation order);
//   * a tile cut into pieces has workspace: n <= splits (the stride) and the tile is a split tile;
//   * stream-K: every piece but piece 0 is the first unit of its cluster, so the fixed summer
//     (piece 0) only ever waits for units that wait on nothing themselves (no circular wait).
// The dynamic tile dispatch is played out in random fetch orders (check_dynamic), the
// half-height tile flag is checked on every decoded tile, and the planned (interleaved) tile
// order is checked (check_interleave).
// Then decode_tile, for random group sizes (empty groups included), widths, bands and both raster
// orders: tile indices map onto every (group, m-tile, n-tile) exactly once.
// Prints "ok <launches> <units> <tables>" and exits 0, or prints the first violation and exits 1.
// With `choose B,M,N,K ...` it prints the cost model's automatic choice for each problem instead.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "gg_b200.h"
#include "gg_kernel.cuh"
#include "gg_sched.h"

namespace {

struct Rng {
    uint64_t s;
    uint64_t next() {
        s ^= s << 13;
        s ^= s >> 7;
        s ^= s << 17;
        return s;
    }
    int range(int lo, int hi) { return lo + int(next() % uint64_t(hi - lo + 1)); }  // [lo, hi]
};

struct Seen {
    int piece, npieces, atom0, atom1, cluster, index;
};

bool fail(const char *what, int form, int64_t tiles, int C, int A, int s, int t) {
    std::printf("FAIL %s: form %d tiles %lld clusters %d atoms %d splits %d tile %d\n", what, form, (long long)tiles,
                C, A, s, t);
    return false;
}

// One launch: form 0 whole tiles, 1 plain split-K, 2 last-wave split-K, 3 / 4 stream-K kind 1 / 2.
bool check(int form, int64_t tiles, int slots, int A, int s, long long &units_seen) {
    gg::KernelParams p{};
    p.total_tiles = int32_t(tiles);
    p.num_kb = A;
    int C = slots;
    if (form == 0) {
        p.splits = 1;
    } else if (form == 1 || form == 2) {
        p.splits = s;
        p.split_tiles = int32_t(form == 1 ? tiles : tiles % slots);
        const int64_t units = tiles + int64_t(p.split_tiles) * (s - 1);
        C = int(std::min<int64_t>(slots, units));  // the launch's grid, as prepare sizes it
    } else {
        const int64_t sk = gg::sk_tiles_for(tiles, slots, A, form == 3 ? 1 : 2);
        if (sk == 0)
            return true;  // the library refuses this kind for this tiling
        p.sk_tiles = int32_t(sk);
        p.splits = gg::sk_max_pieces(sk, slots, A);
    }
    std::vector<std::vector<Seen>> by_tile(static_cast<std::size_t>(tiles));
    for (int c = 0; c < C; ++c) {
        const gg::UnitList l = gg::units_of(p, c, C);
        for (int i = 0; i < l.n; ++i) {
            const gg::Unit u = gg::unit_at(p, l, c, C, i);
            if (u.t < 0 || u.t >= tiles)
                return fail("tile index out of range", form, tiles, C, A, s, u.t);
            if (!(0 <= u.atom0 && u.atom0 < u.atom1 && u.atom1 <= A))
                return fail("empty or out-of-range K range", form, tiles, C, A, s, u.t);
            by_tile.at(static_cast<std::size_t>(u.t)).push_back({u.piece, u.npieces, u.atom0, u.atom1, c, i});
            ++units_seen;
        }
    }
    for (int64_t t = 0; t < tiles; ++t) {
        std::vector<Seen> v = by_tile.at(static_cast<std::size_t>(t));
        if (v.empty())
            return fail("tile not covered", form, tiles, C, A, s, int(t));
        std::sort(v.begin(), v.end(), [](const Seen &a, const Seen &b) { return a.atom0 < b.atom0; });
        int at = 0;
        const int n = v[0].npieces;
        for (size_t j = 0; j < v.size(); ++j) {
            if (v[j].atom0 != at)
                return fail("K atoms missing or covered twice", form, tiles, C, A, s, int(t));
            at = v[j].atom1;
            if (v[j].npieces != n || v[j].piece != int(j))
                return fail("pieces not numbered 0..n-1 in K order", form, tiles, C, A, s, int(t));
        }
        if (at != A || int(v.size()) != n)
            return fail("K range not covered to the end", form, tiles, C, A, s, int(t));
        if (n > 1) {
            const bool split_tile = p.sk_tiles > 0 ? t < p.sk_tiles : t < p.split_tiles;
            if (!split_tile || n > p.splits)
                return fail("pieces without workspace", form, tiles, C, A, s, int(t));
            if (p.sk_tiles > 0)
                for (size_t j = 1; j < v.size(); ++j)
                    if (v[j].index != 0)
                        return fail("stream-K piece > 0 not first in its cluster", form, tiles, C, A, s, int(t));
        }
    }
    return true;
}

// decode_tile over one launch's group tables: tiles 0..total-1 map onto every (group, m-tile,
// n-tile) of the non-empty groups exactly once, with the group's row range, for a raster order
// and band; walked in order with one cursor (as each role does) and from a fresh cursor.
template <int kCM, int kOp>
bool check_decode(const std::vector<int64_t> &group_m, int tiles_n, int band, int raster, int tile_rows) {
    const int G = int(group_m.size());
    std::vector<int32_t> tile_off(G + 1), row_off(G + 1);
    int64_t tiles = 0, rows = 0;
    for (int g = 0; g < G; ++g) {
        tile_off[g] = int32_t(tiles);
        row_off[g] = int32_t(rows);
        const int64_t tile_rows_g = kOp == gg::kOpWgrad ? tile_rows : group_m[g];
        tiles += (tile_rows_g + kCM - 1) / kCM * tiles_n;
        rows += group_m[g];
    }
    tile_off[G] = int32_t(tiles);
    row_off[G] = int32_t(rows);
    gg::KernelParams p{};
    p.tile_off = tile_off.data();
    p.row_off = row_off.data();
    p.tiles_n = tiles_n;
    p.band = band;
    p.raster = raster;
    p.num_kb = 7;
    p.tile_rows = tile_rows;
    std::vector<char> hit(size_t(tiles), 0);
    int cursor = 0;
    gg::GroupCursor gcur;
    for (int64_t t = 0; t < tiles; ++t) {
        const gg::TileCoord tc = gg::decode_tile<kCM, kOp>(p, int(t), cursor);
        int fresh = 0;
        const gg::TileCoord tf = gg::decode_tile<kCM, kOp>(p, int(t), fresh);
        const gg::TileCoord tg = gg::decode_tile<kCM, kOp>(p, int(t), gcur);  // the kernel's cached form
        if (tg.g != tc.g || tg.mt != tc.mt || tg.nt != tc.nt || tg.rows != tc.rows || tg.out_row0 != tc.out_row0 ||
            tg.red_atoms != tc.red_atoms || tg.half != tc.half) {
            std::printf("FAIL decode_tile with a group cache: tile %lld\n", (long long)t);
            return false;
        }
        const int g = tc.g;
        const int64_t m_rows = kOp == gg::kOpWgrad ? tile_rows : group_m[size_t(g)];
        const int tiles_m = int((m_rows + kCM - 1) / kCM);
        const bool ok = g >= 0 && g < G && tc.mt >= 0 && tc.mt < tiles_m && tc.nt >= 0 && tc.nt < tiles_n &&
                        tc.rows == int(m_rows) &&
                        tc.out_row0 == (kOp == gg::kOpWgrad ? g * tile_rows : row_off[size_t(g)]) &&
                        tf.g == tc.g && tf.mt == tc.mt && tf.nt == tc.nt;
        if (!ok) {
            std::printf("FAIL decode_tile: cm %d op %d G %d tiles_n %d band %d raster %d tile %lld\n", kCM, kOp, G,
                        tiles_n, band, raster, (long long)t);
            return false;
        }
        // half-height pair tiles: exactly the last m-tile of a group whose remainder is 1..128 rows
        // (tiles of 256 rows, forward / dgrad); never with the option off, for 128-row tiles or wgrad
        const int64_t rem = m_rows % 256;
        const bool want_half = kCM == 256 && kOp != gg::kOpWgrad && rem != 0 && rem <= 128 && tc.mt == tiles_m - 1;
        const bool got_half = gg::is_half_tile<kCM, kOp>(1, tc.rows, tc.mt);
        if (got_half != want_half || tc.half || gg::is_half_tile<kCM, kOp>(0, tc.rows, tc.mt)) {
            std::printf("FAIL half-tile flag: cm %d op %d rows %lld mt %d\n", kCM, kOp, (long long)m_rows, tc.mt);
            return false;
        }
        const int64_t idx = tile_off[size_t(g)] + int64_t(tc.mt) * tiles_n + tc.nt;
        if (hit.at(static_cast<std::size_t>(idx))++) {
            std::printf("FAIL decode_tile: tile (%d, %d, %d) decoded twice\n", g, tc.mt, tc.nt);
            return false;
        }
    }
    // a cluster's strided walk (tiles c, c + C, ...) with one cached cursor, as each role runs it
    for (const int C : {3, 74, 148}) {
        for (int c = 0; c < C && c < tiles; c += 7) {
            gg::GroupCursor gc;
            for (int64_t t = c; t < tiles; t += C) {
                int fresh = 0;
                const gg::TileCoord tf = gg::decode_tile<kCM, kOp>(p, int(t), fresh);
                const gg::TileCoord tg = gg::decode_tile<kCM, kOp>(p, int(t), gc);
                if (tg.g != tf.g || tg.mt != tf.mt || tg.nt != tf.nt || tg.rows != tf.rows || tg.red_atoms != tf.red_atoms) {
                    std::printf("FAIL decode_tile with a group cache, stride %d: tile %lld\n", C, (long long)t);
                    return false;
                }
            }
        }
    }
    return true;
}

// Dynamic tile dispatch (dispatched_tile / is_last_fetch, as the kernel's producer uses them): C
// clusters fetch from one counter in a random interleaving, two launches in a row on the same
// counter. Every tile runs exactly once, each cluster's tiles increase (decode_tile's cursor only
// moves forward), a launch makes exactly `tiles` fetches and leaves the counter at 0.
bool check_dynamic(Rng &rng, int tiles, int C) {
    int ctr = 0;
    for (int launch = 0; launch < 2; ++launch) {
        std::vector<int> cur(static_cast<size_t>(C), -1), last(static_cast<size_t>(C), -1);
        std::vector<char> hit(static_cast<size_t>(tiles), 0);
        std::vector<int> live;
        for (int c = 0; c < C; ++c) {
            cur[size_t(c)] = c < tiles ? c : -1;
            if (cur[size_t(c)] >= 0)
                live.push_back(c);
        }
        int fetches = 0;
        while (!live.empty()) {
            const size_t k = size_t(rng.range(0, int(live.size()) - 1));
            const int c = live[k];
            const int t = cur[size_t(c)];
            if (t <= last[size_t(c)] || hit.at(size_t(t))++) {
                std::printf("FAIL dynamic dispatch: tiles %d clusters %d tile %d repeated or out of order\n", tiles, C,
                            t);
                return false;
            }
            last[size_t(c)] = t;
            const int v = ctr++;  // atomicAdd
            ++fetches;
            if (gg::is_last_fetch(v, tiles))
                ctr = 0;
            cur[size_t(c)] = gg::dispatched_tile(v, C, tiles);
            if (cur[size_t(c)] < 0)
                live.erase(live.begin() + long(k));
        }
        const bool all = std::all_of(hit.begin(), hit.end(), [](char h) { return h == 1; });
        if (!all || ctr != 0 || fetches != tiles) {
            std::printf("FAIL dynamic dispatch: tiles %d clusters %d covered %d counter %d fetches %d\n", tiles, C,
                        int(all), ctr, fetches);
            return false;
        }
    }
    return true;
}

// Planned tile order (interleave_tiles, as gg_prepare builds it for wgrad): for random group
// tables, the merged list is a permutation of the group-order tiles, keeps the group order within
// each kind, keeps the two kinds' dispatched work fractions within one tile's share of each other,
// and decode_tile over the list returns the listed tiles.
bool check_interleave(Rng &rng) {
    const int G = rng.range(1, 40);
    std::vector<int64_t> gm(static_cast<size_t>(G));
    for (auto &m : gm)
        m = rng.range(1, 5) == 1 ? 0 : (rng.range(1, 3) == 1 ? rng.range(1, 120) : rng.range(1, 30000));
    const int tile_rows = 256 * rng.range(1, 6), tiles_n = rng.range(1, 12);
    std::vector<int32_t> tile_off(static_cast<size_t>(G) + 1), row_off(static_cast<size_t>(G) + 1);
    int64_t tiles = 0, rows = 0;
    for (int g = 0; g < G; ++g) {
        tile_off[size_t(g)] = int32_t(tiles);
        row_off[size_t(g)] = int32_t(rows);
        tiles += (tile_rows + 255) / 256 * tiles_n;
        rows += gm[size_t(g)];
    }
    tile_off[size_t(G)] = int32_t(tiles);
    row_off[size_t(G)] = int32_t(rows);
    gg::KernelParams p{};
    p.tile_off = tile_off.data();
    p.row_off = row_off.data();
    p.tiles_n = tiles_n;
    p.band = rng.range(1, 9);
    p.tile_rows = tile_rows;
    std::vector<int32_t> natural(2 * size_t(tiles)), order;
    int cursor = 0;
    for (int64_t t = 0; t < tiles; ++t) {
        const gg::TileCoord tc = gg::decode_tile<256, gg::kOpWgrad>(p, int(t), cursor);
        natural[2 * size_t(t)] = tc.g;
        natural[2 * size_t(t) + 1] = (tc.mt << 16) | tc.nt;
    }
    std::vector<double> cost(static_cast<size_t>(G));
    std::vector<char> sb(static_cast<size_t>(G));
    double total[2] = {0, 0}, most = 0;
    for (int g = 0; g < G; ++g) {
        const double mma = double((gm[size_t(g)] + 63) / 64) * 4.0 * 128.0, epi = 2816.0;
        cost[size_t(g)] = std::max(mma, epi);
        sb[size_t(g)] = mma < epi;
        total[sb[size_t(g)]] += cost[size_t(g)] * tiles_n * ((tile_rows + 255) / 256);
    }
    gg::interleave_tiles(natural, cost, sb, order);
    if (order.size() != natural.size()) {
        std::printf("FAIL interleave: size\n");
        return false;
    }
    std::vector<std::pair<int32_t, int32_t>> a, b;
    for (size_t i = 0; i < natural.size(); i += 2) {
        a.push_back({natural[i], natural[i + 1]});
        b.push_back({order[i], order[i + 1]});
    }
    std::vector<std::pair<int32_t, int32_t>> sa = a, sb2 = b;
    std::sort(sa.begin(), sa.end());
    std::sort(sb2.begin(), sb2.end());
    if (sa != sb2) {
        std::printf("FAIL interleave: not a permutation\n");
        return false;
    }
    // order within each kind, and the balance of dispatched work
    std::vector<std::pair<int32_t, int32_t>> kind_nat[2], kind_ord[2];
    for (auto &x : a)
        kind_nat[sb[size_t(x.first)]].push_back(x);
    double done[2] = {0, 0};
    for (auto &x : b) {
        const int k = sb[size_t(x.first)];
        kind_ord[k].push_back(x);
        done[k] += cost[size_t(x.first)];
        most = std::max(most, cost[size_t(x.first)]);
        if (total[0] > 0 && total[1] > 0 && done[0] < total[0] && done[1] < total[1] &&
            std::fabs(done[0] / total[0] - done[1] / total[1]) > most / std::min(total[0], total[1]) + 1e-9) {
            std::printf("FAIL interleave: kinds out of balance\n");
            return false;
        }
    }
    if (kind_nat[0] != kind_ord[0] || kind_nat[1] != kind_ord[1]) {
        std::printf("FAIL interleave: order within a kind changed\n");
        return false;
    }
    // decode_tile over the planned list returns the listed tiles
    p.tile_list = order.data();
    for (int64_t t = 0; t < tiles; ++t) {
        int unused = 0;
        const gg::TileCoord tc = gg::decode_tile<256, gg::kOpWgrad>(p, int(t), unused);
        if (tc.g != order[2 * size_t(t)] || ((tc.mt << 16) | tc.nt) != order[2 * size_t(t) + 1] ||
            tc.rows != tile_rows || tc.red_atoms != int((gm[size_t(tc.g)] + 63) / 64)) {
            std::printf("FAIL interleave: decode of the list\n");
            return false;
        }
    }
    return true;
}

}  // namespace

// `choose B,M,N,K ...`: the library's automatic choice for balanced problems on a B200 (148 SMs,
// 74 CTA pairs), with the split-K range prepare allows (up to 4 unless the fp32 partials of
// every tile would exceed 512 MB), one line per problem: variant bn splits hybrid stream_k.
int choose(int argc, char **argv) {
    const gg::TileShape shapes[3] = {{2, 256, 256, 2}, {1, 256, 128, 1}, {1, 128, 128, 2}};
    for (int i = 2; i < argc; ++i) {
        int B = 0;
        long long M = 0, N = 0, K = 0;
        if (std::sscanf(argv[i], "%d,%lld,%lld,%lld", &B, &M, &N, &K) != 4)
            return 2;
        std::vector<int64_t> gm(size_t(B), M);
        const gg_problem p{0, B, N, K, gm.data(), nullptr, nullptr, nullptr};
        const int max_splits = double(B) * double(M) * double(N) * 4.0 * 4 > 512.0 * (1 << 20) ? 1 : 4;
        const gg::Choice c = gg::choose_tiling(shapes, 3, &p, 148, 74, -1, 0, max_splits, false, 1, -1, 0);
        std::printf("%d %d %d %d %d\n", c.variant, c.bn, c.splits, c.hybrid ? 1 : 0, c.sk);
    }
    return 0;
}

int main(int argc, char **argv) {
    if (argc > 1 && std::string(argv[1]) == "choose")
        return choose(argc, argv);
    const int launches = argc > 1 ? std::atoi(argv[1]) : 20000;
    Rng rng{0x9E3779B97F4A7C15ull};
    long long units = 0;
    int done = 0;
    for (int n = 0; n < launches; ++n) {
        const int form = n % 5;
        const int slots = rng.range(1, 3) == 1 ? rng.range(1, 12) : rng.range(60, 148);
        const int64_t tiles = rng.range(1, 3) == 1 ? rng.range(1, 2 * slots) : rng.range(1, 9000);
        const int A = rng.range(1, 300);
        const int s = std::max(2, std::min(A, rng.range(2, 8)));  // the library refuses s > A
        if ((form == 1 || form == 2) && A < 2)
            continue;
        if (form == 2 && (tiles < slots || tiles % slots == 0))
            continue;  // no partial last wave: the library does not use this form
        if (!check(form, tiles, slots, A, s, units))
            return 1;
        ++done;
    }
    int decoded = 0;
    for (int n = 0; n < launches / 10; ++n) {
        std::vector<int64_t> gm(size_t(rng.range(1, 24)));
        for (auto &m : gm)
            m = rng.range(1, 4) == 1 ? 0 : rng.range(1, 3000);
        const int tiles_n = rng.range(1, 40), band = rng.range(1, 20), raster = rng.range(0, 1);
        const int tile_rows = rng.range(1, 1500);
        const bool ok = check_decode<256, gg::kOpForward>(gm, tiles_n, band, raster, tile_rows) &&
                        check_decode<128, gg::kOpForward>(gm, tiles_n, band, raster, tile_rows) &&
                        check_decode<256, gg::kOpWgrad>(gm, tiles_n, band, raster, tile_rows) &&
                        check_decode<128, gg::kOpDgrad>(gm, tiles_n, band, raster, tile_rows);
        if (!ok)
            return 1;
        ++decoded;
    }
    for (int n = 0; n < launches / 10; ++n) {
        const int C = rng.range(1, 3) == 1 ? rng.range(1, 12) : rng.range(60, 148);
        const int tiles = rng.range(1, 3) == 1 ? rng.range(C, 3 * C) : rng.range(C, 3000);
        if (!check_dynamic(rng, tiles, C))
            return 1;
    }
    for (int n = 0; n < launches / 100; ++n)
        if (!check_interleave(rng))
            return 1;
    std::printf("ok %d %lld %d\n", done, units, decoded);
    return 0;
}
