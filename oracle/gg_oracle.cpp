// CPU oracle for the forward MoE grouped GEMM  out[g] = x[g] @ w[g]^T  (RCR layout).
//
// TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
// leg load this library, and only as the checker (or as the timed CPU baseline). The product
// path (libgg_b200.so) never links or calls it.
//
// It restates, on the host, the arithmetic of the reference harness
// (TheRealMichaelWang/GroupGEMM-CKTile-Optimized):
//   * input generator      bench/bench_main.cpp:160-176  (splitmix64 + Box-Muller, N(0,1))
//   * sample selection     bench/bench_main.cpp:208-227  (4 corners + 256 random per group,
//                                                         std::mt19937_64(1234))
//   * fp32 reference       bench/bench_main.cpp:184-206  (fp32 dot of the 16-bit inputs;
//                                                         256 strided partials + tree reduce)
//   * pass rule            bench/bench_main.cpp:235-272  (|got-ref| <= 1e-2 + 1e-2*|ref|,
//                                                         NaN fails)
//   * group row mapping    ck_kernel/ck_grouped_gemm.cpp:166-188 (x+row*K, w+g*N*K, out+row*N)
// plus a full-output blocked fp32 GEMM (the "reference op's CPU fp32 path") that is also the
// timed CPU baseline. Parity is pinned against the reference's own generator and fp32
// reference kernels, compiled unmodified from the reference sources (oracle/ref_harness.cu)
// and run once to produce tests/golden/.
//
// Exported with C linkage for ctypes. Element buffers are raw 16-bit patterns
// (dtype 0 = bf16, 1 = fp16).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

namespace {

// ---- 16-bit float conversions (round to nearest even), written from the IEEE formats ----
inline float bf16_to_f32(uint16_t h) {
    uint32_t u = uint32_t(h) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu))  // NaN: keep it quiet
        return uint16_t((u >> 16) | 0x0040u);
    const uint32_t lsb = (u >> 16) & 1u;
    u += 0x7FFFu + lsb;
    return uint16_t(u >> 16);
}

inline float f16_to_f32(uint16_t h) {
    const uint32_t sign = uint32_t(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    uint32_t u;
    if (exp == 0) {
        if (man == 0) {
            u = sign;
        } else {  // subnormal: normalise
            exp = 127 - 15 + 1;
            while ((man & 0x400u) == 0) {
                man <<= 1;
                --exp;
            }
            man &= 0x3FFu;
            u = sign | (exp << 23) | (man << 13);
        }
    } else if (exp == 31) {
        u = sign | 0x7F800000u | (man << 13);
    } else {
        u = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

inline uint16_t f32_to_f16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    const uint16_t sign = uint16_t((u >> 16) & 0x8000u);
    const uint32_t absu = u & 0x7FFFFFFFu;
    if (absu >= 0x7F800000u)  // inf / NaN
        return sign | 0x7C00u | (absu > 0x7F800000u ? 0x200u : 0u);
    if (absu >= 0x477FF000u)  // rounds to >= 65520: overflow to inf
        return sign | 0x7C00u;
    const int e = int(absu >> 23) - 127;
    if (e < -14) {  // subnormal half (or zero)
        if (e < -25)
            return sign;
        const uint32_t man = (absu & 0x7FFFFFu) | 0x800000u;
        const int shift = -e - 14 + 13;  // bits to drop
        uint32_t q = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u)))
            ++q;
        return sign | uint16_t(q);
    }
    uint32_t q = ((uint32_t(e + 15)) << 10) | ((absu >> 13) & 0x3FFu);
    const uint32_t rem = absu & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u)))
        ++q;  // may carry into the exponent, which is the correct rounding
    return sign | uint16_t(q);
}

inline float to_f32(uint16_t h, int dtype) { return dtype == 0 ? bf16_to_f32(h) : f16_to_f32(h); }
inline uint16_t from_f32(float f, int dtype) { return dtype == 0 ? f32_to_bf16(f) : f32_to_f16(f); }

// splitmix64 (Steele, Lea & Flood 2014): the mixer the reference generator uses.
inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// One standard-normal value for element i (bench/bench_main.cpp:171-174), with the same
// sequence of float operations as the reference: u1, u2 in float; log(u1) rounded to float;
// times -2 (exact); square root rounded to float; cos(pi * 2*u2) rounded to float; product
// rounded to float. The two transcendental steps are evaluated in double precision and
// rounded once (correctly rounded in practice); the reference uses the device logf / cospif,
// which may differ by an ulp of float, so very rarely the 16-bit rounding of a value differs
// by one ulp (the golden test bounds how often).
// cos(pi * x) for x in [0, 2], in double, with an exact argument reduction so the result keeps
// full relative precision near the zeros of cos (x = 0.5, 1.5).
inline double cospi_0_2(double x) {
    double y = x > 1.0 ? 2.0 - x : x;  // cos(pi (2 - y)) = cos(pi y); exact
    if (y <= 0.25)
        return std::cos(M_PI * y);
    if (y <= 0.75)
        return std::sin(M_PI * (0.5 - y));  // 0.5 - y exact
    return -std::cos(M_PI * (1.0 - y));     // 1 - y exact
}

inline float randn_at(uint64_t seed, uint64_t i) {
    const uint64_t r = splitmix64(seed ^ (i * 0x2545F4914F6CDD1Dull));
    const float u1 = (float(r >> 40) + 1.0f) * (1.0f / 16777217.0f);
    const float u2 = float((r >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
    const float lg = float(std::log(double(u1)));
    const float mag = std::sqrt(-2.0f * lg);
    const float ang = float(cospi_0_2(double(2.0f * u2)));
    return mag * ang;
}

int pick_threads(int threads) {
    if (threads > 0)
        return threads;
    const unsigned hc = std::thread::hardware_concurrency();
    return hc ? int(hc) : 1;
}

template <typename F> void parallel_for(int64_t n, int threads, F &&fn) {
    threads = int(std::min<int64_t>(pick_threads(threads), std::max<int64_t>(n, 1)));
    if (threads <= 1) {
        for (int64_t i = 0; i < n; ++i)
            fn(i);
        return;
    }
    std::atomic<int64_t> next{0};
    std::vector<std::thread> pool;
    pool.reserve(threads);
    for (int t = 0; t < threads; ++t)
        pool.emplace_back([&] {
            for (int64_t i; (i = next.fetch_add(1)) < n;)
                fn(i);
        });
    for (auto &th : pool)
        th.join();
}

typedef float v8f __attribute__((vector_size(32)));

inline float hsum(v8f v) {
    float s = 0.f;
    for (int i = 0; i < 8; ++i)
        s += v[i];
    return s;
}

// out[r0:r0+4, c0:c0+4] = dot products over k (fp32 accumulate, 8-wide partial sums).
// a: 4 row pointers, b: 4 row pointers, both fp32, length k.
inline void dot4x4(const float *const *a, const float *const *b, int64_t k, float *acc) {
    v8f s[4][4];
    for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 4; ++j)
            s[i][j] = v8f{0, 0, 0, 0, 0, 0, 0, 0};
    int64_t kk = 0;
    for (; kk + 8 <= k; kk += 8) {
        v8f av[4], bv[4];
        for (int i = 0; i < 4; ++i)
            std::memcpy(&av[i], a[i] + kk, 32);
        for (int j = 0; j < 4; ++j)
            std::memcpy(&bv[j], b[j] + kk, 32);
        for (int i = 0; i < 4; ++i)
            for (int j = 0; j < 4; ++j)
                s[i][j] += av[i] * bv[j];
    }
    for (int i = 0; i < 4; ++i)
        for (int j = 0; j < 4; ++j) {
            float t = hsum(s[i][j]);
            for (int64_t q = kk; q < k; ++q)
                t += a[i][q] * b[j][q];
            acc[i * 4 + j] = t;
        }
}

}  // namespace

extern "C" {

int orc_version(void) { return 1; }

int orc_hw_threads(void) { return pick_threads(0); }

uint64_t orc_splitmix64(uint64_t x) { return splitmix64(x); }

float orc_randn_at(uint64_t seed, uint64_t i) { return randn_at(seed, i); }

uint16_t orc_f32_to_16(float f, int dtype) { return from_f32(f, dtype); }
float orc_16_to_f32(uint16_t h, int dtype) { return to_f32(h, dtype); }

// Bulk conversions (n elements).
void orc_to_f32(const uint16_t *in, float *out, int64_t n, int dtype) {
    for (int64_t i = 0; i < n; ++i)
        out[i] = to_f32(in[i], dtype);
}
void orc_from_f32(const float *in, uint16_t *out, int64_t n, int dtype) {
    for (int64_t i = 0; i < n; ++i)
        out[i] = from_f32(in[i], dtype);
}

// The reference input fill: element i of a tensor with `seed` (x uses seed 1, w seed 2,
// bench/bench_main.cpp:450-457), rounded to bf16/fp16.
void orc_fill_randn(uint16_t *out, int64_t n, uint64_t seed, int dtype, int threads) {
    const int64_t chunk = 1 << 16;
    const int64_t nchunks = (n + chunk - 1) / chunk;
    parallel_for(nchunks, threads, [&](int64_t c) {
        const int64_t lo = c * chunk, hi = std::min(n, lo + chunk);
        for (int64_t i = lo; i < hi; ++i)
            out[i] = from_f32(randn_at(seed, uint64_t(i)), dtype);
    });
}

// Full-output fp32 reference of the grouped GEMM, restricted to groups [g0, g1) and, inside
// each, to rows [0, min(M_g, max_rows)) (max_rows < 0 means all rows). Output rows are
// written at their global row (row_off[g] + r) of `out` ([sum(M), n] fp32).
// x: [sum(M), k], w: [G, n, k]; 16-bit patterns of `dtype`.
void orc_grouped_gemm_f32(const uint16_t *x, const uint16_t *w, float *out, int dtype,
                          int group_num, const int64_t *group_m, int64_t n, int64_t k,
                          int g0, int g1, int64_t max_rows, int threads) {
    std::vector<int64_t> row_off(group_num + 1, 0);
    for (int g = 0; g < group_num; ++g)
        row_off[g + 1] = row_off[g] + group_m[g];
    for (int g = g0; g < g1; ++g) {
        const int64_t m = max_rows < 0 ? group_m[g] : std::min(group_m[g], max_rows);
        if (m <= 0)
            continue;
        // Decode this group's operands once.
        std::vector<float> xf(size_t(m) * k), wf(size_t(n) * k);
        const uint16_t *xg = x + row_off[g] * k;
        const uint16_t *wg = w + int64_t(g) * n * k;
        parallel_for((m + 63) / 64, threads, [&](int64_t b) {
            for (int64_t i = b * 64 * k; i < std::min(m, (b + 1) * 64) * k; ++i)
                xf[i] = to_f32(xg[i], dtype);
        });
        parallel_for((n + 63) / 64, threads, [&](int64_t b) {
            for (int64_t i = b * 64 * k; i < std::min(n, (b + 1) * 64) * k; ++i)
                wf[i] = to_f32(wg[i], dtype);
        });
        // 4x4 register blocks; work items are 16-row x 64-column panels.
        const int64_t rb = (m + 15) / 16, cb = (n + 63) / 64;
        float *og = out + row_off[g] * n;
        parallel_for(rb * cb, threads, [&](int64_t item) {
            const int64_t r0 = (item / cb) * 16, c0 = (item % cb) * 64;
            for (int64_t r = r0; r < std::min(m, r0 + 16); r += 4)
                for (int64_t c = c0; c < std::min(n, c0 + 64); c += 4) {
                    const float *a[4], *b[4];
                    for (int i = 0; i < 4; ++i)
                        a[i] = &xf[size_t(std::min(r + i, m - 1)) * k];
                    for (int j = 0; j < 4; ++j)
                        b[j] = &wf[size_t(std::min(c + j, n - 1)) * k];
                    float acc[16];
                    dot4x4(a, b, k, acc);
                    for (int i = 0; i < 4 && r + i < m; ++i)
                        for (int j = 0; j < 4 && c + j < n; ++j)
                            og[(r + i) * n + (c + j)] = acc[i * 4 + j];
                }
        });
    }
}

// Per-group sample list of bench/bench_main.cpp:210-227: four corners, then 256 random
// (row, col) from one std::mt19937_64(1234) stream that runs across groups. Rows are global.
// Returns the number of samples (writes at most `cap`).
int64_t orc_make_samples(int group_num, const int64_t *group_m, int64_t n, int64_t *rows,
                         int64_t *cols, int64_t *groups, int64_t cap) {
    std::mt19937_64 rng(1234);
    int64_t cnt = 0, row0 = 0;
    auto push = [&](int64_t r, int64_t c, int64_t g) {
        if (cnt < cap) {
            rows[cnt] = r;
            cols[cnt] = c;
            groups[cnt] = g;
        }
        ++cnt;
    };
    for (int g = 0; g < group_num; ++g) {
        const int64_t m = group_m[g];
        if (m > 0) {
            for (int64_t r : {row0, row0 + m - 1})
                for (int64_t c : {int64_t(0), n - 1})
                    push(r, c, g);
            for (int i = 0; i < 256; ++i) {
                const int64_t r = row0 + int64_t(rng() % uint64_t(m));
                const int64_t c = int64_t(rng() % uint64_t(n));
                push(r, c, g);
            }
        }
        row0 += m;
    }
    return cnt;
}

// fp32 reference value of each sample in the reference kernel's own summation order
// (bench/bench_main.cpp:185-206): 256 lanes each accumulate elements i = lane, lane+256, ...
// with a fused multiply-add, then a pairwise tree (stride 128 ... 1) adds the partials.
void orc_sampled_ref(const uint16_t *x, const uint16_t *w, int dtype, int64_t n, int64_t k,
                     const int64_t *rows, const int64_t *cols, const int64_t *groups,
                     int64_t count, float *ref, int threads) {
    parallel_for(count, threads, [&](int64_t s) {
        const uint16_t *xr = x + rows[s] * k;
        const uint16_t *wr = w + (groups[s] * n + cols[s]) * k;
        float partial[256];
        for (int t = 0; t < 256; ++t) {
            float acc = 0.f;
            for (int64_t i = t; i < k; i += 256)
                acc = std::fmaf(to_f32(xr[i], dtype), to_f32(wr[i], dtype), acc);
            partial[t] = acc;
        }
        for (int stride = 128; stride > 0; stride /= 2)
            for (int t = 0; t < stride; ++t)
                partial[t] += partial[t + stride];
        ref[s] = partial[0];
    });
}

// Pass rule of bench/bench_main.cpp:263-270. Returns the number of mismatches; writes the
// max absolute error (NaN counts as +inf).
int64_t orc_check(const float *got, const float *ref, int64_t count, double *max_abs) {
    int64_t bad = 0;
    double mx = 0.0;
    for (int64_t i = 0; i < count; ++i) {
        const double err = std::fabs(double(got[i]) - double(ref[i]));
        mx = std::max(mx, std::isnan(err) ? INFINITY : err);
        if (!(err <= 1e-2 + 1e-2 * std::fabs(double(ref[i]))))
            ++bad;
    }
    if (max_abs)
        *max_abs = mx;
    return bad;
}

// Same rule over 16-bit outputs against an fp32 reference (full-output compare).
int64_t orc_check16(const uint16_t *got, const float *ref, int64_t count, int dtype,
                    double *max_abs, int64_t *first_bad) {
    int64_t bad = 0, first = -1;
    double mx = 0.0;
    for (int64_t i = 0; i < count; ++i) {
        const double g = to_f32(got[i], dtype);
        const double err = std::fabs(g - double(ref[i]));
        mx = std::max(mx, std::isnan(err) ? INFINITY : err);
        if (!(err <= 1e-2 + 1e-2 * std::fabs(double(ref[i])))) {
            if (first < 0)
                first = i;
            ++bad;
        }
    }
    if (max_abs)
        *max_abs = mx;
    if (first_bad)
        *first_bad = first;
    return bad;
}

}  // extern "C"
