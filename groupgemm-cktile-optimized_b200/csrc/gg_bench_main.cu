// gg_bench — grouped-GEMM benchmark harness with the reference's command line and CSV contract
// (bench/bench_main.cpp of the reference: shapes CSV in, results CSV out).
//
//   gg_bench --shapes FILE.csv [--dtype bf16|fp16] [--backends b200,cublas_loop,cublas_grouped]
//            [--only ID,...] [--warmup N] [--iters N] [--no-check] [--out FILE.csv] [--device N]
//            [--opt KEY=VALUE ...]
//
// --opt passes a gg_set_option knob to the b200 backend (variant, bn, split, split_tail, stream_k,
// sched, band, raster, store, pdl, max_ctas, timeout_ms): the runtime counterpart of editing the
// reference's compile-time CkTileConfig (ck_kernel/ck_grouped_gemm_config.hpp:26-86) between runs.
//
// What the contract fixes (and this file keeps): the flags above; balanced groups, B groups of M
// rows (bench/bench_main.cpp:436); inputs from the splitmix64 + Box-Muller generator with seeds 1
// (x) and 2 (w); the sample rule (four corners and 256 random elements per group,
// std::mt19937_64(1234)) and pass rule |got-ref| <= 1e-2 + 1e-2|ref| of the fp32 check; output
// zeroed before each backend; prepare untimed, then one checked run, `warmup` runs and CUDA
// events around `iters` back-to-back runs; the results CSV columns
// (TestID,Case,B,M,N,K,Dtype,GPU,Backend,Check,Time_ms,TFLOPS,MaxAbsErr,Detail) with one appended
// column (PctDensePeak, of 2250 TFLOPS), rewritten after every case; exit code 1 if any row is
// FAIL or ERROR. The rest (argument table, one device arena per run, the staged workload, the
// report object) is this harness's own.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <ctime>
#include <fstream>
#include <functional>
#include <iomanip>
#include <iostream>
#include <map>
#include <memory>
#include <random>
#include <set>
#include <sstream>
#include <string>
#include <vector>

#include "gg_backend.hpp"

namespace {

using gg::DType;
using gg::GroupedGemmProblem;

constexpr double kDenseBf16Tflops = 2250.0;  // B200 datasheet dense bf16/fp16 peak

// ================================ command line ================================

struct Options {
    std::string shapes, out;
    DType dtype = DType::BF16;
    std::vector<std::string> backends{"b200", "cublas_loop"};
    std::set<int> only;
    int warmup = 20, iters = 100, device = 0;
    bool check = true;
    std::vector<std::pair<std::string, int64_t>> b200_opts;  // --opt KEY=VALUE
};

const char *const kUsage =
    "usage: gg_bench --shapes FILE.csv [--dtype bf16|fp16] [--backends b200,cublas_loop,cublas_grouped]\n"
    "                [--only ID,...] [--warmup N] [--iters N] [--no-check] [--out FILE.csv] [--device N]\n"
    "                [--opt KEY=VALUE ...]   (b200 knobs: variant, bn, split, split_tail, band, raster,\n"
    "                                         stream_k, sched, store, pdl, max_ctas, timeout_ms)\n";

[[noreturn]] void usage_error(const std::string &msg) {
    std::cerr << "error: " << msg << "\n" << kUsage;
    std::exit(2);
}

// Comma-separated fields, trimmed; empty fields kept (a CSV row) or dropped (a flag's list).
std::vector<std::string> split_fields(const std::string &s, bool keep_empty) {
    std::vector<std::string> out;
    size_t at = 0;
    while (at <= s.size()) {
        const size_t end = std::min(s.find(',', at), s.size());
        const std::string f = s.substr(at, end - at);
        const size_t a = f.find_first_not_of(" \t\r"), b = f.find_last_not_of(" \t\r");
        if (a != std::string::npos)
            out.push_back(f.substr(a, b - a + 1));
        else if (keep_empty)
            out.emplace_back();
        at = end + 1;
    }
    return out;
}
std::vector<std::string> fields(const std::string &s) { return split_fields(s, false); }

int to_int(const std::string &flag, const std::string &v) {
    try {
        size_t used = 0;
        const int x = std::stoi(v, &used);
        if (used == v.size())
            return x;
    } catch (const std::exception &) {
    }
    usage_error(flag + " wants an integer, got '" + v + "'");
}

// One entry per flag: whether it takes a value, and what it does to the options.
struct Flag {
    const char *name;
    bool has_value;
    std::function<void(Options &, const std::string &)> apply;
};

const std::vector<Flag> &flag_table() {
    static const std::vector<Flag> t = {
        {"--shapes", true, [](Options &o, const std::string &v) { o.shapes = v; }},
        {"--out", true, [](Options &o, const std::string &v) { o.out = v; }},
        {"--dtype", true,
         [](Options &o, const std::string &v) {
             if (v != "bf16" && v != "fp16")
                 usage_error("--dtype must be bf16 or fp16");
             o.dtype = v == "bf16" ? DType::BF16 : DType::FP16;
         }},
        {"--backends", true, [](Options &o, const std::string &v) { o.backends = fields(v); }},
        {"--only", true,
         [](Options &o, const std::string &v) {
             for (const auto &id : fields(v))
                 o.only.insert(to_int("--only", id));
         }},
        {"--warmup", true, [](Options &o, const std::string &v) { o.warmup = to_int("--warmup", v); }},
        {"--iters", true, [](Options &o, const std::string &v) { o.iters = to_int("--iters", v); }},
        {"--device", true, [](Options &o, const std::string &v) { o.device = to_int("--device", v); }},
        {"--no-check", false, [](Options &o, const std::string &) { o.check = false; }},
        {"--opt", true,
         [](Options &o, const std::string &kv) {
             const size_t eq = kv.find('=');
             if (eq == std::string::npos || eq == 0)
                 usage_error("--opt wants KEY=VALUE, got " + kv);
             try {
                 size_t used = 0;
                 const std::string v = kv.substr(eq + 1);
                 const long long x = std::stoll(v, &used);
                 if (used != v.size())
                     throw std::invalid_argument(v);
                 o.b200_opts.emplace_back(kv.substr(0, eq), x);
             } catch (const std::exception &) {
                 usage_error("--opt value is not an integer: " + kv);
             }
         }},
        {"--help", false, [](Options &, const std::string &) { usage_error("help requested"); }},
        {"-h", false, [](Options &, const std::string &) { usage_error("help requested"); }},
    };
    return t;
}

Options parse_args(int argc, char **argv) {
    Options o;
    const auto &table = flag_table();
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        const auto f = std::find_if(table.begin(), table.end(), [&](const Flag &x) { return a == x.name; });
        if (f == table.end())
            usage_error("unknown argument " + a);
        std::string v;
        if (f->has_value) {
            if (i + 1 >= argc)
                usage_error("missing value for " + a);
            v = argv[++i];
        }
        f->apply(o, v);
    }
    if (o.shapes.empty())
        usage_error("--shapes is required");
    if (o.iters < 1 || o.warmup < 0)
        usage_error("--iters must be >= 1 and --warmup >= 0");
    return o;
}

// ================================ shapes CSV ================================

struct Case {
    int id = 0;
    std::string name;
    int64_t b = 0, m = 0, n = 0, k = 0;
    double flops() const { return 2.0 * double(b) * double(m) * double(n) * double(k); }
};

// Columns are found by name, so a results CSV (one row per backend) also reads as a shapes file;
// a TestID seen before is skipped.
std::vector<Case> read_shapes(const std::string &path, const std::set<int> &only) {
    std::ifstream f(path);
    if (!f)
        usage_error("cannot open " + path);
    std::string line;
    std::getline(f, line);
    const auto head = split_fields(line, true);
    auto column = [&](const char *name) {
        const auto it = std::find(head.begin(), head.end(), name);
        if (it == head.end())
            usage_error(path + ": missing column " + name);
        return size_t(it - head.begin());
    };
    const size_t c_id = column("TestID"), c_name = column("Case"), c_b = column("B"), c_m = column("M"),
                 c_n = column("N"), c_k = column("K");
    std::vector<Case> cases;
    std::set<int> seen;
    const size_t need = std::max({c_id, c_name, c_b, c_m, c_n, c_k}) + 1;
    while (std::getline(f, line)) {
        const auto v = split_fields(line, true);
        if (v.size() < need || v[c_id].empty())
            continue;
        Case c{std::stoi(v[c_id]), v[c_name], std::stoll(v[c_b]), std::stoll(v[c_m]), std::stoll(v[c_n]),
               std::stoll(v[c_k])};
        if ((only.empty() || only.count(c.id)) && seen.insert(c.id).second)
            cases.push_back(c);
    }
    return cases;
}

// ================================ device side ================================

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

template <typename T> __device__ T to16(float v);
template <> __device__ __nv_bfloat16 to16(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __half to16(float v) { return __float2half_rn(v); }
__device__ __forceinline__ float from16(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float from16(__half v) { return __half2float(v); }

// N(0,1) values, deterministic in (seed, index): splitmix64 -> two uniforms -> Box-Muller.
template <typename T> __global__ void fill_normal(T *p, size_t n, uint64_t seed) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
        const uint64_t r = mix64(seed ^ (i * 0x2545F4914F6CDD1Dull));
        const float u1 = (float(r >> 40) + 1.0f) * (1.0f / 16777217.0f);
        const float u2 = float((r >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
        p[i] = to16<T>(sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2));
    }
}

struct Pos {
    int64_t row, col, group;
};

// One warp per sampled element: fp32 dot of x[row, :] and w[group][col, :], and the output value.
template <typename T>
__global__ void sample_dots(const T *x, const T *w, const T *out, int64_t n, int64_t k, const Pos *pos, int64_t count,
                            float2 *ref_got) {
    const int64_t s = blockIdx.x * int64_t(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    if (s >= count)
        return;
    const Pos q = pos[s];
    const T *xr = x + q.row * k;
    const T *wr = w + (q.group * n + q.col) * k;
    float acc = 0.f;
    for (int64_t i = lane; i < k; i += 32)
        acc += from16(xr[i]) * from16(wr[i]);
    for (int off = 16; off > 0; off /= 2)
        acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0)
        ref_got[s] = make_float2(acc, from16(out[q.row * n + q.col]));
}

// ================================ workload staging ================================

// One device allocation per run, carved into x | w | out | sample positions | sample results
// (256-byte aligned parts) and grown when a case needs more; plus the pinned group lengths.
class Workspace {
public:
    ~Workspace() {
        if (base_)
            cudaFree(base_);
        if (lens_)
            cudaFreeHost(lens_);
    }

    // Device parts of the given sizes, in order.
    std::vector<void *> carve(const std::vector<size_t> &sizes) {
        size_t total = 0;
        std::vector<size_t> at;
        for (size_t s : sizes) {
            at.push_back(total);
            total += (s + 255) / 256 * 256;
        }
        if (total > cap_) {
            if (base_)
                GG_CUDA_CHECK(cudaFree(base_));
            base_ = nullptr;
            cap_ = 0;
            GG_CUDA_CHECK(cudaMalloc(&base_, total));
            cap_ = total;
        }
        std::vector<void *> parts;
        for (size_t a : at)
            parts.push_back(static_cast<char *>(base_) + a);
        return parts;
    }

    int64_t *pinned_lens(const std::vector<int64_t> &lens) {
        if (lens.size() > lens_cap_) {
            if (lens_)
                GG_CUDA_CHECK(cudaFreeHost(lens_));
            lens_ = nullptr;
            GG_CUDA_CHECK(cudaMallocHost(&lens_, lens.size() * sizeof(int64_t)));
            lens_cap_ = lens.size();
        }
        std::copy(lens.begin(), lens.end(), lens_);
        return lens_;
    }

private:
    void *base_ = nullptr;
    size_t cap_ = 0;
    int64_t *lens_ = nullptr;
    size_t lens_cap_ = 0;
};

// One case on the device: the problem the backends see, and what the check needs.
struct Workload {
    GroupedGemmProblem p;
    size_t out_bytes = 0;
    std::vector<Pos> samples;
    Pos *d_samples = nullptr;
    float2 *d_results = nullptr;
};

// The reference's sample rule: per non-empty group its four corners, then 256 random
// (row, column) pairs from std::mt19937_64(1234) (row first), in group order.
std::vector<Pos> sample_rule(const GroupedGemmProblem &p) {
    std::mt19937_64 rng(1234);
    std::vector<Pos> s;
    int64_t row0 = 0;
    for (int g = 0; g < p.group_num; ++g) {
        const int64_t m = p.group_m[size_t(g)];
        if (m > 0) {
            for (int64_t r : {row0, row0 + m - 1})
                for (int64_t c : {int64_t(0), p.n - 1})
                    s.push_back({r, c, g});
            for (int i = 0; i < 256; ++i) {
                const int64_t r = row0 + int64_t(rng() % uint64_t(m));
                const int64_t c = int64_t(rng() % uint64_t(p.n));
                s.push_back({r, c, g});
            }
        }
        row0 += m;
    }
    return s;
}

template <typename T> void fill_inputs(const GroupedGemmProblem &p, cudaStream_t stream) {
    fill_normal<T><<<4096, 256, 0, stream>>>(static_cast<T *>(const_cast<void *>(p.x)), size_t(p.total_m()) * p.k, 1);
    fill_normal<T><<<4096, 256, 0, stream>>>(static_cast<T *>(const_cast<void *>(p.w)),
                                             size_t(p.group_num) * p.n * p.k, 2);
    GG_CUDA_CHECK(cudaGetLastError());
}

Workload stage(const Case &c, DType dt, Workspace &ws, cudaStream_t stream) {
    Workload wl;
    GroupedGemmProblem &p = wl.p;
    p.dtype = dt;
    p.group_num = int(c.b);
    p.n = c.n;
    p.k = c.k;
    p.group_m.assign(size_t(c.b), c.m);
    wl.samples = sample_rule(p);
    const size_t es = gg::dtype_bytes(dt);
    wl.out_bytes = size_t(p.total_m()) * size_t(p.n) * es;
    const auto parts = ws.carve({size_t(p.total_m()) * size_t(p.k) * es, size_t(p.group_num) * size_t(p.n) * size_t(p.k) * es,
                                 wl.out_bytes, wl.samples.size() * sizeof(Pos), wl.samples.size() * sizeof(float2)});
    p.x = parts[0];
    p.w = parts[1];
    p.out = parts[2];
    wl.d_samples = static_cast<Pos *>(parts[3]);
    wl.d_results = static_cast<float2 *>(parts[4]);
    p.group_lens_pinned = ws.pinned_lens(p.group_m);
    if (dt == DType::BF16)
        fill_inputs<__nv_bfloat16>(p, stream);
    else
        fill_inputs<__half>(p, stream);
    GG_CUDA_CHECK(cudaMemcpyAsync(wl.d_samples, wl.samples.data(), wl.samples.size() * sizeof(Pos),
                                  cudaMemcpyHostToDevice, stream));
    return wl;
}

// ================================ check and timing ================================

struct Verdict {
    int64_t off = 0;      // samples outside the tolerance (NaN counts)
    double max_abs = 0.0;  // largest |got - ref| (infinite for NaN)
};

template <typename T> void launch_sample_dots(const Workload &wl, cudaStream_t stream) {
    const int64_t ns = int64_t(wl.samples.size());
    constexpr int kWarps = 8;
    sample_dots<T><<<unsigned((ns + kWarps - 1) / kWarps), kWarps * 32, 0, stream>>>(
        static_cast<const T *>(wl.p.x), static_cast<const T *>(wl.p.w), static_cast<const T *>(wl.p.out), wl.p.n,
        wl.p.k, wl.d_samples, ns, wl.d_results);
    GG_CUDA_CHECK(cudaGetLastError());
}

Verdict check_output(const Workload &wl, cudaStream_t stream) {
    if (wl.samples.empty())
        return Verdict{};  // every group empty: nothing to compare
    if (wl.p.dtype == DType::BF16)
        launch_sample_dots<__nv_bfloat16>(wl, stream);
    else
        launch_sample_dots<__half>(wl, stream);
    std::vector<float2> rg(wl.samples.size());
    GG_CUDA_CHECK(cudaMemcpyAsync(rg.data(), wl.d_results, rg.size() * sizeof(float2), cudaMemcpyDeviceToHost, stream));
    GG_CUDA_CHECK(cudaStreamSynchronize(stream));
    Verdict v;
    for (const float2 &x : rg) {
        const double err = std::fabs(double(x.y) - double(x.x));
        const bool ok = err <= 1e-2 + 1e-2 * std::fabs(double(x.x));  // false for NaN
        v.off += ok ? 0 : 1;
        v.max_abs = std::max(v.max_abs, std::isnan(err) ? double(INFINITY) : err);
    }
    return v;
}

// CUDA events around `iters` back-to-back calls on one stream: mean milliseconds per call.
class Stopwatch {
public:
    Stopwatch() {
        GG_CUDA_CHECK(cudaEventCreate(&a_));
        GG_CUDA_CHECK(cudaEventCreate(&b_));
    }
    ~Stopwatch() {
        cudaEventDestroy(a_);
        cudaEventDestroy(b_);
    }
    double mean_ms(const std::function<void()> &call, int iters, cudaStream_t stream) {
        GG_CUDA_CHECK(cudaEventRecord(a_, stream));
        for (int i = 0; i < iters; ++i)
            call();
        GG_CUDA_CHECK(cudaEventRecord(b_, stream));
        GG_CUDA_CHECK(cudaEventSynchronize(b_));
        GG_CUDA_CHECK(cudaGetLastError());
        float ms = 0.f;
        GG_CUDA_CHECK(cudaEventElapsedTime(&ms, a_, b_));
        return double(ms) / iters;
    }

private:
    cudaEvent_t a_{}, b_{};
};

struct Result {
    Case c;
    std::string backend, check, detail;
    double ms = NAN, tflops = NAN, max_abs = NAN;
};

// One backend on one staged case: prepare (untimed; a reason means N/A), one run that the fp32
// sample check and the device status judge, warm-up, then the timed runs.
Result evaluate(gg::Backend &be, const Case &c, Workload &wl, const Options &opt, Stopwatch &sw, cudaStream_t stream) {
    Result r{c, be.name(), "ERROR", "", NAN, NAN, NAN};
    try {
        GG_CUDA_CHECK(cudaMemsetAsync(wl.p.out, 0, wl.out_bytes, stream));  // an idle backend must fail
        const std::string why = be.prepare(wl.p, stream);
        if (!why.empty()) {
            r.check = "N/A";
            r.detail = why;
            be.release();
            return r;
        }
        r.detail = be.detail();
        be.run(stream);
        GG_CUDA_CHECK(cudaGetLastError());
        GG_CUDA_CHECK(cudaStreamSynchronize(stream));
        const uint32_t status = be.device_status(stream);
        bool good = status == 0;
        if (opt.check) {
            const Verdict v = check_output(wl, stream);
            r.max_abs = v.max_abs;
            good = good && v.off == 0;
            if (v.off)
                r.detail += " | " + std::to_string(v.off) + "/" + std::to_string(wl.samples.size()) + " samples off";
        }
        if (status)
            r.detail += " | device status " + std::to_string(status);
        r.check = !good ? "FAIL" : opt.check ? "PASS" : "SKIP";
        auto call = [&] { be.run(stream); };
        for (int i = 0; i < opt.warmup; ++i)
            call();
        r.ms = sw.mean_ms(call, opt.iters, stream);
        r.tflops = wl.p.flops() / (r.ms * 1e-3) / 1e12;
    } catch (const std::exception &ex) {
        (void)cudaStreamSynchronize(stream);
        r.check = "ERROR";
        r.detail = ex.what();
    }
    be.release();
    return r;
}

// ================================ report ================================

class Report {
public:
    Report(std::string path, std::string gpu, DType dt) : path_(std::move(path)), gpu_(std::move(gpu)), dt_(dt) {}

    void add(const Result &r) {
        rows_.push_back(r);
        std::ostringstream line;
        line << "  " << std::left << std::setw(16) << r.backend << std::setw(6) << r.check << std::right << std::fixed;
        if (std::isnan(r.ms))
            line << std::setw(12) << "-" << std::setw(14) << "-";
        else
            line << std::setprecision(3) << std::setw(10) << r.ms << " ms" << std::setprecision(1) << std::setw(9)
                 << r.tflops << " TFLOPS";
        std::cout << line.str() << "  " << r.detail.substr(0, 100) << "\n";
    }

    // Rewrites the whole CSV (called after every case, so a crash keeps what finished).
    void save() const {
        std::ofstream f(path_);
        if (!f) {
            std::cerr << "error: cannot write " << path_ << "\n";
            std::exit(1);
        }
        f << "TestID,Case,B,M,N,K,Dtype,GPU,Backend,Check,Time_ms,TFLOPS,MaxAbsErr,Detail,PctDensePeak\n";
        for (const auto &r : rows_) {
            std::vector<std::string> col = {std::to_string(r.c.id), r.c.name, std::to_string(r.c.b),
                                            std::to_string(r.c.m), std::to_string(r.c.n), std::to_string(r.c.k),
                                            gg::dtype_name(dt_), csv_text(gpu_), r.backend, r.check,
                                            fixed(r.ms, 4), fixed(r.tflops, 2), fixed(r.max_abs, 4),
                                            csv_text(r.detail), fixed(100.0 * r.tflops / kDenseBf16Tflops, 2)};
            for (size_t i = 0; i < col.size(); ++i)
                f << (i ? "," : "") << col[i];
            f << "\n";
        }
    }

    // Over the cases that every backend PASSed: per backend the summed time, the mean TFLOPS (and
    // its share of the 2250 TFLOPS dense peak) and the geometric mean of its time over the first
    // backend's.
    void print_summary(const std::vector<std::string> &backends) const {
        std::map<int, std::map<std::string, const Result *>> by_case;
        for (const auto &r : rows_)
            by_case[r.c.id][r.backend] = &r;
        std::vector<const std::map<std::string, const Result *> *> common;
        for (const auto &kv : by_case) {
            const auto &m = kv.second;
            const bool all_pass = m.size() == backends.size() &&
                                  std::all_of(m.begin(), m.end(), [](const auto &e) { return e.second->check == "PASS"; });
            if (all_pass)
                common.push_back(&m);
        }
        std::cout << "\n==== Summary over " << common.size() << " of " << by_case.size()
                  << " cases where all backends passed ====\n";
        if (common.empty())
            return;
        const std::string &base = backends.front();
        std::printf("%-18s%12s%14s%12s%24s\n", "backend", "sum ms", "mean TFLOPS", "% 2250",
                    ("geomean time / " + base).c_str());
        for (const auto &b : backends) {
            double ms = 0, tf = 0, log_ratio = 0;
            for (const auto *m : common) {
                const Result *r = m->at(b);
                ms += r->ms;
                tf += r->tflops;
                log_ratio += std::log(r->ms / m->at(base)->ms);
            }
            const double n = double(common.size());
            std::printf("%-18s%12.3f%14.1f%12.1f%23.3fx\n", b.c_str(), ms, tf / n, 100.0 * tf / n / kDenseBf16Tflops,
                        std::exp(log_ratio / n));
        }
    }

    bool any_failed() const {
        return std::any_of(rows_.begin(), rows_.end(), [](const Result &r) { return r.check == "FAIL" || r.check == "ERROR"; });
    }

    const std::string &path() const { return path_; }

private:
    static std::string csv_text(const std::string &s) {
        std::string q = "\"";
        for (char ch : s) {
            if (ch == '"')
                q += '"';
            q += ch;
        }
        return q + "\"";
    }
    static std::string fixed(double v, int digits) {
        if (std::isnan(v))
            return "";
        char buf[64];
        std::snprintf(buf, sizeof(buf), "%.*f", digits, v);
        return buf;
    }

    std::string path_, gpu_;
    DType dt_;
    std::vector<Result> rows_;
};

std::string default_results_path(const Options &opt) {
    std::string stem = opt.shapes.substr(opt.shapes.find_last_of('/') + 1);
    stem = stem.substr(0, stem.find_last_of('.'));
    char ts[32];
    const std::time_t now = std::time(nullptr);
    std::strftime(ts, sizeof(ts), "%Y%m%d-%H%M%S", std::localtime(&now));
    return "results_" + stem + "_" + gg::dtype_name(opt.dtype) + "_" + ts + ".csv";
}

std::unique_ptr<gg::Backend> make_backend(const std::string &name, const Options &opt) {
    if (name == "b200") {
        auto b = std::make_unique<gg::B200Backend>();
        for (const auto &kv : opt.b200_opts)
            b->set_option(kv.first.c_str(), kv.second);  // throws on an unknown key or bad value
        return b;
    }
    if (name == "cublas_loop")
        return gg::make_cublas_loop_backend();
    if (name == "cublas_grouped")
        return gg::make_cublas_grouped_backend();
    usage_error("unknown backend " + name);
}

int run(const Options &opt) {
    GG_CUDA_CHECK(cudaSetDevice(opt.device));
    cudaDeviceProp prop;
    GG_CUDA_CHECK(cudaGetDeviceProperties(&prop, opt.device));
    const std::string gpu = std::string(prop.name) + " (sm_" + std::to_string(prop.major) + std::to_string(prop.minor) + ")";
    std::vector<std::unique_ptr<gg::Backend>> backends;
    for (const auto &b : opt.backends)
        backends.push_back(make_backend(b, opt));
    const std::vector<Case> cases = read_shapes(opt.shapes, opt.only);
    Report report(opt.out.empty() ? default_results_path(opt) : opt.out, gpu, opt.dtype);
    std::cout << "GPU: " << gpu << "\nshapes: " << opt.shapes << " (" << cases.size() << " cases), dtype "
              << gg::dtype_name(opt.dtype) << ", warmup " << opt.warmup << ", iters " << opt.iters << "\n";

    cudaStream_t stream;
    GG_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    {
        Workspace ws;
        Stopwatch sw;
        for (const Case &c : cases) {
            Workload wl = stage(c, opt.dtype, ws, stream);
            std::cout << "\n[" << c.id << "] " << c.name << "  B=" << c.b << " M=" << c.m << " N=" << c.n
                      << " K=" << c.k << "  (" << std::setprecision(3) << c.flops() / 1e12 << " TFLOP)\n";
            for (auto &be : backends)
                report.add(evaluate(*be, c, wl, opt, sw, stream));
            report.save();
        }
    }
    report.print_summary(opt.backends);
    std::cout << "\nresults: " << report.path() << "\n";
    cudaStreamDestroy(stream);
    return report.any_failed() ? 1 : 0;
}

}  // namespace

int main(int argc, char **argv) {
    try {
        return run(parse_args(argc, argv));
    } catch (const std::exception &e) {
        std::cerr << "fatal: " << e.what() << "\n";
        return 1;
    }
}
