// gg_bench — grouped-GEMM benchmark harness with the reference's command line and CSV contract
// (bench/bench_main.cpp of the reference: shapes CSV in, results CSV out).
//
//   gg_bench --shapes FILE.csv [--dtype bf16|fp16] [--backends b200,cublas_loop,cublas_grouped]
//            [--only ID,...] [--warmup N] [--iters N] [--no-check] [--out FILE.csv] [--device N]
//            [--opt KEY=VALUE ...]
//
// --opt passes a gg_set_option knob to the b200 backend (variant, bn, split, split_tail, stream_k,
// band, raster, store, pdl, max_ctas, timeout_ms): the runtime counterpart of editing the reference's
// compile-time CkTileConfig (ck_kernel/ck_grouped_gemm_config.hpp:26-86) between runs.
//
// Per case (balanced groups: B groups of M rows, like the reference, bench/bench_main.cpp:436):
// device inputs from the splitmix64 + Box-Muller generator (seeds 1 and 2), output zeroed, then
// per backend prepare (untimed), one run + sampled fp32 check (four corners and 256 random
// elements per group, std::mt19937_64(1234); |got-ref| <= 1e-2 + 1e-2|ref|), warm-up, and
// CUDA events around `iters` back-to-back runs. Results CSV columns are the reference's
// (TestID,Case,B,M,N,K,Dtype,GPU,Backend,Check,Time_ms,TFLOPS,MaxAbsErr,Detail) followed by
// PctDensePeak (of 2250 TFLOPS). The file is rewritten after every case. Exit code 1 if any
// row is FAIL or ERROR.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <ctime>
#include <fstream>
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

struct Options {
    std::string shapes, out;
    DType dtype = DType::BF16;
    std::vector<std::string> backends{"b200", "cublas_loop"};
    std::set<int> only;
    int warmup = 20, iters = 100, device = 0;
    bool check = true;
    std::vector<std::pair<std::string, int64_t>> b200_opts;  // --opt KEY=VALUE
};

std::vector<std::string> split_list(const std::string &s, char sep) {
    std::vector<std::string> out;
    std::string cur;
    std::stringstream ss(s);
    while (std::getline(ss, cur, sep)) {
        cur.erase(cur.find_last_not_of(" \r\t") + 1);
        cur.erase(0, cur.find_first_not_of(" \t"));
        if (!cur.empty())
            out.push_back(cur);
    }
    return out;
}

[[noreturn]] void die_usage(const std::string &msg) {
    std::cerr << "error: " << msg << "\n"
              << "usage: gg_bench --shapes FILE.csv [--dtype bf16|fp16] [--backends b200,cublas_loop,cublas_grouped]\n"
              << "                [--only ID,...] [--warmup N] [--iters N] [--no-check] [--out FILE.csv] [--device N]\n"
              << "                [--opt KEY=VALUE ...]   (b200 knobs: variant, bn, split, split_tail, band, raster,\n"
              << "                                         stream_k, store, pdl, max_ctas, timeout_ms)\n";
    std::exit(2);
}

Options parse(int argc, char **argv) {
    Options o;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        auto value = [&]() -> std::string {
            if (i + 1 >= argc)
                die_usage("missing value for " + a);
            return argv[++i];
        };
        if (a == "--shapes")
            o.shapes = value();
        else if (a == "--out")
            o.out = value();
        else if (a == "--dtype") {
            const std::string d = value();
            if (d != "bf16" && d != "fp16")
                die_usage("--dtype must be bf16 or fp16");
            o.dtype = d == "bf16" ? DType::BF16 : DType::FP16;
        } else if (a == "--backends")
            o.backends = split_list(value(), ',');
        else if (a == "--only")
            for (const auto &id : split_list(value(), ','))
                o.only.insert(std::stoi(id));
        else if (a == "--warmup")
            o.warmup = std::stoi(value());
        else if (a == "--iters")
            o.iters = std::stoi(value());
        else if (a == "--device")
            o.device = std::stoi(value());
        else if (a == "--no-check")
            o.check = false;
        else if (a == "--opt") {
            const std::string kv = value();
            const size_t eq = kv.find('=');
            if (eq == std::string::npos || eq == 0)
                die_usage("--opt wants KEY=VALUE, got " + kv);
            try {
                o.b200_opts.emplace_back(kv.substr(0, eq), std::stoll(kv.substr(eq + 1)));
            } catch (const std::exception &) {
                die_usage("--opt value is not an integer: " + kv);
            }
        }
        else if (a == "-h" || a == "--help")
            die_usage("help requested");
        else
            die_usage("unknown argument " + a);
    }
    if (o.shapes.empty())
        die_usage("--shapes is required");
    if (o.iters < 1 || o.warmup < 0)
        die_usage("--iters must be >= 1 and --warmup >= 0");
    return o;
}

struct Case {
    int id = 0;
    std::string name;
    int64_t b = 0, m = 0, n = 0, k = 0;
};

std::vector<Case> load_cases(const std::string &path) {
    std::ifstream f(path);
    if (!f)
        die_usage("cannot open " + path);
    std::string line;
    std::getline(f, line);
    const auto head = split_list(line, ',');
    std::map<std::string, size_t> col;
    for (size_t i = 0; i < head.size(); ++i)
        col[head[i]] = i;
    for (const char *c : {"TestID", "Case", "B", "M", "N", "K"})
        if (!col.count(c))
            die_usage(path + ": missing column " + c);
    std::vector<Case> cases;
    while (std::getline(f, line)) {
        const auto v = split_list(line, ',');
        if (v.size() < head.size())
            continue;
        cases.push_back({std::stoi(v[col["TestID"]]), v[col["Case"]], std::stoll(v[col["B"]]), std::stoll(v[col["M"]]),
                         std::stoll(v[col["N"]]), std::stoll(v[col["K"]])});
    }
    return cases;
}

// ---- device helpers: input fill and sampled fp32 check ----
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

// One warp per sampled element: fp32 dot of x[row, :] and w[group][col, :].
template <typename T>
__global__ void sample_dots(const T *x, const T *w, const T *out, int64_t n, int64_t k, const Pos *pos, int64_t count,
                            float *ref, float *got) {
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
    if (lane == 0) {
        ref[s] = acc;
        got[s] = from16(out[q.row * n + q.col]);
    }
}

std::vector<Pos> sample_positions(const GroupedGemmProblem &p) {
    std::mt19937_64 rng(1234);
    std::vector<Pos> s;
    int64_t row0 = 0;
    for (int g = 0; g < p.group_num; ++g) {
        const int64_t m = p.group_m[g];
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

struct CheckOut {
    bool pass = false;
    double max_abs = 0.0;
    int64_t bad = 0;
};

template <typename T>
CheckOut check_samples(const GroupedGemmProblem &p, const std::vector<Pos> &pos, cudaStream_t stream) {
    const int64_t ns = int64_t(pos.size());
    Pos *d_pos = nullptr;
    float *d_ref = nullptr, *d_got = nullptr;
    GG_CUDA_CHECK(cudaMalloc(&d_pos, ns * sizeof(Pos)));
    GG_CUDA_CHECK(cudaMalloc(&d_ref, ns * sizeof(float)));
    GG_CUDA_CHECK(cudaMalloc(&d_got, ns * sizeof(float)));
    GG_CUDA_CHECK(cudaMemcpyAsync(d_pos, pos.data(), ns * sizeof(Pos), cudaMemcpyHostToDevice, stream));
    const int warps = 8;
    sample_dots<T><<<unsigned((ns + warps - 1) / warps), warps * 32, 0, stream>>>(
        static_cast<const T *>(p.x), static_cast<const T *>(p.w), static_cast<const T *>(p.out), p.n, p.k, d_pos, ns,
        d_ref, d_got);
    GG_CUDA_CHECK(cudaGetLastError());
    std::vector<float> ref(ns), got(ns);
    GG_CUDA_CHECK(cudaMemcpyAsync(ref.data(), d_ref, ns * sizeof(float), cudaMemcpyDeviceToHost, stream));
    GG_CUDA_CHECK(cudaMemcpyAsync(got.data(), d_got, ns * sizeof(float), cudaMemcpyDeviceToHost, stream));
    GG_CUDA_CHECK(cudaStreamSynchronize(stream));
    cudaFree(d_pos);
    cudaFree(d_ref);
    cudaFree(d_got);
    CheckOut c;
    for (int64_t i = 0; i < ns; ++i) {
        const double err = std::fabs(double(got[i]) - double(ref[i]));
        c.max_abs = std::max(c.max_abs, std::isnan(err) ? INFINITY : err);
        if (!(err <= 1e-2 + 1e-2 * std::fabs(double(ref[i]))))
            ++c.bad;
    }
    c.pass = c.bad == 0;
    return c;
}

struct Buffer {
    void *p = nullptr;
    size_t bytes = 0;
    void *need(size_t n) {
        if (n > bytes) {
            if (p)
                GG_CUDA_CHECK(cudaFree(p));
            p = nullptr;
            GG_CUDA_CHECK(cudaMalloc(&p, n));
            bytes = n;
        }
        return p;
    }
    ~Buffer() {
        if (p)
            cudaFree(p);
    }
};

struct Result {
    Case c;
    std::string backend, check, detail;
    double ms = NAN, tflops = NAN, max_abs = NAN;
};

std::string quoted(const std::string &s) {
    std::string q = "\"";
    for (char ch : s)
        q += ch == '"' ? std::string("\"\"") : std::string(1, ch);
    return q + "\"";
}

void save_csv(const std::string &path, const std::vector<Result> &rows, const std::string &gpu, DType dt) {
    std::ofstream f(path);
    if (!f) {
        std::cerr << "error: cannot write " << path << "\n";
        std::exit(1);
    }
    f << "TestID,Case,B,M,N,K,Dtype,GPU,Backend,Check,Time_ms,TFLOPS,MaxAbsErr,Detail,PctDensePeak\n" << std::fixed;
    for (const auto &r : rows) {
        f << r.c.id << ',' << r.c.name << ',' << r.c.b << ',' << r.c.m << ',' << r.c.n << ',' << r.c.k << ','
          << gg::dtype_name(dt) << ',' << quoted(gpu) << ',' << r.backend << ',' << r.check << ',';
        if (std::isnan(r.ms))
            f << ",,";
        else
            f << std::setprecision(4) << r.ms << ',' << std::setprecision(2) << r.tflops << ',';
        if (!std::isnan(r.max_abs))
            f << std::setprecision(4) << r.max_abs;
        f << ',' << quoted(r.detail) << ',';
        if (!std::isnan(r.tflops))
            f << std::setprecision(2) << 100.0 * r.tflops / kDenseBf16Tflops;
        f << '\n';
    }
}

// Mean over the cases every backend passed, and geometric-mean time ratio to the first backend.
void summary(const std::vector<Result> &rows, const std::vector<std::string> &names) {
    std::map<int, std::map<std::string, const Result *>> by_case;
    for (const auto &r : rows)
        by_case[r.c.id][r.backend] = &r;
    std::vector<int> common;
    for (const auto &[id, m] : by_case) {
        bool all = m.size() == names.size();
        for (const auto &[b, r] : m)
            all = all && r->check == "PASS";
        if (all)
            common.push_back(id);
    }
    std::cout << "\n==== Summary over " << common.size() << " of " << by_case.size()
              << " cases where all backends passed ====\n";
    if (common.empty())
        return;
    const std::string first = names.front();
    std::cout << std::left << std::setw(18) << "backend" << std::right << std::setw(12) << "sum ms" << std::setw(14)
              << "mean TFLOPS" << std::setw(12) << "% 2250" << std::setw(24) << ("geomean time / " + first) << "\n";
    for (const auto &b : names) {
        double ms = 0, tf = 0, lr = 0;
        for (int id : common) {
            const Result *r = by_case[id][b];
            ms += r->ms;
            tf += r->tflops;
            lr += std::log(r->ms / by_case[id][first]->ms);
        }
        const double mean_tf = tf / common.size();
        std::cout << std::left << std::setw(18) << b << std::right << std::fixed << std::setprecision(3)
                  << std::setw(12) << ms << std::setprecision(1) << std::setw(14) << mean_tf << std::setw(12)
                  << 100.0 * mean_tf / kDenseBf16Tflops << std::setprecision(3) << std::setw(23)
                  << std::exp(lr / common.size()) << "x\n";
    }
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
    die_usage("unknown backend " + name);
}

int run(const Options &opt) {
    GG_CUDA_CHECK(cudaSetDevice(opt.device));
    cudaDeviceProp prop;
    GG_CUDA_CHECK(cudaGetDeviceProperties(&prop, opt.device));
    const std::string gpu = std::string(prop.name) + " (sm_" + std::to_string(prop.major) + std::to_string(prop.minor) + ")";

    std::vector<std::unique_ptr<gg::Backend>> backends;
    for (const auto &b : opt.backends)
        backends.push_back(make_backend(b, opt));
    std::vector<Case> cases;
    for (const auto &c : load_cases(opt.shapes))
        if (opt.only.empty() || opt.only.count(c.id))
            cases.push_back(c);
    std::string out_path = opt.out;
    if (out_path.empty()) {
        std::string stem = opt.shapes.substr(opt.shapes.find_last_of('/') + 1);
        stem = stem.substr(0, stem.find_last_of('.'));
        char ts[32];
        const std::time_t now = std::time(nullptr);
        std::strftime(ts, sizeof(ts), "%Y%m%d-%H%M%S", std::localtime(&now));
        out_path = "results_" + stem + "_" + gg::dtype_name(opt.dtype) + "_" + ts + ".csv";
    }
    std::cout << "GPU: " << gpu << "\nshapes: " << opt.shapes << " (" << cases.size() << " cases), dtype "
              << gg::dtype_name(opt.dtype) << ", warmup " << opt.warmup << ", iters " << opt.iters << "\n";

    cudaStream_t stream;
    GG_CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    cudaEvent_t e0, e1;
    GG_CUDA_CHECK(cudaEventCreate(&e0));
    GG_CUDA_CHECK(cudaEventCreate(&e1));
    Buffer xb, wb, ob;
    int64_t *lens = nullptr;
    size_t lens_cap = 0;
    std::vector<Result> rows;

    for (const auto &c : cases) {
        GroupedGemmProblem p;
        p.dtype = opt.dtype;
        p.group_num = int(c.b);
        p.n = c.n;
        p.k = c.k;
        p.group_m.assign(size_t(c.b), c.m);
        const size_t es = gg::dtype_bytes(p.dtype);
        const size_t nx = size_t(p.total_m()) * p.k, nw = size_t(p.group_num) * p.n * p.k;
        const size_t nout_bytes = size_t(p.total_m()) * p.n * es;
        p.x = xb.need(nx * es);
        p.w = wb.need(nw * es);
        p.out = ob.need(nout_bytes);
        if (lens_cap < size_t(p.group_num)) {
            if (lens)
                GG_CUDA_CHECK(cudaFreeHost(lens));
            GG_CUDA_CHECK(cudaMallocHost(&lens, size_t(p.group_num) * sizeof(int64_t)));
            lens_cap = size_t(p.group_num);
        }
        std::copy(p.group_m.begin(), p.group_m.end(), lens);
        p.group_lens_pinned = lens;
        if (p.dtype == DType::BF16) {
            fill_normal<__nv_bfloat16><<<4096, 256, 0, stream>>>(static_cast<__nv_bfloat16 *>(const_cast<void *>(p.x)), nx, 1);
            fill_normal<__nv_bfloat16><<<4096, 256, 0, stream>>>(static_cast<__nv_bfloat16 *>(const_cast<void *>(p.w)), nw, 2);
        } else {
            fill_normal<__half><<<4096, 256, 0, stream>>>(static_cast<__half *>(const_cast<void *>(p.x)), nx, 1);
            fill_normal<__half><<<4096, 256, 0, stream>>>(static_cast<__half *>(const_cast<void *>(p.w)), nw, 2);
        }
        GG_CUDA_CHECK(cudaGetLastError());
        const auto positions = sample_positions(p);
        std::cout << "\n[" << c.id << "] " << c.name << "  B=" << c.b << " M=" << c.m << " N=" << c.n << " K=" << c.k
                  << "  (" << std::setprecision(3) << p.flops() / 1e12 << " TFLOP)\n";

        for (auto &be : backends) {
            Result r{c, be->name(), "", "", NAN, NAN, NAN};
            try {
                GG_CUDA_CHECK(cudaMemsetAsync(p.out, 0, nout_bytes, stream));
                const std::string why = be->prepare(p, stream);
                if (!why.empty()) {
                    r.check = "N/A";
                    r.detail = why;
                } else {
                    r.detail = be->detail();
                    be->run(stream);
                    GG_CUDA_CHECK(cudaGetLastError());
                    GG_CUDA_CHECK(cudaStreamSynchronize(stream));
                    const uint32_t st = be->device_status(stream);
                    if (opt.check) {
                        const CheckOut k = p.dtype == DType::BF16 ? check_samples<__nv_bfloat16>(p, positions, stream)
                                                                  : check_samples<__half>(p, positions, stream);
                        r.check = k.pass && st == 0 ? "PASS" : "FAIL";
                        r.max_abs = k.max_abs;
                        if (!k.pass)
                            r.detail += " | " + std::to_string(k.bad) + "/" + std::to_string(positions.size()) +
                                        " samples off";
                    } else {
                        r.check = st == 0 ? "SKIP" : "FAIL";
                    }
                    if (st != 0)
                        r.detail += " | device status " + std::to_string(st);
                    for (int i = 0; i < opt.warmup; ++i)
                        be->run(stream);
                    GG_CUDA_CHECK(cudaEventRecord(e0, stream));
                    for (int i = 0; i < opt.iters; ++i)
                        be->run(stream);
                    GG_CUDA_CHECK(cudaEventRecord(e1, stream));
                    GG_CUDA_CHECK(cudaEventSynchronize(e1));
                    GG_CUDA_CHECK(cudaGetLastError());
                    float ms = 0.f;
                    GG_CUDA_CHECK(cudaEventElapsedTime(&ms, e0, e1));
                    r.ms = double(ms) / opt.iters;
                    r.tflops = p.flops() / (r.ms * 1e-3) / 1e12;
                }
            } catch (const std::exception &ex) {
                (void)cudaStreamSynchronize(stream);
                r.check = "ERROR";
                r.detail = ex.what();
            }
            be->release();
            std::cout << "  " << std::left << std::setw(16) << r.backend << std::setw(6) << r.check << std::right
                      << std::fixed;
            if (std::isnan(r.ms))
                std::cout << std::setw(12) << "-" << std::setw(14) << "-";
            else
                std::cout << std::setprecision(3) << std::setw(10) << r.ms << " ms" << std::setprecision(1)
                          << std::setw(9) << r.tflops << " TFLOPS";
            std::cout << "  " << r.detail.substr(0, 100) << "\n";
            std::cout.unsetf(std::ios::fixed);
            rows.push_back(r);
        }
        save_csv(out_path, rows, gpu, opt.dtype);  // after every case, so a crash keeps what finished
    }
    summary(rows, opt.backends);
    std::cout << "\nresults: " << out_path << "\n";
    if (lens)
        cudaFreeHost(lens);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaStreamDestroy(stream);
    for (const auto &r : rows)
        if (r.check == "FAIL" || r.check == "ERROR")
            return 1;
    return 0;
}

}  // namespace

int main(int argc, char **argv) {
    try {
        return run(parse(argc, argv));
    } catch (const std::exception &e) {
        std::cerr << "fatal: " << e.what() << "\n";
        return 1;
    }
}
