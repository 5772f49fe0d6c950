// Reference harness, built from the reference's own sources (test infrastructure only).
//
// This file #includes the reference's bench/bench_main.cpp UNMODIFIED (through the HIP->CUDA
// shim in ref_shim/) so that its own device input generator (fill_randn), sample rule
// (make_samples), fp32 reference kernel (sampled_reference), pass rule (check_output),
// shapes-CSV reader and results-CSV writer run on the B200. Nothing of the reference is copied
// here; the build recipe (oracle/build.py) compiles it from where it lies.
//
// Modes
//   ref_harness golden DIR DTYPE B M N K [full]
//       Writes the reference generator's x/w bits, its sample list and its fp32 reference
//       value per sample (and, with `full`, at every output element) to DIR. These files pin
//       the CPU oracle (tests/golden/).
//   ref_harness check LIBGG --shapes FILE.csv [--dtype bf16|fp16] [--only IDS] [--warmup N] [--iters N]
//                     [--out FILE.csv]
//       The reference's per-case bench loop (bench/bench_main.cpp:430-523) with one backend,
//       "b200": the B200 library loaded from LIBGG through its C ABI, wrapped in the reference's
//       own Backend interface exactly as a maintainer would register it. Exit code 1 if any
//       case FAILs or ERRORs, like the reference (bench/bench_main.cpp:534-537).
#include <dlfcn.h>

#include <fstream>
#include <stdexcept>

#define main tunemax_reference_bench_main
#include "bench/bench_main.cpp"
#undef main

#include "../include/gg_b200.h"

namespace tunemax {

// The reference's own backends need ROCm (CK Tile on gfx950, hipBLASLt); they are not
// buildable here. These stand-ins only satisfy the reference harness's factory symbols.
namespace {
class UnavailableBackend final : public Backend {
public:
    explicit UnavailableBackend(std::string n) : name_(std::move(n)) {}
    std::string name() const override { return name_; }
    std::string prepare(const GroupedGemmProblem &, hipStream_t) override {
        return "not buildable on this box (needs ROCm and a gfx950 GPU)";
    }
    void run(hipStream_t) override {}

private:
    std::string name_;
};
}  // namespace

std::unique_ptr<Backend> make_ck_tile_backend() { return std::make_unique<UnavailableBackend>("ck_tile"); }
std::unique_ptr<Backend> make_hipblaslt_grouped_backend() {
    return std::make_unique<UnavailableBackend>("hipblaslt_grouped");
}
std::unique_ptr<Backend> make_hipblaslt_loop_backend() {
    return std::make_unique<UnavailableBackend>("hipblaslt_loop");
}

// The B200 backend as the reference's harness sees it: tunemax::Backend over the C ABI.
class B200Backend final : public Backend {
public:
    explicit B200Backend(const std::string &lib_path) {
        so_ = dlopen(lib_path.c_str(), RTLD_NOW | RTLD_LOCAL);
        if (!so_)
            throw std::runtime_error(std::string("dlopen: ") + dlerror());
        create_ = reinterpret_cast<decltype(create_)>(sym("gg_create"));
        prepare_ = reinterpret_cast<decltype(prepare_)>(sym("gg_prepare"));
        run_ = reinterpret_cast<decltype(run_)>(sym("gg_run"));
        release_ = reinterpret_cast<decltype(release_)>(sym("gg_release"));
        detail_ = reinterpret_cast<decltype(detail_)>(sym("gg_detail"));
        last_error_ = reinterpret_cast<decltype(last_error_)>(sym("gg_last_error"));
        status_ = reinterpret_cast<decltype(status_)>(sym("gg_device_status"));
        destroy_ = reinterpret_cast<decltype(destroy_)>(sym("gg_destroy"));
        h_ = create_();
    }
    ~B200Backend() override {
        if (h_)
            destroy_(h_);
    }
    std::string name() const override { return "b200"; }
    std::string prepare(const GroupedGemmProblem &p, hipStream_t stream) override {
        gg_problem q{p.dtype == DType::BF16 ? GG_BF16 : GG_FP16, p.group_num, p.n, p.k, p.group_m.data(), p.x, p.w,
                     p.out};
        char why[256];
        const int rc = prepare_(h_, &q, stream, why, sizeof(why));
        if (rc == GG_OK)
            return "";
        if (rc == GG_NOT_SUPPORTED)
            return why;
        throw std::runtime_error(last_error_(h_));
    }
    void run(hipStream_t stream) override {
        if (run_(h_, stream) != GG_OK)
            throw std::runtime_error(last_error_(h_));
    }
    void release() override { release_(h_); }
    std::string detail() const override { return detail_(h_); }
    uint32_t device_status(hipStream_t stream) {
        uint32_t st = 0;
        status_(h_, stream, &st);
        return st;
    }

private:
    void *sym(const char *n) {
        void *p = dlsym(so_, n);
        if (!p)
            throw std::runtime_error(std::string("missing symbol ") + n);
        return p;
    }
    void *so_ = nullptr;
    gg_handle *h_ = nullptr;
    gg_handle *(*create_)() = nullptr;
    int (*prepare_)(gg_handle *, const gg_problem *, gg_stream_t, char *, size_t) = nullptr;
    int (*run_)(gg_handle *, gg_stream_t) = nullptr;
    void (*release_)(gg_handle *) = nullptr;
    const char *(*detail_)(const gg_handle *) = nullptr;
    const char *(*last_error_)(const gg_handle *) = nullptr;
    int (*status_)(gg_handle *, gg_stream_t, uint32_t *) = nullptr;
    void (*destroy_)(gg_handle *) = nullptr;
};

namespace harness {

template <typename T> void write_bin(const std::string &path, const std::vector<T> &v) {
    std::ofstream f(path, std::ios::binary);
    if (!f)
        throw std::runtime_error("cannot write " + path);
    f.write(reinterpret_cast<const char *>(v.data()), std::streamsize(v.size() * sizeof(T)));
}

template <typename T>
int golden(const std::string &dir, DType dtype, int64_t b, int64_t m, int64_t n, int64_t k, bool full) {
    GroupedGemmProblem p;
    p.dtype = dtype;
    p.group_num = int(b);
    p.n = n;
    p.k = k;
    p.group_m.assign(b, m);
    const size_t nx = size_t(p.total_m()) * k, nw = size_t(b) * n * k;
    hipStream_t stream;
    TUNEMAX_HIP_CHECK(hipStreamCreateWithFlags(&stream, hipStreamNonBlocking));
    DeviceBuffer xb, wb, ob;
    p.x = xb.get(nx * 2);
    p.w = wb.get(nw * 2);
    p.out = ob.get(size_t(p.total_m()) * n * 2);
    TUNEMAX_HIP_CHECK(hipMemsetAsync(p.out, 0, size_t(p.total_m()) * n * 2, stream));
    fill<T>(const_cast<void *>(p.x), nx, 1, stream);  // the reference's seeds (bench_main.cpp:450-457)
    fill<T>(const_cast<void *>(p.w), nw, 2, stream);
    std::vector<uint16_t> hx(nx), hw(nw);
    TUNEMAX_HIP_CHECK(hipMemcpyAsync(hx.data(), p.x, nx * 2, hipMemcpyDeviceToHost, stream));
    TUNEMAX_HIP_CHECK(hipMemcpyAsync(hw.data(), p.w, nw * 2, hipMemcpyDeviceToHost, stream));

    auto eval = [&](const std::vector<Sample> &samples) {
        const size_t ns = samples.size();
        Sample *d_s;
        float *d_ref, *d_got;
        TUNEMAX_HIP_CHECK(hipMalloc(&d_s, ns * sizeof(Sample)));
        TUNEMAX_HIP_CHECK(hipMalloc(&d_ref, ns * sizeof(float)));
        TUNEMAX_HIP_CHECK(hipMalloc(&d_got, ns * sizeof(float)));
        TUNEMAX_HIP_CHECK(hipMemcpyAsync(d_s, samples.data(), ns * sizeof(Sample), hipMemcpyHostToDevice, stream));
        sampled_reference<T><<<ns, 256, 0, stream>>>(static_cast<const T *>(p.x), static_cast<const T *>(p.w),
                                                     static_cast<const T *>(p.out), p.n, p.k, d_s, d_ref, d_got);
        TUNEMAX_HIP_CHECK(hipGetLastError());
        std::vector<float> ref(ns);
        TUNEMAX_HIP_CHECK(hipMemcpyAsync(ref.data(), d_ref, ns * sizeof(float), hipMemcpyDeviceToHost, stream));
        TUNEMAX_HIP_CHECK(hipStreamSynchronize(stream));
        TUNEMAX_HIP_CHECK(hipFree(d_s));
        TUNEMAX_HIP_CHECK(hipFree(d_ref));
        TUNEMAX_HIP_CHECK(hipFree(d_got));
        return ref;
    };

    const std::vector<Sample> samples = make_samples(p);
    const std::vector<float> ref = eval(samples);
    std::vector<int64_t> sflat;
    for (const Sample &s : samples) {
        sflat.push_back(s.row);
        sflat.push_back(s.col);
        sflat.push_back(s.group);
    }
    write_bin(dir + "/x.u16", hx);
    write_bin(dir + "/w.u16", hw);
    write_bin(dir + "/samples.i64", sflat);
    write_bin(dir + "/sample_ref.f32", ref);
    if (full) {
        std::vector<Sample> all;
        int64_t row0 = 0;
        for (int g = 0; g < p.group_num; ++g) {
            for (int64_t r = 0; r < p.group_m[g]; ++r)
                for (int64_t c = 0; c < n; ++c)
                    all.push_back({row0 + r, c, g});
            row0 += p.group_m[g];
        }
        write_bin(dir + "/full_ref.f32", eval(all));
    }
    std::ofstream meta(dir + "/meta.txt");
    meta << "dtype " << dtype_name(dtype) << "\nB " << b << "\nM " << m << "\nN " << n << "\nK " << k
         << "\nsamples " << samples.size() << "\nfull " << (full ? 1 : 0) << "\n";
    TUNEMAX_HIP_CHECK(hipStreamDestroy(stream));
    return 0;
}

// The reference bench loop of bench/bench_main.cpp:392-538, restricted to one backend.
int check(const std::string &lib, const Options &opt) {
    B200Backend backend(lib);
    hipDeviceProp_t prop;
    TUNEMAX_HIP_CHECK(hipGetDeviceProperties(&prop, 0));
    const std::string gpu = std::string(prop.name) + " (" + prop.gcnArchName + ")";
    std::vector<TestCase> cases;
    for (const auto &c : read_cases(opt.shapes))
        if (opt.only.empty() || opt.only.count(c.id))
            cases.push_back(c);
    const std::string out_path = opt.out.empty() ? "ref_harness_results.csv" : opt.out;
    std::cout << "GPU: " << gpu << "\nshapes: " << opt.shapes << " (" << cases.size() << " cases), dtype "
              << dtype_name(opt.dtype) << ", warmup " << opt.warmup << ", iters " << opt.iters << "\n";
    hipStream_t stream;
    TUNEMAX_HIP_CHECK(hipStreamCreateWithFlags(&stream, hipStreamNonBlocking));
    hipEvent_t start, stop;
    TUNEMAX_HIP_CHECK(hipEventCreate(&start));
    TUNEMAX_HIP_CHECK(hipEventCreate(&stop));
    DeviceBuffer x_buf, w_buf, out_buf;
    std::vector<Row> rows;
    for (const auto &tc : cases) {
        GroupedGemmProblem p;
        p.dtype = opt.dtype;
        p.group_num = int(tc.b);
        p.n = tc.n;
        p.k = tc.k;
        p.group_m.assign(tc.b, tc.m);
        const size_t es = dtype_bytes(p.dtype);
        p.x = x_buf.get(size_t(p.total_m()) * p.k * es);
        p.w = w_buf.get(size_t(p.group_num) * p.n * p.k * es);
        p.out = out_buf.get(size_t(p.total_m()) * p.n * es);
        if (p.dtype == DType::BF16) {
            fill<__hip_bfloat16>(const_cast<void *>(p.x), size_t(p.total_m()) * p.k, 1, stream);
            fill<__hip_bfloat16>(const_cast<void *>(p.w), size_t(p.group_num) * p.n * p.k, 2, stream);
        } else {
            fill<__half>(const_cast<void *>(p.x), size_t(p.total_m()) * p.k, 1, stream);
            fill<__half>(const_cast<void *>(p.w), size_t(p.group_num) * p.n * p.k, 2, stream);
        }
        const std::vector<Sample> samples = make_samples(p);
        Row row{tc, backend.name(), "", "", NAN, NAN, NAN};
        try {
            TUNEMAX_HIP_CHECK(hipMemsetAsync(p.out, 0, size_t(p.total_m()) * p.n * es, stream));
            const std::string why_not = backend.prepare(p, stream);
            if (!why_not.empty()) {
                row.check = "N/A";
                row.detail = why_not;
            } else {
                row.detail = backend.detail();
                backend.run(stream);
                TUNEMAX_HIP_CHECK(hipGetLastError());
                TUNEMAX_HIP_CHECK(hipStreamSynchronize(stream));
                const uint32_t st = backend.device_status(stream);
                const CheckResult c = p.dtype == DType::BF16 ? check_output<__hip_bfloat16>(p, samples, stream)
                                                             : check_output<__half>(p, samples, stream);
                row.check = (c.pass && st == 0) ? "PASS" : "FAIL";
                row.max_abs = c.max_abs;
                if (!c.pass)
                    row.detail += " | " + std::to_string(c.mismatches) + "/" + std::to_string(samples.size()) +
                                  " samples off";
                if (st != 0)
                    row.detail += " | device status " + std::to_string(st);
                for (int i = 0; i < opt.warmup; ++i)
                    backend.run(stream);
                TUNEMAX_HIP_CHECK(hipEventRecord(start, stream));
                for (int i = 0; i < opt.iters; ++i)
                    backend.run(stream);
                TUNEMAX_HIP_CHECK(hipEventRecord(stop, stream));
                TUNEMAX_HIP_CHECK(hipEventSynchronize(stop));
                float total_ms = 0.f;
                TUNEMAX_HIP_CHECK(hipEventElapsedTime(&total_ms, start, stop));
                row.ms = double(total_ms) / opt.iters;
                row.tflops = p.flops() / (row.ms * 1e-3) / 1e12;
            }
        } catch (const std::exception &e) {
            (void)hipStreamSynchronize(stream);
            row.check = "ERROR";
            row.detail = e.what();
        }
        backend.release();
        std::cout << "  [" << tc.id << "] " << tc.name << " " << row.check << " " << row.ms << " ms "
                  << row.tflops << " TFLOPS maxabs " << row.max_abs << "  " << row.detail << "\n";
        rows.push_back(row);
        write_csv(out_path, rows, gpu, opt.dtype);
    }
    print_summary(rows, {"b200"});
    TUNEMAX_HIP_CHECK(hipEventDestroy(start));
    TUNEMAX_HIP_CHECK(hipEventDestroy(stop));
    TUNEMAX_HIP_CHECK(hipStreamDestroy(stream));
    for (const auto &r : rows)
        if (r.check == "FAIL" || r.check == "ERROR")
            return 1;
    return 0;
}

}  // namespace harness
}  // namespace tunemax

int main(int argc, char **argv) {
    using namespace tunemax;
    if (argc >= 8 && std::string(argv[1]) == "golden") {
        const DType dt = std::string(argv[3]) == "fp16" ? DType::FP16 : DType::BF16;
        const bool full = argc >= 9 && std::string(argv[8]) == "full";
        const int64_t b = std::stoll(argv[4]), m = std::stoll(argv[5]), n = std::stoll(argv[6]),
                      k = std::stoll(argv[7]);
        return dt == DType::BF16 ? harness::golden<__hip_bfloat16>(argv[2], dt, b, m, n, k, full)
                                 : harness::golden<__half>(argv[2], dt, b, m, n, k, full);
    }
    if (argc >= 3 && std::string(argv[1]) == "check") {
        // The reference's own option parser, fed the arguments after the library path.
        std::vector<char *> args{argv[0]};
        for (int i = 3; i < argc; ++i)
            args.push_back(argv[i]);
        const Options opt = parse_args(int(args.size()), args.data());
        return harness::check(argv[2], opt);
    }
    std::fprintf(stderr,
                 "usage: ref_harness golden DIR bf16|fp16 B M N K [full]\n"
                 "       ref_harness check LIBGG --shapes FILE.csv [bench_main options]\n");
    return 2;
}
