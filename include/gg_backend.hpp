// gg_backend.hpp — C++ host interface of the B200 grouped GEMM.
//
// Restates the reference's common/backend.hpp (TheRealMichaelWang/GroupGEMM-CKTile-Optimized)
// for CUDA: the same problem descriptor (GroupedGemmProblem, common/backend.hpp:39-60) and the
// same backend interface (Backend, common/backend.hpp:62-79), with cudaStream_t for hipStream_t.
// B200Backend implements it over the C ABI of gg_b200.h and is created by make_b200_backend(),
// the factory that sits beside the reference's make_ck_tile_backend()
// (common/backend.hpp:81-83).
//
// Differences from the reference, on purpose: a failing CUDA call throws gg::CudaError instead
// of exit(1) (TUNEMAX_HIP_CHECK, common/backend.hpp:15-23), so a harness can record an ERROR row
// and continue; device-side bounded-wait timeouts are reported by device_status().
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "gg_b200.h"

namespace gg {

struct CudaError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

#define GG_CUDA_CHECK(expr)                                                                              \
    do {                                                                                                 \
        const cudaError_t gg_err_ = (expr);                                                              \
        if (gg_err_ != cudaSuccess)                                                                      \
            throw ::gg::CudaError(std::string(#expr) + ": " + cudaGetErrorString(gg_err_) + " (" __FILE__ \
                                  ":" + std::to_string(__LINE__) + ")");                                 \
    } while (0)

enum class DType { BF16, FP16 };

inline const char *dtype_name(DType t) { return t == DType::BF16 ? "bf16" : "fp16"; }
inline size_t dtype_bytes(DType) { return 2; }

// out[rows of group g] = x[rows of group g] @ w[g]^T, fp32 accumulation, output in the input
// dtype. x [sum(group_m), k] row-major, w [group_num, n, k] row-major, out [sum(group_m), n]
// row-major; x, w, out are device pointers owned by the caller.
struct GroupedGemmProblem {
    DType dtype = DType::BF16;
    int group_num = 0;
    int64_t n = 0;
    int64_t k = 0;
    std::vector<int64_t> group_m;  // host copy, one entry per group

    const void *x = nullptr;
    const void *w = nullptr;
    void *out = nullptr;

    // Same values as group_m in pinned host memory (backends that read lengths per call).
    const int64_t *group_lens_pinned = nullptr;

    int64_t total_m() const {
        int64_t s = 0;
        for (int64_t m : group_m)
            s += m;
        return s;
    }
    double flops() const { return 2.0 * double(total_m()) * double(n) * double(k); }
};

// One grouped GEMM implementation.
//   prepare(): untimed; returns "" when ready, or why this problem cannot run (N/A).
//   run():     timed; enqueues exactly one grouped GEMM on `stream`, no synchronisation.
//   release(): frees what prepare() allocated; called after each problem.
class Backend {
public:
    virtual ~Backend() = default;
    virtual std::string name() const = 0;
    virtual std::string prepare(const GroupedGemmProblem &problem, cudaStream_t stream) = 0;
    virtual void run(cudaStream_t stream) = 0;
    virtual void release() {}
    virtual std::string detail() const { return ""; }
    // 0 when every kernel launched since the last call finished its waits (synchronises).
    virtual uint32_t device_status(cudaStream_t) { return 0; }
};

// The sm_100a grouped GEMM through the C ABI.
class B200Backend final : public Backend {
public:
    B200Backend() : h_(gg_create()) {
        if (!h_)
            throw std::bad_alloc();
    }
    ~B200Backend() override { gg_destroy(h_); }
    B200Backend(const B200Backend &) = delete;
    B200Backend &operator=(const B200Backend &) = delete;

    std::string name() const override { return gg_name(h_); }

    std::string prepare(const GroupedGemmProblem &p, cudaStream_t stream) override {
        const gg_problem q{p.dtype == DType::BF16 ? GG_BF16 : GG_FP16, p.group_num, p.n, p.k, p.group_m.data(),
                           p.x, p.w, p.out};
        char why[256];
        const int rc = gg_prepare(h_, &q, stream, why, sizeof(why));
        if (rc == GG_OK)
            return "";
        if (rc == GG_NOT_SUPPORTED)
            return why;
        throw CudaError(gg_last_error(h_));
    }

    // Backward grouped GEMM of the same layer (GG_OP_DGRAD or GG_OP_WGRAD, gg_prepare_grad);
    // run()/release()/detail() then apply to it. Returns "" or the N/A reason.
    std::string prepare_grad(const gg_grad_problem &q, int32_t op, cudaStream_t stream) {
        char why[256];
        const int rc = gg_prepare_grad(h_, &q, op, stream, why, sizeof(why));
        if (rc == GG_OK)
            return "";
        if (rc == GG_NOT_SUPPORTED)
            return why;
        throw CudaError(gg_last_error(h_));
    }

    void run(cudaStream_t stream) override {
        if (gg_run(h_, stream) != GG_OK)
            throw CudaError(gg_last_error(h_));
    }

    void release() override { gg_release(h_); }
    std::string detail() const override { return gg_detail(h_); }

    uint32_t device_status(cudaStream_t stream) override {
        uint32_t st = 0;
        const int rc = gg_device_status(h_, stream, &st);
        if (rc != GG_OK && rc != GG_ERR_DEVICE)
            throw CudaError(gg_last_error(h_));
        return st;
    }

    // Knobs of gg_set_option ("variant", "bn", "split", "stream_k", "max_ctas", ...; gg_b200.h).
    void set_option(const char *key, int64_t value) {
        if (gg_set_option(h_, key, value) != GG_OK)
            throw std::invalid_argument(gg_last_error(h_));
    }

private:
    gg_handle *h_;
};

inline std::unique_ptr<Backend> make_b200_backend() { return std::make_unique<B200Backend>(); }

// cuBLAS comparison backends of the C++ harness (gg_bench), the analogues of the reference's
// hipBLASLt baselines (backends/hipblaslt_loop_backend.cpp, backends/hipblaslt_grouped_backend.cpp).
// Not on the product path. Defined in groupgemm-cktile-optimized_b200/csrc/gg_cublas_backends.cpp.
std::unique_ptr<Backend> make_cublas_loop_backend();
std::unique_ptr<Backend> make_cublas_grouped_backend();

}  // namespace gg
