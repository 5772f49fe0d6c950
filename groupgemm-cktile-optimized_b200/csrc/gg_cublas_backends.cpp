// cuBLAS comparison backends for the C++ harness (gg_bench). They are the B200 analogues of the
// reference's two hipBLASLt baselines and are NOT on the product path:
//
//   cublas_loop    one cublasGemmEx per group, round-robin over 4 streams with event fork/join
//                  and per-call host argument setup from the pinned group lengths — what
//                  Primus-Turbo's hipblaslt_grouped_gemm does (backends/hipblaslt_loop_backend.cpp,
//                  third_party/primus_turbo/kernels/hipblaslt_grouped_gemm.cu:99-163).
//   cublas_grouped one cublasGemmGroupedBatchedEx call with device pointer arrays built in prepare,
//                  like the hipBLASLt GroupedGemm backend (backends/hipblaslt_grouped_backend.cpp:45-98).
//
// Both compute out_g = x_g @ w_g^T in cuBLAS's column-major terms as
//   C[N x M_g] = op(A)[N x K] * B[K x M_g],  A = w_g viewed as K x N (op = T), B = x_g as K x M_g.
#include <cublas_v2.h>

#include <array>
#include <string>
#include <vector>

#include "gg_backend.hpp"

namespace gg {
namespace {

void cublas_check(cublasStatus_t s, const char *what) {
    if (s != CUBLAS_STATUS_SUCCESS)
        throw CudaError(std::string(what) + ": cuBLAS status " + std::to_string(int(s)));
}

cudaDataType_t cuda_type(DType t) { return t == DType::BF16 ? CUDA_R_16BF : CUDA_R_16F; }

class CublasLoopBackend final : public Backend {
public:
    static constexpr int kStreams = 4;

    ~CublasLoopBackend() override {
        for (int i = 0; i < kStreams; ++i) {
            if (handles_[i])
                cublasDestroy(handles_[i]);
            if (streams_[i])
                cudaStreamDestroy(streams_[i]);
            if (join_[i])
                cudaEventDestroy(join_[i]);
        }
        if (fork_)
            cudaEventDestroy(fork_);
    }

    std::string name() const override { return "cublas_loop"; }

    std::string prepare(const GroupedGemmProblem &p, cudaStream_t) override {
        if (!fork_) {
            GG_CUDA_CHECK(cudaEventCreateWithFlags(&fork_, cudaEventDisableTiming));
            for (int i = 0; i < kStreams; ++i) {
                GG_CUDA_CHECK(cudaStreamCreateWithFlags(&streams_[i], cudaStreamNonBlocking));
                GG_CUDA_CHECK(cudaEventCreateWithFlags(&join_[i], cudaEventDisableTiming));
                cublas_check(cublasCreate(&handles_[i]), "cublasCreate");
                cublas_check(cublasSetStream(handles_[i], streams_[i]), "cublasSetStream");
            }
        }
        p_ = p;
        return "";
    }

    void run(cudaStream_t stream) override {
        const float alpha = 1.f, beta = 0.f;
        const auto t = cuda_type(p_.dtype);
        const size_t es = dtype_bytes(p_.dtype);
        GG_CUDA_CHECK(cudaEventRecord(fork_, stream));
        for (int i = 0; i < kStreams; ++i)
            GG_CUDA_CHECK(cudaStreamWaitEvent(streams_[i], fork_, 0));
        int64_t row = 0;
        for (int g = 0; g < p_.group_num; ++g) {
            // group lengths read on the host every call, as the Primus-Turbo loop does
            const int64_t m = p_.group_lens_pinned ? p_.group_lens_pinned[g] : p_.group_m[g];
            if (m > 0) {
                const auto *x = static_cast<const char *>(p_.x) + size_t(row) * p_.k * es;
                const auto *w = static_cast<const char *>(p_.w) + size_t(g) * p_.n * p_.k * es;
                auto *o = static_cast<char *>(p_.out) + size_t(row) * p_.n * es;
                cublas_check(cublasGemmEx(handles_[g % kStreams], CUBLAS_OP_T, CUBLAS_OP_N, int(p_.n), int(m),
                                          int(p_.k), &alpha, w, t, int(p_.k), x, t, int(p_.k), &beta, o, t,
                                          int(p_.n), CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT),
                             "cublasGemmEx");
            }
            row += m;
        }
        for (int i = 0; i < kStreams; ++i) {
            GG_CUDA_CHECK(cudaEventRecord(join_[i], streams_[i]));
            GG_CUDA_CHECK(cudaStreamWaitEvent(stream, join_[i], 0));
        }
    }

    std::string detail() const override { return "cublasGemmEx per group over 4 streams"; }

private:
    GroupedGemmProblem p_;
    std::array<cublasHandle_t, kStreams> handles_{};
    std::array<cudaStream_t, kStreams> streams_{};
    std::array<cudaEvent_t, kStreams> join_{};
    cudaEvent_t fork_ = nullptr;
};

class CublasGroupedBackend final : public Backend {
public:
    ~CublasGroupedBackend() override {
        release();
        if (handle_)
            cublasDestroy(handle_);
    }

    std::string name() const override { return "cublas_grouped"; }

    std::string prepare(const GroupedGemmProblem &p, cudaStream_t stream) override {
        if (!handle_)
            cublas_check(cublasCreate(&handle_), "cublasCreate");
        release();
        p_ = p;
        type_ = cuda_type(p.dtype);
        const size_t es = dtype_bytes(p.dtype);
        // one cuBLAS "group" per non-empty expert (each has its own m)
        std::vector<const void *> a, b;
        std::vector<void *> c;
        int64_t row = 0;
        for (int g = 0; g < p.group_num; ++g) {
            const int64_t m = p.group_m[g];
            if (m > 0) {
                a.push_back(static_cast<const char *>(p.w) + size_t(g) * p.n * p.k * es);
                b.push_back(static_cast<const char *>(p.x) + size_t(row) * p.k * es);
                c.push_back(static_cast<char *>(p.out) + size_t(row) * p.n * es);
                transa_.push_back(CUBLAS_OP_T);
                transb_.push_back(CUBLAS_OP_N);
                m_.push_back(int(p.n));
                n_.push_back(int(m));
                k_.push_back(int(p.k));
                lda_.push_back(int(p.k));
                ldb_.push_back(int(p.k));
                ldc_.push_back(int(p.n));
                alpha_.push_back(1.f);
                beta_.push_back(0.f);
                size_.push_back(1);
            }
            row += m;
        }
        count_ = int(a.size());
        if (count_ == 0)
            return "";
        GG_CUDA_CHECK(cudaMalloc(&d_ptrs_, 3 * size_t(count_) * sizeof(void *)));
        std::vector<const void *> all(a);
        all.insert(all.end(), b.begin(), b.end());
        for (void *pc : c)
            all.push_back(pc);
        GG_CUDA_CHECK(cudaMemcpyAsync(d_ptrs_, all.data(), all.size() * sizeof(void *), cudaMemcpyHostToDevice, stream));
        GG_CUDA_CHECK(cudaStreamSynchronize(stream));
        return "";
    }

    void run(cudaStream_t stream) override {
        if (count_ == 0)
            return;
        cublas_check(cublasSetStream(handle_, stream), "cublasSetStream");
        auto **ptrs = static_cast<void **>(d_ptrs_);
        cublas_check(cublasGemmGroupedBatchedEx(handle_, transa_.data(), transb_.data(), m_.data(), n_.data(),
                                                k_.data(), alpha_.data(), const_cast<const void *const *>(ptrs),
                                                type_, lda_.data(), const_cast<const void *const *>(ptrs + count_),
                                                type_, ldb_.data(), beta_.data(), ptrs + 2 * count_, type_,
                                                ldc_.data(), count_, size_.data(), CUBLAS_COMPUTE_32F),
                     "cublasGemmGroupedBatchedEx");
    }

    void release() override {
        if (d_ptrs_)
            cudaFree(d_ptrs_);
        d_ptrs_ = nullptr;
        count_ = 0;
        transa_.clear();
        transb_.clear();
        m_.clear();
        n_.clear();
        k_.clear();
        lda_.clear();
        ldb_.clear();
        ldc_.clear();
        alpha_.clear();
        beta_.clear();
        size_.clear();
    }

    std::string detail() const override { return "cublasGemmGroupedBatchedEx, one call"; }

private:
    GroupedGemmProblem p_;
    cublasHandle_t handle_ = nullptr;
    cudaDataType_t type_ = CUDA_R_16BF;
    void *d_ptrs_ = nullptr;
    int count_ = 0;
    std::vector<cublasOperation_t> transa_, transb_;
    std::vector<int> m_, n_, k_, lda_, ldb_, ldc_, size_;
    std::vector<float> alpha_, beta_;
};

}  // namespace

std::unique_ptr<Backend> make_cublas_loop_backend() { return std::make_unique<CublasLoopBackend>(); }
std::unique_ptr<Backend> make_cublas_grouped_backend() { return std::make_unique<CublasGroupedBackend>(); }

}  // namespace gg
