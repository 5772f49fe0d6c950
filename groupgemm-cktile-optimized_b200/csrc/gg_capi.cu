// Host side of the B200 grouped-GEMM backend: the C ABI of include/gg_b200.h.
//
// gg_prepare() plays the role of CkTileBackend::prepare_typed + finish
// (ck_kernel/ck_grouped_gemm.cpp:153-218): it validates the problem, builds the per-group
// argument buffer on the device (tile and row offsets instead of CK's GemmTransKernelArg
// array), encodes the TMA descriptors, picks the kernel variant and sizes the persistent grid.
// gg_run() is the single launch of CkGroupedGemm::launch (ck_kernel/ck_grouped_gemm.cpp:114-121).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "gg_b200.h"
#include "gg_kernel.cuh"
#include "gg_sched.h"

#ifndef GG_ATOMS_V0
#define GG_ATOMS_V0 2
#endif
#ifndef GG_ATOMS_V1
#define GG_ATOMS_V1 1
#endif
#ifndef GG_ATOMS_V2
#define GG_ATOMS_V2 2
#endif

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// One compiled instance of the kernel: a tile shape, for each operation and dtype.
struct Variant {
    int cg;        // CTAs per tile (1 or 2)
    int bn;        // tile N
    int cluster_m; // tile M
    int stages;
    int smem;
    const void *fn[3][2];  // [operation: forward, dgrad, wgrad][dtype: bf16, fp16]
    int atoms;     // 64-element K atoms per stage
    int (*stages_for)(int b_rows);  // ring stages of a launch whose tile loads b_rows B rows per CTA
};

template <int kCG, int kBN, int kAtoms, int kOp> void set_fns(Variant &v) {
    v.fn[kOp][GG_BF16] = reinterpret_cast<const void *>(&gg::grouped_gemm_sm100<__nv_bfloat16, kCG, kBN, kAtoms, kOp>);
    v.fn[kOp][GG_FP16] = reinterpret_cast<const void *>(&gg::grouped_gemm_sm100<__half, kCG, kBN, kAtoms, kOp>);
}

template <int kCG, int kBN, int kAtoms> Variant make_variant() {
    using C = gg::TileCfg<kCG, kBN, kAtoms>;
    Variant v{kCG, kBN, C::kClusterM, C::kStages, C::kSmemBytes, {}, kAtoms, &C::stages_for};
    set_fns<kCG, kBN, kAtoms, gg::kOpForward>(v);
    set_fns<kCG, kBN, kAtoms, gg::kOpDgrad>(v);
    set_fns<kCG, kBN, kAtoms, gg::kOpWgrad>(v);
    return v;
}

const Variant &variant_at(int i) {
    static const Variant v[3] = {make_variant<2, 256, GG_ATOMS_V0>(), make_variant<1, 256, GG_ATOMS_V1>(),
                                 make_variant<1, 128, GG_ATOMS_V2>()};
    return v[i];
}
constexpr int kNumVariants = 3;

// The variants' shapes for the cost model (gg_sched.h).
const gg::TileShape *tile_shapes() {
    static const gg::TileShape t[kNumVariants] = {
        {variant_at(0).cg, variant_at(0).bn, variant_at(0).cluster_m, variant_at(0).atoms},
        {variant_at(1).cg, variant_at(1).bn, variant_at(1).cluster_m, variant_at(1).atoms},
        {variant_at(2).cg, variant_at(2).bn, variant_at(2).cluster_m, variant_at(2).atoms}};
    return t;
}

using gg::Choice;

}  // namespace

struct gg_handle {
    // options
    int opt_variant = -1;
    int opt_band = 0;
    int opt_raster = -1;
    int opt_bn = 0;
    int opt_split = 0;
    int opt_sk_tail = -1;
    int opt_stream_k = 0;  // 0 off (default), -1 cost model decides, 1 / 2 stream-K over the partial
                           // last wave (+ one wave)
    int opt_max_ctas = 0;
    int64_t opt_timeout_ms = 2000;
    int opt_test_stall = 0;
    int opt_test_bounds = 0;  // test only: declare the output one row short to the debug build's checks
    int opt_pdl = 1;
    int opt_store = -1;  // -1 auto, 0 = staging + TMA stores, 1 = direct stores
    int opt_tail = -1;   // split launch for skewed routing: -1 auto, 0 off, 1 on
    int opt_chunks = 1;  // wgrad: 3-D chunk views for the MN-major operand loads where the shape allows
    int opt_order = 0;  // planned tile order (wgrad with store-bound and tensor-bound groups): -1 auto, 0 off, 1 on
    int opt_half = 0;    // 1 on (half-height last tiles where a group allows), 0 off (default), -1 = on
    int opt_sched = 0;  // -1 auto (dynamic for multi-wave launches of whole tiles), 0 static, 1 dynamic
    int opt_l2_a = -1;  // L2 eviction priority of the A / B operand loads (forward):
    int opt_l2_b = 0;   // 0 no hint, 1 evict_first, 2 evict_last; l2_a -1 = automatic

    // prepared state
    bool ready = false;
    int device = -1;
    int dtype = 0;
    int variant = 0;
    int64_t total_m = 0;
    int32_t *d_meta = nullptr;  // tile_off[G+1] then row_off[G+1]
    size_t meta_cap = 0;        // int32 entries
    uint32_t *d_status = nullptr;
    float *d_ws = nullptr;  // split-K partial sums
    size_t ws_cap = 0;      // bytes
    int32_t *d_counters = nullptr;
    size_t counters_cap = 0;  // bytes
    int32_t *d_tiles = nullptr;      // planned tile order: (group, mt << 16 | nt) per tile
    size_t tiles_cap = 0;            // int32 entries
    CUtensorMap *d_gmaps = nullptr;  // wgrad: per-group tensor maps
    size_t gmaps_cap = 0;            // maps
    int op = 0;                      // gg::kOpForward / kOpDgrad / kOpWgrad
    CUtensorMap tmap_a{}, tmap_b{}, tmap_out{};
    CUtensorMap tmap_a_half{};  // A in 64-row boxes, for half-height pair tiles
    // Second launch of a split launch: the one-CTA kernel over the groups' remainders of at most
    // 128 rows (tmap_a / tmap_out are shared with the first launch).
    struct {
        bool active = false;
        const void *fn = nullptr;
        int grid = 0, smem = 0;
        CUtensorMap tmap_b{};
        gg::KernelParams params{};
    } tail;
    gg::KernelParams params{};
    int grid = 0;
    const void *fn = nullptr;
    int smem = 0;
    int cg = 1;

    std::string detail, last_error;
};

namespace {

int fail(gg_handle *h, int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    h->last_error = buf;
    return code;
}

int refuse(gg_handle *h, char *why, size_t why_len, const char *msg) {
    h->last_error = msg;
    if (why && why_len > 0) {
        std::strncpy(why, msg, why_len - 1);
        why[why_len - 1] = '\0';
    }
    return GG_NOT_SUPPORTED;
}

#define GG_CUDA(h, expr)                                                                                  \
    do {                                                                                                  \
        cudaError_t e_ = (expr);                                                                          \
        if (e_ != cudaSuccess)                                                                            \
            return fail((h), GG_ERR_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(e_), __FILE__, __LINE__); \
    } while (0)

}  // namespace

extern "C" {

int gg_abi_version(void) { return 1; }

gg_handle *gg_create(void) { return new (std::nothrow) gg_handle(); }

const char *gg_name(const gg_handle *) { return "b200"; }

const char *gg_detail(const gg_handle *h) { return h ? h->detail.c_str() : ""; }

const char *gg_last_error(const gg_handle *h) { return h ? h->last_error.c_str() : "null handle"; }

int gg_set_option(gg_handle *h, const char *key, int64_t value) {
    if (!h || !key)
        return GG_ERR_ARG;
    if (!std::strcmp(key, "variant")) {
        if (value < -1 || value >= kNumVariants)
            return fail(h, GG_ERR_ARG, "variant must be -1..%d", kNumVariants - 1);
        h->opt_variant = int(value);
    } else if (!std::strcmp(key, "band")) {
        if (value < 0 || value > 1024)
            return fail(h, GG_ERR_ARG, "band must be 0..1024");
        h->opt_band = int(value);
    } else if (!std::strcmp(key, "raster")) {
        if (value < -1 || value > 1)
            return fail(h, GG_ERR_ARG, "raster must be -1 (auto), 0 (m-tile bands) or 1 (n-tile bands)");
        h->opt_raster = int(value);
    } else if (!std::strcmp(key, "split")) {
        if (value < 0 || value > 8)
            return fail(h, GG_ERR_ARG, "split must be 0 (auto) or 1..8");
        h->opt_split = int(value);
    } else if (!std::strcmp(key, "split_tail")) {
        if (value < -1 || value > 1)
            return fail(h, GG_ERR_ARG, "split_tail must be -1 (auto), 0 (split every tile) or 1 (only the last wave)");
        h->opt_sk_tail = int(value);
    } else if (!std::strcmp(key, "stream_k")) {
        if (value < -1 || value > 2)
            return fail(h, GG_ERR_ARG, "stream_k must be -1 (auto), 0 (off), 1 (partial last wave) or 2 (+ one wave)");
        h->opt_stream_k = int(value);
    } else if (!std::strcmp(key, "bn")) {
        if (value != 0 && (value < 16 || value > 256 || value % 16 != 0))
            return fail(h, GG_ERR_ARG, "bn must be 0 (auto) or a multiple of 16 in 16..256");
        h->opt_bn = int(value);
    } else if (!std::strcmp(key, "max_ctas")) {
        if (value < 0)
            return fail(h, GG_ERR_ARG, "max_ctas must be >= 0");
        h->opt_max_ctas = int(value);
    } else if (!std::strcmp(key, "timeout_ms")) {
        if (value < 1 || value > 60000)
            return fail(h, GG_ERR_ARG, "timeout_ms must be 1..60000");
        h->opt_timeout_ms = value;
    } else if (!std::strcmp(key, "store")) {
        if (value < -1 || value > 1)
            return fail(h, GG_ERR_ARG, "store must be -1 (auto), 0 (TMA stores) or 1 (direct stores)");
        h->opt_store = int(value);
    } else if (!std::strcmp(key, "tma_chunks")) {
        if (value < 0 || value > 1)
            return fail(h, GG_ERR_ARG, "tma_chunks must be 0 (one 2-D box per 64-column chunk) or 1");
        h->opt_chunks = int(value);
    } else if (!std::strcmp(key, "tile_order")) {
        if (value < -1 || value > 1)
            return fail(h, GG_ERR_ARG, "tile_order must be -1 (auto), 0 (group order) or 1 (interleaved)");
        h->opt_order = int(value);
    } else if (!std::strcmp(key, "tail_launch")) {
        if (value < -1 || value > 1)
            return fail(h, GG_ERR_ARG, "tail_launch must be -1 (auto), 0 (off) or 1 (on)");
        h->opt_tail = int(value);
    } else if (!std::strcmp(key, "half_tiles")) {
        if (value < -1 || value > 1)
            return fail(h, GG_ERR_ARG, "half_tiles must be -1 (auto), 0 (off) or 1 (on)");
        h->opt_half = int(value);
    } else if (!std::strcmp(key, "sched")) {
        if (value < -1 || value > 1)
            return fail(h, GG_ERR_ARG, "sched must be -1 (auto), 0 (static) or 1 (dynamic tile dispatch)");
        h->opt_sched = int(value);
    } else if (!std::strcmp(key, "l2_a")) {
        if (value < -1 || value > 2)
            return fail(h, GG_ERR_ARG, "l2_a must be -1 (auto), 0 (no hint), 1 (evict_first) or 2 (evict_last)");
        h->opt_l2_a = int(value);
    } else if (!std::strcmp(key, "l2_b")) {
        if (value < 0 || value > 2)
            return fail(h, GG_ERR_ARG, "l2_b must be 0 (no hint), 1 (evict_first) or 2 (evict_last)");
        h->opt_l2_b = int(value);
    } else if (!std::strcmp(key, "pdl")) {
        if (value != 0 && value != 1)
            return fail(h, GG_ERR_ARG, "pdl must be 0 or 1");
        h->opt_pdl = int(value);
    } else if (!std::strcmp(key, "test_bounds")) {
        if (value != 0 && value != 1)
            return fail(h, GG_ERR_ARG, "test_bounds must be 0 or 1");
        h->opt_test_bounds = int(value);
    } else if (!std::strcmp(key, "test_stall")) {
        if (value != 0 && value != 1)
            return fail(h, GG_ERR_ARG, "test_stall must be 0 or 1");
        h->opt_test_stall = int(value);
    } else {
        return fail(h, GG_ERR_ARG, "unknown option '%s'", key);
    }
    return GG_OK;
}

void gg_release(gg_handle *h) {
    if (!h)
        return;
    if (h->d_meta)
        cudaFree(h->d_meta);
    if (h->d_status)
        cudaFree(h->d_status);
    if (h->d_ws)
        cudaFree(h->d_ws);
    if (h->d_counters)
        cudaFree(h->d_counters);
    if (h->d_gmaps)
        cudaFree(h->d_gmaps);
    if (h->d_tiles)
        cudaFree(h->d_tiles);
    h->d_tiles = nullptr;
    h->tiles_cap = 0;
    h->d_gmaps = nullptr;
    h->gmaps_cap = 0;
    h->d_meta = nullptr;
    h->d_status = nullptr;
    h->d_ws = nullptr;
    h->d_counters = nullptr;
    h->ws_cap = 0;
    h->counters_cap = 0;
    h->meta_cap = 0;
    h->tail.active = false;
    h->ready = false;
    h->detail.clear();
}

void gg_destroy(gg_handle *h) {
    if (!h)
        return;
    gg_release(h);
    delete h;
}

int gg_expert_shard(int32_t group_num, int32_t world, int32_t rank, int32_t *g0, int32_t *g1) {
    if (group_num < 0 || world < 1 || rank < 0 || rank >= world || !g0 || !g1)
        return GG_ERR_ARG;
    const int32_t base = group_num / world, extra = group_num % world;
    *g0 = rank * base + std::min(rank, extra);
    *g1 = *g0 + base + (rank < extra ? 1 : 0);
    return GG_OK;
}

}  // extern "C"

namespace {

// One grouped GEMM of the layer, in the kernel's terms: A rows x B columns over a reduction.
//   forward: a = x,  b = w, out = out [sum(M), n]  (reduction k)
//   dgrad:   a = dy, b = w, out = dx  [sum(M), k]  (reduction n)
//   wgrad:   a = dy, b = x, out = dw  [G*n, k]     (reduction: the group's tokens)
struct OpProblem {
    int op;
    int32_t dtype;
    int32_t group_num;
    int64_t n, k;  // the layer's N and K
    const int64_t *group_m;
    const void *a, *b;
    void *out;
};

const char *op_name(int op) { return op == gg::kOpDgrad ? "dgrad" : op == gg::kOpWgrad ? "wgrad" : "forward"; }

int encode_2d(EncodeTiledFn encode, CUtensorMap *m, CUtensorMapDataType dt, const void *base, int64_t cols,
              int64_t rows, uint32_t box_cols, uint32_t box_rows, CUtensorMapL2promotion promo) {
    const cuuint64_t dim[2] = {cuuint64_t(cols), cuuint64_t(rows)};
    const cuuint64_t stride[1] = {cuuint64_t(cols) * 2};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estride[2] = {1, 1};
    return int(encode(m, dt, 2, const_cast<void *>(base), dim, stride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, promo, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
}

// w [G, n, k] as a 3-D map (k, n, G): a box never crosses into the next expert.
int encode_w(EncodeTiledFn encode, CUtensorMap *m, CUtensorMapDataType dt, const void *w, int64_t n, int64_t k,
             int64_t G, uint32_t box_k, uint32_t box_n) {
    const cuuint64_t dim[3] = {cuuint64_t(k), cuuint64_t(n), cuuint64_t(G)};
    const cuuint64_t stride[2] = {cuuint64_t(k) * 2, cuuint64_t(n) * cuuint64_t(k) * 2};
    const cuuint32_t box[3] = {box_k, box_n, 1};
    const cuuint32_t estride[3] = {1, 1, 1};
    return int(encode(m, dt, 3, const_cast<void *>(w), dim, stride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
}

// A row-major [rows, cols] operand read MN-major (cols % 64 == 0) as a 3-D view: 64 columns, rows,
// cols / 64 chunks 128 bytes apart. One box (64 x box_rows x chunks) lands in shared memory as
// `chunks` consecutive 64 x box_rows boxes with the same 128-byte swizzle, so it replaces that many
// 2-D box loads; every address it reads stays inside its row (column c * 64 + i < cols).
int encode_mn_chunks(EncodeTiledFn encode, CUtensorMap *m, CUtensorMapDataType dt, const void *base, int64_t cols,
                     int64_t rows, uint32_t box_rows, uint32_t chunks) {
    const cuuint64_t dim[3] = {64, cuuint64_t(rows), cuuint64_t(cols / 64)};
    const cuuint64_t stride[2] = {cuuint64_t(cols) * 2, 128};
    const cuuint32_t box[3] = {64, box_rows, chunks};
    const cuuint32_t estride[3] = {1, 1, 1};
    return int(encode(m, dt, 3, const_cast<void *>(base), dim, stride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
}

int prepare_op(gg_handle *h, const OpProblem &q, gg_stream_t stream, char *why, size_t why_len) {
    const int op = q.op;
    // ---- argument checks (host only; an unsupported shape is an N/A, not an error) ----
    if (q.dtype != GG_BF16 && q.dtype != GG_FP16)
        return refuse(h, why, why_len, "dtype must be bf16 (0) or fp16 (1)");
    if (q.group_num < 1)
        return refuse(h, why, why_len, "group_num must be >= 1");
    if (!q.group_m)
        return refuse(h, why, why_len, "group_m is null");
    if (q.n < 1 || q.k < 1)
        return refuse(h, why, why_len, "n and k must be >= 1");
    if (q.k % 8 != 0)
        return refuse(h, why, why_len, "k must be a multiple of 8 (16-byte TMA row stride)");
    if (q.n % 8 != 0)
        return refuse(h, why, why_len, "n must be a multiple of 8 (16-byte output row stride)");
    if (q.n > (int64_t(1) << 30) || q.k > (int64_t(1) << 30))
        return refuse(h, why, why_len, "n and k must be below 2^30");
    int64_t total_m = 0;
    for (int g = 0; g < q.group_num; ++g) {
        if (q.group_m[g] < 0)
            return refuse(h, why, why_len, "group_m entries must be >= 0");
        total_m += q.group_m[g];
        if (total_m >= (int64_t(1) << 31))
            return refuse(h, why, why_len, "sum(group_m) must be below 2^31");
    }
    if (op == gg::kOpForward) {
        if (total_m > 0 && (!q.a || !q.b || !q.out))
            return refuse(h, why, why_len, "x, w and out must be non-null device pointers");
        if ((reinterpret_cast<uintptr_t>(q.a) | reinterpret_cast<uintptr_t>(q.b) | reinterpret_cast<uintptr_t>(q.out)) &
            15u)
            return refuse(h, why, why_len, "x, w and out must be 16-byte aligned");
    } else {
        const char *names = op == gg::kOpDgrad ? "dy, w and dx" : "dy, x and dw";
        char msg[96];
        if ((total_m > 0 && (!q.a || !q.b)) || ((total_m > 0 || op == gg::kOpWgrad) && !q.out)) {
            std::snprintf(msg, sizeof(msg), "%s must be non-null device pointers", names);
            return refuse(h, why, why_len, msg);
        }
        if ((reinterpret_cast<uintptr_t>(q.a) | reinterpret_cast<uintptr_t>(q.b) | reinterpret_cast<uintptr_t>(q.out)) &
            15u) {
            std::snprintf(msg, sizeof(msg), "%s must be 16-byte aligned", names);
            return refuse(h, why, why_len, msg);
        }
    }
    if (int64_t(q.group_num) * q.n * q.k >= (int64_t(1) << 40) / 2)
        return refuse(h, why, why_len, "weight tensor too large for one TMA descriptor");
    if (op == gg::kOpWgrad && int64_t(q.group_num) * q.n >= (int64_t(1) << 31))
        return refuse(h, why, why_len, "group_num * n must be below 2^31 for wgrad");
    if (op == gg::kOpWgrad && h->opt_split > 1)
        return refuse(h, why, why_len, "split-K is not available for wgrad (per-group reduction lengths)");
    if (op == gg::kOpWgrad && h->opt_stream_k > 0)
        return refuse(h, why, why_len, "stream-K is not available for wgrad (per-group reduction lengths)");
    if (h->opt_split > 1 && h->opt_stream_k > 0)
        return refuse(h, why, why_len, "split > 1 and stream_k > 0 exclude each other");

    // The problem as the cost model sees it: rows per group, output columns, reduction length.
    const int G = q.group_num;
    const int64_t out_cols = op == gg::kOpForward ? q.n : q.k;
    std::vector<int64_t> wrows;
    gg_problem cm{q.dtype, G, out_cols, op == gg::kOpForward ? q.k : q.n, q.group_m, q.a, q.b, q.out};
    if (op == gg::kOpWgrad) {
        wrows.assign(size_t(G), q.n);
        cm.group_m = wrows.data();
        cm.k = std::max<int64_t>(8, (total_m + G - 1) / G);  // mean tokens per expert
    }
    const bool mn_b = op != gg::kOpForward;

    // ---- device + variant ----
    int dev = 0;
    GG_CUDA(h, cudaGetDevice(&dev));
    int num_sms = 0, cc_major = 0, cc_minor = 0;
    GG_CUDA(h, cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev));
    GG_CUDA(h, cudaDeviceGetAttribute(&cc_major, cudaDevAttrComputeCapabilityMajor, dev));
    GG_CUDA(h, cudaDeviceGetAttribute(&cc_minor, cudaDevAttrComputeCapabilityMinor, dev));
    if (cc_major != 10 || cc_minor != 0)
        return refuse(h, why, why_len, "needs an sm_100 GPU (B200/GB200)");
    EncodeTiledFn encode = get_encode_fn();
    if (!encode)
        return fail(h, GG_ERR_CUDA, "cuTensorMapEncodeTiled not available from the driver");

    // Co-resident CTA pairs of the 2-CTA variant (the cost model's slot count for it).
    int pairs = 0;
    {
        const Variant &v0 = variant_at(0);
        const void *fn0 = v0.fn[op][q.dtype];
        GG_CUDA(h, cudaFuncSetAttribute(fn0, cudaFuncAttributeMaxDynamicSharedMemorySize, v0.smem));
        cudaLaunchConfig_t cfg{};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(num_sms, 1, 1);
        cfg.blockDim = dim3(gg::kThreads, 1, 1);
        cfg.dynamicSmemBytes = size_t(v0.smem);
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        GG_CUDA(h, cudaOccupancyMaxActiveClusters(&pairs, fn0, &cfg));
    }
    if (h->opt_max_ctas > 0) {
        pairs = std::min(pairs, h->opt_max_ctas / 2);
        num_sms = std::min(num_sms, h->opt_max_ctas);
    }
    if (h->opt_bn > 0 && h->opt_variant >= 0 && h->opt_bn > variant_at(h->opt_variant).bn)
        return refuse(h, why, why_len, "bn is wider than the variant's tile");
    // split-K candidates: auto (up to 4) unless forced; never when the fp32 partials would be
    // large; wgrad never splits
    int max_splits = h->opt_split > 0 ? h->opt_split : 4;
    if (double(total_m) * double(out_cols) * 4.0 * max_splits > 512.0 * (1 << 20))
        max_splits = h->opt_split > 0 ? h->opt_split : 1;
    if (op == gg::kOpWgrad)
        max_splits = 1;
    if (h->opt_split > 1 && h->opt_split > (cm.k + gg::kBK - 1) / gg::kBK)
        return refuse(h, why, why_len, "split exceeds the number of 64-wide K atoms");
    // a forced split count is used exactly (the tiling is chosen for it)
    // stream-K is tried unless split-K is forced (or for wgrad)
    const int stream_k = op == gg::kOpWgrad || h->opt_split > 1 ? 0 : h->opt_stream_k;
    const Choice ch = gg::choose_tiling(tile_shapes(), kNumVariants, &cm, num_sms, pairs, h->opt_variant, h->opt_bn, max_splits, mn_b,
                                    h->opt_split > 1 && op != gg::kOpWgrad ? h->opt_split : 1, h->opt_sk_tail,
                                    stream_k);
    if (ch.variant < 0)
        return refuse(h, why, why_len,
                      mn_b && h->opt_bn > 0    ? "bn must be a multiple of 64 per CTA for a backward operation"
                      : stream_k > 0        ? "stream_k: this tiling has no partial last wave (or too few tiles) to "
                                              "spread"
                      : h->opt_sk_tail == 1 ? "split_tail=1: this tiling has no partial last wave to split"
                                            : "no kernel variant fits this device and these options");
    const int vi = ch.variant;
    const int bn = ch.bn;
    const Variant &v = variant_at(vi);
    const void *fn = v.fn[op][q.dtype];

    // ---- split launch for skewed routing ----
    // A group whose last 256-row pair tile would hold at most 128 rows (a small expert, or the
    // remainder of a larger one) wastes over half of that tile. With the 2-CTA variant chosen for
    // forward / dgrad and whole tiles, such remainders go to a second launch of the one-CTA kernel
    // (128-row tiles), and the pair kernel covers each group's other rows; automatic when at least
    // 5% of the pair m-tiles are such remainders.
    std::vector<int64_t> small(size_t(G), 0);
    bool tail = false;
    if (v.cg == 2 && op != gg::kOpWgrad && ch.splits <= 1 && ch.sk == 0 && h->opt_tail != 0) {
        int64_t n_small = 0, n_mt = 0;
        for (int g = 0; g < G; ++g) {
            const int64_t rem = q.group_m[g] % 256;
            if (rem > 0 && rem <= 128) {
                small[size_t(g)] = rem;
                ++n_small;
            }
            n_mt += (q.group_m[g] + 255) / 256;
        }
        tail = n_small > 0 && (h->opt_tail == 1 || 20 * n_small >= n_mt);
        if (!tail)
            std::fill(small.begin(), small.end(), 0);
    }

    // ---- group arguments: tile offsets (this tiling) and row (token) offsets; with a split launch
    // also the rows each launch covers per group, then the tail launch's tables ----
    const int64_t tiles_n = (out_cols + bn - 1) / bn;
    const size_t T1 = size_t(G + 1);  // entries of one offset table
    std::vector<int32_t> meta(tail ? 6 * size_t(G) + 4 : 2 * T1);
    int64_t tiles = 0, rows = 0, tail_tiles = 0;
    for (int g = 0; g < G; ++g) {
        meta[size_t(g)] = int32_t(tiles);
        meta[T1 + size_t(g)] = int32_t(rows);
        tiles += (cm.group_m[g] - small[size_t(g)] + v.cluster_m - 1) / v.cluster_m * tiles_n;
        if (tail) {
            meta[2 * T1 + size_t(g)] = int32_t(q.group_m[g] - small[size_t(g)]);              // pair rows
            meta[2 * T1 + size_t(G) + size_t(g)] = int32_t(tail_tiles);                         // tail tile_off
            meta[3 * T1 + size_t(G) + size_t(g)] = int32_t(rows + q.group_m[g] - small[size_t(g)]);  // tail row_off
            meta[4 * T1 + size_t(G) + size_t(g)] = int32_t(small[size_t(g)]);                   // tail rows
            tail_tiles += small[size_t(g)] > 0 ? tiles_n : 0;
        }
        rows += q.group_m[g];
        if (tiles >= (int64_t(1) << 31))
            return refuse(h, why, why_len, "too many tiles");
    }
    meta[size_t(G)] = int32_t(tiles);
    meta[T1 + size_t(G)] = int32_t(rows);
    if (tail) {
        meta[2 * T1 + 2 * size_t(G)] = int32_t(tail_tiles);
        meta[3 * T1 + 2 * size_t(G)] = int32_t(rows);
    }
    // Split-K form: every tile split, or (hybrid) only as many tiles as would form a partial last
    // wave; the split tiles' units run first, the whole tiles after them.
    // Stream-K instead: the first sk_tiles tiles' atoms dealt out evenly to every cluster.
    const int64_t clusters = std::max(1, v.cg == 2 ? pairs : num_sms);
    const int64_t atoms = (cm.k + gg::kBK - 1) / gg::kBK;
    const int64_t sk_tiles = ch.sk > 0 ? gg::sk_tiles_for(tiles, clusters, atoms, ch.sk) : 0;
    const bool partials = ch.splits > 1 || sk_tiles > 0;  // fp32 workspace + arrival counters
    const int64_t split_tiles = sk_tiles > 0 ? sk_tiles : ch.splits > 1 ? (ch.hybrid ? tiles % clusters : tiles) : 0;
    const int64_t units = sk_tiles > 0 ? clusters : tiles + split_tiles * (ch.splits - 1);

    if (h->meta_cap < meta.size()) {
        if (h->d_meta)
            cudaFree(h->d_meta);
        h->d_meta = nullptr;
        h->meta_cap = 0;
        GG_CUDA(h, cudaMalloc(&h->d_meta, meta.size() * sizeof(int32_t)));
        h->meta_cap = meta.size();
    }
    // status word [0] and the dynamic-dispatch tile counter [1], both zero between launches
    if (!h->d_status)
        GG_CUDA(h, cudaMalloc(&h->d_status, 16));
    GG_CUDA(h, cudaMemsetAsync(h->d_status, 0, 16, stream));
    if (partials) {
        // tile-private partials: per split tile and CTA, 128 rows x bn fp32 (rounded up to whole
        // 32-column chunks) per split / piece
        const size_t ws_bytes = size_t(split_tiles) * size_t(v.cg) * size_t(ch.splits) * 128 *
                                size_t((bn + 31) / 32 * 32) * sizeof(float);
        const size_t ctr_bytes = size_t(split_tiles) * size_t(v.cg) * 4 * sizeof(int32_t);
        if (h->ws_cap < ws_bytes) {
            if (h->d_ws)
                cudaFree(h->d_ws);
            h->d_ws = nullptr;
            h->ws_cap = 0;
            GG_CUDA(h, cudaMalloc(&h->d_ws, ws_bytes));
            h->ws_cap = ws_bytes;
        }
        if (h->counters_cap < ctr_bytes) {
            if (h->d_counters)
                cudaFree(h->d_counters);
            h->d_counters = nullptr;
            h->counters_cap = 0;
            GG_CUDA(h, cudaMalloc(&h->d_counters, ctr_bytes));
            h->counters_cap = ctr_bytes;
        }
        GG_CUDA(h, cudaMemsetAsync(h->d_counters, 0, ctr_bytes, stream));
    }
    GG_CUDA(h, cudaMemcpyAsync(h->d_meta, meta.data(), meta.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                               stream));

    // Half-height pair tiles for groups that end in a remainder of at most 128 rows (pair variant,
    // forward / dgrad, whole tiles, a tile width the M = 128 pair MMA takes).
    bool half_tiles = false;
    if (v.cg == 2 && op != gg::kOpWgrad && !partials && bn % 32 == 0 && h->opt_half != 0)
        for (int g = 0; g < G && !half_tiles; ++g)
            half_tiles = ((q.group_m[g] - small[size_t(g)]) % 256) != 0 && ((q.group_m[g] - small[size_t(g)]) % 256) <= 128;

    // ---- TMA descriptors ----
    const CUtensorMapDataType dt =
        q.dtype == GG_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint32_t b_box = uint32_t(bn / v.cg);
    h->tmap_a = CUtensorMap{};
    h->tmap_a_half = CUtensorMap{};
    h->tmap_b = CUtensorMap{};
    h->tmap_out = CUtensorMap{};
    std::vector<CUtensorMap> gmaps;
    int mn_chunks = 0;
    if (op == gg::kOpForward && total_m > 0) {
        if (encode_2d(encode, &h->tmap_a, dt, q.a, q.k, total_m, gg::kBK, gg::kBM, CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
            return fail(h, GG_ERR_CUDA, "cuTensorMapEncodeTiled(x) failed");
        if (half_tiles && encode_2d(encode, &h->tmap_a_half, dt, q.a, q.k, total_m, gg::kBK, 64,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
            return fail(h, GG_ERR_CUDA, "cuTensorMapEncodeTiled(x, 64-row boxes) failed");
        if (encode_w(encode, &h->tmap_b, dt, q.b, q.n, q.k, G, gg::kBK, b_box))
            return fail(h, GG_ERR_CUDA, "cuTensorMapEncodeTiled(w) failed");
        // out [sum(M), N]: the epilogue's TMA stores, 32 rows x 64 columns per box
        if (encode_2d(encode, &h->tmap_out, dt, q.out, q.n, total_m, 64, 32, CU_TENSOR_MAP_L2_PROMOTION_NONE))
            return fail(h, GG_ERR_CUDA, "cuTensorMapEncodeTiled(out) failed");
    } else if (op == gg::kOpDgrad && total_m > 0) {
        // A = dy [sum(M), N], K-major over N; B = w[g] read as 64 (K) x 64 (N) MN-major boxes
        if (encode_2d(encode, &h->tmap_a, dt, q.a, q.n, total_m, gg::kBK, gg::kBM, CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
            return fail(h, GG_ERR_CUDA, "cuTensorMapEncodeTiled(dy) failed");
        if (half_tiles && encode_2d(encode, &h->tmap_a_half, dt, q.a, q.n, total_m, gg::kBK, 64,
                                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B))
            return fail(h, GG_ERR_CUDA, "cuTensorMapEncodeTiled(dy, 64-row boxes) failed");
        if (encode_w(encode, &h->tmap_b, dt, q.b, q.n, q.k, G, 64, gg::kBK))
            return fail(h, GG_ERR_CUDA, "cuTensorMapEncodeTiled(w) failed");
        if (encode_2d(encode, &h->tmap_out, dt, q.out, q.k, total_m, 64, 32, CU_TENSOR_MAP_L2_PROMOTION_NONE))
            return fail(h, GG_ERR_CUDA, "cuTensorMapEncodeTiled(dx) failed");
    } else if (op == gg::kOpWgrad) {
        // Per group: dy rows and x rows of the group's tokens, each bounded by the group so that the
        // token tail reads zeros; 64 x 64 MN-major boxes, or (N, resp. K, a multiple of 64) the 3-D
        // chunk view that loads a CTA's 64-column chunks of an atom in one box. An empty group's
        // maps are never read.
        mn_chunks = h->opt_chunks != 0 ? (q.n % 64 == 0 ? 1 : 0) | (q.k % 64 == 0 ? 2 : 0) : 0;
        gmaps.assign(2 * size_t(G), CUtensorMap{});
        int64_t r0 = 0;
        for (int g = 0; g < G; ++g) {
            const int64_t m = q.group_m[g];
            if (m > 0) {
                const char *dy = static_cast<const char *>(q.a) + r0 * q.n * 2;
                const char *x = static_cast<const char *>(q.b) + r0 * q.k * 2;
                const int ea = (mn_chunks & 1)
                                   ? encode_mn_chunks(encode, &gmaps[2 * g], dt, dy, q.n, m, gg::kBK, uint32_t(gg::kBM / 64))
                                   : encode_2d(encode, &gmaps[2 * g], dt, dy, q.n, m, 64, gg::kBK, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
                const int eb = (mn_chunks & 2)
                                   ? encode_mn_chunks(encode, &gmaps[2 * g + 1], dt, x, q.k, m, gg::kBK, b_box / 64)
                                   : encode_2d(encode, &gmaps[2 * g + 1], dt, x, q.k, m, 64, gg::kBK, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
                if (ea || eb)
                    return fail(h, GG_ERR_CUDA, "cuTensorMapEncodeTiled(group %d) failed", g);
            }
            r0 += m;
        }
        if (encode_2d(encode, &h->tmap_out, dt, q.out, q.k, int64_t(G) * q.n, 64, 32, CU_TENSOR_MAP_L2_PROMOTION_NONE))
            return fail(h, GG_ERR_CUDA, "cuTensorMapEncodeTiled(dw) failed");
        if (h->gmaps_cap < gmaps.size()) {
            if (h->d_gmaps)
                cudaFree(h->d_gmaps);
            h->d_gmaps = nullptr;
            h->gmaps_cap = 0;
            GG_CUDA(h, cudaMalloc(&h->d_gmaps, gmaps.size() * sizeof(CUtensorMap)));
            h->gmaps_cap = gmaps.size();
        }
        GG_CUDA(h, cudaMemcpyAsync(h->d_gmaps, gmaps.data(), gmaps.size() * sizeof(CUtensorMap),
                                   cudaMemcpyHostToDevice, stream));
    }

    // ---- raster band and persistent grid ----
    int band = h->opt_band;
    const int raster = h->opt_raster < 0 ? 0 : h->opt_raster;
    if (band <= 0) {
        // Enough m-tiles per band that one wave of tiles spans few weight panels.
        band = v.cg == 2 ? 8 : 16;
    }
    GG_CUDA(h, cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, v.smem));
    const int slots = v.cg == 2 ? 2 * pairs : num_sms;  // CTAs that can be resident at once
    if (slots < v.cg)
        return refuse(h, why, why_len, "no CTA of this kernel fits on the device");
    const int64_t want = units * v.cg;
    h->grid = int(std::max<int64_t>(v.cg, std::min<int64_t>(slots, want)));

    gg::KernelParams &kp = h->params;
    kp = gg::KernelParams{};
    kp.tile_off = h->d_meta;
    kp.row_off = h->d_meta + (G + 1);
    kp.row_cnt = tail ? h->d_meta + 2 * (G + 1) : nullptr;
    kp.out = q.out;
    kp.status = h->d_status;
    kp.gmaps = op == gg::kOpWgrad ? h->d_gmaps : nullptr;
    kp.group_num = G;
    kp.n = int32_t(out_cols);
    kp.k = int32_t(op == gg::kOpForward ? q.k : q.n);
    kp.tile_rows = op == gg::kOpWgrad ? int32_t(q.n) : 0;
    kp.num_kb = int32_t((kp.k + gg::kBK - 1) / gg::kBK);
    kp.tiles_n = int32_t(tiles_n);
    kp.bn = bn;
    kp.total_tiles = int32_t(tiles);
    kp.splits = ch.splits;
    kp.split_tiles = sk_tiles > 0 ? 0 : int32_t(split_tiles);
    kp.sk_tiles = int32_t(sk_tiles);
    kp.ws = partials ? h->d_ws : nullptr;
    kp.counters = partials ? h->d_counters : nullptr;
    kp.band = band;
    kp.raster = raster;
    // epilogue store path: direct stores for tiles with >= 16 K atoms (1024 of reduction)
    kp.store_min_atoms = h->opt_store == 0 ? (1 << 30) : h->opt_store == 1 ? 0 : 16;
    kp.test_stall = h->opt_test_stall;
    kp.half_tiles = half_tiles && total_m > 0 ? 1 : 0;
    kp.mn_chunks = mn_chunks;
    // L2 policy of the operand loads. Automatic: where the weights outweigh the activations at
    // least 4 : 1 (few tokens per expert, many experts: config E) and the launch runs at least 64
    // waves, the weights stream through L2 once while the clusters drift apart, and they push out
    // activation rows that later n-tiles of the same expert still read; those loads are marked
    // evict_last. Measured (interleaved, 8-10 rounds, both orders on one box): E (110 waves) +9.5%
    // on two boxes, +0.6% on a third that ran E power-capped at ~1100 TFLOPS; its 2-, 4- and 8-GPU
    // shares (55 / 28 / 14 waves) unchanged within noise, so they keep no hint; L / P / D slower.
    const double act_elems = double(total_m) * double(kp.k);
    const double w_elems = double(G) * double(q.n) * double(q.k);
    const bool long_launch = tiles >= 64 * int64_t(std::max(1, h->grid / v.cg));
    kp.l2_a = op != gg::kOpForward ? 0
              : h->opt_l2_a >= 0 ? h->opt_l2_a
                                 : (w_elems >= 4.0 * act_elems && long_launch ? 2 : 0);
    kp.l2_b = op != gg::kOpForward ? 0 : h->opt_l2_b;
    kp.out_rows = int32_t(op == gg::kOpWgrad ? int64_t(G) * q.n : total_m) - h->opt_test_bounds;
    kp.ws_float4s = partials ? int64_t(h->ws_cap / 16) : 0;
    kp.ctr_entries = partials ? int32_t(h->counters_cap / sizeof(int32_t)) : 0;
    kp.timeout_ns = uint64_t(h->opt_timeout_ms) * 1000000ull;
    // Planned tile order (skewed routing): tiles of two kinds, bound by different resources, run
    // as separate phases in group order; the interleaved order (gg::interleave_tiles) with dynamic
    // dispatch lets them overlap.
    //   wgrad: an expert with few tokens has a short reduction, so its tiles are bound by their
    //     stores (a whole tile of output each), a large expert's by the tensor pipe. Estimates per
    //     tile: bn/2 cycles per MMA (the tensor rate), ~11 bn cycles for the epilogue's stores.
    //   forward / dgrad (one launch, no split launch): a tile streams its weight panel (bn/kCG rows
    //     of the reduction per CTA) from DRAM once per group, shared by the group's m-tiles; an
    //     expert with few tokens has few m-tiles to share it, so its tiles are bound by DRAM
    //     (~40 B/cycle per SM, its share of HBM), a large expert's by the tensor pipe (bn/2 cycles
    //     per MMA, half that for a half-height tile).
    bool planned = false;
    const bool plan_ok = op == gg::kOpWgrad || !tail;
    if (plan_ok && !partials && h->opt_order != 0 && tiles > 0) {
        std::vector<double> cost(size_t(G), 0.0);
        std::vector<char> store_bound(size_t(G), 0);
        double work[2] = {0, 0};
        const double epi = 11.0 * bn;
        for (int g = 0; g < G; ++g) {
            double mma, other;
            if (op == gg::kOpWgrad) {
                mma = double((q.group_m[g] + gg::kBK - 1) / gg::kBK) * 4.0 * 0.5 * bn;
                other = epi;
            } else {
                const int64_t mtiles = std::max<int64_t>(1, (q.group_m[g] + v.cluster_m - 1) / v.cluster_m);
                const bool half_only = half_tiles && mtiles == 1 && q.group_m[g] <= v.cluster_m / 2;
                mma = double(kp.num_kb) * 4.0 * 0.5 * bn * (half_only ? 0.5 : 1.0);
                other = double(bn / v.cg) * double(kp.k) * 2.0 / 40.0 / double(mtiles);
            }
            cost[size_t(g)] = std::max(mma, other);
            store_bound[size_t(g)] = mma < other ? 1 : 0;
            work[store_bound[size_t(g)]] += cost[size_t(g)] * double(meta[size_t(g) + 1] - meta[size_t(g)]);
        }
        const double all = work[0] + work[1];
        planned = h->opt_order == 1 || (work[0] > 0.05 * all && work[1] > 0.05 * all);
        if (planned) {
            // the tiles in group order, from the kernel's own decode over the host tables
            gg::KernelParams hp = kp;
            hp.tile_off = meta.data();
            hp.row_off = meta.data() + (G + 1);
            hp.row_cnt = nullptr;
            hp.tile_list = nullptr;
            std::vector<int32_t> natural(2 * size_t(tiles)), order;
            int cursor = 0;
            for (int64_t t = 0; t < tiles; ++t) {
                gg::TileCoord tc;
                if (op == gg::kOpWgrad)
                    tc = v.cluster_m == 256 ? gg::decode_tile<256, gg::kOpWgrad>(hp, int(t), cursor)
                                            : gg::decode_tile<128, gg::kOpWgrad>(hp, int(t), cursor);
                else
                    tc = v.cluster_m == 256 ? gg::decode_tile<256, gg::kOpForward>(hp, int(t), cursor)
                                            : gg::decode_tile<128, gg::kOpForward>(hp, int(t), cursor);
                natural[2 * size_t(t)] = tc.g;
                natural[2 * size_t(t) + 1] = (tc.mt << 16) | tc.nt;
            }
            gg::interleave_tiles(natural, cost, store_bound, order);
            if (h->tiles_cap < order.size()) {
                if (h->d_tiles)
                    cudaFree(h->d_tiles);
                h->d_tiles = nullptr;
                h->tiles_cap = 0;
                GG_CUDA(h, cudaMalloc(&h->d_tiles, order.size() * sizeof(int32_t)));
                h->tiles_cap = order.size();
            }
            GG_CUDA(h, cudaMemcpyAsync(h->d_tiles, order.data(), order.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                                       stream));
            GG_CUDA(h, cudaStreamSynchronize(stream));  // `order` is a host temporary
        }
    }
    kp.tile_list = planned ? h->d_tiles : nullptr;
    // Dynamic tile dispatch (whole tiles only): clusters take the next tile from a counter as they
    // finish one, so tiles that share a weight panel run at the same time all through the launch
    // (a static round-robin lets clusters drift apart); automatic for launches of more than one
    // wave. A planned tile order is dealt out either way.
    const bool dynamic = !partials && (h->opt_sched == 1 || (h->opt_sched < 0 && units * v.cg > h->grid));
    kp.tile_ctr = dynamic ? reinterpret_cast<int32_t *>(h->d_status) + 1 : nullptr;

    // The tail launch: the one-CTA 128-row kernel over the remainders, same tile width, static
    // schedule, whole tiles; its own weight map (each CTA loads all bn weight rows of a tile).
    h->tail.active = false;
    h->tail.tmap_b = CUtensorMap{};
    if (tail && tail_tiles > 0) {
        const Variant &tv = variant_at(1);
        if (op == gg::kOpForward) {
            if (encode_w(encode, &h->tail.tmap_b, dt, q.b, q.n, q.k, G, gg::kBK, uint32_t(bn)))
                return fail(h, GG_ERR_CUDA, "cuTensorMapEncodeTiled(w, tail launch) failed");
        } else {
            h->tail.tmap_b = h->tmap_b;  // dgrad: 64 x 64 MN-major boxes either way
        }
        GG_CUDA(h, cudaFuncSetAttribute(tv.fn[op][q.dtype], cudaFuncAttributeMaxDynamicSharedMemorySize, tv.smem));
        gg::KernelParams &tp = h->tail.params;
        tp = kp;
        tp.tile_off = h->d_meta + 2 * (G + 1) + G;
        tp.row_off = h->d_meta + 3 * (G + 1) + G;
        tp.row_cnt = h->d_meta + 4 * (G + 1) + G;
        tp.total_tiles = int32_t(tail_tiles);
        tp.band = 16;
        tp.tile_ctr = nullptr;
        tp.tile_list = nullptr;
        tp.half_tiles = 0;
        tp.test_stall = 0;
        h->tail.fn = tv.fn[op][q.dtype];
        h->tail.smem = tv.smem;
        h->tail.grid = int(std::min<int64_t>(num_sms, tail_tiles));
        h->tail.active = true;
    }

    GG_CUDA(h, cudaStreamSynchronize(stream));

    h->device = dev;
    h->dtype = q.dtype;
    h->op = op;
    h->variant = vi;
    h->total_m = total_m;
    h->fn = fn;
    h->smem = v.smem;
    h->cg = v.cg;
    char form[224];
    if (sk_tiles > 0)
        std::snprintf(form, sizeof(form), "split=1 stream_k=%lld tiles(<=%d pieces)", (long long)sk_tiles, ch.splits);
    else
        std::snprintf(form, sizeof(form), "split=%d%s%s%s%s%s%s%s", ch.splits,
                      split_tiles > 0 && split_tiles < tiles ? "(last wave)" : "", dynamic ? " dynamic" : "",
                      half_tiles ? " half-tiles" : "", planned ? " interleaved" : "",
                      mn_chunks == 3 ? " chunk-boxes" : mn_chunks == 1 ? " chunk-boxes(dy)" : mn_chunks == 2 ? " chunk-boxes(x)" : "",
                      kp.l2_a == 2 ? " a:evict_last" : kp.l2_a == 1 ? " a:evict_first" : "",
                      kp.l2_b == 2 ? " b:evict_last" : kp.l2_b == 1 ? " b:evict_first" : "");
    char tail_form[96] = "";
    if (h->tail.active)
        std::snprintf(tail_form, sizeof(tail_form), " +tail gg_sm100 tile=128x%d cta_group=1 tiles=%lld grid=%d", bn,
                      (long long)tail_tiles, h->tail.grid);
    char d[384];
    std::snprintf(d, sizeof(d), "gg_sm100<%s%s%s> tile=%dx%dx%d cta_group=%d stages=%d tiles=%lld %s grid=%d band=%d%s%s",
                  q.dtype == GG_BF16 ? "bf16" : "fp16", op == gg::kOpForward ? "" : ",", op == gg::kOpForward ? "" : op_name(op),
                  v.cluster_m, bn, gg::kBK * v.atoms, v.cg, v.stages_for(bn / v.cg), (long long)tiles, form, h->grid, band,
                  raster ? "n" : "", tail_form);
    h->detail = d;
    h->ready = true;
    return GG_OK;
}

}  // namespace

extern "C" {

int gg_prepare(gg_handle *h, const gg_problem *p, gg_stream_t stream, char *why, size_t why_len) {
    if (!h)
        return GG_ERR_ARG;
    h->ready = false;
    h->last_error.clear();
    if (why && why_len)
        why[0] = '\0';
    if (!p)
        return fail(h, GG_ERR_ARG, "null problem");
    const OpProblem q{gg::kOpForward, p->dtype, p->group_num, p->n, p->k, p->group_m, p->x, p->w, p->out};
    return prepare_op(h, q, stream, why, why_len);
}

int gg_prepare_grad(gg_handle *h, const gg_grad_problem *p, int32_t op, gg_stream_t stream, char *why,
                    size_t why_len) {
    if (!h)
        return GG_ERR_ARG;
    h->ready = false;
    h->last_error.clear();
    if (why && why_len)
        why[0] = '\0';
    if (!p)
        return fail(h, GG_ERR_ARG, "null problem");
    if (op == GG_OP_DGRAD) {
        const OpProblem q{gg::kOpDgrad, p->dtype, p->group_num, p->n, p->k, p->group_m, p->dy, p->w, p->dx};
        return prepare_op(h, q, stream, why, why_len);
    }
    if (op == GG_OP_WGRAD) {
        const OpProblem q{gg::kOpWgrad, p->dtype, p->group_num, p->n, p->k, p->group_m, p->dy, p->x, p->dw};
        return prepare_op(h, q, stream, why, why_len);
    }
    return fail(h, GG_ERR_ARG, "op must be GG_OP_DGRAD (1) or GG_OP_WGRAD (2)");
}

int gg_run(gg_handle *h, gg_stream_t stream) {
    if (!h)
        return GG_ERR_ARG;
    if (!h->ready)
        return fail(h, GG_ERR_ARG, "gg_run before a successful gg_prepare");
    if (h->params.total_tiles == 0 && !h->tail.active)
        return GG_OK;  // every group empty: nothing to write
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(h->cg);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // Programmatic dependent launch: this grid may be scheduled while the previous kernel in the
    // stream finishes; the kernel waits for it (griddepcontrol.wait) before reading or writing
    // global memory, so only launch latency and on-chip set-up overlap.
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(unsigned(h->grid), 1, 1);
    cfg.blockDim = dim3(gg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = size_t(h->smem);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = h->opt_pdl ? 2 : 1;
    if (h->params.total_tiles > 0) {
        void *args[5] = {&h->tmap_a, &h->tmap_b, &h->tmap_out, &h->tmap_a_half, &h->params};
        GG_CUDA(h, cudaLaunchKernelExC(&cfg, h->fn, args));
    }
    if (h->tail.active) {
        // split launch: the one-CTA kernel over the groups' remainders (rows disjoint from the first
        // launch's), behind it in the stream
        attr[0].val.clusterDim.x = 1;
        cfg.gridDim = dim3(unsigned(h->tail.grid), 1, 1);
        cfg.dynamicSmemBytes = size_t(h->tail.smem);
        void *args[5] = {&h->tmap_a, &h->tail.tmap_b, &h->tmap_out, &h->tmap_a_half, &h->tail.params};
        GG_CUDA(h, cudaLaunchKernelExC(&cfg, h->tail.fn, args));
    }
    return GG_OK;
}

int gg_device_status(gg_handle *h, gg_stream_t stream, uint32_t *status) {
    if (!h || !status)
        return GG_ERR_ARG;
    *status = 0;
    if (!h->d_status)
        return GG_OK;
    GG_CUDA(h, cudaStreamSynchronize(stream));
    GG_CUDA(h, cudaMemcpy(status, h->d_status, sizeof(uint32_t), cudaMemcpyDeviceToHost));
    GG_CUDA(h, cudaMemset(h->d_status, 0, sizeof(uint32_t)));
    if (*status != 0) {
        // an aborted launch can leave the dynamic-dispatch tile counter behind: clear it
        GG_CUDA(h, cudaMemset(h->d_status, 0, 16));
        // an aborted launch can leave split-K arrival counts behind: clear them
        if (h->d_counters)
            GG_CUDA(h, cudaMemset(h->d_counters, 0, h->counters_cap));
        return fail(h, GG_ERR_DEVICE, "%s: status 0x%x",
                    (*status & gg::kStatusBounds) ? "debug bounds check failed" : "kernel bounded wait timed out", *status);
    }
    return GG_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Entry point that allocates nothing: gg_run_noalloc.
//
// Some callers cannot allocate device memory at the moment they want the GEMM: an inference
// engine that has reserved (nearly) all HBM up front for weights and KV cache through its own
// pool and fails any allocation outside it; a plugin host that hands out a fixed memory budget;
// a latency-critical path where cudaMalloc/cudaFree are off limits because they can synchronise
// the device. gg_prepare() allocates two small device buffers per handle (the per-group tile and
// row offsets, and the kernel's status word), so those callers cannot use it.
//
// gg_run_noalloc keeps that scratch instead in one file-scope device array, g_noalloc_scratch,
// sized for at most kNoAllocMaxGroups groups (about 8 KB). It is part of the library image, so
// every GPU that loads the library holds it until the process exits. The caller still passes x,
// w and out; the library allocates nothing, neither device nor host memory on the heap.
// ---------------------------------------------------------------------------------------------
namespace {

constexpr int kNoAllocMaxGroups = 1024;
constexpr size_t kNoAllocHeader = 256;  // status word, padded to keep the offsets 256-aligned
constexpr size_t kNoAllocScratchBytes = kNoAllocHeader + 2 * (kNoAllocMaxGroups + 1) * sizeof(int32_t);

// Device-side scratch shared by every gg_run_noalloc call on a device. In host code this name
// is only a stand-in for the symbol, never a device address: the address comes from
// cudaGetSymbolAddress (see noalloc_device_setup).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// The group offsets of one call travel to the device as a kernel parameter (a by-value copy
// taken when the launch is enqueued, up to 32 KB on CUDA 12.1+ drivers), and a one-block kernel
// writes them into the scratch array in stream order. So the host neither waits for the stream
// (as a copy from pageable memory would) nor leaves a pointer to its stack behind.
struct NoAllocOffsets {
    int32_t count;                              // entries used: 2 (G + 1)
    int32_t v[2 * (kNoAllocMaxGroups + 1)];     // tile_off[G+1] then row_off[G+1]
};
static_assert(sizeof(NoAllocOffsets) < 32000, "kernel parameter limit");

__global__ void noalloc_publish_offsets(const __grid_constant__ NoAllocOffsets a, int32_t *dst) {
    for (int i = int(threadIdx.x); i < a.count; i += int(blockDim.x))
        dst[i] = a.v[i];
}

constexpr int kNoAllocMaxDevices = 64;

struct NoAllocDevice {
    bool ready = false;
    unsigned char *scratch = nullptr;  // device address of g_noalloc_scratch on this device
    int num_sms = 0;
    int clusters_v0 = 0;  // co-resident CTA pairs of the 256x256 variant (any dtype)
};

std::mutex g_noalloc_mutex;
NoAllocDevice g_noalloc_dev[kNoAllocMaxDevices];

void copy_msg(char *why, size_t why_len, const char *msg) {
    if (why && why_len > 0) {
        std::strncpy(why, msg, why_len - 1);
        why[why_len - 1] = '\0';
    }
}

// One-time set-up of device `dev` (the current device): the scratch address, the SM count, the
// dynamic shared-memory limit of every kernel variant and the pair occupancy of the 2-CTA one.
cudaError_t noalloc_device_setup(int dev, NoAllocDevice &d) {
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void **>(&d.scratch), g_noalloc_scratch);
    if (e != cudaSuccess)
        return e;
    if ((e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return e;
    for (int i = 0; i < kNumVariants; ++i) {
        const Variant &v = variant_at(i);
        for (const void *fn : {v.fn[gg::kOpForward][GG_BF16], v.fn[gg::kOpForward][GG_FP16]})
            if ((e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, v.smem)) != cudaSuccess)
                return e;
    }
    const Variant &v0 = variant_at(0);
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(unsigned(d.num_sms), 1, 1);
    cfg.blockDim = dim3(gg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = size_t(v0.smem);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if ((e = cudaOccupancyMaxActiveClusters(&d.clusters_v0, v0.fn[gg::kOpForward][GG_BF16], &cfg)) != cudaSuccess)
        return e;
    d.ready = true;
    return cudaSuccess;
}

}  // namespace

extern "C" int gg_run_noalloc(const gg_problem *p, gg_stream_t stream, uint32_t *status_out, char *why,
                              size_t why_len) {
    if (why && why_len)
        why[0] = '\0';
    if (status_out)
        *status_out = 0;
    if (!p) {
        copy_msg(why, why_len, "null problem");
        return GG_ERR_ARG;
    }
    // ---- the same shape rules as gg_prepare, plus the scratch limit ----
    const char *bad = nullptr;
    if (p->dtype != GG_BF16 && p->dtype != GG_FP16)
        bad = "dtype must be bf16 (0) or fp16 (1)";
    else if (p->group_num < 1)
        bad = "group_num must be >= 1";
    else if (p->group_num > kNoAllocMaxGroups)
        bad = "group_num exceeds the 1024 groups that gg_run_noalloc's fixed scratch holds";
    else if (!p->group_m)
        bad = "group_m is null";
    else if (p->n < 1 || p->k < 1)
        bad = "n and k must be >= 1";
    else if (p->k % 8 != 0)
        bad = "k must be a multiple of 8 (16-byte TMA row stride)";
    else if (p->n % 8 != 0)
        bad = "n must be a multiple of 8 (16-byte output row stride)";
    else if (p->n > (int64_t(1) << 30) || p->k > (int64_t(1) << 30))
        bad = "n and k must be below 2^30";
    else if (int64_t(p->group_num) * p->n * p->k >= (int64_t(1) << 40) / 2)
        bad = "weight tensor too large for one TMA descriptor";
    int64_t total_m = 0;
    for (int g = 0; !bad && g < p->group_num; ++g) {
        if (p->group_m[g] < 0)
            bad = "group_m entries must be >= 0";
        total_m += p->group_m[g];
        if (total_m >= (int64_t(1) << 31))
            bad = "sum(group_m) must be below 2^31";
    }
    if (!bad && total_m > 0 && (!p->x || !p->w || !p->out))
        bad = "x, w and out must be non-null device pointers";
    if (!bad && ((reinterpret_cast<uintptr_t>(p->x) | reinterpret_cast<uintptr_t>(p->w) |
                  reinterpret_cast<uintptr_t>(p->out)) & 15u))
        bad = "x, w and out must be 16-byte aligned";
    if (bad) {
        copy_msg(why, why_len, bad);
        return GG_NOT_SUPPORTED;
    }

    char msg[256];
    auto cuda_fail = [&](const char *what, cudaError_t e) {
        std::snprintf(msg, sizeof(msg), "%s: %s", what, cudaGetErrorString(e));
        copy_msg(why, why_len, msg);
        return GG_ERR_CUDA;
    };

    // ---- per-device set-up on the first call ----
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return cuda_fail("cudaGetDevice", e);
    if (dev < 0 || dev >= kNoAllocMaxDevices) {
        copy_msg(why, why_len, "device ordinal out of range");
        return GG_ERR_ARG;
    }
    int cc_major = 0, cc_minor = 0;
    if ((e = cudaDeviceGetAttribute(&cc_major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
        (e = cudaDeviceGetAttribute(&cc_minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
        return cuda_fail("cudaDeviceGetAttribute", e);
    if (cc_major != 10 || cc_minor != 0) {
        copy_msg(why, why_len, "needs an sm_100 GPU (B200/GB200)");
        return GG_NOT_SUPPORTED;
    }
    NoAllocDevice *d = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        d = &g_noalloc_dev[dev];
        if (!d->ready && (e = noalloc_device_setup(dev, *d)) != cudaSuccess)
            return cuda_fail("gg_run_noalloc device set-up", e);
    }
    EncodeTiledFn encode = get_encode_fn();
    if (!encode) {
        copy_msg(why, why_len, "cuTensorMapEncodeTiled not available from the driver");
        return GG_ERR_CUDA;
    }

    // ---- variant, group arguments (host stack), descriptors ----
    const Choice ch = gg::choose_tiling(tile_shapes(), kNumVariants, p, d->num_sms, d->clusters_v0, -1, 0, 1);
    if (ch.variant < 0) {
        copy_msg(why, why_len, "no kernel variant fits this device");
        return GG_NOT_SUPPORTED;
    }
    const Variant &v = variant_at(ch.variant);
    const int bn = ch.bn;
    const int G = p->group_num;
    const int64_t tiles_n = (p->n + bn - 1) / bn;
    NoAllocOffsets offs;
    offs.count = 2 * (G + 1);
    int32_t *meta = offs.v;
    int64_t tiles = 0, rows = 0;
    for (int g = 0; g < G; ++g) {
        meta[g] = int32_t(tiles);
        meta[G + 1 + g] = int32_t(rows);
        tiles += (p->group_m[g] + v.cluster_m - 1) / v.cluster_m * tiles_n;
        rows += p->group_m[g];
    }
    if (tiles >= (int64_t(1) << 31)) {
        copy_msg(why, why_len, "too many tiles");
        return GG_NOT_SUPPORTED;
    }
    meta[G] = int32_t(tiles);
    meta[2 * G + 1] = int32_t(rows);
    if (tiles == 0)
        return GG_OK;  // every group empty: nothing to write

    uint32_t *d_status = reinterpret_cast<uint32_t *>(d->scratch);
    int32_t *d_meta = reinterpret_cast<int32_t *>(d->scratch + kNoAllocHeader);
    // The previous call's offsets are still in the array: overwrite them, in stream order behind
    // any earlier call on the same stream. The status word is left alone: a timeout of an earlier
    // call stays recorded until a call with status_out reads and clears it.
    noalloc_publish_offsets<<<1, 256, 0, stream>>>(offs, d_meta);
    if ((e = cudaGetLastError()) != cudaSuccess)
        return cuda_fail("group-offset publish launch", e);

    const CUtensorMapDataType dt =
        p->dtype == GG_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap tmap_a, tmap_b, tmap_out, tmap_unused{};  // no half-height tiles on this path
    if (encode_2d(encode, &tmap_a, dt, p->x, p->k, total_m, gg::kBK, gg::kBM, CU_TENSOR_MAP_L2_PROMOTION_L2_256B)) {
        copy_msg(why, why_len, "cuTensorMapEncodeTiled(x) failed");
        return GG_ERR_CUDA;
    }
    if (encode_w(encode, &tmap_b, dt, p->w, p->n, p->k, G, gg::kBK, uint32_t(bn / v.cg))) {
        copy_msg(why, why_len, "cuTensorMapEncodeTiled(w) failed");
        return GG_ERR_CUDA;
    }
    if (encode_2d(encode, &tmap_out, dt, p->out, p->n, total_m, 64, 32, CU_TENSOR_MAP_L2_PROMOTION_NONE)) {
        copy_msg(why, why_len, "cuTensorMapEncodeTiled(out) failed");
        return GG_ERR_CUDA;
    }

    gg::KernelParams kp{};
    kp.tile_off = d_meta;
    kp.row_off = d_meta + (G + 1);
    kp.out = p->out;
    kp.status = d_status;
    kp.group_num = G;
    kp.n = int32_t(p->n);
    kp.k = int32_t(p->k);
    kp.num_kb = int32_t((p->k + gg::kBK - 1) / gg::kBK);
    kp.tiles_n = int32_t(tiles_n);
    kp.bn = bn;
    kp.total_tiles = int32_t(tiles);
    kp.band = v.cg == 2 ? 8 : 16;
    kp.store_min_atoms = 16;  // the same epilogue store policy as gg_run's default
    kp.out_rows = int32_t(total_m);
    kp.timeout_ns = 2000ull * 1000000ull;

    const int slots = v.cg == 2 ? 2 * d->clusters_v0 : d->num_sms;
    if (slots < v.cg) {
        copy_msg(why, why_len, "no CTA of this kernel fits on the device");
        return GG_NOT_SUPPORTED;
    }
    const int grid = int(std::max<int64_t>(v.cg, std::min<int64_t>(slots, tiles * v.cg)));
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = unsigned(v.cg);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(unsigned(grid), 1, 1);
    cfg.blockDim = dim3(gg::kThreads, 1, 1);
    cfg.dynamicSmemBytes = size_t(v.smem);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void *args[5] = {&tmap_a, &tmap_b, &tmap_out, &tmap_unused, &kp};
    if ((e = cudaLaunchKernelExC(&cfg, v.fn[gg::kOpForward][p->dtype], args)) != cudaSuccess)
        return cuda_fail("kernel launch", e);

    if (status_out) {
        // Wait for this call's kernel, then read the shared status word: the first timeout of any
        // call on this device since the last read. Clear it once reported.
        uint32_t st = 0;
        if ((e = cudaStreamSynchronize(stream)) != cudaSuccess)
            return cuda_fail("cudaStreamSynchronize", e);
        if ((e = cudaMemcpy(&st, d_status, sizeof(uint32_t), cudaMemcpyDeviceToHost)) != cudaSuccess)
            return cuda_fail("cudaMemcpy(status)", e);
        *status_out = st;
        if (st != 0) {
            if ((e = cudaMemset(d_status, 0, sizeof(uint32_t))) != cudaSuccess)
                return cuda_fail("cudaMemset(status)", e);
            std::snprintf(msg, sizeof(msg), "%s: status 0x%x",
                          (st & gg::kStatusBounds) ? "debug bounds check failed" : "kernel bounded wait timed out", st);
            copy_msg(why, why_len, msg);
            return GG_ERR_DEVICE;
        }
    }
    return GG_OK;
}
