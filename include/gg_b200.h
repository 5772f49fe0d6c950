/*
 * gg_b200.h — C ABI of the B200 (sm_100a) grouped-GEMM backend.
 *
 * Operation (forward MoE grouped GEMM, RCR layout), the op of the reference's
 * GroupedGemmProblem (common/backend.hpp:32-60):
 *
 *     out[rows of group g] = x[rows of group g] @ w[g]^T
 *     x   [sum(group_m), k]  row-major   (tokens of all experts, back to back)
 *     w   [group_num, n, k]  row-major   (one weight matrix per expert)
 *     out [sum(group_m), n]  row-major
 *     bf16 or fp16 in, fp32 accumulation, output in the input dtype.
 *
 * The entry points mirror the reference's `class Backend` (common/backend.hpp:62-79):
 * prepare() is untimed set-up that returns "" or a reason the shape cannot run, run() enqueues
 * exactly one grouped GEMM without synchronising, release() frees what prepare() allocated.
 * Instead of exiting on a device error (TUNEMAX_HIP_CHECK, common/backend.hpp:15-23) every call
 * returns a status code and the library never terminates the process.
 *
 * Plain pointers and sizes only. `gg_stream_t` is the same type as CUDA's cudaStream_t
 * (NULL = the legacy default stream). A handle is bound to the device that is current when
 * gg_prepare() is called; it is not thread-safe (one handle per thread and device).
 */
#ifndef GG_B200_H
#define GG_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *gg_stream_t; /* == cudaStream_t */
typedef struct gg_handle gg_handle;

/* Element types (tunemax::DType, common/backend.hpp:27). */
enum gg_dtype { GG_BF16 = 0, GG_FP16 = 1 };

/* Return codes. */
enum gg_status {
    GG_OK = 0,            /* ready / done */
    GG_NOT_SUPPORTED = 1, /* gg_prepare: shape or arguments refused; `why` holds the reason (N/A) */
    GG_ERR_ARG = -1,      /* invalid call (null handle, run before prepare, ...) */
    GG_ERR_CUDA = -2,     /* a CUDA runtime/driver call failed; see gg_last_error() */
    GG_ERR_DEVICE = -3    /* the kernel reported a bounded-wait timeout; see gg_device_status() */
};

/* Problem descriptor: tunemax::GroupedGemmProblem (common/backend.hpp:39-60). group_m is a host
 * array of group_num entries (any value >= 0; zero-length groups are skipped); x, w, out are
 * device pointers owned by the caller, 16-byte aligned. Requirements checked by gg_prepare:
 * k % 8 == 0 and n % 8 == 0 (16-byte row strides for TMA and the vector epilogue),
 * sum(group_m) < 2^31. */
typedef struct gg_problem {
    int32_t dtype;          /* enum gg_dtype */
    int32_t group_num;      /* B: number of groups (experts) */
    int64_t n;              /* N: output columns = rows of each w[g] */
    int64_t k;              /* K: reduction length */
    const int64_t *group_m; /* host, [group_num] rows per group */
    const void *x;          /* device, [sum(group_m), k] */
    const void *w;          /* device, [group_num, n, k] */
    void *out;              /* device, [sum(group_m), n] */
} gg_problem;

/* Create a backend instance (tunemax::make_ck_tile_backend(), common/backend.hpp:81, is the
 * factory this one sits beside). Returns NULL only when out of host memory. */
gg_handle *gg_create(void);

/* Backend::name() (common/backend.hpp:65). Returns "b200". */
const char *gg_name(const gg_handle *h);

/* Backend::prepare() (common/backend.hpp:66; the CK version is ck_kernel/ck_grouped_gemm.cpp:
 * 130-218). Untimed: validates the problem, builds the device group-argument buffer (per-group
 * tile and row offsets), encodes the TMA descriptors and picks the kernel variant, then waits
 * for `stream`. Returns GG_OK when ready, GG_NOT_SUPPORTED with a reason in `why` (if why != NULL
 * and why_len > 0) when the shape is refused, or a negative error. */
int gg_prepare(gg_handle *h, const gg_problem *p, gg_stream_t stream, char *why, size_t why_len);

/* Backward grouped GEMMs of the same layer (MoE training). The reference benchmarks the forward
 * op only; its vendored Primus-Turbo grouped GEMM carries the two backward calls this replaces
 * (third_party/primus_turbo/kernels/hipblaslt_grouped_gemm.cu:80-96 shape rules,
 * :199-240 per-group arguments, zero-filled gradient for an expert without tokens :201-214):
 *
 *   GG_OP_DGRAD: dx[rows of g] = dy[rows of g] @ w[g]     dx [sum(group_m), k]
 *   GG_OP_WGRAD: dw[g] = dy[rows of g]^T @ x[rows of g]   dw [group_num, n, k]; an expert with
 *                                                         group_m[g] == 0 gets dw[g] = 0
 *
 * with dy [sum(group_m), n] (the gradient of out), x and w as in gg_problem. Same dtype rules,
 * fp32 accumulation, output in the input dtype (dw is overwritten, not accumulated into). */
enum gg_op { GG_OP_FORWARD = 0, GG_OP_DGRAD = 1, GG_OP_WGRAD = 2 };

typedef struct gg_grad_problem {
    int32_t dtype;          /* enum gg_dtype */
    int32_t group_num;      /* B */
    int64_t n;              /* N: columns of dy = rows of each w[g] */
    int64_t k;              /* K: columns of x, dx and each w[g] */
    const int64_t *group_m; /* host, [group_num] tokens per group */
    const void *dy;         /* device, [sum(group_m), n] */
    const void *x;          /* device, [sum(group_m), k]  (GG_OP_WGRAD) */
    const void *w;          /* device, [group_num, n, k]  (GG_OP_DGRAD) */
    void *dx;               /* device, [sum(group_m), k]  (GG_OP_DGRAD output) */
    void *dw;               /* device, [group_num, n, k]  (GG_OP_WGRAD output) */
} gg_grad_problem;

/* Backend::prepare() for a backward operation `op` (GG_OP_DGRAD or GG_OP_WGRAD); afterwards
 * gg_run() enqueues it as one kernel launch and gg_detail() describes it. The operands the
 * operation does not use may be NULL. Extra refusals: "split" > 1 for wgrad (its reduction
 * length differs per group), group_num * n >= 2^31 for wgrad, and a forced "bn" that is not a
 * multiple of 64 per CTA (the MN-major operand boxes are 64 columns wide). */
int gg_prepare_grad(gg_handle *h, const gg_grad_problem *p, int32_t op, gg_stream_t stream, char *why,
                    size_t why_len);

/* Backend::run() (common/backend.hpp:67; ck_kernel/ck_grouped_gemm.cpp:140, :114-121). Timed:
 * enqueues one grouped GEMM on `stream` and does not synchronise: one kernel launch, or two for
 * a split launch ("tail_launch" below). */
int gg_run(gg_handle *h, gg_stream_t stream);

/* Backend::release() (common/backend.hpp:69; ck_kernel/ck_grouped_gemm.cpp:142-146): frees
 * what gg_prepare() allocated. The handle can be prepared again. */
void gg_release(gg_handle *h);

/* Backend::detail() (common/backend.hpp:71; ck_kernel/ck_grouped_gemm.cpp:216): kernel variant,
 * tile shape, stages and grid of the prepared problem. Valid until the next prepare/release. */
const char *gg_detail(const gg_handle *h);

/* Message of the last failed call on this handle ("" if none). */
const char *gg_last_error(const gg_handle *h);

/* Synchronises `stream`, then reads and clears the kernel's device status word: 0 when every
 * launch since the last read finished normally, otherwise the first bounded-wait timeout code
 * (0x1000 | role << 8 | barrier) or, in the bounds-checked debug build, the first failed check
 * (0x2000 | site: 1 tile decode, 2 direct store, 3 TMA store box, 4 split-K workspace,
 * 5 arrival counter; the checked access was skipped). The outputs of every launch since the last read are then
 * unreliable (an aborted launch stops part-way and can leave the dynamic-dispatch tile counter
 * and split-K arrival counts behind; this call resets them, so later launches are sound again).
 * No counterpart in the reference, whose kernel cannot time out (its only device-side guard is
 * a trap, ck_kernel/fast_epilogue.hpp:38-41). */
int gg_device_status(gg_handle *h, gg_stream_t stream, uint32_t *status);

/* Override the automatic choices of gg_prepare / gg_prepare_grad (takes effect at the next
 * prepare):
 *   "variant"    -1 auto, 0 = 2-CTA 256x256 tile, 1 = 1-CTA 128x256, 2 = 1-CTA 128x128
 *   "band"       tiles per raster band (default chosen per shape), 0 = auto
 *   "raster"     -1 auto (= 0), 0 = bands of M tiles (weight panels shared), 1 = bands of N tiles
 *   "bn"         tile width (multiple of 16, <= the variant's), 0 = auto (cost model)
 *   "split"      K splits per split tile (split-K with an fp32 workspace), 0 = auto, 1 = none
 *   "split_tail" -1 auto, 0 = split every tile, 1 = split only the tiles of what would be a
 *                partial last wave (their units run first, whole tiles after them)
 *   "stream_k"   0 (default) = off, -1 = the cost model decides, 1 = stream-K over the tiles of
 *                what would be a partial last wave, 2 = over those and one full wave more: their
 *                K atoms are dealt out in equal contiguous ranges to all CTAs (pairs), tiles cut
 *                at arbitrary atoms are summed through an fp32 workspace (forward and dgrad;
 *                refused with "split" > 1, for wgrad, and where the tiling has no partial wave)
 *   "store"      -1 auto (direct stores from registers for tiles with >= 16 K atoms, staging +
 *                TMA stores for shorter ones), 0 = always TMA stores, 1 = always direct stores
 *   "sched"      0 (default) = static round-robin (cluster c runs tiles c, c + C, ...), 1 = dynamic
 *                dispatch: a cluster takes its next tile from a counter in the handle's device
 *                memory as it finishes one, so tiles that share a weight panel stay in step all
 *                launch long (fewer DRAM re-reads, but measured slower at the power cap), -1 =
 *                dynamic for launches of whole tiles with more tiles than CTAs / pairs. The counter
 *                is zero between launches, so launches of one handle must not overlap on the GPU
 *                (order them on one stream, as for any handle)
 *   "l2_a", "l2_b" forward op: L2 eviction priority of the A operand's (x) and the B operand's
 *                (weights) TMA loads: 0 no hint, 1 evict_first, 2 evict_last; l2_a -1
 *                (its default) = evict_last where the launch's weights outweigh its activations at
 *                least 4 : 1 and it runs at least 64 waves of tiles (many experts with few tokens
 *                each: over a long launch the streaming weights would push out activation rows
 *                that later tiles of the expert still read), no hint otherwise; l2_b defaults to 0.
 *                Results are unchanged by either. Backward operations ignore both (in the dgrad
 *                producer the hinted load form measured slower than any hint saved)
 *   "tail_launch" -1 auto (default), 0 off, 1 on: with the 2-CTA variant (forward and dgrad, no
 *                split-K or stream-K), the rows of each group's last 256-row tile, where they are at
 *                most 128, go to a second launch of the one-CTA kernel (128-row tiles) right behind
 *                the first in the stream; gg_run then enqueues two kernels. Automatic when at least
 *                5% of the pair m-tiles are such remainders (skewed routing: many small experts)
 *   "half_tiles" 0 off (default), 1 / -1 on: with the 2-CTA variant (forward and dgrad, no
 *                split-K or stream-K, a tile width that is a multiple of 32), a group whose last
 *                256-row tile holds at most 128 rows runs that tile half height (an M = 128 pair
 *                MMA, 64 rows per CTA). Measured slower than the split launch and than padding on
 *                B200 (a half tile costs ~0.9 of a whole one), so it is off unless asked for
 *   "tile_order" whole tiles (no split-K), and for forward / dgrad one launch (no split launch):
 *                0 group order (default), 1 interleaved, -1 interleaved when each kind below holds
 *                at least 5% of the launch's cost. With interleaving, gg_prepare plans the launch's
 *                tile order on the host: tiles of two kinds are merged so that both are dealt out
 *                at the same fraction of their total cost, and the list is copied to the handle's
 *                device memory; "sched" still picks static or dynamic dispatch over it. The kinds:
 *                wgrad, groups with a short reduction (few rows, bound by their output stores) and
 *                groups with a long one (bound by the tensor cores); forward / dgrad, groups with
 *                few m-tiles (bound by reading their weight panels from DRAM) and groups with many.
 *                Measured on B200 under skewed routing (256 experts): wgrad slower than group order
 *                (707 static / 764 dynamic vs 815 TFLOPS); forward with half tiles and dynamic
 *                dispatch level with the split launch at the power cap (1034 vs 1059 TFLOPS), so
 *                it is off unless asked for
 *   "pdl"        1 (default) = launch with programmatic stream serialisation, so the launch and
 *                on-chip set-up overlap the previous kernel in the stream; 0 = plain launch
 *   "max_ctas"   cap on the persistent grid (0 = one CTA per SM)
 *   "timeout_ms" bounded-wait limit inside the kernel (default 2000)
 *   "test_bounds" test only: 1 = the kernel is told the output has one row fewer than it has, so
 *                the bounds-checked debug build (lib/libgg_b200_debug.so, -DGG_DEBUG) finds the last
 *                row's stores out of bounds, skips them and reports 0x2002 in the status word (the
 *                release build has no checks and stores every row); used to test the checks
 *   "test_stall" test only: 1 = the kernel never loads the first stage of its first CTA (pair),
 *                so that wait runs out after timeout_ms and gg_device_status() reports it;
 *                used to test failure detection without faulting the GPU
 * Returns GG_OK or GG_ERR_ARG for an unknown key. The knobs are the analogue of the compile-time
 * CkTileConfig (ck_kernel/ck_grouped_gemm_config.hpp:26-86) that the reference edits to tune. */
int gg_set_option(gg_handle *h, const char *key, int64_t value);

/* Destroy the handle (calls gg_release first). */
void gg_destroy(gg_handle *h);

/* Expert-parallel shard of `group_num` groups over `world` GPUs: contiguous ranges, the first
 * (group_num % world) ranks get one extra group. Writes [*g0, *g1) for `rank`. Pure host
 * arithmetic (no CUDA). The reference has no multi-GPU path; its only split of experts is the
 * shape generator's EP divisor (scripts/gen_shapes.py:43-48). Returns GG_ERR_ARG on bad input. */
int gg_expert_shard(int32_t group_num, int32_t world, int32_t rank, int32_t *g0, int32_t *g1);

/* Library ABI version (incremented on incompatible change). */
int gg_abi_version(void);

/* One grouped GEMM with no allocation at all: the same computation and result as
 * gg_prepare() + gg_run(), for callers that cannot allocate device memory when they call, e.g. an
 * engine that has reserved the GPU's memory for its own pool, a plugin host with a fixed memory
 * budget, or a latency-critical path that must not call cudaMalloc/cudaFree (they can
 * synchronise the device). No counterpart in the reference, whose backend allocates its
 * argument buffer in prepare (ck_kernel/ck_grouped_gemm.cpp:209).
 *
 * The per-group tile/row offsets and the kernel's status word live in one fixed device array
 * inside the library (about 8 KB, held by every GPU that loads the library until the process
 * exits), so group_num is limited to 1024; larger problems are refused with GG_NOT_SUPPORTED and
 * a reason in `why`. Nothing is allocated, neither device memory nor host heap memory.
 * Enqueues two kernels on `stream` (one writes the call's group offsets into the array, passed
 * by value as its launch parameter; then the grouped GEMM) and returns without waiting for the
 * GPU, unless `status_out` is non-NULL: then it waits for the stream and stores the status word
 * there (0 = every bounded wait finished; GG_ERR_DEVICE is returned otherwise).
 *
 * The status word is shared by every call on the device and is sticky: a bounded-wait timeout
 * in any call stays recorded (and makes the waits of later calls give up early, leaving their
 * output incomplete) until a call with a non-NULL `status_out` reports it and clears it. A call
 * with `status_out == NULL` therefore reports nothing itself; a caller that never passes
 * `status_out` cannot detect a timeout.
 *
 * The first call on each device does a one-time set-up (it looks up the array's device address
 * and the kernels' launch limits); make that first call before any stream capture. Every call
 * on a device shares the one array and each call overwrites it, so calls whose kernels may
 * overlap on the GPU (different streams without ordering between them) race; calls in order on
 * one stream do not. Errors are reported in `why` (there is no handle for gg_last_error). */
int gg_run_noalloc(const gg_problem *p, gg_stream_t stream, uint32_t *status_out, char *why, size_t why_len);

#ifdef __cplusplus
}
#endif

#endif /* GG_B200_H */
