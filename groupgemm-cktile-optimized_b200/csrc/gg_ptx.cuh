// Thin inline-PTX wrappers for the sm_100a features the grouped GEMM uses: mbarriers, TMA
// tensor loads, Tensor Memory (tcgen05.alloc/ld) and the 5th-generation tensor-core MMA
// (tcgen05.mma). Each wrapper is one instruction; the kernel composes them.
#pragma once

#include <cstdint>

namespace gg {
namespace ptx {

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lane_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%laneid;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// One lane of the (converged) warp: 1 there, 0 in the others. The warp keeps running the issuing
// code together and predicates the single-thread instructions (TMA, MMA, commit) on this value.
__device__ __forceinline__ uint32_t elect_one_sync() {
    uint32_t r;
    asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\tselp.b32 %0, 1, 0, e;\n\t}" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Address of the same shared-memory variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// ---- programmatic dependent launch ----
// Wait until the grids this one depends on (the previous kernel in the stream, when launched
// with programmatic stream serialisation) have completed and their memory is visible. Returns
// at once when there is none.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next grid in the stream (if launched with programmatic stream serialisation) to be
// scheduled; it still waits in its own griddep_wait() for this grid to complete.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Order this thread's later async-proxy (TMA) accesses of global memory after the generic-proxy
// writes it can see (used after griddep_wait()).
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---- mbarrier ----
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Executed only where `pred` != 0 (the other lanes of the warp pass over it).
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes, uint32_t pred) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %2, 0;\n\t"
                 "@q mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(bar), "r"(bytes), "r"(pred)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Arrive on a barrier given by its shared::cluster address (possibly the peer CTA's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
                 : "memory");
}

// The same arrive with CTA-scope release, for a signal that publishes no memory the waiter reads:
// an accumulator's release to the MMA warp after tcgen05.wait::ld (the tcgen05 fences around the
// barrier order the TMEM accesses). A cluster-scope release would first wait until this warp's
// earlier global stores are performed at cluster scope, which costs the epilogue of a short tile
// about as much as its own stores.
__device__ __forceinline__ void mbar_arrive_cluster_cta(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// Test (and briefly wait for) completion of the phase with the given parity.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.b32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(bar), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Same with cluster-scope acquire: for barriers whose arrivals publish generic-proxy writes of
// the peer CTA.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.b32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(bar), "r"(parity)
                 : "memory");
    return ok != 0;
}

// ---- TMA (tensor) loads: global -> shared, completion counted on an mbarrier ----
// The load wrappers issue only where `pred` != 0, so a converged warp can run the producer loop
// with one elected lane issuing.
__device__ __forceinline__ void prefetch_tmap(const void *tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Before the first use of a tensor map that lives in global memory and was written through the
// generic proxy (a host copy): order that write before the tensor-map proxy reads it.
__device__ __forceinline__ void fence_tensormap_acquire(const void *tmap) {
    asm volatile("fence.proxy.tensormap::generic.acquire.sys [%0], 128;" ::"l"(tmap) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *tmap, uint32_t bar, int32_t c0,
                                            int32_t c1, uint32_t pred) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t"
                 "@q cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];\n\t}" ::"r"(dst),
                 "l"(tmap), "r"(bar), "r"(c0), "r"(c1), "r"(pred)
                 : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void *tmap, uint32_t bar, int32_t c0,
                                            int32_t c1, int32_t c2, uint32_t pred) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %6, 0;\n\t"
                 "@q cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4, %5}], [%2];\n\t}" ::"r"(dst),
                 "l"(tmap), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(pred)
                 : "memory");
}

// CTA-pair forms: the destination is this CTA's shared memory, the completion barrier may be
// the pair leader's (a shared::cluster address from mapa). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void *tmap, uint32_t bar,
                                                 int32_t c0, int32_t c1, uint32_t pred) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t"
                 "@q cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];\n\t}" ::"r"(dst),
                 "l"(tmap), "r"(bar), "r"(c0), "r"(c1), "r"(pred)
                 : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const void *tmap, uint32_t bar,
                                                 int32_t c0, int32_t c1, int32_t c2, uint32_t pred) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %6, 0;\n\t"
                 "@q cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4, %5}], [%2];\n\t}" ::"r"(dst),
                 "l"(tmap), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(pred)
                 : "memory");
}

// The same four loads with an L2 eviction-priority hint (`policy` from l2_policy_*): the lines a
// load brings into L2 are kept longer (evict_last) or dropped first (evict_first).
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const void *tmap, uint32_t bar, int32_t c0,
                                                 int32_t c1, uint64_t policy, uint32_t pred) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t"
                 "@q cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
                 " [%0], [%1, {%3, %4}], [%2], %6;\n\t}" ::"r"(dst),
                 "l"(tmap), "r"(bar), "r"(c0), "r"(c1), "r"(pred), "l"(policy)
                 : "memory");
}

__device__ __forceinline__ void tma_load_3d_hint(uint32_t dst, const void *tmap, uint32_t bar, int32_t c0,
                                                 int32_t c1, int32_t c2, uint64_t policy, uint32_t pred) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %6, 0;\n\t"
                 "@q cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
                 " [%0], [%1, {%3, %4, %5}], [%2], %7;\n\t}" ::"r"(dst),
                 "l"(tmap), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(pred), "l"(policy)
                 : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair_hint(uint32_t dst, const void *tmap, uint32_t bar, int32_t c0,
                                                      int32_t c1, uint64_t policy, uint32_t pred) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %5, 0;\n\t"
                 "@q cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
                 ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %6;\n\t}" ::"r"(dst),
                 "l"(tmap), "r"(bar), "r"(c0), "r"(c1), "r"(pred), "l"(policy)
                 : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair_hint(uint32_t dst, const void *tmap, uint32_t bar, int32_t c0,
                                                      int32_t c1, int32_t c2, uint64_t policy, uint32_t pred) {
    asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %6, 0;\n\t"
                 "@q cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
                 ".L2::cache_hint [%0], [%1, {%3, %4, %5}], [%2], %7;\n\t}" ::"r"(dst),
                 "l"(tmap), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(pred), "l"(policy)
                 : "memory");
}

// 32-byte streaming store (evict-first): the 16 bf16/fp16 values of one half-chunk of a row.
// `p` must be 32-byte aligned.
__device__ __forceinline__ void st_cs_v8(void *p, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t a4, uint32_t a5, uint32_t a6, uint32_t a7) {
    asm volatile("st.global.cs.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(a0), "r"(a1), "r"(a2),
                 "r"(a3), "r"(a4), "r"(a5), "r"(a6), "r"(a7)
                 : "memory");
}

// ---- TMA stores: shared -> global, tracked in bulk groups of the issuing thread ----
// L2 cache policy: evict first (data that is written once and not re-read by this kernel).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void tma_store_2d(const void *tmap, uint32_t src, int32_t c0, int32_t c1, uint64_t policy) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
                     tmap),
                 "r"(src), "r"(c0), "r"(c1), "l"(policy)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N bulk groups still read their shared-memory source.
template <int N> __device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until all bulk groups of this thread have completed (writes done).
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// ---- Tensor Memory ----
template <int kCG> __device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
    if constexpr (kCG == 1)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                     "r"(ncols)
                     : "memory");
    else
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                     "r"(ncols)
                     : "memory");
}

template <int kCG> __device__ __forceinline__ void tmem_relinquish() {
    if constexpr (kCG == 1)
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    else
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

template <int kCG> __device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    if constexpr (kCG == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                     : "memory");
    else
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                     : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i gets lane (base + i), columns col..col+31.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32"
                 " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
                 " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31},"
                 " [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                   "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
                   "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                   "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
                   "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}

// Wait for this thread's outstanding tcgen05.ld. The registers are tied through the asm so
// the compiler cannot move their uses above the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                   "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                   "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                   "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// Order the uses of `r` after a preceding tcgen05.wait::ld (for a second register array loaded
// before the same wait): an empty volatile statement that ties the registers.
__device__ __forceinline__ void tmem_tie(uint32_t (&r)[32]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                   "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                   "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                   "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                   "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                   "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// 32-bit stores into shared memory: this CTA's (shared::cta address) or any CTA's of the cluster
// (shared::cluster address from mapa).
__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

// ---- MMA ----
// Shared-memory matrix descriptor for a K-major operand tile written by TMA with the 128-byte
// swizzle: rows of 128 bytes (64 16-bit elements), 8-row swizzle atoms of 1024 bytes.
//   bits  0-13  start address >> 4
//   bits 16-29  leading-dimension byte offset >> 4 (unused for swizzled K-major; 1)
//   bits 32-45  stride-dimension byte offset >> 4 (1024 B between 8-row groups)
//   bits 46-47  descriptor version (1 on sm_100)
//   bits 61-63  layout: 2 = 128-byte swizzle
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
    return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Shared-memory matrix descriptor for an MN-major operand tile written by TMA as boxes of 64
// MN elements (one 128-byte row) x 64 K rows with the 128-byte swizzle: within a box the K rows
// are 128 bytes apart in 8-row swizzle atoms of 1024 bytes; boxes of successive 64-element MN
// chunks are 8 KB apart.
//   leading-dimension byte offset = 8192 (between 64-element MN chunks)
//   stride-dimension byte offset  = 1024 (between 8-row groups along K)
// Sixteen K rows (one kind::f16 MMA) span 2048 bytes.
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t saddr) {
    return uint64_t((saddr & 0x3FFFFu) >> 4) | (uint64_t(8192 >> 4) << 16) | (uint64_t(1024 >> 4) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Instruction descriptor of tcgen05.mma kind::f16 with fp32 accumulation: bits 4-5 D format
// (1 = f32), 7-9 A format, 10-12 B format (0 = f16, 1 = bf16), 15/16 A/B major (0 = K-major,
// 1 = MN-major), 17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t f16_idesc(uint32_t ab_fmt, int m, int n, uint32_t a_mn = 0,
                                                 uint32_t b_mn = 0) {
    return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (a_mn << 15) | (b_mn << 16) | (uint32_t(n >> 3) << 17) |
           (uint32_t(m >> 4) << 24);
}

// Issued only where `pred` != 0: the MMA warp runs its loop converged and one elected lane
// issues. (Measured on B200: issued this way a pair MMA of width N takes the tensor pipe's N/2
// cycles for every N, with a commit every 4 or 8 MMAs; issued from a lone lane inside a divergent
// branch the same loop takes ~120-130 cycles per MMA below N = 256.)
template <int kCG>
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate, uint32_t pred) {
    if constexpr (kCG == 1)
        asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.b32 p, %4, 0;\n\tsetp.ne.b32 q, %5, 0;\n\t"
                     "@q tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
                     "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(pred)
                     : "memory");
    else
        asm volatile("{\n\t.reg .pred p, q;\n\tsetp.ne.b32 p, %4, 0;\n\tsetp.ne.b32 q, %5, 0;\n\t"
                     "@q tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
                     "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(pred)
                     : "memory");
}

// Arrive (once) on `bar` when all tcgen05.mma issued so far by this thread have completed.
// `bar` is a shared::cluster address, so it may name the peer CTA's barrier. Only where
// `pred` != 0 (the lane that issued the MMAs).
template <int kCG> __device__ __forceinline__ void umma_commit(uint32_t bar, uint32_t pred) {
    if constexpr (kCG == 1)
        asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %1, 0;\n\t"
                     "@q tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar),
                     "r"(pred)
                     : "memory");
    else
        asm volatile("{\n\t.reg .pred q;\n\tsetp.ne.b32 q, %1, 0;\n\t"
                     "@q tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(bar),
                     "r"(pred)
                     : "memory");
}

}  // namespace ptx
}  // namespace gg
