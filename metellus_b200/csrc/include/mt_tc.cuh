// sm_100a tensor-core helpers: mbarriers, TMA, tcgen05 / TMEM, and the 3xTF32 GEMM
// mainloop used by every tcgen05 matmul group (standalone, with prologue / epilogue,
// and the two-anchor diamond).
//
// 3xTF32: each fp32 operand x is split as hi = x rounded to tf32, lo = x - hi
// and the product is accumulated in fp32 TMEM as hi*hi + hi*lo + lo*hi, which keeps
// about 22 bits of each operand (fp32 carries 24): normwise error close to an fp32
// dot product, at tensor-core rate.
//
// All spin-waits are bounded by wall time (%globaltimer). On timeout the waiting
// thread records a code in the kernel's status word, raises the CTA abort flag and
// returns false; every role then leaves its loop, in-flight copies are drained with
// a bounded wait, TMEM is freed and the kernel returns. The host reads the status
// word after the launch and raises.
#pragma once

// The limit can be set before this header (a test shortens it to exercise the
// timeout path on a kernel whose producer is told to stop early, below).
#ifndef MT_WAIT_LIMIT_NS
#define MT_WAIT_LIMIT_NS 2000000000ull  // 2 s per wait
#endif
// MT_TEST_STALL_KTILE (test builds only, never defined by the planner): the TMA
// producer stops before that k-tile, so the consumers' bounded waits run out and the
// kernel takes its abort path (status word, drained copies, TMEM freed, return).

struct alignas(64) mt_tmap { unsigned long long v[16]; };

__device__ __forceinline__ uint32_t mt_smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t mt_globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- mbarrier ------------------------------------------------------------------

__device__ __forceinline__ void mt_mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(mt_smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mt_fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mt_mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}"
                 :: "r"(mt_smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mt_mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 :: "r"(mt_smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mt_mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.b32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(mt_smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Non-blocking check of an mbarrier phase.
__device__ __forceinline__ bool mt_mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.b32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(mt_smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Bounded wait: true when the phase completed, false on timeout or CTA abort.
__device__ __forceinline__ bool mt_mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                             int* status, int code) {
    if (mt_mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = mt_globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mt_mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (*abort_flag) return false;
            if (mt_globaltimer() - t0 > MT_WAIT_LIMIT_NS) {
                if (status) atomicCAS(status, 0, code);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// Bounded wait that ignores the abort flag: used on the abort path to let this CTA's
// own in-flight bulk copies land before it exits (0.5 s limit).
__device__ __forceinline__ void mt_mbar_drain(uint64_t* bar, uint32_t parity) {
    const uint64_t t0 = mt_globaltimer();
    while (!mt_mbar_try_wait(bar, parity)) {
        if (mt_globaltimer() - t0 > 500000000ull) return;
    }
}

// ---- thread-block clusters (split-K pairs) ---------------------------------------

__device__ __forceinline__ uint32_t mt_cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Address of `p` (this CTA's shared memory) in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t mt_cluster_map(const void* p, uint32_t rank) {
    uint32_t a;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(mt_smem_u32(p)), "r"(rank));
    return a;
}
__device__ __forceinline__ void mt_st_cluster_v4(uint32_t addr, float4 v) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};"
                 :: "r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w) : "memory");
}
// Arrive on an mbarrier in another cluster CTA's shared memory; release at cluster
// scope, so this thread's earlier shared::cluster stores are visible to its waiters.
__device__ __forceinline__ void mt_mbar_arrive_remote(uint32_t remote_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" :: "r"(remote_bar) : "memory");
}
__device__ __forceinline__ bool mt_mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.b32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(mt_smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// Bounded wait for arrivals from another cluster CTA (acquire at cluster scope). With
// `ignore_abort` the wait runs to its time limit even when this CTA is aborting: a
// split-K partner keeps its shared memory alive until the remote arrive it expects.
__device__ __forceinline__ bool mt_mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                     int* status, int code, bool ignore_abort) {
    const uint64_t t0 = mt_globaltimer();
    for (uint32_t it = 1;; ++it) {
        if (mt_mbar_try_wait_cluster(bar, parity)) return true;
        if ((it & 255u) == 0) {
            if (!ignore_abort && *abort_flag) return false;
            if (mt_globaltimer() - t0 > MT_WAIT_LIMIT_NS) {
                if (status) atomicCAS(status, 0, code);
                *abort_flag = 1;
                return false;
            }
        }
    }
}
// Arrive on an mbarrier in another cluster CTA's shared memory with the default
// release at CTA scope: no cluster-scope fence (a release.cluster arrive stalls the
// warp on a memory barrier). For hand-offs that publish no generic-proxy data to
// the other CTA: tensor-memory reads done (tcgen05.wait::ld), or operands this CTA
// wrote into its own shared memory for the pair's MMAs, made visible to the async
// proxy by fence.proxy.async first.
__device__ __forceinline__ void mt_mbar_arrive_peer(uint32_t remote_bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" :: "r"(remote_bar) : "memory");
}
// Cluster-wide barrier: every thread of both CTAs executes it right after set-up
// (mbarrier initialisation), before any role can wait on anything.
__device__ __forceinline__ void mt_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Prologue / epilogue adaptors around lambdas generated per kernel.
template <class F>
struct mt_prologue {
    F f;
    static constexpr bool kActive = true;
    __device__ __forceinline__ float operator()(float x, int r, int k) const { return f(x, r, k); }
};
template <class F>
struct mt_epilogue {
    F f;
    template <class V>
    __device__ __forceinline__ void store(int row, int col0, V& v) const { f(row, col0, v); }
};

// ---- TMA -------------------------------------------------------------------------

__device__ __forceinline__ void mt_tma_prefetch(const mt_tmap* m) {
    asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
__device__ __forceinline__ void mt_tma_load_2d(void* dst, const mt_tmap* m, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        :: "r"(mt_smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(m)), "r"(mt_smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void mt_tma_load_3d(void* dst, const mt_tmap* m, uint64_t* bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        :: "r"(mt_smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(m)), "r"(mt_smem_u32(bar)), "r"(c0), "r"(c1),
           "r"(c2)
        : "memory");
}
__device__ __forceinline__ void mt_tma_load_4d(void* dst, const mt_tmap* m, uint64_t* bar, int c0, int c1, int c2,
                                               int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];"
        :: "r"(mt_smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(m)), "r"(mt_smem_u32(bar)), "r"(c0), "r"(c1),
           "r"(c2), "r"(c3)
        : "memory");
}
// Generic-proxy writes to shared memory become visible to the async proxy
// (tcgen05.mma operand reads) after this fence.
__device__ __forceinline__ void mt_fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 / TMEM ----------------------------------------------------------------

__device__ __forceinline__ void mt_tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(mt_smem_u32(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void mt_tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mt_tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void mt_tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc), kind::tf32, one CTA.
__device__ __forceinline__ void mt_mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// D(tmem) (+)= A(tmem) * B(smem desc), kind::tf32, one CTA. A sits K-major in tensor
// memory: lane = row (M = 128), one 32-bit column per k.
__device__ __forceinline__ void mt_mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive on `bar` once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void mt_mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(mt_smem_u32(bar)) : "memory");
}
// ---- CTA-pair (cta_group::2) forms, used by mt_gemm_3xtf32_pair. A kernel uses
// either these or the one-CTA forms above for all of its tcgen05 instructions.

// One warp in each CTA of the pair: the same columns are allocated in both CTAs'
// tensor memory and each CTA's slot receives the address.
__device__ __forceinline__ void mt_tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(mt_smem_u32(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void mt_tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}
// D (+)= A * B over the pair, issued by one thread of the even CTA: M = 256, rows
// [0, 128) from the even CTA and [128, 256) from the odd one; A from each CTA's
// tensor memory at `a_tmem`, B's N columns split in halves between the two CTAs'
// shared memory at the descriptor's address; each CTA's D holds its 128 rows.
__device__ __forceinline__ void mt_mma_tf32_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                    uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive on the mbarrier at `bar`'s offset in both CTAs of the pair once this
// thread's earlier pair MMAs complete.
__device__ __forceinline__ void mt_mma_commit_pair_both(uint64_t* bar) {
    const unsigned short both = 3;
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 :: "r"(mt_smem_u32(bar)), "h"(both) : "memory");
}
// The same for this CTA's barrier only.
__device__ __forceinline__ void mt_mma_commit_pair_local(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(mt_smem_u32(bar)) : "memory");
}

// 32 lanes x 32 consecutive fp32 columns: thread t of the warp gets lane (base+t).
__device__ __forceinline__ void mt_tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16-column forms of the two accesses above (lower register pressure).
__device__ __forceinline__ void mt_tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
template <int W>
__device__ __forceinline__ void mt_tmem_ldw(uint32_t taddr, float (&v)[W]) {
    static_assert(W == 16 || W == 32, "16- or 32-column loads");
    if constexpr (W == 32) mt_tmem_ld32(taddr, v);
    else mt_tmem_ld16(taddr, v);
}

__device__ __forceinline__ void mt_tmem_st16(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        :: "r"(taddr),
           "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
           "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
           "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
           "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void mt_tmem_st16_nowait(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        :: "r"(taddr),
           "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
           "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
           "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
           "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
        : "memory");
}

// Thread t of the warp writes 32 consecutive fp32 columns of lane (base+t); returns
// once the writes are done (tcgen05.wait::st).
__device__ __forceinline__ void mt_tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        :: "r"(taddr),
           "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
           "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
           "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
           "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
           "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
           "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
           "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
           "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void mt_tmem_st32_nowait(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        :: "r"(taddr),
           "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
           "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
           "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
           "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
           "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
           "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
           "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
           "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}

// The stores above without their wait: issue several, then one mt_tmem_wait_st, and
// leave their source registers unchanged until that wait.
__device__ __forceinline__ void mt_tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 layout type 2, version 1).
__device__ __forceinline__ uint64_t mt_sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor for kind::tf32 with fp32 accumulation.
__host__ __device__ constexpr uint32_t mt_idesc_tf32(int M, int N, bool a_mn_major, bool b_mn_major) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Split x into hi + lo with hi exact as a tf32 (x's leading 11 significant bits,
// rounded to nearest on the magnitude, ties away from zero) and lo = x - hi, exact in
// fp32 with at most 12 significant bits (the MMA's truncating read keeps 11 of them).
// Rounding is done on the bit pattern: adding half a tf32 ulp (bit 12) to the
// magnitude bits carries into the kept bits exactly when the dropped part is at least
// half an ulp, then the 13 low bits are cleared. Two integer operations and one fp32
// subtraction per element; this measured 6 % faster in the pair GEMM than Veltkamp's
// splitting with an overflow guard (4 fp32 operations plus 3 for the guard), at
// the same error. Rounding hi to nearest rather than letting the MMA truncate x halves
// |lo| and quarters the lo*lo term that 3xTF32 omits (truncated hi measured 4.5e-7
// normwise at 4096^3, nearest 3.2e-7; fp32 dot products 3.7e-7).
// Range: exact for every finite |x| below (2 - 2^-11) * 2^127 (within half a tf32 ulp
// of FLT_MAX the rounding carries to inf); inf stays inf and NaN stays NaN, and lo is
// then NaN, so an inf or NaN operand makes the products it enters NaN.
__device__ __forceinline__ void mt_split_tf32(float x, float& hi, float& lo) {
    hi = __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u);
    lo = __fsub_rn(x, hi);
}

// ---------------------------------------------------------------------------------
// The GEMM mainloop.
//
// Tile BM=128 rows x BN columns, K chunks of BK=32 fp32 (one 128-byte swizzle row);
// warp roles are listed at mt_gemm_3xtf32.
//
// Operand tiles in shared memory, per stage:
//   A          : TMA box {32 (k), 128 (m)}, K-major, rows of 128 B, 8-row atoms
//                (SBO 1024 B); split into tensor memory, where the MMA reads it.
//   B K-major  : TMA box {32 (k), BN (n)}, as A; MMA k-step of 8 = +32 B.
//   B MN-major : TMA 3-D box {32 (n), 32 (k), BN/32}: 32-column chunks of 4 KB
//                (LBO 4096 B), k rows of 128 B in 4-row swizzle atoms (SBO 512 B),
//                MMA k-step = +1024 B.
// ---------------------------------------------------------------------------------

template <int BN, int RSTAGES, int CSTAGES, bool A_MN, bool B_MN, int NB>
struct mt_gemm_layout {
    static_assert(!A_MN, "A tiles must be K-major");
    static constexpr uint32_t kABytes = 128u * 32u * 4u;            // 16 KB
    static constexpr uint32_t kBBytes = (uint32_t)BN * 32u * 4u;
    // Raw ring (TMA targets): A, then B of every anchor side by side.
    static constexpr uint32_t kRawBytes = kABytes + (uint32_t)NB * kBBytes;
    // Converted ring (MMA operands): B hi of every anchor side by side, then B lo. A's
    // hi / lo split goes to tensor memory (one 64-column slot per converted stage).
    static constexpr uint32_t kConvBytes = 2u * (uint32_t)NB * kBBytes;
    static constexpr uint32_t kRawOffset = 0;
    static constexpr uint32_t kConvOffset = RSTAGES * kRawBytes;
    static constexpr uint32_t kTileBytes = RSTAGES * kRawBytes + CSTAGES * kConvBytes;
    static constexpr uint32_t kBarOffset = kTileBytes;  // rfull, rempty per raw stage; cfull, cempty per converted stage; accum
    static constexpr uint32_t kBytes = kTileBytes + (2 * RSTAGES + 2 * CSTAGES + 6) * 8 + 16;
};

// K-major 128-byte-swizzled operand tile (rows of 32 fp32 = 128 B, 8-row atoms of
// 1 KB): descriptor for MMA k-step kk (8 tf32 = 32 B into each row).
//
__device__ __forceinline__ uint64_t mt_operand_desc_k(uint32_t base, int kk) {
    return mt_sdesc_sw128(base + (uint32_t)kk * 32u, 16u, 1024u);
}

// N-contiguous (MN-major) B tile, as TMA writes it with SWIZZLE_128B_ATOM_32B from a
// 3-D box {32 (n), 32 (k), BN/32}: 128-byte rows of 32 n-values, one row per k;
// 32-byte chunks swizzled within 4-row atoms (512 B, SBO); 32-column chunks 4 KB
// apart (LBO). tf32 MN-major operands use this layout (sm_100 layout type 1,
// 128-byte swizzle on a 32-byte base); with the plain 128-byte swizzle a B200 run
// left the accumulator unchanged. MMA k-step kk = 8 rows = +1024 B.
__device__ __forceinline__ uint64_t mt_operand_desc_mn(uint32_t base, int kk) {
    const uint32_t a = base + (uint32_t)kk * 1024u;
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)((4096u >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((512u >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (1ull << 61);
}


// Coordinates of element `i` (0..rows*32-1 in storage order) of an operand tile:
// row within the tile (m or n) and k within the chunk, undoing the 128-byte swizzle.
template <bool MN>
__device__ __forceinline__ void mt_tile_coord(uint32_t byte_off, int& r, int& k) {
    const uint32_t line = byte_off >> 7;               // 128-byte line index
    const uint32_t chunk = ((byte_off >> 4) & 7u) ^ (line & 7u);
    const uint32_t in = (byte_off >> 2) & 3u;
    const uint32_t inner = chunk * 4u + in;            // logical position within the 128 B line
    if (MN) {
        // line = kk_row + 32 * chunk32 ; inner = column within the 32-wide chunk
        k = (int)(line & 31u);
        r = (int)((line >> 5) * 32u + inner);
    } else {
        r = (int)line;
        k = (int)inner;
    }
}

// Identity prologue (no transform, no coordinates needed).
struct mt_no_prologue {
    static constexpr bool kActive = false;
    __device__ __forceinline__ float operator()(float x, int, int) const { return x; }
};

// Split one landed fp32 tile: hi to `hi` (the tile itself for an in-place split), lo
// to `lo`. `ROWS` is the tile extent along M (A) or N (B); `r0` / `k0` its global origin;
// `rlim` / `klim` the global bounds (prologue transforms only touch in-bounds
// elements; out-of-bounds elements were zero-filled by TMA and stay 0).
// Convert one landed tile in two phases so every shared-memory load of the thread is
// in flight before the first split (the converter is latency bound otherwise): load
// this thread's IT float4 chunks, then apply the prologue (global coordinates
// recovered from the swizzled offset), split, and store hi (to `hi`, which may be the
// landed tile itself) and lo.
template <bool MN, bool A_SIDE, int ROWS, int NT, class Pro>
__device__ __forceinline__ void mt_convert_tile(const float* tile, float* hi, float* lo, int r0, int k0, int rlim,
                                                int klim, const Pro& pro, int tid) {
    constexpr int N4 = ROWS * 32 / 4;
    constexpr int IT = (N4 + NT - 1) / NT;
    float4 v[IT];
#pragma unroll
    for (int j = 0; j < IT; ++j) {
        const int i = tid + j * NT;
        if (N4 % NT == 0 || i < N4) v[j] = reinterpret_cast<const float4*>(tile)[i];
    }
#pragma unroll
    for (int j = 0; j < IT; ++j) {
        const int i = tid + j * NT;
        if (!(N4 % NT == 0 || i < N4)) continue;
        if constexpr (Pro::kActive) {
            int r, k;
            mt_tile_coord<MN>((uint32_t)i * 16u, r, k);
            const int gr = r0 + r, gk = k0 + k;
            float* e = reinterpret_cast<float*>(&v[j]);
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                if (gr < rlim && gk + l < klim) {
                    if constexpr (A_SIDE) e[l] = pro(e[l], gr, gk + l);
                    else e[l] = pro(e[l], gk + l, gr);
                }
            }
        }
        float4 h, w;
        mt_split_tf32(v[j].x, h.x, w.x);
        mt_split_tf32(v[j].y, h.y, w.y);
        mt_split_tf32(v[j].z, h.z, w.z);
        mt_split_tf32(v[j].w, h.w, w.w);
        reinterpret_cast<float4*>(hi)[i] = h;
        reinterpret_cast<float4*>(lo)[i] = w;
    }
}

// Split this thread's row of a landed K-major A tile (row q*32+lane: 32 k values in
// one 128-byte line, 16-byte chunks swizzled by row & 7) into tf32 hi / lo and write
// them to tensor memory: hi to columns [0, 32) and lo to [32, 64) past `t_hi`, lane =
// row. Conflict-free: 8 consecutive rows cover all 8 chunk positions.
template <class Pro>
__device__ __forceinline__ void mt_convert_a_rows(const float* tile, uint32_t t_hi, int q, int lane, int m0, int k0,
                                                  int M, int K, const Pro& pro) {
    const int r = q * 32 + lane;
    const float4* line = reinterpret_cast<const float4*>(tile + r * 32);
    float hi[32], lo[32];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float4 x = line[c ^ (r & 7)];
        hi[4 * c] = x.x;
        hi[4 * c + 1] = x.y;
        hi[4 * c + 2] = x.z;
        hi[4 * c + 3] = x.w;
    }
    if constexpr (Pro::kActive) {
        const int gr = m0 + r;
#pragma unroll
        for (int k = 0; k < 32; ++k)
            if (gr < M && k0 + k < K) hi[k] = pro(hi[k], gr, k0 + k);
    }
#pragma unroll
    for (int k = 0; k < 32; ++k) {
        const float x = hi[k];
        mt_split_tf32(x, hi[k], lo[k]);
    }
    const uint32_t t = t_hi + ((uint32_t)(q * 32) << 16);
    mt_tmem_st32_nowait(t, hi);
    mt_tmem_st32_nowait(t + 32u, lo);
    mt_tmem_wait_st();
}

// C-tile = A(128 x K) * B_b(K x BN) for b < NB (NB = 2: two anchors sharing A).
//
// 544 threads, 17 warps:
//   warps 0, 1   MMA issuers (one elected lane each: warp 1 the even chunks, warp 0
//                the odd ones, each into its own accumulator buffer; see the pair
//                kernel below for why); warp 1 also owns tensor memory
//   warp 16      TMA producer (one elected lane)
//   warps 2..7   converters: warps 4..7 split the A rows of their TMEM lane quarter
//                into tf32 hi / lo in tensor memory (the MMA reads A from there, so
//                shared memory carries only the TMA write and one read of A); then
//                all six split the B tiles from the raw ring into hi / lo in the
//                converted ring
//   warps 8..15  accumulators + epilogue: warp w owns TMEM lane quarter (w % 4) and
//                half (w - 8) / 4 of the columns of every anchor.
//
// Accuracy: the tensor core's fp32 accumulation loses bits on every add (the error
// grows linearly with K: ~7e-6 normwise at K = 1024 when one TMEM accumulator runs
// the whole K loop). So each chunk of CHUNK k-tiles is accumulated into a fresh TMEM
// buffer (double buffered), and the accumulator warps add every finished chunk into
// fp32 registers with round-to-nearest adds, which keeps the normwise error at the
// level of an fp32 dot product.
//
// Split-K (SPLITK = 2): the launch is in clusters of two CTAs along x that share one
// output tile; CTA rank r runs the r-th half of the k-tiles. Rank 0's accumulator
// warps, once their mainloop is done, signal rank 1 (remote mbarrier arrive); rank 1
// writes its fp32 partial sums into rank 0's (now free) stage memory through
// distributed shared memory and signals back; rank 0 adds them (fixed order: its own
// half first) and runs the epilogue. Used when the output has too few tiles to fill
// the SMs (C = 1024^3: 64 tiles of 128 x 128 -> 128 CTAs).
template <int BN, int RST, int CST, bool A_MN, bool B_MN, int NB, int SPLITK = 1, class ProA, class ProB,
          class Epi, int CHUNK = 1>
__device__ __forceinline__ void mt_gemm_3xtf32(const mt_tmap* tmA, const mt_tmap* tmB0, const mt_tmap* tmB1,
                                               int M, int N, int K, const ProA& proA, const ProB& proB,
                                               const Epi& epi, int* status, void* smem_raw) {
    using L = mt_gemm_layout<BN, RST, CST, A_MN, B_MN, NB>;
    constexpr int HALF = BN / 2;                  // columns per accumulator warp per anchor
    constexpr uint32_t ACOLS = 2u * NB * BN;      // two chunk buffers of accumulators
    constexpr uint32_t TCOLS = ACOLS + 64u * CST;  // + A hi / lo per converted stage
    constexpr uint32_t NCOLS = TCOLS <= 32 ? 32 : TCOLS <= 64 ? 64 : TCOLS <= 128 ? 128 : TCOLS <= 256 ? 256 : 512;
    static_assert(TCOLS <= 512, "accumulators and A stages exceed TMEM");
    static_assert(BN == 64 || BN == 128, "BN must be 64 or 128");
    static_assert(NB * BN <= 256, "one MMA covers every anchor: N = NB * BN <= 256");
    static_assert(NB * HALF <= 64, "at most 64 accumulator registers per thread");
    static_assert(SPLITK == 1 || (SPLITK == 2 && NB == 1), "split-K pairs: one anchor");
    static_assert(SPLITK == 1 || 128u * NB * BN * 4u <= L::kTileBytes, "partial sums must fit the stage memory");
    constexpr int NCONV = 6;
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* rfull = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);  // [RST] TMA landed
    uint64_t* rempty = rfull + RST;     // [RST] converters done reading the raw stage
    uint64_t* cfull = rempty + RST;     // [CST] converted operands ready
    uint64_t* cempty = cfull + CST;     // [CST] MMAs done with the converted stage
    uint64_t* tfull = cempty + CST;     // [2]
    uint64_t* tempty = tfull + 2;       // [2]
    uint64_t* xready = tempty + 2;      // split-K: rank 0's stage memory is free (on rank 1)
    uint64_t* xfull = xready + 1;       // split-K: rank 1's partial sums landed (on rank 0)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xfull + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = (int)(threadIdx.x >> 5), lane = (int)(threadIdx.x & 31);
    // Tile order: the launch is (N tiles, M tiles); CTAs are mapped so that the ~148
    // resident at a time cover groups of 8 M tiles x ~18 N tiles, so each A row block
    // and each B column block is fetched from DRAM about once per group instead of
    // once per M tile (row-major order streams all of B once per M tile when B does
    // not fit L2).
    const int rank = SPLITK > 1 ? (int)mt_cluster_rank() : 0;
    int m0, n0;
    {
        constexpr int kGroupM = 8;
        const int n_tiles = (int)gridDim.x / SPLITK, m_tiles = (int)gridDim.y;
        const int id = (int)(blockIdx.y * n_tiles + blockIdx.x / SPLITK);
        const int group = id / (kGroupM * n_tiles);
        const int first_m = group * kGroupM;
        const int gsize = min(m_tiles - first_m, kGroupM);
        const int in_group = id - group * kGroupM * n_tiles;
        m0 = (first_m + in_group % gsize) * 128;
        n0 = (in_group / gsize) * BN;
    }
    // this CTA's k-tiles: [kbeg, kbeg + nk) of ceil(K / 32)
    const int nk_all = (K + 31) / 32;
    const int per = (nk_all + SPLITK - 1) / SPLITK;
    const int kbeg = SPLITK > 1 ? rank * per : 0;
    const int nk = SPLITK > 1 ? max(0, min(nk_all, kbeg + per) - kbeg) : nk_all;
    const int nchunks = (nk + CHUNK - 1) / CHUNK;
    // Raw ring: what TMA writes (A, then B of every anchor). Converted ring: B hi of
    // every anchor side by side, then B lo, so one MMA with N = NB * BN covers every
    // anchor (anchor b's columns land at accumulator columns [b * BN, (b + 1) * BN)).
    // A raw stage is free as soon as it is converted, so TMA runs ahead of the MMAs by
    // RST + CST stages rather than by the stages the converted operands occupy.
    auto A_raw = [&](int r) { return reinterpret_cast<float*>(smem + L::kRawOffset + r * L::kRawBytes); };
    auto B_raw = [&](int r, int b) {
        return reinterpret_cast<float*>(smem + L::kRawOffset + r * L::kRawBytes + L::kABytes + b * L::kBBytes);
    };
    auto B_cv = [&](int c, int b, int j) {
        return reinterpret_cast<float*>(smem + L::kConvOffset + c * L::kConvBytes + (j * NB + b) * L::kBBytes);
    };

    if (threadIdx.x == 0) {
        for (int r = 0; r < RST; ++r) {
            mt_mbar_init(&rfull[r], 1);
            mt_mbar_init(&rempty[r], NCONV);
        }
        for (int c = 0; c < CST; ++c) {
            mt_mbar_init(&cfull[c], NCONV);
            mt_mbar_init(&cempty[c], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mt_mbar_init(&tfull[b], 1);
            mt_mbar_init(&tempty[b], 8);
        }
        mt_mbar_init(xready, 256);
        mt_mbar_init(xfull, 256);
        *abort_flag = 0;
        mt_fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        mt_tma_prefetch(tmA);
        mt_tma_prefetch(tmB0);
        if (NB > 1) mt_tma_prefetch(tmB1);
    }
    if (warp == 1) mt_tmem_alloc(tmem_slot, NCOLS);
    mt_tc_fence_before();
    __syncthreads();
    if constexpr (SPLITK > 1) mt_cluster_sync();  // partner's barriers initialised
    mt_tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 16) {
        if (lane == 0) {
            int issued = 0;
            for (int kt = 0; kt < nk; ++kt) {
                const int r = kt % RST;
                if (kt >= RST && !mt_mbar_wait(&rempty[r], (uint32_t)((kt / RST) - 1) & 1u, abort_flag, status, 1))
                    break;
#ifdef MT_TEST_STALL_KTILE
                if (kt == MT_TEST_STALL_KTILE) break;
#endif
                mt_mbar_expect_tx(&rfull[r], L::kRawBytes);
                const int kg = (kbeg + kt) * 32;
                mt_tma_load_2d(A_raw(r), tmA, &rfull[r], kg, m0);
                for (int b = 0; b < NB; ++b) {
                    const mt_tmap* tb = b == 0 ? tmB0 : tmB1;
                    if (B_MN) mt_tma_load_3d(B_raw(r, b), tb, &rfull[r], 0, kg, n0 / 32);
                    else mt_tma_load_2d(B_raw(r, b), tb, &rfull[r], kg, n0);
                }
                issued = kt + 1;
            }
            if (*abort_flag) {  // let this CTA's own copies land before it can exit
                for (int kt = (issued > RST ? issued - RST : 0); kt < issued; ++kt)
                    mt_mbar_drain(&rfull[kt % RST], (uint32_t)(kt / RST) & 1u);
            }
        }
    } else if (warp == 0 || warp == 1) {
        // two MMA issuers: warp 1 the even chunks, warp 0 the odd ones, each into its
        // own accumulator buffer, so one issuer's waits overlap the other's MMAs
        const int issuer = warp == 1 ? 0 : 1;
        if (lane == 0) {
            constexpr uint32_t idesc = mt_idesc_tf32(128, NB * BN, false, B_MN);
            bool ok = true;
            for (int ch = issuer; ch < nchunks && ok; ch += 2) {
                const int tb = ch & 1;
                if (ch >= 2 && !mt_mbar_wait(&tempty[tb], (uint32_t)((ch >> 1) - 1) & 1u, abort_flag, status, 2))
                    break;
                mt_tc_fence_after();
                const int kt0 = ch * CHUNK, kt1 = min(kt0 + CHUNK, nk);
                for (int kt = kt0; kt < kt1; ++kt) {
                    const int c = kt % CST;
                    if (!mt_mbar_wait(&cfull[c], (uint32_t)(kt / CST) & 1u, abort_flag, status, 2)) {
                        ok = false;
                        break;
                    }
                    mt_tc_fence_after();
                    const uint32_t ah = tmem + ACOLS + 64u * (uint32_t)c;
                    const uint32_t bh = mt_smem_u32(B_cv(c, 0, 0)), bl = mt_smem_u32(B_cv(c, 0, 1));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t dah = ah + 8u * (uint32_t)kk;
                        const uint32_t dal = dah + 32u;
                        const uint32_t d = tmem + (uint32_t)(tb * NB * BN);
                        const uint64_t dbh = B_MN ? mt_operand_desc_mn(bh, kk) : mt_operand_desc_k(bh, kk);
                        const uint64_t dbl = B_MN ? mt_operand_desc_mn(bl, kk) : mt_operand_desc_k(bl, kk);
                        mt_mma_tf32_ts(d, dah, dbl, idesc, (kt != kt0 || kk) ? 1u : 0u);
                        mt_mma_tf32_ts(d, dal, dbh, idesc, 1u);
                        mt_mma_tf32_ts(d, dah, dbh, idesc, 1u);
                    }
                    mt_mma_commit(&cempty[c]);
                }
                mt_mma_commit(&tfull[tb]);
            }
        }
    } else if (warp >= 2 && warp < 8) {
        const int cw = warp - 2;                    // converter warp 0..5
        const int ct = cw * 32 + lane;              // 0..191
        for (int kt = 0; kt < nk; ++kt) {
            const int r = kt % RST, c = kt % CST;
            if (!mt_mbar_wait(&rfull[r], (uint32_t)(kt / RST) & 1u, abort_flag, status, 3)) break;
            // the converted stage (B buffers and A's TMEM slot) is free once the MMAs
            // of k-tile kt - CST completed
            if (kt >= CST && !mt_mbar_wait(&cempty[c], (uint32_t)((kt / CST) - 1) & 1u, abort_flag, status, 3)) break;
            mt_tc_fence_after();
            if (warp >= 4)
                mt_convert_a_rows(A_raw(r), tmem + ACOLS + 64u * (uint32_t)c, warp & 3, lane, m0, (kbeg + kt) * 32, M,
                                  K, proA);
            // the prologue (coordinates) is only supported on K-major B tiles
            for (int b = 0; b < NB; ++b)
                mt_convert_tile<false, false, BN, NCONV * 32>(B_raw(r, b), B_cv(c, b, 0), B_cv(c, b, 1), n0,
                                                              (kbeg + kt) * 32, N, K, proB, ct);
            mt_fence_proxy_async();
            mt_tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mt_mbar_arrive(&rempty[r]);
                mt_mbar_arrive(&cfull[c]);
            }
        }
    } else if (warp >= 8 && warp < 16) {
        const int q = warp & 3;                     // TMEM lane quarter
        const int h = (warp - 8) >> 2;              // column half
        float acc[NB][HALF];
#pragma unroll
        for (int b = 0; b < NB; ++b)
#pragma unroll
            for (int j = 0; j < HALF; ++j) acc[b][j] = 0.0f;
        bool ok = true;
        for (int c = 0; c < nchunks; ++c) {
            const int tb = c & 1;
            if (!mt_mbar_wait(&tfull[tb], (uint32_t)(c >> 1) & 1u, abort_flag, status, 5)) {
                ok = false;
                break;
            }
            mt_tc_fence_after();
#pragma unroll
            for (int b = 0; b < NB; ++b) {
#pragma unroll
                for (int j = 0; j < HALF / 16; ++j) {  // 16-column loads: 96 registers at 544 threads
                    float v[16];
                    mt_tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((tb * NB + b) * BN + h * HALF + j * 16), v);
#pragma unroll
                    for (int i = 0; i < 16; ++i) acc[b][j * 16 + i] = __fadd_rn(acc[b][j * 16 + i], v[i]);
                }
            }
            mt_tc_fence_before();
            __syncwarp();
            if (lane == 0) mt_mbar_arrive(&tempty[tb]);
        }
        if constexpr (SPLITK > 1) {
            const int t = (warp - 8) * 32 + lane;                // 0..255
            float4* xbuf = reinterpret_cast<float4*>(smem);      // stage memory, free after the mainloop
            if (rank == 1) {
                // wait until rank 0's stages are free, even when aborting (keeps this
                // CTA alive for rank 0's remote arrive)
                const bool ready = mt_mbar_wait_cluster(xready, 0, abort_flag, status, 6, true);
                if (ok && ready) {
#pragma unroll
                    for (int g = 0; g < HALF / 4; ++g)
                        mt_st_cluster_v4(mt_cluster_map(&xbuf[g * 256 + t], 0),
                                         make_float4(acc[0][4 * g], acc[0][4 * g + 1], acc[0][4 * g + 2],
                                                     acc[0][4 * g + 3]));
                    mt_mbar_arrive_remote(mt_cluster_map(xfull, 0));
                }
                ok = false;  // rank 0 runs the epilogue
            } else if (ok) {
                mt_mbar_arrive_remote(mt_cluster_map(xready, 1));
                ok = mt_mbar_wait_cluster(xfull, 0, abort_flag, status, 7, false);
                if (ok) {
#pragma unroll
                    for (int g = 0; g < HALF / 4; ++g) {
                        const float4 p = xbuf[g * 256 + t];
                        acc[0][4 * g] = __fadd_rn(acc[0][4 * g], p.x);
                        acc[0][4 * g + 1] = __fadd_rn(acc[0][4 * g + 1], p.y);
                        acc[0][4 * g + 2] = __fadd_rn(acc[0][4 * g + 2], p.z);
                        acc[0][4 * g + 3] = __fadd_rn(acc[0][4 * g + 3], p.w);
                    }
                }
            }
        }
        if (ok) {
            const int row = m0 + q * 32 + lane;
#pragma unroll
            for (int j = 0; j < HALF / 32; ++j) {
                float v[NB][32];
#pragma unroll
                for (int b = 0; b < NB; ++b)
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[b][i] = acc[b][j * 32 + i];
                epi.store(row, n0 + h * HALF + j * 32, v);
            }
        }
    }
    mt_tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        mt_tc_fence_after();
        mt_tmem_dealloc(tmem, NCOLS);
    }
}

// Optional wait-time counters for the pair GEMM (compile with MT_GEMM_PROFILE): clock64
// cycles each role spends in its mbarrier waits, summed over CTAs into the 64-bit slots
// 1..7 of the status buffer (slot 0 stays the timeout code). Off by default.
#ifdef MT_GEMM_PROFILE
#define MT_PROF_DECL() unsigned long long p_mma_issue = 0, p_mma_tempty = 0, p_mma_cfull = 0, p_mma_loop = 0, \
    p_conv_rfull = 0, p_conv_cempty = 0, p_acc_tfull = 0
#define MT_PROF_BEGIN(t) const long long t = clock64()
#define MT_PROF_END(t, acc) (acc) += (unsigned long long)(clock64() - (t))
#define MT_PROF_FLUSH(st) do { \
    unsigned long long* q = reinterpret_cast<unsigned long long*>(st); \
    if (p_mma_cfull | p_mma_tempty | p_mma_loop) { atomicAdd(q + 1, p_mma_cfull); atomicAdd(q + 2, p_mma_tempty); \
        atomicAdd(q + 3, p_mma_loop); } \
    if (p_conv_rfull | p_conv_cempty) { atomicAdd(q + 4, p_conv_rfull); atomicAdd(q + 5, p_conv_cempty); } \
    if (p_mma_issue) atomicAdd(q + 6, p_mma_issue); \
    if (p_acc_tfull) atomicAdd(q + 7, p_acc_tfull); } while (0)
#else
#define MT_PROF_DECL() do { } while (0)
#define MT_PROF_BEGIN(t) do { } while (0)
#define MT_PROF_END(t, acc) do { } while (0)
#define MT_PROF_FLUSH(st) do { } while (0)
#endif

// ---------------------------------------------------------------------------------

// Columns per tensor-memory load when the accumulator warps drain a chunk buffer.
#ifndef MT_PAIR_DRAIN_W
#define MT_PAIR_DRAIN_W 16
#endif

// CTA-pair GEMM: a 256 x 128 output tile per cluster of two CTAs (cta_group::2).
//
// The even CTA (rank 0) issues every MMA for both: M = 256 (its 128 A rows and the
// odd CTA's 128, each from its own tensor memory) x N = 128, with B's 128 columns
// split between the two CTAs' shared memory (64 each). Per CTA and k-tile this moves
// half of the B bytes of the one-CTA 128 x 128 tile through TMA, the converters and
// the MMA operand reads, for the same MMA work per SM: shared-memory traffic per
// k-tile drops from ~144 KB to ~88 KB, below what the MMAs need in issue time.
//
// Columns: one anchor (NB = 1, BN = 128): rank r holds B columns [n0 + 64r, +64).
// Two anchors sharing A (NB = 2, BN = 64): rank b holds anchor b's 64 columns, so D
// columns [0, 64) are anchor 0 and [64, 128) anchor 1, as in the one-CTA layout.
//
// Warp roles (544 threads, 17 warps) in each CTA: warps 0 and 1 issue the MMAs (one
// elected thread each, on the even CTA only): warp 1 the even k-tiles, warp 0 the odd
// ones, each into its own accumulator buffer. tcgen05.mma issue from one thread keeps
// almost nothing queued (measured: an N-cycle gap between groups of 12 MMAs costs
// ~N cycles of tensor-pipe time), so with a single issuer every barrier wait and fence
// between k-tiles idled the pipe; with two, one issuer's waits overlap the other's
// MMAs. Warps 2-7 split the operands (4-7: A rows into tensor memory; 2-3: B), warps
// 8-15 drain the accumulators and run the epilogue, warp 16 issues the TMA loads. 544
// threads leave 96 registers per thread: the drains use 16-column tensor-memory loads.
// Hand-offs across the pair: the odd
// CTA's converters arrive on the even CTA's cfull (remote arrive, release at CTA
// scope, after the proxy and tcgen05 fences), its accumulator warps on the even
// CTA's tempty; the even CTA's MMA commits arrive on both CTAs' cempty / tfull
// (multicast commit). Every wait is bounded; both CTAs meet at a cluster barrier
// before tensor memory is freed and either exits.
template <int BN, int RST, int CST, bool B_MN, int NB, int CHUNK, bool BAL, int NACC, int NISSUE, bool SACC,
          int GROUP_M, class ProA, class ProB, class Epi>
__device__ __forceinline__ void mt_gemm_3xtf32_pair(const mt_tmap* tmA, const mt_tmap* tmB0, const mt_tmap* tmB1,
                                                    int M, int N, int K, const ProA& proA, const ProB& proB,
                                                    const Epi& epi, int* status, void* smem_raw) {
    constexpr int NMMA = NB * BN;                 // MMA N: 128
    constexpr int BROWS = NMMA / 2;               // B rows (n) per CTA and stage: 64
    constexpr int HALF = BN / 2;                  // columns per accumulator warp per anchor
    constexpr uint32_t kABytes = 128u * 32u * 4u;
    constexpr uint32_t kBBytes = (uint32_t)BROWS * 32u * 4u;
    constexpr uint32_t kRawBytes = kABytes + kBBytes;
    constexpr uint32_t kConvBytes = 2u * kBBytes;
    constexpr uint32_t kConvOffset = RST * kRawBytes;
    constexpr uint32_t kBarOffset = kConvOffset + CST * kConvBytes;
    // NACC chunk buffers of accumulators (+ SACC: one buffer of the small products)
    constexpr uint32_t ACOLS = (uint32_t)(NACC + (SACC ? 1 : 0)) * NMMA;
    static_assert(NMMA == 128, "pair tiles are 256 x 128");
    static_assert(NB * HALF <= 64, "at most 64 accumulator registers per thread");
    static_assert(ACOLS + 64u * CST <= 512, "accumulators and A stages exceed TMEM");
    static_assert(SACC ? (NISSUE == 2 && NACC == 1)
                       : (NISSUE == 1 || (NISSUE == 2 && NACC == 2)),
                  "two issuers own one accumulator buffer each (SACC: one issues hi*hi, the other the small products)");
    constexpr uint32_t NCOLS = 512;
    constexpr int NCONV = 6;
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* rfull = reinterpret_cast<uint64_t*>(smem + kBarOffset);
    uint64_t* rempty = rfull + RST;
    uint64_t* cfull = rempty + RST;     // used on rank 0: both CTAs' converters
    uint64_t* cempty = cfull + CST;     // both CTAs: rank 0's MMA commit
    uint64_t* tfull = cempty + CST;     // [NACC] both CTAs: rank 0's MMA commit
    uint64_t* tempty = tfull + NACC;    // [NACC] used on rank 0: both CTAs' accumulator warps
    uint64_t* mdone = tempty + NACC;    // [2] rank 0: each issuer's MMAs drained on the abort path
    uint64_t* sdone = mdone + 2;        // SACC, both CTAs: the small-product issuer's last commit
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sdone + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = (int)(threadIdx.x >> 5), lane = (int)(threadIdx.x & 31);
    const int rank = (int)mt_cluster_rank();
    MT_PROF_DECL();
    int m0, n0;
    {
        // consecutive clusters walk the N tiles of a group of GROUP_M M tiles, so the
        // ~74 clusters resident at once share A and B tiles in L2
        constexpr int kGroupM = GROUP_M;        // in 256-row pair tiles
        const int n_tiles = (int)gridDim.x / 2, m_tiles = (int)gridDim.y;
        const int id = (int)(blockIdx.y * n_tiles + blockIdx.x / 2);
        const int group = id / (kGroupM * n_tiles);
        const int first_m = group * kGroupM;
        const int gsize = min(m_tiles - first_m, kGroupM);
        const int in_group = id - group * kGroupM * n_tiles;
        m0 = (first_m + in_group % gsize) * 256 + rank * 128;
        n0 = (in_group / gsize) * BN;
    }
    const int nb0 = NB == 1 ? n0 + rank * BROWS : n0;   // first B column this CTA loads
    const mt_tmap* tmB = (NB > 1 && rank == 1) ? tmB1 : tmB0;
    const int nk = (K + 31) / 32;
    auto A_raw = [&](int r) { return reinterpret_cast<float*>(smem + r * kRawBytes); };
    auto B_raw = [&](int r) { return reinterpret_cast<float*>(smem + r * kRawBytes + kABytes); };
    auto B_cv = [&](int c, int j) { return reinterpret_cast<float*>(smem + kConvOffset + c * kConvBytes + j * kBBytes); };

    if (threadIdx.x == 0) {
        for (int r = 0; r < RST; ++r) {
            mt_mbar_init(&rfull[r], 1);
            mt_mbar_init(&rempty[r], NCONV);
        }
        for (int c = 0; c < CST; ++c) {
            mt_mbar_init(&cfull[c], 2 * NCONV);
            mt_mbar_init(&cempty[c], SACC ? 2 : 1);   // SACC: both issuers read every stage
        }
        for (int b = 0; b < NACC; ++b) {
            mt_mbar_init(&tfull[b], 1);
            mt_mbar_init(&tempty[b], 16);
        }
        mt_mbar_init(&mdone[0], 1);
        mt_mbar_init(&mdone[1], 1);
        mt_mbar_init(sdone, 1);
        *abort_flag = 0;
        mt_fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        mt_tma_prefetch(tmA);
        mt_tma_prefetch(tmB);
    }
    if (warp == 1) mt_tmem_alloc_pair(tmem_slot, NCOLS);
    mt_tc_fence_before();
    __syncthreads();
    mt_cluster_sync();  // both CTAs' barriers initialised and tensor memory allocated
    mt_tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // TMA loads of k-tile kt into raw stage kt % RST (warp 16)
    auto tma_issue = [&](int kt) {
        const int r = kt % RST;
        mt_mbar_expect_tx(&rfull[r], kRawBytes);
        const int kg = kt * 32;
        mt_tma_load_2d(A_raw(r), tmA, &rfull[r], kg, m0);
        if (B_MN) mt_tma_load_3d(B_raw(r), tmB, &rfull[r], 0, kg, nb0 / 32);
        else mt_tma_load_2d(B_raw(r), tmB, &rfull[r], kg, nb0);
    };

    if (warp == 16) {
        if (lane == 0) {
            int issued = 0;
            for (int kt = 0; kt < nk; ++kt) {
                const int r = kt % RST;
                if (kt >= RST && !mt_mbar_wait(&rempty[r], (uint32_t)((kt / RST) - 1) & 1u, abort_flag, status, 1))
                    break;
                tma_issue(kt);
                issued = kt + 1;
            }
            if (*abort_flag) {
                for (int kt = (issued > RST ? issued - RST : 0); kt < issued; ++kt)
                    mt_mbar_drain(&rfull[kt % RST], (uint32_t)(kt / RST) & 1u);
            }
        }
    } else if (warp == 1 || (NISSUE == 2 && warp == 0)) {
        // NISSUE = 2: warp 1 issues the even chunks and warp 0 the odd ones (with
        // NACC = 2 each owns one accumulator buffer), so one issuer's barrier waits and
        // fences overlap the other's MMAs: a single issuing thread leaves the tensor
        // pipe idle for every cycle it spends between two MMAs (measured: an N-cycle
        // gap per 12 MMAs costs ~N cycles of pipe time).
        const int issuer = warp == 1 ? 0 : 1;
        if (SACC && rank == 0 && lane == 0) {
            // SACC: issuer 0 (warp 1) accumulates hi*hi of CHUNK k-tiles at a time into
            // the one chunk buffer, which the accumulator warps promote into fp32
            // registers; issuer 1 (warp 0) accumulates the small products hi*lo + lo*hi
            // of the whole K into their own buffer, read once at the end (they are
            // ~2^-11 of the result, so the tensor core's accumulation error on them is
            // negligible). While the chunk buffer drains, issuer 1 keeps the pipe busy.
            constexpr uint32_t idesc = mt_idesc_tf32(256, NMMA, false, B_MN);
            bool ok = true;
            const uint32_t dH = tmem, dS = tmem + (uint32_t)NMMA;
            if (issuer == 0) {
                const int nchunks = (nk + CHUNK - 1) / CHUNK;
                MT_PROF_BEGIN(tloop);
                for (int ch = 0; ch < nchunks && ok; ++ch) {
                    MT_PROF_BEGIN(w1);
                    if (ch >= 1 && !mt_mbar_wait(&tempty[0], (uint32_t)(ch - 1) & 1u, abort_flag, status, 2)) {
                        ok = false;
                        break;
                    }
                    MT_PROF_END(w1, p_mma_tempty);
                    const int kt0 = ch * CHUNK, kt1 = min(kt0 + CHUNK, nk);
                    for (int kt = kt0; kt < kt1; ++kt) {
                        const int c = kt % CST;
                        MT_PROF_BEGIN(w2);
                        if (!mt_mbar_wait(&cfull[c], (uint32_t)(kt / CST) & 1u, abort_flag, status, 2)) {
                            ok = false;
                            break;
                        }
                        MT_PROF_END(w2, p_mma_cfull);
                        mt_tc_fence_after();
                        const uint32_t ah = tmem + ACOLS + 64u * (uint32_t)c;
                        const uint32_t bh = mt_smem_u32(B_cv(c, 0));
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {
                            const uint64_t dbh = B_MN ? mt_operand_desc_mn(bh, kk) : mt_operand_desc_k(bh, kk);
                            mt_mma_tf32_ts_pair(dH, ah + 8u * (uint32_t)kk, dbh, idesc, (kt != kt0 || kk) ? 1u : 0u);
                        }
                        mt_mma_commit_pair_both(&cempty[c]);
                    }
                    if (ok) mt_mma_commit_pair_both(&tfull[0]);
                }
                MT_PROF_END(tloop, p_mma_loop);
            } else {
                for (int kt = 0; kt < nk && ok; ++kt) {
                    const int c = kt % CST;
                    MT_PROF_BEGIN(w6);
                    if (!mt_mbar_wait(&cfull[c], (uint32_t)(kt / CST) & 1u, abort_flag, status, 2)) {
                        ok = false;
                        break;
                    }
                    MT_PROF_END(w6, p_mma_issue);
                    mt_tc_fence_after();
                    const uint32_t ah = tmem + ACOLS + 64u * (uint32_t)c;
                    const uint32_t bh = mt_smem_u32(B_cv(c, 0)), bl = mt_smem_u32(B_cv(c, 1));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t dah = ah + 8u * (uint32_t)kk;
                        const uint32_t dal = dah + 32u;
                        const uint64_t dbh = B_MN ? mt_operand_desc_mn(bh, kk) : mt_operand_desc_k(bh, kk);
                        const uint64_t dbl = B_MN ? mt_operand_desc_mn(bl, kk) : mt_operand_desc_k(bl, kk);
                        mt_mma_tf32_ts_pair(dS, dah, dbl, idesc, (kt || kk) ? 1u : 0u);
                        mt_mma_tf32_ts_pair(dS, dal, dbh, idesc, 1u);
                    }
                    mt_mma_commit_pair_both(&cempty[c]);
                }
                if (ok) mt_mma_commit_pair_both(sdone);
            }
            if (!ok) {  // let the MMAs in flight finish before tensor memory is freed
                mt_mma_commit_pair_local(&mdone[issuer]);
                mt_mbar_drain(&mdone[issuer], 0);
            }
        } else if (!SACC && rank == 0 && lane == 0) {
            constexpr uint32_t idesc = mt_idesc_tf32(256, NMMA, false, B_MN);
            bool ok = true;
            const int nchunks = (nk + CHUNK - 1) / CHUNK;
            MT_PROF_BEGIN(tloop);
            for (int ch = issuer; ch < nchunks && ok; ch += NISSUE) {
                const int tb = ch % NACC;
                MT_PROF_BEGIN(w1);
                if (ch >= NACC && !mt_mbar_wait(&tempty[tb], (uint32_t)((ch / NACC) - 1) & 1u, abort_flag, status, 2)) {
                    ok = false;
                    break;
                }
                MT_PROF_END(w1, p_mma_tempty);
                // one tcgen05.fence::after_thread_sync per k-tile, after both waits
                const int kt0 = ch * CHUNK, kt1 = min(kt0 + CHUNK, nk);
                const uint32_t d = tmem + (uint32_t)(tb * NMMA);
                for (int kt = kt0; kt < kt1; ++kt) {
                    const int c = kt % CST;
                    MT_PROF_BEGIN(w2);
                    if (!mt_mbar_wait(&cfull[c], (uint32_t)(kt / CST) & 1u, abort_flag, status, 2)) {
                        ok = false;
                        break;
                    }
                    MT_PROF_END(w2, p_mma_cfull);
                    mt_tc_fence_after();
                    MT_PROF_BEGIN(w6);
                    const uint32_t ah = tmem + ACOLS + 64u * (uint32_t)c;
                    const uint32_t bh = mt_smem_u32(B_cv(c, 0)), bl = mt_smem_u32(B_cv(c, 1));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint32_t dah = ah + 8u * (uint32_t)kk;
                        const uint32_t dal = dah + 32u;
                        const uint64_t dbh = B_MN ? mt_operand_desc_mn(bh, kk) : mt_operand_desc_k(bh, kk);
                        const uint64_t dbl = B_MN ? mt_operand_desc_mn(bl, kk) : mt_operand_desc_k(bl, kk);
                        mt_mma_tf32_ts_pair(d, dah, dbl, idesc, (kt != kt0 || kk) ? 1u : 0u);
                        mt_mma_tf32_ts_pair(d, dal, dbh, idesc, 1u);
                        mt_mma_tf32_ts_pair(d, dah, dbh, idesc, 1u);
                    }
                    mt_mma_commit_pair_both(&cempty[c]);
                    MT_PROF_END(w6, p_mma_issue);
                }
                if (ok) mt_mma_commit_pair_both(&tfull[tb]);
            }
            MT_PROF_END(tloop, p_mma_loop);
            if (!ok) {  // let the MMAs in flight finish before tensor memory is freed
                mt_mma_commit_pair_local(&mdone[issuer]);
                mt_mbar_drain(&mdone[issuer], 0);
            }
        }
    } else if (warp >= 2 && warp < 8) {
        const int cw = warp - 2;
        const int ct = cw * 32 + lane;
        const uint32_t cfull_r0 = mt_cluster_map(cfull, 0);
        for (int kt = 0; kt < nk; ++kt) {
            const int r = kt % RST, c = kt % CST;
            MT_PROF_BEGIN(w3);
            if (!mt_mbar_wait(&rfull[r], (uint32_t)(kt / RST) & 1u, abort_flag, status, 3)) break;
            if (warp == 4 && lane == 0) MT_PROF_END(w3, p_conv_rfull);
            MT_PROF_BEGIN(w4);
            if (kt >= CST && !mt_mbar_wait(&cempty[c], (uint32_t)((kt / CST) - 1) & 1u, abort_flag, status, 3)) break;
            if (warp == 4 && lane == 0) MT_PROF_END(w4, p_conv_cempty);
            mt_tc_fence_after();
            if (warp >= 4)
                mt_convert_a_rows(A_raw(r), tmem + ACOLS + 64u * (uint32_t)c, warp & 3, lane, m0, kt * 32, M, K, proA);
            // BAL: warps 2-3 split B (32 elements per thread, as many as an A row) while
            // warps 4-7 split A; otherwise all six share B after their A rows
            if (!BAL)
                mt_convert_tile<false, false, BROWS, NCONV * 32>(B_raw(r), B_cv(c, 0), B_cv(c, 1), nb0, kt * 32, N, K,
                                                                 proB, ct);
            else if (warp < 4)
                mt_convert_tile<false, false, BROWS, 64>(B_raw(r), B_cv(c, 0), B_cv(c, 1), nb0, kt * 32, N, K, proB,
                                                         ct);
            mt_fence_proxy_async();
            mt_tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mt_mbar_arrive(&rempty[r]);
                mt_mbar_arrive_peer(cfull_r0 + (uint32_t)(c * 8));
            }
        }
    } else if (warp >= 8 && warp < 16) {
        const int q = warp & 3;
        const int h = (warp - 8) >> 2;
        const uint32_t tempty_r0 = mt_cluster_map(tempty, 0);
        float acc[NB][HALF];
#pragma unroll
        for (int b = 0; b < NB; ++b)
#pragma unroll
            for (int j = 0; j < HALF; ++j) acc[b][j] = 0.0f;
        bool ok = true;
        const int nchunks = (nk + CHUNK - 1) / CHUNK;
        for (int c = 0; c < nchunks; ++c) {
            const int tb = c % NACC;
            const uint32_t par = (uint32_t)(c / NACC) & 1u;
            MT_PROF_BEGIN(w5);
            const bool landed = mt_mbar_wait(&tfull[tb], par, abort_flag, status, 5);
            if (!landed) {
                ok = false;
                break;
            }
            if (warp == 8 && lane == 0) MT_PROF_END(w5, p_acc_tfull);
            __syncwarp();
            mt_tc_fence_after();
            // NB * HALF / 16 loads of 16 columns (544 threads leave 96 registers per
            // thread: 64 accumulators + 16 loaded values); the buffer is released as
            // soon as the last load has landed, before its adds
            constexpr int W = MT_PAIR_DRAIN_W;
            constexpr int PER = HALF / W;
            constexpr int NLD = NB * PER;
            float v[W];
#pragma unroll
            for (int l = 0; l < NLD; ++l) {
                const int b = l / PER, j = l % PER;
                if (l > 0) {
                    const int pb = (l - 1) / PER, pj = (l - 1) % PER;
#pragma unroll
                    for (int i = 0; i < W; ++i) acc[pb][pj * W + i] = __fadd_rn(acc[pb][pj * W + i], v[i]);
                }
                const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(tb * NMMA + b * BN + h * HALF + j * W);
                mt_tmem_ldw<W>(ta, v);
            }
            mt_tc_fence_before();
            __syncwarp();
            if (lane == 0) mt_mbar_arrive_peer(tempty_r0 + (uint32_t)(tb * 8));
            {
                constexpr int lb = (NLD - 1) / PER, lj = (NLD - 1) % PER;
#pragma unroll
                for (int i = 0; i < W; ++i) acc[lb][lj * W + i] = __fadd_rn(acc[lb][lj * W + i], v[i]);
            }
        }
        if constexpr (SACC) {
            // the small products of the whole K, added once
            if (ok && !mt_mbar_wait(sdone, 0, abort_flag, status, 5)) ok = false;
            if (ok) {
                __syncwarp();
                mt_tc_fence_after();
                constexpr int W = 16;
                constexpr int PER = HALF / W;
#pragma unroll
                for (int l = 0; l < NB * PER; ++l) {
                    const int b = l / PER, j = l % PER;
                    float v[W];
                    mt_tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(NACC * NMMA + b * BN + h * HALF + j * W), v);
#pragma unroll
                    for (int i = 0; i < W; ++i) acc[b][j * W + i] = __fadd_rn(acc[b][j * W + i], v[i]);
                }
            }
        }
        if (ok) {
            const int row = m0 + q * 32 + lane;
#pragma unroll
            for (int j = 0; j < HALF / 32; ++j) {
                float v[NB][32];
#pragma unroll
                for (int b = 0; b < NB; ++b)
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[b][i] = acc[b][j * 32 + i];
                epi.store(row, n0 + h * HALF + j * 32, v);
            }
        }
    }
    MT_PROF_FLUSH(status);
    mt_tc_fence_before();
    __syncthreads();
    mt_cluster_sync();  // no CTA frees tensor memory or exits while its partner may still use it
    if (warp == 1) {
        mt_tc_fence_after();
        mt_tmem_dealloc_pair(tmem, NCOLS);
    }
}
