// tcgen05 kind::tf32 issue-rate microbenchmark: one CTA per SM, one thread issuing
// back-to-back 128 x N x 8 MMAs (A from shared memory "SS" or from tensor memory
// "TS", B from shared memory) and timing them with clock64 and CUDA events. Variants:
// zero or random operand data, and the 3xTF32 pattern (per 8-deep k step three MMAs
// over A hi / lo and B hi / lo: hi*lo, lo*hi, hi*hi, as the GEMM kernels issue them).
// Gives the tensor-pipe ceiling the 3xTF32 kernels are measured against (three MMAs per
// 8-deep k step). Build and run:
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -o mma_peak metellus_b200/csrc/mma_peak.cu && ./mma_peak
// The completion wait is bounded (the kernel reports -1 cycles if it gives up).
#include <cstdio>
#include <cstdint>
#include <cuda_runtime.h>
__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t sdesc(uint32_t a) {
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
__host__ __device__ constexpr uint32_t idesc(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ float rnd(uint32_t i) {  // deterministic pseudo-random tf32-ish value in [-1, 1)
    uint32_t x = i * 2654435761u + 12345u;
    x ^= x >> 13; x *= 0x5bd1e995u; x ^= x >> 15;
    return (float)(x & 0xFFFFFu) * (2.0f / 1048576.0f) - 1.0f;
}
// NOISE: other warps run alongside the MMA thread until it finishes: 1 = tcgen05.st
// streams into free tensor-memory columns (as the A split does), 2 = tcgen05.ld streams
// (as the accumulator drain does), 3 = both.
template <int N, bool TS, bool RANDOM, bool PAT3, int NOISE = 0>
__global__ void __launch_bounds__(128, 1) bench(long long* out, int iters) {
    extern __shared__ __align__(1024) unsigned char raw[];
    unsigned char* sm = (unsigned char*)(((uintptr_t)raw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bar;
    __shared__ uint32_t slot;
    __shared__ volatile int done;
    if (threadIdx.x == 0) done = 0;
    // A tile 16 KB at 0 (hi) and 16 KB (lo); B tiles (N x 32 fp32, up to 32 KB each) at 32 KB (hi) and 64 KB (lo)
    for (int i = threadIdx.x; i < (32768 + 65536) / 4; i += blockDim.x)
        ((float*)sm)[i] = RANDOM ? ((i >= 4096 && i < 8192) || i >= 16384 ? 1e-3f * rnd(i) : rnd(i)) : 0.0f;  // lo tiles small
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" :: "r"(su32(&slot)) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(su32(&bar)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = slot;
    if (TS) {  // A hi / lo into tensor memory columns [256, 320): lane = row
        const int w = threadIdx.x >> 5;
        for (int c = 0; c < 64; ++c) {
            const float v = RANDOM ? (c >= 32 ? 1e-3f * rnd(threadIdx.x * 64 + c + 7) : rnd(threadIdx.x * 64 + c + 7)) : 0.0f;
            asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};"
                         :: "r"(tmem + ((uint32_t)(w * 32) << 16) + 256u + (uint32_t)c), "r"(__float_as_uint(v)) : "memory");
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (NOISE && threadIdx.x >= 32) {
        const int w = threadIdx.x >> 5;
        const uint32_t lanes = (uint32_t)(w * 32) << 16;
        const bool st = (NOISE == 1) || (NOISE == 3 && w < 3);
        uint32_t r[32];
        for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(1.0f + i);
        for (long long it = 0; it < 50000000 && !done; ++it) {
            if (st) {
                asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
                             "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
                             :: "r"(tmem + lanes + 384u + 32u * (uint32_t)(it & 1)), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
                                "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
                                "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]),
                                "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]),
                                "r"(r[31]) : "memory");
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            } else {
                asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                             "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                             : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                               "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                               "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                               "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                             : "r"(tmem + lanes + 448u + 32u * (uint32_t)(it & 1)));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            }
        }
        if (r[0] == 12345u) out[148 + blockIdx.x] = r[1];  // keep the loads
    }
    if (threadIdx.x == 0 && PAT3) {
        const uint32_t ah = su32(sm), al = su32(sm + 16384), bh = su32(sm + 32768), bl = su32(sm + 65536);
        const long long t0 = clock64();
        for (int it = 0; it < iters; ++it) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint32_t acc = (it | kk) ? 1u : 0u;
                if (TS) {
                    const uint32_t th = tmem + 256u + 8u * kk, tl = th + 32u;
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
                                 :: "r"(tmem), "r"(th), "l"(sdesc(bl + 32u * kk)), "r"(idesc(128, N)), "r"(acc) : "memory");
                    asm volatile("tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, 1;"
                                 :: "r"(tmem), "r"(tl), "l"(sdesc(bh + 32u * kk)), "r"(idesc(128, N)) : "memory");
                    asm volatile("tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, 1;"
                                 :: "r"(tmem), "r"(th), "l"(sdesc(bh + 32u * kk)), "r"(idesc(128, N)) : "memory");
                } else {
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
                                 :: "r"(tmem), "l"(sdesc(ah + 32u * kk)), "l"(sdesc(bl + 32u * kk)), "r"(idesc(128, N)), "r"(acc) : "memory");
                    asm volatile("tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, 1;"
                                 :: "r"(tmem), "l"(sdesc(al + 32u * kk)), "l"(sdesc(bh + 32u * kk)), "r"(idesc(128, N)) : "memory");
                    asm volatile("tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, 1;"
                                 :: "r"(tmem), "l"(sdesc(ah + 32u * kk)), "l"(sdesc(bh + 32u * kk)), "r"(idesc(128, N)) : "memory");
                }
            }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(su32(&bar)) : "memory");
        uint32_t ok = 0;
        for (long long w = 0; w < 200000000 && !ok; ++w) {
            asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\tselp.b32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(su32(&bar)) : "memory");
        }
        const long long t1 = clock64();
        out[blockIdx.x] = ok ? (t1 - t0) : -1;
        done = 1;
    } else if (threadIdx.x == 0) {
        const uint32_t a = su32(sm), b = su32(sm + 32768);
        const long long t0 = clock64();
        for (int it = 0; it < iters; ++it) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint32_t acc = (it | kk) ? 1u : 0u;
                if (TS) {
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
                                 :: "r"(tmem), "r"(tmem + 256u + 8u * kk), "l"(sdesc(b + 32u * kk)), "r"(idesc(128, N)), "r"(acc) : "memory");
                } else {
                    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                                 "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
                                 :: "r"(tmem), "l"(sdesc(a + 32u * kk)), "l"(sdesc(b + 32u * kk)), "r"(idesc(128, N)), "r"(acc) : "memory");
                }
            }
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(su32(&bar)) : "memory");
        uint32_t ok = 0;
        for (long long w = 0; w < 200000000 && !ok; ++w) {
            asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\tselp.b32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(su32(&bar)) : "memory");
        }
        const long long t1 = clock64();
        out[blockIdx.x] = ok ? (t1 - t0) : -1;
        done = 1;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" :: "r"(tmem) : "memory");
    }
}
// CTA pairs: clusters of two CTAs, the even one issuing tcgen05.mma.cta_group::2
// (M = 256: 128 A rows from each CTA's tensor memory; N columns of B split between the
// two CTAs' shared memory), the 3xTF32 pattern on random data.
// COMMITS: per 12 MMAs (one 32-deep k-tile of the GEMM) that many multicast commits to
// spare barriers, as the GEMM's MMA thread issues (stage free + accumulator ready).
// SWITCH: every 12 MMAs start a fresh accumulator in the other of two TMEM buffers, as
// the GEMM does per k-tile (one buffer per 32-deep chunk, ping-pong).
// FENCE: before every 12 MMAs a tcgen05.fence::after_thread_sync, as the GEMM's MMA
// thread issues after each barrier wait.
// DELAY: the issuing thread spins that many cycles before every 12 MMAs (stand-in for
// the barrier waits between k-tiles): shows how much work the tensor pipe has queued.
template <int N, int COMMITS = 0, bool SWITCH = false, bool FENCE = false, int DELAY = 0>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(128, 1) bench_pair(long long* out, int iters) {
    extern __shared__ __align__(1024) unsigned char raw[];
    unsigned char* sm = (unsigned char*)(((uintptr_t)raw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bar;
    __shared__ uint64_t spare[2];
    __shared__ uint32_t slot;
    uint32_t rank;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    for (int i = threadIdx.x; i < (32768 + 65536) / 4; i += blockDim.x)
        ((float*)sm)[i] = (i >= 16384 ? 1e-3f : 1.0f) * rnd(i + 77 * rank);
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" :: "r"(su32(&slot)) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(su32(&bar)) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(su32(&spare[0])) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(su32(&spare[1])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = slot;
    {
        const int w = threadIdx.x >> 5;
        for (int c = 0; c < 64; ++c) {
            const float v = (c >= 32 ? 1e-3f : 1.0f) * rnd(threadIdx.x * 64 + c + 7 + 999 * rank);
            asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};"
                         :: "r"(tmem + ((uint32_t)(w * 32) << 16) + 256u + (uint32_t)c), "r"(__float_as_uint(v)) : "memory");
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (threadIdx.x == 0 && rank == 0) {
        const uint32_t bh = su32(sm + 32768), bl = su32(sm + 65536);
        const long long t0 = clock64();
        for (int it = 0; it < iters; ++it) {
            if (DELAY) {
                const long long d0 = clock64();
                while (clock64() - d0 < DELAY) { }
            }
            if (FENCE) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t dd = tmem + (SWITCH ? 128u * (uint32_t)(it & 1) : 0u);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint32_t acc = (SWITCH ? kk : (it | kk)) ? 1u : 0u;
                const uint32_t th = tmem + 256u + 8u * kk, tl = th + 32u;
                asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                             "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
                             :: "r"(dd), "r"(th), "l"(sdesc(bl + 32u * kk)), "r"(idesc(256, N)), "r"(acc) : "memory");
                asm volatile("tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, 1;"
                             :: "r"(dd), "r"(tl), "l"(sdesc(bh + 32u * kk)), "r"(idesc(256, N)) : "memory");
                asm volatile("tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, 1;"
                             :: "r"(dd), "r"(th), "l"(sdesc(bh + 32u * kk)), "r"(idesc(256, N)) : "memory");
            }
            for (int c = 0; c < COMMITS; ++c) {
                const unsigned short both = 3;
                asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                             :: "r"(su32(&spare[c & 1])), "h"(both) : "memory");
            }
        }
        asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(su32(&bar)) : "memory");
        uint32_t ok = 0;
        for (long long w = 0; w < 200000000 && !ok; ++w) {
            asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\tselp.b32 %0, 1, 0, p;\n\t}" : "=r"(ok) : "r"(su32(&bar)) : "memory");
        }
        const long long t1 = clock64();
        out[blockIdx.x / 2] = ok ? (t1 - t0) : -1;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" :: "r"(tmem) : "memory");
    }
}
template <int N, int COMMITS = 0, bool SWITCH = false, bool FENCE = false, int DELAY = 0>
void run_pair(long long* d, int iters) {
    auto k = bench_pair<N, COMMITS, SWITCH, FENCE, DELAY>;
    const int smem = 32768 + 65536 + 1024;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    k<<<148, 128, smem>>>(d, iters);
    cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
    cudaEventRecord(e0);
    k<<<148, 128, smem>>>(d, iters);
    cudaEventRecord(e1); cudaEventSynchronize(e1);
    float ms; cudaEventElapsedTime(&ms, e0, e1);
    long long h[74]; cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    double flops = 2.0 * 256 * N * 8 * 12 * (double)iters * 74;
    printf("pair M=256 N=%3d TS random 3xTF32 pattern, %d commits per 12 MMAs%s, %d-cycle gap: %.1f cycles/MMA (cluster 0), %.1f TF/s (1x tf32), err=%s\n", N, COMMITS,
           SWITCH ? (FENCE ? ", fresh accumulator buffer and a tcgen05.fence::after_thread_sync per 12 MMAs"
                           : ", fresh accumulator buffer per 12 MMAs") : "", DELAY,
           (double)h[0] / (iters * 12), flops / ms / 1e9, cudaGetErrorString(cudaGetLastError()));
}
template <int N, bool TS, bool RANDOM = false, bool PAT3 = false, int NOISE = 0>
void run(long long* d, int iters) {
    auto k = bench<N, TS, RANDOM, PAT3, NOISE>;
    const int smem = 32768 + 65536 + 1024;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    k<<<148, 128, smem>>>(d, iters);
    cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
    cudaEventRecord(e0);
    k<<<148, 128, smem>>>(d, iters);
    cudaEventRecord(e1); cudaEventSynchronize(e1);
    float ms; cudaEventElapsedTime(&ms, e0, e1);
    long long h[148]; cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    const int per_it = PAT3 ? 12 : 4;
    double flops = 2.0 * 128 * N * 8 * per_it * (double)iters * 148;
    printf("N=%3d %s %s %s%s: %.1f cycles/MMA (CTA0), %.1f TF/s (1x tf32), err=%s\n", N, TS ? "TS" : "SS",
           RANDOM ? "random" : "zeros ", PAT3 ? "3xTF32 pattern" : "one operand pair",
           NOISE == 1 ? " + TMEM stores" : NOISE == 2 ? " + TMEM loads" : NOISE == 3 ? " + TMEM stores and loads" : "",
           (double)h[0] / (iters * per_it), flops / ms / 1e9, cudaGetErrorString(cudaGetLastError()));
}
int main() {
    long long* d; cudaMalloc(&d, 2 * 148 * sizeof(long long));
    const int it = 4096;
    run<64, false>(d, it); run<64, true>(d, it);
    run<128, false>(d, it); run<128, true>(d, it);
    run<256, false>(d, it); run<256, true>(d, it);
    run<128, true, true>(d, it);
    run<128, true, false, true>(d, it / 3);
    run<128, true, true, true>(d, it / 3);
    run<128, false, true, true>(d, it / 3);
    run<256, true, true, true>(d, it / 3);
    run<128, true, true, true, 1>(d, it / 3);
    run<128, true, true, true, 2>(d, it / 3);
    run<128, true, true, true, 3>(d, it / 3);
    run_pair<128>(d, it / 3);
    run_pair<256>(d, it / 3);
    run_pair<128, 2>(d, it / 3);
    run_pair<128, 2, true>(d, it / 3);
    run_pair<128, 2, true, true>(d, it / 3);
    run_pair<128, 2, true, true, 200>(d, it / 3);
    run_pair<128, 2, true, true, 400>(d, it / 3);
    run_pair<128, 2, true, true, 800>(d, it / 3);
    return 0;
}
