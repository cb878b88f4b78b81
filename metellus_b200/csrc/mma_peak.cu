// tcgen05 kind::tf32 issue-rate microbenchmark: one CTA per SM, one thread issuing
// back-to-back 128 x N x 8 MMAs (A from shared memory "SS" or from tensor memory
// "TS", B from shared memory, zero data) and timing them with clock64 and CUDA events.
// Gives the tensor-pipe ceiling the 3xTF32 kernels are judged against (three MMAs per
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
template <int N, bool TS>
__global__ void __launch_bounds__(128, 1) bench(long long* out, int iters) {
    extern __shared__ __align__(1024) unsigned char raw[];
    unsigned char* sm = (unsigned char*)(((uintptr_t)raw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bar;
    __shared__ uint32_t slot;
    for (int i = threadIdx.x; i < (16384 + 32768) / 4; i += blockDim.x) ((float*)sm)[i] = 0.0f;
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
    if (threadIdx.x == 0) {
        const uint32_t a = su32(sm), b = su32(sm + 16384);
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
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" :: "r"(tmem) : "memory");
    }
}
template <int N, bool TS>
void run(long long* d, int iters) {
    auto k = bench<N, TS>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 60000);
    k<<<148, 128, 60000>>>(d, iters);
    cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
    cudaEventRecord(e0);
    k<<<148, 128, 60000>>>(d, iters);
    cudaEventRecord(e1); cudaEventSynchronize(e1);
    float ms; cudaEventElapsedTime(&ms, e0, e1);
    long long h[148]; cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
    double flops = 2.0 * 128 * N * 8 * 4 * (double)iters * 148;
    printf("N=%3d %s: %.1f cycles/MMA (CTA0), %.1f TF/s (1x tf32), err=%s\n", N, TS ? "TS" : "SS",
           (double)h[0] / (iters * 4), flops / ms / 1e9, cudaGetErrorString(cudaGetLastError()));
}
int main() {
    long long* d; cudaMalloc(&d, 148 * sizeof(long long));
    const int it = 4096;
    run<64, false>(d, it); run<64, true>(d, it);
    run<128, false>(d, it); run<128, true>(d, it);
    run<256, false>(d, it); run<256, true>(d, it);
    return 0;
}
