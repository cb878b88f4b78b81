// Native backend of Metellus for NVIDIA B200 (sm_100a): the C ABI declared in
// include/metellus_b200.h. It takes over from the reference's Objective-C++ Metal
// backend (src/metal_backend.mm): where that module recompiles MSL on every
// run_kernel call and waits for each command buffer, this one compiles once with
// NVRTC (the Python layer keeps an on-disk cubin cache), allocates from a
// stream-ordered memory pool, launches asynchronously on one stream per device and
// only synchronises on reads, explicit syncs and profile-mode launches.
#include <cuda.h>
#include <cuda_runtime.h>
#include <nvrtc.h>

#include <dlfcn.h>
#include <nccl.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/metellus_b200.h"

namespace {

thread_local std::string g_err;

// Driver API entry points, resolved through the runtime at first use so that the
// library loads (and exports its symbols) on machines without a GPU driver.
struct DriverApi {
    decltype(&cuModuleLoadData) ModuleLoadData = nullptr;
    decltype(&cuModuleGetFunction) ModuleGetFunction = nullptr;
    decltype(&cuFuncSetAttribute) FuncSetAttribute = nullptr;
    decltype(&cuFuncGetAttribute) FuncGetAttribute = nullptr;
    decltype(&cuLaunchKernel) LaunchKernel = nullptr;
    decltype(&cuLaunchKernelEx) LaunchKernelEx = nullptr;
    decltype(&cuTensorMapEncodeTiled) TensorMapEncodeTiled = nullptr;
    decltype(&cuGetErrorString) GetErrorString = nullptr;
    bool ok = false;
} g_drv;

int fail(const char* fmt, ...) {
    char buf[2048];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return 1;
}

#define RT_CHECK(call)                                                               \
    do {                                                                             \
        cudaError_t e_ = (call);                                                     \
        if (e_ != cudaSuccess)                                                       \
            return fail("%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_),      \
                        __FILE__, __LINE__);                                         \
    } while (0)

#define DRV_CHECK(call)                                                              \
    do {                                                                             \
        if (load_driver()) return 1;                                                 \
        CUresult r_ = (g_drv.call);                                                  \
        if (r_ != CUDA_SUCCESS) {                                                    \
            const char* s_ = nullptr;                                                \
            if (g_drv.GetErrorString) g_drv.GetErrorString(r_, &s_);                 \
            return fail("%s failed: %s (%s:%d)", #call, s_ ? s_ : "?", __FILE__,     \
                        __LINE__);                                                   \
        }                                                                            \
    } while (0)

int load_driver() {
    if (g_drv.ok) return 0;
    cudaDriverEntryPointQueryResult q;
#define MT_SYM(field, name)                                                                   \
    if (cudaGetDriverEntryPoint(name, (void**)&g_drv.field, cudaEnableDefault, &q) != cudaSuccess || \
        !g_drv.field)                                                                         \
        return fail("driver entry point %s unavailable", name);
    MT_SYM(ModuleLoadData, "cuModuleLoadData")
    MT_SYM(ModuleGetFunction, "cuModuleGetFunction")
    MT_SYM(FuncSetAttribute, "cuFuncSetAttribute")
    MT_SYM(FuncGetAttribute, "cuFuncGetAttribute")
    MT_SYM(LaunchKernel, "cuLaunchKernel")
    MT_SYM(LaunchKernelEx, "cuLaunchKernelEx")
    MT_SYM(TensorMapEncodeTiled, "cuTensorMapEncodeTiled")
    MT_SYM(GetErrorString, "cuGetErrorString")
#undef MT_SYM
    g_drv.ok = true;
    return 0;
}

constexpr int kMaxDev = 16;

struct Device {
    bool ready = false;
    cudaStream_t stream = nullptr;
    cudaStream_t d2h = nullptr;  // copy stream for downloads that overlap the next uploads
    cudaMemPool_t pool = nullptr;
    ncclComm_t comm = nullptr;  // set by mt_nccl_init
};

struct Buffer {
    int dev;
    void* ptr;
    size_t size;
};

struct KernelEntry {
    std::vector<char> cubin;
    std::string fn;
    CUmodule mod[kMaxDev] = {};
    CUfunction func[kMaxDev] = {};
    int smem_attr[kMaxDev] = {};
};

std::mutex g_mu;
Device g_dev[kMaxDev];
std::map<uint64_t, Buffer> g_bufs;
std::map<uint64_t, std::unique_ptr<KernelEntry>> g_kernels;
std::map<uint64_t, cudaEvent_t> g_events;
std::map<uint64_t, cudaGraphExec_t> g_graphs;
uint64_t g_next = 1;

int ensure_dev(int dev) {
    if (dev < 0 || dev >= kMaxDev) return fail("device index %d out of range", dev);
    Device& d = g_dev[dev];
    RT_CHECK(cudaSetDevice(dev));
    if (d.ready) return 0;
    RT_CHECK(cudaFree(nullptr));  // create / bind the primary context
    RT_CHECK(cudaStreamCreateWithFlags(&d.stream, cudaStreamNonBlocking));
    RT_CHECK(cudaStreamCreateWithFlags(&d.d2h, cudaStreamNonBlocking));
    RT_CHECK(cudaDeviceGetDefaultMemPool(&d.pool, dev));
    uint64_t keep = ~0ull;  // keep freed blocks cached in the pool
    RT_CHECK(cudaMemPoolSetAttribute(d.pool, cudaMemPoolAttrReleaseThreshold, &keep));
    d.ready = true;
    return 0;
}

int get_buf(uint64_t h, Buffer* out) {
    auto it = g_bufs.find(h);
    if (it == g_bufs.end()) return fail("unknown buffer handle %llu", (unsigned long long)h);
    *out = it->second;
    return 0;
}

int get_func(KernelEntry* k, int dev, CUfunction* f) {
    if (!k->func[dev]) {
        DRV_CHECK(ModuleLoadData(&k->mod[dev], k->cubin.data()));
        DRV_CHECK(ModuleGetFunction(&k->func[dev], k->mod[dev], k->fn.c_str()));
    }
    *f = k->func[dev];
    return 0;
}

}  // namespace

// ---- native split-row reduction ------------------------------------------------

namespace {

constexpr int kRedThreads = 256;

struct RedSum { static __device__ double id() { return 0.0; }
                static __device__ double op(double a, double b) { return a + b; } };
struct RedProd { static __device__ double id() { return 1.0; }
                 static __device__ double op(double a, double b) { return a * b; } };
struct RedMax { static __device__ double id() { return -__longlong_as_double(0x7ff0000000000000ll); }
                static __device__ double op(double a, double b) { return fmax(a, b); } };
struct RedMin { static __device__ double id() { return __longlong_as_double(0x7ff0000000000000ll); }
                static __device__ double op(double a, double b) { return fmin(a, b); } };

template <class R>
__device__ double block_reduce(double v, double* sh) {
    for (int o = 16; o > 0; o >>= 1) v = R::op(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    double r = R::id();
    if (threadIdx.x < 32) {
        r = (lane < kRedThreads / 32) ? sh[lane] : R::id();
        for (int o = 16; o > 0; o >>= 1) r = R::op(r, __shfl_xor_sync(0xffffffffu, r, o));
    }
    return r;  // valid in thread 0
}

// grid (splits, rows): block (s, r) reduces columns [s*chunk, min((s+1)*chunk, cols))
// of row r into partials[r * splits + s]; the last block of the row (ticket) combines
// the partials in split order and writes out[r] (fp32, or the fp64 value itself for
// a partial that another GPU's partials are combined with).
template <class R, class OutT>
__global__ void __launch_bounds__(kRedThreads) reduce_rows_split(const float* __restrict__ in,
                                                                 OutT* __restrict__ out, double* partials,
                                                                 unsigned* tickets, unsigned long long cols,
                                                                 unsigned long long ld, unsigned long long chunk) {
    __shared__ double sh[kRedThreads / 32];
    __shared__ bool last;
    const unsigned long long r = blockIdx.y, s = blockIdx.x, splits = gridDim.x;
    const unsigned long long c0 = s * chunk, c1 = (c0 + chunk < cols) ? c0 + chunk : cols;
    const float* row = in + r * ld;
    double acc = R::id();
    // 16-byte aligned vector body when the row start and c0 allow it
    unsigned long long c = c0;
    const bool vec = ((reinterpret_cast<uintptr_t>(row + c0) & 15u) == 0);
    if (vec) {
        const unsigned long long n4 = (c1 - c0) / 4;
        const float4* p4 = reinterpret_cast<const float4*>(row + c0);
        for (unsigned long long i = threadIdx.x; i < n4; i += kRedThreads) {
            const float4 v = __ldcs(p4 + i);
            acc = R::op(acc, R::op(R::op((double)v.x, (double)v.y), R::op((double)v.z, (double)v.w)));
        }
        c = c0 + n4 * 4;
    }
    for (unsigned long long i = c + threadIdx.x; i < c1; i += kRedThreads) acc = R::op(acc, (double)row[i]);
    const double part = block_reduce<R>(acc, sh);
    if (threadIdx.x == 0) {
        partials[r * splits + s] = part;
        __threadfence();
        last = (atomicAdd(&tickets[r], 1u) == (unsigned)(splits - 1));
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    double tot = R::id();
    for (unsigned long long i = threadIdx.x; i < splits; i += kRedThreads)
        tot = R::op(tot, ((volatile double*)partials)[r * splits + i]);
    tot = block_reduce<R>(tot, sh);
    if (threadIdx.x == 0) {
        out[r] = (OutT)tot;
        tickets[r] = 0;  // ready for the next launch on the same scratch
    }
}

// Grid shape for a rows x cols reduction: about 8 blocks per SM in total, at least
// 4096 columns per block.
void reduce_plan(unsigned long long rows, unsigned long long cols, int sms, unsigned long long* splits,
                 unsigned long long* chunk) {
    unsigned long long want = (unsigned long long)sms * 8ull / (rows ? rows : 1);
    unsigned long long max_by_len = (cols + 4095) / 4096;
    unsigned long long sp = want < max_by_len ? want : max_by_len;
    if (sp < 1) sp = 1;
    if (sp > 65535) sp = 65535;
    unsigned long long ch = (cols + sp - 1) / sp;
    ch = (ch + 3) / 4 * 4;  // keep every split start 16-byte aligned when the row is
    *chunk = ch;
    *splits = (cols + ch - 1) / ch;
}

// op 0..3 = sum / max / min / product with fp32 output; 4..7 the same with fp64 output.
int launch_reduce(int op, cudaStream_t st, unsigned long long splits, unsigned long long rows, const float* in,
                  void* out, double* partials, unsigned* tickets, unsigned long long cols, unsigned long long ld,
                  unsigned long long chunk) {
    dim3 grid((unsigned)splits, (unsigned)rows);
    float* o32 = (float*)out;
    double* o64 = (double*)out;
    switch (op) {
        case 0: reduce_rows_split<RedSum><<<grid, kRedThreads, 0, st>>>(in, o32, partials, tickets, cols, ld, chunk); break;
        case 1: reduce_rows_split<RedMax><<<grid, kRedThreads, 0, st>>>(in, o32, partials, tickets, cols, ld, chunk); break;
        case 2: reduce_rows_split<RedMin><<<grid, kRedThreads, 0, st>>>(in, o32, partials, tickets, cols, ld, chunk); break;
        case 3: reduce_rows_split<RedProd><<<grid, kRedThreads, 0, st>>>(in, o32, partials, tickets, cols, ld, chunk); break;
        case 4: reduce_rows_split<RedSum><<<grid, kRedThreads, 0, st>>>(in, o64, partials, tickets, cols, ld, chunk); break;
        case 5: reduce_rows_split<RedMax><<<grid, kRedThreads, 0, st>>>(in, o64, partials, tickets, cols, ld, chunk); break;
        case 6: reduce_rows_split<RedMin><<<grid, kRedThreads, 0, st>>>(in, o64, partials, tickets, cols, ld, chunk); break;
        case 7: reduce_rows_split<RedProd><<<grid, kRedThreads, 0, st>>>(in, o64, partials, tickets, cols, ld, chunk); break;
        default: return fail("mt_reduce_rows: op %d is not 0..7", op);
    }
    RT_CHECK(cudaGetLastError());
    return 0;
}

}  // namespace

// ---- allocation-free variant of mt_reduce_rows -------------------------------------
//
// Scratch for mt_reduce_rows_noalloc: one fixed array per device, part of this
// library's device image, so the entry point never allocates. 256 KiB holds the fp64
// partials and tickets of any plan with rows * splits * 8 + rows * 4 <= 256 KiB: a
// whole-tensor or few-row reduction needs about 10 KB (8 blocks per SM in total), and
// one-split plans fit up to 21,845 rows. Every GPU that loads the library keeps this
// array until the process exits.
static constexpr size_t kNoAllocScratchBytes = size_t(256) << 10;
static __device__ __align__(256) unsigned char mt_noalloc_scratch[kNoAllocScratchBytes];

namespace {
void* g_noalloc_scratch_ptr[kMaxDev] = {};  // device address of mt_noalloc_scratch per device
std::mutex g_noalloc_mu;
}  // namespace

extern "C" {

int mt_last_error(char* buf, size_t n) {
    if (!buf || n == 0) return 1;
    snprintf(buf, n, "%s", g_err.c_str());
    return 0;
}

int mt_device_count(int* n) {
    int c = 0;
    cudaError_t e = cudaGetDeviceCount(&c);
    if (e != cudaSuccess) {
        *n = 0;
        cudaGetLastError();
        return 0;
    }
    *n = c;
    return 0;
}

int mt_init(int dev) {
    std::lock_guard<std::mutex> lk(g_mu);
    return ensure_dev(dev);
}

int mt_device_attr(int dev, int which, int64_t* out) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (ensure_dev(dev)) return 1;
    int v = 0;
    switch (which) {
        case 0: RT_CHECK(cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev)); break;
        case 1: RT_CHECK(cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)); break;
        case 2: {
            int a = 0, b = 0;
            RT_CHECK(cudaDeviceGetAttribute(&a, cudaDevAttrComputeCapabilityMajor, dev));
            RT_CHECK(cudaDeviceGetAttribute(&b, cudaDevAttrComputeCapabilityMinor, dev));
            v = a * 10 + b;
            break;
        }
        case 3: RT_CHECK(cudaDeviceGetAttribute(&v, cudaDevAttrL2CacheSize, dev)); break;
        default: return fail("unknown attribute %d", which);
    }
    *out = v;
    return 0;
}

int mt_buffer_create(int dev, size_t nbytes, uint64_t* handle) {
    if (nbytes == 0) return fail("buffer nbytes must be > 0");
    std::lock_guard<std::mutex> lk(g_mu);
    if (ensure_dev(dev)) return 1;
    void* p = nullptr;
    RT_CHECK(cudaMallocAsync(&p, nbytes, g_dev[dev].pool, g_dev[dev].stream));
    uint64_t h = g_next++;
    g_bufs[h] = Buffer{dev, p, nbytes};
    *handle = h;
    return 0;
}

int mt_buffer_release(uint64_t handle) {
    std::lock_guard<std::mutex> lk(g_mu);
    Buffer b;
    if (get_buf(handle, &b)) return 1;
    RT_CHECK(cudaSetDevice(b.dev));
    RT_CHECK(cudaFreeAsync(b.ptr, g_dev[b.dev].stream));
    g_bufs.erase(handle);
    return 0;
}

int mt_buffer_size(uint64_t handle, size_t* nbytes) {
    std::lock_guard<std::mutex> lk(g_mu);
    Buffer b;
    if (get_buf(handle, &b)) return 1;
    *nbytes = b.size;
    return 0;
}

int mt_buffer_ptr(uint64_t handle, uint64_t* dptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    Buffer b;
    if (get_buf(handle, &b)) return 1;
    *dptr = (uint64_t)(uintptr_t)b.ptr;
    return 0;
}

static int copy_common(uint64_t handle, void* host, size_t nbytes, bool to_dev, bool wait) {
    Buffer b;
    cudaStream_t s;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (get_buf(handle, &b)) return 1;
        s = g_dev[b.dev].stream;
    }
    if (nbytes > b.size) return fail("copy of %zu bytes exceeds buffer of %zu bytes", nbytes, b.size);
    RT_CHECK(cudaSetDevice(b.dev));
    if (to_dev)
        RT_CHECK(cudaMemcpyAsync(b.ptr, host, nbytes, cudaMemcpyHostToDevice, s));
    else
        RT_CHECK(cudaMemcpyAsync(host, b.ptr, nbytes, cudaMemcpyDeviceToHost, s));
    if (wait) RT_CHECK(cudaStreamSynchronize(s));
    return 0;
}

int mt_buffer_write(uint64_t h, const void* src, size_t n) { return copy_common(h, (void*)src, n, true, true); }
int mt_buffer_read(uint64_t h, void* dst, size_t n) { return copy_common(h, dst, n, false, true); }
int mt_buffer_write_async(uint64_t h, const void* src, size_t n) { return copy_common(h, (void*)src, n, true, false); }
int mt_buffer_read_async(uint64_t h, void* dst, size_t n) { return copy_common(h, dst, n, false, false); }

int mt_buffer_read_after(uint64_t h, void* dst, size_t n, uint64_t after, uint64_t done) {
    Buffer b;
    cudaStream_t s;
    cudaEvent_t ea = nullptr, ed = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (get_buf(h, &b)) return 1;
        s = g_dev[b.dev].d2h;
        if (after) {
            auto it = g_events.find(after);
            if (it == g_events.end()) return fail("mt_buffer_read_after: unknown event %llu", (unsigned long long)after);
            ea = it->second;
        }
        if (done) {
            auto it = g_events.find(done);
            if (it == g_events.end()) return fail("mt_buffer_read_after: unknown event %llu", (unsigned long long)done);
            ed = it->second;
        }
    }
    if (n > b.size) return fail("copy of %zu bytes exceeds buffer of %zu bytes", n, b.size);
    RT_CHECK(cudaSetDevice(b.dev));
    if (ea) RT_CHECK(cudaStreamWaitEvent(s, ea, 0));
    RT_CHECK(cudaMemcpyAsync(dst, b.ptr, n, cudaMemcpyDeviceToHost, s));
    if (ed) RT_CHECK(cudaEventRecord(ed, s));
    return 0;
}

int mt_buffer_fill(uint64_t handle, uint8_t value) {
    Buffer b;
    cudaStream_t s;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (get_buf(handle, &b)) return 1;
        s = g_dev[b.dev].stream;
    }
    RT_CHECK(cudaSetDevice(b.dev));
    RT_CHECK(cudaMemsetAsync(b.ptr, value, b.size, s));
    RT_CHECK(cudaStreamSynchronize(s));
    return 0;
}

int mt_buffer_fill_async(uint64_t handle, uint8_t value) {
    Buffer b;
    cudaStream_t s;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (get_buf(handle, &b)) return 1;
        s = g_dev[b.dev].stream;
    }
    RT_CHECK(cudaSetDevice(b.dev));
    RT_CHECK(cudaMemsetAsync(b.ptr, value, b.size, s));
    return 0;
}

int mt_host_alloc(size_t nbytes, void** ptr) {
    RT_CHECK(cudaHostAlloc(ptr, nbytes, cudaHostAllocPortable));
    return 0;
}

int mt_host_free(void* ptr) {
    RT_CHECK(cudaFreeHost(ptr));
    return 0;
}

int mt_nvrtc_compile(const char* src, const char* name, const char* opts, void* cubin, size_t cap,
                     size_t* size, char* log, size_t logcap) {
    nvrtcProgram prog;
    nvrtcResult r = nvrtcCreateProgram(&prog, src, name ? name : "kernel.cu", 0, nullptr, nullptr);
    if (r != NVRTC_SUCCESS) return fail("nvrtcCreateProgram: %s", nvrtcGetErrorString(r));
    std::vector<std::string> args;
    {
        std::string o = opts ? opts : "";
        size_t i = 0;
        while (i < o.size()) {
            while (i < o.size() && o[i] == ' ') ++i;
            size_t j = i;
            while (j < o.size() && o[j] != ' ') ++j;
            if (j > i) args.push_back(o.substr(i, j - i));
            i = j;
        }
    }
    std::vector<const char*> argv;
    for (auto& a : args) argv.push_back(a.c_str());
    r = nvrtcCompileProgram(prog, (int)argv.size(), argv.data());
    size_t lsz = 0;
    nvrtcGetProgramLogSize(prog, &lsz);
    std::string lg(lsz, '\0');
    if (lsz) nvrtcGetProgramLog(prog, &lg[0]);
    if (log && logcap) snprintf(log, logcap, "%s", lg.c_str());
    if (r != NVRTC_SUCCESS) {
        nvrtcDestroyProgram(&prog);
        return fail("NVRTC compile of %s failed: %s\n%s", name ? name : "kernel", nvrtcGetErrorString(r),
                    lg.c_str());
    }
    size_t n = 0;
    r = nvrtcGetCUBINSize(prog, &n);
    if (r != NVRTC_SUCCESS) {
        nvrtcDestroyProgram(&prog);
        return fail("nvrtcGetCUBINSize: %s", nvrtcGetErrorString(r));
    }
    *size = n;
    if (cubin && cap >= n) nvrtcGetCUBIN(prog, (char*)cubin);
    nvrtcDestroyProgram(&prog);
    return 0;
}

int mt_kernel_load(const void* cubin, size_t size, const char* fn, uint64_t* kernel) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto k = std::make_unique<KernelEntry>();
    k->cubin.assign((const char*)cubin, (const char*)cubin + size);
    k->fn = fn;
    uint64_t h = g_next++;
    g_kernels[h] = std::move(k);
    *kernel = h;
    return 0;
}

int mt_kernel_info(int dev, uint64_t kernel, int* regs, int* local_bytes, int* max_threads) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (ensure_dev(dev)) return 1;
    auto it = g_kernels.find(kernel);
    if (it == g_kernels.end()) return fail("unknown kernel handle");
    CUfunction f;
    if (get_func(it->second.get(), dev, &f)) return 1;
    DRV_CHECK(FuncGetAttribute(regs, CU_FUNC_ATTRIBUTE_NUM_REGS, f));
    DRV_CHECK(FuncGetAttribute(local_bytes, CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, f));
    DRV_CHECK(FuncGetAttribute(max_threads, CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, f));
    return 0;
}

int mt_launch(int dev, uint64_t kernel, const uint64_t* buffers, int nbuf, const uint32_t* dims,
              int ndims, const uint32_t grid[3], const uint32_t block[3], uint32_t dyn_smem,
              uint32_t cluster_x, const mt_tmap_spec* tmaps, int ntmaps, float* time_ms) {
    if (ndims < 0 || ndims > 16) return fail("ndims %d out of range (max 16)", ndims);
    if (nbuf < 0 || nbuf > 64) return fail("nbuf %d out of range (max 64)", nbuf);
    if (ntmaps < 0 || ntmaps > 8) return fail("ntmaps %d out of range (max 8)", ntmaps);
    CUfunction f;
    cudaStream_t s;
    std::vector<uint64_t> ptrs(nbuf);
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (ensure_dev(dev)) return 1;
        auto it = g_kernels.find(kernel);
        if (it == g_kernels.end()) return fail("unknown kernel handle %llu", (unsigned long long)kernel);
        KernelEntry* k = it->second.get();
        if (get_func(k, dev, &f)) return 1;
        if ((int)dyn_smem > k->smem_attr[dev]) {
            DRV_CHECK(FuncSetAttribute(f, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)dyn_smem));
            k->smem_attr[dev] = (int)dyn_smem;
        }
        for (int i = 0; i < nbuf; ++i) {
            Buffer b;
            if (get_buf(buffers[i], &b)) return 1;
            if (b.dev != dev) return fail("buffer %d lives on device %d, launch is on %d", i, b.dev, dev);
            ptrs[i] = (uint64_t)(uintptr_t)b.ptr;
        }
        s = g_dev[dev].stream;
    }
    struct alignas(64) Dims { uint32_t d[16]; } dimblk;
    memset(&dimblk, 0, sizeof dimblk);
    for (int i = 0; i < ndims; ++i) dimblk.d[i] = dims[i];
    std::vector<CUtensorMap> maps(ntmaps > 0 ? ntmaps : 1);
    for (int t = 0; t < ntmaps; ++t) {
        const mt_tmap_spec& sp = tmaps[t];
        if (sp.buf_index < 0 || sp.buf_index >= nbuf) return fail("tmap %d: bad buffer index", t);
        static const CUtensorMapSwizzle sw[] = {CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_SWIZZLE_32B,
                                                CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_SWIZZLE_128B,
                                                CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B};
        static const CUtensorMapL2promotion l2[] = {
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B};
        if (sp.swizzle < 0 || sp.swizzle > 4 || sp.l2_promo < 0 || sp.l2_promo > 3)
            return fail("tmap %d: bad swizzle / l2 promotion", t);
        cuuint64_t gdim[5], gstr[4];
        cuuint32_t box[5], es[5];
        for (uint32_t i = 0; i < sp.rank; ++i) {
            gdim[i] = sp.dims[i];
            box[i] = sp.box[i];
            es[i] = sp.elem_strides[i] ? sp.elem_strides[i] : 1;
        }
        for (uint32_t i = 0; i + 1 < sp.rank; ++i) gstr[i] = sp.strides[i];
        void* base = (void*)(uintptr_t)(ptrs[sp.buf_index] + sp.byte_offset);
        DRV_CHECK(TensorMapEncodeTiled(&maps[t], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, sp.rank, base, gdim,
                                         gstr, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw[sp.swizzle],
                                         l2[sp.l2_promo], CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
    }
    std::vector<void*> params;
    for (int i = 0; i < nbuf; ++i) params.push_back(&ptrs[i]);
    params.push_back(&dimblk);
    for (int t = 0; t < ntmaps; ++t) params.push_back(&maps[t]);

    cudaEvent_t e0 = nullptr, e1 = nullptr;
    RT_CHECK(cudaSetDevice(dev));
    if (time_ms) {
        RT_CHECK(cudaEventCreate(&e0));
        RT_CHECK(cudaEventCreate(&e1));
        RT_CHECK(cudaEventRecord(e0, s));
    }
    if (cluster_x > 1) {
        CUlaunchConfig cfg;
        memset(&cfg, 0, sizeof cfg);
        cfg.gridDimX = grid[0]; cfg.gridDimY = grid[1]; cfg.gridDimZ = grid[2];
        cfg.blockDimX = block[0]; cfg.blockDimY = block[1]; cfg.blockDimZ = block[2];
        cfg.sharedMemBytes = dyn_smem;
        cfg.hStream = (CUstream)s;
        CUlaunchAttribute attr;
        memset(&attr, 0, sizeof attr);
        attr.id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
        attr.value.clusterDim.x = cluster_x;
        attr.value.clusterDim.y = 1;
        attr.value.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        DRV_CHECK(LaunchKernelEx(&cfg, f, params.data(), nullptr));
    } else {
        DRV_CHECK(LaunchKernel(f, grid[0], grid[1], grid[2], block[0], block[1], block[2], dyn_smem,
                                 (CUstream)s, params.data(), nullptr));
    }
    if (time_ms) {
        RT_CHECK(cudaEventRecord(e1, s));
        RT_CHECK(cudaEventSynchronize(e1));
        RT_CHECK(cudaEventElapsedTime(time_ms, e0, e1));
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    return 0;
}

int mt_reduce_rows(int dev, uint64_t in_buf, uint64_t out_buf, uint64_t rows, uint64_t cols, uint64_t ld, int op,
                   float* time_ms) {
    if (rows == 0 || cols == 0) return fail("mt_reduce_rows: empty matrix (%llu x %llu)",
                                           (unsigned long long)rows, (unsigned long long)cols);
    if (rows > 65535) return fail("mt_reduce_rows: %llu rows exceed 65535", (unsigned long long)rows);
    Buffer bi, bo;
    cudaStream_t st;
    cudaMemPool_t pool;
    int sms = 148;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (ensure_dev(dev)) return 1;
        if (get_buf(in_buf, &bi) || get_buf(out_buf, &bo)) return 1;
        st = g_dev[dev].stream;
        pool = g_dev[dev].pool;
        RT_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    }
    if (bi.dev != dev || bo.dev != dev) return fail("mt_reduce_rows: buffers are not on device %d", dev);
    if (((rows - 1) * ld + cols) * sizeof(float) > bi.size) return fail("mt_reduce_rows: input buffer too small");
    if (op < 0 || op > 7) return fail("mt_reduce_rows: op %d is not 0..7", op);
    if (rows * (op >= 4 ? sizeof(double) : sizeof(float)) > bo.size)
        return fail("mt_reduce_rows: output buffer too small");
    unsigned long long splits, chunk;
    reduce_plan(rows, cols, sms, &splits, &chunk);
    void* scratch = nullptr;
    const size_t pbytes = rows * splits * sizeof(double), tbytes = rows * sizeof(unsigned);
    RT_CHECK(cudaSetDevice(dev));
    RT_CHECK(cudaMallocAsync(&scratch, pbytes + tbytes, pool, st));
    double* partials = (double*)scratch;
    unsigned* tickets = (unsigned*)((char*)scratch + pbytes);
    RT_CHECK(cudaMemsetAsync(tickets, 0, tbytes, st));
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (time_ms) {
        RT_CHECK(cudaEventCreate(&e0));
        RT_CHECK(cudaEventCreate(&e1));
        RT_CHECK(cudaEventRecord(e0, st));
    }
    int rc = launch_reduce(op, st, splits, rows, (const float*)bi.ptr, bo.ptr, partials, tickets, cols, ld,
                           chunk);
    if (time_ms) {
        RT_CHECK(cudaEventRecord(e1, st));
        RT_CHECK(cudaEventSynchronize(e1));
        RT_CHECK(cudaEventElapsedTime(time_ms, e0, e1));
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    RT_CHECK(cudaFreeAsync(scratch, st));
    return rc;
}

// Allocation-free reduction for callers that cannot allocate device memory: code
// that runs inside another framework's device-memory budget (a serving process whose
// caching allocator has reserved the GPU, where an extra cudaMalloc can fail or
// fragment that pool) and latency-critical loops where an allocation may synchronise
// the device. Same kernel and plan as mt_reduce_rows; the scratch is the static
// array above. `in` / `out` are device pointers the caller owns (in: (rows - 1) * ld
// + cols floats, out: rows floats).
int mt_reduce_rows_noalloc(int dev, const float* in, float* out, uint64_t rows, uint64_t cols, uint64_t ld,
                           int op, void* stream) {
    if (!in || !out) return fail("mt_reduce_rows_noalloc: null input or output pointer");
    if (op < 0 || op > 3) return fail("mt_reduce_rows_noalloc: op %d is not 0..3 (fp32 output)", op);
    if (rows == 0 || cols == 0)
        return fail("mt_reduce_rows_noalloc: empty matrix (%llu x %llu)", (unsigned long long)rows,
                    (unsigned long long)cols);
    if (rows > 65535) return fail("mt_reduce_rows_noalloc: %llu rows exceed 65535", (unsigned long long)rows);
    if (dev < 0 || dev >= kMaxDev) return fail("mt_reduce_rows_noalloc: device index %d out of range", dev);
    cudaStream_t st = (cudaStream_t)stream;
    if (!st) {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_dev[dev].ready)
            return fail("mt_reduce_rows_noalloc: no stream given and device %d not initialised "
                        "(pass a stream or call mt_init first)", dev);
        st = g_dev[dev].stream;
    } else {
        int sdev = -1;
        RT_CHECK(cudaStreamGetDevice(st, &sdev));
        if (sdev != dev)
            return fail("mt_reduce_rows_noalloc: the stream belongs to device %d, not device %d", sdev, dev);
    }
    // The caller (often another framework) keeps its own current device: switch to
    // `dev` for the set-up and the launch and switch back on every return path.
    int caller_dev = -1;
    RT_CHECK(cudaGetDevice(&caller_dev));
    struct RestoreDevice {
        int d;
        ~RestoreDevice() { if (d >= 0) cudaSetDevice(d); }
    } restore{caller_dev};
    RT_CHECK(cudaSetDevice(dev));
    int sms = 148;
    RT_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    unsigned long long splits, chunk;
    reduce_plan(rows, cols, sms, &splits, &chunk);
    const size_t pbytes = rows * splits * sizeof(double);
    const size_t need = pbytes + rows * sizeof(unsigned);
    if (need > kNoAllocScratchBytes)
        return fail("mt_reduce_rows_noalloc: this reduction needs %zu bytes of scratch (rows * splits * 8 + "
                    "rows * 4 with %llu splits per row); the allocation-free entry point has %zu bytes per device "
                    "- use mt_reduce_rows", need, splits, kNoAllocScratchBytes);
    void* base = nullptr;
    {
        // Set-up, once per device, with that device current: the host-side name of
        // the __device__ array is not a device address, so look the address up.
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_scratch_ptr[dev]) {
            void* p = nullptr;
            RT_CHECK(cudaGetSymbolAddress(&p, mt_noalloc_scratch));
            g_noalloc_scratch_ptr[dev] = p;
        }
        base = g_noalloc_scratch_ptr[dev];
    }
    double* partials = (double*)base;
    unsigned* tickets = (unsigned*)((char*)base + pbytes);
    // The array keeps the previous call's contents: the tickets must start at zero.
    RT_CHECK(cudaMemsetAsync(tickets, 0, rows * sizeof(unsigned), st));
    return launch_reduce(op, st, splits, rows, in, out, partials, tickets, cols, ld, chunk);
}

// ---- NCCL: combining whole-tensor reductions across GPUs ------------------------
//
// libnccl is opened at first use (dlopen by soname), so the library still loads where
// NCCL is absent and shares the copy a host framework (torch.distributed) has loaded.

}  // extern "C"

namespace {

struct NcclApi {
    bool ok = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};
NcclApi g_nccl;
std::mutex g_nccl_mu;

int nccl_api() {
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.ok) return 0;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return fail("NCCL: cannot open libnccl.so.2 (%s)", dlerror());
#define MT_NCCL(name) \
    g_nccl.name = reinterpret_cast<decltype(g_nccl.name)>(dlsym(h, "nccl" #name)); \
    if (!g_nccl.name) return fail("NCCL: symbol nccl" #name " missing");
    MT_NCCL(GetUniqueId)
    MT_NCCL(CommInitRank)
    MT_NCCL(AllReduce)
    MT_NCCL(CommDestroy)
    MT_NCCL(GetErrorString)
#undef MT_NCCL
    g_nccl.ok = true;
    return 0;
}

#define NCCL_CHECK(x)                                                                    \
    do {                                                                                \
        ncclResult_t r_ = (x);                                                          \
        if (r_ != ncclSuccess) return fail("%s: %s", #x, g_nccl.GetErrorString(r_));    \
    } while (0)

__global__ void f64_to_f32(const double* in, float* out, unsigned long long n) {
    const unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x;
    if (i < n) out[i] = (float)in[i];
}

}  // namespace

extern "C" {

int mt_nccl_unique_id(unsigned char* out, uint64_t cap) {
    if (!out || cap < sizeof(ncclUniqueId)) return fail("mt_nccl_unique_id: buffer below %zu bytes", sizeof(ncclUniqueId));
    if (nccl_api()) return 1;
    ncclUniqueId id;
    NCCL_CHECK(g_nccl.GetUniqueId(&id));
    memcpy(out, &id, sizeof(id));
    return 0;
}

int mt_nccl_init(int dev, int nranks, int rank, const unsigned char* id) {
    if (!id || nranks < 1 || rank < 0 || rank >= nranks)
        return fail("mt_nccl_init: rank %d of %d or id invalid", rank, nranks);
    if (nccl_api()) return 1;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (ensure_dev(dev)) return 1;
        if (g_dev[dev].comm) return fail("mt_nccl_init: device %d already has a communicator", dev);
    }
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclComm_t c = nullptr;
    RT_CHECK(cudaSetDevice(dev));
    NCCL_CHECK(g_nccl.CommInitRank(&c, nranks, uid, rank));
    std::lock_guard<std::mutex> lk(g_mu);
    g_dev[dev].comm = c;
    return 0;
}

int mt_nccl_destroy(int dev) {
    ncclComm_t c = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (dev < 0 || dev >= kMaxDev) return fail("device index %d out of range", dev);
        c = g_dev[dev].comm;
        g_dev[dev].comm = nullptr;
    }
    if (c) NCCL_CHECK(g_nccl.CommDestroy(c));
    return 0;
}

int mt_allreduce_f64(int dev, uint64_t buf, uint64_t count, int op, uint64_t out_f32) {
    static const ncclRedOp_t kOps[4] = {ncclSum, ncclMax, ncclMin, ncclProd};
    if (op < 0 || op > 3) return fail("mt_allreduce_f64: op %d is not 0..3", op);
    Buffer b, o{};
    cudaStream_t st;
    ncclComm_t c;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (ensure_dev(dev)) return 1;
        if (get_buf(buf, &b)) return 1;
        if (out_f32 && get_buf(out_f32, &o)) return 1;
        st = g_dev[dev].stream;
        c = g_dev[dev].comm;
    }
    if (!c) return fail("mt_allreduce_f64: device %d has no communicator (mt_nccl_init)", dev);
    if (b.dev != dev || count * sizeof(double) > b.size) return fail("mt_allreduce_f64: buffer too small or on another device");
    if (out_f32 && (o.dev != dev || count * sizeof(float) > o.size))
        return fail("mt_allreduce_f64: output buffer too small or on another device");
    RT_CHECK(cudaSetDevice(dev));
    NCCL_CHECK(g_nccl.AllReduce(b.ptr, b.ptr, count, ncclFloat64, kOps[op], c, st));
    if (out_f32) {
        const unsigned threads = 256;
        const unsigned blocks = (unsigned)((count + threads - 1) / threads);
        f64_to_f32<<<blocks, threads, 0, st>>>((const double*)b.ptr, (float*)o.ptr, count);
        RT_CHECK(cudaGetLastError());
    }
    return 0;
}

int mt_stream_wait_event(int dev, uint64_t ev) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (ensure_dev(dev)) return 1;
    auto it = g_events.find(ev);
    if (it == g_events.end()) return fail("mt_stream_wait_event: unknown event %llu", (unsigned long long)ev);
    RT_CHECK(cudaStreamWaitEvent(g_dev[dev].stream, it->second, 0));
    return 0;
}

int mt_sync(int dev) {
    cudaStream_t s, s2;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (ensure_dev(dev)) return 1;
        s = g_dev[dev].stream;
        s2 = g_dev[dev].d2h;
    }
    RT_CHECK(cudaStreamSynchronize(s2));
    RT_CHECK(cudaStreamSynchronize(s));
    RT_CHECK(cudaGetLastError());
    return 0;
}

int mt_event_create(uint64_t* ev) {
    cudaEvent_t e;
    RT_CHECK(cudaEventCreate(&e));
    std::lock_guard<std::mutex> lk(g_mu);
    uint64_t h = g_next++;
    g_events[h] = e;
    *ev = h;
    return 0;
}

int mt_event_record(int dev, uint64_t ev) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (ensure_dev(dev)) return 1;
    auto it = g_events.find(ev);
    if (it == g_events.end()) return fail("unknown event");
    RT_CHECK(cudaEventRecord(it->second, g_dev[dev].stream));
    return 0;
}

int mt_event_elapsed(uint64_t start, uint64_t end, float* ms) {
    cudaEvent_t a, b;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto i = g_events.find(start), j = g_events.find(end);
        if (i == g_events.end() || j == g_events.end()) return fail("unknown event");
        a = i->second;
        b = j->second;
    }
    RT_CHECK(cudaEventSynchronize(b));
    RT_CHECK(cudaEventElapsedTime(ms, a, b));
    return 0;
}

int mt_event_destroy(uint64_t ev) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_events.find(ev);
    if (it == g_events.end()) return fail("unknown event");
    cudaEventDestroy(it->second);
    g_events.erase(it);
    return 0;
}

int mt_graph_begin(int dev) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (ensure_dev(dev)) return 1;
    RT_CHECK(cudaStreamBeginCapture(g_dev[dev].stream, cudaStreamCaptureModeThreadLocal));
    return 0;
}

int mt_graph_end(int dev, uint64_t* graph) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (ensure_dev(dev)) return 1;
    cudaGraph_t g;
    RT_CHECK(cudaStreamEndCapture(g_dev[dev].stream, &g));
    cudaGraphExec_t ex;
    RT_CHECK(cudaGraphInstantiate(&ex, g, 0));
    cudaGraphDestroy(g);
    uint64_t h = g_next++;
    g_graphs[h] = ex;
    *graph = h;
    return 0;
}

int mt_graph_launch(int dev, uint64_t graph) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (ensure_dev(dev)) return 1;
    auto it = g_graphs.find(graph);
    if (it == g_graphs.end()) return fail("unknown graph");
    RT_CHECK(cudaGraphLaunch(it->second, g_dev[dev].stream));
    return 0;
}

int mt_graph_destroy(uint64_t graph) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_graphs.find(graph);
    if (it == g_graphs.end()) return fail("unknown graph");
    cudaGraphExecDestroy(it->second);
    g_graphs.erase(it);
    return 0;
}

}  // extern "C"
