/*
 * metellus_b200.h — C ABI of the Metellus B200 backend (libmetellus_cuda.so).
 *
 * This library replaces the reference's Objective-C++ nanobind module
 * `metal_backend` (src/metal_backend.mm:253-261). Every entry point returns an int
 * status: 0 = success, nonzero = failure, with the message available from
 * mt_last_error(). The Python layer raises RuntimeError on nonzero, matching the
 * reference's std::runtime_error -> RuntimeError behaviour (metal_backend.mm:78,
 * 192-207, 230-232).
 *
 * Threading: one CUDA stream per device; the buffer registry and kernel table are
 * mutex-guarded. Device work is stream ordered; reads synchronise the stream.
 */
#ifndef METELLUS_B200_H
#define METELLUS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- errors / devices --------------------------------------------------- */

/* Copy the calling thread's last error message into buf (NUL terminated). */
int mt_last_error(char* buf, size_t n);
/* Number of visible CUDA devices. */
int mt_device_count(int* n);
/* Initialise device `dev` (primary context, stream, memory pool). Idempotent.
 * The reference creates its device and queue statically (metal_backend.mm:21-35). */
int mt_init(int dev);
/* Query a device attribute: 0 = SM count, 1 = max opt-in shared memory per block,
 * 2 = compute capability major*10+minor, 3 = L2 bytes. */
int mt_device_attr(int dev, int which, int64_t* out);

/* ---- buffers (replace create_buffer / release_buffer / buffer_size /
 *      write_buffer / read_buffer / fill_buffer, metal_backend.mm:94-141) ---- */

/* Allocate nbytes of device memory on `dev` from a stream-ordered pool. */
int mt_buffer_create(int dev, size_t nbytes, uint64_t* handle);
/* Release a buffer (stream ordered: pending kernels that use it finish first). */
int mt_buffer_release(uint64_t handle);
int mt_buffer_size(uint64_t handle, size_t* nbytes);
/* Device address of the buffer (for interop and for the C-level tests). */
int mt_buffer_ptr(uint64_t handle, uint64_t* dptr);
/* Host -> device copy of nbytes from src (pinned or pageable); waits for completion. */
int mt_buffer_write(uint64_t handle, const void* src, size_t nbytes);
/* Device -> host copy into dst; waits for all earlier work on the stream. */
int mt_buffer_read(uint64_t handle, void* dst, size_t nbytes);
/* Asynchronous variants (stream ordered); src/dst must be pinned for true overlap. */
int mt_buffer_write_async(uint64_t handle, const void* src, size_t nbytes);
int mt_buffer_read_async(uint64_t handle, void* dst, size_t nbytes);
/* Set every byte to `value`. */
int mt_buffer_fill(uint64_t handle, uint8_t value);
/* Stream-ordered form of mt_buffer_fill: returns without waiting for the device. */
int mt_buffer_fill_async(uint64_t handle, uint8_t value);
/* Device-to-host copy on the device's copy stream (not the main stream): waits for
 * event `after` (recorded on the main stream, e.g. after the kernels that produce the
 * data; 0 = no wait), then records event `done` (0 = none) when the copy finishes.
 * A step's download then overlaps the next step's uploads (PCIe is full duplex; the
 * main stream carries uploads and kernels). No counterpart in the reference (its
 * read_buffer is synchronous). */
int mt_buffer_read_after(uint64_t handle, void* dst, size_t nbytes, uint64_t after, uint64_t done);
/* The device's main stream waits for event `ev` before its next operation. */
int mt_stream_wait_event(int dev, uint64_t ev);
/* Pinned host memory for fast host<->device copies. */
int mt_host_alloc(size_t nbytes, void** ptr);
int mt_host_free(void* ptr);

/* ---- kernels (replace run_kernel's per-call compile, metal_backend.mm:178-249) */

/* NVRTC: compile CUDA C++ `src` for `arch` (e.g. "sm_100a") with extra options
 * (space separated) into a cubin. On success *size is the cubin size; if cap is
 * too small nothing is copied and the call still succeeds (query then retry).
 * The compile log goes to `log` (may be NULL). */
int mt_nvrtc_compile(const char* src, const char* name, const char* opts,
                     void* cubin, size_t cap, size_t* size, char* log, size_t logcap);
/* Load a cubin and look up `fn`; returns a kernel handle usable on any device. */
int mt_kernel_load(const void* cubin, size_t size, const char* fn, uint64_t* kernel);
/* Register count and local (spill) bytes per thread of a loaded kernel. */
int mt_kernel_info(int dev, uint64_t kernel, int* regs, int* local_bytes, int* max_threads);

/* TMA tensor-map description, encoded by the backend at launch time. */
typedef struct mt_tmap_spec {
    int32_t buf_index;     /* index into the launch's buffer list */
    uint32_t rank;         /* 1..5 */
    uint64_t dims[5];      /* elements, innermost first */
    uint64_t strides[4];   /* bytes, for dims 1..rank-1 */
    uint32_t box[5];       /* elements per copy, innermost first */
    uint32_t elem_strides[5];
    int32_t swizzle;       /* 0 none, 1 32B, 2 64B, 3 128B, 4 128B with 32-byte atoms */
    int32_t l2_promo;      /* 0 none, 1 64B, 2 128B, 3 256B */
    uint64_t byte_offset;  /* added to the buffer base address */
} mt_tmap_spec;

/* Launch `kernel` on device `dev`'s stream. Parameters are the buffers' device
 * addresses in order, then a 64-byte block holding `ndims` uint32 dims, then one
 * CUtensorMap per tmap spec. If time_ms is non-NULL the launch is bracketed by
 * events, waited for, and its device time is returned (profile mode). cluster_x
 * > 1 launches thread-block clusters of that size along x. */
int mt_launch(int dev, uint64_t kernel, const uint64_t* buffers, int nbuf,
              const uint32_t* dims, int ndims, const uint32_t grid[3],
              const uint32_t block[3], uint32_t dyn_smem, uint32_t cluster_x,
              const mt_tmap_spec* tmaps, int ntmaps, float* time_ms);
/* Wait for all work on the device's streams (main and copy). */
int mt_sync(int dev);

/* ---- native kernels ------------------------------------------------------- */

/* Last-axis reduction of a rows x cols fp32 matrix stored with row stride `ld`
 * elements (column stride 1): out[r] = op over c of in[r * ld + c], op 0 = sum,
 * 1 = max, 2 = min, 3 = product. Sum and product accumulate in fp64 and round once
 * to fp32. Ops 4..7 are the same four with an fp64 `out` (rows doubles): the
 * per-GPU partial of a sharded whole-tensor reduction, combined by mt_allreduce_f64. Long rows are split across blocks; each block writes an fp64 partial to
 * scratch and the last block of a row (atomic ticket) combines the partials in a
 * fixed order, so results are deterministic. The scratch (partials + tickets) comes
 * from the device's stream-ordered pool and is returned to it after the launch.
 * Replaces the reference's reduction kernel for few, long rows (a whole-tensor
 * sum viewed as (1, M*K) runs on ONE threadgroup there:
 * src/compute/reduction/reduction.py:24-111, src/orchestrator/assembly/
 * reduction.py:105-106). `time_ms` as in mt_launch. */
int mt_reduce_rows(int dev, uint64_t in_buf, uint64_t out_buf, uint64_t rows, uint64_t cols, uint64_t ld,
                   int op, float* time_ms);

/* Allocation-free variant of mt_reduce_rows (no counterpart in the reference).
 * For callers that cannot allocate device memory: code running inside another
 * framework's device-memory budget (e.g. a serving process whose caching allocator
 * owns the GPU) or a latency-critical loop that must not allocate. It calls no
 * cudaMalloc / cudaFree: its scratch is a fixed 256 KiB array in this library's device
 * image (kept on every GPU that loads the library until exit). `in` and `out` are
 * device pointers owned by the caller; `stream` is a cudaStream_t (NULL = this
 * library's stream for `dev`, which then must have been initialised by mt_init).
 * Rejects, with an error message, reductions whose partials do not fit
 * (rows * splits * 8 + rows * 4 > 256 KiB, splits ~ 8 blocks per SM / rows: a few-row
 * reduction needs ~10 KB; one-split plans fit up to 21,845 rows).
 * The first call on a device looks up the array's device address (module set-up):
 * make it before any stream capture. That address is kept for the life of the
 * process, so do not call cudaDeviceReset between calls. All calls share the array,
 * so calls that overlap on the GPU (different streams) race; the tickets are cleared
 * per call. A caller's stream must belong to `dev`; the caller's current device is
 * restored before returning. */
int mt_reduce_rows_noalloc(int dev, const float* in, float* out, uint64_t rows, uint64_t cols, uint64_t ld,
                           int op, void* stream);

/* ---- multi-GPU: combining sharded whole-tensor reductions -------------------
 * No counterpart in the reference (its Metal backend drives one GPU); a sharded
 * whole-tensor reduction (sum(X) with X's rows split across GPUs) computes one fp64
 * partial per GPU (mt_reduce_rows op 4..7) and combines the partials with one NCCL
 * all-reduce over NVLink. One process per GPU; libnccl.so.2 is opened at first use. */

/* NCCL unique id (ncclGetUniqueId) into `out` (cap >= 128 bytes); rank 0 makes it
 * and the host plumbing (torch.distributed) broadcasts it to the other ranks. */
int mt_nccl_unique_id(unsigned char* out, uint64_t cap);
/* Create the device's communicator (ncclCommInitRank): rank `rank` of `nranks`. */
int mt_nccl_init(int dev, int nranks, int rank, const unsigned char* id);
int mt_nccl_destroy(int dev);
/* In-place all-reduce of `count` doubles in `buf` on the device's stream, op 0 = sum,
 * 1 = max, 2 = min, 3 = product; if `out_f32` is nonzero the result is also written
 * there rounded to fp32 (the program's output tensor). Stream ordered, no host wait. */
int mt_allreduce_f64(int dev, uint64_t buf, uint64_t count, int op, uint64_t out_f32);

/* ---- timing and graphs --------------------------------------------------- */

int mt_event_create(uint64_t* ev);
int mt_event_record(int dev, uint64_t ev);
int mt_event_elapsed(uint64_t start, uint64_t end, float* ms);
int mt_event_destroy(uint64_t ev);
/* Capture subsequent launches on the device's stream into a CUDA graph. */
int mt_graph_begin(int dev);
int mt_graph_end(int dev, uint64_t* graph);
int mt_graph_launch(int dev, uint64_t graph);
int mt_graph_destroy(uint64_t graph);

#ifdef __cplusplus
}
#endif
#endif /* METELLUS_B200_H */
