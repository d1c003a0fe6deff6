/*
 * porch_b200 runtime C-ABI: the thin layer between porch's C++ front-end and
 * the CUDA driver API, NVRTC and NCCL. Every symbol is resolved at run time
 * with dlopen/dlsym, so a program that links this library needs no CUDA
 * toolkit at build time and no nvcc.
 *
 * Conventions
 *  - Every entry point returns an int status (PBRT_OK == 0). On failure the
 *    calling thread's message is available from pbrt_last_error() until the
 *    next failing call on that thread.
 *  - Device pointers are plain uint64_t addresses, streams/events/functions are
 *    opaque handles (CUstream, CUevent, CUfunction underneath).
 *  - Each (thread, device) pair owns one non-blocking "current" stream, the
 *    multi-device counterpart of the reference's thread-local stream.
 *
 * Reference interfaces replaced (paths within AkhilSamavedam/porch):
 *  - src/cuda_jit.cpp:30-356   dynamic driver/NVRTC loader and error formatting
 *  - src/cuda_jit.cpp:437-528  cuda_environment (device 0 only) and thread-local
 *                              stream_handle; here: primary context per device,
 *                              stream per (thread, device)
 *  - src/cuda_jit.cpp:532-627  device_buffer_state cuMemAllocAsync/cuMemFreeAsync;
 *                              here: both kept, plus cuMemAlloc for the
 *                              library's caching allocator (pbrt_mem_alloc)
 *  - src/cuda_jit.cpp:647-703  compile_to_ptx + ptx_cache (source-text keyed);
 *                              here: NVRTC -> sm_100a cubin keyed by a 64-bit hash
 *  - src/cuda_jit.cpp:705-761  copy_to_device / copy_to_host / synchronize
 *  - src/cuda_jit.cpp:763-948  launch_* (cuModuleLoadData on every launch);
 *                              here: module loaded once per (device, key)
 *  The reference has no NCCL, tensor-map, profiling or fault-injection layer;
 *  those entry points are new and have no counterpart there.
 */
#ifndef PORCH_B200_RT_H
#define PORCH_B200_RT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum pbrt_status {
    PBRT_OK = 0,
    PBRT_ERR_INVALID = 1,     /* bad argument: maps to std::invalid_argument  */
    PBRT_ERR_RANGE = 2,       /* index out of range: std::out_of_range        */
    PBRT_ERR_DRIVER = 3,      /* "<api> failed: NAME: description"            */
    PBRT_ERR_COMPILE = 4,     /* NVRTC compile failed; message is the log     */
    PBRT_ERR_UNAVAILABLE = 5, /* libcuda / libnvrtc / libnccl or device absent */
    PBRT_ERR_INJECTED = 6,    /* host-side fault injection fired              */
    PBRT_ERR_DEVICE = 7,      /* a kernel raised the per-device error word    */
    PBRT_ERR_NCCL = 8,        /* NCCL call failed, timed out or was aborted   */
};

typedef struct pbrt_stream_s* pbrt_stream;
typedef struct pbrt_event_s* pbrt_event;
typedef struct pbrt_function_s* pbrt_function;
typedef struct pbrt_comm_s* pbrt_comm;

/* ---- errors, availability, devices ------------------------------------ */
const char* pbrt_last_error(void);
/* 1 when libcuda and libnvrtc load, cuInit succeeds and a device exists.
 * Never fails (the reference's is_available() is noexcept,
 * src/cuda_jit.cpp:634-645). */
int pbrt_available(void);
int pbrt_init(void);
int pbrt_device_count(int* count);
int pbrt_device_attribute(int device, int attribute, int* value);
int pbrt_device_name(int device, char* buffer, size_t length);
int pbrt_driver_version(int* version);
int pbrt_nvrtc_version(int* major, int* minor);

/* ---- streams and events ------------------------------------------------ */
int pbrt_stream_current(int device, pbrt_stream* stream);
int pbrt_stream_create(int device, pbrt_stream* stream);
int pbrt_stream_destroy(int device, pbrt_stream stream);
int pbrt_stream_synchronize(int device, pbrt_stream stream);
int pbrt_event_create(int device, int enable_timing, pbrt_event* event);
int pbrt_event_destroy(int device, pbrt_event event);
int pbrt_event_record(int device, pbrt_event event, pbrt_stream stream);
int pbrt_event_synchronize(int device, pbrt_event event);
/* *done = 1 when every operation before the event has completed, else 0. */
int pbrt_event_query(int device, pbrt_event event, int* done);
int pbrt_event_elapsed_ms(pbrt_event start, pbrt_event end, float* ms);
int pbrt_stream_wait_event(int device, pbrt_stream stream, pbrt_event event);

/* ---- memory ------------------------------------------------------------ */
/* Stream-ordered allocation from the device's default pool. The pool keeps
 * freed memory cached (release threshold = max) so steady-state graphs never
 * return to the OS allocator. */
int pbrt_mem_alloc_async(int device, size_t bytes, pbrt_stream stream,
                         uint64_t* pointer);
int pbrt_mem_free_async(int device, uint64_t pointer, pbrt_stream stream);
/* Plain allocation (cuMemAlloc), usable on any stream at once. Growing the
 * stream-ordered pool can block the calling thread until the stream's queued
 * work drains (measured: up to 116 ms for 64 MB behind a busy GEMM queue),
 * so the library's caching allocator takes its blocks from here. The free
 * waits for all work on the device (cuMemFree), so it is used only when the
 * cache is trimmed. */
int pbrt_mem_alloc(int device, size_t bytes, uint64_t* pointer);
int pbrt_mem_free(int device, uint64_t pointer);
int pbrt_host_alloc(size_t bytes, void** pointer); /* page-locked */
int pbrt_host_free(void* pointer);
int pbrt_memcpy_h2d_async(int device, uint64_t dst, const void* src,
                          size_t bytes, pbrt_stream stream);
int pbrt_memcpy_d2h_async(int device, void* dst, uint64_t src, size_t bytes,
                          pbrt_stream stream);
int pbrt_memcpy_d2d_async(int device, uint64_t dst, uint64_t src,
                          size_t bytes, pbrt_stream stream);
int pbrt_memcpy_peer_async(int dst_device, uint64_t dst, int src_device,
                           uint64_t src, size_t bytes, pbrt_stream stream);
int pbrt_memset_d32_async(int device, uint64_t dst, uint32_t value,
                          size_t count, pbrt_stream stream);
int pbrt_enable_peer_access(int device, int peer);

/* ---- NVRTC + modules + launches -------------------------------------- */
/* Compile `source` with NVRTC. want_cubin=1 asks for a cubin (the options
 * must then name a real architecture, e.g. --gpu-architecture=sm_100a),
 * 0 for PTX. The result is cached by a 64-bit hash of source and options;
 * *key receives that hash. A compile failure returns PBRT_ERR_COMPILE with the
 * NVRTC log as the message. */
int pbrt_compile(const char* source, const char* const* options,
                 int option_count, int want_cubin, uint64_t* key);
/* Image bytes (cubin or NUL-terminated PTX) of a compiled key. The pointer
 * stays valid for the life of the process. */
int pbrt_compiled_image(uint64_t key, const void** image, size_t* size);
/* Loads an image given directly (e.g. user PTX) and returns its key. */
int pbrt_register_image(const void* image, size_t size, uint64_t* key);
/* Function lookup; the module is loaded once per (device, key). */
int pbrt_get_function(int device, uint64_t key, const char* name,
                  pbrt_function* function);
int pbrt_function_set_max_dynamic_smem(pbrt_function function, int bytes);
/* CTAs of `function` that fit on one SM of `device` at this block size and
 * dynamic shared memory (registers, shared memory and thread limits). */
int pbrt_occupancy(int device, pbrt_function function, int block_threads, size_t dynamic_smem,
                   int* blocks_per_sm);
/* Clusters of `cluster_x` CTAs of `function` that can be resident on
 * `device` at once (cuOccupancyMaxActiveClusters). */
int pbrt_max_active_clusters(int device, pbrt_function function, int block_threads, size_t dynamic_smem,
                             unsigned cluster_x, int* clusters);
int pbrt_function_attribute(pbrt_function function, int attribute,
                            int* value);
/* grid/block are 3-vectors; cluster may be NULL (no cluster attribute). */
int pbrt_launch(int device, pbrt_function function, const uint32_t* grid,
                const uint32_t* block, uint32_t dynamic_smem,
                pbrt_stream stream, void** params, const uint32_t* cluster);
/* pbrt_launch with flags. PBRT_LAUNCH_PDL: programmatic stream serialization
 * -- the launch may begin while the stream's previous kernel finishes, so
 * the kernel must execute `griddepcontrol.wait` before it touches memory
 * that earlier work in the stream reads or writes (the generated kernels do
 * so first thing). */
#define PBRT_LAUNCH_PDL 1u
int pbrt_launch_ex(int device, pbrt_function function, const uint32_t* grid,
                   const uint32_t* block, uint32_t dynamic_smem,
                   pbrt_stream stream, void** params, const uint32_t* cluster,
                   unsigned flags);
/* cuTensorMapEncodeTiled with plain integers; out must hold 128 bytes. */
int pbrt_tensor_map_encode_tiled(void* out, int data_type, uint32_t rank,
                                 uint64_t global_address,
                                 const uint64_t* global_dims,
                                 const uint64_t* global_strides_bytes,
                                 const uint32_t* box_dims,
                                 const uint32_t* element_strides,
                                 int interleave, int swizzle,
                                 int l2_promotion, int oob_fill);

/* ---- device error word ------------------------------------------------- */
/* Each device owns one zero-initialised 64-byte error block. Kernels whose
 * waits are bounded write a non-zero code there instead of spinning forever;
 * pbrt_error_check synchronises `stream`, reads and clears it. */
int pbrt_error_word(int device, uint64_t* pointer);
int pbrt_error_check(int device, pbrt_stream stream, int* code);

/* ---- profiling -------------------------------------------------------- */
/* When enabled, every pbrt_launch is bracketed by a pair of timing events on
 * its stream. pbrt_profile_read synchronises the recorded events and writes
 * "name<TAB>launches<TAB>total_ms\n" lines (then clears the record). */
int pbrt_profile_enable(int enable);
int pbrt_profile_read(char* buffer, size_t length);
uint64_t pbrt_launch_count(void);
/* NVRTC compilations run by this process, and images loaded instead from
 * the on-disk cache ($PORCH_B200_CACHE_DIR), since start. */
void pbrt_compile_stats(uint64_t* nvrtc_compiles, uint64_t* disk_cache_hits);

/* ---- fault injection (host side only) --------------------------------- */
/* spec: comma-separated "<site>:<n>" entries; the n-th subsequent call at that
 * site fails with PBRT_ERR_INJECTED. Sites: compile, alloc, launch, h2d, d2h,
 * nccl_init, nccl_coll. An empty spec clears all. PORCH_FAULT in the
 * environment is read once at first use. */
int pbrt_fault_inject(const char* spec);

/* ---- NCCL (dlopen'ed libnccl.so.2) ------------------------------------- */
int pbrt_nccl_available(void);
int pbrt_nccl_unique_id(char id[128]);
/* One process driving `count` devices (ncclCommInitAll). */
int pbrt_nccl_init_all(int count, const int* devices, pbrt_comm* comms);
/* One rank of a multi-process communicator, created non-blocking and
 * completed with a deadline (seconds). */
int pbrt_nccl_init_rank(int nranks, const char id[128], int rank, int device,
                        double timeout_s, pbrt_comm* comm);
int pbrt_nccl_group_start(void);
/* Ends a group. On non-blocking communicators the group's operations may
 * still be enqueueing when this returns: call pbrt_nccl_settle on every
 * communicator of the group before ordering other work behind them. */
int pbrt_nccl_group_end(void);
/* Waits (bounded by the communicator's timeout, aborting it on expiry or on
 * an asynchronous error) until the communicator's pending host-side enqueue
 * has finished. Collectives issued outside a group settle by themselves. */
int pbrt_nccl_settle(pbrt_comm comm);
int pbrt_nccl_allgather_f32(pbrt_comm comm, uint64_t send, uint64_t recv,
                            size_t count_per_rank, pbrt_stream stream);
int pbrt_nccl_send_f32(pbrt_comm comm, uint64_t send, size_t count, int peer,
                       pbrt_stream stream);
int pbrt_nccl_recv_f32(pbrt_comm comm, uint64_t recv, size_t count, int peer,
                       pbrt_stream stream);
/* Waits until `stream` drains or the communicator reports an async error;
 * after timeout_s the communicator is aborted and PBRT_ERR_NCCL returned. */
int pbrt_nccl_wait(pbrt_comm comm, int device, pbrt_stream stream,
                   double timeout_s);
int pbrt_nccl_abort(pbrt_comm comm);
/* Bound (seconds) on the communicator's host-side waits from now on. */
int pbrt_nccl_set_timeout(pbrt_comm comm, double timeout_s);
int pbrt_nccl_destroy(pbrt_comm comm);

#ifdef __cplusplus
}
#endif

#endif /* PORCH_B200_RT_H */
