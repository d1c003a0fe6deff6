/*
 * porch_b200 flat C-ABI over the porch tensor API.
 *
 * The reference is a C++20 library (include/porch/tensor.hpp, ops.hpp,
 * cuda_jit.hpp) and has no FFI of its own; this header is the binding a
 * maintainer would add to reach it from C, Python (ctypes), Go (cgo) or any
 * other FFI. Each entry point forwards to the C++ call named in its comment,
 * with the same argument meaning, and turns that call's exception into a
 * status code:
 *   std::invalid_argument -> PB_ERR_INVALID_ARGUMENT
 *   std::out_of_range     -> PB_ERR_OUT_OF_RANGE
 *   cuda_jit::compilation_error -> PB_ERR_COMPILATION
 *   any other exception   -> PB_ERR_RUNTIME
 * The message of the last failure on the calling thread is pb_last_error().
 *
 * Handles: pb_tensor wraps porch::tensor (a shared handle), pb_expr wraps
 * porch::tensor_expr. Release every handle you receive; releasing does not
 * invalidate other handles that share the same storage.
 */
#ifndef PORCH_B200_H
#define PORCH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum pb_status {
    PB_OK = 0,
    PB_ERR_INVALID_ARGUMENT = 1,
    PB_ERR_OUT_OF_RANGE = 2,
    PB_ERR_RUNTIME = 3,
    PB_ERR_COMPILATION = 4,
};

enum pb_op {
    PB_ADD = 0,        /* operator+   (include/porch/tensor.hpp:221) */
    PB_SUBTRACT = 1,   /* operator-   (tensor.hpp:222)               */
    PB_MULTIPLY = 2,   /* operator*   (tensor.hpp:223)               */
    PB_DIVIDE = 3,     /* operator/   (tensor.hpp:224)               */
    PB_MAXIMUM = 4,    /* maximum     (tensor.hpp:212)               */
    PB_MINIMUM = 5,    /* minimum     (tensor.hpp:213)               */
    PB_MATMUL = 6,     /* matmul      (tensor.hpp:196)               */
    PB_EXP = 7,        /* exp         (tensor.hpp:214)               */
    PB_RECIPROCAL = 8, /* reciprocal  (tensor.hpp:215)               */
    PB_TRANSPOSE = 9,  /* transpose   (tensor.hpp:201)               */
    PB_RELU = 10,      /* relu        (include/porch/ops.hpp:7)      */
    PB_LOGISTIC = 11,  /* logistic    (ops.hpp:9)                    */
    PB_SUM = 12,       /* sum         (tensor.hpp:208)               */
    PB_MAX = 13,       /* max         (tensor.hpp:210)               */
};

enum pb_index_kind { PB_INDEX = 0, PB_SLICE = 1, PB_ALL = 2 };

/* One element of tensor::operator[] (tensor.hpp:43-69: index, slice, all). */
typedef struct pb_index {
    int kind;
    int64_t index;
    int64_t start;
    int64_t stop;
    int64_t step;
} pb_index;

typedef struct pb_tensor_s pb_tensor;
typedef struct pb_expr_s pb_expr;

const char* pb_last_error(void);
/* cuda_jit::is_available (include/porch/cuda_jit.hpp:60) */
int pb_is_available(void);
/* backend_name(backend_for(device)) (include/porch/backend.hpp:35-37) */
const char* pb_backend_name(void);
/* cuda_jit::synchronize (cuda_jit.hpp:73): drain this thread's streams. */
int pb_synchronize(void);

/* ---- tensors ------------------------------------------------------------ */
/* tensor(shape, values, device{device}) (tensor.hpp:99-102). `values` is
 * read synchronously before return; page-locked memory (pb_host_alloc) makes
 * the copy a direct DMA. Unlike the C++ constructor no host mirror is kept,
 * so a later read copies from the device. */
int pb_tensor_create(const int64_t* shape, size_t rank, const float* values,
                     size_t count, int device, pb_tensor** out);
/* The same tensor with the host-to-device copy enqueued on this thread's
 * upload stream and not waited for: the call returns at once, and every
 * kernel or copy that later reads the tensor waits (on the device) for the
 * copy, so an upload overlaps work that does not read it. `values` must stay
 * unchanged and allocated until the copy is done (any read of the tensor, or
 * pb_synchronize); page-locked memory (pb_host_alloc) makes it a DMA. No
 * counterpart in the reference, whose copies are synchronous
 * (src/cuda_jit.cpp:711-734). */
int pb_tensor_create_async(const int64_t* shape, size_t rank, const float* values,
                           size_t count, int device, pb_tensor** out);
/* full(shape, value, device) (tensor.hpp:184-186) */
int pb_tensor_full(const int64_t* shape, size_t rank, float value, int device,
                   pb_tensor** out);
/* A shape-only tensor without device storage: usable only to build
 * expressions passed to pb_expr_describe (plan inspection without a GPU). */
int pb_tensor_placeholder(const int64_t* shape, size_t rank, int device,
                          pb_tensor** out);
void pb_tensor_release(pb_tensor* tensor);
int pb_tensor_rank(const pb_tensor* tensor, size_t* rank);
int pb_tensor_shape(const pb_tensor* tensor, int64_t* shape, size_t capacity);
int pb_tensor_strides(const pb_tensor* tensor, int64_t* strides, size_t capacity);
int pb_tensor_numel(const pb_tensor* tensor, size_t* numel);
int pb_tensor_storage_offset(const pb_tensor* tensor, int64_t* offset);
int pb_tensor_is_contiguous(const pb_tensor* tensor, int* contiguous);
int pb_tensor_device(const pb_tensor* tensor, int* device);
/* tensor::realize / tensor::synchronize (tensor.hpp:118-119) */
int pb_tensor_realize(const pb_tensor* tensor);
int pb_tensor_synchronize(const pb_tensor* tensor);
/* tensor::cpu() copied into `values` (tensor.hpp:116). Materialises first.
 * Copies straight from device memory into `values`. */
int pb_tensor_read(const pb_tensor* tensor, float* values, size_t count);
/* tensor::device_data() (tensor.hpp:117): device address and size in bytes. */
int pb_tensor_device_pointer(const pb_tensor* tensor, uint64_t* pointer,
                             size_t* bytes);
/* tensor::operator[] (tensor.hpp:120-123) */
int pb_tensor_index(const pb_tensor* tensor, const pb_index* indices,
                    size_t count, pb_expr** out);

/* ---- expressions -------------------------------------------------------- */
/* tensor_expr(const tensor&) / tensor_expr(float) (tensor.hpp:146-147) */
int pb_expr_from_tensor(const pb_tensor* tensor, pb_expr** out);
int pb_expr_scalar(float value, pb_expr** out);
void pb_expr_release(pb_expr* expr);
/* PB_ADD..PB_MATMUL */
int pb_expr_binary(int op, const pb_expr* lhs, const pb_expr* rhs, pb_expr** out);
/* PB_EXP, PB_RECIPROCAL, PB_TRANSPOSE, PB_RELU, PB_LOGISTIC */
int pb_expr_unary(int op, const pb_expr* value, pb_expr** out);
/* reshape / broadcast_to (tensor.hpp:197-204) */
int pb_expr_reshape(const pb_expr* value, const int64_t* shape, size_t rank,
                    pb_expr** out);
int pb_expr_broadcast(const pb_expr* value, const int64_t* shape, size_t rank,
                      pb_expr** out);
/* unsqueeze / concat (tensor.hpp:200, 205-207) */
int pb_expr_unsqueeze(const pb_expr* value, size_t axis, pb_expr** out);
int pb_expr_concat(const pb_expr* lhs, const pb_expr* rhs, size_t axis,
                   pb_expr** out);
/* N-D permutation of the axes: output axis d is input axis perm[d]. No
 * counterpart in the reference, whose transpose is rank 2 only
 * (src/tensor.cpp:430-437); PB_TRANSPOSE keeps that rule. Realised alone
 * (or with slices and unsqueezes) it is a strided view: no copy until the
 * values are read out. */
int pb_expr_permute(const pb_expr* value, const int64_t* perm, size_t rank,
                    pb_expr** out);
/* Batched matmul: [B,M,K] @ [B,K,N] -> [B,M,N], one fp32 product per batch
 * (3xTF32 on the tensor cores, every batch in one launch, when
 * B*M*N*K >= 2^27; else the CUDA-core GEMM). No counterpart in the
 * reference, whose matmul is rank 2 only (src/tensor.cpp:366-381);
 * PB_MATMUL keeps that rule. */
int pb_expr_batched_matmul(const pb_expr* lhs, const pb_expr* rhs, pb_expr** out);
/* sum / max with keepdim (PB_SUM, PB_MAX) */
int pb_expr_reduce(int op, const pb_expr* value, size_t axis, int keepdim,
                   pb_expr** out);
/* softmax(value, axis) (ops.hpp:8) */
int pb_expr_softmax(const pb_expr* value, size_t axis, pb_expr** out);
/* tensor_expr::shape() (tensor.hpp:150). *rank receives the rank; up to
 * `capacity` extents are written. A scalar expression has rank 0. */
int pb_expr_shape(const pb_expr* expr, int64_t* shape, size_t capacity,
                  size_t* rank);
/* tensor_expr::operator tensor() (tensor.hpp:154): a lazy tensor. */
int pb_expr_to_tensor(const pb_expr* expr, pb_tensor** out);
/* materialize(expr) (tensor.hpp:217): a realised tensor. */
int pb_materialize(const pb_expr* expr, pb_tensor** out);
/* Describes the kernel plan for `expr` (kernels, schedules, and with
 * with_source != 0 the generated CUDA). *needed receives the full length
 * including the terminating NUL; the text is truncated to `capacity`. */
int pb_expr_describe(const pb_expr* expr, int with_source, char* text,
                     size_t capacity, size_t* needed);

/* ---- host memory, timing, counters -------------------------------------- */
int pb_host_alloc(size_t bytes, void** pointer); /* page-locked */
int pb_host_free(void* pointer);
/* Device timer on this thread's porch stream of `device`: begin records a
 * start event, end records a stop event, waits for it and returns the
 * elapsed milliseconds. */
int pb_timer_begin(int device, void** timer);
int pb_timer_end(void* timer, float* milliseconds);
/* Synchronise this thread's porch stream on `device`. */
int pb_device_synchronize(int device);
/* Drops every cached device block of `device` (*released receives the
 * bytes; may be NULL). Blocks freed by porch stay cached per stream for
 * reuse without a driver call until then; they are carved from 256 MiB
 * slabs (a larger block has a slab of its own), and a slab goes back to the
 * driver once every block carved from it has been dropped. */
int pb_empty_cache(int device, size_t* released);
/* Kernel launches issued by this library since process start. */
uint64_t pb_launch_count(void);
/* Per-launch kernel timing (events around each launch); see
 * pbrt_profile_read for the text format. */
int pb_profile_enable(int enable);
int pb_profile_read(char* text, size_t capacity);
/* Host-side phase timers of materialize (bind = inference, canonical graph
 * and plan lookup; inputs = stream ordering and allocations; launch; wrap).
 * Read returns "<phase>_us_per_call<TAB><value>" lines and resets. */
int pb_host_profile_enable(int enable);
int pb_host_profile_read(char* text, size_t capacity);
/* Fills `values` (count floats) with seeded synthetic data: dist 0 = uniform
 * on [a, b), dist 1 = normal(mean a, stddev b). Deterministic for a given
 * (seed, count, dist, a, b), independent of thread count. Host side only. */
int pb_fill_synthetic(float* values, size_t count, uint64_t seed, int dist,
                      double a, double b);

/* ---- row sharding across GPUs (one process per GPU) --------------------- */
/* No counterpart in the reference, which runs on one device only
 * (src/backend.cpp, src/cuda_jit.cpp:437-528). A graph whose rows are
 * independent is realised per row block on each rank's GPU; these calls move
 * data only where a consumer needs the whole tensor. */
typedef struct pb_comm_s pb_comm;
/* 128-byte NCCL unique id, made on one rank and passed to the others. */
int pb_comm_unique_id(char id[128]);
/* Joins rank `rank` of `nranks` on `device`; every host-side wait of this
 * communicator (init included) gives up after timeout_s seconds, aborting
 * the communicator and returning PB_ERR_RUNTIME. */
int pb_comm_init(int nranks, const char id[128], int rank, int device, double timeout_s,
                 pb_comm** out);
int pb_comm_info(const pb_comm* comm, int* rank, int* nranks, int* device);
/* Bound (seconds) on this communicator's host-side waits from now on. */
int pb_comm_set_timeout(pb_comm* comm, double timeout_s);
/* Aborts outstanding work; later calls on the communicator fail. */
int pb_comm_abort(pb_comm* comm);
int pb_comm_release(pb_comm* comm);
/* Rows [*begin, *end) of a `rows`-row tensor owned by `rank` of `nranks`:
 * contiguous blocks, the first rows % nranks ranks holding one extra row. */
int pb_row_block(int64_t rows, int rank, int nranks, int64_t* begin, int64_t* end);
/* Every rank passes its row block `shard` (realised first if lazy; its row
 * count must be pb_row_block's for this rank) and receives the whole
 * [total_rows, ...] tensor, row blocks concatenated in rank order, on its own
 * device: one ncclAllGather for equal blocks, grouped Send/Recv otherwise.
 * Returns once the gather has completed on the device. */
int pb_allgather_rows(pb_comm* comm, const pb_tensor* shard, int64_t total_rows,
                      pb_tensor** out);
/* The same gather enqueued on the communicator's own stream, returning at
 * once: it waits (on the device) for the shard's producer, and whatever
 * later reads the result waits for the gather the same way, so the gather
 * overlaps compute enqueued after it. pb_comm_wait is the bounded
 * completion check (it aborts the communicator on timeout or error); call it
 * before reading results on the host if a peer may fail. */
int pb_allgather_rows_async(pb_comm* comm, const pb_tensor* shard, int64_t total_rows,
                            pb_tensor** out);
/* Waits, bounded by the communicator's timeout, until every asynchronous
 * gather issued so far has completed. */
int pb_comm_wait(pb_comm* comm);

/* ---- failure-detection test hook ---------------------------------------- */
/* No counterpart in the reference, which has no device-side waits. While
 * enabled (it is off by default), tensor-core GEMM plans built from then on
 * (a plan key of their own) make one CTA wait on an mbarrier that nothing
 * arrives on: its bounded wait gives up (about two seconds), the kernel
 * records code 0x7c07 in the device error word, waits for its own copies in
 * flight, frees its tensor memory and returns; the next synchronisation
 * raises PB_ERR_RUNTIME. Only for tests of that path. */
int pb_test_gemm_stall(int enable);

/* ---- matmul without allocation ------------------------------------------ */
/* C = A @ B in fp32 (3xTF32 on tcgen05), on raw device pointers, allocating
 * nothing. No counterpart in the reference: it is for callers that must not
 * let a library allocate device memory (a custom arena or allocator hook
 * owns the device, or an allocation would synchronise or fail where they
 * call). A, B, C are row-major device arrays on the current device:
 * A [M,K], B [K,N], C [M,N]; M % 128 == 0, N % 256 == 0, K % 64 == 0.
 * A and C must be 16-byte aligned (they are read and written in float4s),
 * B 4-byte aligned; all three must be device (or managed) memory of the
 * current device. Misaligned, host or other-device pointers, and buffers
 * that end before their shape does within one allocation, are rejected
 * with PB_ERR_INVALID_ARGUMENT before anything is enqueued.
 * The split operands live in a fixed 64 MiB device array that every GPU
 * loading this library holds until exit; calls needing more than that
 * (2 * (M*K + N*K) floats) are rejected with PB_ERR_INVALID_ARGUMENT.
 * Operands must be finite: with Inf or NaN in A or B the call returns
 * PB_ERR_INVALID_ARGUMENT and C is unspecified (pb_materialize handles them).
 * All calls share the array, so calls that overlap on the GPU race. The first
 * call on each device sets that device up (symbol address, kernel limits);
 * make it outside any stream capture. The call enqueues on `stream`
 * (a cudaStream_t, NULL for the default stream) and waits for the result. */
int pb_matmul_3xtf32_noalloc(const float* a, const float* b, float* c,
                             int64_t m, int64_t n, int64_t k, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PORCH_B200_H */
