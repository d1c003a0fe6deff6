// Internal declarations shared by the porch_b200 C++ front-end.
#pragma once

#include "porch/tensor.hpp"
#include "porch_b200_rt.h"

#include <atomic>
#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

namespace porch::detail {

    // ------------------------------------------------------------ errors --
    // Maps a runtime status to the reference's exception conventions
    // (std::invalid_argument / std::out_of_range / compilation_error /
    // std::runtime_error; src/cuda_jit.cpp:304-339, include/porch/cuda_jit.hpp:50-58).
    [[noreturn]] void throw_status(int status);
    inline void check(int status) {
        if (status != PBRT_OK) throw_status(status);
    }

    // ----------------------------------------------------------- streams --
    // A stream with shared lifetime: buffers keep their producer stream alive
    // until their stream-ordered free has been enqueued (the same guarantee
    // as the reference's shared stream_handle, src/cuda_jit.cpp:479-528).
    struct stream_ref {
        int device = 0;
        pbrt_stream stream = nullptr;
        stream_ref(int device_index, pbrt_stream s)
            : device(device_index), stream(s) {}
        stream_ref(const stream_ref&) = delete;
        stream_ref& operator=(const stream_ref&) = delete;
        ~stream_ref();
    };

    // The calling thread's stream on `device`.
    std::shared_ptr<stream_ref> current_stream(int device);
    // Streams the calling thread has created so far.
    std::vector<std::shared_ptr<stream_ref>> thread_streams();
    // The calling thread's host-to-device upload stream on `device`
    // (pb_tensor_create_async); readers order behind it with events.
    std::shared_ptr<stream_ref> upload_stream(int device);

    // ------------------------------------------------------- dry run --
    // True while a plan is being inspected without a device (placeholder
    // tensors); never set on the execution path.
    bool placeholder_mode();

} // namespace porch::detail

namespace porch::cuda_jit {

    struct device_buffer_state {
        int device = 0;
        uint64_t ptr = 0;
        size_t bytes = 0;
        size_t capacity = 0; // allocator size class; 0 = not from the cache
        std::mutex mutex;
        std::shared_ptr<detail::stream_ref> producer;
        std::vector<std::shared_ptr<detail::stream_ref>> readers;
        // Set for an asynchronous upload: recorded on the producer stream
        // right after the copy; readers wait on it rather than on
        // everything the producer stream holds.
        pbrt_event ready = nullptr;

        device_buffer_state() = default;
        device_buffer_state(const device_buffer_state&) = delete;
        device_buffer_state& operator=(const device_buffer_state&) = delete;
        ~device_buffer_state();
    };

    struct buffer_access {
        static const std::shared_ptr<device_buffer_state>& state(
            const device_buffer& buffer
        ) {
            return buffer.state_;
        }
        static device_buffer wrap(std::shared_ptr<device_buffer_state> state) {
            device_buffer b;
            b.state_ = std::move(state);
            return b;
        }
    };

} // namespace porch::cuda_jit

namespace porch::detail {

    // Allocates `bytes` on `device`, stream-ordered on `stream`, from the
    // per-device caching allocator.
    cuda_jit::device_buffer allocate(
        int device, size_t bytes, const std::shared_ptr<stream_ref>& stream
    );
    // Returns a block to the cache (called when its last owner drops it).
    void recycle(int device, uint64_t ptr, size_t capacity, std::shared_ptr<stream_ref> stream);
    // Returns a block to `stream`'s free list once every (device, event) in
    // `events` -- recorded behind reads on other streams -- has completed.
    void defer_recycle(int device, uint64_t ptr, size_t capacity, std::shared_ptr<stream_ref> stream,
                       std::vector<std::pair<int, pbrt_event>> events);
    // Drops every cached block of `device` (slabs left with no block go back
    // to the driver); returns the bytes dropped.
    size_t release_cached_blocks(int device);
    // Gives one block back (a slab block: to its slab; any other: to the
    // driver). The caller has ordered it after every use.
    void release_block(int device, uint64_t ptr, size_t capacity);
    // Makes `stream` wait for the buffer's producer when they differ, and
    // records `stream` as a reader so the eventual free is ordered after it.
    void order_read(
        cuda_jit::device_buffer_state& buffer,
        const std::shared_ptr<stream_ref>& stream
    );
    void set_producer(
        cuda_jit::device_buffer_state& buffer, std::shared_ptr<stream_ref> stream
    );

    // Realised storage of a tensor: device values plus a lazily filled host
    // mirror (the reference zero-fills a host vector of numel floats twice per
    // materialisation, src/tensor.cpp:1019 and :1073-1076; here the mirror is
    // allocated only when data()/cpu() is called).
    //
    // A storage may instead be a strided view of another storage's device
    // values: materialising a graph that only slices, transposes,
    // unsqueezes or (contiguously) reshapes one realised tensor launches
    // nothing and records element (i0, i1, ...) at
    // view_offset + sum_d i_d * view_strides[d] of `view_base`. Later graphs
    // read the view in place (canonicalised as a slice over the base); the
    // public accessors still see a contiguous tensor, copied out on the
    // first request for its values (make_contiguous). A view is a snapshot:
    // before a raw handle to a base's values is handed out (device_data()),
    // its live views are copied out, and no view is made of a storage whose
    // handle has been handed out.
    struct realized_storage {
        cuda_jit::device_buffer device_values; // a view: the base's buffer
        size_t count = 0;
        int device = 0;
        std::mutex host_mutex;
        std::vector<float32_t> host;
        bool host_current = false;
        bool placeholder = false; // shape-only tensor for plan inspection

        std::mutex view_mutex;
        std::shared_ptr<realized_storage> view_base; // null: contiguous values
        std::vector<index_t> view_shape;
        std::vector<index_t> view_strides;
        index_t view_offset = 0;
        // Bumped when a view turns into contiguous values (bound graphs that
        // read it through its base are then rebuilt).
        std::atomic<uint32_t> layout_epoch{0};
        bool escaped = false; // a handle to device_values was handed out
        std::vector<std::weak_ptr<realized_storage>> views;

        // 3xTF32 splits of these values kept for later GEMMs (hi, lo and the
        // non-finite flag, per operand layout key); dropped when a handle to
        // the values is handed out. Guarded by view_mutex.
        struct kept_split {
            std::string key;
            cuda_jit::device_buffer hi, lo, flag;
        };
        std::vector<kept_split> splits;
    };

    // A strided layout over a storage's linear values.
    struct strided_layout {
        std::vector<index_t> shape;
        std::vector<index_t> strides;
        index_t offset = 0;
    };

    // The view fields of `s` under its view_mutex: false when `s` holds
    // contiguous values.
    bool view_of(realized_storage& s, std::shared_ptr<realized_storage>& base, strided_layout& layout);
    // Turns a view into contiguous values of its own (one copy kernel);
    // no-op for contiguous storage.
    void make_contiguous(const std::shared_ptr<realized_storage>& s);
    // Before a handle to `s`'s device values leaves the library: copies out
    // its live views (so they stay snapshots), makes `s` itself contiguous
    // and marks it so that no new view is made of it.
    void escape(const std::shared_ptr<realized_storage>& s);

    enum class expr_kind : uint8_t {
        input,
        scalar,
        add,
        subtract,
        multiply,
        divide,
        matmul,
        slice,
        reshape,
        unsqueeze,
        transpose,
        broadcast,
        concat,
        sum,
        max,
        maximum,
        minimum,
        exp,
        reciprocal,
        // Internal N-D permutation (no reference counterpart: its transpose
        // is rank 2 only, src/tensor.cpp:430-437); `shape` holds the
        // permutation, output dim d = input dim perm[d].
        permute,
        // Internal batched matmul [B, M, K] @ [B, K, N] -> [B, M, N] (the
        // reference's matmul is rank 2 only, src/tensor.cpp:366-381).
        batched_matmul,
    };

    const char* kind_name(expr_kind kind);

} // namespace porch::detail

namespace porch {

    // IR node. Same 19 kinds and parameters as the reference
    // (src/tensor.cpp:26-60) plus the internal permute, except that an input
    // holds shared ownership of the realised storage instead of a raw
    // `const tensor*`.
    struct tensor_expr::node {
        detail::expr_kind kind = detail::expr_kind::scalar;
        std::shared_ptr<detail::realized_storage> storage; // input
        std::vector<index_t> input_shape;                  // input
        device placement{};                                // input
        float32_t scalar = 0.0F;
        std::shared_ptr<const node> lhs;
        std::shared_ptr<const node> rhs;
        std::vector<index_t> slice_shape;
        std::vector<index_t> slice_strides;
        std::vector<index_t> shape; // reshape / broadcast target
        index_t slice_offset = 0;
        size_t axis = 0;
        bool keepdim = false;
        // Lowering bound to this exact root (canonical graph + plan), filled
        // on its first materialisation so repeat realisations of the same
        // expression skip inference, canonicalisation and plan lookup.
        mutable std::shared_ptr<const void> bound;
    };

    struct expr_access {
        static const std::shared_ptr<const tensor_expr::node>& root(
            const tensor_expr& e
        ) {
            return e.root_;
        }
        static tensor_expr make(std::shared_ptr<const tensor_expr::node> n) {
            return tensor_expr{std::move(n)};
        }
    };

    struct index_access {
        static int kind(const tensor_index& i) {
            return static_cast<int>(i.kind_);
        }
        static index_t index(const tensor_index& i) { return i.index_; }
        static slice range(const tensor_index& i) { return i.slice_; }
    };

    // Internal access to tensor state for the C-ABI binding and the planner.
    struct tensor_access {
        static tensor from_storage(
            std::vector<index_t> shape,
            std::shared_ptr<detail::realized_storage> storage, device placement
        );
        static std::shared_ptr<detail::realized_storage> storage(
            const tensor& t
        );
        static bool is_lazy(const tensor& t);
        static tensor placeholder(std::vector<index_t> shape, device placement);
    };

} // namespace porch

namespace porch::detail {

    // Shape inference with the reference's validation and messages
    // (src/tensor.cpp:279-496). Returns false for scalar expressions.
    struct shape_info {
        std::vector<index_t> shape;
        bool scalar = true;
        bool has_input = false;
        device placement{};
    };
    shape_info infer(const tensor_expr::node& root);

    size_t checked_numel(std::span<const index_t> shape);
    std::vector<index_t> contiguous_strides(std::span<const index_t> shape);
    // The GPU that device{ordinal} runs on among `count` visible devices:
    // the ordinal itself when present, else device 0 (the reference's only
    // device); a negative ordinal throws std::invalid_argument.
    int checked_ordinal(int ordinal, int count);

    // Lower, compile and launch `root`; the result is a realised tensor on the
    // graph's device (src/tensor.cpp:1002-1066 is the reference's driver).
    tensor materialize_graph(const tensor_expr::node& root);

    // Host-side phase timers of materialize (nanoseconds): enabled by
    // host_profile_enable; read and reset by host_profile_read.
    enum host_phase {
        phase_bind,
        phase_stream,
        phase_order,
        phase_alloc,
        phase_launch,
        phase_wrap,
        phase_total,
        phase_count
    };
    void host_count(const char* what); // allocator hit/miss counters
    void host_profile_enable(bool on);
    std::string host_profile_read();

    // ---------------------------------------------------- row sharding --
    // One rank of a one-process-per-GPU communicator (NCCL over NVLink).
    struct communicator {
        pbrt_comm comm = nullptr;
        int rank = 0;
        int nranks = 1;
        int device = 0;
        double timeout_s = 60.0; // bound on every host-side wait
        bool aborted = false;
        // Stream of the asynchronous gathers (created on first use), so a
        // gather overlaps the compute that the caller enqueues next.
        std::shared_ptr<stream_ref> stream;
        communicator() = default;
        communicator(const communicator&) = delete;
        communicator& operator=(const communicator&) = delete;
        ~communicator();
    };
    std::unique_ptr<communicator> make_communicator(
        int nranks, const char id[128], int rank, int device, double timeout_s
    );
    void abort_communicator(communicator& c);
    // Rows [begin, end) of `rows` owned by `rank` of `nranks` (contiguous
    // blocks, the first rows % nranks ranks one row longer).
    std::pair<index_t, index_t> row_block(index_t rows, int rank, int nranks);
    // Every rank passes its realised row block; every rank receives the whole
    // [total_rows, ...] tensor (row blocks concatenated in rank order).
    // Synchronous: on the caller's stream, returns after a bounded wait for
    // completion. Asynchronous: on the communicator's own stream, ordered
    // after the shard's producer by an event; the result's readers order
    // after it the same way; wait_communicator() is the bounded completion
    // (and failure) check.
    tensor allgather_rows(communicator& c, const tensor& shard, index_t total_rows,
                          bool asynchronous = false);
    void wait_communicator(communicator& c);

    // Human-readable description of the plan chosen for `root` (kernels,
    // schedules and generated sources). Works on placeholder inputs without a
    // device, so the lowering can be inspected on a build machine.
    std::string describe_plan(const tensor_expr::node& root, bool with_source);

} // namespace porch::detail
