// Row sharding across GPUs, one process per GPU.
//
// The reference runs on one device only (src/backend.cpp keeps a single
// context; src/cuda_jit.cpp:437-528 binds device 0). Graphs whose leading
// (row) axis is independent -- elementwise maps, row softmax, a matmul whose
// left operand is row-blocked -- give the same rows whether they run whole
// or per row block, so each rank realises its own block of rows on its own
// GPU with no exchange, and NCCL over NVLink moves data only where a
// consumer needs the whole tensor: allgather_rows below.
//
// Partition: rows [begin, end) of rank r of n are the contiguous block
// partition, the first rows % n ranks holding one extra row. Equal blocks
// gather with one ncclAllGather straight into the output (the concatenation
// of row blocks in rank order is the whole tensor, because a row-major
// tensor's row block is one contiguous range); unequal blocks with one
// grouped Send/Recv per peer into the output's row offsets.
#include "detail.hpp"

#include <stdexcept>
#include <string>
#include <utility>

namespace porch::detail {

    std::pair<index_t, index_t> row_block(index_t rows, int rank, int nranks) {
        if (nranks <= 0 || rank < 0 || rank >= nranks)
            throw std::invalid_argument("rank must lie in [0, nranks)");
        if (rows < 0) throw std::invalid_argument("row count must be non-negative");
        const index_t n = nranks;
        const index_t base = rows / n;
        const index_t extra = rows % n;
        const index_t r = rank;
        const index_t begin = r * base + (r < extra ? r : extra);
        return {begin, begin + base + (r < extra ? 1 : 0)};
    }

    communicator::~communicator() {
        if (comm != nullptr) (void)pbrt_nccl_destroy(comm);
        comm = nullptr;
    }

    std::unique_ptr<communicator> make_communicator(
        int nranks, const char id[128], int rank, int device, double timeout_s
    ) {
        if (nranks <= 0 || rank < 0 || rank >= nranks)
            throw std::invalid_argument("rank must lie in [0, nranks)");
        if (!(timeout_s > 0.0)) throw std::invalid_argument("timeout must be positive");
        auto c = std::make_unique<communicator>();
        c->rank = rank;
        c->nranks = nranks;
        c->device = device;
        c->timeout_s = timeout_s;
        check(pbrt_nccl_init_rank(nranks, id, rank, device, timeout_s, &c->comm));
        return c;
    }

    tensor allgather_rows(communicator& c, const tensor& shard, index_t total_rows,
                          bool asynchronous) {
        if (c.comm == nullptr || c.aborted)
            throw std::runtime_error("communicator is not usable (aborted or destroyed)");
        if (shard.rank() == 0) throw std::invalid_argument("allgather_rows needs a tensor of rank >= 1");
        if (shard.placement().ordinal() != c.device)
            throw std::invalid_argument("shard lives on a different device than the communicator");
        const auto [begin, end] = row_block(total_rows, c.rank, c.nranks);
        const std::vector<index_t> shape(shard.shape().begin(), shard.shape().end());
        if (shape[0] != end - begin)
            throw std::invalid_argument(
                "shard has " + std::to_string(shape[0]) + " rows; the block partition of " +
                std::to_string(total_rows) + " rows gives rank " + std::to_string(c.rank) + " " +
                std::to_string(end - begin));
        index_t inner = 1;
        for (size_t d = 1; d < shape.size(); ++d) inner *= shape[d];
        std::vector<index_t> out_shape = shape;
        out_shape[0] = total_rows;
        const size_t out_count = checked_numel(out_shape);

        auto storage_in = tensor_access::storage(shard); // realises a lazy shard
        make_contiguous(storage_in);                      // a view: its rows copied out
        if (asynchronous && c.stream == nullptr) {
            pbrt_stream s = nullptr;
            check(pbrt_stream_create(c.device, &s));
            c.stream = std::make_shared<stream_ref>(c.device, s);
        }
        auto stream = asynchronous ? c.stream : current_stream(c.device);
        auto storage = std::make_shared<realized_storage>();
        storage->count = out_count;
        storage->device = c.device;
        storage->device_values = allocate(c.device, out_count * sizeof(float32_t), stream);
        if (out_count == 0) {
            storage->host_current = true;
            return tensor_access::from_storage(std::move(out_shape), std::move(storage),
                                               shard.placement());
        }
        auto& in_state = *cuda_jit::buffer_access::state(storage_in->device_values);
        auto& out_state = *cuda_jit::buffer_access::state(storage->device_values);
        order_read(in_state, stream);

        const bool equal = total_rows % c.nranks == 0;
        int status = PBRT_OK;
        if (equal) {
            status = pbrt_nccl_allgather_f32(c.comm, in_state.ptr, out_state.ptr,
                                             static_cast<size_t>((end - begin) * inner),
                                             stream->stream);
        } else {
            const size_t row_bytes = static_cast<size_t>(inner) * sizeof(float32_t);
            if (end > begin)
                status = pbrt_memcpy_d2d_async(c.device, out_state.ptr + begin * row_bytes,
                                               in_state.ptr, (end - begin) * row_bytes,
                                               stream->stream);
            if (status == PBRT_OK) status = pbrt_nccl_group_start();
            if (status == PBRT_OK) {
                for (int p = 0; p < c.nranks && status == PBRT_OK; ++p) {
                    if (p == c.rank) continue;
                    const auto [pb, pe] = row_block(total_rows, p, c.nranks);
                    if (end > begin)
                        status = pbrt_nccl_send_f32(c.comm, in_state.ptr,
                                                    static_cast<size_t>((end - begin) * inner), p,
                                                    stream->stream);
                    if (status == PBRT_OK && pe > pb)
                        status = pbrt_nccl_recv_f32(c.comm, out_state.ptr + pb * row_bytes,
                                                    static_cast<size_t>((pe - pb) * inner), p,
                                                    stream->stream);
                }
                const int end_status = pbrt_nccl_group_end();
                if (status == PBRT_OK) status = end_status;
                if (status == PBRT_OK) status = pbrt_nccl_settle(c.comm);
            }
        }
        // Bounded wait: a peer that never arrives (or an asynchronous NCCL
        // error) aborts the communicator and surfaces here as an exception,
        // instead of hanging a later synchronize.
        if (status == PBRT_OK && !asynchronous)
            status = pbrt_nccl_wait(c.comm, c.device, stream->stream, c.timeout_s);
        if (status != PBRT_OK) {
            abort_communicator(c);
            throw_status(status);
        }
        set_producer(out_state, stream);
        return tensor_access::from_storage(std::move(out_shape), std::move(storage),
                                           shard.placement());
    }

    void wait_communicator(communicator& c) {
        if (c.comm == nullptr || c.aborted)
            throw std::runtime_error("communicator is not usable (aborted or destroyed)");
        if (c.stream == nullptr) return;
        const int status = pbrt_nccl_wait(c.comm, c.device, c.stream->stream, c.timeout_s);
        if (status != PBRT_OK) {
            abort_communicator(c);
            throw_status(status);
        }
    }

    void abort_communicator(communicator& c) {
        if (c.comm != nullptr && !c.aborted) (void)pbrt_nccl_abort(c.comm);
        c.aborted = true;
    }

} // namespace porch::detail
