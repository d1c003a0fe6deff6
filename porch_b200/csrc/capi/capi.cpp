// Flat C-ABI over the porch C++ API (include/porch_b200.h).
#include "porch_b200.h"
#include "lower.hpp"

#include "../front/detail.hpp"
#include "porch/backend.hpp"
#include "porch/ops.hpp"

#include <cmath>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

struct pb_tensor_s {
    porch::tensor value;
};

struct pb_expr_s {
    porch::tensor_expr value;
};

struct pb_comm_s {
    std::unique_ptr<porch::detail::communicator> value;
};

namespace {

    thread_local std::string tl_error;

    template <typename F>
    int guarded(F&& f) {
        try {
            f();
            return PB_OK;
        } catch (const porch::cuda_jit::compilation_error& e) {
            tl_error = e.log();
            return PB_ERR_COMPILATION;
        } catch (const std::invalid_argument& e) {
            tl_error = e.what();
            return PB_ERR_INVALID_ARGUMENT;
        } catch (const std::out_of_range& e) {
            tl_error = e.what();
            return PB_ERR_OUT_OF_RANGE;
        } catch (const std::exception& e) {
            tl_error = e.what();
            return PB_ERR_RUNTIME;
        } catch (...) {
            tl_error = "unknown error";
            return PB_ERR_RUNTIME;
        }
    }

    void require(const void* p, const char* what) {
        if (p == nullptr) throw std::invalid_argument(std::string{what} + " is null");
    }

    std::vector<porch::index_t> shape_of(const int64_t* shape, size_t rank) {
        if (rank != 0) require(shape, "shape");
        return std::vector<porch::index_t>(shape, shape + rank);
    }

    pb_expr* wrap(porch::tensor_expr e) { return new pb_expr_s{std::move(e)}; }
    pb_tensor* wrap(porch::tensor t) { return new pb_tensor_s{std::move(t)}; }

} // namespace

namespace porch::detail {
    // Lets other translation units of the C-ABI (the no-allocation matmul)
    // report through pb_last_error().
    void set_last_error(const std::string& message) { tl_error = message; }
} // namespace porch::detail

extern "C" {

const char* pb_last_error(void) { return tl_error.c_str(); }

int pb_is_available(void) { return porch::cuda_jit::is_available() ? 1 : 0; }

const char* pb_backend_name(void) {
    static const std::string name{porch::backend_name(porch::backend_for(porch::device{}))};
    return name.c_str();
}

int pb_synchronize(void) {
    return guarded([] { porch::cuda_jit::synchronize(); });
}

int pb_tensor_create(const int64_t* shape, size_t rank, const float* values, size_t count,
                     int device, pb_tensor** out) {
    return guarded([&] {
        require(out, "out");
        auto s = shape_of(shape, rank);
        const size_t expected = porch::detail::checked_numel(s);
        if (count != expected)
            throw std::invalid_argument("tensor data size does not match shape");
        if (count != 0) require(values, "values");
        int ndev = 0;
        porch::detail::check(pbrt_device_count(&ndev));
        auto storage = std::make_shared<porch::detail::realized_storage>();
        storage->count = count;
        storage->device = porch::detail::checked_ordinal(device, ndev);
        auto stream = porch::detail::current_stream(storage->device);
        storage->device_values =
            porch::detail::allocate(storage->device, count * sizeof(float), stream);
        if (count != 0) {
            const auto& st = porch::cuda_jit::buffer_access::state(storage->device_values);
            porch::detail::check(pbrt_memcpy_h2d_async(storage->device, st->ptr, values,
                                                       count * sizeof(float), stream->stream));
            porch::detail::check(pbrt_stream_synchronize(storage->device, stream->stream));
        }
        *out = wrap(porch::tensor_access::from_storage(std::move(s), std::move(storage),
                                                       porch::device{device}));
    });
}

int pb_tensor_create_async(const int64_t* shape, size_t rank, const float* values, size_t count,
                           int device, pb_tensor** out) {
    return guarded([&] {
        require(out, "out");
        auto s = shape_of(shape, rank);
        const size_t expected = porch::detail::checked_numel(s);
        if (count != expected)
            throw std::invalid_argument("tensor data size does not match shape");
        if (count != 0) require(values, "values");
        int ndev = 0;
        porch::detail::check(pbrt_device_count(&ndev));
        auto storage = std::make_shared<porch::detail::realized_storage>();
        storage->count = count;
        storage->device = porch::detail::checked_ordinal(device, ndev);
        // The block and its copy belong to the upload stream: the first
        // kernel (or copy) that reads the tensor waits for it with an event.
        auto stream = porch::detail::upload_stream(storage->device);
        storage->device_values =
            porch::detail::allocate(storage->device, count * sizeof(float), stream);
        if (count != 0) {
            const auto& st = porch::cuda_jit::buffer_access::state(storage->device_values);
            porch::detail::check(pbrt_memcpy_h2d_async(storage->device, st->ptr, values,
                                                       count * sizeof(float), stream->stream));
            pbrt_event e = nullptr;
            porch::detail::check(pbrt_event_create(storage->device, 0, &e));
            st->ready = e;
            porch::detail::check(pbrt_event_record(storage->device, e, stream->stream));
        }
        *out = wrap(porch::tensor_access::from_storage(std::move(s), std::move(storage),
                                                       porch::device{device}));
    });
}

int pb_tensor_full(const int64_t* shape, size_t rank, float value, int device,
                   pb_tensor** out) {
    return guarded([&] {
        require(out, "out");
        *out = wrap(porch::full(shape_of(shape, rank), value, porch::device{device}));
    });
}

int pb_tensor_placeholder(const int64_t* shape, size_t rank, int device, pb_tensor** out) {
    return guarded([&] {
        require(out, "out");
        *out = wrap(porch::tensor_access::placeholder(shape_of(shape, rank), porch::device{device}));
    });
}

void pb_tensor_release(pb_tensor* tensor) { delete tensor; }

int pb_tensor_rank(const pb_tensor* t, size_t* rank) {
    return guarded([&] {
        require(t, "tensor");
        require(rank, "rank");
        *rank = t->value.rank();
    });
}

int pb_tensor_shape(const pb_tensor* t, int64_t* shape, size_t capacity) {
    return guarded([&] {
        require(t, "tensor");
        auto s = t->value.shape();
        for (size_t i = 0; i < s.size() && i < capacity; ++i) shape[i] = s[i];
    });
}

int pb_tensor_strides(const pb_tensor* t, int64_t* strides, size_t capacity) {
    return guarded([&] {
        require(t, "tensor");
        auto s = t->value.strides();
        for (size_t i = 0; i < s.size() && i < capacity; ++i) strides[i] = s[i];
    });
}

int pb_tensor_numel(const pb_tensor* t, size_t* numel) {
    return guarded([&] {
        require(t, "tensor");
        require(numel, "numel");
        *numel = t->value.numel();
    });
}

int pb_tensor_storage_offset(const pb_tensor* t, int64_t* offset) {
    return guarded([&] {
        require(t, "tensor");
        require(offset, "offset");
        *offset = t->value.storage_offset();
    });
}

int pb_tensor_is_contiguous(const pb_tensor* t, int* contiguous) {
    return guarded([&] {
        require(t, "tensor");
        require(contiguous, "contiguous");
        *contiguous = t->value.is_contiguous() ? 1 : 0;
    });
}

int pb_tensor_device(const pb_tensor* t, int* device) {
    return guarded([&] {
        require(t, "tensor");
        require(device, "device");
        *device = t->value.placement().ordinal();
    });
}

int pb_tensor_realize(const pb_tensor* t) {
    return guarded([&] {
        require(t, "tensor");
        t->value.realize();
    });
}

int pb_tensor_synchronize(const pb_tensor* t) {
    return guarded([&] {
        require(t, "tensor");
        t->value.synchronize();
    });
}

int pb_tensor_read(const pb_tensor* t, float* values, size_t count) {
    return guarded([&] {
        require(t, "tensor");
        if (count != t->value.numel())
            throw std::invalid_argument("host buffer size does not match tensor");
        if (count == 0) return;
        require(values, "values");
        auto storage = porch::tensor_access::storage(t->value);
        {
            std::scoped_lock lock{storage->host_mutex};
            if (storage->host_current) {
                std::memcpy(values, storage->host.data(), count * sizeof(float));
                return;
            }
        }
        if (storage->placeholder)
            throw std::runtime_error("placeholder tensors hold no values");
        porch::detail::make_contiguous(storage);
        porch::cuda_jit::copy_to_host(storage->device_values, std::span<float>(values, count));
    });
}

int pb_tensor_device_pointer(const pb_tensor* t, uint64_t* pointer, size_t* bytes) {
    return guarded([&] {
        require(t, "tensor");
        const auto& b = t->value.device_data();
        const auto& st = porch::cuda_jit::buffer_access::state(b);
        if (pointer) *pointer = st ? st->ptr : 0;
        if (bytes) *bytes = b.size_bytes();
    });
}

int pb_tensor_index(const pb_tensor* t, const pb_index* indices, size_t count, pb_expr** out) {
    return guarded([&] {
        require(t, "tensor");
        require(out, "out");
        if (count != 0) require(indices, "indices");
        std::vector<porch::tensor_index> idx;
        idx.reserve(count);
        for (size_t i = 0; i < count; ++i) {
            const pb_index& x = indices[i];
            switch (x.kind) {
                case PB_INDEX: idx.emplace_back(porch::index_t{x.index}); break;
                case PB_SLICE: idx.emplace_back(porch::slice{x.start, x.stop, x.step}); break;
                case PB_ALL: idx.emplace_back(porch::all); break;
                default: throw std::invalid_argument("unknown tensor index kind");
            }
        }
        // operator[] takes an initializer_list; forward a runtime-sized list.
        porch::tensor_expr result = [&]() -> porch::tensor_expr {
            switch (idx.size()) {
                case 0: return t->value[{}];
                case 1: return t->value[{idx[0]}];
                case 2: return t->value[{idx[0], idx[1]}];
                case 3: return t->value[{idx[0], idx[1], idx[2]}];
                case 4: return t->value[{idx[0], idx[1], idx[2], idx[3]}];
                case 5: return t->value[{idx[0], idx[1], idx[2], idx[3], idx[4]}];
                case 6: return t->value[{idx[0], idx[1], idx[2], idx[3], idx[4], idx[5]}];
                case 7: return t->value[{idx[0], idx[1], idx[2], idx[3], idx[4], idx[5], idx[6]}];
                case 8:
                    return t->value[{idx[0], idx[1], idx[2], idx[3], idx[4], idx[5], idx[6], idx[7]}];
                default: throw std::invalid_argument("too many tensor indices");
            }
        }();
        *out = wrap(std::move(result));
    });
}

int pb_expr_from_tensor(const pb_tensor* t, pb_expr** out) {
    return guarded([&] {
        require(t, "tensor");
        require(out, "out");
        *out = wrap(porch::tensor_expr{t->value});
    });
}

int pb_expr_scalar(float value, pb_expr** out) {
    return guarded([&] {
        require(out, "out");
        *out = wrap(porch::tensor_expr{value});
    });
}

void pb_expr_release(pb_expr* e) { delete e; }

int pb_expr_binary(int op, const pb_expr* lhs, const pb_expr* rhs, pb_expr** out) {
    return guarded([&] {
        require(lhs, "lhs");
        require(rhs, "rhs");
        require(out, "out");
        const porch::tensor_expr& l = lhs->value;
        const porch::tensor_expr& r = rhs->value;
        switch (op) {
            case PB_ADD: *out = wrap(l + r); break;
            case PB_SUBTRACT: *out = wrap(l - r); break;
            case PB_MULTIPLY: *out = wrap(l * r); break;
            case PB_DIVIDE: *out = wrap(l / r); break;
            case PB_MAXIMUM: *out = wrap(porch::maximum(l, r)); break;
            case PB_MINIMUM: *out = wrap(porch::minimum(l, r)); break;
            case PB_MATMUL: *out = wrap(porch::matmul(l, r)); break;
            default: throw std::invalid_argument("unknown binary op");
        }
    });
}

int pb_expr_unary(int op, const pb_expr* value, pb_expr** out) {
    return guarded([&] {
        require(value, "value");
        require(out, "out");
        const porch::tensor_expr& v = value->value;
        switch (op) {
            case PB_EXP: *out = wrap(porch::exp(v)); break;
            case PB_RECIPROCAL: *out = wrap(porch::reciprocal(v)); break;
            case PB_TRANSPOSE: *out = wrap(porch::transpose(v)); break;
            case PB_RELU: *out = wrap(porch::relu(v)); break;
            case PB_LOGISTIC: *out = wrap(porch::logistic(v)); break;
            default: throw std::invalid_argument("unknown unary op");
        }
    });
}

int pb_expr_reshape(const pb_expr* value, const int64_t* shape, size_t rank, pb_expr** out) {
    return guarded([&] {
        require(value, "value");
        require(out, "out");
        *out = wrap(porch::reshape(value->value, shape_of(shape, rank)));
    });
}

int pb_expr_broadcast(const pb_expr* value, const int64_t* shape, size_t rank, pb_expr** out) {
    return guarded([&] {
        require(value, "value");
        require(out, "out");
        *out = wrap(porch::broadcast_to(value->value, shape_of(shape, rank)));
    });
}

int pb_expr_unsqueeze(const pb_expr* value, size_t axis, pb_expr** out) {
    return guarded([&] {
        require(value, "value");
        require(out, "out");
        *out = wrap(porch::unsqueeze(value->value, axis));
    });
}

int pb_test_gemm_stall(int enable) {
    return guarded([&] { porch::detail::set_test_gemm_stall(enable != 0); });
}

int pb_expr_batched_matmul(const pb_expr* lhs, const pb_expr* rhs, pb_expr** out) {
    return guarded([&] {
        require(lhs, "lhs");
        require(rhs, "rhs");
        require(out, "out");
        auto n = std::make_shared<porch::tensor_expr::node>();
        n->kind = porch::detail::expr_kind::batched_matmul;
        n->lhs = porch::expr_access::root(lhs->value);
        n->rhs = porch::expr_access::root(rhs->value);
        porch::tensor_expr e = porch::expr_access::make(std::move(n));
        (void)porch::detail::infer(*porch::expr_access::root(e));
        *out = wrap(std::move(e));
    });
}

int pb_expr_permute(const pb_expr* value, const int64_t* perm, size_t rank, pb_expr** out) {
    return guarded([&] {
        require(value, "value");
        require(out, "out");
        if (rank != 0) require(perm, "perm");
        auto n = std::make_shared<porch::tensor_expr::node>();
        n->kind = porch::detail::expr_kind::permute;
        n->lhs = porch::expr_access::root(value->value);
        n->shape.assign(perm, perm + rank);
        porch::tensor_expr e = porch::expr_access::make(std::move(n));
        (void)porch::detail::infer(*porch::expr_access::root(e)); // validates now, as the builders do
        *out = wrap(std::move(e));
    });
}

int pb_expr_concat(const pb_expr* lhs, const pb_expr* rhs, size_t axis, pb_expr** out) {
    return guarded([&] {
        require(lhs, "lhs");
        require(rhs, "rhs");
        require(out, "out");
        *out = wrap(porch::concat(lhs->value, rhs->value, axis));
    });
}

int pb_expr_reduce(int op, const pb_expr* value, size_t axis, int keepdim, pb_expr** out) {
    return guarded([&] {
        require(value, "value");
        require(out, "out");
        if (op == PB_SUM)
            *out = wrap(porch::sum(value->value, axis, keepdim != 0));
        else if (op == PB_MAX)
            *out = wrap(porch::max(value->value, axis, keepdim != 0));
        else
            throw std::invalid_argument("unknown reduction op");
    });
}

int pb_expr_softmax(const pb_expr* value, size_t axis, pb_expr** out) {
    return guarded([&] {
        require(value, "value");
        require(out, "out");
        *out = wrap(porch::softmax(value->value, axis));
    });
}

int pb_expr_shape(const pb_expr* e, int64_t* shape, size_t capacity, size_t* rank) {
    return guarded([&] {
        require(e, "expr");
        const std::vector<porch::index_t> s = e->value.shape();
        if (rank) *rank = s.size();
        for (size_t i = 0; i < s.size() && i < capacity; ++i) shape[i] = s[i];
    });
}

int pb_expr_to_tensor(const pb_expr* e, pb_tensor** out) {
    return guarded([&] {
        require(e, "expr");
        require(out, "out");
        *out = wrap(static_cast<porch::tensor>(e->value));
    });
}

int pb_materialize(const pb_expr* e, pb_tensor** out) {
    return guarded([&] {
        require(e, "expr");
        require(out, "out");
        *out = wrap(porch::materialize(e->value));
    });
}

int pb_expr_describe(const pb_expr* e, int with_source, char* text, size_t capacity,
                     size_t* needed) {
    return guarded([&] {
        require(e, "expr");
        const std::string s =
            porch::detail::describe_plan(*porch::expr_access::root(e->value), with_source != 0);
        if (needed) *needed = s.size() + 1;
        if (text != nullptr && capacity > 0) {
            const size_t n = std::min(s.size(), capacity - 1);
            std::memcpy(text, s.data(), n);
            text[n] = '\0';
        }
    });
}

int pb_host_alloc(size_t bytes, void** pointer) {
    return guarded([&] {
        require(pointer, "pointer");
        porch::detail::check(pbrt_host_alloc(bytes, pointer));
    });
}

int pb_host_free(void* pointer) {
    return guarded([&] { porch::detail::check(pbrt_host_free(pointer)); });
}

namespace {
    struct device_timer {
        int device;
        pbrt_event start;
        pbrt_event stop;
        std::shared_ptr<porch::detail::stream_ref> stream;
    };
} // namespace

int pb_timer_begin(int device, void** timer) {
    return guarded([&] {
        require(timer, "timer");
        auto* t = new device_timer{device, nullptr, nullptr, porch::detail::current_stream(device)};
        porch::detail::check(pbrt_event_create(device, 1, &t->start));
        porch::detail::check(pbrt_event_create(device, 1, &t->stop));
        porch::detail::check(pbrt_event_record(device, t->start, t->stream->stream));
        *timer = t;
    });
}

int pb_timer_end(void* timer, float* milliseconds) {
    return guarded([&] {
        require(timer, "timer");
        auto* t = static_cast<device_timer*>(timer);
        std::unique_ptr<device_timer> owner{t};
        porch::detail::check(pbrt_event_record(t->device, t->stop, t->stream->stream));
        porch::detail::check(pbrt_event_synchronize(t->device, t->stop));
        float ms = 0.0F;
        porch::detail::check(pbrt_event_elapsed_ms(t->start, t->stop, &ms));
        (void)pbrt_event_destroy(t->device, t->start);
        (void)pbrt_event_destroy(t->device, t->stop);
        if (milliseconds) *milliseconds = ms;
    });
}

int pb_device_synchronize(int device) {
    return guarded([&] {
        auto s = porch::detail::current_stream(device);
        porch::detail::check(pbrt_stream_synchronize(device, s->stream));
        int code = 0;
        porch::detail::check(pbrt_error_check(device, s->stream, &code));
    });
}

uint64_t pb_launch_count(void) { return pbrt_launch_count(); }

int pb_empty_cache(int device, size_t* released) {
    return guarded([&] {
        const size_t n = porch::detail::release_cached_blocks(device);
        if (released) *released = n;
    });
}

int pb_host_profile_enable(int enable) {
    return guarded([&] { porch::detail::host_profile_enable(enable != 0); });
}

int pb_host_profile_read(char* text, size_t capacity) {
    return guarded([&] {
        const std::string s = porch::detail::host_profile_read();
        if (text != nullptr && capacity > 0) {
            const size_t n = std::min(s.size(), capacity - 1);
            std::memcpy(text, s.data(), n);
            text[n] = '\0';
        }
    });
}

int pb_comm_unique_id(char id[128]) {
    return guarded([&] {
        require(id, "id");
        porch::detail::check(pbrt_nccl_unique_id(id));
    });
}

int pb_comm_init(int nranks, const char id[128], int rank, int device, double timeout_s,
                 pb_comm** out) {
    return guarded([&] {
        require(id, "id");
        require(out, "out");
        *out = nullptr;
        auto c = porch::detail::make_communicator(nranks, id, rank, device, timeout_s);
        *out = new pb_comm_s{std::move(c)};
    });
}

int pb_comm_info(const pb_comm* comm, int* rank, int* nranks, int* device) {
    return guarded([&] {
        require(comm, "communicator");
        if (rank) *rank = comm->value->rank;
        if (nranks) *nranks = comm->value->nranks;
        if (device) *device = comm->value->device;
    });
}

int pb_comm_set_timeout(pb_comm* comm, double timeout_s) {
    return guarded([&] {
        require(comm, "communicator");
        if (!(timeout_s > 0.0)) throw std::invalid_argument("timeout must be positive");
        porch::detail::check(pbrt_nccl_set_timeout(comm->value->comm, timeout_s));
        comm->value->timeout_s = timeout_s;
    });
}

int pb_comm_abort(pb_comm* comm) {
    return guarded([&] {
        require(comm, "communicator");
        porch::detail::abort_communicator(*comm->value);
    });
}

int pb_comm_release(pb_comm* comm) {
    return guarded([&] { delete comm; });
}

int pb_row_block(int64_t rows, int rank, int nranks, int64_t* begin, int64_t* end) {
    return guarded([&] {
        const auto [b, e] = porch::detail::row_block(rows, rank, nranks);
        if (begin) *begin = b;
        if (end) *end = e;
    });
}

int pb_allgather_rows(pb_comm* comm, const pb_tensor* shard, int64_t total_rows,
                      pb_tensor** out) {
    return guarded([&] {
        require(comm, "communicator");
        require(shard, "shard");
        require(out, "out");
        *out = nullptr;
        *out = wrap(porch::detail::allgather_rows(*comm->value, shard->value, total_rows));
    });
}

int pb_allgather_rows_async(pb_comm* comm, const pb_tensor* shard, int64_t total_rows,
                            pb_tensor** out) {
    return guarded([&] {
        require(comm, "communicator");
        require(shard, "shard");
        require(out, "out");
        *out = nullptr;
        *out = wrap(porch::detail::allgather_rows(*comm->value, shard->value, total_rows, true));
    });
}

int pb_comm_wait(pb_comm* comm) {
    return guarded([&] {
        require(comm, "communicator");
        porch::detail::wait_communicator(*comm->value);
    });
}

int pb_profile_enable(int enable) {
    return guarded([&] { porch::detail::check(pbrt_profile_enable(enable)); });
}

int pb_profile_read(char* text, size_t capacity) {
    return guarded([&] { porch::detail::check(pbrt_profile_read(text, capacity)); });
}

} // extern "C"
