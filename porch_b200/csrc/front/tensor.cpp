// porch tensor front-end: handles, layouts, slicing, the lazy IR builders and
// shape inference. Public behaviour follows the reference
// (src/tensor.cpp:1081-1513); the lowering behind materialize() lives in
// graph.cpp / lower.cpp.
#include "detail.hpp"

#include "porch/ops.hpp"

#include <algorithm>
#include <stdexcept>

namespace porch {

    // ------------------------------------------------------------- state --
    struct tensor::state {
        struct lazy_t {
            std::shared_ptr<const tensor_expr::node> expression;
            std::once_flag once;
            std::shared_ptr<detail::realized_storage> result;
            std::atomic<bool> done{false};
        };

        state(tensor_layout l, device p) : layout(std::move(l)), placement(p) {}

        std::shared_ptr<detail::realized_storage> storage() const {
            if (realized != nullptr) return realized;
            lazy_t& z = *lazy;
            std::call_once(z.once, [&] {
                tensor t = detail::materialize_graph(*z.expression);
                z.result = t.state_->realized;
                z.done.store(true, std::memory_order_release);
            });
            return z.result;
        }

        tensor_layout layout;
        device placement;
        std::shared_ptr<detail::realized_storage> realized;
        std::shared_ptr<lazy_t> lazy;
    };

    namespace detail {

        const char* kind_name(expr_kind kind) {
            switch (kind) {
                case expr_kind::input: return "input";
                case expr_kind::scalar: return "scalar";
                case expr_kind::add: return "add";
                case expr_kind::subtract: return "subtract";
                case expr_kind::multiply: return "multiply";
                case expr_kind::divide: return "divide";
                case expr_kind::matmul: return "matmul";
                case expr_kind::slice: return "slice";
                case expr_kind::reshape: return "reshape";
                case expr_kind::unsqueeze: return "unsqueeze";
                case expr_kind::transpose: return "transpose";
                case expr_kind::broadcast: return "broadcast";
                case expr_kind::concat: return "concat";
                case expr_kind::sum: return "sum";
                case expr_kind::max: return "max";
                case expr_kind::maximum: return "maximum";
                case expr_kind::minimum: return "minimum";
                case expr_kind::exp: return "exp";
                case expr_kind::reciprocal: return "reciprocal";
                case expr_kind::permute: return "permute";
                case expr_kind::batched_matmul: return "batched_matmul";
            }
            return "?";
        }

        size_t checked_numel(std::span<const index_t> shape) {
            size_t count = 1;
            for (const index_t extent : shape) {
                if (extent < 0)
                    throw std::invalid_argument("tensor shape extents must be non-negative");
                count *= static_cast<size_t>(extent);
            }
            return count;
        }

        int checked_ordinal(int ordinal, int count) {
            if (ordinal < 0)
                throw std::invalid_argument("CUDA device ordinal must be non-negative");
            // An ordinal with no GPU behind it keeps the reference's meaning
            // (metadata; the work runs on device 0, src/cuda_jit.cpp:446-450):
            // its own tests build device{1} tensors on one GPU. It never
            // lands on another present GPU.
            return ordinal < count ? ordinal : 0;
        }

        std::vector<index_t> contiguous_strides(std::span<const index_t> shape) {
            std::vector<index_t> strides(shape.size(), 1);
            index_t stride = 1;
            for (size_t i = shape.size(); i > 0; --i) {
                strides[i - 1] = stride;
                stride *= shape[i - 1];
            }
            return strides;
        }

        namespace {
            bool contiguous_layout(std::span<const index_t> shape,
                                   std::span<const index_t> strides) {
                if (shape.size() != strides.size()) return false;
                index_t expected = 1;
                for (size_t i = shape.size(); i > 0; --i) {
                    if (strides[i - 1] != expected) return false;
                    expected *= shape[i - 1];
                }
                return true;
            }

            index_t normalize_index(index_t index, index_t extent) {
                if (index < 0) index += extent;
                if (index < 0 || index >= extent)
                    throw std::out_of_range("tensor index is out of bounds");
                return index;
            }

            index_t normalize_endpoint(index_t index, index_t extent) {
                if (index < 0) index += extent;
                if (index < 0) return 0;
                if (index > extent) return extent;
                return index;
            }

            size_t slice_length(index_t start, index_t stop, index_t step) {
                if (step <= 0)
                    throw std::invalid_argument("tensor slice step must be positive");
                if (stop <= start) return 0;
                return static_cast<size_t>((stop - start + step - 1) / step);
            }

            std::vector<index_t> reduced_shape(std::span<const index_t> shape, size_t axis,
                                               bool keepdim) {
                if (keepdim) {
                    std::vector<index_t> r{shape.begin(), shape.end()};
                    r[axis] = 1;
                    return r;
                }
                std::vector<index_t> r;
                for (size_t d = 0; d < shape.size(); ++d)
                    if (d != axis) r.push_back(shape[d]);
                if (r.empty()) r.push_back(1);
                return r;
            }

            struct infer_context {
                bool initialized = false;
                device placement{};
            };

            void record_device(infer_context& c, device p) {
                if (!c.initialized) {
                    c.placement = p;
                    c.initialized = true;
                } else if (c.placement != p) {
                    throw std::invalid_argument("tensor expression devices must match");
                }
            }

            struct info {
                std::vector<index_t> shape;
                bool scalar = true;
            };

            void require_same_shape(const info& l, const info& r) {
                if (l.scalar || r.scalar) return;
                if (std::ranges::equal(l.shape, r.shape)) return;
                throw std::invalid_argument("tensor expression shapes must match");
            }

            void require_axis(size_t axis, size_t rank, const char* op) {
                if (axis >= rank)
                    throw std::invalid_argument(std::string{op} + " axis is out of bounds");
            }

            void require_broadcastable(std::span<const index_t> src,
                                       std::span<const index_t> dst) {
                if (src.size() > dst.size())
                    throw std::invalid_argument(
                        "broadcast target rank must be at least source rank");
                const size_t off = dst.size() - src.size();
                for (size_t d = 0; d < src.size(); ++d) {
                    if (src[d] != 1 && src[d] != dst[off + d])
                        throw std::invalid_argument("broadcast shapes are not compatible");
                }
            }

            info infer_rec(const tensor_expr::node& n, infer_context& c) {
                switch (n.kind) {
                    case expr_kind::input:
                        record_device(c, n.placement);
                        return {n.input_shape, false};
                    case expr_kind::scalar:
                        return {};
                    case expr_kind::add:
                    case expr_kind::subtract:
                    case expr_kind::multiply:
                    case expr_kind::divide:
                    case expr_kind::maximum:
                    case expr_kind::minimum: {
                        info l = infer_rec(*n.lhs, c);
                        info r = infer_rec(*n.rhs, c);
                        require_same_shape(l, r);
                        return l.scalar ? r : l;
                    }
                    case expr_kind::matmul: {
                        info l = infer_rec(*n.lhs, c);
                        info r = infer_rec(*n.rhs, c);
                        if (l.scalar || r.scalar)
                            throw std::invalid_argument("matmul operands must be tensors");
                        if (l.shape.size() != 2 || r.shape.size() != 2)
                            throw std::invalid_argument("matmul requires rank-2 tensors");
                        if (l.shape[1] != r.shape[0])
                            throw std::invalid_argument("matmul inner dimensions must match");
                        return {{l.shape[0], r.shape[1]}, false};
                    }
                    case expr_kind::batched_matmul: {
                        info l = infer_rec(*n.lhs, c);
                        info r = infer_rec(*n.rhs, c);
                        if (l.scalar || r.scalar)
                            throw std::invalid_argument("batched matmul operands must be tensors");
                        if (l.shape.size() != 3 || r.shape.size() != 3)
                            throw std::invalid_argument("batched matmul requires rank-3 tensors");
                        if (l.shape[0] != r.shape[0])
                            throw std::invalid_argument("batched matmul batch dimensions must match");
                        if (l.shape[2] != r.shape[1])
                            throw std::invalid_argument("batched matmul inner dimensions must match");
                        return {{l.shape[0], l.shape[1], r.shape[2]}, false};
                    }
                    case expr_kind::slice:
                        (void)infer_rec(*n.lhs, c);
                        return {n.slice_shape, false};
                    case expr_kind::reshape: {
                        info s = infer_rec(*n.lhs, c);
                        if (s.scalar)
                            throw std::invalid_argument("reshape operand must be a tensor");
                        if (checked_numel(s.shape) != checked_numel(n.shape))
                            throw std::invalid_argument(
                                "reshape must preserve tensor element count");
                        return {n.shape, false};
                    }
                    case expr_kind::unsqueeze: {
                        info s = infer_rec(*n.lhs, c);
                        if (s.scalar)
                            throw std::invalid_argument("unsqueeze operand must be a tensor");
                        if (n.axis > s.shape.size())
                            throw std::invalid_argument("unsqueeze axis is out of bounds");
                        std::vector<index_t> shape = s.shape;
                        shape.insert(shape.begin() + static_cast<ptrdiff_t>(n.axis), 1);
                        return {std::move(shape), false};
                    }
                    case expr_kind::permute: {
                        info s = infer_rec(*n.lhs, c);
                        if (s.scalar)
                            throw std::invalid_argument("permute operand must be a tensor");
                        if (n.shape.size() != s.shape.size())
                            throw std::invalid_argument("permutation length must equal the tensor rank");
                        std::vector<bool> seen(s.shape.size(), false);
                        std::vector<index_t> shape(s.shape.size());
                        for (size_t d = 0; d < n.shape.size(); ++d) {
                            const index_t p = n.shape[d];
                            if (p < 0 || static_cast<size_t>(p) >= s.shape.size() || seen[static_cast<size_t>(p)])
                                throw std::invalid_argument("permute needs a permutation of the tensor's axes");
                            seen[static_cast<size_t>(p)] = true;
                            shape[d] = s.shape[static_cast<size_t>(p)];
                        }
                        return {std::move(shape), false};
                    }
                    case expr_kind::transpose: {
                        info s = infer_rec(*n.lhs, c);
                        if (s.scalar)
                            throw std::invalid_argument("transpose operand must be a tensor");
                        if (s.shape.size() != 2)
                            throw std::invalid_argument(
                                "transpose currently requires a rank-2 tensor");
                        return {{s.shape[1], s.shape[0]}, false};
                    }
                    case expr_kind::broadcast: {
                        info s = infer_rec(*n.lhs, c);
                        if (s.scalar) return {n.shape, false};
                        require_broadcastable(s.shape, n.shape);
                        return {n.shape, false};
                    }
                    case expr_kind::concat: {
                        info l = infer_rec(*n.lhs, c);
                        info r = infer_rec(*n.rhs, c);
                        if (l.scalar || r.scalar)
                            throw std::invalid_argument("concat operands must be tensors");
                        if (l.shape.size() != r.shape.size())
                            throw std::invalid_argument(
                                "concat operands must have the same rank");
                        require_axis(n.axis, l.shape.size(), "concat");
                        std::vector<index_t> shape = l.shape;
                        for (size_t d = 0; d < shape.size(); ++d) {
                            if (d == n.axis) continue;
                            if (l.shape[d] != r.shape[d])
                                throw std::invalid_argument(
                                    "concat non-axis dimensions must match");
                        }
                        shape[n.axis] += r.shape[n.axis];
                        return {std::move(shape), false};
                    }
                    case expr_kind::sum:
                    case expr_kind::max: {
                        info s = infer_rec(*n.lhs, c);
                        if (s.scalar)
                            throw std::invalid_argument("reduction operand must be a tensor");
                        require_axis(n.axis, s.shape.size(), "reduction");
                        return {reduced_shape(s.shape, n.axis, n.keepdim), false};
                    }
                    case expr_kind::exp:
                    case expr_kind::reciprocal: {
                        info s = infer_rec(*n.lhs, c);
                        return s;
                    }
                }
                throw std::invalid_argument("unknown tensor expression node");
            }
        } // namespace

        shape_info infer(const tensor_expr::node& root) {
            infer_context c;
            info i = infer_rec(root, c);
            shape_info out;
            out.shape = std::move(i.shape);
            out.scalar = i.scalar;
            out.has_input = c.initialized;
            out.placement = c.placement;
            return out;
        }

        namespace {
            int physical_device(device placement) {
                int count = 0;
                check(pbrt_device_count(&count));
                // The reference treats the ordinal as metadata and always runs on
                // device 0 (src/cuda_jit.cpp:446-450). Here ordinals address real
                // devices; one that is not present runs on device 0.
                return checked_ordinal(placement.ordinal(), count);
            }
        } // namespace

        int device_for(device placement) { return physical_device(placement); }

    } // namespace detail

    // ----------------------------------------------------- tensor_index --
    tensor_index::tensor_index(index_t index) : kind_(kind::index), index_(index) {}
    tensor_index::tensor_index(slice range) : kind_(kind::slice), slice_(range) {}
    tensor_index::tensor_index(all_t) : kind_(kind::all) {}

    // ---------------------------------------------------- tensor_layout --
    tensor_layout::tensor_layout(std::vector<index_t> shape)
        : shape_(std::move(shape)), strides_(detail::contiguous_strides(shape_)) {
        (void)detail::checked_numel(shape_);
    }

    tensor_layout::tensor_layout(std::vector<index_t> shape, std::vector<index_t> strides,
                                 index_t storage_offset)
        : shape_(std::move(shape)), strides_(std::move(strides)),
          storage_offset_(storage_offset) {
        if (shape_.size() != strides_.size())
            throw std::invalid_argument("tensor layout rank mismatch");
        if (storage_offset_ < 0)
            throw std::invalid_argument("tensor layout offset must be non-negative");
        for (const index_t s : strides_)
            if (s < 0) throw std::invalid_argument("tensor layout strides must be non-negative");
        (void)detail::checked_numel(shape_);
    }

    std::span<const index_t> tensor_layout::shape() const noexcept { return shape_; }
    std::span<const index_t> tensor_layout::strides() const noexcept { return strides_; }
    index_t tensor_layout::storage_offset() const noexcept { return storage_offset_; }
    size_t tensor_layout::rank() const noexcept { return shape_.size(); }
    size_t tensor_layout::numel() const noexcept {
        size_t n = 1;
        for (const index_t e : shape_) n *= static_cast<size_t>(e);
        return n;
    }
    bool tensor_layout::is_contiguous() const noexcept {
        return storage_offset_ == 0 && detail::contiguous_layout(shape_, strides_);
    }

    // ------------------------------------------------------------ tensor --
    namespace detail {
        int device_for(device placement);
    }

    tensor::tensor(std::vector<index_t> shape, std::vector<float32_t> values,
                   device placement)
        : state_(std::make_shared<state>(tensor_layout{std::move(shape)}, placement)) {
        const size_t expected = state_->layout.numel();
        if (values.size() != expected)
            throw std::invalid_argument("tensor data size does not match shape");
        auto storage = std::make_shared<detail::realized_storage>();
        storage->count = expected;
        storage->device = detail::device_for(placement);
        auto stream = detail::current_stream(storage->device);
        storage->device_values =
            detail::allocate(storage->device, expected * sizeof(float32_t), stream);
        if (expected != 0) {
            auto& st = *cuda_jit::buffer_access::state(storage->device_values);
            detail::check(pbrt_memcpy_h2d_async(storage->device, st.ptr, values.data(),
                                                expected * sizeof(float32_t),
                                                stream->stream));
            // Pageable source: complete before returning (src/cuda_jit.cpp:711-734).
            detail::check(pbrt_stream_synchronize(storage->device, stream->stream));
        }
        storage->host = std::move(values);
        storage->host_current = true;
        state_->realized = std::move(storage);
    }

    tensor::tensor(std::vector<index_t> shape, std::vector<float32_t> values,
                   cuda_jit::device_buffer device_values, device placement)
        : tensor(std::move(shape), std::move(values), std::move(device_values), true,
                 placement) {}

    tensor::tensor(std::vector<index_t> shape, std::vector<float32_t> values,
                   cuda_jit::device_buffer device_values, bool host_current,
                   device placement)
        : tensor(tensor_layout{std::move(shape)}, std::move(values),
                 std::move(device_values), host_current, placement) {}

    tensor::tensor(tensor_layout layout, std::vector<float32_t> values,
                   cuda_jit::device_buffer device_values, bool host_current,
                   device placement)
        : state_(std::make_shared<state>(std::move(layout), placement)) {
        const size_t expected = state_->layout.numel();
        if (values.size() != expected)
            throw std::invalid_argument("tensor data size does not match shape");
        if (!state_->layout.is_contiguous())
            throw std::invalid_argument(
                "non-contiguous tensor storage is not implemented yet");
        if (device_values.size_bytes() < values.size() * sizeof(float32_t))
            throw std::invalid_argument("tensor device storage is too small");
        auto storage = std::make_shared<detail::realized_storage>();
        storage->count = expected;
        const auto& bst = cuda_jit::buffer_access::state(device_values);
        storage->device = bst ? bst->device : 0;
        storage->device_values = std::move(device_values);
        storage->host = std::move(values);
        storage->host_current = host_current;
        state_->realized = std::move(storage);
    }

    tensor::tensor(std::shared_ptr<state> handle) noexcept : state_(std::move(handle)) {}

    std::span<const index_t> tensor::shape() const noexcept { return state_->layout.shape(); }
    std::span<const index_t> tensor::strides() const noexcept {
        return state_->layout.strides();
    }
    const tensor_layout& tensor::layout() const noexcept { return state_->layout; }
    index_t tensor::storage_offset() const noexcept {
        return state_->layout.storage_offset();
    }
    bool tensor::is_contiguous() const noexcept { return state_->layout.is_contiguous(); }
    size_t tensor::rank() const noexcept { return state_->layout.rank(); }
    size_t tensor::numel() const noexcept { return state_->layout.numel(); }
    device tensor::placement() const noexcept { return state_->placement; }

    std::span<const float32_t> tensor::data() const {
        std::shared_ptr<detail::realized_storage> storage = state_->storage();
        detail::make_contiguous(storage);
        std::scoped_lock lock{storage->host_mutex};
        if (!storage->host_current) {
            if (storage->placeholder)
                throw std::runtime_error("placeholder tensors hold no values");
            storage->host.resize(storage->count);
            cuda_jit::copy_to_host(storage->device_values, storage->host);
            storage->host_current = true;
        }
        return storage->host;
    }

    std::vector<float32_t> tensor::cpu() const {
        const std::span<const float32_t> host = data();
        return {host.begin(), host.end()};
    }

    const cuda_jit::device_buffer& tensor::device_data() const {
        // The handle may be written through: contiguous values of its own,
        // and its live views copied out first.
        const std::shared_ptr<detail::realized_storage>& storage = state_->storage();
        detail::escape(storage);
        return storage->device_values;
    }

    const tensor& tensor::realize() const {
        ensure_materialized();
        return *this;
    }

    void tensor::synchronize() const {
        ensure_materialized();
        cuda_jit::synchronize();
    }

    void tensor::ensure_materialized() const { (void)state_->storage(); }

    tensor_expr tensor::operator[](std::initializer_list<tensor_index> indices) const {
        if (indices.size() > rank()) throw std::invalid_argument("too many tensor indices");
        std::vector<index_t> out_shape;
        std::vector<index_t> out_strides;
        index_t offset = storage_offset();
        size_t dim = 0;
        for (const tensor_index& index : indices) {
            const index_t extent = shape()[dim];
            const index_t stride = strides()[dim];
            switch (index.kind_) {
                case tensor_index::kind::index:
                    offset += detail::normalize_index(index.index_, extent) * stride;
                    break;
                case tensor_index::kind::slice: {
                    const index_t start = detail::normalize_endpoint(index.slice_.start, extent);
                    const index_t stop = detail::normalize_endpoint(index.slice_.stop, extent);
                    const size_t length = detail::slice_length(start, stop, index.slice_.step);
                    offset += start * stride;
                    out_shape.push_back(static_cast<index_t>(length));
                    out_strides.push_back(stride * index.slice_.step);
                    break;
                }
                case tensor_index::kind::all:
                    out_shape.push_back(extent);
                    out_strides.push_back(stride);
                    break;
            }
            ++dim;
        }
        for (; dim < rank(); ++dim) {
            out_shape.push_back(shape()[dim]);
            out_strides.push_back(strides()[dim]);
        }
        (void)detail::checked_numel(out_shape);
        auto n = std::make_shared<tensor_expr::node>();
        n->kind = detail::expr_kind::slice;
        n->lhs = tensor_expr{*this}.root_;
        n->slice_shape = std::move(out_shape);
        n->slice_strides = std::move(out_strides);
        n->slice_offset = offset;
        return tensor_expr{std::shared_ptr<const tensor_expr::node>(std::move(n))};
    }

    tensor_expr tensor::operator[](tensor_index index) const { return (*this)[{index}]; }

    // ------------------------------------------------------- tensor_expr --
    namespace {
        std::shared_ptr<const tensor_expr::node> input_node(
            const std::vector<index_t>& shape,
            std::shared_ptr<detail::realized_storage> storage, device placement
        ) {
            auto n = std::make_shared<tensor_expr::node>();
            n->kind = detail::expr_kind::input;
            n->storage = std::move(storage);
            n->input_shape = shape;
            n->placement = placement;
            return n;
        }
    } // namespace

    tensor_expr::tensor_expr(const tensor& value) {
        const auto& st = *value.state_;
        const std::vector<index_t> shape{st.layout.shape().begin(), st.layout.shape().end()};
        if (st.realized != nullptr) {
            root_ = input_node(shape, st.realized, st.placement);
        } else if (st.lazy->done.load(std::memory_order_acquire)) {
            // Already materialised: read the stored result instead of
            // re-inlining (and recomputing) the graph as src/tensor.cpp:1321-1326 does.
            root_ = input_node(shape, st.lazy->result, st.placement);
        } else {
            root_ = st.lazy->expression;
        }
    }

    tensor_expr::tensor_expr(float32_t value) {
        auto n = std::make_shared<tensor_expr::node>();
        n->kind = detail::expr_kind::scalar;
        n->scalar = value;
        root_ = std::move(n);
    }

    tensor_expr::tensor_expr(std::shared_ptr<const node> root) : root_(std::move(root)) {}

    tensor tensor_expr::eval() const { return materialize(*this); }

    std::vector<index_t> tensor_expr::shape() const {
        detail::shape_info i = detail::infer(*root_);
        if (i.scalar) return {};
        return i.shape;
    }

    size_t tensor_expr::rank() const { return shape().size(); }
    size_t tensor_expr::numel() const { return detail::checked_numel(shape()); }

    tensor_expr::operator tensor() const {
        detail::shape_info i = detail::infer(*root_);
        if (!i.has_input)
            throw std::invalid_argument("tensor expression must reference at least one tensor");
        if (i.scalar)
            throw std::invalid_argument("scalar expression cannot convert to a tensor");
        auto st = std::make_shared<tensor::state>(tensor_layout{std::move(i.shape)},
                                                  i.placement);
        st->lazy = std::make_shared<tensor::state::lazy_t>();
        st->lazy->expression = root_;
        return tensor{std::move(st)};
    }

    // --------------------------------------------------------- builders --
    tensor full(std::vector<index_t> shape, float32_t value, device placement) {
        const size_t count = detail::checked_numel(shape);
        return tensor{std::move(shape), std::vector<float32_t>(count, value), placement};
    }

    tensor zeros(std::vector<index_t> shape, device placement) {
        return full(std::move(shape), 0.0F, placement);
    }

    tensor add(const tensor& lhs, const tensor& rhs) {
        return materialize(tensor_expr{lhs} + tensor_expr{rhs});
    }
    tensor subtract(const tensor& lhs, const tensor& rhs) {
        return materialize(tensor_expr{lhs} - tensor_expr{rhs});
    }
    tensor multiply(const tensor& lhs, const tensor& rhs) {
        return materialize(tensor_expr{lhs} * tensor_expr{rhs});
    }
    tensor divide(const tensor& lhs, const tensor& rhs) {
        return materialize(tensor_expr{lhs} / tensor_expr{rhs});
    }

    tensor make_materialized_tensor(std::vector<index_t> shape, std::vector<float32_t> values,
                                    cuda_jit::device_buffer device_values, bool host_current,
                                    device placement) {
        return tensor{std::move(shape), std::move(values), std::move(device_values),
                      host_current, placement};
    }

    namespace {
        using node_ptr = std::shared_ptr<const tensor_expr::node>;
        node_ptr binary(detail::expr_kind k, node_ptr l, node_ptr r) {
            auto n = std::make_shared<tensor_expr::node>();
            n->kind = k;
            n->lhs = std::move(l);
            n->rhs = std::move(r);
            return n;
        }
        node_ptr unary(detail::expr_kind k, node_ptr v) { return binary(k, std::move(v), nullptr); }
        node_ptr shaped(detail::expr_kind k, node_ptr v, std::vector<index_t> shape) {
            auto n = std::make_shared<tensor_expr::node>();
            n->kind = k;
            n->lhs = std::move(v);
            n->shape = std::move(shape);
            return n;
        }
        node_ptr axis_node(detail::expr_kind k, node_ptr v, node_ptr r, size_t axis,
                           bool keepdim) {
            auto n = std::make_shared<tensor_expr::node>();
            n->kind = k;
            n->lhs = std::move(v);
            n->rhs = std::move(r);
            n->axis = axis;
            n->keepdim = keepdim;
            return n;
        }
    } // namespace

    tensor_expr matmul(tensor_expr lhs, tensor_expr rhs) {
        return tensor_expr{binary(detail::expr_kind::matmul, std::move(lhs.root_),
                                  std::move(rhs.root_))};
    }
    tensor_expr reshape(tensor_expr value, std::vector<index_t> shape) {
        return tensor_expr{shaped(detail::expr_kind::reshape, std::move(value.root_),
                                  std::move(shape))};
    }
    tensor_expr unsqueeze(tensor_expr value, size_t axis) {
        return tensor_expr{axis_node(detail::expr_kind::unsqueeze, std::move(value.root_),
                                     nullptr, axis, false)};
    }
    tensor_expr transpose(tensor_expr value) {
        return tensor_expr{unary(detail::expr_kind::transpose, std::move(value.root_))};
    }
    tensor_expr broadcast_to(tensor_expr value, std::vector<index_t> shape) {
        return tensor_expr{shaped(detail::expr_kind::broadcast, std::move(value.root_),
                                  std::move(shape))};
    }
    tensor_expr concat(tensor_expr lhs, tensor_expr rhs, size_t axis) {
        return tensor_expr{axis_node(detail::expr_kind::concat, std::move(lhs.root_),
                                     std::move(rhs.root_), axis, false)};
    }
    tensor_expr sum(tensor_expr value, size_t axis, bool keepdim) {
        return tensor_expr{axis_node(detail::expr_kind::sum, std::move(value.root_), nullptr,
                                     axis, keepdim)};
    }
    tensor_expr max(tensor_expr value, size_t axis, bool keepdim) {
        return tensor_expr{axis_node(detail::expr_kind::max, std::move(value.root_), nullptr,
                                     axis, keepdim)};
    }
    tensor_expr maximum(tensor_expr lhs, tensor_expr rhs) {
        return tensor_expr{binary(detail::expr_kind::maximum, std::move(lhs.root_),
                                  std::move(rhs.root_))};
    }
    tensor_expr minimum(tensor_expr lhs, tensor_expr rhs) {
        return tensor_expr{binary(detail::expr_kind::minimum, std::move(lhs.root_),
                                  std::move(rhs.root_))};
    }
    tensor_expr exp(tensor_expr value) {
        return tensor_expr{unary(detail::expr_kind::exp, std::move(value.root_))};
    }
    tensor_expr reciprocal(tensor_expr value) {
        return tensor_expr{unary(detail::expr_kind::reciprocal, std::move(value.root_))};
    }

    tensor materialize(const tensor_expr& expression) {
        return detail::materialize_graph(*expression.root_);
    }

    tensor_expr operator+(tensor_expr lhs, tensor_expr rhs) {
        return tensor_expr{binary(detail::expr_kind::add, std::move(lhs.root_),
                                  std::move(rhs.root_))};
    }
    tensor_expr operator-(tensor_expr lhs, tensor_expr rhs) {
        return tensor_expr{binary(detail::expr_kind::subtract, std::move(lhs.root_),
                                  std::move(rhs.root_))};
    }
    tensor_expr operator*(tensor_expr lhs, tensor_expr rhs) {
        return tensor_expr{binary(detail::expr_kind::multiply, std::move(lhs.root_),
                                  std::move(rhs.root_))};
    }
    tensor_expr operator/(tensor_expr lhs, tensor_expr rhs) {
        return tensor_expr{binary(detail::expr_kind::divide, std::move(lhs.root_),
                                  std::move(rhs.root_))};
    }

    // ---------------------------------------------------- tensor_access --
    tensor tensor_access::from_storage(std::vector<index_t> shape,
                                       std::shared_ptr<detail::realized_storage> storage,
                                       device placement) {
        auto st = std::make_shared<tensor::state>(tensor_layout{std::move(shape)}, placement);
        st->realized = std::move(storage);
        return tensor{std::move(st)};
    }

    std::shared_ptr<detail::realized_storage> tensor_access::storage(const tensor& t) {
        return t.state_->storage();
    }

    bool tensor_access::is_lazy(const tensor& t) { return t.state_->realized == nullptr; }

    tensor tensor_access::placeholder(std::vector<index_t> shape, device placement) {
        auto storage = std::make_shared<detail::realized_storage>();
        storage->count = detail::checked_numel(shape);
        storage->device = placement.ordinal();
        storage->placeholder = true;
        return from_storage(std::move(shape), std::move(storage), placement);
    }

    // -------------------------------------------------------------- ops --
    // Same graph formulas as the reference (src/ops.cpp:5-18); the lowering
    // recognises the softmax shape and runs it as one fused row kernel.
    tensor_expr relu(tensor_expr value) { return maximum(value, 0.0F); }

    tensor_expr softmax(tensor_expr value, size_t axis) {
        const std::vector<index_t> output_shape = value.shape();
        tensor_expr shifted = value - broadcast_to(max(value, axis, true), output_shape);
        tensor_expr numerator = exp(shifted);
        return numerator / broadcast_to(sum(numerator, axis, true), output_shape);
    }

    tensor_expr logistic(tensor_expr value) { return reciprocal(1.0F + exp(0.0F - value)); }

} // namespace porch
