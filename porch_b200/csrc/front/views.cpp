// Strided views of realised storage.
//
// The reference realises every graph into a new contiguous buffer
// (src/tensor.cpp:1002-1066) and refuses non-contiguous storage
// (src/tensor.cpp:1193-1197). Here a graph that only moves data of one
// realised tensor -- slices, transposes, internal permutes, unsqueezes and
// reshapes of contiguous layouts -- is realised as a strided view of that
// tensor's device values: no kernel runs, and later graphs read the view in
// place through the same affine index maps a slice uses (the canonical graph
// turns the view into slice(input(base), layout)). Values are copied out
// into a contiguous buffer only when someone asks for them (data(), cpu(),
// device_data(), a gather), or before a raw handle to the base's values is
// handed out, so a view keeps the snapshot semantics of the reference's
// copy.
#include "plan.hpp"

#include <stdexcept>

namespace porch::detail {

    tensor materialize_graph_copy(const tensor_expr::node& root);

    bool view_of(realized_storage& s, std::shared_ptr<realized_storage>& base, strided_layout& layout) {
        std::scoped_lock lock{s.view_mutex};
        if (!s.view_base) return false;
        base = s.view_base;
        layout.shape = s.view_shape;
        layout.strides = s.view_strides;
        layout.offset = s.view_offset;
        return true;
    }

    bool compose_slice(const strided_layout& src, index_t offset, const std::vector<index_t>& strides,
                       const std::vector<index_t>& shape, strided_layout& out) {
        // The slice addresses src's logical (contiguous) index space:
        // L = offset + sum_j i_j strides[j]. Unravel the offset into src
        // coordinates, then give every sliced dimension the src dimension
        // its stride steps along, provided no coordinate carries over.
        const size_t R = src.shape.size();
        const std::vector<index_t> cs = contiguous_strides(src.shape);
        index_t numel = 1;
        for (index_t e : src.shape) numel *= e;
        if (numel <= 0 || offset < 0 || offset >= numel) return false;
        std::vector<index_t> c(R, 0), reach(R, 0);
        index_t rem = offset;
        for (size_t d = 0; d < R; ++d) {
            c[d] = rem / cs[d];
            rem %= cs[d];
        }
        out.shape = shape;
        out.strides.assign(shape.size(), 0);
        out.offset = src.offset;
        for (size_t d = 0; d < R; ++d) out.offset += c[d] * src.strides[d];
        for (size_t j = 0; j < shape.size(); ++j) {
            if (shape[j] <= 1 || strides[j] == 0) continue;
            if (strides[j] < 0) return false;
            size_t d = 0;
            while (d < R && (strides[j] % cs[d] != 0 || strides[j] / cs[d] >= src.shape[d])) ++d;
            if (d == R) return false;
            const index_t m = strides[j] / cs[d];
            reach[d] += m * (shape[j] - 1);
            out.strides[j] = m * src.strides[d];
        }
        for (size_t d = 0; d < R; ++d)
            if (c[d] + reach[d] >= src.shape[d]) return false;
        return true;
    }

    bool pure_view(const graph& g, int& slot, strided_layout& layout) {
        // The chain of data-movement nodes from the root down to one input.
        std::vector<int> chain;
        int id = g.root;
        for (;;) {
            const gnode& n = g.nodes[static_cast<size_t>(id)];
            if (n.kind == expr_kind::input) break;
            if (n.kind != expr_kind::slice && n.kind != expr_kind::transpose && n.kind != expr_kind::unsqueeze &&
                n.kind != expr_kind::reshape && n.kind != expr_kind::permute)
                return false;
            chain.push_back(id);
            id = n.a;
        }
        if (chain.empty()) return false; // the input itself: nothing to view
        const gnode& in = g.nodes[static_cast<size_t>(id)];
        slot = in.slot;
        strided_layout l;
        l.shape = in.shape;
        l.strides = contiguous_strides(in.shape);
        l.offset = 0;
        for (size_t i = chain.size(); i > 0; --i) {
            const gnode& n = g.nodes[static_cast<size_t>(chain[i - 1])];
            strided_layout next;
            switch (n.kind) {
                case expr_kind::slice:
                    if (!compose_slice(l, n.p_offset, n.p_strides, n.p_shape, next)) return false;
                    break;
                case expr_kind::transpose:
                    next.shape = {l.shape[1], l.shape[0]};
                    next.strides = {l.strides[1], l.strides[0]};
                    next.offset = l.offset;
                    break;
                case expr_kind::permute:
                    next.offset = l.offset;
                    for (index_t p : n.p_shape) {
                        next.shape.push_back(l.shape[static_cast<size_t>(p)]);
                        next.strides.push_back(l.strides[static_cast<size_t>(p)]);
                    }
                    break;
                case expr_kind::unsqueeze:
                    next = l;
                    next.shape.insert(next.shape.begin() + static_cast<ptrdiff_t>(n.axis), 1);
                    next.strides.insert(next.strides.begin() + static_cast<ptrdiff_t>(n.axis), 0);
                    break;
                case expr_kind::reshape:
                    // Only a contiguous layout reshapes without a copy here.
                    if (l.strides != contiguous_strides(l.shape)) return false;
                    next.shape = n.p_shape;
                    next.strides = contiguous_strides(n.p_shape);
                    next.offset = l.offset;
                    break;
                default:
                    return false;
            }
            l = std::move(next);
        }
        layout = std::move(l);
        return true;
    }

    bool make_view(const std::shared_ptr<realized_storage>& base, const strided_layout& layout,
                   const std::shared_ptr<realized_storage>& view) {
        std::scoped_lock lock{base->view_mutex};
        if (base->escaped || base->placeholder || base->view_base) return false;
        view->view_base = base;
        view->view_shape = layout.shape;
        view->view_strides = layout.strides;
        view->view_offset = layout.offset;
        view->device_values = base->device_values;
        // Forget views that no longer exist, then record this one.
        std::erase_if(base->views, [](const std::weak_ptr<realized_storage>& w) { return w.expired(); });
        base->views.push_back(view);
        return true;
    }

    void make_contiguous(const std::shared_ptr<realized_storage>& s) {
        std::shared_ptr<realized_storage> base;
        strided_layout l;
        if (!view_of(*s, base, l)) return;
        auto in = std::make_shared<tensor_expr::node>();
        in->kind = expr_kind::input;
        in->storage = base;
        in->input_shape = {static_cast<index_t>(base->count)};
        in->placement = device{base->device};
        auto sl = std::make_shared<tensor_expr::node>();
        sl->kind = expr_kind::slice;
        sl->lhs = in;
        sl->slice_shape = l.shape;
        sl->slice_strides = l.strides;
        sl->slice_offset = l.offset;
        tensor t = materialize_graph_copy(*sl);
        std::shared_ptr<realized_storage> r = tensor_access::storage(t);
        std::scoped_lock lock{s->view_mutex};
        if (!s->view_base) return; // another thread copied it out first
        s->device_values = r->device_values;
        s->view_base.reset();
        s->layout_epoch.fetch_add(1, std::memory_order_acq_rel);
    }

    void escape(const std::shared_ptr<realized_storage>& s) {
        make_contiguous(s);
        // A raw handle carries no stream order: an upload still in flight
        // (pb_tensor_create_async) completes first.
        if (const auto& st = cuda_jit::buffer_access::state(s->device_values); st && st->ready != nullptr)
            check(pbrt_event_synchronize(st->device, st->ready));
        std::vector<std::shared_ptr<realized_storage>> live;
        {
            std::scoped_lock lock{s->view_mutex};
            s->escaped = true;
            s->splits.clear(); // the values may now be written
            for (auto& w : s->views)
                if (auto v = w.lock()) live.push_back(std::move(v));
            s->views.clear();
        }
        for (auto& v : live) make_contiguous(v);
        if (!live.empty()) {
            // The copies run on this thread's stream; whatever the caller
            // does with the handle next (its own stream, a raw pointer) must
            // find them done.
            auto stream = current_stream(s->device);
            check(pbrt_stream_synchronize(s->device, stream->stream));
        }
    }

} // namespace porch::detail
