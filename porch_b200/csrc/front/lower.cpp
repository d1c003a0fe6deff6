// Lowering of canonical graphs to sm_100a kernel templates.
//
// Reference counterpart: lower_nested_reductions + emit_expression +
// fused_kernel_source / fused_reduction_kernel_source (src/tensor.cpp:498-989).
// The reference turns every graph into one of two string templates (one
// thread per output element with 64-bit div/mod index chains, or one
// 256-thread block per reduced output) and materialises every non-root
// reduction separately.
//
// Here a graph is lowered to a short list of kernels chosen from templates:
//  - elementwise/view graphs: every leaf access is analysed as an affine map
//    of the output coordinates. concat splits the output into boxes, each
//    box with its own maps. A box whose leaves stream along the innermost
//    output dimension runs the ROW schedule (128-bit loads/stores, 4 vectors
//    per thread in flight); a box with a transposed leaf runs the TILE
//    schedule (64x64 tiles staged through XOR-swizzled shared memory so
//    both global reads and writes stay coalesced and shared memory is
//    bank-conflict free). Graphs that are not affine (reshape of an
//    unaligned slice and the like) fall back to a per-element gather kernel.
//  - sum/max along an axis, the operand expression fused in: a warp per row
//    (contiguous axis), a CTA per row for few long rows, 128-column tiles
//    for the second-to-last axis of an operand with aligned rows (axis 0
//    of [A, C], the middle axis of [B, A, C]), else a thread per
//    output (strided axis); dimensions after the axis that every load
//    walks contiguously merge first; tall inputs split into row chunks whose
//    partials a second pass combines in a fixed order.
//  - the ops.hpp softmax shape over the last axis: one row kernel, not four
//    kernels -- rows held in registers (one HBM read and one write); for few
//    long rows a thread-block cluster per row exchanging max and sum through
//    distributed shared memory; otherwise an online max/sum pass and a write
//    pass.
//  - matmul: the pending elementwise consumer is fused as the epilogue.
//    Large shapes use the tcgen05 3xTF32 path (gemm_tc.cpp); the rest
//    use a tiled CUDA-core kernel whose per-output FMA chain runs in k order,
//    the same order as the reference's generated loop.
#include "plan.hpp"

#include "lower.hpp"

#include <algorithm>
#include <cinttypes>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <sstream>
#include <stdexcept>

namespace porch::detail {

    const std::vector<std::string>& kernel_options() {
        static const std::vector<std::string> options = {
            "--gpu-architecture=sm_100a", "-std=c++17", "--fmad=false",
            "--prec-div=true", "--prec-sqrt=true", "--ftz=false", "-lineinfo",
            "--diag-suppress=177", "-DPB_NVRTC=1"};
        return options;
    }

    std::string float_literal(float v) {
        uint32_t bits = 0;
        std::memcpy(&bits, &v, 4);
        char buf[64];
        if (std::isfinite(v)) {
            std::snprintf(buf, sizeof buf, "%af", static_cast<double>(v));
        } else {
            std::snprintf(buf, sizeof buf, "__int_as_float(0x%08xu)", bits);
        }
        return buf;
    }

    const char* kernel_prelude() {
        return R"PB(
typedef unsigned int pb_u32;
typedef unsigned long long pb_u64;
#define PB_NEG_FLT_MAX (-3.4028234663852886e+38f)
static __device__ __forceinline__ float4 pb_ld4(const float* p) {
    return __ldg(reinterpret_cast<const float4*>(p));
}
static __device__ __forceinline__ float pb_ld(const float* p) { return __ldg(p); }
static __device__ __forceinline__ void pb_st4(float* p, float4 v) {
    *reinterpret_cast<float4*>(p) = v;
}
static __device__ __forceinline__ float pb_get(const float4& v, int e) {
    return e == 0 ? v.x : (e == 1 ? v.y : (e == 2 ? v.z : v.w));
}
)PB";
    }

    namespace {

        // ------------------------------------------------------ helpers --
        std::string lit(int64_t v, bool wide) {
            if (wide) return "((pb_u64)(" + std::to_string(v) + "ll))";
            return "((pb_u32)(" + std::to_string(v) + "ll))";
        }

        std::string hex64(uint64_t v) {
            char b[32];
            std::snprintf(b, sizeof b, "%016" PRIx64, v);
            return b;
        }

        uint64_t hash_string(const std::string& s) {
            uint64_t h = 0xcbf29ce484222325ULL;
            for (unsigned char c : s) {
                h ^= c;
                h *= 0x100000001b3ULL;
            }
            return h;
        }

    } // namespace

    // ============================================================ lowerer ==
    lowerer::lowerer(const graph& g, plan& p) : g_(g), p_(p) {}

    int lowerer::new_temp(size_t bytes) {
        p_.temp_bytes.push_back(bytes == 0 ? 4 : bytes);
        return static_cast<int>(p_.temp_bytes.size()) - 1;
    }

    int lowerer::kernel::leaf(arg_kind kind, int index) {
        for (size_t i = 0; i < leaves.size(); ++i)
            if (leaves[i].kind == kind && leaves[i].index == index) return static_cast<int>(i);
        kernel_arg a;
        a.kind = kind;
        a.index = index;
        leaves.push_back(a);
        return static_cast<int>(leaves.size()) - 1;
    }

    bool lowerer::match_softmax(int id, int& x, size_t& axis) const {
        const gnode& n = g_.nodes[static_cast<size_t>(id)];
        if (n.kind != expr_kind::divide || n.a < 0 || n.b < 0) return false;
        const gnode& den = g_.nodes[static_cast<size_t>(n.b)];
        if (den.kind != expr_kind::broadcast) return false;
        const gnode& s = g_.nodes[static_cast<size_t>(den.a)];
        if (s.kind != expr_kind::sum || !s.keepdim || s.a != n.a) return false;
        const gnode& num = g_.nodes[static_cast<size_t>(n.a)];
        if (num.kind != expr_kind::exp) return false;
        const gnode& sub = g_.nodes[static_cast<size_t>(num.a)];
        if (sub.kind != expr_kind::subtract) return false;
        const gnode& bm = g_.nodes[static_cast<size_t>(sub.b)];
        if (bm.kind != expr_kind::broadcast) return false;
        const gnode& m = g_.nodes[static_cast<size_t>(bm.a)];
        if (m.kind != expr_kind::max || !m.keepdim || m.a != sub.a || m.axis != s.axis)
            return false;
        const gnode& xv = g_.nodes[static_cast<size_t>(sub.a)];
        if (xv.is_scalar) return false;
        if (den.p_shape != xv.shape || bm.p_shape != xv.shape) return false;
        x = sub.a;
        axis = s.axis;
        return true;
    }

    bool lowerer::is_barrier(int id) const {
        const gnode& n = g_.nodes[static_cast<size_t>(id)];
        if (n.kind == expr_kind::matmul || n.kind == expr_kind::batched_matmul || n.kind == expr_kind::sum ||
            n.kind == expr_kind::max)
            return true;
        // Only a softmax over the last axis has a kernel of its own; over
        // another axis the pattern lowers as its reductions and elementwise
        // ops, so it must not stop the elementwise walk (materialize would
        // hand it straight back here).
        int x = 0;
        size_t axis = 0;
        return match_softmax(id, x, axis) && axis + 1 == n.shape.size();
    }

    // Finds the single matmul (rank 2) or batched matmul (rank 3) whose
    // output feeds `id` through elementwise ops only (the fusable
    // epilogue). Returns -1 when there is none.
    int lowerer::match_gemm(int id) const {
        const gnode& root = g_.nodes[static_cast<size_t>(id)];
        if (root.is_scalar || (root.shape.size() != 2 && root.shape.size() != 3)) return -1;
        const expr_kind product = root.shape.size() == 2 ? expr_kind::matmul : expr_kind::batched_matmul;
        int found = -1;
        bool ambiguous = false;
        std::function<void(int)> walk = [&](int v) {
            const gnode& n = g_.nodes[static_cast<size_t>(v)];
            switch (n.kind) {
                case expr_kind::matmul:
                case expr_kind::batched_matmul:
                    if (n.kind == product && n.shape == root.shape) {
                        if (found >= 0 && found != v) ambiguous = true;
                        found = v;
                    }
                    return;
                case expr_kind::add:
                case expr_kind::subtract:
                case expr_kind::multiply:
                case expr_kind::divide:
                case expr_kind::maximum:
                case expr_kind::minimum:
                    walk(n.a);
                    walk(n.b);
                    return;
                case expr_kind::exp:
                case expr_kind::reciprocal:
                    walk(n.a);
                    return;
                default:
                    return;
            }
        };
        walk(id);
        if (ambiguous) return -1;
        return found;
    }

    int lowerer::materialize(int id) {
        auto it = done_.find(id);
        if (it != done_.end()) return it->second;
        // Nested lowering (a barrier met while building an outer kernel)
        // must not disturb the outer kernel's coordinate rank.
        struct rank_guard {
            int& r;
            int saved;
            ~rank_guard() { r = saved; }
        } guard{rank_, rank_};
        const gnode& n = g_.nodes[static_cast<size_t>(id)];
        int t = -1;
        int x = 0;
        size_t axis = 0;
        if (match_softmax(id, x, axis) && axis + 1 == n.shape.size()) {
            if (n.shape.size() == 2) {
                const int mm = match_gemm(x);
                if (mm >= 0) t = emit_gemm_softmax(id, x, mm);
            }
            if (t < 0) t = emit_softmax(id, x);
        } else if (n.kind == expr_kind::sum || n.kind == expr_kind::max) {
            t = emit_reduce(id);
        } else if (n.kind == expr_kind::batched_matmul) {
            t = emit_batched_gemm(id, id);
        } else if ((n.kind == expr_kind::reshape || n.kind == expr_kind::unsqueeze) &&
                   g_.nodes[static_cast<size_t>(n.a)].kind != expr_kind::input) {
            // A contiguous result holds the same bytes under any shape:
            // realise the operand under its own shape (its schedules see
            // no carries), and read that buffer as this node.
            t = materialize(n.a);
        } else {
            const int mm = match_gemm(id);
            if (mm >= 0) t = n.shape.size() == 3 ? emit_batched_gemm(id, mm) : emit_gemm(id, mm);
            if (t < 0) t = emit_elementwise(id);
        }
        done_[id] = t;
        return t;
    }

    // Operand of a matmul or reduction as a realised contiguous buffer.
    kernel_arg lowerer::as_buffer(int id) {
        const gnode& n = g_.nodes[static_cast<size_t>(id)];
        kernel_arg a;
        if (n.kind == expr_kind::input) {
            a.kind = arg_kind::slot;
            a.index = n.slot;
        } else {
            a.kind = arg_kind::temp;
            a.index = materialize(id);
        }
        return a;
    }

    gemm_operand lowerer::as_gemm_operand(int id) {
        const gnode& n = g_.nodes[static_cast<size_t>(id)];
        gemm_operand o;
        // Peel one transpose (it swaps the strides), then a slice of an
        // input or the input itself.
        bool transposed = false;
        int v = id;
        if (n.kind == expr_kind::transpose) {
            transposed = true;
            v = n.a;
        }
        const gnode& m = g_.nodes[static_cast<size_t>(v)];
        bool in_place = false;
        if (m.kind == expr_kind::input && m.shape.size() == 2) {
            o.arg.kind = arg_kind::slot;
            o.arg.index = m.slot;
            o.s0 = m.shape[1];
            o.s1 = 1;
            in_place = true;
        } else if (m.kind == expr_kind::slice && m.shape.size() == 2 &&
                   g_.nodes[static_cast<size_t>(m.a)].kind == expr_kind::input && m.p_strides[0] >= 0 &&
                   m.p_strides[1] >= 0) {
            o.arg.kind = arg_kind::slot;
            o.arg.index = g_.nodes[static_cast<size_t>(m.a)].slot;
            o.off = m.p_offset;
            o.s0 = m.p_strides[0];
            o.s1 = m.p_strides[1];
            in_place = true;
        }
        if (!in_place) {
            o.arg = as_buffer(id);
            o.s0 = n.shape[1];
            o.s1 = 1;
            return o;
        }
        if (transposed) std::swap(o.s0, o.s1);
        return o;
    }

    // ================================================= affine analysis ==
    std::string lowerer::pos_key(const position& p) {
        std::string k = p.linear ? "L" : "C";
        auto put = [&](const affine& a) {
            k += std::to_string(a.off);
            for (int64_t s : a.st) k += "," + std::to_string(s);
            k += ";";
        };
        if (p.linear)
            put(p.lin);
        else
            for (const affine& a : p.coords) put(a);
        return k;
    }

    affine lowerer::to_linear(const position& p, const std::vector<index_t>& shape) const {
        if (p.linear) return p.lin;
        affine r;
        r.st.assign(static_cast<size_t>(rank_), 0);
        const std::vector<index_t> cs = contiguous_strides(shape);
        for (size_t k = 0; k < p.coords.size(); ++k) {
            r.off += p.coords[k].off * cs[k];
            for (int d = 0; d < rank_; ++d) r.st[static_cast<size_t>(d)] += p.coords[k].st[static_cast<size_t>(d)] * cs[k];
        }
        return r;
    }

    std::vector<affine> lowerer::to_coords(const position& p, const std::vector<index_t>& shape,
                                           const box& b) const {
        if (!p.linear) return p.coords;
        // Unravel a linear position into the node's coordinates; affine only
        // when no digit carries inside the box.
        const size_t R = shape.size();
        const std::vector<index_t> cs = contiguous_strides(shape);
        int64_t base = p.lin.off;
        for (int d = 0; d < rank_; ++d) base += p.lin.st[static_cast<size_t>(d)] * b.lo[static_cast<size_t>(d)];
        const int64_t numel = static_cast<int64_t>(checked_numel(shape));
        if (base < 0 || (numel > 0 && base >= numel)) throw not_affine{};
        std::vector<affine> out(R);
        std::vector<int64_t> digit(R, 0), reach(R, 0);
        for (size_t k = 0; k < R; ++k) {
            digit[k] = shape[k] == 0 ? 0 : (base / cs[k]) % shape[k];
            out[k].st.assign(static_cast<size_t>(rank_), 0);
            out[k].off = digit[k];
        }
        for (int d = 0; d < rank_; ++d) {
            const int64_t s = p.lin.st[static_cast<size_t>(d)];
            const int64_t extent = b.hi[static_cast<size_t>(d)] - b.lo[static_cast<size_t>(d)];
            if (s == 0 || extent <= 1) continue;
            if (s < 0) throw not_affine{};
            size_t k = 0;
            while (k < R && s % cs[k] != 0) ++k;
            if (k == R) throw not_affine{};
            const int64_t m = s / cs[k];
            out[k].st[static_cast<size_t>(d)] += m;
            out[k].off -= m * b.lo[static_cast<size_t>(d)];
            reach[k] += m * (extent - 1);
        }
        for (size_t k = 0; k < R; ++k)
            if (digit[k] + reach[k] >= shape[k]) throw not_affine{};
        return out;
    }

    int lowerer::push(box& b, vnode v) {
        b.nodes.push_back(std::move(v));
        return static_cast<int>(b.nodes.size()) - 1;
    }

    int lowerer::build(kernel& k, box& b, int id, const position& pos, int acc_id,
                       std::map<std::string, int>& memo) {
        const std::string key = std::to_string(id) + pos_key(pos);
        auto it = memo.find(key);
        if (it != memo.end()) return it->second;
        const gnode& n = g_.nodes[static_cast<size_t>(id)];
        int out = -1;
        auto load_from = [&](arg_kind kind, int index) {
            vnode v;
            v.kind = vnode::op::load;
            v.buffer = k.leaf(kind, index);
            v.map = to_linear(pos, n.shape);
            return push(b, std::move(v));
        };
        if (id == acc_id) {
            // The GEMM accumulator is only defined at the output position.
            if (pos.linear) throw not_fusable{};
            for (int d = 0; d < rank_; ++d) {
                const affine& a = pos.coords[static_cast<size_t>(d)];
                if (a.off != 0) throw not_fusable{};
                for (int e = 0; e < rank_; ++e)
                    if (a.st[static_cast<size_t>(e)] != (d == e ? 1 : 0)) throw not_fusable{};
            }
            vnode v;
            v.kind = vnode::op::acc;
            out = push(b, std::move(v));
            memo.emplace(key, out);
            return out;
        }
        switch (n.kind) {
            case expr_kind::scalar: {
                vnode v;
                v.kind = vnode::op::scalar;
                v.scalar = n.scalar;
                out = push(b, std::move(v));
                break;
            }
            case expr_kind::input:
                out = load_from(arg_kind::slot, n.slot);
                break;
            case expr_kind::add:
            case expr_kind::subtract:
            case expr_kind::multiply:
            case expr_kind::divide:
            case expr_kind::maximum:
            case expr_kind::minimum: {
                if (is_barrier(id)) {
                    out = load_from(arg_kind::temp, materialize(id));
                    break;
                }
                const int l = build(k, b, n.a, pos, acc_id, memo);
                const int r = build(k, b, n.b, pos, acc_id, memo);
                vnode v;
                v.kind = vnode::op::binary;
                v.ek = n.kind;
                v.a = l;
                v.b = r;
                out = push(b, std::move(v));
                break;
            }
            case expr_kind::exp:
            case expr_kind::reciprocal: {
                const int l = build(k, b, n.a, pos, acc_id, memo);
                vnode v;
                v.kind = vnode::op::unary;
                v.ek = n.kind;
                v.a = l;
                out = push(b, std::move(v));
                break;
            }
            case expr_kind::matmul:
            case expr_kind::batched_matmul:
            case expr_kind::sum:
            case expr_kind::max:
                out = load_from(arg_kind::temp, materialize(id));
                break;
            case expr_kind::slice: {
                const std::vector<affine> c = to_coords(pos, n.shape, b);
                position child;
                child.linear = true;
                child.lin.off = n.p_offset;
                child.lin.st.assign(static_cast<size_t>(rank_), 0);
                for (size_t d = 0; d < c.size(); ++d) {
                    child.lin.off += c[d].off * n.p_strides[d];
                    for (int e = 0; e < rank_; ++e)
                        child.lin.st[static_cast<size_t>(e)] += c[d].st[static_cast<size_t>(e)] * n.p_strides[d];
                }
                out = build(k, b, n.a, child, acc_id, memo);
                break;
            }
            case expr_kind::reshape:
            case expr_kind::unsqueeze: {
                position child;
                child.linear = true;
                child.lin = to_linear(pos, n.shape);
                out = build(k, b, n.a, child, acc_id, memo);
                break;
            }
            case expr_kind::transpose: {
                const std::vector<affine> c = to_coords(pos, n.shape, b);
                position child;
                child.coords = {c[1], c[0]};
                out = build(k, b, n.a, child, acc_id, memo);
                break;
            }
            case expr_kind::permute: {
                // Output dim d is input dim perm[d].
                const std::vector<affine> c = to_coords(pos, n.shape, b);
                position child;
                child.coords.resize(c.size());
                for (size_t d = 0; d < c.size(); ++d) child.coords[static_cast<size_t>(n.p_shape[d])] = c[d];
                out = build(k, b, n.a, child, acc_id, memo);
                break;
            }
            case expr_kind::broadcast: {
                const gnode& src = g_.nodes[static_cast<size_t>(n.a)];
                if (src.is_scalar) {
                    out = build(k, b, n.a, pos, acc_id, memo);
                    break;
                }
                const std::vector<affine> c = to_coords(pos, n.shape, b);
                position child;
                const size_t off = n.shape.size() - src.shape.size();
                for (size_t d = 0; d < src.shape.size(); ++d) {
                    if (src.shape[d] == 1) {
                        affine z;
                        z.st.assign(static_cast<size_t>(rank_), 0);
                        child.coords.push_back(z);
                    } else {
                        child.coords.push_back(c[off + d]);
                    }
                }
                out = build(k, b, n.a, child, acc_id, memo);
                break;
            }
            case expr_kind::concat: {
                const std::vector<affine> c = to_coords(pos, n.shape, b);
                const size_t ax = n.axis;
                const int64_t L = g_.nodes[static_cast<size_t>(n.a)].shape[ax];
                const affine& ca = c[ax];
                int dim = -1;
                for (int d = 0; d < rank_; ++d) {
                    if (ca.st[static_cast<size_t>(d)] == 0) continue;
                    if (b.hi[static_cast<size_t>(d)] - b.lo[static_cast<size_t>(d)] <= 1) continue;
                    if (dim >= 0) throw not_affine{};
                    dim = d;
                }
                bool left = false;
                if (dim < 0) {
                    int64_t v = ca.off;
                    for (int d = 0; d < rank_; ++d)
                        v += ca.st[static_cast<size_t>(d)] * b.lo[static_cast<size_t>(d)];
                    left = v < L;
                } else {
                    const int64_t kk = ca.st[static_cast<size_t>(dim)];
                    if (kk < 0) throw not_affine{};
                    int64_t base = ca.off;
                    for (int d = 0; d < rank_; ++d)
                        if (d != dim) base += ca.st[static_cast<size_t>(d)] * b.lo[static_cast<size_t>(d)];
                    const int64_t lo_v = base + kk * b.lo[static_cast<size_t>(dim)];
                    const int64_t hi_v = base + kk * (b.hi[static_cast<size_t>(dim)] - 1);
                    if (hi_v < L) {
                        left = true;
                    } else if (lo_v >= L) {
                        left = false;
                    } else {
                        // First coordinate on the right-hand side.
                        const int64_t t = (L - base + kk - 1) / kk;
                        throw need_split{dim, t};
                    }
                }
                position child;
                child.coords = c;
                if (!left) child.coords[ax].off -= L;
                out = build(k, b, left ? n.a : n.b, child, acc_id, memo);
                break;
            }
        }
        memo.emplace(key, out);
        return out;
    }

    std::vector<box> lowerer::build_boxes(kernel& k, int root, const std::vector<index_t>& shape,
                                          int acc_id) {
        rank_ = static_cast<int>(shape.size());
        std::vector<box> boxes;
        std::function<void(std::vector<int64_t>, std::vector<int64_t>)> rec =
            [&](std::vector<int64_t> lo, std::vector<int64_t> hi) {
                for (int d = 0; d < rank_; ++d)
                    if (lo[static_cast<size_t>(d)] >= hi[static_cast<size_t>(d)]) return;
                box b;
                b.lo = lo;
                b.hi = hi;
                std::map<std::string, int> memo;
                position root_pos;
                for (int d = 0; d < rank_; ++d) {
                    affine a;
                    a.st.assign(static_cast<size_t>(rank_), 0);
                    a.st[static_cast<size_t>(d)] = 1;
                    root_pos.coords.push_back(a);
                }
                try {
                    b.root = build(k, b, root, root_pos, acc_id, memo);
                } catch (const need_split& s) {
                    auto hi1 = hi;
                    hi1[static_cast<size_t>(s.dim)] = s.at;
                    rec(lo, hi1);
                    auto lo2 = lo;
                    lo2[static_cast<size_t>(s.dim)] = s.at;
                    rec(lo2, hi);
                    return;
                }
                boxes.push_back(std::move(b));
            };
        std::vector<int64_t> lo(shape.size(), 0);
        std::vector<int64_t> hi(shape.begin(), shape.end());
        rec(lo, hi);
        return boxes;
    }

    // ================================================= code emission ==
    // Emits `float pb_e<tag>(float l0, ...)`: the per-element arithmetic of a
    // box, in the reference's operator order (src/tensor.cpp:629-683, 856-869).
    std::string lowerer::emit_expr_function(const box& b, const std::string& tag,
                                            std::vector<int>& load_order) const {
        load_order.clear();
        std::ostringstream os;
        std::vector<std::string> names(b.nodes.size());
        std::ostringstream body;
        int params = 0;
        bool has_acc = false;
        for (size_t i = 0; i < b.nodes.size(); ++i) {
            const vnode& v = b.nodes[i];
            switch (v.kind) {
                case vnode::op::load:
                    names[i] = "l" + std::to_string(params++);
                    load_order.push_back(static_cast<int>(i));
                    break;
                case vnode::op::acc:
                    names[i] = "acc";
                    has_acc = true;
                    break;
                case vnode::op::scalar:
                    names[i] = float_literal(v.scalar);
                    break;
                case vnode::op::unary: {
                    names[i] = "t" + std::to_string(i);
                    const std::string& a = names[static_cast<size_t>(v.a)];
                    body << "    const float " << names[i] << " = ";
                    if (v.ek == expr_kind::exp)
                        body << "__expf(" << a << ");\n";
                    else
                        body << "(1.0f / " << a << ");\n";
                    break;
                }
                case vnode::op::binary: {
                    names[i] = "t" + std::to_string(i);
                    const std::string& a = names[static_cast<size_t>(v.a)];
                    const std::string& c = names[static_cast<size_t>(v.b)];
                    body << "    const float " << names[i] << " = ";
                    switch (v.ek) {
                        case expr_kind::add: body << "(" << a << " + " << c << ");\n"; break;
                        case expr_kind::subtract: body << "(" << a << " - " << c << ");\n"; break;
                        case expr_kind::multiply: body << "(" << a << " * " << c << ");\n"; break;
                        case expr_kind::divide: body << "(" << a << " / " << c << ");\n"; break;
                        case expr_kind::maximum:
                            body << "((" << a << ") > (" << c << ") ? (" << a << ") : (" << c << "));\n";
                            break;
                        case expr_kind::minimum:
                            body << "((" << a << ") < (" << c << ") ? (" << a << ") : (" << c << "));\n";
                            break;
                        default: body << "0.0f;\n"; break;
                    }
                    break;
                }
            }
        }
        os << "static __device__ __forceinline__ float pb_e" << tag << "(";
        bool first = true;
        if (has_acc) {
            os << "float acc";
            first = false;
        }
        for (int i = 0; i < params; ++i) {
            if (!first) os << ", ";
            os << "float l" << i;
            first = false;
        }
        if (first) os << "void";
        os << ") {\n" << body.str() << "    return " << names[static_cast<size_t>(b.root)] << ";\n}\n";
        return os.str();
    }

    namespace {
        // Value of an affine map at the box's low corner and its maximum over
        // the box (to pick 32- or 64-bit index arithmetic).
        int64_t affine_at(const affine& a, const std::vector<int64_t>& c) {
            int64_t v = a.off;
            for (size_t d = 0; d < c.size(); ++d) v += a.st[d] * c[d];
            return v;
        }
        int64_t affine_max(const affine& a, const std::vector<int64_t>& lo,
                           const std::vector<int64_t>& hi) {
            int64_t v = a.off;
            for (size_t d = 0; d < lo.size(); ++d)
                v += a.st[d] * (a.st[d] >= 0 ? hi[d] - 1 : lo[d]);
            return v;
        }
    } // namespace

    bool lowerer::needs_wide(const std::vector<box>& boxes, const std::vector<index_t>& shape) const {
        const int64_t numel = static_cast<int64_t>(checked_numel(shape));
        if (numel >= (int64_t{1} << 31) - 4096) return true;
        for (const box& b : boxes)
            for (const vnode& v : b.nodes)
                if (v.kind == vnode::op::load) {
                    const int64_t mx = affine_max(v.map, b.lo, b.hi);
                    if (mx >= (int64_t{1} << 31) - 4096) return true;
                    if (std::llabs(v.map.off) >= (int64_t{1} << 31) - 4096) return true;
                }
        return false;
    }

    // Address expression of a load for coordinate variables c0..c{R-1}.
    std::string lowerer::address(const affine& a, const std::vector<std::string>& cvar, bool wide,
                                 int skip_dim) const {
        std::string s = lit(a.off, wide);
        for (int d = 0; d < rank_; ++d) {
            if (d == skip_dim) continue;
            const int64_t st = a.st[static_cast<size_t>(d)];
            if (st == 0) continue;
            if (st == 1)
                s += " + " + cvar[static_cast<size_t>(d)];
            else
                s += " + " + cvar[static_cast<size_t>(d)] + " * " + lit(st, wide);
        }
        return "(" + s + ")";
    }

    // ROW schedule: 256 threads, U vectors of V consecutive innermost
    // elements per thread; all loads issued before any arithmetic.
    std::string lowerer::emit_row_box(const box& b, int tag, const std::vector<index_t>& shape,
                                      bool wide, int64_t& ctas, std::string& desc) const {
        const int R = rank_;
        const int q = R - 1;
        std::vector<int64_t> E(static_cast<size_t>(R));
        for (int d = 0; d < R; ++d) E[static_cast<size_t>(d)] = b.hi[static_cast<size_t>(d)] - b.lo[static_cast<size_t>(d)];
        const std::vector<index_t> ocs = contiguous_strides(shape);
        bool vec = (E[static_cast<size_t>(q)] % 4 == 0) && (b.lo[static_cast<size_t>(q)] % 4 == 0) &&
                   (R == 1 || shape[static_cast<size_t>(q)] % 4 == 0);
        for (const vnode& v : b.nodes)
            if (v.kind == vnode::op::load) {
                const int64_t sq = v.map.st[static_cast<size_t>(q)];
                if (sq != 0 && sq != 1) vec = false;
            }
        const int V = vec ? 4 : 1;
        const int U = 4;
        int64_t rows = 1;
        for (int d = 0; d < q; ++d) rows *= E[static_cast<size_t>(d)];
        const int64_t ipv = E[static_cast<size_t>(q)] / V;
        const int64_t nvec = rows * ipv;
        ctas = (nvec + 256 * U - 1) / (256 * U);
        const std::string I = wide ? "pb_u64" : "pb_u32";

        std::vector<int> order;
        std::ostringstream os;
        os << emit_expr_function(b, std::to_string(tag), order);
        os << "static __device__ __forceinline__ void pb_box" << tag << "(const float* const* L, float* __restrict__ out, pb_u32 cta) {\n";
        os << "    const " << I << " v0 = (" << I << ")cta * " << 256 * U << "u + threadIdx.x;\n";
        // Per-leaf load mode: 0 broadcast scalar, 1 vector, 2 strided scalars.
        std::vector<int> mode(order.size());
        int nvec_leaves = 0;
        for (size_t li = 0; li < order.size(); ++li) {
            const vnode& v = b.nodes[static_cast<size_t>(order[li])];
            const int64_t sq = v.map.st[static_cast<size_t>(q)];
            if (sq == 0) {
                mode[li] = 0;
            } else if (V == 4 && sq == 1) {
                bool aligned = affine_at(v.map, b.lo) % 4 == 0;
                for (int d = 0; d < q; ++d)
                    if (E[static_cast<size_t>(d)] > 1 && v.map.st[static_cast<size_t>(d)] % 4 != 0) aligned = false;
                mode[li] = aligned ? 1 : 2;
                nvec_leaves += aligned;
            } else {
                mode[li] = 2;
            }
        }
        os << "    float x[" << U << "][" << (order.empty() ? 1 : order.size()) << "][" << V << "];\n";
        os << "    " << I << " oa[" << U << "];\n";
        os << "    #pragma unroll\n    for (int u = 0; u < " << U << "; ++u) {\n";
        os << "        const " << I << " v = v0 + (" << I << ")u * 256u;\n";
        os << "        oa[u] = ~(" << I << ")0;\n";
        os << "        if (v < " << lit(nvec, wide) << ") {\n";
        std::vector<std::string> cvar(static_cast<size_t>(R));
        for (int d = 0; d < R; ++d) cvar[static_cast<size_t>(d)] = "c" + std::to_string(d);
        os << "            " << I << " t = v;\n";
        os << "            const " << I << " c" << q << " = " << lit(b.lo[static_cast<size_t>(q)], wide)
           << " + (t % " << lit(ipv, wide) << ") * " << V << "u;\n";
        if (q > 0) os << "            t /= " << lit(ipv, wide) << ";\n";
        for (int d = q - 1; d >= 0; --d) {
            if (d > 0) {
                os << "            const " << I << " c" << d << " = " << lit(b.lo[static_cast<size_t>(d)], wide)
                   << " + t % " << lit(E[static_cast<size_t>(d)], wide) << ";\n";
                os << "            t /= " << lit(E[static_cast<size_t>(d)], wide) << ";\n";
            } else {
                os << "            const " << I << " c0 = " << lit(b.lo[0], wide) << " + t;\n";
            }
        }
        // Output address.
        affine oaff;
        oaff.st.assign(static_cast<size_t>(R), 0);
        for (int d = 0; d < R; ++d) oaff.st[static_cast<size_t>(d)] = ocs[static_cast<size_t>(d)];
        os << "            oa[u] = " << address(oaff, cvar, wide, -1) << ";\n";
        for (size_t li = 0; li < order.size(); ++li) {
            const vnode& v = b.nodes[static_cast<size_t>(order[li])];
            const std::string base = "L[" + std::to_string(v.buffer) + "]";
            const std::string addr = address(v.map, cvar, wide, -1);
            if (mode[li] == 0) {
                os << "            { const float s = pb_ld(" << base << " + " << addr << ");";
                for (int e = 0; e < V; ++e) os << " x[u][" << li << "][" << e << "] = s;";
                os << " }\n";
            } else if (mode[li] == 1) {
                os << "            { const float4 w = pb_ld4(" << base << " + " << addr
                   << "); x[u][" << li << "][0] = w.x; x[u][" << li << "][1] = w.y; x[u][" << li
                   << "][2] = w.z; x[u][" << li << "][3] = w.w; }\n";
            } else {
                const int64_t sq = v.map.st[static_cast<size_t>(q)];
                for (int e = 0; e < V; ++e)
                    os << "            x[u][" << li << "][" << e << "] = pb_ld(" << base << " + " << addr
                       << " + " << lit(sq * e, wide) << ");\n";
            }
        }
        os << "        }\n    }\n";
        os << "    #pragma unroll\n    for (int u = 0; u < " << U << "; ++u) {\n";
        os << "        if (oa[u] != ~(" << I << ")0) {\n";
        for (int e = 0; e < V; ++e) {
            os << "            const float y" << e << " = pb_e" << tag << "(";
            for (size_t li = 0; li < order.size(); ++li) {
                if (li) os << ", ";
                os << "x[u][" << li << "][" << e << "]";
            }
            os << ");\n";
        }
        if (V == 4)
            os << "            pb_st4(out + oa[u], make_float4(y0, y1, y2, y3));\n";
        else
            os << "            out[oa[u]] = y0;\n";
        os << "        }\n    }\n}\n";
        std::ostringstream d;
        d << "box" << tag << " ROW V=" << V << " U=" << U << " vec_leaves=" << nvec_leaves << "/"
          << order.size() << " ctas=" << ctas;
        desc = d.str();
        return os.str();
    }

    // TILE schedule for boxes with a transposed leaf: see the file comment.
    std::string lowerer::emit_tile_box(const box& b, int tag, const std::vector<index_t>& shape,
                                       bool wide, int p, int64_t& ctas, int& smem_tiles,
                                       std::string& desc) const {
        const int R = rank_;
        const int q = R - 1;
        std::vector<int64_t> E(static_cast<size_t>(R));
        for (int d = 0; d < R; ++d) E[static_cast<size_t>(d)] = b.hi[static_cast<size_t>(d)] - b.lo[static_cast<size_t>(d)];
        const std::vector<index_t> ocs = contiguous_strides(shape);
        const int64_t tp_n = (E[static_cast<size_t>(p)] + 63) / 64;
        const int64_t tq_n = (E[static_cast<size_t>(q)] + 63) / 64;
        int64_t batch = 1;
        for (int d = 0; d < R; ++d)
            if (d != p && d != q) batch *= E[static_cast<size_t>(d)];
        ctas = tp_n * tq_n * batch;
        const std::string I = wide ? "pb_u64" : "pb_u32";
        std::vector<int> order;
        std::ostringstream os;
        os << emit_expr_function(b, std::to_string(tag), order);
        // Classify leaves.
        std::vector<int> tslot(order.size(), -1);
        std::vector<bool> tvec(order.size(), false);
        std::vector<int> mode(order.size(), 0);
        int nt = 0;
        for (size_t li = 0; li < order.size(); ++li) {
            const vnode& v = b.nodes[static_cast<size_t>(order[li])];
            const int64_t sq = v.map.st[static_cast<size_t>(q)];
            if (sq != 0 && sq != 1) {
                tslot[li] = nt++;
                bool aligned = affine_at(v.map, b.lo) % 4 == 0 && sq % 4 == 0;
                for (int d = 0; d < R; ++d)
                    if (d != p && d != q && E[static_cast<size_t>(d)] > 1 &&
                        v.map.st[static_cast<size_t>(d)] % 4 != 0)
                        aligned = false;
                tvec[li] = aligned;
            } else if (sq == 0) {
                mode[li] = 0;
            } else {
                bool aligned = affine_at(v.map, b.lo) % 4 == 0;
                for (int d = 0; d < q; ++d)
                    if (E[static_cast<size_t>(d)] > 1 && v.map.st[static_cast<size_t>(d)] % 4 != 0) aligned = false;
                mode[li] = aligned ? 1 : 2;
            }
        }
        smem_tiles = nt;
        std::vector<std::string> cvar(static_cast<size_t>(R));
        for (int d = 0; d < R; ++d) cvar[static_cast<size_t>(d)] = "c" + std::to_string(d);
        os << "static __device__ __forceinline__ void pb_box" << tag
           << "(const float* const* L, float* __restrict__ out, pb_u32 cta, float* sm) {\n";
        os << "    pb_u32 t = cta;\n";
        os << "    const pb_u32 tq = t % " << tq_n << "u; t /= " << tq_n << "u;\n";
        os << "    const pb_u32 tp = t % " << tp_n << "u; t /= " << tp_n << "u;\n";
        // Batch coordinates.
        for (int d = R - 1; d >= 0; --d) {
            if (d == p || d == q) continue;
            os << "    const " << I << " c" << d << " = " << lit(b.lo[static_cast<size_t>(d)], wide) << " + ("
               << I << ")(t % " << E[static_cast<size_t>(d)] << "u); t /= " << E[static_cast<size_t>(d)] << "u;\n";
        }
        os << "    const " << I << " bp = " << lit(b.lo[static_cast<size_t>(p)], wide) << " + (" << I << ")tp * 64u;\n";
        os << "    const " << I << " bq = " << lit(b.lo[static_cast<size_t>(q)], wide) << " + (" << I << ")tq * 64u;\n";
        const std::string hp = lit(b.hi[static_cast<size_t>(p)], wide);
        const std::string hq = lit(b.hi[static_cast<size_t>(q)], wide);
        // Load phase.
        os << "    #pragma unroll\n    for (int u = 0; u < 4; ++u) {\n";
        os << "        const pb_u32 f = threadIdx.x + 256u * u;\n";
        os << "        const pb_u32 ci = (f & 7u) | ((f >> 9) << 3);\n";
        os << "        const pb_u32 j = (f >> 3) & 63u;\n";
        os << "        const pb_u32 i = ci * 4u;\n";
        os << "        const " << I << " c" << p << " = bp + i;\n";
        os << "        const " << I << " c" << q << " = bq + j;\n";
        os << "        const pb_u32 sw = 4u * ((j >> 2) ^ (ci & 7u)) + (j & 3u);\n";
        for (size_t li = 0; li < order.size(); ++li) {
            if (tslot[li] < 0) continue;
            const vnode& v = b.nodes[static_cast<size_t>(order[li])];
            const std::string base = "L[" + std::to_string(v.buffer) + "]";
            const std::string addr = address(v.map, cvar, wide, -1);
            const int64_t sp = v.map.st[static_cast<size_t>(p)];
            os << "        {\n            float4 w = make_float4(0.f, 0.f, 0.f, 0.f);\n";
            os << "            if (c" << p << " < " << hp << " && c" << q << " < " << hq << ") {\n";
            if (tvec[li] && sp == 1) {
                os << "                w = pb_ld4(" << base << " + " << addr << ");\n";
            } else {
                os << "                const " << I << " a = " << addr << ";\n";
                for (int e = 0; e < 4; ++e) {
                    const char* comp = e == 0 ? "x" : (e == 1 ? "y" : (e == 2 ? "z" : "w"));
                    if (e == 0)
                        os << "                w." << comp << " = pb_ld(" << base << " + a);\n";
                    else
                        os << "                if (c" << p << " + " << e << "u < " << hp << ") w." << comp
                           << " = pb_ld(" << base << " + a + " << lit(sp * e, wide) << ");\n";
                }
            }
            os << "            }\n";
            const int base_off = tslot[li] * 4096;
            os << "            float* s = sm + " << base_off << " + i * 64u + sw;\n";
            os << "            s[0] = w.x; s[64] = w.y; s[128] = w.z; s[192] = w.w;\n";
            os << "        }\n";
        }
        os << "    }\n    __syncthreads();\n";
        // Output phase.
        os << "    #pragma unroll\n    for (int u = 0; u < 4; ++u) {\n";
        os << "        const pb_u32 f = threadIdx.x + 256u * u;\n";
        os << "        const pb_u32 ch = f & 15u;\n";
        os << "        const pb_u32 i = f >> 4;\n";
        os << "        const " << I << " c" << p << " = bp + i;\n";
        os << "        const " << I << " c" << q << " = bq + 4u * ch;\n";
        os << "        if (c" << p << " < " << hp << " && c" << q << " < " << hq << ") {\n";
        for (size_t li = 0; li < order.size(); ++li) {
            const vnode& v = b.nodes[static_cast<size_t>(order[li])];
            const std::string base = "L[" + std::to_string(v.buffer) + "]";
            if (tslot[li] >= 0) {
                os << "            const float4 x" << li << " = *reinterpret_cast<const float4*>(sm + "
                   << tslot[li] * 4096 << " + i * 64u + 4u * (ch ^ ((i >> 2) & 7u)));\n";
            } else if (mode[li] == 0) {
                const std::string addr = address(v.map, cvar, wide, -1);
                os << "            const float s" << li << " = pb_ld(" << base << " + " << addr << ");\n";
                os << "            const float4 x" << li << " = make_float4(s" << li << ", s" << li << ", s"
                   << li << ", s" << li << ");\n";
            } else if (mode[li] == 1) {
                const std::string addr = address(v.map, cvar, wide, -1);
                os << "            const float4 x" << li << " = pb_ld4(" << base << " + " << addr << ");\n";
            } else {
                const std::string addr = address(v.map, cvar, wide, -1);
                os << "            const float4 x" << li << " = make_float4(pb_ld(" << base << " + " << addr
                   << "), pb_ld(" << base << " + " << addr << " + 1u), pb_ld(" << base << " + " << addr
                   << " + 2u), pb_ld(" << base << " + " << addr << " + 3u));\n";
            }
        }
        const char* comps[4] = {"x", "y", "z", "w"};
        for (int e = 0; e < 4; ++e) {
            os << "            const float y" << e << " = pb_e" << tag << "(";
            for (size_t li = 0; li < order.size(); ++li) {
                if (li) os << ", ";
                os << "x" << li << "." << comps[e];
            }
            os << ");\n";
        }
        affine oaff;
        oaff.st.assign(static_cast<size_t>(R), 0);
        for (int d = 0; d < R; ++d) oaff.st[static_cast<size_t>(d)] = ocs[static_cast<size_t>(d)];
        os << "            pb_st4(out + " << address(oaff, cvar, wide, -1) << ", make_float4(y0, y1, y2, y3));\n";
        os << "        }\n    }\n}\n";
        std::ostringstream d;
        d << "box" << tag << " TILE p=" << p << " tiles=" << tp_n << "x" << tq_n << "x" << batch
          << " transposed_leaves=" << nt;
        desc = d.str();
        return os.str();
    }

    // Every generated kernel first waits for the stream's previous kernel
    // (griddepcontrol.wait: returns at once when there is no programmatic
    // dependency), so all of them can launch with programmatic stream
    // serialization and their launch overlaps the previous kernel's tail.
    void lowerer::finish_kernel(launch_spec& l) {
        const size_t g = l.source.find("__global__");
        const size_t open = g == std::string::npos ? g : l.source.find('{', g);
        if (open == std::string::npos || l.source.find("__global__", g + 10) != std::string::npos)
            throw std::logic_error("generated source must define exactly one kernel: " + l.name);
        l.source.insert(open + 1, "\n    asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");");
        l.pdl = true;
        const auto& opts = kernel_options();
        std::vector<const char*> o;
        for (const auto& s : opts) o.push_back(s.c_str());
        check(pbrt_compile(l.source.c_str(), o.data(), static_cast<int>(o.size()), 1, &l.image_key));
    }

    int lowerer::emit_elementwise(int id) {
        const gnode& n = g_.nodes[static_cast<size_t>(id)];
        std::vector<index_t> shape = n.shape;
        if (shape.empty()) shape = {1};
        kernel k;
        std::vector<box> boxes;
        try {
            boxes = build_boxes(k, id, shape, -1);
        } catch (const not_affine&) {
            return emit_generic(id);
        }
        const int out = new_temp(checked_numel(shape) * sizeof(float));
        const bool wide = needs_wide(boxes, shape);
        std::ostringstream src;
        src << kernel_prelude();
        std::vector<int64_t> ctas(boxes.size());
        std::vector<bool> tiled(boxes.size(), false);
        std::string desc;
        int max_tiles = 0;
        for (size_t bi = 0; bi < boxes.size(); ++bi) {
            const box& b = boxes[bi];
            const int R = rank_;
            const int q = R - 1;
            // Transposed leaves and the dim along which they are contiguous.
            int p = -1;
            bool has_t = false;
            for (const vnode& v : b.nodes) {
                if (v.kind != vnode::op::load) continue;
                const int64_t sq = v.map.st[static_cast<size_t>(q)];
                if (sq != 0 && sq != 1) has_t = true;
            }
            if (has_t && R >= 2) {
                int64_t best = 0;
                for (int d = 0; d < q; ++d) {
                    bool ok = true;
                    for (const vnode& v : b.nodes) {
                        if (v.kind != vnode::op::load) continue;
                        const int64_t sq = v.map.st[static_cast<size_t>(q)];
                        if (sq != 0 && sq != 1 && v.map.st[static_cast<size_t>(d)] != 1) ok = false;
                    }
                    const int64_t ext = b.hi[static_cast<size_t>(d)] - b.lo[static_cast<size_t>(d)];
                    if (ok && ext > best) {
                        best = ext;
                        p = d;
                    }
                }
                const int64_t eq = b.hi[static_cast<size_t>(q)] - b.lo[static_cast<size_t>(q)];
                if (p >= 0 && !(eq % 4 == 0 && b.lo[static_cast<size_t>(q)] % 4 == 0 &&
                                shape[static_cast<size_t>(q)] % 4 == 0 && best >= 4))
                    p = -1;
            }
            std::string d;
            if (p >= 0) {
                int tiles = 0;
                src << emit_tile_box(b, static_cast<int>(bi), shape, wide, p, ctas[bi], tiles, d);
                tiled[bi] = true;
                max_tiles = std::max(max_tiles, tiles);
            } else {
                src << emit_row_box(b, static_cast<int>(bi), shape, wide, ctas[bi], d);
            }
            desc += (desc.empty() ? "" : "; ") + d;
        }
        launch_spec l;
        const std::string body = src.str();
        l.name = "pb_elem_" + hex64(hash_string(body)).substr(0, 8);
        std::ostringstream ker;
        ker << body;
        ker << "extern \"C\" __global__ void __launch_bounds__(256) " << l.name << "(";
        for (size_t i = 0; i < k.leaves.size(); ++i) ker << "const float* __restrict__ in" << i << ", ";
        ker << "float* __restrict__ out) {\n";
        ker << "    const float* L[" << std::max<size_t>(1, k.leaves.size()) << "] = {";
        for (size_t i = 0; i < k.leaves.size(); ++i) ker << (i ? ", " : "") << "in" << i;
        if (k.leaves.empty()) ker << "nullptr";
        ker << "};\n";
        if (max_tiles > 0) ker << "    extern __shared__ float4 pb_dyn_smem[];\n    float* sm = reinterpret_cast<float*>(pb_dyn_smem);\n";
        ker << "    pb_u32 cta = blockIdx.x;\n";
        int64_t total = 0;
        for (size_t bi = 0; bi < boxes.size(); ++bi) {
            ker << "    if (cta < " << ctas[bi] << "u) { pb_box" << bi << "(L, out, cta"
                << (tiled[bi] ? ", sm" : "") << "); return; }\n";
            ker << "    cta -= " << ctas[bi] << "u;\n";
            total += ctas[bi];
        }
        ker << "}\n";
        l.source = ker.str();
        l.schedule = "elementwise " + desc;
        if (total > 0x7fffffff) throw std::invalid_argument("tensor is too large for one launch");
        l.grid = {static_cast<uint32_t>(std::max<int64_t>(1, total)), 1, 1};
        l.block = {256, 1, 1};
        l.smem = static_cast<uint32_t>(max_tiles) * 4096u * 4u;
        l.args = k.leaves;
        kernel_arg o;
        o.kind = arg_kind::temp;
        o.index = out;
        l.args.push_back(o);
        finish_kernel(l);
        p_.launches.push_back(std::move(l));
        return out;
    }

    // ---------------------------------------------------- generic gather --
    // Fallback for graphs whose index maps are not affine: one thread per
    // output element, index arithmetic composed node by node on the linear
    // output index (the same composition rules as src/tensor.cpp:511-614).
    std::string lowerer::gen_value(kernel& k, int id, const std::string& idx,
                                   std::ostringstream& stmts, int& counter) {
        const gnode& n = g_.nodes[static_cast<size_t>(id)];
        auto coord = [&](const std::vector<index_t>& shape, size_t d) {
            const std::vector<index_t> cs = contiguous_strides(shape);
            return "((" + idx + " / " + std::to_string(cs[d]) + "ull) % " + std::to_string(shape[d]) + "ull)";
        };
        switch (n.kind) {
            case expr_kind::scalar:
                return float_literal(n.scalar);
            case expr_kind::input:
                return "pb_ld(in" + std::to_string(k.leaf(arg_kind::slot, n.slot)) + " + (" + idx + "))";
            case expr_kind::matmul:
            case expr_kind::batched_matmul:
            case expr_kind::sum:
            case expr_kind::max:
                return "pb_ld(in" + std::to_string(k.leaf(arg_kind::temp, materialize(id))) + " + (" +
                       idx + "))";
            case expr_kind::add:
            case expr_kind::subtract:
            case expr_kind::multiply:
            case expr_kind::divide:
            case expr_kind::maximum:
            case expr_kind::minimum: {
                if (is_barrier(id))
                    return "pb_ld(in" + std::to_string(k.leaf(arg_kind::temp, materialize(id))) +
                           " + (" + idx + "))";
                const std::string a = gen_value(k, n.a, idx, stmts, counter);
                const std::string c = gen_value(k, n.b, idx, stmts, counter);
                const std::string t = "g" + std::to_string(counter++);
                stmts << "    const float " << t << " = ";
                switch (n.kind) {
                    case expr_kind::add: stmts << "(" << a << " + " << c << ");\n"; break;
                    case expr_kind::subtract: stmts << "(" << a << " - " << c << ");\n"; break;
                    case expr_kind::multiply: stmts << "(" << a << " * " << c << ");\n"; break;
                    case expr_kind::divide: stmts << "(" << a << " / " << c << ");\n"; break;
                    case expr_kind::maximum: stmts << "((" << a << ") > (" << c << ") ? (" << a << ") : (" << c << "));\n"; break;
                    default: stmts << "((" << a << ") < (" << c << ") ? (" << a << ") : (" << c << "));\n"; break;
                }
                return t;
            }
            case expr_kind::exp:
            case expr_kind::reciprocal: {
                const std::string a = gen_value(k, n.a, idx, stmts, counter);
                const std::string t = "g" + std::to_string(counter++);
                if (n.kind == expr_kind::exp)
                    stmts << "    const float " << t << " = __expf(" << a << ");\n";
                else
                    stmts << "    const float " << t << " = (1.0f / " << a << ");\n";
                return t;
            }
            case expr_kind::slice: {
                std::string s = std::to_string(n.p_offset) + "ull";
                for (size_t d = 0; d < n.shape.size(); ++d)
                    if (n.p_strides[d] != 0)
                        s += " + " + coord(n.shape, d) + " * " + std::to_string(n.p_strides[d]) + "ull";
                const std::string v = "x" + std::to_string(counter++);
                stmts << "    const pb_u64 " << v << " = " << s << ";\n";
                return gen_value(k, n.a, v, stmts, counter);
            }
            case expr_kind::reshape:
            case expr_kind::unsqueeze:
                return gen_value(k, n.a, idx, stmts, counter);
            case expr_kind::permute: {
                const gnode& src = g_.nodes[static_cast<size_t>(n.a)];
                const std::vector<index_t> scs = contiguous_strides(src.shape);
                std::string s = "0ull";
                for (size_t d = 0; d < n.shape.size(); ++d)
                    s += " + " + coord(n.shape, d) + " * " + std::to_string(scs[static_cast<size_t>(n.p_shape[d])]) + "ull";
                const std::string v = "x" + std::to_string(counter++);
                stmts << "    const pb_u64 " << v << " = " << s << ";\n";
                return gen_value(k, n.a, v, stmts, counter);
            }
            case expr_kind::transpose: {
                const gnode& src = g_.nodes[static_cast<size_t>(n.a)];
                const std::string v = "x" + std::to_string(counter++);
                stmts << "    const pb_u64 " << v << " = ((" << idx << ") % " << src.shape[0] << "ull) * "
                      << src.shape[1] << "ull + (" << idx << ") / " << src.shape[0] << "ull;\n";
                return gen_value(k, n.a, v, stmts, counter);
            }
            case expr_kind::broadcast: {
                const gnode& src = g_.nodes[static_cast<size_t>(n.a)];
                if (src.is_scalar) return gen_value(k, n.a, idx, stmts, counter);
                const std::vector<index_t> scs = contiguous_strides(src.shape);
                const size_t off = n.shape.size() - src.shape.size();
                std::string s = "0ull";
                for (size_t d = 0; d < src.shape.size(); ++d)
                    if (src.shape[d] != 1)
                        s += " + " + coord(n.shape, off + d) + " * " + std::to_string(scs[d]) + "ull";
                const std::string v = "x" + std::to_string(counter++);
                stmts << "    const pb_u64 " << v << " = " << s << ";\n";
                return gen_value(k, n.a, v, stmts, counter);
            }
            case expr_kind::concat: {
                const gnode& l = g_.nodes[static_cast<size_t>(n.a)];
                const gnode& r = g_.nodes[static_cast<size_t>(n.b)];
                const std::vector<index_t> lcs = contiguous_strides(l.shape);
                const std::vector<index_t> rcs = contiguous_strides(r.shape);
                std::string li = "0ull", ri = "0ull";
                for (size_t d = 0; d < n.shape.size(); ++d) {
                    const std::string c = coord(n.shape, d);
                    li += " + " + c + " * " + std::to_string(lcs[d]) + "ull";
                    if (d == n.axis)
                        ri += " + (" + c + " - " + std::to_string(l.shape[d]) + "ull) * " + std::to_string(rcs[d]) + "ull";
                    else
                        ri += " + " + c + " * " + std::to_string(rcs[d]) + "ull";
                }
                const std::string ax = "x" + std::to_string(counter++);
                stmts << "    const pb_u64 " << ax << " = " << coord(n.shape, n.axis) << ";\n";
                const std::string t = "g" + std::to_string(counter++);
                stmts << "    float " << t << ";\n    if (" << ax << " < " << l.shape[n.axis] << "ull) {\n";
                std::ostringstream lst;
                const std::string lv = gen_value(k, n.a, "(" + li + ")", lst, counter);
                stmts << lst.str() << "    " << t << " = " << lv << ";\n    } else {\n";
                std::ostringstream rst;
                const std::string rv = gen_value(k, n.b, "(" + ri + ")", rst, counter);
                stmts << rst.str() << "    " << t << " = " << rv << ";\n    }\n";
                return t;
            }
        }
        return "0.0f";
    }

    int lowerer::emit_generic(int id) {
        const gnode& n = g_.nodes[static_cast<size_t>(id)];
        const size_t count = checked_numel(n.shape.empty() ? std::vector<index_t>{1} : n.shape);
        const int out = new_temp(count * sizeof(float));
        kernel k;
        std::ostringstream stmts;
        int counter = 0;
        const std::string v = gen_value(k, id, "i", stmts, counter);
        std::ostringstream src;
        src << kernel_prelude();
        std::ostringstream body;
        body << "    for (pb_u64 i = (pb_u64)blockIdx.x * 256u + threadIdx.x; i < " << count
             << "ull; i += (pb_u64)gridDim.x * 256u) {\n"
             << stmts.str() << "    out[i] = " << v << ";\n    }\n";
        launch_spec l;
        l.name = "pb_gather_" + hex64(hash_string(body.str())).substr(0, 8);
        src << "extern \"C\" __global__ void __launch_bounds__(256) " << l.name << "(";
        for (size_t i = 0; i < k.leaves.size(); ++i) src << "const float* __restrict__ in" << i << ", ";
        src << "float* __restrict__ out) {\n" << body.str() << "}\n";
        l.source = src.str();
        l.schedule = "gather (non-affine index maps)";
        const uint64_t blocks = std::min<uint64_t>((count + 255) / 256, 148u * 16u);
        l.grid = {static_cast<uint32_t>(std::max<uint64_t>(1, blocks)), 1, 1};
        l.args = k.leaves;
        kernel_arg o;
        o.kind = arg_kind::temp;
        o.index = out;
        l.args.push_back(o);
        finish_kernel(l);
        p_.launches.push_back(std::move(l));
        return out;
    }

    // ------------------------------------------------------ reductions --
    // Builds the operand of a row-wise kernel (reduction or softmax) as a
    // single affine box over the operand's coordinates. Falls back to
    // materialising the operand when it is not a single affine box or its
    // leaves are not contiguous along `axis`.
    lowerer::row_operand lowerer::row_prologue(int operand, size_t axis) {
        const gnode& s = g_.nodes[static_cast<size_t>(operand)];
        row_operand r;
        r.shape = s.shape;
        auto try_build = [&](int src_id) -> bool {
            r.k = kernel{};
            std::vector<box> boxes;
            try {
                boxes = build_boxes(r.k, src_id, r.shape, -1);
            } catch (const not_affine&) {
                return false;
            }
            if (boxes.size() != 1) return false;
            for (const vnode& v : boxes[0].nodes)
                if (v.kind == vnode::op::load) {
                    const int64_t sa = v.map.st[axis];
                    if (axis + 1 == r.shape.size() && sa != 0 && sa != 1) return false;
                }
            r.b = std::move(boxes[0]);
            return true;
        };
        if (!try_build(operand)) {
            // Materialise the operand, then read it back as a plain input.
            const int t = materialize(operand);
            r.k = kernel{};
            rank_ = static_cast<int>(r.shape.size());
            r.b = box{};
            r.b.lo.assign(r.shape.size(), 0);
            r.b.hi.assign(r.shape.begin(), r.shape.end());
            vnode v;
            v.kind = vnode::op::load;
            v.buffer = r.k.leaf(arg_kind::temp, t);
            v.map.st.assign(r.shape.size(), 0);
            const std::vector<index_t> cs = contiguous_strides(r.shape);
            for (size_t d = 0; d < r.shape.size(); ++d) v.map.st[d] = cs[d];
            r.b.nodes.push_back(v);
            r.b.root = 0;
        }
        return r;
    }

    int lowerer::emit_reduce(int id) {
        const gnode& n = g_.nodes[static_cast<size_t>(id)];
        const bool is_sum = n.kind == expr_kind::sum;
        row_operand r = row_prologue(n.a, n.axis);
        // Dimensions after the reduced axis that every load walks
        // contiguously (or not at all) merge into one: [A, B, C] over axis
        // 0 becomes [A, B*C], which the column-tile schedule reads as
        // float4. The outputs keep their order, so nothing else changes.
        if (n.axis + 2 < r.shape.size()) {
            const size_t a0 = n.axis + 1, last = r.shape.size() - 1;
            bool ok = true;
            for (size_t d = a0; d <= last && ok; ++d)
                ok = r.b.lo[d] == 0 && r.b.hi[d] == r.shape[d];
            for (const vnode& v : r.b.nodes) {
                if (!ok) break;
                if (v.kind != vnode::op::load) continue;
                for (size_t d = a0; d < last && ok; ++d)
                    ok = r.shape[d] == 1 || v.map.st[d] == v.map.st[d + 1] * r.shape[d + 1];
            }
            if (ok) {
                int64_t merged = 1;
                for (size_t d = a0; d <= last; ++d) merged *= r.shape[d];
                for (vnode& v : r.b.nodes)
                    if (v.kind == vnode::op::load) {
                        const int64_t st_last = v.map.st[last];
                        v.map.st.resize(a0);
                        v.map.st.push_back(st_last);
                    }
                r.shape.resize(a0);
                r.shape.push_back(merged);
                r.b.lo.resize(a0);
                r.b.lo.push_back(0);
                r.b.hi.resize(a0);
                r.b.hi.push_back(merged);
            }
        }
        const std::vector<index_t>& S = r.shape;
        rank_ = static_cast<int>(S.size());
        const int R = rank_;
        const size_t ax = n.axis;
        int64_t outer = 1, inner = 1;
        for (size_t d = 0; d < ax; ++d) outer *= S[d];
        for (size_t d = ax + 1; d < S.size(); ++d) inner *= S[d];
        const int64_t A = S[ax];
        const int64_t outputs = outer * inner;
        const int out = new_temp(static_cast<size_t>(outputs) * sizeof(float));
        bool wide = needs_wide({r.b}, S);
        const std::string I = wide ? "pb_u64" : "pb_u32";
        std::vector<int> order;
        std::ostringstream src;
        src << kernel_prelude();
        src << emit_expr_function(r.b, "0", order);
        const std::string init = is_sum ? "0.0f" : "PB_NEG_FLT_MAX";
        auto combine = [&](const std::string& acc, const std::string& v) {
            if (is_sum) return acc + " = " + acc + " + " + v + ";";
            return acc + " = " + acc + " > " + v + " ? " + acc + " : " + v + ";";
        };
        std::vector<std::string> cvar(static_cast<size_t>(R));
        for (int d = 0; d < R; ++d) cvar[static_cast<size_t>(d)] = "c" + std::to_string(d);
        std::ostringstream body;
        launch_spec l;
        std::string desc;
        int threads = 256;
        // The loop over the reduction axis of a strided reduction: eight
        // independent loads (and prologues) per step, then combined in k
        // order -- the same result as one at a time, with eight loads in
        // flight per thread.
        auto emit_strided_loop = [&](std::ostringstream& os, const std::string& from, const std::string& to) {
            auto value_at = [&](const std::string& k, const std::string& dst, const std::string& ind) {
                os << ind << "{\n" << ind << "    const " << I << " c" << ax << " = " << k << ";\n";
                for (size_t li = 0; li < order.size(); ++li) {
                    const vnode& v = r.b.nodes[static_cast<size_t>(order[li])];
                    os << ind << "    const float x" << li << " = pb_ld(in" << v.buffer << " + "
                       << address(v.map, cvar, wide, -1) << ");\n";
                }
                os << ind << "    " << dst << " = pb_e0(";
                for (size_t li = 0; li < order.size(); ++li) os << (li ? ", " : "") << "x" << li;
                os << ");\n" << ind << "}\n";
            };
            os << "    " << I << " k = " << from << ";\n";
            os << "    for (; k + 8u <= " << to << "; k += 8u) {\n        float vv[8];\n";
            os << "        #pragma unroll\n        for (int u = 0; u < 8; ++u)\n";
            value_at("k + (" + I + ")u", "vv[u]", "        ");
            os << "        #pragma unroll\n        for (int u = 0; u < 8; ++u) { const float v = vv[u]; "
               << combine("acc", "v") << " }\n    }\n";
            os << "    for (; k < " << to << "; ++k) {\n        float v;\n";
            value_at("k", "v", "        ");
            os << "        " << combine("acc", "v") << "\n    }\n";
        };
        // Pass 2 of a reduction split into row chunks: `chunks` partials per
        // output, laid out [chunk][output]. A CTA of 512 threads covers W
        // outputs (32, or 8 when there are too few outputs to spread 32-wide
        // CTAs over the GPU) with G = 512 / W groups; group g combines chunks
        // g, g+G, ... in order (eight loads in flight). The G group results
        // are then combined in a fixed two-level order through shared
        // memory, so the result does not depend on scheduling.
        auto emit_chunk_combine = [&](int partial, int64_t chunks, const std::string& what) {
            const bool pwide = wide || chunks * outputs >= (int64_t{1} << 31) - 4096;
            const std::string PI = pwide ? "pb_u64" : "pb_u32";
            const int W = outputs >= 32 * 148 ? 32 : 8;
            const int G = 512 / W;
            const std::string Ws = std::to_string(W), Gs = std::to_string(G), Ss = std::to_string(G / 8);
            std::ostringstream b2;
            b2 << "    __shared__ float red[" << Gs << "][" << W + 1 << "];\n";
            b2 << "    __shared__ float red2[8][" << W + 1 << "];\n";
            b2 << "    const pb_u32 j = threadIdx.x % " << Ws << "u, g = threadIdx.x / " << Ws << "u;\n";
            b2 << "    const " << PI << " o = (" << PI << ")blockIdx.x * " << Ws << "u + j;\n";
            b2 << "    float acc = " << init << ";\n";
            b2 << "    if (o < " << lit(outputs, pwide) << ") {\n";
            b2 << "        " << PI << " c = g;\n";
            b2 << "        for (; c + " << 7 * G << "u < " << lit(chunks, pwide) << "; c += " << 8 * G
               << "u) {\n            float vv[8];\n";
            b2 << "            #pragma unroll\n            for (int u = 0; u < 8; ++u) vv[u] = part[(c + " << Gs
               << "u * (" << PI << ")u) * " << lit(outputs, pwide) << " + o];\n";
            b2 << "            #pragma unroll\n            for (int u = 0; u < 8; ++u) { const float v = vv[u]; "
               << combine("acc", "v") << " }\n        }\n";
            b2 << "        for (; c < " << lit(chunks, pwide) << "; c += " << Gs << "u) {\n";
            b2 << "            const float v = part[c * " << lit(outputs, pwide) << " + o]; " << combine("acc", "v")
               << "\n        }\n    }\n";
            b2 << "    red[g][j] = acc;\n    __syncthreads();\n";
            b2 << "    if (g < 8u) {\n        float s = red[g * " << Ss << "u][j];\n";
            b2 << "        #pragma unroll\n        for (int w = 1; w < " << Ss << "; ++w) { const float v = red[g * "
               << Ss << "u + w][j]; " << combine("s", "v") << " }\n";
            b2 << "        red2[g][j] = s;\n    }\n    __syncthreads();\n";
            b2 << "    if (g == 0u && o < " << lit(outputs, pwide) << ") {\n";
            b2 << "        float s = red2[0][j];\n";
            b2 << "        #pragma unroll\n        for (int w = 1; w < 8; ++w) { const float v = red2[w][j]; "
               << combine("s", "v") << " }\n";
            b2 << "        out[o] = s;\n    }\n";
            launch_spec l2;
            l2.name = "pb_reduce_comb_" + hex64(hash_string(b2.str())).substr(0, 8);
            std::ostringstream s2;
            s2 << kernel_prelude() << "extern \"C\" __global__ void __launch_bounds__(512) " << l2.name
               << "(const float* __restrict__ part, float* __restrict__ out) {\n" << b2.str() << "}\n";
            l2.source = s2.str();
            l2.schedule = std::string(is_sum ? "sum " : "max ") + what + " pass 2 (combine " +
                          std::to_string(chunks) + " partials, " + Gs + " interleaved groups, in fixed order)";
            l2.grid = {static_cast<uint32_t>((outputs + W - 1) / W), 1, 1};
            l2.block = {512, 1, 1};
            kernel_arg pa;
            pa.kind = arg_kind::temp;
            pa.index = partial;
            kernel_arg oa;
            oa.kind = arg_kind::temp;
            oa.index = out;
            l2.args = {pa, oa};
            finish_kernel(l2);
            p_.launches.push_back(std::move(l2));
        };
        if (inner == 1) {
            // Row reduction: one warp per output row, 8 rows per CTA.
            // Four consecutive elements per load: leaves must be unit-stride
            // (or broadcast) along the axis. A reduced axis followed by
            // extent-1 dimensions can carry any stride, so check it here.
            bool vec = A % 4 == 0;
            for (int li : order) {
                const vnode& v = r.b.nodes[static_cast<size_t>(li)];
                const int64_t sa = v.map.st[ax];
                if (sa == 1) {
                    if (affine_at(v.map, r.b.lo) % 4 != 0) vec = false;
                    for (size_t d = 0; d < ax; ++d)
                        if (v.map.st[d] % 4 != 0 && S[d] > 1) vec = false;
                } else if (sa != 0) {
                    vec = false;
                }
            }
            const int V = vec ? 4 : 1;
            // Few long rows: a warp per row would leave too few CTAs to
            // spread evenly over the SMs, so the 8 warps of a CTA share one
            // row instead (threads stride the row, four loads in flight per
            // leaf, then the warps combine in warp order).
            const bool block_row = outer < 148 * 8 * 8 && A >= 2048;
            if (block_row) {
                // Longer rows take bigger CTAs: more, shorter waves of equal
                // CTAs leave a smaller partial last wave.
                threads = A >= 16384 ? 1024 : (A >= 8192 ? 512 : 256);
                const int64_t step = static_cast<int64_t>(threads) * V;
                const int warps = threads / 32;
                body << "    __shared__ float red[" << warps << "];\n";
                body << "    const pb_u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;\n";
                body << "    const " << I << " row = (" << I << ")blockIdx.x;\n";
                body << "    " << I << " t = row;\n";
                for (int d = static_cast<int>(ax) - 1; d >= 0; --d) {
                    body << "    const " << I << " c" << d << " = t % " << lit(S[static_cast<size_t>(d)], wide)
                         << "; t /= " << lit(S[static_cast<size_t>(d)], wide) << ";\n";
                }
                for (int d = static_cast<int>(ax) + 1; d < R; ++d) body << "    const " << I << " c" << d << " = 0;\n";
                const char* comps[4] = {"x", "y", "z", "w"};
                // Loads of the leaves at row offset `kexpr` into x<u>_<leaf>.
                auto loads = [&](const std::string& kexpr, const std::string& u, const std::string& ind) {
                    body << ind << "const " << I << " c" << ax << "_" << u << " = " << kexpr << ";\n";
                    std::vector<std::string> cv = cvar;
                    cv[ax] = "c" + std::to_string(ax) + "_" + u;
                    for (size_t li = 0; li < order.size(); ++li) {
                        const vnode& v = r.b.nodes[static_cast<size_t>(order[li])];
                        const std::string base = "in" + std::to_string(v.buffer);
                        const std::string addr = address(v.map, cv, wide, -1);
                        const std::string nm = "x" + u + "_" + std::to_string(li);
                        if (V == 4 && v.map.st[ax] == 1)
                            body << ind << "const float4 " << nm << " = pb_ld4(" << base << " + " << addr << ");\n";
                        else if (V == 4)
                            body << ind << "const float " << nm << "s = pb_ld(" << base << " + " << addr
                                 << "); const float4 " << nm << " = make_float4(" << nm << "s, " << nm << "s, " << nm
                                 << "s, " << nm << "s);\n";
                        else
                            body << ind << "const float " << nm << " = pb_ld(" << base << " + " << addr << ");\n";
                    }
                };
                auto fold = [&](const std::string& u, const std::string& ind) {
                    for (int e = 0; e < V; ++e) {
                        body << ind << "{ const float v = pb_e0(";
                        for (size_t li = 0; li < order.size(); ++li)
                            body << (li ? ", " : "") << "x" << u << "_" << li
                                 << (V == 4 ? std::string(".") + comps[e] : "");
                        body << "); " << combine("acc", "v") << " }\n";
                    }
                };
                body << "    float acc = " << init << ";\n";
                body << "    " << I << " k = threadIdx.x * " << V << "u;\n";
                body << "    for (; k + " << 3 * step << "u < " << lit(A, wide) << "; k += " << 4 * step << "u) {\n";
                for (int u = 0; u < 4; ++u)
                    loads("k + " + std::to_string(u * step) + "u", std::to_string(u), "        ");
                for (int u = 0; u < 4; ++u) fold(std::to_string(u), "        ");
                body << "    }\n";
                body << "    for (; k < " << lit(A, wide) << "; k += " << step << "u) {\n";
                loads("k", "0", "        ");
                fold("0", "        ");
                body << "    }\n";
                body << "    #pragma unroll\n    for (int o = 16; o > 0; o >>= 1) { const float v = "
                        "__shfl_xor_sync(0xffffffffu, acc, o); "
                     << combine("acc", "v") << " }\n";
                body << "    if (lane == 0) red[warp] = acc;\n    __syncthreads();\n";
                body << "    if (threadIdx.x == 0) {\n        float s2 = red[0];\n";
                body << "        #pragma unroll\n        for (int w = 1; w < " << warps << "; ++w) { const float v = red[w]; "
                     << combine("s2", "v") << " }\n        out[row] = s2;\n    }\n";
                l.grid = {static_cast<uint32_t>(outer), 1, 1};
                desc = "row reduction (CTA of " + std::to_string(threads) + " per row, 4 loads in flight) V=" +
                       std::to_string(V);
            } else {
                body << "    const pb_u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;\n";
                body << "    const " << I << " row = (" << I << ")blockIdx.x * 8u + warp;\n";
                body << "    if (row >= " << lit(outer, wide) << ") return;\n";
                body << "    " << I << " t = row;\n";
                for (int d = static_cast<int>(ax) - 1; d >= 0; --d) {
                    body << "    const " << I << " c" << d << " = t % " << lit(S[static_cast<size_t>(d)], wide) << "; t /= "
                         << lit(S[static_cast<size_t>(d)], wide) << ";\n";
                }
                // Dimensions after the axis all have extent 1 here.
                for (int d = static_cast<int>(ax) + 1; d < R; ++d)
                    body << "    const " << I << " c" << d << " = 0;\n";
                body << "    float acc = " << init << ";\n";
                body << "    for (" << I << " k = lane * " << V << "u; k < " << lit(A, wide) << "; k += " << 32 * V << "u) {\n";
                body << "        const " << I << " c" << ax << " = k;\n";
                for (size_t li = 0; li < order.size(); ++li) {
                    const vnode& v = r.b.nodes[static_cast<size_t>(order[li])];
                    const std::string base = "in" + std::to_string(v.buffer);
                    const std::string addr = address(v.map, cvar, wide, -1);
                    const int64_t sa = v.map.st[ax];
                    if (V == 4 && sa == 1)
                        body << "        const float4 x" << li << " = pb_ld4(" << base << " + " << addr << ");\n";
                    else if (V == 4)
                        body << "        const float s" << li << " = pb_ld(" << base << " + " << addr
                             << "); const float4 x" << li << " = make_float4(s" << li << ", s" << li << ", s" << li
                             << ", s" << li << ");\n";
                    else
                        body << "        const float x" << li << " = pb_ld(" << base << " + " << addr << ");\n";
                }
                const char* comps[4] = {"x", "y", "z", "w"};
                for (int e = 0; e < V; ++e) {
                    body << "        { const float v = pb_e0(";
                    for (size_t li = 0; li < order.size(); ++li) {
                        if (li) body << ", ";
                        body << "x" << li << (V == 4 ? std::string(".") + comps[e] : "");
                    }
                    body << "); " << combine("acc", "v") << " }\n";
                }
                body << "    }\n";
                body << "    #pragma unroll\n    for (int o = 16; o > 0; o >>= 1) { const float v = __shfl_xor_sync(0xffffffffu, acc, o); "
                     << combine("acc", "v") << " }\n";
                body << "    if (lane == 0) out[row] = acc;\n";
                const int64_t ctas = (outer + 7) / 8;
                l.grid = {static_cast<uint32_t>(ctas), 1, 1};
                desc = "row reduction (warp per row) V=" + std::to_string(V);
            }
        } else if (R >= 2 && static_cast<int>(ax) == R - 2 && S[static_cast<size_t>(R - 1)] % 4 == 0 &&
                   S[static_cast<size_t>(R - 1)] >= 4 && outer <= 65535 && [&] {
                       for (int li : order) {
                           const vnode& v = r.b.nodes[static_cast<size_t>(li)];
                           const int64_t sc = v.map.st[static_cast<size_t>(R - 1)];
                           if (sc != 0 && sc != 1) return false;
                           if (sc == 0) continue;
                           if (affine_at(v.map, r.b.lo) % 4 != 0) return false;
                           for (int d = 0; d < R - 1; ++d)
                               if (v.map.st[static_cast<size_t>(d)] % 4 != 0 && S[static_cast<size_t>(d)] > 1) return false;
                       }
                       return true;
                   }()) {
            // Reduction over the second-to-last axis of an [..., A, C]
            // operand whose rows are unit-stride and 16-byte aligned (axis 0
            // of a 2-D operand; the middle axis of [B, A, C], one batch per
            // blockIdx.z): column tiles of 128 (a float4 per lane);
            // the 8 warps of a CTA take every 8th row of the CTA's row chunk
            // (eight float4 loads in flight per lane), then combine their
            // partials in warp order through shared memory. Rows narrower
            // than 128 columns (down to 4) pack several rows into one warp
            // load: LPR
            // lanes per row (a power of two covering the row), RPW = 32 / LPR
            // rows per warp; lanes holding the same columns are combined in
            // (warp, row) order. Row chunks fill the GPU as in the strided
            // form; chunk partials are combined in chunk order, so results
            // do not depend on scheduling.
            const int64_t C = S[static_cast<size_t>(R - 1)];
            const int64_t col_tiles = (C + 127) / 128;
            int lpr = 32;
            if (C < 128) {
                lpr = 1;
                while (lpr * 4 < C) lpr *= 2;
            }
            const int rpw = 32 / lpr;
            // Four CTAs per SM already keep 128 KB of loads in flight per SM;
            // more row chunks would only lengthen pass 2.
            const int64_t target = 148 * 4;
            int64_t chunks = std::max<int64_t>(
                1, std::min<int64_t>((target + col_tiles * outer - 1) / (col_tiles * outer), A / (64 * rpw)));
            const int64_t per = (A + chunks - 1) / chunks;
            chunks = (A + per - 1) / per;
            const int part = chunks > 1 ? new_temp(static_cast<size_t>(chunks * outputs) * sizeof(float)) : out;
            const bool pwide = wide || chunks * outputs >= (int64_t{1} << 31) - 4096;
            const std::string cax = "c" + std::to_string(ax), ccol = "c" + std::to_string(R - 1);
            const std::string PI = pwide ? "pb_u64" : "pb_u32";
            const char* comps[4] = {"x", "y", "z", "w"};
            auto combine4 = [&](std::ostringstream& os, const std::string& acc, const std::string& v,
                                const std::string& ind) {
                for (int e = 0; e < 4; ++e)
                    os << ind << combine(acc + "." + comps[e], v + "." + comps[e]) << "\n";
            };
            auto value4 = [&](std::ostringstream& os, const std::string& k, const std::string& dst,
                              const std::string& ind) {
                os << ind << "{\n" << ind << "    const " << I << " " << cax << " = " << k << ";\n";
                for (size_t li = 0; li < order.size(); ++li) {
                    const vnode& v = r.b.nodes[static_cast<size_t>(order[li])];
                    const std::string addr = address(v.map, cvar, wide, -1);
                    if (v.map.st[static_cast<size_t>(R - 1)] == 1)
                        os << ind << "    const float4 x" << li << " = pb_ld4(in" << v.buffer << " + " << addr << ");\n";
                    else
                        os << ind << "    const float s" << li << " = pb_ld(in" << v.buffer << " + " << addr
                           << "); const float4 x" << li << " = make_float4(s" << li << ", s" << li << ", s" << li
                           << ", s" << li << ");\n";
                }
                for (int e = 0; e < 4; ++e) {
                    os << ind << "    " << dst << "." << comps[e] << " = pb_e0(";
                    for (size_t li = 0; li < order.size(); ++li) os << (li ? ", " : "") << "x" << li << "." << comps[e];
                    os << ");\n";
                }
                os << ind << "}\n";
            };
            std::ostringstream b1;
            b1 << "    __shared__ float4 red[8][32];\n";
            b1 << "    const pb_u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;\n";
            b1 << "    const pb_u32 sub = lane / " << lpr << "u, lc = lane % " << lpr << "u;\n";
            b1 << "    (void)sub;\n";
            b1 << "    const " << I << " " << ccol << " = (" << I << ")blockIdx.x * 128u + lc * 4u;\n";
            b1 << "    const bool active = " << ccol << " < " << lit(C, wide) << ";\n";
            // Batch coordinates (the dimensions before the reduced axis).
            b1 << "    " << I << " bt = blockIdx.z;\n    (void)bt;\n";
            for (int d = static_cast<int>(ax) - 1; d >= 0; --d)
                b1 << "    const " << I << " c" << d << " = bt % " << lit(S[static_cast<size_t>(d)], wide) << "; bt /= "
                   << lit(S[static_cast<size_t>(d)], wide) << ";\n";
            b1 << "    const " << I << " k0 = (" << I << ")blockIdx.y * " << lit(per, wide) << ";\n";
            b1 << "    const " << I << " k1 = k0 + " << lit(per, wide) << " < " << lit(A, wide) << " ? k0 + "
               << lit(per, wide) << " : " << lit(A, wide) << ";\n";
            b1 << "    float4 acc = make_float4(" << init << ", " << init << ", " << init << ", " << init << ");\n";
            b1 << "    if (active) {\n";
            b1 << "        " << I << " k = k0 + warp * " << rpw << "u + sub;\n";
            b1 << "        for (; k + " << 56 * rpw << "u < k1; k += " << 64 * rpw << "u) {\n            float4 vv[8];\n";
            b1 << "            #pragma unroll\n            for (int u = 0; u < 8; ++u)\n";
            value4(b1, "k + " + std::to_string(8 * rpw) + "u * (" + I + ")u", "vv[u]", "            ");
            b1 << "            #pragma unroll\n            for (int u = 0; u < 8; ++u) {\n";
            combine4(b1, "acc", "vv[u]", "                ");
            b1 << "            }\n        }\n";
            b1 << "        for (; k < k1; k += " << 8 * rpw << "u) {\n            float4 v;\n";
            value4(b1, "k", "v", "            ");
            combine4(b1, "acc", "v", "            ");
            b1 << "        }\n    }\n";
            b1 << "    red[warp][lane] = acc;\n    __syncthreads();\n";
            b1 << "    if (warp == 0 && sub == 0u && active) {\n";
            b1 << "        float4 s = red[0][lc];\n";
            b1 << "        #pragma unroll 8\n        for (int q = 1; q < " << 8 * rpw << "; ++q) {\n"
               << "            const float4 v = red[q / " << rpw << "][(q % " << rpw << ") * " << lpr << " + lc];\n";
            combine4(b1, "s", "v", "            ");
            b1 << "        }\n";
            b1 << "        pb_st4(" << (chunks > 1 ? "part" : "out") << " + (" << PI << ")blockIdx.y * "
               << lit(outputs, pwide) << " + (" << PI << ")blockIdx.z * " << lit(C, pwide) << " + (" << PI << ")"
               << ccol << ", s);\n    }\n";
            launch_spec l1;
            l1.name = "pb_reduce_cols_" + hex64(hash_string(src.str() + b1.str())).substr(0, 8);
            std::ostringstream s1;
            s1 << src.str() << "extern \"C\" __global__ void __launch_bounds__(256) " << l1.name << "(";
            for (size_t i = 0; i < r.k.leaves.size(); ++i) s1 << "const float* __restrict__ in" << i << ", ";
            s1 << "float* __restrict__ " << (chunks > 1 ? "part" : "out") << ") {\n" << b1.str() << "}\n";
            l1.source = s1.str();
            l1.schedule = std::string(is_sum ? "sum " : "max ") + "column reduction (128-column tiles, 8 warps on " +
                          "interleaved rows" + (rpw > 1 ? ", " + std::to_string(rpw) + " rows per warp load" : "") +
                          ", " + std::to_string(chunks) + " row chunks of " + std::to_string(per) + ")";
            l1.grid = {static_cast<uint32_t>(col_tiles), static_cast<uint32_t>(chunks), static_cast<uint32_t>(outer)};
            l1.block = {256, 1, 1};
            l1.args = r.k.leaves;
            kernel_arg pa;
            pa.kind = arg_kind::temp;
            pa.index = part;
            l1.args.push_back(pa);
            finish_kernel(l1);
            p_.launches.push_back(std::move(l1));
            if (chunks > 1) emit_chunk_combine(part, chunks, "column reduction");
            return out;
        } else {
            // Strided reduction: one thread per output, coalesced across the
            // inner dimensions. When the outputs alone give too few CTAs to
            // fill the GPU (sum(x, 0) on a tall x), the reduction axis is
            // also split into row chunks: pass 1 writes one partial per
            // (chunk, output), pass 2 combines the partials of each output in
            // chunk order, so the result does not depend on scheduling.
            const int64_t col_ctas = (outputs + 255) / 256;
            const int64_t target = 148 * 8;
            int64_t chunks = 1;
            if (col_ctas * 2 < target && A >= 64)
                chunks = std::min<int64_t>((target + col_ctas - 1) / col_ctas, A / 32);
            if (chunks > 1) {
                const int64_t per = (A + chunks - 1) / chunks;
                chunks = (A + per - 1) / per;
                const int partial = new_temp(static_cast<size_t>(chunks * outputs) * sizeof(float));
                const bool pwide = wide || chunks * outputs >= (int64_t{1} << 31) - 4096;
                const std::string PI = pwide ? "pb_u64" : "pb_u32";
                std::ostringstream b1;
                b1 << "    const " << I << " o = (" << I << ")blockIdx.x * 256u + threadIdx.x;\n";
                b1 << "    if (o >= " << lit(outputs, wide) << ") return;\n";
                b1 << "    " << I << " t = o;\n";
                for (int d = R - 1; d >= 0; --d) {
                    if (static_cast<size_t>(d) == ax) continue;
                    b1 << "    const " << I << " c" << d << " = t % " << lit(S[static_cast<size_t>(d)], wide)
                       << "; t /= " << lit(S[static_cast<size_t>(d)], wide) << ";\n";
                }
                b1 << "    const " << I << " k0 = (" << I << ")blockIdx.y * " << lit(per, wide) << ";\n";
                b1 << "    const " << I << " k1 = k0 + " << lit(per, wide) << " < " << lit(A, wide) << " ? k0 + "
                   << lit(per, wide) << " : " << lit(A, wide) << ";\n";
                b1 << "    float acc = " << init << ";\n";
                emit_strided_loop(b1, "k0", "k1");
                b1 << "    part[(" << PI << ")blockIdx.y * " << lit(outputs, pwide) << " + (" << PI << ")o] = acc;\n";
                launch_spec l1;
                l1.name = "pb_reduce_part_" + hex64(hash_string(src.str() + b1.str())).substr(0, 8);
                std::ostringstream s1;
                s1 << src.str() << "extern \"C\" __global__ void __launch_bounds__(256) " << l1.name << "(";
                for (size_t i = 0; i < r.k.leaves.size(); ++i) s1 << "const float* __restrict__ in" << i << ", ";
                s1 << "float* __restrict__ part) {\n" << b1.str() << "}\n";
                l1.source = s1.str();
                l1.schedule = std::string(is_sum ? "sum " : "max ") + "strided reduction pass 1 (" +
                              std::to_string(chunks) + " row chunks of " + std::to_string(per) + ")";
                l1.grid = {static_cast<uint32_t>(col_ctas), static_cast<uint32_t>(chunks), 1};
                l1.block = {256, 1, 1};
                l1.args = r.k.leaves;
                kernel_arg pa;
                pa.kind = arg_kind::temp;
                pa.index = partial;
                l1.args.push_back(pa);
                finish_kernel(l1);
                p_.launches.push_back(std::move(l1));

                emit_chunk_combine(partial, chunks, "strided reduction");
                return out;
            }
            body << "    const " << I << " o = (" << I << ")blockIdx.x * 256u + threadIdx.x;\n";
            body << "    if (o >= " << lit(outputs, wide) << ") return;\n";
            body << "    " << I << " t = o;\n";
            for (int d = R - 1; d >= 0; --d) {
                if (static_cast<size_t>(d) == ax) continue;
                body << "    const " << I << " c" << d << " = t % " << lit(S[static_cast<size_t>(d)], wide) << "; t /= "
                     << lit(S[static_cast<size_t>(d)], wide) << ";\n";
            }
            body << "    float acc = " << init << ";\n";
            emit_strided_loop(body, "(" + I + ")0", lit(A, wide));
            body << "    out[o] = acc;\n";
            const int64_t ctas = (outputs + 255) / 256;
            l.grid = {static_cast<uint32_t>(ctas), 1, 1};
            desc = "strided reduction (thread per output)";
        }
        l.name = "pb_reduce_" + hex64(hash_string(src.str() + body.str())).substr(0, 8);
        src << "extern \"C\" __global__ void __launch_bounds__(" << threads << ") " << l.name << "(";
        for (size_t i = 0; i < r.k.leaves.size(); ++i) src << "const float* __restrict__ in" << i << ", ";
        src << "float* __restrict__ out) {\n" << body.str() << "}\n";
        l.source = src.str();
        l.schedule = std::string(is_sum ? "sum " : "max ") + desc;
        l.block = {static_cast<uint32_t>(threads), 1, 1};
        l.args = r.k.leaves;
        kernel_arg o;
        o.kind = arg_kind::temp;
        o.index = out;
        l.args.push_back(o);
        finish_kernel(l);
        p_.launches.push_back(std::move(l));
        return out;
    }

    // --------------------------------------------------------- softmax --
    int lowerer::emit_softmax(int id, int x) {
        const gnode& n = g_.nodes[static_cast<size_t>(id)];
        const size_t ax = n.shape.size() - 1;
        row_operand r = row_prologue(x, ax);
        const std::vector<index_t>& S = r.shape;
        rank_ = static_cast<int>(S.size());
        const int R = rank_;
        int64_t rows = 1;
        for (size_t d = 0; d < ax; ++d) rows *= S[d];
        const int64_t A = S[ax];
        const int out = new_temp(static_cast<size_t>(rows * A) * sizeof(float));
        bool wide = needs_wide({r.b}, S) || rows * A >= (int64_t{1} << 31) - 4096;
        const std::string I = wide ? "pb_u64" : "pb_u32";
        std::vector<int> order;
        std::ostringstream src;
        src << kernel_prelude();
        src << emit_expr_function(r.b, "0", order);
        bool vec = A % 4 == 0;
        for (int li : order) {
            const vnode& v = r.b.nodes[static_cast<size_t>(li)];
            if (v.map.st[ax] == 1) {
                if (affine_at(v.map, r.b.lo) % 4 != 0) vec = false;
                for (size_t d = 0; d < ax; ++d)
                    if (v.map.st[d] % 4 != 0 && S[d] > 1) vec = false;
            } else if (v.map.st[ax] != 0) {
                vec = false;  // strided along the axis (trailing extent-1 dimensions)
            }
        }
        const int V = vec ? 4 : 1;
        const int T0 = A >= 2048 ? 256 : (A >= 512 ? 128 : 32);
        const int64_t NI = (A + static_cast<int64_t>(T0) * V - 1) / (static_cast<int64_t>(T0) * V);
        const bool in_registers = NI * V <= 64;
        // Longer rows stream twice (online max/sum, then the write). The
        // CTAs resident at once are capped so that their rows stay in L2
        // and the second read comes from L2, not HBM: four 256-thread CTAs
        // per SM while their rows take at most 48 MB, three up to 64 MB
        // (16 KB of loads in flight per CTA, and enough CTAs to hide each
        // other's barriers), else one 1024-thread CTA per SM (64 KB of loads
        // in flight). Measured on one box against the unlimited 256-thread
        // grid, as fractions of one read + one write: 0.64 -> 0.83 at
        // [8192, 16388], 0.65 -> 0.73 at [16384, 20000], 0.63 -> 0.71 at
        // [4096, 32768], 0.62 -> 0.72 at [2048, 65536].
        const int64_t row_bytes = A * 4;
        const int stream_per_sm = 148 * 4 * row_bytes <= (int64_t{48} << 20)   ? 4
                                  : 148 * 3 * row_bytes <= (int64_t{64} << 20) ? 3
                                                                               : 1;
        // Fewer rows than the streaming form keeps resident, each of up to
        // 8 x 16384 values: a cluster of C CTAs (512 threads, up to 32
        // values each in registers) per row, the CTAs' maxima and sums
        // exchanged through distributed shared memory -- one read and one
        // write, and rows x C CTAs to spread over the SMs. (With rows
        // enough to fill the GPU the persistent streaming CTAs win: on one
        // box [64, 65536] 0.31 -> 0.43 of one read + one write with
        // clusters, but [8192, 16388] 0.83 -> 0.72 and [2048, 65536]
        // 0.72 -> 0.62.)
        const int64_t cl_cap = 16384;
        const int cluster_c = in_registers || A > 8 * cl_cap || rows >= int64_t{148} * stream_per_sm
                                  ? 1
                                  : static_cast<int>((A + cl_cap - 1) / cl_cap);
        const bool clustered = cluster_c > 1;
        const int T = in_registers ? T0 : (clustered ? 512 : (stream_per_sm > 1 ? 256 : 1024));
        std::vector<std::string> cvar(static_cast<size_t>(R));
        for (int d = 0; d < R; ++d) cvar[static_cast<size_t>(d)] = "c" + std::to_string(d);
        const char* comps[4] = {"x", "y", "z", "w"};
        std::ostringstream body;
        // Separate partial arrays for the max and the sum: each reduction
        // then needs one barrier (the other reduction's barrier orders a
        // row's reads before the next row's writes).
        body << "    __shared__ float red_m[32], red_s[32];\n";
        body << "    const pb_u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;\n";
        // Declares the row coordinates c0..c(ax-1) of row `r` in a scope.
        auto emit_row_coords = [&](const std::string& row_expr, const std::string& indent) {
            body << indent << I << " t = " << row_expr << ";\n";
            for (int d = static_cast<int>(ax) - 1; d >= 0; --d)
                body << indent << "const " << I << " c" << d << " = t % " << lit(S[static_cast<size_t>(d)], wide)
                     << "; t /= " << lit(S[static_cast<size_t>(d)], wide) << ";\n";
            body << indent << "(void)t;\n";
        };
        // Loads the operand value vector at column k into float xv[V].
        auto emit_load = [&](const std::string& k, const std::string& dst, const std::string& indent) {
            body << indent << "{\n" << indent << "    const " << I << " c" << ax << " = " << k << ";\n";
            for (size_t li = 0; li < order.size(); ++li) {
                const vnode& v = r.b.nodes[static_cast<size_t>(order[li])];
                const std::string base = "in" + std::to_string(v.buffer);
                const std::string addr = address(v.map, cvar, wide, -1);
                if (V == 4 && v.map.st[ax] == 1)
                    body << indent << "    const float4 x" << li << " = pb_ld4(" << base << " + " << addr << ");\n";
                else if (V == 4)
                    body << indent << "    const float s" << li << " = pb_ld(" << base << " + " << addr
                         << "); const float4 x" << li << " = make_float4(s" << li << ", s" << li << ", s" << li
                         << ", s" << li << ");\n";
                else
                    body << indent << "    const float x" << li << " = pb_ld(" << base << " + " << addr << ");\n";
            }
            for (int e = 0; e < V; ++e) {
                body << indent << "    " << dst << "[" << e << "] = pb_e0(";
                for (size_t li = 0; li < order.size(); ++li) {
                    if (li) body << ", ";
                    body << "x" << li << (V == 4 ? std::string(".") + comps[e] : "");
                }
                body << ");\n";
            }
            body << indent << "}\n";
        };
        auto block_reduce = [&](const std::string& var, bool is_max) {
            const std::string comb = is_max ? (var + " = " + var + " > v ? " + var + " : v;")
                                            : (var + " = " + var + " + v;");
            body << "        #pragma unroll\n        for (int o = 16; o > 0; o >>= 1) { const float v = __shfl_xor_sync(0xffffffffu, "
                 << var << ", o); " << comb << " }\n";
            if (T > 32) {
                // Every thread combines the warps' partials in the same order,
                // so all hold the same value.
                const std::string red = is_max ? "red_m" : "red_s";
                body << "        if (lane == 0) " << red << "[warp] = " << var << ";\n        __syncthreads();\n";
                body << "        " << var << " = " << red << "[0];\n";
                body << "        #pragma unroll\n        for (int w = 1; w < " << T / 32 << "; ++w) { const float v = "
                     << red << "[w]; " << comb << " }\n";
            }
        };
        const std::string orow = "row * " + lit(A, wide);
        if (in_registers) {
            // Software pipeline over the CTA's rows: the next row's loads are
            // issued before this row's reductions, so HBM stays busy while
            // the block waits at its barriers.
            auto emit_row_loads = [&](const std::string& row_expr, const std::string& dst, const std::string& indent) {
                body << indent << "{\n";
                emit_row_coords(row_expr, indent + "    ");
                body << indent << "    #pragma unroll\n" << indent << "    for (int it = 0; it < " << NI << "; ++it) {\n";
                body << indent << "        const " << I << " k = ((" << I << ")it * " << T << "u + threadIdx.x) * " << V
                     << "u;\n";
                body << indent << "        if (k < " << lit(A, wide) << ") ";
                emit_load("k", dst + "[it]", indent + "        ");
                body << indent << "        else { ";
                for (int e = 0; e < V; ++e) body << dst << "[it][" << e << "] = PB_NEG_FLT_MAX; ";
                body << "}\n" << indent << "    }\n" << indent << "}\n";
            };
            body << "    float xn[" << NI << "][" << V << "];\n";
            body << "    if (blockIdx.x < " << lit(rows, wide) << ")\n";
            emit_row_loads("blockIdx.x", "xn", "    ");
            body << "    for (" << I << " row = blockIdx.x; row < " << lit(rows, wide) << "; row += gridDim.x) {\n";
            body << "        float x[" << NI << "][" << V << "];\n";
            body << "        #pragma unroll\n        for (int it = 0; it < " << NI << "; ++it)\n";
            body << "            #pragma unroll\n            for (int e = 0; e < " << V << "; ++e) x[it][e] = xn[it][e];\n";
            body << "        if (row + gridDim.x < " << lit(rows, wide) << ")\n";
            emit_row_loads("row + gridDim.x", "xn", "        ");
            body << "        float m = PB_NEG_FLT_MAX;\n";
            body << "        #pragma unroll\n        for (int it = 0; it < " << NI << "; ++it)\n";
            body << "            #pragma unroll\n            for (int e = 0; e < " << V
                 << "; ++e) m = m > x[it][e] ? m : x[it][e];\n";
            block_reduce("m", true);
            body << "        float s = 0.0f;\n";
            body << "        #pragma unroll\n        for (int it = 0; it < " << NI << "; ++it) {\n";
            body << "            const " << I << " k = ((" << I << ")it * " << T << "u + threadIdx.x) * " << V << "u;\n";
            body << "            if (k < " << lit(A, wide) << ") {\n";
            body << "                #pragma unroll\n                for (int e = 0; e < " << V
                 << "; ++e) { x[it][e] = __expf(x[it][e] - m); s = s + x[it][e]; }\n";
            body << "            }\n        }\n";
            block_reduce("s", false);
            // One IEEE division per row, then multiplies: within 1.5 ulp of
            // x / s (softmax is compared within 1e-5), and 3 % faster than a
            // division per element (measured on [65536, 4096]).
            body << "        const float rs = 1.0f / s;\n";
            body << "        #pragma unroll\n        for (int it = 0; it < " << NI << "; ++it) {\n";
            body << "            const " << I << " k = ((" << I << ")it * " << T << "u + threadIdx.x) * " << V << "u;\n";
            body << "            if (k < " << lit(A, wide) << ") {\n";
            if (V == 4)
                body << "                pb_st4(out + " << orow << " + k, make_float4(x[it][0] * rs, x[it][1] * rs, x[it][2] * rs, x[it][3] * rs));\n";
            else
                body << "                out[" << orow << " + k] = x[it][0] * rs;\n";
            body << "            }\n        }\n";
        } else if (clustered) {
            // CTA `rank` of the row's cluster holds columns [rank * SEG,
            // (rank + 1) * SEG) in registers. Cluster barriers (release /
            // acquire) order each CTA's shared partial before the others
            // read it with ld.shared::cluster; all read the C partials in
            // rank order, so every CTA combines them identically. The last
            // barrier keeps each CTA's shared memory alive until the others
            // have read it.
            const int64_t seg = ((A + cluster_c - 1) / cluster_c + 3) / 4 * 4;
            const int64_t ni = (seg + static_cast<int64_t>(T) * V - 1) / (static_cast<int64_t>(T) * V);
            body << "    __shared__ float cl_part[2];\n";
            body << "    pb_u32 rank;\n    asm volatile(\"mov.u32 %0, %%cluster_ctarank;\" : \"=r\"(rank));\n";
            body << "    const " << I << " row = (" << I << ")blockIdx.x / " << cluster_c << "u;\n";
            body << "    {\n";
            emit_row_coords("row", "        ");
            body << "        const " << I << " k0 = (" << I << ")rank * " << lit(seg, wide) << ";\n";
            body << "        const " << I << " k1 = k0 + " << lit(seg, wide) << " < " << lit(A, wide) << " ? k0 + "
                 << lit(seg, wide) << " : " << lit(A, wide) << ";\n";
            body << "        float x[" << ni << "][" << V << "];\n";
            body << "        float m = PB_NEG_FLT_MAX;\n";
            body << "        #pragma unroll\n        for (int it = 0; it < " << ni << "; ++it) {\n";
            body << "            const " << I << " k = k0 + ((" << I << ")it * " << T << "u + threadIdx.x) * " << V
                 << "u;\n";
            body << "            if (k < k1) {\n";
            emit_load("k", "x[it]", "                ");
            body << "                #pragma unroll\n                for (int e = 0; e < " << V
                 << "; ++e) m = m > x[it][e] ? m : x[it][e];\n";
            body << "            }\n        }\n";
            block_reduce("m", true);
            body << "        if (threadIdx.x == 0) cl_part[0] = m;\n";
            body << "        asm volatile(\"barrier.cluster.arrive.release;\\n\\tbarrier.cluster.wait.acquire;\" ::: \"memory\");\n";
            body << "        m = PB_NEG_FLT_MAX;\n";
            body << "        #pragma unroll\n        for (pb_u32 q = 0; q < " << cluster_c << "u; ++q) {\n"
                 << "            pb_u32 ra;\n            float v;\n"
                 << "            asm volatile(\"mapa.shared::cluster.u32 %0, %1, %2;\" : \"=r\"(ra) : \"r\"((pb_u32)__cvta_generic_to_shared(&cl_part[0])), \"r\"(q));\n"
                 << "            asm volatile(\"ld.shared::cluster.f32 %0, [%1];\" : \"=f\"(v) : \"r\"(ra) : \"memory\");\n"
                 << "            m = m > v ? m : v;\n        }\n";
            body << "        float s = 0.0f;\n";
            body << "        #pragma unroll\n        for (int it = 0; it < " << ni << "; ++it) {\n";
            body << "            const " << I << " k = k0 + ((" << I << ")it * " << T << "u + threadIdx.x) * " << V
                 << "u;\n";
            body << "            if (k < k1) {\n";
            body << "                #pragma unroll\n                for (int e = 0; e < " << V
                 << "; ++e) { x[it][e] = __expf(x[it][e] - m); s = s + x[it][e]; }\n";
            body << "            }\n        }\n";
            block_reduce("s", false);
            body << "        if (threadIdx.x == 0) cl_part[1] = s;\n";
            body << "        asm volatile(\"barrier.cluster.arrive.release;\\n\\tbarrier.cluster.wait.acquire;\" ::: \"memory\");\n";
            body << "        s = 0.0f;\n";
            body << "        #pragma unroll\n        for (pb_u32 q = 0; q < " << cluster_c << "u; ++q) {\n"
                 << "            pb_u32 ra;\n            float v;\n"
                 << "            asm volatile(\"mapa.shared::cluster.u32 %0, %1, %2;\" : \"=r\"(ra) : \"r\"((pb_u32)__cvta_generic_to_shared(&cl_part[1])), \"r\"(q));\n"
                 << "            asm volatile(\"ld.shared::cluster.f32 %0, [%1];\" : \"=f\"(v) : \"r\"(ra) : \"memory\");\n"
                 << "            s = s + v;\n        }\n";
            body << "        asm volatile(\"barrier.cluster.arrive.release;\" ::: \"memory\");\n";
            body << "        const float rs = 1.0f / s;\n";
            body << "        #pragma unroll\n        for (int it = 0; it < " << ni << "; ++it) {\n";
            body << "            const " << I << " k = k0 + ((" << I << ")it * " << T << "u + threadIdx.x) * " << V
                 << "u;\n";
            body << "            if (k < k1) {\n";
            if (V == 4)
                body << "                pb_st4(out + " << orow
                     << " + k, make_float4(x[it][0] * rs, x[it][1] * rs, x[it][2] * rs, x[it][3] * rs));\n";
            else
                body << "                out[" << orow << " + k] = x[it][0] * rs;\n";
            body << "            }\n        }\n";
            body << "        asm volatile(\"barrier.cluster.wait.acquire;\" ::: \"memory\");\n";
        } else {
            // Rows too long for registers: an online pass keeps a running
            // (max, sum) per thread -- four vector loads per step, the sum
            // rescaled once per step by exp(old max - new max) -- and the
            // block combines the pairs; a second pass writes
            // exp(x - m) * (1 / s). Two reads and one write per element.
            const int64_t step = static_cast<int64_t>(T) * V;
            body << "    for (" << I << " row = blockIdx.x; row < " << lit(rows, wide) << "; row += gridDim.x) {\n";
            emit_row_coords("row", "        ");
            body << "        float m = PB_NEG_FLT_MAX, s = 0.0f;\n";
            body << "        " << I << " k = threadIdx.x * " << V << "u;\n";
            body << "        for (; k + " << 3 * step << "u < " << lit(A, wide) << "; k += " << 4 * step << "u) {\n";
            body << "            float xv[4][" << V << "];\n";
            for (int u = 0; u < 4; ++u)
                emit_load("k + " + std::to_string(u * step) + "u", "xv[" + std::to_string(u) + "]", "            ");
            body << "            float bm = m;\n";
            body << "            #pragma unroll\n            for (int u = 0; u < 4; ++u)\n"
                 << "                #pragma unroll\n                for (int e = 0; e < " << V
                 << "; ++e) bm = bm > xv[u][e] ? bm : xv[u][e];\n";
            body << "            s = s * __expf(m - bm);\n            m = bm;\n";
            body << "            #pragma unroll\n            for (int u = 0; u < 4; ++u)\n"
                 << "                #pragma unroll\n                for (int e = 0; e < " << V
                 << "; ++e) s = s + __expf(xv[u][e] - m);\n";
            body << "        }\n";
            body << "        for (; k < " << lit(A, wide) << "; k += " << step << "u) {\n";
            body << "            float xv[" << V << "];\n";
            emit_load("k", "xv", "            ");
            body << "            float bm = m;\n";
            body << "            #pragma unroll\n            for (int e = 0; e < " << V
                 << "; ++e) bm = bm > xv[e] ? bm : xv[e];\n";
            body << "            s = s * __expf(m - bm);\n            m = bm;\n";
            body << "            #pragma unroll\n            for (int e = 0; e < " << V
                 << "; ++e) s = s + __expf(xv[e] - m);\n";
            body << "        }\n";
            // Pair combine: the larger max wins, the other sum is rescaled.
            auto pair_combine = [&](const std::string& om, const std::string& os, const std::string& ind) {
                body << ind << "{ const float nm = m > " << om << " ? m : " << om << "; s = s * __expf(m - nm) + "
                     << os << " * __expf(" << om << " - nm); m = nm; }\n";
            };
            body << "        #pragma unroll\n        for (int o = 16; o > 0; o >>= 1) {\n"
                 << "            const float om = __shfl_xor_sync(0xffffffffu, m, o);\n"
                 << "            const float os = __shfl_xor_sync(0xffffffffu, s, o);\n";
            pair_combine("om", "os", "            ");
            body << "        }\n";
            if (T > 32) {
                body << "        if (lane == 0) { red_m[warp] = m; red_s[warp] = s; }\n        __syncthreads();\n";
                body << "        m = red_m[0];\n        s = red_s[0];\n";
                body << "        #pragma unroll\n        for (int w = 1; w < " << T / 32 << "; ++w) {\n"
                     << "            const float om = red_m[w], os = red_s[w];\n";
                pair_combine("om", "os", "            ");
                body << "        }\n        __syncthreads();  // red_m/red_s are rewritten by the next row\n";
            }
            // The write pass walks the row from its end: the online pass
            // read the end last, so that part is the likeliest still in L2.
            body << "        const float rs = 1.0f / s;\n";
            body << "        {\n";
            body << "            const " << I << " k0 = threadIdx.x * " << V << "u;\n";
            body << "            long long j = k0 < " << lit(A, wide) << " ? (long long)((" << lit(A, wide)
                 << " - 1u - k0) / " << step << "u) : -1;\n";
            body << "            for (; j >= 3; j -= 4) {\n";
            body << "                float xv[4][" << V << "];\n";
            for (int u = 0; u < 4; ++u)
                emit_load("k0 + (" + I + ")(j - " + std::to_string(u) + ") * " + std::to_string(step) + "u",
                          "xv[" + std::to_string(u) + "]", "                ");
            for (int u = 0; u < 4; ++u) {
                const std::string kk = "k0 + (" + I + ")(j - " + std::to_string(u) + ") * " + std::to_string(step) + "u";
                if (V == 4)
                    body << "                pb_st4(out + " << orow << " + " << kk << ", make_float4(__expf(xv[" << u
                         << "][0] - m) * rs, __expf(xv[" << u << "][1] - m) * rs, __expf(xv[" << u
                         << "][2] - m) * rs, __expf(xv[" << u << "][3] - m) * rs));\n";
                else
                    body << "                out[" << orow << " + " << kk << "] = __expf(xv[" << u
                         << "][0] - m) * rs;\n";
            }
            body << "            }\n";
            body << "            for (; j >= 0; --j) {\n";
            body << "                const " << I << " kj = k0 + (" << I << ")j * " << step << "u;\n";
            body << "                float xv[" << V << "];\n";
            emit_load("kj", "xv", "                ");
            body << "                #pragma unroll\n                for (int e = 0; e < " << V << "; ++e) out["
                 << orow << " + kj + e] = __expf(xv[e] - m) * rs;\n";
            body << "            }\n        }\n";
        }
        body << "    }\n";
        launch_spec l;
        l.name = "pb_softmax_" + hex64(hash_string(src.str() + body.str())).substr(0, 8);
        src << "extern \"C\" __global__ void __launch_bounds__(" << T << ") " << l.name << "(";
        for (size_t i = 0; i < r.k.leaves.size(); ++i) src << "const float* __restrict__ in" << i << ", ";
        src << "float* __restrict__ out) {\n" << body.str() << "}\n";
        l.source = src.str();
        const int64_t per_sm = 2048 / T;
        l.grid = {static_cast<uint32_t>(std::min<int64_t>(rows, 148 * per_sm)), 1, 1};
        l.persistent_units = rows; // grid = CTAs resident at once, fixed at first launch
        if (clustered) {
            l.grid[0] = static_cast<uint32_t>(rows * cluster_c);
            l.persistent_units = 0;
            l.cluster_x = static_cast<uint32_t>(cluster_c);
        } else if (!in_registers) {
            l.grid[0] = static_cast<uint32_t>(std::min<int64_t>(rows, 148 * stream_per_sm));
            l.persistent_per_sm = stream_per_sm;
        }
        l.block = {static_cast<uint32_t>(T), 1, 1};
        l.schedule = "softmax row kernel T=" + std::to_string(T) + " V=" + std::to_string(V) +
                     (in_registers ? " (row in registers, next row prefetched, 1 read + 1 write)"
                      : clustered ? " (cluster of " + std::to_string(cluster_c) +
                                        " CTAs per row, row in registers, partials through DSMEM, 1 read + 1 write)"
                                  : std::string(" (online max/sum pass + write pass, 2 reads + 1 write)"));
        l.args = r.k.leaves;
        kernel_arg o;
        o.kind = arg_kind::temp;
        o.index = out;
        l.args.push_back(o);
        finish_kernel(l);
        p_.launches.push_back(std::move(l));
        return out;
    }

    // ------------------------------------------------------------- GEMM --
    int lowerer::emit_gemm(int id, int mm) {
        const gnode& m = g_.nodes[static_cast<size_t>(mm)];
        const gnode& root = g_.nodes[static_cast<size_t>(id)];
        const int64_t M = m.shape[0], N = m.shape[1];
        const int64_t K = g_.nodes[static_cast<size_t>(m.a)].shape[1];
        // Epilogue over the output coordinates, accumulator at `mm`.
        kernel k;
        std::vector<box> boxes;
        try {
            boxes = build_boxes(k, id, root.shape, mm);
        } catch (const not_fusable&) {
            if (id != mm) return -1;
            throw;
        } catch (const not_affine&) {
            return -1;
        }
        if (boxes.size() != 1) return -1;
        // A produced by a GEMM that nothing else reads arrives as 3xTF32
        // halves from that GEMM's epilogue: no split pass, no fp32 copy.
        gemm_temps shared;
        gemm_operand A;
        if (!presplit_operand(m.a, M, N, K, shared, A)) A = as_gemm_operand(m.a);
        const gemm_operand B = as_gemm_operand(m.b);
        int nonfinite = -1;
        if (const int t = emit_gemm_tc(id, boxes[0], k, A, B, M, N, K, &nonfinite, nullptr, -1, 0, &shared);
            t >= 0) {
            // Inf or NaN in an operand: the 3xTF32 expansion turns inf * 0
            // (an inf hi times a zero lo) into NaN where the reference's fp32
            // chain gives +-inf, so that case reruns on the CUDA cores with
            // the reference's own arithmetic (a k-ordered FMA chain), into
            // the same output; it returns at once when every value is finite.
            emit_gemm_simt(boxes[0], k, A, B, M, N, K, t, nonfinite);
            return t;
        }
        return emit_gemm_simt(boxes[0], k, A, B, M, N, K);
    }

    bool lowerer::presplit_operand(int a, int64_t M, int64_t N, int64_t K, gemm_temps& t, gemm_operand& op) {
        const gnode& h = g_.nodes[static_cast<size_t>(a)];
        if (a == g_.root || h.kind == expr_kind::input || g_.uses[static_cast<size_t>(a)] != 1 ||
            done_.count(a) != 0)
            return false;
        if (K % 32 != 0 || !tensor_core_gemm(M, N, K)) return false;
        const int mh = match_gemm(a);
        if (mh < 0) return false;
        const gnode& hm = g_.nodes[static_cast<size_t>(mh)];
        const int64_t Kh = g_.nodes[static_cast<size_t>(hm.a)].shape[1];
        if (hm.shape[0] != M || hm.shape[1] != K || !tensor_core_gemm(M, K, Kh)) return false;
        kernel kh;
        std::vector<box> boxes;
        try {
            boxes = build_boxes(kh, a, h.shape, mh);
        } catch (const not_fusable&) {
            return false;
        } catch (const not_affine&) {
            return false;
        }
        if (boxes.size() != 1) return false;
        auto temp = [](int i) {
            kernel_arg x;
            x.kind = arg_kind::temp;
            x.index = i;
            return x;
        };
        // The consumer's A halves and flag; the flag is cleared before the
        // producer runs (the consumer's own clear then leaves it alone).
        t.a_hi = new_temp(static_cast<size_t>(M * K) * 4);
        t.a_lo = new_temp(static_cast<size_t>(M * K) * 4);
        t.fa = new_temp(256);
        {
            launch_spec l;
            l.name = "pb_flag_clear";
            l.source = std::string(kernel_prelude()) +
                       "extern \"C\" __global__ void pb_flag_clear(int* f) { f[0] = 0; }\n";
            l.schedule = "clear the next GEMM's operand flag (its A comes from a split-output epilogue)";
            l.grid = {1, 1, 1};
            l.block = {1, 1, 1};
            l.args = {temp(t.fa)};
            finish_kernel(l);
            p_.launches.push_back(std::move(l));
        }
        const split_output so{t.a_hi, t.a_lo, t.fa, K};
        const gemm_operand Ah = as_gemm_operand(hm.a);
        const gemm_operand Bh = as_gemm_operand(hm.b);
        int nfh = -1;
        if (emit_gemm_tc(a, boxes[0], kh, Ah, Bh, M, K, Kh, &nfh, nullptr, -1, 0, nullptr, &so) < 0)
            throw std::logic_error("split-output GEMM was not eligible");
        emit_gemm_simt(boxes[0], kh, Ah, Bh, M, K, Kh, -1, nfh, 0, 1, &so);
        t.a_ready = true;
        op = gemm_operand{};
        op.arg = temp(t.a_hi);
        op.s0 = K;
        op.s1 = 1;
        op.has_lo = true;
        op.lo = temp(t.a_lo);
        done_[a] = -1; // its only reader takes the halves
        return true;
    }

    int lowerer::emit_batched_gemm(int id, int mm) {
        const gnode& n = g_.nodes[static_cast<size_t>(mm)];
        const int64_t Bt = n.shape[0], M = n.shape[1], N = n.shape[2];
        const int64_t K = g_.nodes[static_cast<size_t>(n.a)].shape[2];
        kernel k;
        box b;
        // Per epilogue leaf: elements between consecutive batches.
        std::vector<int64_t> batch_stride;
        if (id == mm) {
            // The plain product as the epilogue: one box over [M, N]
            // holding the accumulator.
            b.lo = {0, 0};
            b.hi = {M, N};
            vnode acc;
            acc.kind = vnode::op::acc;
            b.nodes.push_back(acc);
            b.root = 0;
        } else {
            // The elementwise graph over [B, M, N] as one box, its leaves'
            // batch coordinate moved into per-batch pointer offsets: each
            // batch's GEMM then runs the same [M, N] epilogue. Leaves whose
            // batch stride would misalign their float4 loads, or a buffer
            // read at two batch strides, are not fused.
            // The same rule as the grouped tensor-core GEMM's.
            const bool tc = Bt == 1 ? tensor_core_gemm(M, N, K)
                                    : N > 1 && Bt * M <= (int64_t{1} << 30) && Bt * N <= (int64_t{1} << 30) &&
                                          tensor_core_gemm(Bt * M, N, K);
            if (!tc) return -1;
            std::vector<box> boxes;
            try {
                boxes = build_boxes(k, id, g_.nodes[static_cast<size_t>(id)].shape, mm);
            } catch (const not_fusable&) {
                return -1;
            } catch (const not_affine&) {
                return -1;
            }
            if (boxes.size() != 1) return -1;
            b = std::move(boxes[0]);
            batch_stride.assign(k.leaves.size(), -1);
            for (vnode& v : b.nodes) {
                if (v.kind != vnode::op::load) continue;
                const int64_t s0 = v.map.st[0];
                int64_t& bs = batch_stride[static_cast<size_t>(v.buffer)];
                if (s0 < 0 || s0 % 4 != 0 || (bs >= 0 && bs != s0)) return -1;
                bs = s0;
                v.map.st = {v.map.st[1], v.map.st[2]};
            }
            b.lo = {0, 0};
            b.hi = {M, N};
        }
        const kernel_arg A = as_buffer(n.a); // contiguous [Bt, M, K]
        const kernel_arg B = as_buffer(n.b); // contiguous [Bt, K, N]
        const int out = new_temp(static_cast<size_t>(Bt * M * N) * sizeof(float));
        if (Bt == 0 || M == 0 || N == 0) return out;
        rank_ = 2;
        auto at = [](const kernel_arg& base, int64_t off, int64_t s0) {
            gemm_operand o;
            o.arg = base;
            o.arg.elem_offset = off;
            o.s0 = s0;
            o.s1 = 1;
            return o;
        };
        // Tensor cores: every batch's tiles in one grouped launch (A's rows
        // of all batches split as one matrix, B's batches transposed side
        // by side), the epilogue's leaves moved by their batch strides.
        // Realised operands keep their splits, as a 2-D matmul's do.
        gemm_temps shared;
        gemm_batches groups;
        groups.count = Bt;
        groups.leaf_stride.assign(k.leaves.size(), 0);
        for (size_t i = 0; i < batch_stride.size() && i < k.leaves.size(); ++i)
            if (batch_stride[i] > 0) groups.leaf_stride[i] = batch_stride[i];
        int nonfinite = -1;
        if (emit_gemm_tc(id, b, k, at(A, 0, K), at(B, 0, N), M, N, K, &nonfinite, nullptr, out, 0, &shared,
                         nullptr, &groups) >= 0) {
            // Inf or NaN in an operand: the CUDA-core GEMM over every batch
            // (blockIdx.y) into the same output; it returns at once otherwise.
            emit_gemm_simt(b, k, at(A, 0, K), at(B, 0, N), M, N, K, out, nonfinite, 0, Bt, nullptr,
                           &groups.leaf_stride);
            return out;
        }
        if (id != mm) throw std::logic_error("batched GEMM epilogue planned for tensor cores that do not apply");
        // CUDA cores: every batch in one launch (blockIdx.y).
        emit_gemm_simt(b, k, at(A, 0, K), at(B, 0, N), M, N, K, out, -1, 0, Bt);
        return out;
    }

    int lowerer::emit_gemm_softmax(int id, int x, int mm) {
        (void)id;
        const gnode& m = g_.nodes[static_cast<size_t>(mm)];
        const gnode& xv = g_.nodes[static_cast<size_t>(x)];
        if (m.shape != xv.shape) return -1;
        const int64_t M = m.shape[0], N = m.shape[1];
        const int64_t K = g_.nodes[static_cast<size_t>(m.a)].shape[1];
        const int64_t T = (N + 255) / 256; // column tiles of the GEMM
        if (T > 1536) return -1;           // the pass keeps a row's T factors in shared memory
        kernel k;
        std::vector<box> boxes;
        try {
            boxes = build_boxes(k, x, xv.shape, mm);
        } catch (const not_fusable&) {
            return -1;
        } catch (const not_affine&) {
            return -1;
        }
        if (boxes.size() != 1) return -1;
        if (!tensor_core_gemm(M, N, K)) return -1;
        gemm_temps shared;
        gemm_operand A;
        if (!presplit_operand(m.a, M, N, K, shared, A)) A = as_gemm_operand(m.a);
        const gemm_operand B = as_gemm_operand(m.b);
        int nonfinite = -1, stats = -1;
        const int out = emit_gemm_tc(x, boxes[0], k, A, B, M, N, K, &nonfinite, &stats, -1, 0, &shared);
        if (out < 0) throw std::logic_error("softmax GEMM was not eligible");
        auto temp = [](int t) {
            kernel_arg a;
            a.kind = arg_kind::temp;
            a.index = t;
            return a;
        };
        // Inf or NaN in an operand: the CUDA-core GEMM writes y = tree(A@B)
        // into the output, then a row softmax with the reference's own
        // steps (max with -FLT_MAX as seed and (l > r ? l : r), exp(y - max)
        // summed, then divided; src/ops.cpp:7-14) runs in place. Both return
        // at once for finite operands.
        emit_gemm_simt(boxes[0], k, A, B, M, N, K, out, nonfinite);
        {
            std::ostringstream src;
            src << kernel_prelude();
            std::ostringstream body;
            body << "    if (*(const volatile int*)nf == 0) return;\n"
                 << "    __shared__ float red[256];\n"
                 << "    for (pb_u64 r = blockIdx.x; r < " << M << "ull; r += gridDim.x) {\n"
                 << "        float* row = p + r * " << N << "ull;\n"
                 << "        float m = -3.40282347e+38f;\n"
                 << "        for (pb_u64 c = threadIdx.x; c < " << N << "ull; c += 256u) { const float v = row[c]; m = v > m ? v : m; }\n"
                 << "        red[threadIdx.x] = m;\n        __syncthreads();\n"
                 << "        for (pb_u32 h = 128u; h > 0u; h >>= 1) {\n"
                 << "            if (threadIdx.x < h) { const float a = red[threadIdx.x], b = red[threadIdx.x + h]; red[threadIdx.x] = a > b ? a : b; }\n"
                 << "            __syncthreads();\n        }\n"
                 << "        m = red[0];\n        __syncthreads();\n"
                 << "        float s = 0.0f;\n"
                 << "        for (pb_u64 c = threadIdx.x; c < " << N << "ull; c += 256u) s = s + __expf(row[c] - m);\n"
                 << "        red[threadIdx.x] = s;\n        __syncthreads();\n"
                 << "        for (pb_u32 h = 128u; h > 0u; h >>= 1) {\n"
                 << "            if (threadIdx.x < h) red[threadIdx.x] = red[threadIdx.x] + red[threadIdx.x + h];\n"
                 << "            __syncthreads();\n        }\n"
                 << "        s = red[0];\n        __syncthreads();\n"
                 << "        for (pb_u64 c = threadIdx.x; c < " << N << "ull; c += 256u) row[c] = __expf(row[c] - m) / s;\n"
                 << "        __syncthreads();\n    }\n";
            launch_spec l;
            l.name = "pb_softmax_rows_nonfinite";
            src << "extern \"C\" __global__ void __launch_bounds__(256) " << l.name
                << "(float* __restrict__ p, const int* __restrict__ nf) {\n" << body.str() << "}\n";
            l.source = src.str();
            l.schedule = "row softmax in place (runs only for non-finite matmul operands)";
            l.grid = {static_cast<uint32_t>(std::min<int64_t>(M, 148 * 8)), 1, 1};
            l.block = {256, 1, 1};
            l.args = {temp(out), temp(nonfinite)};
            finish_kernel(l);
            p_.launches.push_back(std::move(l));
        }
        // The normalising pass, in place: per row, M = max of the tiles'
        // maxima, S = sum_t s_t exp(m_t - M), and each tile's values times
        // f_t = exp(m_t - M) * (1 / S). A warp per row; the row's T factors
        // in shared memory. (With split-K its combine did the whole
        // softmax: no row statistics, no pass.)
        if (stats >= 0) {
            const bool vec = N % 4 == 0;
            std::ostringstream src;
            src << kernel_prelude();
            std::ostringstream body;
            body << "    if (*(const volatile int*)nf != 0) return;  // the fallback above wrote the rows\n"
                 << "    __shared__ float f[8][" << T << "];\n"
                 << "    const pb_u32 warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;\n"
                 << "    for (pb_u64 r = (pb_u64)blockIdx.x * 8u + warp; r < " << M << "ull; r += (pb_u64)gridDim.x * 8u) {\n"
                 << "        const float2* st = stats + r * " << T << "ull;\n"
                 << "        float m = __int_as_float(0xff800000);\n"
                 << "        for (pb_u32 t = lane; t < " << T << "u; t += 32u) { const float v = st[t].x; m = v > m ? v : m; }\n"
                 << "        #pragma unroll\n"
                 << "        for (int o = 16; o > 0; o >>= 1) { const float v = __shfl_xor_sync(0xffffffffu, m, o); m = v > m ? v : m; }\n"
                 << "        float s = 0.0f;\n"
                 << "        for (pb_u32 t = lane; t < " << T << "u; t += 32u) s = s + st[t].y * __expf(st[t].x - m);\n"
                 << "        #pragma unroll\n"
                 << "        for (int o = 16; o > 0; o >>= 1) s = s + __shfl_xor_sync(0xffffffffu, s, o);\n"
                 << "        const float inv = 1.0f / s;\n"
                 << "        for (pb_u32 t = lane; t < " << T << "u; t += 32u) f[warp][t] = __expf(st[t].x - m) * inv;\n"
                 << "        __syncwarp();\n"
                 << "        float* row = p + r * " << N << "ull;\n";
            if (vec)
                body << "        for (pb_u32 c = lane; c < " << N / 4 << "u; c += 32u) {\n"
                     << "            float4 v = pb_ld4(row + 4u * c);\n"
                     << "            const float g = f[warp][(4u * c) >> 8];\n"
                     << "            v.x = v.x * g; v.y = v.y * g; v.z = v.z * g; v.w = v.w * g;\n"
                     << "            pb_st4(row + 4u * c, v);\n"
                     << "        }\n";
            else
                body << "        for (pb_u32 c = lane; c < " << N << "u; c += 32u) row[c] = row[c] * f[warp][c >> 8];\n";
            body << "        __syncwarp();\n    }\n";
            launch_spec l;
            l.name = "pb_softmax_norm_" + hex64(hash_string(body.str())).substr(0, 8);
            src << "extern \"C\" __global__ void __launch_bounds__(256) " << l.name
                << "(float* __restrict__ p, const float2* __restrict__ stats, const int* __restrict__ nf) {\n"
                << body.str() << "}\n";
            l.source = src.str();
            l.schedule = "softmax normalising pass over the GEMM's exp tiles: a warp per row, " +
                         std::to_string(T) + " tile factors per row";
            l.grid = {static_cast<uint32_t>(std::min<int64_t>((M + 7) / 8, 148 * 16)), 1, 1};
            l.block = {256, 1, 1};
            l.args = {temp(out), temp(stats), temp(nonfinite)};
            finish_kernel(l);
            p_.launches.push_back(std::move(l));
        }
        return out;
    }

    int lowerer::emit_gemm_simt(const box& b, kernel& k, const gemm_operand& A, const gemm_operand& B,
                                int64_t M, int64_t N, int64_t K, int out_temp, int guard_temp, int64_t out_off,
                                int64_t batches, const split_output* so,
                                const std::vector<int64_t>* leaf_batch_stride) {
        const int out = so != nullptr ? so->hi
                        : out_temp >= 0 ? out_temp
                                        : new_temp(static_cast<size_t>(batches * M * N) * sizeof(float));
        rank_ = 2;
        const bool wide = M * N >= (int64_t{1} << 31) - 4096 || M * K >= (int64_t{1} << 31) - 4096 ||
                          K * N >= (int64_t{1} << 31) - 4096 ||
                          A.off + (M - 1) * A.s0 + (K - 1) * A.s1 >= (int64_t{1} << 31) - 4096 ||
                          B.off + (K - 1) * B.s0 + (N - 1) * B.s1 >= (int64_t{1} << 31) - 4096;
        // Operand element addresses: the contiguous forms keep their
        // original text; strided operands add offset and strides.
        auto a_at = [&](const std::string& r, const std::string& c) {
            if (A.contiguous(K)) return "A + (" + r + ") * " + lit(K, wide) + " + " + c;
            return "A + " + lit(A.off, wide) + " + (" + r + ") * " + lit(A.s0, wide) + " + (" + c + ") * " +
                   lit(A.s1, wide);
        };
        // A held as 3xTF32 halves: its value is hi + lo at the same place.
        auto a_val = [&](const std::string& r, const std::string& c) {
            const std::string at = a_at(r, c);
            if (!A.has_lo) return "pb_ld(" + at + ")";
            return "(pb_ld(" + at + ") + pb_ld(Alo" + at.substr(1) + "))";
        };
        auto b_at = [&](const std::string& r, const std::string& c) {
            if (B.contiguous(N)) return "B + (" + r + ") * " + lit(N, wide) + " + " + c;
            return "B + " + lit(B.off, wide) + " + (" + r + ") * " + lit(B.s0, wide) + " + (" + c + ") * " +
                   lit(B.s1, wide);
        };
        const std::string I = wide ? "pb_u64" : "pb_u32";
        std::vector<int> order;
        std::ostringstream src;
        src << kernel_prelude();
        src << emit_expr_function(b, "0", order);
        std::vector<std::string> cvar = {"r", "c"};
        std::ostringstream body;
        // 64x64 output tiles, walked with a grid-stride loop: the guarded
        // fallback of the tensor-core GEMM gets a small grid, so when every
        // operand is finite it costs one short launch, not tiles' worth.
        const int64_t tiles_n = (N + 63) / 64, tiles = tiles_n * ((M + 63) / 64);
        if (guard_temp >= 0) body << "    if (*(const volatile int*)guard == 0) return;\n";
        if (batches > 1) {
            // One matrix product per blockIdx.y over contiguous [M, K] and
            // [K, N] operands and [M, N] outputs; epilogue leaves move by
            // their own batch strides.
            body << "    A += (pb_u64)blockIdx.y * " << M * K << "ull;\n    B += (pb_u64)blockIdx.y * " << K * N
                 << "ull;\n    out += (pb_u64)blockIdx.y * " << M * N << "ull;\n";
            if (leaf_batch_stride != nullptr)
                for (size_t i = 0; i < leaf_batch_stride->size(); ++i)
                    if ((*leaf_batch_stride)[i] > 0)
                        body << "    in" << i << " += (pb_u64)blockIdx.y * " << (*leaf_batch_stride)[i] << "ull;\n";
        }
        body << "    __shared__ float As[16][68];\n    __shared__ float Bs[16][68];\n";
        body << "    const pb_u32 tx = threadIdx.x & 15u, ty = threadIdx.x >> 4;\n";
        body << "    for (" << I << " tile = blockIdx.x; tile < " << lit(tiles, wide) << "; tile += gridDim.x) {\n";
        body << "    const " << I << " row0 = (tile / " << lit(tiles_n, wide) << ") * 64u, col0 = (tile % "
             << lit(tiles_n, wide) << ") * 64u;\n";
        body << "    float acc[4][4];\n";
        body << "    #pragma unroll\n    for (int i = 0; i < 4; ++i)\n        #pragma unroll\n        for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;\n";
        body << "    for (" << I << " k0 = 0; k0 < " << lit(K, wide) << "; k0 += 16u) {\n";
        body << "        #pragma unroll\n        for (int u = 0; u < 4; ++u) {\n";
        body << "            const pb_u32 f = threadIdx.x + 256u * u;\n";
        body << "            const pb_u32 ar = f >> 4, ak = f & 15u;\n";
        body << "            As[ak][ar] = (row0 + ar < " << lit(M, wide) << " && k0 + ak < " << lit(K, wide)
             << ") ? " << a_val("row0 + ar", "k0 + ak") << " : 0.0f;\n";
        body << "            const pb_u32 bk = f >> 6, bc = f & 63u;\n";
        body << "            Bs[bk][bc] = (k0 + bk < " << lit(K, wide) << " && col0 + bc < " << lit(N, wide)
             << ") ? pb_ld(" << b_at("k0 + bk", "col0 + bc") << ") : 0.0f;\n";
        body << "        }\n        __syncthreads();\n";
        body << "        const pb_u32 kmax = (" << lit(K, wide) << " - k0) < 16u ? (pb_u32)(" << lit(K, wide)
             << " - k0) : 16u;\n";
        body << "        for (pb_u32 kk = 0; kk < kmax; ++kk) {\n";
        body << "            float a[4], bv[4];\n";
        body << "            #pragma unroll\n            for (int i = 0; i < 4; ++i) { a[i] = As[kk][ty * 4u + i]; bv[i] = Bs[kk][tx * 4u + i]; }\n";
        body << "            #pragma unroll\n            for (int i = 0; i < 4; ++i)\n                #pragma unroll\n                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);\n";
        body << "        }\n        __syncthreads();\n    }\n";
        body << "    #pragma unroll\n    for (int i = 0; i < 4; ++i)\n        #pragma unroll\n        for (int j = 0; j < 4; ++j) {\n";
        body << "            const " << I << " r = row0 + ty * 4u + i, c = col0 + tx * 4u + j;\n";
        body << "            if (r < " << lit(M, wide) << " && c < " << lit(N, wide) << ") {\n";
        for (size_t li = 0; li < order.size(); ++li) {
            const vnode& v = b.nodes[static_cast<size_t>(order[li])];
            body << "                const float x" << li << " = pb_ld(in" << v.buffer << " + " << address(v.map, cvar, wide, -1)
                 << ");\n";
        }
        body << "                const float y = pb_e0(acc[i][j]";
        for (size_t li = 0; li < order.size(); ++li) body << ", x" << li;
        body << ");\n";
        if (so != nullptr)
            // Split output (see split_output): hi, lo and the Inf/NaN flag.
            body << "                const float h = pb_tf32_hi_s(y);\n"
                 << "                out[r * " << lit(N, wide) << " + c] = h;\n"
                 << "                lo_out[r * " << lit(N, wide) << " + c] = isfinite(y) ? pb_tf32_rn_s(y - h) : 0.0f;\n"
                 << "                if (!isfinite(y)) atomicOr(split_flag, 1);\n";
        else
            body << "                out[r * " << lit(N, wide) << " + c] = y;\n";
        body << "            }\n        }\n";
        body << "    __syncthreads();  // shared tiles are reused by the next output tile\n    }\n";
        launch_spec l;
        l.name = "pb_gemm_simt_" + hex64(hash_string(src.str() + body.str())).substr(0, 8);
        if (so != nullptr)
            // Round to nearest TF32 (hi truncated where rounding would
            // overflow), as the split passes do.
            src << "static __device__ __forceinline__ float pb_tf32_rn_s(float x) {\n"
                   "    unsigned r;\n    asm(\"cvt.rna.tf32.f32 %0, %1;\" : \"=r\"(r) : \"f\"(x));\n"
                   "    return __uint_as_float(r);\n}\n"
                   "static __device__ __forceinline__ float pb_tf32_hi_s(float x) {\n"
                   "    const float r = pb_tf32_rn_s(x);\n"
                   "    return isinf(r) && !isinf(x) ? __uint_as_float(__float_as_uint(x) & 0xFFFFE000u) : r;\n}\n";
        src << "extern \"C\" __global__ void __launch_bounds__(256) " << l.name
            << "(const float* __restrict__ A, " << (A.has_lo ? "const float* __restrict__ Alo, " : "")
            << "const float* __restrict__ B, ";
        for (size_t i = 0; i < k.leaves.size(); ++i) src << "const float* __restrict__ in" << i << ", ";
        src << "float* __restrict__ out" << (so != nullptr ? ", float* __restrict__ lo_out, int* split_flag" : "")
            << (guard_temp >= 0 ? ", const int* guard" : "") << ") {\n" << body.str() << "}\n";
        l.source = src.str();
        if (tiles > 0x7fffffff) throw std::invalid_argument("matmul output is too large for one launch");
        l.grid = {static_cast<uint32_t>(guard_temp >= 0 ? std::min<int64_t>(tiles, 148 * 8) : tiles),
                  static_cast<uint32_t>(batches), 1};
        if (batches > 65535) throw std::invalid_argument("batched matmul has too many batches for one launch");
        l.block = {256, 1, 1};
        l.schedule = "gemm CUDA-core 64x64x16 tiles, k-ordered FMA chain, fused epilogue";
        if (guard_temp >= 0) l.schedule += " (runs only for non-finite operands)";
        l.args.push_back(A.arg);
        if (A.has_lo) l.args.push_back(A.lo);
        l.args.push_back(B.arg);
        for (const kernel_arg& a : k.leaves) l.args.push_back(a);
        kernel_arg o;
        o.kind = arg_kind::temp;
        o.index = out;
        o.elem_offset = out_off;
        l.args.push_back(o);
        if (so != nullptr) {
            kernel_arg lo, fl;
            lo.kind = fl.kind = arg_kind::temp;
            lo.index = so->lo;
            fl.index = so->flag;
            l.args.push_back(lo);
            l.args.push_back(fl);
        }
        if (guard_temp >= 0) {
            kernel_arg gk;
            gk.kind = arg_kind::temp;
            gk.index = guard_temp;
            l.args.push_back(gk);
        }
        finish_kernel(l);
        p_.launches.push_back(std::move(l));
        return out;
    }

    std::shared_ptr<plan> build_plan(const graph& g) {
        auto p = std::make_shared<plan>();
        lowerer low{g, *p};
        p->result_temp = low.materialize(g.root);
        p->out_shape = g.nodes[static_cast<size_t>(g.root)].shape;
        return p;
    }

} // namespace porch::detail
