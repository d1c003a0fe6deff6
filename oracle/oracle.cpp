// Host scalar oracle for porch's lazy tensor graphs.
//
// TEST INFRASTRUCTURE ONLY. This file is the checker that tests/,
// __graft_entry__.smoke() and bench.py's cpu_baseline leg run against the
// CUDA path; nothing in porch_b200/ links, loads or calls it.
//
// It restates the reference's graph semantics (AkhilSamavedam/porch) in plain
// C++ with no GPU:
//  - the builders and slicing of src/tensor.cpp:1261-1315 and 1406-1511, and
//    the compound ops of src/ops.cpp:5-18 (relu, softmax, logistic);
//  - shape inference and validation with the same messages,
//    src/tensor.cpp:279-496;
//  - the per-element index maps of the generated kernels: strided slice
//    (src/tensor.cpp:511-530), broadcast (:532-560), rank-2 transpose
//    (:562-571), reduction source index (:573-614) and concat (:766-818);
//  - operator forms and order (:629-683, 856-869): IEEE fp32 + - * /,
//    maximum/minimum as `(l > r) ? l : r` / `(l < r) ? l : r`,
//    reciprocal as 1.0f / x; built with -ffp-contract=off so nothing fuses;
//  - reductions materialised before their consumer, as
//    lower_nested_reductions does (:964-989): sum starts at 0, max starts at
//    -FLT_MAX and keeps `t > v ? t : v`.
// Where the reference's arithmetic is not reproducible on a host it is
// computed more accurately and compared with a tolerance by the tests:
//  - exp uses std::exp in double (the reference calls the __expf intrinsic);
//  - sum reductions accumulate in double (the reference's order is a
//    256-thread strided partial sum followed by a shared-memory tree);
//  - matmul accumulates in double (the reference runs an fp32 FMA chain).
//
// Input: a text program, one op per line, "<id> <op> <args...>":
//   input <slot> | scalar <hex float bits> | add|subtract|multiply|divide|
//   maximum|minimum|matmul <a> <b> | exp|reciprocal|transpose|relu|logistic
//   <a> | reshape|broadcast <a> <d0,d1,..> | unsqueeze <a> <axis> |
//   concat <a> <b> <axis> | sum|max <a> <axis> <keepdim> |
//   softmax <a> <axis> | index <a> <spec;spec;..> (spec: i<k> | s<start>:<stop>:<step> | a)
//   | tensor <a> | materialize <a>
// The last line is the output.
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

    using index_t = int64_t;

    enum class kind {
        input, scalar, add, subtract, multiply, divide, matmul, slice, reshape,
        unsqueeze, transpose, broadcast, concat, sum, max, maximum, minimum, exp,
        reciprocal
    };

    struct node;
    using node_ptr = std::shared_ptr<const node>;

    // A realised array (an input or a materialised intermediate).
    struct array {
        std::vector<index_t> shape;
        std::vector<float> values;
    };
    using array_ptr = std::shared_ptr<const array>;

    struct node {
        kind k = kind::scalar;
        array_ptr input;
        float scalar = 0.0F;
        node_ptr lhs, rhs;
        std::vector<index_t> slice_shape, slice_strides, shape;
        index_t slice_offset = 0;
        size_t axis = 0;
        bool keepdim = false;
        // Operand shapes, filled by evaluator::prepare before evaluation.
        std::vector<index_t> lshape, rshape;
        bool lscalar = false;
    };

    // Program values: expressions, or "tensor" handles (lazy or realised).
    struct value {
        node_ptr expr;
        bool is_tensor = false;
        std::vector<index_t> tensor_shape; // for tensors
    };

    size_t numel(const std::vector<index_t>& s) {
        size_t n = 1;
        for (index_t e : s) {
            if (e < 0) throw std::invalid_argument("tensor shape extents must be non-negative");
            n *= static_cast<size_t>(e);
        }
        return n;
    }

    std::vector<index_t> contiguous(const std::vector<index_t>& s) {
        std::vector<index_t> st(s.size(), 1);
        index_t acc = 1;
        for (size_t i = s.size(); i > 0; --i) {
            st[i - 1] = acc;
            acc *= s[i - 1];
        }
        return st;
    }

    node_ptr make(kind k, node_ptr a = nullptr, node_ptr b = nullptr) {
        auto n = std::make_shared<node>();
        n->k = k;
        n->lhs = std::move(a);
        n->rhs = std::move(b);
        return n;
    }

    // ------------------------------------------------------- inference --
    struct info {
        std::vector<index_t> shape;
        bool scalar = true;
    };

    std::vector<index_t> reduced(const std::vector<index_t>& s, size_t axis, bool keepdim) {
        std::vector<index_t> r;
        if (keepdim) {
            r = s;
            r[axis] = 1;
            return r;
        }
        for (size_t d = 0; d < s.size(); ++d)
            if (d != axis) r.push_back(s[d]);
        if (r.empty()) r.push_back(1);
        return r;
    }

    info infer(const node& n, bool& has_input) {
        auto same = [](const info& a, const info& b) {
            if (a.scalar || b.scalar) return;
            if (a.shape != b.shape) throw std::invalid_argument("tensor expression shapes must match");
        };
        switch (n.k) {
            case kind::input:
                has_input = true;
                return {n.input->shape, false};
            case kind::scalar:
                return {};
            case kind::add: case kind::subtract: case kind::multiply: case kind::divide:
            case kind::maximum: case kind::minimum: {
                info a = infer(*n.lhs, has_input), b = infer(*n.rhs, has_input);
                same(a, b);
                return a.scalar ? b : a;
            }
            case kind::matmul: {
                info a = infer(*n.lhs, has_input), b = infer(*n.rhs, has_input);
                if (a.scalar || b.scalar) throw std::invalid_argument("matmul operands must be tensors");
                if (a.shape.size() != 2 || b.shape.size() != 2)
                    throw std::invalid_argument("matmul requires rank-2 tensors");
                if (a.shape[1] != b.shape[0]) throw std::invalid_argument("matmul inner dimensions must match");
                return {{a.shape[0], b.shape[1]}, false};
            }
            case kind::slice:
                (void)infer(*n.lhs, has_input);
                return {n.slice_shape, false};
            case kind::reshape: {
                info a = infer(*n.lhs, has_input);
                if (a.scalar) throw std::invalid_argument("reshape operand must be a tensor");
                if (numel(a.shape) != numel(n.shape))
                    throw std::invalid_argument("reshape must preserve tensor element count");
                return {n.shape, false};
            }
            case kind::unsqueeze: {
                info a = infer(*n.lhs, has_input);
                if (a.scalar) throw std::invalid_argument("unsqueeze operand must be a tensor");
                if (n.axis > a.shape.size()) throw std::invalid_argument("unsqueeze axis is out of bounds");
                a.shape.insert(a.shape.begin() + static_cast<ptrdiff_t>(n.axis), 1);
                return a;
            }
            case kind::transpose: {
                info a = infer(*n.lhs, has_input);
                if (a.scalar) throw std::invalid_argument("transpose operand must be a tensor");
                if (a.shape.size() != 2)
                    throw std::invalid_argument("transpose currently requires a rank-2 tensor");
                return {{a.shape[1], a.shape[0]}, false};
            }
            case kind::broadcast: {
                info a = infer(*n.lhs, has_input);
                if (a.scalar) return {n.shape, false};
                if (a.shape.size() > n.shape.size())
                    throw std::invalid_argument("broadcast target rank must be at least source rank");
                const size_t off = n.shape.size() - a.shape.size();
                for (size_t d = 0; d < a.shape.size(); ++d)
                    if (a.shape[d] != 1 && a.shape[d] != n.shape[off + d])
                        throw std::invalid_argument("broadcast shapes are not compatible");
                return {n.shape, false};
            }
            case kind::concat: {
                info a = infer(*n.lhs, has_input), b = infer(*n.rhs, has_input);
                if (a.scalar || b.scalar) throw std::invalid_argument("concat operands must be tensors");
                if (a.shape.size() != b.shape.size())
                    throw std::invalid_argument("concat operands must have the same rank");
                if (n.axis >= a.shape.size()) throw std::invalid_argument("concat axis is out of bounds");
                for (size_t d = 0; d < a.shape.size(); ++d)
                    if (d != n.axis && a.shape[d] != b.shape[d])
                        throw std::invalid_argument("concat non-axis dimensions must match");
                a.shape[n.axis] += b.shape[n.axis];
                return a;
            }
            case kind::sum: case kind::max: {
                info a = infer(*n.lhs, has_input);
                if (a.scalar) throw std::invalid_argument("reduction operand must be a tensor");
                if (n.axis >= a.shape.size()) throw std::invalid_argument("reduction axis is out of bounds");
                return {reduced(a.shape, n.axis, n.keepdim), false};
            }
            case kind::exp: case kind::reciprocal:
                return infer(*n.lhs, has_input);
        }
        throw std::invalid_argument("unknown tensor expression node");
    }

    // ------------------------------------------------------ evaluation --
    struct evaluator {
        int threads = 1;

        array_ptr materialize(const node& root);

        // Value of `n` at linear index `i` of its contiguous layout. Matmul
        // and reduction nodes have been replaced by realised inputs.
        float at(const node& n, index_t i) const {
            switch (n.k) {
                case kind::input:
                    return n.input->values[static_cast<size_t>(i)];
                case kind::scalar:
                    return n.scalar;
                case kind::add: return at(*n.lhs, i) + at(*n.rhs, i);
                case kind::subtract: return at(*n.lhs, i) - at(*n.rhs, i);
                case kind::multiply: return at(*n.lhs, i) * at(*n.rhs, i);
                case kind::divide: return at(*n.lhs, i) / at(*n.rhs, i);
                case kind::maximum: {
                    const float l = at(*n.lhs, i), r = at(*n.rhs, i);
                    return (l > r) ? l : r;
                }
                case kind::minimum: {
                    const float l = at(*n.lhs, i), r = at(*n.rhs, i);
                    return (l < r) ? l : r;
                }
                case kind::exp:
                    return static_cast<float>(std::exp(static_cast<double>(at(*n.lhs, i))));
                case kind::reciprocal:
                    return 1.0F / at(*n.lhs, i);
                case kind::slice: {
                    // off + sum_d ((i / prod_{>d}) % shape_d) * stride_d
                    index_t src = n.slice_offset, rest = i;
                    for (size_t d = n.slice_shape.size(); d > 0; --d) {
                        const index_t ext = n.slice_shape[d - 1];
                        src += (rest % ext) * n.slice_strides[d - 1];
                        rest /= ext;
                    }
                    return at(*n.lhs, src);
                }
                case kind::reshape:
                case kind::unsqueeze:
                    return at(*n.lhs, i);
                case kind::transpose: {
                    // out [s1, s0] from [s0, s1]: src = (i % s0) * s1 + i / s0
                    const std::vector<index_t>& s = n.lshape;
                    return at(*n.lhs, (i % s[0]) * s[1] + i / s[0]);
                }
                case kind::broadcast: {
                    if (n.lscalar) return at(*n.lhs, i);
                    const std::vector<index_t>& s = n.lshape;
                    const size_t off = n.shape.size() - s.size();
                    // Right-aligned: the source index keeps the coordinates of
                    // non-unit source dims in the source's contiguous layout.
                    index_t src = 0, rest = i, sstride = 1;
                    for (size_t d = n.shape.size(); d > 0; --d) {
                        const index_t c = rest % n.shape[d - 1];
                        rest /= n.shape[d - 1];
                        if (d - 1 >= off) {
                            const size_t sd = d - 1 - off;
                            if (s[sd] != 1) src += c * sstride;
                            sstride *= s[sd];
                        }
                    }
                    return at(*n.lhs, src);
                }
                case kind::concat: {
                    const std::vector<index_t>& l = n.lshape;
                    const std::vector<index_t>& r = n.rshape;
                    const size_t R = l.size();
                    index_t li = 0, ri = 0, ls = 1, rs = 1, rest = i, ac = 0;
                    for (size_t d = R; d > 0; --d) {
                        const index_t ext = d - 1 == n.axis ? l[d - 1] + r[d - 1] : l[d - 1];
                        const index_t c = rest % ext;
                        rest /= ext;
                        if (d - 1 == n.axis) ac = c;
                        li += c * ls;
                        ri += (d - 1 == n.axis ? c - l[d - 1] : c) * rs;
                        ls *= l[d - 1];
                        rs *= r[d - 1];
                    }
                    return ac < l[n.axis] ? at(*n.lhs, li) : at(*n.rhs, ri);
                }
                default:
                    throw std::logic_error("unlowered node in oracle evaluation");
            }
        }

        template <typename F>
        void parallel(size_t count, F&& f) const {
            const size_t nt = std::max<size_t>(1, std::min<size_t>(static_cast<size_t>(threads),
                                                                  count / 4096 + 1));
            if (nt <= 1) {
                f(size_t{0}, count);
                return;
            }
            std::vector<std::thread> pool;
            const size_t chunk = (count + nt - 1) / nt;
            for (size_t t = 0; t < nt; ++t) {
                const size_t b = t * chunk, e = std::min(count, b + chunk);
                if (b < e) pool.emplace_back([&, b, e] { f(b, e); });
            }
            for (auto& th : pool) th.join();
        }

        // Records operand shapes on every node (evaluation is per element, so
        // shape inference must not run inside it).
        void prepare(const node_ptr& n) {
            if (!n) return;
            prepare(n->lhs);
            prepare(n->rhs);
            auto* m = const_cast<node*>(n.get());
            bool h = false;
            if (n->lhs) {
                const info a = infer(*n->lhs, h);
                m->lshape = a.shape;
                m->lscalar = a.scalar;
            }
            if (n->rhs) m->rshape = infer(*n->rhs, h).shape;
        }

        // Replaces every matmul / sum / max below the root with a realised
        // input (children first, lhs before rhs).
        node_ptr lower(const node_ptr& n, bool is_root) {
            if (!n) return n;
            if (!is_root && (n->k == kind::sum || n->k == kind::max || n->k == kind::matmul)) {
                auto in = make(kind::input);
                std::const_pointer_cast<node>(in)->input = materialize(*n);
                return in;
            }
            auto copy = std::make_shared<node>(*n);
            copy->lhs = lower(n->lhs, false);
            copy->rhs = lower(n->rhs, false);
            return copy;
        }
    };

    array_ptr evaluator::materialize(const node& root_in) {
        bool has_input = false;
        node_ptr root = lower(std::make_shared<node>(root_in), true);
        const info out_info = infer(*root, has_input);
        if (!has_input)
            throw std::invalid_argument("tensor expression must reference at least one tensor");
        if (out_info.scalar)
            throw std::invalid_argument("scalar expression cannot materialize to a tensor");
        auto result = std::make_shared<array>();
        result->shape = out_info.shape;
        const size_t count = numel(out_info.shape);
        result->values.assign(count, 0.0F);
        if (count == 0) return result;
        // A launch with a non-empty output refuses an empty input buffer
        // (src/cuda_jit.cpp:794-803 elementwise, :875-884 reductions); the
        // nested reductions were materialised (and checked) first above.
        {
            bool empty = false;
            std::vector<const node*> stack{root.get()};
            while (!stack.empty()) {
                const node* n = stack.back();
                stack.pop_back();
                if (n == nullptr) continue;
                if (n->k == kind::input && n->input && numel(n->input->shape) == 0) empty = true;
                stack.push_back(n->lhs.get());
                stack.push_back(n->rhs.get());
            }
            if (empty)
                throw std::invalid_argument(root->k == kind::sum || root->k == kind::max
                                                ? "CUDA reduction input is empty"
                                                : "CUDA elementwise input is empty");
        }
        float* out = result->values.data();

        if (root->k == kind::matmul) {
            const array_ptr a = materialize(*root->lhs);
            const array_ptr b = materialize(*root->rhs);
            const index_t M = a->shape[0], K = a->shape[1], N = b->shape[1];
            parallel(static_cast<size_t>(M), [&](size_t r0, size_t r1) {
                std::vector<double> acc(static_cast<size_t>(N));
                for (size_t r = r0; r < r1; ++r) {
                    std::fill(acc.begin(), acc.end(), 0.0);
                    for (index_t k = 0; k < K; ++k) {
                        const double av = a->values[r * static_cast<size_t>(K) + static_cast<size_t>(k)];
                        const float* brow = b->values.data() + static_cast<size_t>(k * N);
                        for (index_t c = 0; c < N; ++c) acc[static_cast<size_t>(c)] += av * brow[c];
                    }
                    for (index_t c = 0; c < N; ++c)
                        out[r * static_cast<size_t>(N) + static_cast<size_t>(c)] =
                            static_cast<float>(acc[static_cast<size_t>(c)]);
                }
            });
            return result;
        }
        if (root->k == kind::sum || root->k == kind::max) {
            const array_ptr src = materialize(*root->lhs);
            const std::vector<index_t>& S = src->shape;
            index_t outer = 1, inner = 1;
            for (size_t d = 0; d < root->axis; ++d) outer *= S[d];
            for (size_t d = root->axis + 1; d < S.size(); ++d) inner *= S[d];
            const index_t A = S[root->axis];
            const bool is_sum = root->k == kind::sum;
            parallel(static_cast<size_t>(outer * inner), [&](size_t o0, size_t o1) {
                for (size_t o = o0; o < o1; ++o) {
                    const index_t ou = static_cast<index_t>(o) / inner, in = static_cast<index_t>(o) % inner;
                    double s = 0.0;
                    float m = -FLT_MAX;
                    for (index_t k = 0; k < A; ++k) {
                        const float v = src->values[static_cast<size_t>((ou * A + k) * inner + in)];
                        if (is_sum)
                            s += v;
                        else
                            m = m > v ? m : v;
                    }
                    out[o] = is_sum ? static_cast<float>(s) : m;
                }
            });
            return result;
        }
        prepare(root);
        parallel(count, [&](size_t b, size_t e) {
            for (size_t i = b; i < e; ++i) out[i] = at(*root, static_cast<index_t>(i));
        });
        return result;
    }

    // ---------------------------------------------------- program parse --
    std::vector<index_t> parse_dims(const std::string& s) {
        std::vector<index_t> d;
        if (s == "-") return d;
        std::stringstream ss(s);
        std::string item;
        while (std::getline(ss, item, ',')) d.push_back(std::stoll(item));
        return d;
    }

    node_ptr expr_of(const value& v, const std::vector<array_ptr>& inputs) {
        (void)inputs;
        return v.expr;
    }

    // tensor::operator[] (src/tensor.cpp:1261-1315) for a contiguous tensor.
    node_ptr index_tensor(const value& t, const std::string& spec_text) {
        const std::vector<index_t>& shape = t.tensor_shape;
        const std::vector<index_t> strides = contiguous(shape);
        std::vector<std::string> specs;
        {
            std::stringstream ss(spec_text);
            std::string s;
            while (std::getline(ss, s, ';'))
                if (!s.empty()) specs.push_back(s);
        }
        if (specs.size() > shape.size()) throw std::invalid_argument("too many tensor indices");
        std::vector<index_t> oshape, ostr;
        index_t offset = 0;
        size_t dim = 0;
        for (const std::string& sp : specs) {
            const index_t ext = shape[dim], st = strides[dim];
            if (sp[0] == 'i') {
                index_t k = std::stoll(sp.substr(1));
                if (k < 0) k += ext;
                if (k < 0 || k >= ext) throw std::out_of_range("tensor index is out of bounds");
                offset += k * st;
            } else if (sp[0] == 's') {
                index_t start = 0, stop = 0, step = 1;
                std::sscanf(sp.c_str() + 1, "%ld:%ld:%ld", &start, &stop, &step);
                auto norm = [&](index_t x) {
                    if (x < 0) x += ext;
                    if (x < 0) return index_t{0};
                    if (x > ext) return ext;
                    return x;
                };
                start = norm(start);
                stop = norm(stop);
                if (step <= 0) throw std::invalid_argument("tensor slice step must be positive");
                const index_t len = stop <= start ? 0 : (stop - start + step - 1) / step;
                offset += start * st;
                oshape.push_back(len);
                ostr.push_back(st * step);
            } else {
                oshape.push_back(ext);
                ostr.push_back(st);
            }
            ++dim;
        }
        for (; dim < shape.size(); ++dim) {
            oshape.push_back(shape[dim]);
            ostr.push_back(strides[dim]);
        }
        auto n = std::make_shared<node>();
        n->k = kind::slice;
        n->lhs = t.expr;
        n->slice_shape = oshape;
        n->slice_strides = ostr;
        n->slice_offset = offset;
        return n;
    }

    node_ptr run_program(const std::string& program, const std::vector<array_ptr>& inputs,
                         evaluator& ev, bool& materialized_root) {
        std::vector<value> vals;
        std::stringstream lines(program);
        std::string line;
        node_ptr last;
        while (std::getline(lines, line)) {
            if (line.empty()) continue;
            std::stringstream ls(line);
            size_t id = 0;
            std::string op;
            ls >> id >> op;
            if (vals.size() <= id) vals.resize(id + 1);
            auto arg = [&]() {
                size_t a = 0;
                ls >> a;
                if (a >= vals.size() || !vals[a].expr) throw std::invalid_argument("bad program reference");
                return vals[a];
            };
            value out;
            if (op == "input") {
                size_t slot = 0;
                ls >> slot;
                auto n = make(kind::input);
                std::const_pointer_cast<node>(n)->input = inputs.at(slot);
                out.expr = n;
                out.is_tensor = true;
                out.tensor_shape = inputs.at(slot)->shape;
            } else if (op == "scalar") {
                std::string hex;
                ls >> hex;
                uint32_t bits = static_cast<uint32_t>(std::stoul(hex, nullptr, 16));
                auto n = std::make_shared<node>();
                n->k = kind::scalar;
                std::memcpy(&n->scalar, &bits, 4);
                out.expr = n;
            } else if (op == "add" || op == "subtract" || op == "multiply" || op == "divide" ||
                       op == "maximum" || op == "minimum" || op == "matmul") {
                value a = arg(), b = arg();
                kind k = op == "add" ? kind::add : op == "subtract" ? kind::subtract
                       : op == "multiply" ? kind::multiply : op == "divide" ? kind::divide
                       : op == "maximum" ? kind::maximum : op == "minimum" ? kind::minimum : kind::matmul;
                out.expr = make(k, a.expr, b.expr);
            } else if (op == "exp" || op == "reciprocal" || op == "transpose") {
                value a = arg();
                out.expr = make(op == "exp" ? kind::exp : op == "reciprocal" ? kind::reciprocal
                                                                            : kind::transpose,
                                a.expr);
            } else if (op == "relu") {
                // relu(x) = maximum(x, 0) (src/ops.cpp:5)
                value a = arg();
                auto zero = std::make_shared<node>();
                zero->k = kind::scalar;
                out.expr = make(kind::maximum, a.expr, zero);
            } else if (op == "logistic") {
                // 1 / (1 + exp(0 - x)) (src/ops.cpp:16-18)
                value a = arg();
                auto zero = std::make_shared<node>();
                zero->k = kind::scalar;
                auto one = std::make_shared<node>();
                one->k = kind::scalar;
                one->scalar = 1.0F;
                out.expr = make(kind::reciprocal,
                                make(kind::add, one, make(kind::exp, make(kind::subtract, zero, a.expr))));
            } else if (op == "softmax") {
                // max-keepdim, subtract, exp, sum-keepdim, divide (src/ops.cpp:7-14)
                value a = arg();
                size_t axis = 0;
                ls >> axis;
                bool h = false;
                const info s = infer(*a.expr, h);
                const std::vector<index_t> shape = s.scalar ? std::vector<index_t>{} : s.shape;
                auto mx = std::make_shared<node>();
                mx->k = kind::max;
                mx->lhs = a.expr;
                mx->axis = axis;
                mx->keepdim = true;
                auto bm = std::make_shared<node>();
                bm->k = kind::broadcast;
                bm->lhs = mx;
                bm->shape = shape;
                auto numerator = make(kind::exp, make(kind::subtract, a.expr, bm));
                auto sm = std::make_shared<node>();
                sm->k = kind::sum;
                sm->lhs = numerator;
                sm->axis = axis;
                sm->keepdim = true;
                auto bs = std::make_shared<node>();
                bs->k = kind::broadcast;
                bs->lhs = sm;
                bs->shape = shape;
                out.expr = make(kind::divide, numerator, bs);
            } else if (op == "reshape" || op == "broadcast") {
                value a = arg();
                std::string dims;
                ls >> dims;
                auto n = std::make_shared<node>();
                n->k = op == "reshape" ? kind::reshape : kind::broadcast;
                n->lhs = a.expr;
                n->shape = parse_dims(dims);
                out.expr = n;
            } else if (op == "unsqueeze") {
                value a = arg();
                auto n = std::make_shared<node>();
                n->k = kind::unsqueeze;
                n->lhs = a.expr;
                ls >> n->axis;
                out.expr = n;
            } else if (op == "concat") {
                value a = arg(), b = arg();
                auto n = std::make_shared<node>();
                n->k = kind::concat;
                n->lhs = a.expr;
                n->rhs = b.expr;
                ls >> n->axis;
                out.expr = n;
            } else if (op == "sum" || op == "max") {
                value a = arg();
                auto n = std::make_shared<node>();
                n->k = op == "sum" ? kind::sum : kind::max;
                n->lhs = a.expr;
                int keep = 0;
                ls >> n->axis >> keep;
                n->keepdim = keep != 0;
                out.expr = n;
            } else if (op == "tensor") {
                // `tensor t = expr;` validates and keeps the graph lazy.
                value a = arg();
                bool h = false;
                const info s = infer(*a.expr, h);
                if (!h) throw std::invalid_argument("tensor expression must reference at least one tensor");
                if (s.scalar) throw std::invalid_argument("scalar expression cannot convert to a tensor");
                out.expr = a.expr;
                out.is_tensor = true;
                out.tensor_shape = s.shape;
            } else if (op == "materialize") {
                value a = arg();
                array_ptr r = ev.materialize(*a.expr);
                auto n = make(kind::input);
                std::const_pointer_cast<node>(n)->input = r;
                out.expr = n;
                out.is_tensor = true;
                out.tensor_shape = r->shape;
            } else if (op == "index") {
                value a = arg();
                std::string spec;
                ls >> spec;
                if (!a.is_tensor) throw std::invalid_argument("index applies to a tensor");
                if (spec == "-") spec.clear();
                out.expr = index_tensor(a, spec);
            } else {
                throw std::invalid_argument("unknown program op " + op + " in line: " + line);
            }
            vals[id] = out;
            last = out.expr;
        }
        materialized_root = false;
        return last;
    }

    thread_local std::string tl_error;

    int status_of(const std::exception_ptr& e) {
        try {
            std::rethrow_exception(e);
        } catch (const std::invalid_argument& x) {
            tl_error = x.what();
            return 1;
        } catch (const std::out_of_range& x) {
            tl_error = x.what();
            return 2;
        } catch (const std::exception& x) {
            tl_error = x.what();
            return 3;
        }
    }

} // namespace

extern "C" {

const char* oracle_last_error(void) { return tl_error.c_str(); }

// Shape of the program's output (rank written to *rank). Validates.
int oracle_shape(const char* program, const float* const* inputs, const int64_t* const* shapes,
                 const size_t* ranks, size_t n_inputs, int64_t* out_shape, size_t capacity,
                 size_t* rank) {
    try {
        std::vector<array_ptr> ins;
        for (size_t i = 0; i < n_inputs; ++i) {
            auto a = std::make_shared<array>();
            a->shape.assign(shapes[i], shapes[i] + ranks[i]);
            // Values are needed when the program materialises an intermediate.
            if (inputs != nullptr && inputs[i] != nullptr)
                a->values.assign(inputs[i], inputs[i] + numel(a->shape));
            ins.push_back(a);
        }
        evaluator ev;
        bool mat = false;
        node_ptr root = run_program(program, ins, ev, mat);
        bool has_input = false;
        const info s = infer(*root, has_input);
        *rank = s.scalar ? 0 : s.shape.size();
        for (size_t d = 0; d < *rank && d < capacity; ++d) out_shape[d] = s.shape[d];
        return 0;
    } catch (...) {
        return status_of(std::current_exception());
    }
}

// Evaluates the program; `out` receives the materialised output.
int oracle_eval(const char* program, const float* const* inputs, const int64_t* const* shapes,
                const size_t* ranks, size_t n_inputs, float* out, size_t out_count, int threads) {
    try {
        std::vector<array_ptr> ins;
        for (size_t i = 0; i < n_inputs; ++i) {
            auto a = std::make_shared<array>();
            a->shape.assign(shapes[i], shapes[i] + ranks[i]);
            const size_t n = numel(a->shape);
            a->values.assign(inputs[i], inputs[i] + n);
            ins.push_back(a);
        }
        evaluator ev;
        ev.threads = threads > 0 ? threads : 1;
        bool mat = false;
        node_ptr root = run_program(program, ins, ev, mat);
        array_ptr r = ev.materialize(*root);
        if (r->values.size() != out_count) {
            tl_error = "output buffer size does not match the result";
            return 1;
        }
        std::memcpy(out, r->values.data(), out_count * sizeof(float));
        return 0;
    } catch (...) {
        return status_of(std::current_exception());
    }
}

} // extern "C"
