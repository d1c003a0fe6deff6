// Graph canonicalisation, the plan cache and plan execution.
//
// Reference counterpart: materialize_expression (src/tensor.cpp:1002-1066),
// which re-runs shape inference and code emission and recompiles (cache
// lookup by full source text) on every call, allocates a zero-filled host
// vector of numel floats, and loads the PTX module on every launch. Here a
// repeat graph costs one hash walk, the stream-ordered allocations and the
// launches.
#include "lower.hpp"
#include "plan.hpp"

#include <atomic>
#include <chrono>
#include <cstring>
#include <sstream>
#include <stdexcept>
#include <unordered_map>

namespace porch::detail {

    namespace {

        uint64_t mix(uint64_t h, uint64_t v) {
            h ^= v + 0x9e3779b97f4a7c15ULL + (h << 6) + (h >> 2);
            return h;
        }

        struct canonicalizer {
            graph g;
            std::unordered_map<const tensor_expr::node*, int> memo;
            std::map<std::string, int> numbering;
            std::unordered_map<const realized_storage*, int> slot_of;

            // Interns a node under its structural key (value numbering).
            int intern(gnode gn, std::string key) {
                auto num = numbering.find(key);
                if (num != numbering.end()) return num->second;
                shape_of(gn);
                const int id = static_cast<int>(g.nodes.size());
                g.nodes.push_back(std::move(gn));
                g.uses.push_back(0);
                if (g.nodes[id].a >= 0) ++g.uses[g.nodes[id].a];
                if (g.nodes[id].b >= 0) ++g.uses[g.nodes[id].b];
                g.hash = mix(g.hash, std::hash<std::string>{}(key));
                g.key += key;
                numbering.emplace(std::move(key), id);
                return id;
            }

            static void put_i(std::string& key, int64_t v) { key.append(reinterpret_cast<const char*>(&v), sizeof v); }
            static void put_v(std::string& key, const std::vector<index_t>& v) {
                put_i(key, static_cast<int64_t>(v.size()));
                for (index_t x : v) put_i(key, x);
            }

            int slot_for(const std::shared_ptr<realized_storage>& s, const std::vector<index_t>& shape) {
                auto it = slot_of.find(s.get());
                if (it != slot_of.end()) return it->second;
                const int slot = static_cast<int>(g.slots.size());
                slot_of.emplace(s.get(), slot);
                g.slots.push_back(s);
                g.slot_shapes.push_back(shape);
                return slot;
            }

            // A strided view read in place: slice(input(base as [count]), layout).
            int view_node(const std::shared_ptr<realized_storage>& base, const strided_layout& l) {
                gnode in;
                in.kind = expr_kind::input;
                in.shape = {static_cast<index_t>(base->count)};
                in.slot = slot_for(base, in.shape);
                std::string ik;
                put_i(ik, static_cast<int64_t>(expr_kind::input));
                put_i(ik, -1);
                put_i(ik, -1);
                put_i(ik, in.slot);
                put_v(ik, in.shape);
                const int bi = intern(std::move(in), std::move(ik));
                gnode sl;
                sl.kind = expr_kind::slice;
                sl.a = bi;
                sl.p_shape = l.shape;
                sl.p_strides = l.strides;
                sl.p_offset = l.offset;
                std::string sk;
                put_i(sk, static_cast<int64_t>(expr_kind::slice));
                put_i(sk, bi);
                put_i(sk, -1);
                put_v(sk, sl.p_shape);
                put_v(sk, sl.p_strides);
                put_i(sk, sl.p_offset);
                return intern(std::move(sl), std::move(sk));
            }

            int visit(const tensor_expr::node& n) {
                auto it = memo.find(&n);
                if (it != memo.end()) return it->second;
                // Inputs that are strided views (and slices of them) read the
                // base storage in place.
                if (n.kind == expr_kind::input || (n.kind == expr_kind::slice && n.lhs &&
                                                   n.lhs->kind == expr_kind::input)) {
                    const tensor_expr::node& in = n.kind == expr_kind::input ? n : *n.lhs;
                    std::shared_ptr<realized_storage> base;
                    strided_layout l;
                    if (in.storage && view_of(*in.storage, base, l)) {
                        g.view_inputs.emplace_back(in.storage, in.storage->layout_epoch.load());
                        int id = -1;
                        if (n.kind == expr_kind::input) {
                            id = view_node(base, l);
                        } else {
                            strided_layout c;
                            if (compose_slice(l, n.slice_offset, n.slice_strides, n.slice_shape, c))
                                id = view_node(base, c);
                        }
                        if (id >= 0) {
                            memo.emplace(&n, id);
                            return id;
                        }
                    }
                }
                gnode gn;
                gn.kind = n.kind;
                if (n.lhs) gn.a = visit(*n.lhs);
                if (n.rhs) gn.b = visit(*n.rhs);
                std::string key;
                key.reserve(64);
                put_i(key, static_cast<int64_t>(n.kind));
                put_i(key, gn.a);
                put_i(key, gn.b);
                switch (n.kind) {
                    case expr_kind::input: {
                        gn.slot = slot_for(n.storage, n.input_shape);
                        put_i(key, gn.slot);
                        put_v(key, n.input_shape);
                        gn.shape = n.input_shape;
                        break;
                    }
                    case expr_kind::scalar: {
                        gn.scalar = n.scalar;
                        gn.is_scalar = true;
                        uint32_t bits = 0;
                        std::memcpy(&bits, &n.scalar, 4);
                        put_i(key, bits);
                        break;
                    }
                    case expr_kind::slice:
                        gn.p_shape = n.slice_shape;
                        gn.p_strides = n.slice_strides;
                        gn.p_offset = n.slice_offset;
                        put_v(key, gn.p_shape);
                        put_v(key, gn.p_strides);
                        put_i(key, gn.p_offset);
                        break;
                    case expr_kind::reshape:
                    case expr_kind::broadcast:
                    case expr_kind::permute:
                        gn.p_shape = n.shape;
                        put_v(key, gn.p_shape);
                        break;
                    case expr_kind::unsqueeze:
                    case expr_kind::concat:
                    case expr_kind::sum:
                    case expr_kind::max:
                        gn.axis = n.axis;
                        gn.keepdim = n.keepdim;
                        put_i(key, static_cast<int64_t>(n.axis));
                        put_i(key, n.keepdim ? 1 : 0);
                        break;
                    default:
                        break;
                }
                const int id = intern(std::move(gn), std::move(key));
                memo.emplace(&n, id);
                return id;
            }

            // Output shape of an already-validated node.
            void shape_of(gnode& n) {
                const gnode* a = n.a >= 0 ? &g.nodes[n.a] : nullptr;
                const gnode* b = n.b >= 0 ? &g.nodes[n.b] : nullptr;
                switch (n.kind) {
                    case expr_kind::input:
                        n.is_scalar = false;
                        return;
                    case expr_kind::scalar:
                        n.is_scalar = true;
                        return;
                    case expr_kind::add:
                    case expr_kind::subtract:
                    case expr_kind::multiply:
                    case expr_kind::divide:
                    case expr_kind::maximum:
                    case expr_kind::minimum: {
                        const gnode* t = a->is_scalar ? b : a;
                        n.is_scalar = t->is_scalar;
                        n.shape = t->shape;
                        return;
                    }
                    case expr_kind::exp:
                    case expr_kind::reciprocal:
                        n.is_scalar = a->is_scalar;
                        n.shape = a->shape;
                        return;
                    case expr_kind::matmul:
                        n.shape = {a->shape[0], b->shape[1]};
                        return;
                    case expr_kind::batched_matmul:
                        n.shape = {a->shape[0], a->shape[1], b->shape[2]};
                        return;
                    case expr_kind::slice:
                        n.shape = n.p_shape;
                        return;
                    case expr_kind::reshape:
                    case expr_kind::broadcast:
                        n.shape = n.p_shape;
                        return;
                    case expr_kind::unsqueeze:
                        n.shape = a->shape;
                        n.shape.insert(n.shape.begin() + static_cast<ptrdiff_t>(n.axis), 1);
                        return;
                    case expr_kind::transpose:
                        n.shape = {a->shape[1], a->shape[0]};
                        return;
                    case expr_kind::permute:
                        n.shape.resize(a->shape.size());
                        for (size_t d = 0; d < n.p_shape.size(); ++d)
                            n.shape[d] = a->shape[static_cast<size_t>(n.p_shape[d])];
                        return;
                    case expr_kind::concat:
                        n.shape = a->shape;
                        n.shape[n.axis] += b->shape[n.axis];
                        return;
                    case expr_kind::sum:
                    case expr_kind::max: {
                        if (n.keepdim) {
                            n.shape = a->shape;
                            n.shape[n.axis] = 1;
                        } else {
                            for (size_t d = 0; d < a->shape.size(); ++d)
                                if (d != n.axis) n.shape.push_back(a->shape[d]);
                            if (n.shape.empty()) n.shape.push_back(1);
                        }
                        return;
                    }
                }
            }
        };

        struct plan_cache {
            std::mutex mutex;
            std::unordered_map<uint64_t, std::vector<std::pair<std::string, std::shared_ptr<plan>>>>
                plans;
        };

        plan_cache& plans() {
            static plan_cache* c = new plan_cache();
            return *c;
        }

        std::shared_ptr<plan> lookup_plan(const graph& g) {
            // Plans built under the GEMM test hook never serve normal calls,
            // nor plans of another GEMM form.
            const std::string key = g.key + gemm_form_key() + (test_gemm_stall() ? "|test-stall" : "");
            plan_cache& c = plans();
            {
                std::scoped_lock lock{c.mutex};
                auto it = c.plans.find(g.hash);
                if (it != c.plans.end()) {
                    for (auto& [k, p] : it->second)
                        if (k == key) return p;
                }
            }
            std::shared_ptr<plan> p = build_plan(g);
            std::scoped_lock lock{c.mutex};
            c.plans[g.hash].emplace_back(key, p);
            return p;
        }

    } // namespace

    graph canonicalize(const tensor_expr::node& root) {
        canonicalizer c;
        c.g.hash = 0x6a09e667f3bcc909ULL;
        c.g.root = c.visit(root);
        c.g.hash = mix(c.g.hash, static_cast<uint64_t>(c.g.root));
        c.g.key += "|root=" + std::to_string(c.g.root);
        return std::move(c.g);
    }

    bool placeholder_mode() { return false; }

    namespace {

        struct bound_graph {
            graph g;
            std::shared_ptr<plan> p;
            shape_info info;
            int device = 0;
            // A pure view builds its (copy) plan only if a view cannot be
            // made when it is materialised.
            mutable std::once_flag plan_once;
            mutable std::shared_ptr<plan> view_copy_plan;
            plan* get_plan() const {
                if (p) return p.get();
                std::call_once(plan_once, [&] { view_copy_plan = lookup_plan(g); });
                return view_copy_plan.get();
            }
        };

        bool stale(const bound_graph& b) {
            for (const auto& [s, epoch] : b.g.view_inputs)
                if (s->layout_epoch.load(std::memory_order_acquire) != epoch) return true;
            return false;
        }

        struct host_profiler {
            std::atomic<bool> on{false};
            std::atomic<uint64_t> ns[phase_count]{};
            std::atomic<uint64_t> calls{0};
            std::mutex counter_mutex;
            std::map<std::string, uint64_t> counters;
        };

        host_profiler& hprof() {
            static host_profiler* h = new host_profiler();
            return *h;
        }

        uint64_t now_ns() {
            return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                             std::chrono::steady_clock::now().time_since_epoch())
                                             .count());
        }

        std::shared_ptr<const bound_graph> bind(const tensor_expr::node& root) {
            auto cached = std::static_pointer_cast<const bound_graph>(std::atomic_load(&root.bound));
            if (cached && !stale(*cached)) return cached;
            auto b = std::make_shared<bound_graph>();
            b->info = infer(root);
            if (!b->info.has_input)
                throw std::invalid_argument("tensor expression must reference at least one tensor");
            if (b->info.scalar)
                throw std::invalid_argument("scalar expression cannot materialize to a tensor");
            b->g = canonicalize(root);
            int device = -1;
            for (const auto& s : b->g.slots) {
                if (s->placeholder)
                    throw std::runtime_error("placeholder tensors can only be used to describe plans");
                if (device < 0) device = s->device;
            }
            b->device = device < 0 ? 0 : device;
            b->g.pure_view = pure_view(b->g, b->g.view_slot, b->g.view_layout);
            if (checked_numel(b->info.shape) != 0 && !b->g.pure_view) b->p = lookup_plan(b->g);
            std::shared_ptr<const void> erased = b;
            std::atomic_store(&root.bound, erased);
            return b;
        }

    } // namespace

    void host_profile_enable(bool on) { hprof().on.store(on); }

    void host_count(const char* what) {
        host_profiler& h = hprof();
        if (!h.on.load(std::memory_order_relaxed)) return;
        std::scoped_lock lock{h.counter_mutex};
        ++h.counters[what];
    }

    std::string host_profile_read() {
        host_profiler& h = hprof();
        static const char* names[phase_count] = {"bind", "stream", "order", "alloc",
                                                 "launch", "wrap", "total"};
        std::ostringstream os;
        const uint64_t calls = h.calls.exchange(0);
        os << "materialize_calls\t" << calls << "\n";
        {
            std::scoped_lock lock{h.counter_mutex};
            for (const auto& [k, v] : h.counters) os << k << "\t" << v << "\n";
            h.counters.clear();
        }
        for (int i = 0; i < phase_count; ++i) {
            const uint64_t v = h.ns[i].exchange(0);
            os << names[i] << "_us_per_call\t" << (calls ? double(v) / 1000.0 / double(calls) : 0.0)
               << "\n";
        }
        return os.str();
    }

    // The reference launches every nested sum/max first and the root graph
    // last, each refusing an empty input buffer when its own output is not
    // empty (src/cuda_jit.cpp:794-803, 875-884); the first launch to meet an
    // empty slot names the kind of launch it is.
    std::string empty_input_message(const graph& g, int slot) {
        std::vector<char> reads(g.nodes.size(), 0); // node's subtree reads `slot`
        for (size_t i = 0; i < g.nodes.size(); ++i) { // children precede parents
            const gnode& n = g.nodes[i];
            reads[i] = (n.kind == expr_kind::input && n.slot == slot) ||
                       (n.a >= 0 && reads[static_cast<size_t>(n.a)]) ||
                       (n.b >= 0 && reads[static_cast<size_t>(n.b)]);
            if ((n.kind == expr_kind::sum || n.kind == expr_kind::max) && n.a >= 0 &&
                reads[static_cast<size_t>(n.a)] && checked_numel(n.shape) != 0)
                return "CUDA reduction input is empty";
        }
        return "CUDA elementwise input is empty";
    }

    namespace {
        tensor materialize_impl(const tensor_expr::node& root, bool allow_view);
    }

    tensor materialize_graph(const tensor_expr::node& root) { return materialize_impl(root, true); }
    tensor materialize_graph_copy(const tensor_expr::node& root) { return materialize_impl(root, false); }

    namespace {
    tensor materialize_impl(const tensor_expr::node& root, bool allow_view) {
        host_profiler& hp = hprof();
        const bool timing = hp.on.load(std::memory_order_relaxed);
        uint64_t t0 = timing ? now_ns() : 0, t1 = 0, t2 = 0, t3 = 0, ta = 0, tb = 0;

        std::shared_ptr<const bound_graph> b = bind(root);
        const graph& g = b->g;
        const int device = b->device;
        const size_t count = checked_numel(b->info.shape);
        if (timing) t1 = now_ns();

        auto storage = std::make_shared<realized_storage>();
        storage->count = count;
        storage->device = device;
        auto stream = current_stream(device);
        if (count == 0) {
            // Empty result: no launch (src/tensor.cpp:1023-1028).
            storage->device_values = allocate(device, 0, stream);
            storage->host_current = true;
            return tensor_access::from_storage(b->info.shape, std::move(storage),
                                               b->info.placement);
        }
        if (allow_view && g.pure_view &&
            make_view(g.slots[static_cast<size_t>(g.view_slot)], g.view_layout, storage)) {
            // Data movement of one realised tensor: a strided view, no kernel.
            storage->count = count;
            storage->device = device;
            host_count("materialize_view");
            return tensor_access::from_storage(b->info.shape, std::move(storage), b->info.placement);
        }
        plan* p = b->get_plan();
        if (timing) ta = now_ns();

        for (size_t si = 0; si < g.slots.size(); ++si) {
            const auto& s = g.slots[si];
            const auto& st = cuda_jit::buffer_access::state(s->device_values);
            if (st == nullptr || st->ptr == 0)
                throw std::invalid_argument(empty_input_message(g, static_cast<int>(si)));
            if (st->device != device)
                throw std::invalid_argument("tensor expression devices must match");
            // Ordered behind its producer at its first launch (below), so a
            // launch waits only for the inputs it reads: an input still
            // uploading on another stream holds back only its readers.
        }
        if (timing) tb = now_ns();

        // Operand splits kept by their input's storage: the launch is
        // skipped and its hi / lo / flag temps are the kept buffers.
        std::vector<char> skip(p->launches.size(), 0);
        std::vector<cuda_jit::device_buffer> kept(p->temp_bytes.size());
        for (size_t li = 0; li < p->launches.size(); ++li) {
            const launch_spec& l = p->launches[li];
            if (l.cache_slot < 0) continue;
            realized_storage& st = *g.slots[static_cast<size_t>(l.cache_slot)];
            std::scoped_lock lock{st.view_mutex};
            for (const auto& e : st.splits) {
                if (e.key != l.cache_key) continue;
                skip[li] = 1;
                kept[static_cast<size_t>(l.cache_temps[0])] = e.hi;
                kept[static_cast<size_t>(l.cache_temps[1])] = e.lo;
                kept[static_cast<size_t>(l.cache_temps[2])] = e.flag;
                break;
            }
        }
        std::vector<cuda_jit::device_buffer> temps;
        temps.reserve(p->temp_bytes.size());
        for (size_t ti = 0; ti < p->temp_bytes.size(); ++ti) {
            if (const auto& ks = cuda_jit::buffer_access::state(kept[ti]); ks != nullptr) {
                order_read(*ks, stream);
                temps.push_back(kept[ti]);
                host_count("split_kept");
            } else {
                temps.push_back(allocate(device, p->temp_bytes[ti], stream));
            }
        }
        if (timing) t2 = now_ns();

        uint64_t error_word = 0;
        // Kernel arguments: one 8-byte pointer or value per argument (tensor
        // maps apart); up to 2048 of them fit the 32 KB parameter space of
        // sm_100 launches, so a graph may read that many distinct tensors.
        constexpr size_t kMaxArgs = 2048;
        thread_local std::vector<uint64_t> values;
        thread_local std::vector<void*> params;
        struct alignas(64) tensor_map_storage {
            unsigned char bytes[128];
        };
        tensor_map_storage maps[8];
        int nmaps = 0;
        std::vector<char> slot_ordered(g.slots.size(), 0);
        for (size_t li = 0; li < p->launches.size(); ++li) {
            if (skip[li]) continue;
            launch_spec& l = p->launches[li];
            pbrt_function fn = nullptr;
            const bool slot = device < static_cast<int>(l.per_device->function.size());
            if (slot) fn = l.per_device->function[device].load(std::memory_order_acquire);
            if (fn == nullptr) {
                std::scoped_lock lock{p->resolve_mutex};
                check(pbrt_get_function(device, l.image_key, l.name.c_str(), &fn));
                if (l.smem > 48 * 1024)
                    check(pbrt_function_set_max_dynamic_smem(fn, static_cast<int>(l.smem)));
                uint32_t pgrid = 0;
                if (l.persistent_units > 0) {
                    int per_sm = 0, sms = 0;
                    check(pbrt_occupancy(device, fn, static_cast<int>(l.block[0] * l.block[1] * l.block[2]),
                                         l.smem, &per_sm));
                    check(pbrt_device_attribute(device, 16 /* multiprocessor count */, &sms));
                    if (l.persistent_per_sm > 0) per_sm = std::min(per_sm, l.persistent_per_sm);
                    int64_t fit = std::max<int64_t>(1, int64_t{per_sm} * sms);
                    // Work units of a clustered kernel are clusters of
                    // cluster_x CTAs, as many as can be resident at once.
                    const int64_t cx = std::max<uint32_t>(1, l.cluster_x);
                    if (cx > 1) {
                        int clusters = 0;
                        check(pbrt_max_active_clusters(device, fn,
                                                       static_cast<int>(l.block[0] * l.block[1] * l.block[2]),
                                                       l.smem, l.cluster_x, &clusters));
                        fit = std::max<int64_t>(1, std::min<int64_t>(clusters, fit / cx));
                    }
                    pgrid = static_cast<uint32_t>(cx * std::min<int64_t>(l.persistent_units, fit));
                }
                if (slot) {
                    l.per_device->persistent_grid[device].store(pgrid, std::memory_order_relaxed);
                    l.per_device->function[device].store(fn, std::memory_order_release);
                }
            }
            if (l.args.size() > kMaxArgs) throw std::runtime_error("kernel has too many arguments");
            // Parameters are copied at launch: the tensor-map scratch serves
            // each launch afresh.
            nmaps = 0;
            if (values.size() < l.args.size()) {
                values.resize(l.args.size());
                params.resize(l.args.size());
            }
            for (size_t i = 0; i < l.args.size(); ++i) {
                const kernel_arg& a = l.args[i];
                switch (a.kind) {
                    case arg_kind::slot:
                        if (!slot_ordered[static_cast<size_t>(a.index)]) {
                            slot_ordered[static_cast<size_t>(a.index)] = 1;
                            order_read(*cuda_jit::buffer_access::state(
                                           g.slots[static_cast<size_t>(a.index)]->device_values),
                                       stream);
                        }
                        values[i] = cuda_jit::buffer_access::state(
                                        g.slots[static_cast<size_t>(a.index)]->device_values)
                                        ->ptr + static_cast<uint64_t>(a.elem_offset) * 4u;
                        break;
                    case arg_kind::temp:
                        values[i] = cuda_jit::buffer_access::state(
                                        temps[static_cast<size_t>(a.index)])
                                        ->ptr + static_cast<uint64_t>(a.elem_offset) * 4u;
                        break;
                    case arg_kind::error_word:
                        if (error_word == 0) check(pbrt_error_word(device, &error_word));
                        values[i] = error_word;
                        break;
                    case arg_kind::u64:
                        values[i] = a.value;
                        break;
                    case arg_kind::flag_clear: {
                        const bool is_kept = cuda_jit::buffer_access::state(kept[static_cast<size_t>(a.index)]) != nullptr;
                        const size_t t = is_kept ? static_cast<size_t>(a.value) : static_cast<size_t>(a.index);
                        values[i] = cuda_jit::buffer_access::state(temps[t])->ptr;
                        break;
                    }
                    case arg_kind::tmap: {
                        if (nmaps >= 8) throw std::runtime_error("a kernel has more than 8 tensor maps");
                        const uint64_t base =
                            cuda_jit::buffer_access::state(temps[static_cast<size_t>(a.index)])->ptr;
                        const uint64_t dims[2] = {static_cast<uint64_t>(a.cols), a.value};
                        const uint64_t strides[1] = {static_cast<uint64_t>(a.cols) * 4u};
                        const uint32_t box[2] = {static_cast<uint32_t>(a.box_cols),
                                                 static_cast<uint32_t>(a.box_rows)};
                        const uint32_t estride[2] = {1, 1};
                        // fp32, no interleave, the kernel's swizzle, 256-byte
                        // L2 promotion, zero fill.
                        check(pbrt_tensor_map_encode_tiled(maps[nmaps].bytes, 7, 2, base, dims,
                                                           strides, box, estride, 0, a.swizzle, 3, 0));
                        params[i] = maps[nmaps].bytes;
                        ++nmaps;
                        continue;
                    }
                }
                params[i] = &values[i];
            }
            std::array<uint32_t, 3> grid = l.grid;
            if (l.persistent_units > 0 && slot) {
                const uint32_t pg = l.per_device->persistent_grid[device].load(std::memory_order_relaxed);
                if (pg != 0) grid[0] = pg;
            }
            const uint32_t cluster[3] = {l.cluster_x, 1, 1};
            check(pbrt_launch_ex(device, fn, grid.data(), l.block.data(), l.smem, stream->stream,
                                 params.data(), l.cluster_x > 1 ? cluster : nullptr,
                                 l.pdl ? PBRT_LAUNCH_PDL : 0u));
        }
        // A slot whose every read was served by kept splits still joins the
        // stream's readers, so its eventual free is ordered after this work.
        for (size_t si = 0; si < g.slots.size(); ++si)
            if (!slot_ordered[si] && !p->launches.empty())
                order_read(*cuda_jit::buffer_access::state(g.slots[si]->device_values), stream);
        // Splits computed now are kept by their input's storage (a few per
        // storage, the oldest dropped first), unless a handle to its values
        // has been handed out.
        for (size_t li = 0; li < p->launches.size(); ++li) {
            const launch_spec& l = p->launches[li];
            if (l.cache_slot < 0 || skip[li]) continue;
            realized_storage& st = *g.slots[static_cast<size_t>(l.cache_slot)];
            std::scoped_lock lock{st.view_mutex};
            if (st.escaped || st.placeholder) continue;
            if (st.splits.size() >= 4) st.splits.erase(st.splits.begin());
            st.splits.push_back({l.cache_key, temps[static_cast<size_t>(l.cache_temps[0])],
                                 temps[static_cast<size_t>(l.cache_temps[1])],
                                 temps[static_cast<size_t>(l.cache_temps[2])]});
        }
        if (timing) t3 = now_ns();

        storage->device_values = temps[static_cast<size_t>(p->result_temp)];
        set_producer(*cuda_jit::buffer_access::state(storage->device_values), stream);
        tensor result = tensor_access::from_storage(b->info.shape, std::move(storage),
                                                    b->info.placement);
        if (timing) {
            const uint64_t t4 = now_ns();
            hp.ns[phase_bind] += t1 - t0;
            hp.ns[phase_stream] += ta - t1;
            hp.ns[phase_order] += tb - ta;
            hp.ns[phase_alloc] += t2 - tb;
            hp.ns[phase_launch] += t3 - t2;
            hp.ns[phase_wrap] += t4 - t3;
            hp.ns[phase_total] += t4 - t0;
            hp.calls += 1;
        }
        return result;
    }
    } // namespace

    std::string describe_plan(const tensor_expr::node& root, bool with_source) {
        shape_info info = infer(root);
        if (!info.has_input)
            throw std::invalid_argument("tensor expression must reference at least one tensor");
        if (info.scalar)
            throw std::invalid_argument("scalar expression cannot materialize to a tensor");
        graph g = canonicalize(root);
        std::shared_ptr<plan> p = lookup_plan(g);
        std::ostringstream os;
        os << "graph nodes=" << g.nodes.size() << " slots=" << g.slots.size()
           << " hash=" << std::hex << g.hash << std::dec << "\n";
        os << "temps=" << p->temp_bytes.size() << " result=t" << p->result_temp << "\n";
        for (const launch_spec& l : p->launches) {
            os << "kernel " << l.name << " grid=" << l.grid[0] << "x" << l.grid[1] << "x"
               << l.grid[2] << " block=" << l.block[0] << " smem=" << l.smem;
            if (l.cluster_x > 1) os << " cluster=" << l.cluster_x;
            os << " : " << l.schedule << "\n";
            if (with_source) os << l.source << "\n";
        }
        return os.str();
    }

} // namespace porch::detail
