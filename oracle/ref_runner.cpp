// Graph runner over porch's public C++ API (TEST / BENCHMARK INFRASTRUCTURE).
//
// The same source is compiled twice by oracle/build.py:
//  - against the reference's own headers and sources (oracle/_ref/ref_runner):
//    this is how the reference's NVRTC-JIT path is run on the GPU box, as a
//    separate process because both libraries define `porch::`;
//  - against this repository's drop-in headers and libporch_b200.so
//    (oracle/_build/pb_runner), which shows that code written against the
//    reference's API compiles and links unchanged.
//
// Modes
//   eval <program file> <inputs file> <output file>
//       Builds the program (the oracle's text format, see oracle/oracle.cpp)
//       through the porch API, materialises it and writes the result.
//       Inputs file: repeated [int64 rank][int64 dims...][float32 data...].
//       Output file: [int64 rank][int64 dims...][float32 data...].
//   bench <config> <steps> <warmup> [e2e]
//       Times the benchmark config with synthetic inputs (pb_fill_synthetic)
//       and prints one JSON object: device-resident materialize+synchronize
//       per step, and with "e2e" also host tensor construction and cpu().
#include "porch/ops.hpp"
#include "porch/tensor.hpp"

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <fstream>
#include <iostream>
#include <map>
#include <optional>
#include <sstream>
#include <string>
#include <vector>

extern "C" int pb_fill_synthetic(float* values, size_t count, uint64_t seed, int dist, double a,
                                 double b);

namespace {

    using porch::index_t;

    struct value {
        std::optional<porch::tensor_expr> expr;
        std::optional<porch::tensor> tensor;
    };

    std::vector<index_t> dims(const std::string& s) {
        std::vector<index_t> d;
        if (s == "-") return d;
        std::stringstream ss(s);
        std::string x;
        while (std::getline(ss, x, ',')) d.push_back(std::stoll(x));
        return d;
    }

    porch::tensor_expr E(const value& v) {
        if (v.expr) return *v.expr;
        return porch::tensor_expr{*v.tensor};
    }

    porch::tensor_expr index(const porch::tensor& t, const std::string& spec_text) {
        std::vector<porch::tensor_index> idx;
        std::stringstream ss(spec_text);
        std::string s;
        while (std::getline(ss, s, ';')) {
            if (s.empty() || s == "-") continue;
            if (s[0] == 'i') {
                idx.emplace_back(porch::index_t{std::stoll(s.substr(1))});
            } else if (s[0] == 's') {
                long a = 0, b = 0, c = 1;
                std::sscanf(s.c_str() + 1, "%ld:%ld:%ld", &a, &b, &c);
                idx.emplace_back(porch::slice{a, b, c});
            } else {
                idx.emplace_back(porch::all);
            }
        }
        switch (idx.size()) {
            case 0: return t[{}];
            case 1: return t[{idx[0]}];
            case 2: return t[{idx[0], idx[1]}];
            case 3: return t[{idx[0], idx[1], idx[2]}];
            case 4: return t[{idx[0], idx[1], idx[2], idx[3]}];
            default: throw std::invalid_argument("too many tensor indices");
        }
    }

    porch::tensor run_program(const std::string& program, const std::vector<porch::tensor>& inputs) {
        // A deque keeps element addresses stable: the reference's expression
        // nodes hold raw `const tensor*` pointers to the tensors stored here
        // (src/tensor.cpp:50), so they must never move.
        std::deque<value> vals;
        std::stringstream lines(program);
        std::string line;
        size_t last = 0;
        while (std::getline(lines, line)) {
            if (line.empty()) continue;
            std::stringstream ls(line);
            size_t id = 0;
            std::string op;
            ls >> id >> op;
            if (vals.size() <= id) vals.resize(id + 1);
            auto arg = [&]() -> value& {
                size_t a = 0;
                ls >> a;
                return vals.at(a);
            };
            value out;
            if (op == "input") {
                size_t slot = 0;
                ls >> slot;
                out.tensor = inputs.at(slot);
            } else if (op == "scalar") {
                std::string hex;
                ls >> hex;
                uint32_t bits = static_cast<uint32_t>(std::stoul(hex, nullptr, 16));
                float f;
                std::memcpy(&f, &bits, 4);
                out.expr = porch::tensor_expr{f};
            } else if (op == "add" || op == "subtract" || op == "multiply" || op == "divide" ||
                       op == "maximum" || op == "minimum" || op == "matmul") {
                porch::tensor_expr a = E(arg());
                porch::tensor_expr b = E(arg());
                if (op == "add") out.expr = a + b;
                else if (op == "subtract") out.expr = a - b;
                else if (op == "multiply") out.expr = a * b;
                else if (op == "divide") out.expr = a / b;
                else if (op == "maximum") out.expr = porch::maximum(a, b);
                else if (op == "minimum") out.expr = porch::minimum(a, b);
                else out.expr = porch::matmul(a, b);
            } else if (op == "exp") {
                out.expr = porch::exp(E(arg()));
            } else if (op == "reciprocal") {
                out.expr = porch::reciprocal(E(arg()));
            } else if (op == "transpose") {
                out.expr = porch::transpose(E(arg()));
            } else if (op == "relu") {
                out.expr = porch::relu(E(arg()));
            } else if (op == "logistic") {
                out.expr = porch::logistic(E(arg()));
            } else if (op == "softmax") {
                porch::tensor_expr a = E(arg());
                size_t axis = 0;
                ls >> axis;
                out.expr = porch::softmax(a, axis);
            } else if (op == "reshape" || op == "broadcast") {
                porch::tensor_expr a = E(arg());
                std::string d;
                ls >> d;
                out.expr = op == "reshape" ? porch::reshape(a, dims(d)) : porch::broadcast_to(a, dims(d));
            } else if (op == "unsqueeze") {
                porch::tensor_expr a = E(arg());
                size_t axis = 0;
                ls >> axis;
                out.expr = porch::unsqueeze(a, axis);
            } else if (op == "concat") {
                porch::tensor_expr a = E(arg());
                porch::tensor_expr b = E(arg());
                size_t axis = 0;
                ls >> axis;
                out.expr = porch::concat(a, b, axis);
            } else if (op == "sum" || op == "max") {
                porch::tensor_expr a = E(arg());
                size_t axis = 0;
                int keep = 0;
                ls >> axis >> keep;
                out.expr = op == "sum" ? porch::sum(a, axis, keep != 0) : porch::max(a, axis, keep != 0);
            } else if (op == "tensor") {
                porch::tensor t = E(arg());
                out.tensor = t;
            } else if (op == "materialize") {
                out.tensor = porch::materialize(E(arg()));
            } else if (op == "index") {
                value& a = arg();
                std::string spec;
                ls >> spec;
                out.expr = index(*a.tensor, spec);
            } else {
                throw std::invalid_argument("unknown op " + op);
            }
            vals[id] = std::move(out);
            last = id;
        }
        return porch::materialize(E(vals.at(last)));
    }

    int eval_mode(const char* program_file, const char* inputs_file, const char* output_file) {
        std::ifstream pf(program_file);
        std::string program((std::istreambuf_iterator<char>(pf)), {});
        std::ifstream inf(inputs_file, std::ios::binary);
        std::vector<porch::tensor> inputs;
        for (;;) {
            int64_t rank = 0;
            if (!inf.read(reinterpret_cast<char*>(&rank), 8)) break;
            std::vector<index_t> shape(static_cast<size_t>(rank));
            size_t n = 1;
            for (auto& d : shape) {
                inf.read(reinterpret_cast<char*>(&d), 8);
                n *= static_cast<size_t>(d);
            }
            std::vector<float> data(n);
            inf.read(reinterpret_cast<char*>(data.data()), static_cast<std::streamsize>(n * 4));
            inputs.emplace_back(shape, std::move(data));
        }
        try {
            porch::tensor out = run_program(program, inputs);
            std::vector<float> host = out.cpu();
            std::ofstream of(output_file, std::ios::binary);
            const int64_t rank = static_cast<int64_t>(out.rank());
            of.write(reinterpret_cast<const char*>(&rank), 8);
            for (index_t d : out.shape()) of.write(reinterpret_cast<const char*>(&d), 8);
            of.write(reinterpret_cast<const char*>(host.data()),
                     static_cast<std::streamsize>(host.size() * 4));
        } catch (const std::invalid_argument& e) {
            std::cerr << "invalid_argument: " << e.what() << "\n";
            return 3;
        } catch (const std::out_of_range& e) {
            std::cerr << "out_of_range: " << e.what() << "\n";
            return 4;
        }
        return 0;
    }

    // ------------------------------------------------------------ bench --
    struct input_spec {
        std::vector<index_t> shape;
        int dist;
        double a, b;
    };

    constexpr uint64_t kSeed = 20261201ULL;

    std::map<std::string, std::vector<input_spec>> config_inputs() {
        const double s8192 = 1.0 / 90.50966799187808;  // 1/sqrt(8192)
        return {
            {"c1_elementwise", {{{1 << 24}, 0, -1, 1}, {{1 << 24}, 0, -1, 1}}},
            {"c2_view", {{{8192, 8192}, 1, 0, 1}, {{4096}, 0, -0.5, 0.5}, {{6144, 4096}, 1, 0, 1}}},
            {"c3a_softmax", {{{65536, 4096}, 1, 0, 2}}},
            {"c3b_relu_logistic", {{{65536, 4096}, 1, 0, 2}}},
            {"c4_matmul",
             {{{8192, 8192}, 0, -s8192, s8192}, {{8192, 8192}, 0, -s8192, s8192}, {{8192}, 0, -0.1, 0.1}}},
            {"c5_mlp",
             {{{16384, 4096}, 1, 0, 1},
              {{4096, 16384}, 1, 0, 1.0 / 64.0},
              {{16384}, 0, -0.1, 0.1},
              {{16384, 4096}, 1, 0, 1.0 / 128.0},
              {{4096}, 0, -0.1, 0.1}}},
        };
    }

    porch::tensor run_config(const std::string& name, const std::vector<porch::tensor>& t,
                             bool staged) {
        using namespace porch;
        if (name == "c1_elementwise") return materialize((t[0] + t[1]) * 2.0F - 1.0F);
        if (name == "c2_view") {
            tensor_expr xs = t[0][{slice{0, 8192, 2}, slice{1024, 7168}}];
            return materialize(concat(transpose(xs) + broadcast_to(t[1], {6144, 4096}), t[2], 0));
        }
        if (name == "c3a_softmax") return materialize(softmax(t[0], 1));
        if (name == "c3b_relu_logistic") return materialize(logistic(relu(t[0])));
        if (name == "c4_matmul")
            return materialize(relu(matmul(t[0], t[1]) + broadcast_to(t[2], {8192, 8192})));
        if (name == "c5_mlp") {
            const index_t m = t[0].shape()[0];
            if (staged) {
                tensor h = materialize(logistic(matmul(t[0], t[1]) + broadcast_to(t[2], {m, 16384})));
                tensor z = materialize(matmul(h, t[3]) + broadcast_to(t[4], {m, 4096}));
                return materialize(softmax(z, 1));
            }
            tensor_expr h = logistic(matmul(t[0], t[1]) + broadcast_to(t[2], {m, 16384}));
            return materialize(softmax(matmul(h, t[3]) + broadcast_to(t[4], {m, 4096}), 1));
        }
        throw std::invalid_argument("unknown config " + name);
    }

    int bench_mode(const std::string& name, int steps, int warmup, bool e2e, index_t rows) {
        auto specs = config_inputs().at(name);
        if (rows > 0 && (name == "c3a_softmax" || name == "c3b_relu_logistic" || name == "c5_mlp"))
            specs[0].shape[0] = rows;
        std::vector<std::vector<float>> host;
        for (size_t i = 0; i < specs.size(); ++i) {
            size_t n = 1;
            for (index_t d : specs[i].shape) n *= static_cast<size_t>(d);
            host.emplace_back(n);
            pb_fill_synthetic(host.back().data(), n, kSeed + i, specs[i].dist, specs[i].a, specs[i].b);
        }
        const bool staged = true;
        std::vector<porch::tensor> t;
        for (size_t i = 0; i < specs.size(); ++i) t.emplace_back(specs[i].shape, host[i]);
        using clock = std::chrono::steady_clock;
        auto cold0 = clock::now();
        porch::tensor first = run_config(name, t, staged);
        first.synchronize();
        const double cold_ms = std::chrono::duration<double, std::milli>(clock::now() - cold0).count();
        for (int w = 0; w < warmup; ++w) run_config(name, t, staged).synchronize();
        auto t0 = clock::now();
        for (int s = 0; s < steps; ++s) run_config(name, t, staged).synchronize();
        const double warm_ms =
            std::chrono::duration<double, std::milli>(clock::now() - t0).count() / std::max(1, steps);
        double e2e_ms = -1.0;
        size_t h2d = 0, d2h = 0;
        if (e2e) {
            std::vector<float> out_host;
            for (int w = 0; w < std::max(1, warmup / 2); ++w) {
                std::vector<porch::tensor> tt;
                for (size_t i = 0; i < specs.size(); ++i) tt.emplace_back(specs[i].shape, host[i]);
                out_host = run_config(name, tt, staged).cpu();
            }
            auto e0 = clock::now();
            for (int s = 0; s < steps; ++s) {
                std::vector<porch::tensor> tt;
                for (size_t i = 0; i < specs.size(); ++i) tt.emplace_back(specs[i].shape, host[i]);
                out_host = run_config(name, tt, staged).cpu();
            }
            e2e_ms = std::chrono::duration<double, std::milli>(clock::now() - e0).count() /
                     std::max(1, steps);
            for (auto& h : host) h2d += h.size() * 4;
            d2h = out_host.size() * 4;
        }
        std::printf(
            "{\"config\": \"%s\", \"steps\": %d, \"warmup\": %d, \"cold_ms\": %.6f, "
            "\"warm_ms\": %.6f, \"e2e_ms\": %.6f, \"h2d_bytes\": %zu, \"d2h_bytes\": %zu, "
            "\"staged\": %s, \"rows\": %lld}\n",
            name.c_str(), steps, warmup, cold_ms, warm_ms, e2e_ms, h2d, d2h, staged ? "true" : "false",
            static_cast<long long>(specs[0].shape[0]));
        return 0;
    }

} // namespace

int main(int argc, char** argv) {
    if (argc >= 5 && std::string{argv[1]} == "eval") return eval_mode(argv[2], argv[3], argv[4]);
    if (argc >= 5 && std::string{argv[1]} == "bench") {
        const bool e2e = argc >= 6 && std::string{argv[5]} == "e2e";
        const index_t rows = argc >= 7 ? std::stoll(argv[6]) : 0;
        return bench_mode(argv[2], std::atoi(argv[3]), std::atoi(argv[4]), e2e, rows);
    }
    std::fprintf(stderr,
                 "usage: %s eval <program> <inputs> <output> | bench <config> <steps> <warmup> [e2e [rows]]\n",
                 argv[0]);
    return 2;
}
