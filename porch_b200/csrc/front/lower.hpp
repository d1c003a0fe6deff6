// Lowering internals shared by lower.cpp and the tensor-core GEMM emitter.
#pragma once

#include "plan.hpp"

#include <map>
#include <sstream>
#include <string>
#include <vector>

namespace porch::detail {

    // Integer affine map of the output (root) coordinates:
    // value(c) = off + sum_d st[d] * c[d].
    struct affine {
        int64_t off = 0;
        std::vector<int64_t> st;
    };

    // Where a node is evaluated: either as coordinates of the node's own
    // shape (one affine map per dimension) or as a linear index into the
    // node's contiguous layout.
    struct position {
        bool linear = false;
        affine lin;
        std::vector<affine> coords;
    };

    struct need_split {
        int dim;
        int64_t at;
    };
    struct not_affine {};
    struct not_fusable {};

    // Straight-line value graph of one output box.
    struct vnode {
        enum class op : uint8_t { load, scalar, acc, unary, binary } kind = op::scalar;
        expr_kind ek = expr_kind::add;
        int a = -1;
        int b = -1;
        int buffer = -1; // kernel leaf index
        affine map;      // element index of the load
        float scalar = 0.0F;
    };

    struct box {
        std::vector<int64_t> lo;
        std::vector<int64_t> hi;
        std::vector<vnode> nodes;
        int root = -1;
    };

    const char* kernel_prelude();

    // Test hook (off by default; part of the plan key): tcgen05 GEMMs built
    // while it is on make CTA 0 wait on a barrier nothing arrives on, so the
    // bounded wait expires and the kernel reports and tears down.
    void set_test_gemm_stall(bool on);
    // Whether an [M, K] @ [K, N] product runs on the tensor cores.
    bool tensor_core_gemm(int64_t M, int64_t N, int64_t K);
    bool test_gemm_stall();
    // PORCH_B200_GEMM ("simt": no tensor-core GEMMs; "single": one CTA per
    // tile instead of CTA pairs, cta_group::2), as a suffix of the plan key.
    std::string gemm_form_key();

    // A matmul operand [rows, cols] read in place: element (i, j) at
    // off + i * s0 + j * s1 of `arg` (an input slot, or a contiguous temp).
    // Temps of one tensor-core GEMM's operand splits and flags (a caller may
    // supply them, e.g. when A's halves come from the GEMM that produced A).
    struct gemm_temps {
        int a_hi = -1, a_lo = -1, b_hi = -1, b_lo = -1, nf = -1, fa = -1, fb = -1;
        // A's hi / lo / flag were written by the GEMM that produced A (its
        // split-output epilogue): no split pass for A, and fa not cleared.
        bool a_ready = false;
    };

    // A GEMM epilogue that writes its result as the 3xTF32 halves a
    // following GEMM reads for its A operand: hi / lo temps of rows of `kp`
    // floats (kp = the result's columns, a multiple of 32) and a flag set
    // when a result is Inf or NaN (lo is then 0, so hi + lo is the result).
    struct split_output {
        int hi = -1, lo = -1, flag = -1;
        int64_t kp = 0;
    };

    // A grouped batched GEMM: `count` products [M, K] @ [K, N] of contiguous
    // operands ([count, M, K] and [count, K, N]) into [count, M, N], every
    // batch's tiles in one launch; leaf_stride[i] = elements between
    // consecutive batches of epilogue leaf i (0: the same for every batch).
    struct gemm_batches {
        int64_t count = 1;
        std::vector<int64_t> leaf_stride;
    };

    struct gemm_operand {
        kernel_arg arg;
        int64_t off = 0;
        int64_t s0 = 0;
        int64_t s1 = 1;
        // Set when the operand exists only as 3xTF32 halves: element
        // (i, j) = arg[..] + lo[..] at the same offsets (a GEMM's
        // split-output result, read by the CUDA-core fallback).
        bool has_lo = false;
        kernel_arg lo;
        bool contiguous(int64_t cols) const { return off == 0 && s1 == 1 && s0 == cols; }
    };

    class lowerer {
      public:
        lowerer(const graph& g, plan& p);
        int materialize(int id);

        struct kernel {
            std::vector<kernel_arg> leaves;
            int leaf(arg_kind kind, int index);
        };

      private:
        struct row_operand {
            kernel k;
            box b;
            std::vector<index_t> shape;
        };

        int new_temp(size_t bytes);
        bool match_softmax(int id, int& x, size_t& axis) const;
        bool is_barrier(int id) const;
        int match_gemm(int id) const;
        kernel_arg as_buffer(int id);
        // A rank-2 matmul operand: an input, a slice of an input (e.g. a
        // strided view), or a transpose of either, read in place with
        // strides; anything else is materialised into a contiguous temp.
        gemm_operand as_gemm_operand(int id);

        static std::string pos_key(const position& p);
        affine to_linear(const position& p, const std::vector<index_t>& shape) const;
        std::vector<affine> to_coords(const position& p, const std::vector<index_t>& shape,
                                      const box& b) const;
        static int push(box& b, vnode v);
        int build(kernel& k, box& b, int id, const position& pos, int acc_id,
                  std::map<std::string, int>& memo);
        std::vector<box> build_boxes(kernel& k, int root, const std::vector<index_t>& shape,
                                     int acc_id);

        std::string emit_expr_function(const box& b, const std::string& tag,
                                       std::vector<int>& load_order) const;
        bool needs_wide(const std::vector<box>& boxes, const std::vector<index_t>& shape) const;
        std::string address(const affine& a, const std::vector<std::string>& cvar, bool wide,
                            int skip_dim) const;
        std::string emit_row_box(const box& b, int tag, const std::vector<index_t>& shape,
                                 bool wide, int64_t& ctas, std::string& desc) const;
        std::string emit_tile_box(const box& b, int tag, const std::vector<index_t>& shape,
                                  bool wide, int p, int64_t& ctas, int& smem_tiles,
                                  std::string& desc) const;
        static void finish_kernel(launch_spec& l);

        int emit_elementwise(int id);
        std::string gen_value(kernel& k, int id, const std::string& idx,
                              std::ostringstream& stmts, int& counter);
        int emit_generic(int id);
        row_operand row_prologue(int operand, size_t axis);
        int emit_reduce(int id);
        int emit_softmax(int id, int x);
        int emit_gemm(int id, int mm);
        // CUDA-core GEMM (fp32 FMA chain in k order). out_temp >= 0 writes
        // into that temp; guard_temp >= 0 runs only when its first int is set.
        // out_off: the output starts out_off floats into out_temp; batches > 1:
        // that many products over contiguous operands (blockIdx.y).
        int emit_gemm_simt(const box& b, kernel& k, const gemm_operand& A, const gemm_operand& B,
                           int64_t M, int64_t N, int64_t K, int out_temp = -1, int guard_temp = -1,
                           int64_t out_off = 0, int64_t batches = 1, const split_output* so = nullptr,
                           const std::vector<int64_t>* leaf_batch_stride = nullptr);
        // When matmul operand `a` ([M, K]) is a GEMM-with-epilogue read by
        // nothing else, lowers it with a split-output epilogue into `t`'s A
        // temps and returns true; `op` then reads those halves.
        bool presplit_operand(int a, int64_t M, int64_t N, int64_t K, gemm_temps& t, gemm_operand& op);
        // Internal batched matmul [B, M, K] @ [B, K, N] at `mm`, with the
        // elementwise graph `id` (rank 3, the product as one leaf; id == mm
        // for the bare product) as the epilogue: one grouped tensor-core GEMM
        // over every batch's tiles (epilogue leaves moved by their batch
        // strides), or one CUDA-core launch over every batch for a bare
        // product. Returns -1 when the epilogue cannot be fused (the caller
        // then realises the product on its own).
        int emit_batched_gemm(int id, int mm);
        // tcgen05 3xTF32 path; returns -1 when the shape is not eligible. On
        // success *nonfinite receives a temp whose first int is set when an
        // operand holds Inf or NaN (the tensor-core result is then skipped).
        // With row_partials != nullptr the epilogue is a softmax over each
        // output row: the result temp receives exp(y - m) per 128 x 256 tile
        // and *row_partials a temp of [M, ceil(N / 256)] float2 (m, sum) --
        // the tile's row maximum and its sum of exp(y - m).
        int emit_gemm_tc(int id, const box& b, kernel& k, const gemm_operand& A,
                         const gemm_operand& B, int64_t M, int64_t N, int64_t K, int* nonfinite,
                         int* row_partials = nullptr, int out_temp = -1, int64_t out_off = 0,
                         gemm_temps* shared = nullptr, const split_output* so = nullptr,
                         const gemm_batches* batches = nullptr);
        // softmax(x, last axis) where x is an elementwise tree over one
        // rank-2 matmul `mm`: the GEMM's softmax epilogue plus a normalising
        // pass; -1 when the tensor-core GEMM does not apply.
        int emit_gemm_softmax(int id, int x, int mm);

        const graph& g_;
        plan& p_;
        std::map<int, int> done_;
        int rank_ = 0;
    };

} // namespace porch::detail
