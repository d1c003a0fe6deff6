// Canonical graphs, lowering plans and kernel launch descriptions.
//
// A porch expression tree is value-numbered into a `graph` (common
// subexpressions merged, inputs numbered into slots by storage identity).
// The graph's 64-bit structural hash keys a process-wide plan cache, so a
// graph shape seen before skips lowering, code generation and NVRTC entirely
// and costs one hash walk plus its launches.
#pragma once

#include "detail.hpp"

#include <array>
#include <atomic>
#include <map>
#include <string>
#include <vector>

namespace porch::detail {

    struct gnode {
        expr_kind kind = expr_kind::scalar;
        int a = -1;
        int b = -1;
        int slot = -1;
        float scalar = 0.0F;
        bool is_scalar = false;
        std::vector<index_t> shape;     // inferred output shape
        std::vector<index_t> p_shape;   // slice shape / reshape+broadcast target
        std::vector<index_t> p_strides; // slice strides
        index_t p_offset = 0;           // slice offset
        size_t axis = 0;
        bool keepdim = false;
    };

    struct graph {
        std::vector<gnode> nodes;
        int root = -1;
        std::vector<std::shared_ptr<realized_storage>> slots;
        std::vector<std::vector<index_t>> slot_shapes;
        std::vector<int> uses; // number of parents per node
        uint64_t hash = 0;
        std::string key; // full structural key (verifies plan-cache hash hits)
        // Inputs that were strided views, read through their base, with the
        // layout epoch seen: a bound graph is rebuilt once one of them has
        // turned into contiguous values.
        std::vector<std::pair<std::shared_ptr<realized_storage>, uint32_t>> view_inputs;
        // The root is a strided view of one input slot (slice, transpose,
        // unsqueeze, contiguous reshape and permute only): materialising it
        // needs no kernel.
        bool pure_view = false;
        int view_slot = -1;
        strided_layout view_layout;
    };

    graph canonicalize(const tensor_expr::node& root);

    // ------------------------------------------------------ strided views --
    // The layout of slicing `src`'s logical (contiguous) index space with
    // (offset, strides, shape) -- the parameters tensor::operator[] records --
    // over src's own storage; false when a stride does not step along one of
    // src's dimensions without carrying into the next.
    bool compose_slice(const strided_layout& src, index_t offset, const std::vector<index_t>& strides,
                       const std::vector<index_t>& shape, strided_layout& out);
    // True when `g`'s root only moves the data of one input slot (slice,
    // transpose, permute, unsqueeze, reshape of a contiguous layout):
    // `layout` is then the root over that slot's values.
    bool pure_view(const graph& g, int& slot, strided_layout& layout);
    // Makes `view` a view of `base` (false when base's values have been
    // handed out or base is itself a view or a placeholder).
    bool make_view(const std::shared_ptr<realized_storage>& base, const strided_layout& layout,
                   const std::shared_ptr<realized_storage>& view);
    // materialize_graph that always writes a new contiguous result.
    tensor materialize_graph_copy(const tensor_expr::node& root);

    // ---------------------------------------------------------- launches --
    enum class arg_kind : uint8_t {
        slot,       // pointer to an input slot's device values
        temp,       // pointer to a plan temporary
        error_word, // pointer to the device's error block
        u64,        // immediate
        tmap,       // TMA tensor map (128 bytes) over a temp: `value` rows x
                    // `cols` fp32, box `box_rows` x `box_cols`, 128B swizzle
        flag_clear, // temp `index` (an operand's non-finite flag) to clear, or
                    // temp `value` when that operand's split is kept (below)
    };

    struct kernel_arg {
        arg_kind kind = arg_kind::u64;
        int index = 0;
        uint64_t value = 0;
        // slot / temp: the pointer passed is the buffer's + elem_offset floats
        // (one batch of a batched matmul; the kernel source stays the same).
        int64_t elem_offset = 0;
        int64_t cols = 0;
        int box_rows = 0;
        int box_cols = 0;
        int swizzle = 3; // CUtensorMapSwizzle: 1 = 32B, 2 = 64B, 3 = 128B
    };

    struct launch_spec {
        std::string name;      // kernel entry point
        std::string source;    // full NVRTC source
        std::string schedule;  // one-line description for plan dumps
        uint64_t image_key = 0;
        std::array<uint32_t, 3> grid{1, 1, 1};
        std::array<uint32_t, 3> block{256, 1, 1};
        uint32_t smem = 0;
        std::vector<kernel_arg> args;
        // Persistent kernels loop over `persistent_units` work units with a
        // grid-stride loop; their grid is fixed on first launch per device to
        // exactly the CTAs that fit at once (SMs x occupancy; for a clustered
        // kernel, whose units are clusters, the clusters that fit), so no CTA
        // waits for a second wave. 0 = launch `grid` as given.
        int64_t persistent_units = 0;
        // With persistent_units: at most this many CTAs per SM (0: as many
        // as fit), e.g. to keep the rows in flight inside L2.
        int persistent_per_sm = 0;
        // Thread-block cluster size along x (1: no cluster); grid[0] is a
        // multiple of it.
        uint32_t cluster_x = 1;
        // A 3xTF32 operand split of input slot `cache_slot` (>= 0) that the
        // slot's storage may keep under `cache_key`: when it holds one, the
        // launch is skipped and temps cache_temps = {hi, lo, flag} are bound
        // to the kept buffers; otherwise, after the launch, those temps are
        // kept. Storage whose device handle was handed out is never kept.
        int cache_slot = -1;
        std::string cache_key;
        std::array<int, 3> cache_temps{-1, -1, -1};
        // The kernel waits for the stream's previous kernel itself
        // (griddepcontrol.wait first thing), so it may launch with
        // programmatic stream serialization.
        bool pdl = false;
        // Per device, filled on first launch under the plan's resolve mutex
        // and read without it by every later launch (from any thread): the
        // function is published with release order after the grid.
        struct resolved {
            std::array<std::atomic<pbrt_function>, 16> function{};
            std::array<std::atomic<uint32_t>, 16> persistent_grid{};
        };
        std::shared_ptr<resolved> per_device = std::make_shared<resolved>();
    };

    struct plan {
        std::vector<size_t> temp_bytes;
        int result_temp = -1;
        std::vector<launch_spec> launches;
        std::vector<index_t> out_shape;
        std::mutex resolve_mutex;
    };

    // Builds the plan for `g` (lowering + code generation + NVRTC compile).
    std::shared_ptr<plan> build_plan(const graph& g);

    // NVRTC options used for every generated kernel: sm_100a cubin, IEEE
    // division and square root, no FMA contraction (bit-exact elementwise
    // arithmetic against the host oracle), no flush-to-zero.
    const std::vector<std::string>& kernel_options();

    // Formats a float as an exact CUDA literal.
    std::string float_literal(float v);

} // namespace porch::detail
