"""Writes tests/golden/known_answers.json: the known-answer cases of the
reference's own test suite (AkhilSamavedam/porch, tests/tensor_test.cpp),
restated as graph programs (oracle/oracle.cpp's text format) with the
expected values the reference asserts. Each case cites the lines it follows.

Run: python tests/golden/make_known_answers.py
"""

import json
from pathlib import Path

def hx(x):
    import struct
    return f"{struct.unpack('<I', struct.pack('<f', float(x)))[0]:08x}"

CASES = []


def case(name, source, inputs, program, expect=None, interval=None, exact_at=None, error=None,
         shape=None):
    CASES.append({"name": name, "source": source, "inputs": inputs, "program": program,
                  "expect": expect, "interval": interval, "exact_at": exact_at, "error": error,
                  "shape": shape})


L23 = [[2, 2], [1, 2, 3, 4]]
R23 = [[2, 2], [10, 20, 30, 40]]
S6 = [[2, 3], [1, 2, 3, 4, 5, 6]]

case("bracket_slice_selects_contiguous_copy", "tests/tensor_test.cpp:54-70",
     [[[6], [0, 1, 2, 3, 4, 5]]], "0 input 0\n1 index 0 s1:6:2\n", [1, 3, 5], shape=[3])
case("bracket_slice_returns_lazy_expression", "tests/tensor_test.cpp:72-85",
     [[[6], [0, 1, 2, 3, 4, 5]]], f"0 input 0\n1 index 0 s1:6:2\n2 scalar {hx(2)}\n3 multiply 1 2\n",
     [2, 6, 10])
case("bracket_slice_handles_multiple_dimensions", "tests/tensor_test.cpp:87-106",
     [[[3, 4], list(range(12))]], "0 input 0\n1 index 0 i1;s1:4:2\n", [5, 7], shape=[2])
case("add_uses_cuda_backend", "tests/tensor_test.cpp:119-130", [L23, R23],
     "0 input 0\n1 input 1\n2 add 0 1\n", [11, 22, 33, 44])
case("subtract_uses_cuda_backend", "tests/tensor_test.cpp:132-143", [R23, L23],
     "0 input 0\n1 input 1\n2 subtract 0 1\n", [9, 18, 27, 36])
case("multiply_uses_cuda_backend", "tests/tensor_test.cpp:145-156", [L23, R23],
     "0 input 0\n1 input 1\n2 multiply 0 1\n", [10, 40, 90, 160])
EL = [[[2, 3], [-3, -1, 0, 2, 4, 8]], [[2, 3], [6, -5, 3, 2, -4, 0.5]]]
case("elementwise_sum", "tests/tensor_test.cpp:158-169", EL, "0 input 0\n1 input 1\n2 add 0 1\n",
     [3, -6, 3, 4, 0, 8.5])
case("elementwise_difference", "tests/tensor_test.cpp:170-173", EL,
     "0 input 0\n1 input 1\n2 subtract 0 1\n", [-9, 4, -3, 0, 8, 7.5])
case("elementwise_product", "tests/tensor_test.cpp:174-178", EL,
     "0 input 0\n1 input 1\n2 multiply 0 1\n", [-18, 5, 0, 4, -16, 4])
case("chained_arithmetic", "tests/tensor_test.cpp:181-192",
     [[[2, 3], [1, 2, 3, 4, 5, 6]], [[2, 3], [6, 5, 4, 3, 2, 1]]],
     f"0 input 0\n1 input 1\n2 add 0 1\n3 scalar {hx(1)}\n4 subtract 0 3\n5 multiply 2 4\n6 subtract 5 1\n",
     [-6, 2, 10, 18, 26, 34])
case("fused_expression_materializes_once", "tests/tensor_test.cpp:194-206", [L23, R23],
     f"0 input 0\n1 input 1\n2 scalar {hx(2)}\n3 multiply 1 2\n4 add 0 3\n5 scalar {hx(1)}\n6 subtract 4 5\n",
     [20, 41, 62, 83])
case("multiline_expression_stays_lazy", "tests/tensor_test.cpp:208-222", [L23, R23],
     f"0 input 0\n1 input 1\n2 add 0 1\n3 scalar {hx(2)}\n4 multiply 2 3\n5 scalar {hx(1)}\n6 subtract 4 5\n",
     [21, 43, 65, 87])
case("tensor_assignment_keeps_graph_lazy", "tests/tensor_test.cpp:224-243", [L23, R23],
     f"0 input 0\n1 input 1\n2 add 0 1\n3 tensor 2\n4 scalar {hx(2)}\n5 multiply 3 4\n6 scalar {hx(1)}\n7 subtract 5 6\n",
     [21, 43, 65, 87])
case("scalar_elementwise_ops", "tests/tensor_test.cpp:342-353", [[[2, 2], [1, 2, 3, 4]]],
     f"0 input 0\n1 scalar {hx(10)}\n2 scalar {hx(2)}\n3 multiply 0 2\n4 subtract 1 3\n", [8, 6, 4, 2])
SV = [[[2, 3], [-2, -1, 0, 1, 2, 3]]]
case("scalar_order_left", "tests/tensor_test.cpp:355-366", SV,
     f"0 input 0\n1 scalar {hx(10)}\n2 scalar {hx(3)}\n3 multiply 0 2\n4 subtract 1 3\n",
     [16, 13, 10, 7, 4, 1])
case("scalar_order_right", "tests/tensor_test.cpp:367-371", SV,
     f"0 input 0\n1 scalar {hx(5)}\n2 add 0 1\n3 scalar {hx(2)}\n4 multiply 2 3\n",
     [6, 8, 10, 12, 14, 16])
MA = [[[2, 3], [1, 2, 3, 4, 5, 6]], [[3, 2], [7, 8, 9, 10, 11, 12]]]
case("matmul_uses_cuda_backend", "tests/tensor_test.cpp:374-393", MA,
     "0 input 0\n1 input 1\n2 matmul 0 1\n", [58, 64, 139, 154], shape=[2, 2])
case("matmul_rectangular_values_are_correct", "tests/tensor_test.cpp:395-414",
     [[[3, 2], [1, 2, -1, 3, 4, -2]], [[2, 4], [2, 0, -1, 5, 3, -2, 4, 1]]],
     "0 input 0\n1 input 1\n2 matmul 0 1\n", [8, -4, 7, 7, 7, -6, 13, -2, 2, 4, -12, 18], shape=[3, 4])
case("matmul_composes_with_elementwise_ir", "tests/tensor_test.cpp:434-448", MA,
     f"0 input 0\n1 input 1\n2 matmul 0 1\n3 scalar {hx(2)}\n4 multiply 2 3\n5 scalar {hx(1)}\n6 subtract 4 5\n",
     [115, 127, 277, 307])
case("matmul_accepts_expression_operands", "tests/tensor_test.cpp:450-464", MA,
     "0 input 0\n1 input 1\n2 add 0 0\n3 matmul 2 1\n", [116, 128, 278, 308])
case("matmul_rejects_invalid_shapes", "tests/tensor_test.cpp:466-479",
     [[[2, 3], [1, 2, 3, 4, 5, 6]], [[2, 2], [1, 2, 3, 4]]],
     "0 input 0\n1 input 1\n2 matmul 0 1\n", error="invalid_argument")
case("reshape_uses_lazy_device_ir", "tests/tensor_test.cpp:481-497", [S6],
     f"0 input 0\n1 scalar {hx(1)}\n2 add 0 1\n3 reshape 2 3,2\n", [2, 3, 4, 5, 6, 7], shape=[3, 2])
case("transpose_uses_lazy_device_ir", "tests/tensor_test.cpp:499-515", [S6],
     "0 input 0\n1 transpose 0\n", [1, 4, 2, 5, 3, 6], shape=[3, 2])
case("broadcast_to_uses_lazy_device_ir", "tests/tensor_test.cpp:517-526", [[[3], [1, 2, 3]]],
     f"0 input 0\n1 broadcast 0 2,3\n2 scalar {hx(2)}\n3 multiply 1 2\n", [2, 4, 6, 2, 4, 6])
case("concat_uses_lazy_device_ir", "tests/tensor_test.cpp:528-543",
     [[[2, 2], [1, 2, 3, 4]], [[2, 1], [10, 20]]], "0 input 0\n1 input 1\n2 concat 0 1 1\n",
     [1, 2, 10, 3, 4, 20], shape=[2, 3])
case("reductions_column_sums", "tests/tensor_test.cpp:545-555", [S6], "0 input 0\n1 sum 0 0 0\n",
     [5, 7, 9], shape=[3])
case("reductions_row_maxes", "tests/tensor_test.cpp:551-556", [S6], "0 input 0\n1 max 0 1 0\n",
     [3, 6], shape=[2])
case("keepdim_sums", "tests/tensor_test.cpp:559-572", [S6], "0 input 0\n1 sum 0 1 1\n", [6, 15],
     shape=[2, 1])
case("keepdim_maxes", "tests/tensor_test.cpp:565-580", [S6], "0 input 0\n1 max 0 0 1\n", [4, 5, 6],
     shape=[1, 3])
V513 = [float(i + 1) for i in range(513)]
V513m = list(V513)
V513m[400] = 1000.0
case("block_reduction_sum", "tests/tensor_test.cpp:583-596", [[[1, 513], V513m]],
     "0 input 0\n1 sum 0 1 0\n", [132440], shape=[1])
case("block_reduction_max", "tests/tensor_test.cpp:583-596", [[[1, 513], V513m]],
     "0 input 0\n1 max 0 1 0\n", [1000], shape=[1])
case("nested_reductions", "tests/tensor_test.cpp:598-608", [[[1, 513], V513]],
     f"0 input 0\n1 sum 0 1 0\n2 scalar {hx(2)}\n3 multiply 1 2\n4 scalar {hx(1)}\n5 add 3 4\n",
     [263683], shape=[1])
SM = [[[2, 2], [0, 0, 1, 1]]]
case("softmax_style_expression", "tests/tensor_test.cpp:610-623", SM,
     "0 input 0\n1 exp 0\n2 sum 1 1 1\n3 broadcast 2 2,2\n4 divide 1 3\n",
     interval=[[0.49, 0.51]] * 4)
case("relu_compound_op", "tests/tensor_test.cpp:625-634", [[[4], [-2, -0.5, 0, 3]]],
     "0 input 0\n1 relu 0\n", [0, 0, 0, 3])
case("softmax_compound_op", "tests/tensor_test.cpp:636-646", SM, "0 input 0\n1 softmax 0 1\n",
     interval=[[0.49, 0.51]] * 4)
case("logistic_compound_op", "tests/tensor_test.cpp:648-657", [[[3], [-1, 0, 1]]],
     "0 input 0\n1 logistic 0\n", interval=[[0.26, 0.27], [0.5, 0.5], [0.73, 0.74]],
     exact_at={"1": 0.5})
case("exp_uses_lazy_device_ir", "tests/tensor_test.cpp:659-668", [[[3], [-1, 0, 2]]],
     "0 input 0\n1 exp 0\n", interval=[[0.36, 0.37], [1, 1], [7.38, 7.39]], exact_at={"1": 1.0})
case("divide", "tests/tensor_test.cpp:670-680", [[[3], [2, 4, 8]], [[3], [1, 2, 4]]],
     "0 input 0\n1 input 1\n2 divide 0 1\n", [2, 2, 2])
case("reciprocal", "tests/tensor_test.cpp:675-682", [[[3], [2, 4, 8]]], "0 input 0\n1 reciprocal 0\n",
     [0.5, 0.25, 0.125])
MM = [[[4], [-1, 5, 3, 9]], [[4], [2, 4, 7, 1]]]
case("maximum", "tests/tensor_test.cpp:685-694", MM, "0 input 0\n1 input 1\n2 maximum 0 1\n",
     [2, 5, 7, 9])
case("minimum", "tests/tensor_test.cpp:690-697", MM, "0 input 0\n1 input 1\n2 minimum 0 1\n",
     [-1, 4, 3, 1])
case("unsqueeze_expression", "tests/tensor_test.cpp:700-741", [S6],
     f"0 input 0\n1 scalar {hx(1)}\n2 add 0 1\n3 unsqueeze 2 1\n", [2, 3, 4, 5, 6, 7], shape=[2, 1, 3])
case("unsqueeze_leading", "tests/tensor_test.cpp:706-725", [S6], "0 input 0\n1 unsqueeze 0 0\n",
     [1, 2, 3, 4, 5, 6], shape=[1, 2, 3])
case("unsqueeze_trailing", "tests/tensor_test.cpp:707-729", [S6], "0 input 0\n1 unsqueeze 0 2\n",
     [1, 2, 3, 4, 5, 6], shape=[2, 3, 1])

if __name__ == "__main__":
    out = Path(__file__).with_name("known_answers.json")
    out.write_text(json.dumps({"reference": "AkhilSamavedam/porch tests/tensor_test.cpp",
                               "cases": CASES}, indent=1))
    print(f"wrote {len(CASES)} cases to {out}")
