"""Write tests/golden/known_answers.json.

The reference (CHICKEN Scheme) cannot run on this machine, so its pinned
numbers are transcribed here from its own test files: every case records the
reference test (file:line) whose inputs and expected values it restates.
Expressions use a small JSON form evaluated by tests/golden_dsl.py:
  ["in", values, shape, dtype]            morph-from-list
  [op, operand...]                        add sub mul div pow gt lt eq sqrt exp log negate abs ...
  ["map", fname, x]                       morph-map with a named function
  ["reduce", op, x, axes, keepdims]       morph-reduce
  ["reshape", x, shape] ["transpose", x, perm|null] ["slice", x, start, end, step|null]
  ["squeeze", x] ["unsqueeze", x, axis] ["pad", x, pads, mode, value]
  ["im2col", x, k, s, p] ["col2im", x, shape, k, s, p]
  ["stack", [xs], axis] ["concat", [xs], axis] ["split_stack", x, n]
  ["matmul", a, b] ["matvec", a, v] ["dot", a, b] ["attention", q, k, v, scale|null]
The attention cross-validation expectations are computed below by a
restatement of the tests' own list-based ref-attention
(tests/test-attention.scm:53-79) in double precision.

    python tests/golden/make_known_answers.py
"""
import json
import math
from pathlib import Path


def inp(values, shape, dtype="f64"):
    return ["in", values, list(shape), dtype]


def ref_attention(Q, K, V, n, dk, dv, scale):
    """tests/test-attention.scm:53-79: per row scores, max, exp, Z, weights, out."""
    out = []
    for i in range(n):
        qi = Q[i * dk:(i + 1) * dk]
        scores = [scale * sum(a * b for a, b in zip(qi, K[k * dk:(k + 1) * dk])) for k in range(n)]
        rmax = max(scores)
        exps = [math.exp(s - rmax) for s in scores]
        Z = sum(exps)
        w = [e / Z for e in exps]
        out.extend(sum(w[k] * V[k * dv + p] for k in range(n)) for p in range(dv))
    return out


R = "tests/test-realization.scm"
B = "tests/test-blas.scm"
AT = "tests/test-attention.scm"
C2 = "tests/test-col2im.scm"

cases = []


def case(name, src, expr, values=None, shape=None, dtype=None, tol=0.0):
    cases.append({"name": name, "source": src, "expr": expr, "values": values, "shape": shape, "dtype": dtype,
                  "tol": tol})


m23 = inp([1, 2, 3, 4, 5, 6], [6])
case("reshape preserves values", R + ":106-109", ["reshape", m23, [2, 3]], [[1, 2, 3], [4, 5, 6]])
case("reshape flatten", R + ":111-114", ["reshape", inp([[1, 2], [3, 4]], [2, 2]), [4]], [1, 2, 3, 4])
case("reshape with inference", R + ":116-119", ["reshape", m23, [2, -1]], [[1, 2, 3], [4, 5, 6]])
case("reshape 3D shape", R + ":121-126", ["reshape", inp([1.0] * 24, [24]), [2, 3, 4]], shape=[2, 3, 4])
case("2D transpose", R + ":134-137", ["transpose", inp([[1, 2, 3], [4, 5, 6]], [2, 3]), None], [[1, 4], [2, 5], [3, 6]])
case("custom permutation shape", R + ":145-151",
     ["transpose", inp([[[1, 2], [3, 4]], [[5, 6], [7, 8]]], [2, 2, 2]), [2, 1, 0]], shape=[2, 2, 2])
case("transpose identity permutation", R + ":153-156", ["transpose", inp([[1, 2], [3, 4]], [2, 2]), [0, 1]],
     [[1, 2], [3, 4]])
case("1D slice", R + ":164-167", ["slice", inp([0, 1, 2, 3, 4, 5], [6]), [1], [4], None], [1, 2, 3])
case("1D slice with step", R + ":169-172", ["slice", inp(list(range(10)), [10]), [0], [10], 2], [0, 2, 4, 6, 8])
case("2D slice rows and columns", R + ":174-177",
     ["slice", inp([[1, 2, 3], [4, 5, 6], [7, 8, 9]], [3, 3]), [0, 1], [2, 3], None], [[2, 3], [5, 6]])
case("2D slice single row", R + ":179-182", ["slice", inp([[1, 2, 3], [4, 5, 6]], [2, 3]), [1, 0], [2, 3], None],
     [[4, 5, 6]])
case("slice with negative indices", R + ":184-187", ["slice", inp([0, 1, 2, 3, 4], [5]), [-2], [-1], None], [3])
case("addition", R + ":195-199", ["add", inp([1, 2, 3], [3]), inp([4, 5, 6], [3])], [5, 7, 9])
case("subtraction", R + ":201-205", ["sub", inp([10, 20, 30], [3]), inp([1, 2, 3], [3])], [9, 18, 27])
case("multiplication", R + ":207-211", ["mul", inp([2, 3, 4], [3]), inp([5, 6, 7], [3])], [10, 18, 28])
case("division", R + ":213-217", ["div", inp([10.0, 20.0, 30.0], [3]), inp([2.0, 4.0, 5.0], [3])], [5.0, 5.0, 6.0])
case("power", R + ":219-223", ["pow", inp([2.0, 3.0, 4.0], [3]), inp([2.0, 2.0, 2.0], [3])], [4.0, 9.0, 16.0])
case("broadcasting", R + ":225-229", ["add", inp([[1, 2], [3, 4]], [2, 2]), inp([10], [1])], [[11, 12], [13, 14]])
case("sqrt", R + ":237-240", ["sqrt", inp([1.0, 4.0, 9.0, 16.0], [4])], [1.0, 2.0, 3.0, 4.0])
case("exp", R + ":242-245", ["exp", inp([0.0, 1.0], [2])], [1.0, math.exp(1.0)], tol=1e-12)
case("log", R + ":247-250", ["log", inp([1.0, 2.71828], [2])], [0.0, 1.0], tol=1e-4)
case("negate", R + ":252-255", ["negate", inp([1, -2, 3, -4], [4])], [-1, 2, -3, 4])
case("abs", R + ":257-260", ["abs", inp([-1, 2, -3, 4], [4])], [1, 2, 3, 4])
case("transcendental promotes integers", R + ":262-266", ["sqrt", inp([1, 4, 9], [3], "s32")], [1.0, 2.0, 3.0],
     dtype="f64")
case("greater-than", R + ":274-278", ["gt", inp([1, 2, 3], [3]), inp([2, 2, 2], [3])], [0.0, 0.0, 1.0])
case("less-than", R + ":280-284", ["lt", inp([1, 2, 3], [3]), inp([2, 2, 2], [3])], [1.0, 0.0, 0.0])
case("equality", R + ":286-290", ["eq", inp([1, 2, 3], [3]), inp([1, 2, 4], [3])], [1.0, 1.0, 0.0])
case("constant padding", R + ":298-301", ["pad", inp([1, 2, 3], [3]), [[2, 1]], "constant", 0.0],
     [0.0, 0.0, 1.0, 2.0, 3.0, 0.0])
case("edge padding", R + ":303-306", ["pad", inp([1, 2, 3], [3]), [[2, 1]], "edge", 0.0], [1.0, 1.0, 1.0, 2.0, 3.0, 3.0])
case("reflect padding", R + ":308-311", ["pad", inp([1, 2, 3], [3]), [[2, 2]], "reflect", 0.0],
     [2.0, 1.0, 1.0, 2.0, 3.0, 3.0, 2.0])
case("2D constant padding", R + ":313-320", ["pad", inp([[1, 2], [3, 4]], [2, 2]), [[1, 1], [1, 1]], "constant", 0.0],
     [[0, 0, 0, 0], [0, 1, 2, 0], [0, 3, 4, 0], [0, 0, 0, 0]])
case("sum all elements", R + ":328-331", ["reduce", "sum", inp([1, 2, 3, 4], [4]), [], False], 10.0)
case("sum along axis", R + ":333-336", ["reduce", "sum", inp([[1, 2, 3], [4, 5, 6]], [2, 3]), [0], False], [5.0, 7.0, 9.0])
case("sum keepdims", R + ":338-343", ["reduce", "sum", inp([[1, 2], [3, 4]], [2, 2]), [0], True], [[4.0, 6.0]])
case("mean", R + ":345-348", ["reduce", "mean", inp([1.0, 2.0, 3.0, 4.0], [4]), [], False], 2.5)
case("max", R + ":350-353", ["reduce", "max", inp([1, 5, 3, 2, 4], [5]), [], False], 5.0)
case("min along axis", R + ":355-358", ["reduce", "min", inp([[3, 1, 4], [1, 5, 9]], [2, 3]), [1], False], [1.0, 1.0])
case("product", R + ":360-363", ["reduce", "prod", inp([2, 3, 4], [3]), [], False], 24.0)
case("im2col basic shape", R + ":371-378", ["im2col", inp([[[1, 2, 3], [4, 5, 6], [7, 8, 9]]], [1, 3, 3]), [2, 2], 1, 0],
     shape=[4, 4])
case("im2col with padding shape", R + ":380-389", ["im2col", inp([[[1, 2], [3, 4]]], [1, 2, 2]), [3, 3], 1, 1],
     shape=[9, 4])
case("im2col batched shape", R + ":391-396", ["im2col", inp([1.0] * 72, [2, 2, 6, 3]), [2, 2], 1, 0], shape=[2, 8, 10])
case("squeeze", R + ":406-409", ["squeeze", inp([[[1, 2]]], [1, 1, 2])], [1, 2])
case("unsqueeze", R + ":411-416", ["unsqueeze", inp([1, 2, 3], [3]), 0], [[1, 2, 3]])
case("morph-map square", R + ":418-421", ["map", "square", inp([1, 2, 3, 4], [4])], [1, 4, 9, 16])
case("stack", R + ":429-434", ["stack", [inp([1, 2], [2]), inp([3, 4], [2]), inp([5, 6], [2])], 0], [[1, 2], [3, 4], [5, 6]])
case("concat", R + ":436-440", ["concat", [inp([1, 2], [2]), inp([3, 4, 5], [3])], 0], [1, 2, 3, 4, 5])
case("split then stack", R + ":442-446", ["split_stack", inp([1, 2, 3, 4, 5, 6], [6]), 3], [[1, 2], [3, 4], [5, 6]])
case("reshape then transpose", R + ":561-565", ["transpose", ["reshape", m23, [2, 3]], None], [[1, 4], [2, 5], [3, 6]])
case("arithmetic then reduction", R + ":567-572",
     ["reduce", "sum", ["mul", inp([[1, 2], [3, 4]], [2, 2]), inp([[2, 2], [2, 2]], [2, 2])], [], False], 20.0)
case("slice then arithmetic", R + ":574-578",
     ["mul", ["slice", inp([1, 2, 3, 4, 5], [5]), [1], [4], None], inp([2, 2, 2], [3])], [4, 6, 8])
case("complex pipeline", R + ":580-586",
     ["reduce", "sum", ["transpose", ["add", ["reshape", inp([1, 2, 3, 4], [4]), [2, 2]], inp([10], [1])], None], [0],
      False], [23.0, 27.0])
case("nested operations", R + ":588-593",
     ["reduce", "sum", ["mul", ["sqrt", inp([1, 2, 3, 4], [4])], inp([2], [1])], [], False], 12.2925, tol=1e-4)
case("multiple reshapes", R + ":595-603",
     ["reshape", ["reshape", ["reshape", inp([1.0] * 24, [24]), [2, 3, 4]], [6, 4]], [24]], [1.0] * 24)
case("empty reduction produces scalar", R + ":610-615", ["reduce", "sum", inp([42.0], [1]), [], False], 42.0, shape=[])
case("single element operations", R + ":617-620", ["sqrt", inp([5.0], [1])], [math.sqrt(5.0)], tol=1e-6)
case("different dtypes promote", R + ":622-627", ["add", inp([1, 2, 3], [3], "s32"), inp([1.5, 2.5, 3.5], [3])],
     [2.5, 4.5, 6.5], dtype="f64")

case("matmul", B + ":776-782", ["matmul", inp([[1, 2], [3, 4]], [2, 2]), inp([[5, 6], [7, 8]], [2, 2])],
     [[19, 22], [43, 50]])
case("matmul rectangular", B + ":784-788",
     ["matmul", inp([[1, 2, 3], [4, 5, 6]], [2, 3]), inp([[7, 8], [9, 10], [11, 12]], [3, 2])], [[58, 64], [139, 154]])
case("matvec", B + ":790-796", ["matvec", inp([[1, 2, 3], [4, 5, 6]], [2, 3]), inp([1, 2, 3], [3])], [14, 32])
case("dot", B + ":798-804", ["dot", inp([1, 2, 3], [3]), inp([4, 5, 6], [3])], 32, shape=[])
case("matmul of abstract operands", B + ":830-837",
     ["matmul", ["add", inp([[1, 0], [0, 1]], [2, 2]), inp([[0, 0], [0, 0]], [2, 2])],
      ["add", inp([[2, 3], [4, 5]], [2, 2]), inp([[0, 0], [0, 0]], [2, 2])]], [[2, 3], [4, 5]])
case("matmul f32", B + ":839-845", ["matmul", inp([[1, 2], [3, 4]], [2, 2], "f32"), inp([[5, 6], [7, 8]], [2, 2], "f32")],
     [[19, 22], [43, 50]], dtype="f32", tol=1e-4)
case("dot with stride-2 slice operand", B + ":463-470",
     ["dot", ["slice", inp(list(range(10)), [10]), [0], [10], 2], inp([1, 1, 1, 1, 1], [5])], 20, shape=[])
# the stride-aware kernels of test-blas.scm groups 4-6 and the strided GEMM
# group: transposed and sliced operands, identities, zeros, scalars
I2 = inp([[1, 0], [0, 1]], [2, 2])
I3 = inp([[1, 0, 0], [0, 1, 0], [0, 0, 1]], [3, 3])
src32 = inp([[1, 2], [3, 4], [5, 6]], [3, 2])
case("gemm identity", B + ":332-336", ["matmul", inp([[1, 2, 3], [4, 5, 6], [7, 8, 9]], [3, 3]), I3],
     [[1, 2, 3], [4, 5, 6], [7, 8, 9]])
case("gemm zero", B + ":338-342", ["matmul", inp([[1, 2], [3, 4]], [2, 2]), inp([[0, 0], [0, 0]], [2, 2])],
     [[0, 0], [0, 0]])
case("gemm (3,4)x(4,2) shape", B + ":351-355",
     ["matmul", inp(list(range(1, 13)), [3, 4]), inp(list(range(1, 9)), [4, 2])], shape=[3, 2])
case("gemm transposed operand", B + ":357-366", ["matmul", ["transpose", src32, None], I3], [[1, 3, 5], [2, 4, 6]])
case("gemm column-slice operand", B + ":368-377",
     ["matmul", ["slice", inp([[1, 2, 3, 4], [5, 6, 7, 8], [9, 10, 11, 12]], [3, 4]), [0, 1], [3, 4], None], I3],
     [[2, 3, 4], [6, 7, 8], [10, 11, 12]])
case("gemv identity", B + ":393-397", ["matvec", I3, inp([2, 5, 7], [3])], [2, 5, 7])
case("gemv zero", B + ":399-403", ["matvec", inp([[0, 0, 0], [0, 0, 0]], [2, 3]), inp([9, 9, 9], [3])], [0, 0])
case("gemv (1,N) row", B + ":405-411", ["matvec", inp([[1, 2, 3, 4]], [1, 4]), inp([1, 2, 3, 4], [4])], [30])
case("gemv transposed matrix", B + ":413-421", ["matvec", ["transpose", inp([[1, 2], [3, 4]], [2, 2]), None],
                                                 inp([1, 0], [2])], [1, 2])
case("dot orthogonal", B + ":438-442", ["dot", inp([1, 0, 0], [3]), inp([0, 1, 0], [3])], 0, shape=[])
case("dot squared norm", B + ":444-448", ["dot", inp([3, 4], [2]), inp([3, 4], [2])], 25, shape=[])
case("dot single element", B + ":450-454", ["dot", inp([3], [1]), inp([4], [1])], 12, shape=[])
case("dot f32", B + ":456-462", ["dot", inp([1, 2, 3], [3], "f32"), inp([4, 5, 6], [3], "f32")], 32, shape=[],
     dtype="f32", tol=1e-4)
case("strided gemm G x B^T", B + ":1066-1075",
     ["matmul", inp([[1, 2], [4, 5]], [2, 2]), ["transpose", inp([[1, 0], [0, 1], [1, 1]], [3, 2]), None]],
     [[1, 2, 3], [4, 5, 9]])
case("strided gemm A^T x G", B + ":1077-1087",
     ["matmul", ["transpose", src32, None], inp([[1, 0, 1], [0, 1, 0], [1, 1, 0]], [3, 3])], [[6, 8, 1], [8, 10, 2]])
conv_in = inp(list(range(1, 17)), [1, 4, 4])
w1 = inp([1.0] * 9, [1, 1, 3, 3])
case("conv2d non-batched values", B + ":914-921",
     ["reshape", ["matmul", ["reshape", w1, [1, 9]], ["im2col", conv_in, [3, 3], 1, 0]], [1, 2, 2]], [[[54, 63], [90, 99]]])
w2 = inp([1.0] * 9 + [2.0] * 9, [2, 1, 3, 3])
case("conv2d 2-channel values", B + ":951-960",
     ["reshape", ["matmul", ["reshape", w2, [2, 9]], ["im2col", conv_in, [3, 3], 1, 0]], [2, 2, 2]],
     [[[54, 63], [90, 99]], [[108, 126], [180, 198]]])
case("conv2d f32", B + ":971-982",
     ["reshape", ["matmul", ["reshape", inp([1.0] * 9, [1, 1, 3, 3], "f32"), [1, 9]],
                  ["im2col", inp(list(range(1, 17)), [1, 4, 4], "f32"), [3, 3], 1, 0]], [1, 2, 2]],
     [[[54, 63], [90, 99]]], dtype="f32", tol=1e-3)

img = inp([[[1, 2, 3, 4], [5, 6, 7, 8], [9, 10, 11, 12], [13, 14, 15, 16]]], [1, 4, 4])
case("col2im inverts im2col (stride = kernel)", C2 + ":49-63",
     ["col2im", ["im2col", img, [2, 2], 2, 0], [1, 4, 4], [2, 2], 2, 0],
     [[[1, 2, 3, 4], [5, 6, 7, 8], [9, 10, 11, 12], [13, 14, 15, 16]]], tol=1e-10)
case("col2im output shape", C2 + ":65-72", ["col2im", inp([1.0] * 36, [36, 1]), [4, 3, 3], [3, 3], 1, 0], shape=[4, 3, 3])
case("col2im single pixel windows", C2 + ":74-82",
     ["col2im", ["im2col", inp([[[1, 2], [3, 4]]], [1, 2, 2]), [1, 1], 1, 0], [1, 2, 2], [1, 1], 1, 0],
     [[[1, 2], [3, 4]]], tol=1e-10)

# attention (tests/test-attention.scm)
Q3 = [1.0, 2.0, 0.5, -1.0, -0.5, 1.0, 2.0, 0.0, 0.0, -1.0, 1.5, 2.0]
K3 = [1.0, 0.0, 1.0, 0.0, 0.0, 1.0, 0.0, 1.0, -1.0, 1.0, -1.0, 1.0]
V3 = [1.0, 0.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 0.0, 1.0, 0.0]
case("attention uniform inputs", AT + ":202-224",
     ["attention", inp([1.0] * 24, [4, 6]), inp([1.0] * 24, [4, 6]), inp([1.0] * 24, [4, 6]), None], [[1.0] * 6] * 4,
     tol=1e-12)
exp3 = ref_attention(Q3, K3, V3, 3, 4, 4, 1.0 / math.sqrt(4.0))
case("attention cross-validation n=3 dk=4", AT + ":239-252",
     ["attention", inp(Q3, [3, 4]), inp(K3, [3, 4]), inp(V3, [3, 4]), None], exp3, shape=[3, 4], tol=1e-10)
Qi = [1.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 1.0]
Vi = [1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0, 9.0]
case("attention identity Q/K", AT + ":254-266",
     ["attention", inp(Qi, [3, 3]), inp(Qi, [3, 3]), inp(Vi, [3, 3]), None],
     ref_attention(Qi, Qi, Vi, 3, 3, 3, 1.0 / math.sqrt(3.0)), shape=[3, 3], tol=1e-10)
case("attention batched rank 3", AT + ":290-315",
     ["attention", inp(Q3 + Q3, [2, 3, 4]), inp(K3 + K3, [2, 3, 4]), inp(V3 + V3, [2, 3, 4]), None], exp3 + exp3,
     shape=[2, 3, 4], tol=1e-10)

case("attention explicit scale 1/sqrt(dk)", AT + ":366-376",
     ["attention", inp(Q3, [3, 4]), inp(K3, [3, 4]), inp(V3, [3, 4]), 0.5], exp3, shape=[3, 4], tol=1e-10)
# matmul(A, transpose(B)) through the zero-copy view equals the explicit
# transpose: the product Q3 K3^T written out
QKt = [sum(Q3[i * 4 + j] * K3[k * 4 + j] for j in range(4)) for i in range(3) for k in range(3)]
case("matmul with a transposed view operand", AT + ":335-364",
     ["matmul", inp(Q3, [3, 4]), ["transpose", inp(K3, [3, 4]), [1, 0]]], QKt, shape=[3, 3], tol=1e-12)
Q8 = [0.5, -0.3, 1.2, 0.8, 0.1, 0.9, -0.4, 0.6, -0.7, 0.2, 0.5, -0.9, 1.1, -0.5, 0.3, 0.4,
      -0.2, 0.8, -0.6, 1.0, 0.6, 0.1, 0.9, -0.3, -0.8, 0.4, -0.1, 0.7, 0.3, -0.9, 0.6, 0.2]
K8 = [0.4, -0.1, 0.8, 0.3, 0.7, 0.5, -0.2, 0.9, -0.3, 1.0, 0.4, -0.6, 0.2, 0.6, 0.1, 0.5,
      -0.9, 0.3, 0.7, 0.1, 0.5, -0.7, 0.2, 0.8, 0.1, 0.4, -0.5, 0.6, -0.4, 0.8, 0.3, -0.2]
V8 = [0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9, 1.0, 0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8,
      0.9, 1.0, 0.1, 0.2, 0.3, 0.4, 0.5, 0.6, 0.7, 0.8, 0.9, 1.0, 0.1, 0.3, 0.5, 0.7, 0.9, 0.2,
      0.4, 0.6, 0.8, 1.0, 0.2, 0.4, 0.6, 0.8, 1.0, 0.2, 0.4, 0.6]
case("attention n=8 dk=4 dv=6 cross-validation", AT + ":381-427",
     ["attention", inp(Q8, [8, 4]), inp(K8, [8, 4]), inp(V8, [8, 6]), None],
     ref_attention(Q8, K8, V8, 8, 4, 6, 0.5), shape=[8, 6], tol=1e-10)

# tests/test-im2col.scm: buffer sizes and shapes, the one stated value set,
# and im2col of a stacked batch
IC = "tests/test-im2col.scm"
img33 = inp([[[1, 2, 3], [4, 5, 6], [7, 8, 9]]], [1, 3, 3])
case("im2col 3x3 k2 s1 shape", IC + ":42-53", ["im2col", img33, [2, 2], 1, 0], shape=[4, 4])
case("im2col 4x4 ones k2 s2", IC + ":55-65", ["im2col", inp([1.0] * 16, [1, 4, 4]), [2, 2], 2, 0], [[1.0] * 4] * 4,
     shape=[4, 4])
case("im2col 2x2 k2 s1 p1 shape", IC + ":67-79", ["im2col", inp([[[1, 2], [3, 4]]], [1, 2, 2]), [2, 2], 1, 1],
     shape=[4, 9])
case("im2col 2 channels ones", IC + ":81-94", ["im2col", inp([1.0] * 18, [2, 3, 3]), [2, 2], 1, 0], [[1.0] * 4] * 8,
     shape=[8, 4])
case("im2col batched shape (2,1,3,3)", IC + ":111-119", ["im2col", inp([1.0] * 18, [2, 1, 3, 3]), [2, 2], 1, 0],
     shape=[2, 4, 4])
case("im2col 5x5 k3 s2 shape", IC + ":121-130", ["im2col", inp([1.0] * 25, [1, 5, 5]), [3, 3], 2, 0], shape=[9, 4])
case("im2col 2x2 window values", IC + ":150-162", ["im2col", inp([[[1, 2], [3, 4]]], [1, 2, 2]), [2, 2], 1, 0],
     [[1], [2], [3], [4]], shape=[4, 1])
case("im2col of a stacked batch", IC + ":222-241",
     ["im2col", ["stack", [img33, inp([[[9, 8, 7], [6, 5, 4], [3, 2, 1]]], [1, 3, 3])], 0], [2, 2], 1, 0],
     shape=[2, 4, 4])

# test-realization.scm: the stack kernel groups and the integration and
# performance groups that state values or shapes
img_b = inp([[[9, 8, 7], [6, 5, 4], [3, 2, 1]]], [1, 3, 3])
case("stack two 1D arrays", R + ":460-468", ["stack", [inp([1, 2, 3], [3]), inp([4, 5, 6], [3])], 0],
     [[1, 2, 3], [4, 5, 6]], shape=[2, 3])
case("stack two 2D arrays", R + ":470-477", ["stack", [inp([[1, 2], [3, 4]], [2, 2]), inp([[5, 6], [7, 8]], [2, 2])], 0],
     [[[1, 2], [3, 4]], [[5, 6], [7, 8]]], shape=[2, 2, 2])
case("stack 3D images", R + ":489-496", ["stack", [img33, img_b], 0],
     [[[[1, 2, 3], [4, 5, 6], [7, 8, 9]]], [[[9, 8, 7], [6, 5, 4], [3, 2, 1]]]], shape=[2, 1, 3, 3])
case("col2im of im2col of a stacked batch", R + ":509-517",
     ["col2im", ["im2col", ["stack", [img33, img_b], 0], [2, 2], 1, 0], [2, 1, 3, 3], [2, 2], 1, 0], shape=[2, 1, 3, 3])
case("stacked matches direct batch", R + ":519-535",
     ["stack", [inp([[[1, 2], [3, 4]]], [1, 2, 2]), inp([[[5, 6], [7, 8]]], [1, 2, 2])], 0],
     [[[[1, 2], [3, 4]]], [[[5, 6], [7, 8]]]], shape=[2, 1, 2, 2])
case("stack single array", R + ":539-544", ["stack", [inp([1, 2, 3], [3])], 0], [[1, 2, 3]], shape=[1, 3])
case("stack promotes f32 and f64", R + ":546-554", ["stack", [inp([1, 2], [2], "f32"), inp([3, 4], [2])], 0],
     [[1, 2], [3, 4]], dtype="f64")
case("realize large array", R + ":641-646", ["mul", inp([1.0] * 10000, [10000]), inp([2.0], [1])], [2.0] * 10000)
deep = inp([1.0] * 100, [100])
for _ in range(10):
    deep = ["add", deep, inp([0.1], [1])]
acc = 1.0
for _ in range(10):
    acc = acc + 0.1
case("realize deep operation chain", R + ":648-655", deep, [acc] * 100)

# examples/example-08-polyphase-filter-bank.scm: the M=4 polyphase branches
# of x[n] = n as strided slices, a nested stride-2 decimation, and the 4-tap
# average of branch 0
E8 = "examples/example-08-polyphase-filter-bank.scm"
x16 = inp([float(v) for v in range(16)], [16])
for mm in range(4):
    case(f"polyphase branch {mm}", E8 + ":46-49", ["slice", x16, [mm], [16], 4], [float(mm + 4 * k) for k in range(4)])
case("polyphase nested decimation", E8 + ":54", ["slice", ["slice", x16, [0], [16], 4], [0], [4], 2], [0.0, 8.0])
case("polyphase 4-tap average", E8 + ":75-76",
     ["reduce", "sum", ["mul", ["slice", x16, [0], [16], 4], inp([0.25] * 4, [4])], [], False], 6.0, shape=[])

# examples/example-05-reshape-after-slice.scm: reshape of a stride-2 slice
# reads it in logical order; rows of the reshaped view are x[0], x[2] and
# x[4], x[6]
E5 = "examples/example-05-reshape-after-slice.scm"
x8 = inp([float(v) for v in range(8)], [8])
ds = ["slice", x8, [0], [8], 2]
case("reshape of a strided slice to (2,2)", E5 + ":34-38", ["reshape", ds, [2, 2]], [[0.0, 2.0], [4.0, 6.0]])
case("reshape of a strided slice to (1,4)", E5 + ":34-39", ["reshape", ds, [1, 4]], [[0.0, 2.0, 4.0, 6.0]])
case("row 0 of the reshaped slice", E5 + ":56-59", ["slice", ["reshape", ds, [2, 2]], [0, 0], [1, 2], None],
     [[0.0, 2.0]])
case("row 1 of the reshaped slice", E5 + ":57-61", ["slice", ["reshape", ds, [2, 2]], [1, 0], [2, 2], None],
     [[4.0, 6.0]])

# examples/example-04-cross-boundary-fusion.scm: 7 windows of 8 samples,
# hop 4, of x[n] = n by im2col, transposed and weighted by a rectangular window
E4 = "examples/example-04-cross-boundary-fusion.scm"
x32 = ["reshape", inp([float(v) for v in range(32)], [32]), [1, 1, 32]]
win = ["transpose", ["im2col", x32, [1, 8], [1, 4], 0], None]
case("windowed analysis window matrix", E4 + ":40-51", win, [[float(4 * k + j) for j in range(8)] for k in range(7)],
     shape=[7, 8])
case("windowed analysis rectangular window", E4 + ":64-82", ["mul", win, inp([1.0] * 8, [1, 8])],
     [[float(4 * k + j) for j in range(8)] for k in range(7)], shape=[7, 8])

# tests/test-col2im.scm groups 2-6: col2im(im2col(x)) scales each pixel by
# the number of windows covering it (corners once, edges twice, the centre
# of a 3x3 image four times with a 2x2 kernel, stride 1), the pattern the
# tests state; shapes where they state only shapes
cover33 = [[1, 2, 1], [2, 4, 2], [1, 2, 1]]
imgA = [[1, 2, 3], [4, 5, 6], [7, 8, 9]]
imgB = [[9, 8, 7], [6, 5, 4], [3, 2, 1]]
times = lambda im: [[im[i][j] * cover33[i][j] for j in range(3)] for i in range(3)]
case("col2im accumulates overlapping windows", C2 + ":90-112",
     ["col2im", ["im2col", img33, [2, 2], 1, 0], [1, 3, 3], [2, 2], 1, 0], [times(imgA)], shape=[1, 3, 3])
case("col2im single window of ones", C2 + ":114-129",
     ["col2im", ["im2col", inp([[[1, 1], [1, 1]]], [1, 2, 2]), [2, 2], 1, 0], [1, 2, 2], [2, 2], 1, 0],
     [[[1, 1], [1, 1]]])
case("col2im with padding shape", C2 + ":134-146",
     ["col2im", ["im2col", inp([[[1, 2], [3, 4]]], [1, 2, 2]), [2, 2], 1, 1], [1, 2, 2], [2, 2], 1, 1],
     shape=[1, 2, 2])
case("col2im batched matches per-image", C2 + ":211-244",
     ["col2im", ["im2col", ["stack", [img33, img_b], 0], [2, 2], 1, 0], [2, 1, 3, 3], [2, 2], 1, 0],
     [[times(imgA)], [times(imgB)]], shape=[2, 1, 3, 3])
case("col2im batched shape", C2 + ":198-209",
     ["col2im", ["im2col", inp([1.0] * 72, [2, 2, 6, 3]), [2, 2], 1, 0], [2, 2, 6, 3], [2, 2], 1, 0],
     shape=[2, 2, 6, 3])
case("col2im adjoint of ones", C2 + ":251-270", ["col2im", inp([1.0] * 32, [8, 4]), [2, 3, 3], [2, 2], 1, 0],
     [cover33, cover33], shape=[2, 3, 3])
case("col2im gradient of twos", C2 + ":272-290", ["col2im", inp([2.0] * 16, [4, 4]), [1, 3, 3], [2, 2], 1, 0],
     [[[2 * c for c in row] for row in cover33]], shape=[1, 3, 3])
case("col2im large kernel", C2 + ":305-314",
     ["col2im", ["im2col", inp([1.0] * 25, [1, 5, 5]), [5, 5], 1, 0], [1, 5, 5], [5, 5], 1, 0], [[[1.0] * 5] * 5])
case("col2im asymmetric kernel and stride shape", C2 + ":316-324",
     ["col2im", ["im2col", inp([1.0] * 12, [1, 3, 4]), [2, 3], [1, 2], 0], [1, 3, 4], [2, 3], [1, 2], 0],
     shape=[1, 3, 4])

out = Path(__file__).resolve().parent / "known_answers.json"
out.write_text(json.dumps({"generator": "tests/golden/make_known_answers.py", "cases": cases}, indent=1))
print(f"wrote {len(cases)} cases to {out}")
