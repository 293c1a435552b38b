"""Builds morphism trees from the JSON expressions in tests/golden/."""
from __future__ import annotations

import amcuda as am

FUNCS = {
    "square": lambda a: a * a,
}

UNARY = {"sqrt": am.morph_sqrt, "exp": am.morph_exp, "log": am.morph_log, "sin": am.morph_sin, "cos": am.morph_cos,
         "tan": am.morph_tan, "negate": am.morph_negate, "abs": am.morph_abs, "floor": am.morph_floor,
         "ceiling": am.morph_ceiling, "relu": am.morph_relu, "sigmoid": am.morph_sigmoid, "tanh": am.morph_tanh}
BINARY = {"add": am.morph_add, "sub": am.morph_sub, "mul": am.morph_mul, "div": am.morph_div, "pow": am.morph_pow,
          "gt": am.morph_gt, "lt": am.morph_lt, "eq": am.morph_eq, "ge": am.morph_ge, "le": am.morph_le,
          "matmul": am.morph_matmul, "matvec": am.morph_matvec, "dot": am.morph_dot}


def build(e):
    op = e[0]
    if op == "in":
        return am.morph_from_list(e[1], e[2], e[3])
    if op in UNARY:
        return UNARY[op](build(e[1]))
    if op in BINARY:
        return BINARY[op](build(e[1]), build(e[2]))
    if op == "map":
        return am.morph_map(FUNCS[e[1]], build(e[2]))
    if op == "reduce":
        return am.morph_reduce(e[1], build(e[2]), e[3], e[4])
    if op == "reshape":
        return am.morph_reshape(build(e[1]), e[2])
    if op == "transpose":
        return am.morph_transpose(build(e[1]), e[2])
    if op == "slice":
        return am.morph_slice(build(e[1]), e[2], e[3], e[4])
    if op == "squeeze":
        return am.morph_squeeze(build(e[1]))
    if op == "unsqueeze":
        return am.morph_unsqueeze(build(e[1]), e[2])
    if op == "pad":
        return am.morph_pad(build(e[1]), e[2], e[3], e[4])
    if op == "im2col":
        return am.im2col_morph(build(e[1]), e[2], e[3], e[4])
    if op == "col2im":
        return am.col2im_morph(build(e[1]), e[2], e[3], e[4], e[5])
    if op == "stack":
        return am.morph_stack([build(x) for x in e[1]], e[2])
    if op == "concat":
        return am.morph_concat([build(x) for x in e[1]], e[2])
    if op == "split_stack":
        return am.morph_stack(am.morph_split(build(e[1]), e[2]))
    if op == "attention":
        return am.attention_morphism(build(e[1]), build(e[2]), build(e[3]), e[4])
    raise ValueError(op)
