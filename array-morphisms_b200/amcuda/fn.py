"""Functions usable inside morph_map (traced into the element-wise program).

Each accepts a traced operand or a plain number (then computes directly),
mirroring the Scheme procedures a morph-map lambda may call
(get-unary-transformer, basic-ops.scm:258-284).
"""
from __future__ import annotations

import math

from . import _abi as A
from .morph import Sym


def _u(op: str, pyf):
    def f(x):
        if isinstance(x, Sym):
            return Sym(x.prog + [(A.OP[op], 0, 0.0)])
        return pyf(x)
    f.__name__ = op.lower()
    return f


def _relu(x):
    return max(0.0, float(x))


def _sigmoid(x):
    return 1.0 / (1.0 + math.exp(-float(x)))


def _tanh(x):
    e2 = math.exp(2.0 * float(x))
    return (e2 - 1.0) / (e2 + 1.0)


sqrt = _u("SQRT", math.sqrt)
exp = _u("EXP", math.exp)
log = _u("LOG", math.log)
sin = _u("SIN", math.sin)
cos = _u("COS", math.cos)
tan = _u("TAN", math.tan)
floor = _u("FLOOR", math.floor)
ceiling = _u("CEIL", math.ceil)
relu = _u("RELU", _relu)
sigmoid = _u("SIGMOID", _sigmoid)
tanh = _u("TANH", _tanh)


def maximum(a, b):
    if isinstance(a, Sym) or isinstance(b, Sym):
        return Sym._c(a)._b(b, "MAX")
    return max(a, b)


def minimum(a, b):
    if isinstance(a, Sym) or isinstance(b, Sym):
        return Sym._c(a)._b(b, "MIN")
    return min(a, b)


def eq(a, b):
    if isinstance(a, Sym) or isinstance(b, Sym):
        return Sym._c(a)._b(b, "EQ")
    return 1.0 if a == b else 0.0
