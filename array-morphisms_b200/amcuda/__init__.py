"""amcuda — B200 (sm_100a) realization backend for array-morphisms.

The lazy-morphism API of the reference (constructors in amcuda.morph,
realize / realize_ctx) over libamcuda.so, the C-ABI library of hand-written
sm_100a kernels.  The library is loaded by the first call that needs the
device (init, realize, a buffer or a workload entry point) and that call
fails loudly when the library is missing; there is no CPU fallback.
Building morphism trees needs no library, so host-only users (the oracle,
the reference arm of the benchmark) never map it.
"""
from . import _abi
from ._abi import AmcError

from .morph import (Concrete, Expr, Morphism, attention_morphism, broadcast_shapes, col2im_morph,  # noqa: E402
                    compute_strides, im2col_morph, infer_reduction_dtype, morph_abs, morph_add, morph_ceiling,
                    morph_concat, morph_cos, morph_div, morph_dot, morph_eq, morph_exp, morph_floor, morph_from_list,
                    morph_from_numpy, morph_ge, morph_gt, morph_le, morph_log, morph_lt, morph_map, morph_matmul,
                    morph_matvec, morph_mul, morph_negate, morph_pad, morph_pow, morph_reduce, morph_relu,
                    morph_reshape, morph_sigmoid, morph_sin, morph_slice, morph_split, morph_sqrt, morph_squeeze,
                    morph_stack, morph_sub, morph_tan, morph_tanh, morph_transpose, morph_unsqueeze, morph_unstack,
                    promote_types)
from .batch import (add_batch_dimension, batch_fold, batch_map, batch_reduce, batch_scan, batch_size,  # noqa: E402
                    batch_zip, batched, broadcast_to_batch, concat_batch, extract_batch_element,
                    make_batch_aware_binop, morph_add_batch, morph_batch_matmul, morph_div_batch, morph_mul_batch,
                    morph_sub_batch, remove_batch_dimension, stack_into_batch)
from .grad import (Var, accumulate_grad, backward, make_var, topo_sort, var_abs, var_add, var_cos,  # noqa: E402
                   var_div, var_exp, var_grad, var_grad_fn, var_log, var_matmul, var_mean, var_mul, var_name,
                   var_negate, var_parents, var_pow, var_relu, var_requires_grad, var_reshape, var_sigmoid,
                   var_sin, var_sqrt, var_sub, var_sum, var_tanh, var_transpose, var_value, zero_grad)
from .ssa import (morphism_to_ssa, ssa_constant_id, ssa_element_wise_fusion_pass, ssa_loss_binding_val,  # noqa: E402
                  ssa_realize, ssa_realize_ctx, ssa_vjp)
from .realize import DeviceBuffer, Plan, force_morphism, init, morph_to_list, realize, to_numpy  # noqa: E402
from .context import (MorphismContext, context_stats, finalize_context, make_morphism_context, plan_ctx,  # noqa: E402
                      realize_ctx, reset_context)
from . import fn  # noqa: E402

__all__ = [n for n in dir() if not n.startswith("_")]
