"""The five realize workloads: seeded synthetic inputs, their morphism trees,
and direct device entry points on torch CUDA tensors.

Inputs come from SplitMix64 (Steele, Lea, Flood 2014), counter-based so the
host (numpy) and device (torch) generators produce identical bits:
  z = seed + (i + 1) * 0x9E3779B97F4A7C15
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9
  z = (z ^ (z >> 27)) * 0x94D049BB133111EB
  z =  z ^ (z >> 31)
uniform u = (z >> 11) * 2^-53; normals by Box-Muller on consecutive pairs
(u1, u2): sqrt(-2 ln(1 - u1)) cos(2 pi u2).  Seed of workload k, tensor j:
0xA11CE000 + k + (j << 32).
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

from . import _abi as A
from .morph import (im2col_morph, morph_add, morph_from_numpy, morph_map, morph_mul, morph_reduce, morph_reshape,
                    morph_slice, morph_transpose)

GOLD = 0x9E3779B97F4A7C15
M1 = 0xBF58476D1CE4E5B9
M2 = 0x94D049BB133111EB


def seed_of(workload: int, tensor: int) -> int:
    return (0xA11CE000 + workload + (tensor << 32)) & 0xFFFFFFFFFFFFFFFF


# ---------------------------------------------------------------------------- generators (host)
def splitmix_u64(seed: int, start: int, n: int) -> np.ndarray:
    i = np.arange(start + 1, start + n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + i * np.uint64(GOLD)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(M1)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(M2)
        z = z ^ (z >> np.uint64(31))
    return z


def uniform(seed: int, n: int, lo: float = 0.0, hi: float = 1.0, start: int = 0) -> np.ndarray:
    u = (splitmix_u64(seed, start, n) >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)
    return lo + (hi - lo) * u


def normal(seed: int, n: int, start: int = 0) -> np.ndarray:
    u = (splitmix_u64(seed, 2 * start, 2 * n) >> np.uint64(11)).astype(np.float64) * (2.0 ** -53)
    u1, u2 = u[0::2], u[1::2]
    return np.sqrt(-2.0 * np.log1p(-u1)) * np.cos(2.0 * math.pi * u2)


def randint(seed: int, n: int, lo: int, hi: int) -> np.ndarray:
    """Integers uniform on [lo, hi] (inclusive) by multiply-shift of the top 32 bits."""
    z = splitmix_u64(seed, 0, n) >> np.uint64(32)
    span = np.uint64(hi - lo + 1)
    return (lo + ((z * span) >> np.uint64(32)).astype(np.int64)).astype(np.int64)


# ---------------------------------------------------------------------------- generators (device)
def _torch_splitmix(seed: int, start: int, n: int, device):
    import torch
    i = torch.arange(start + 1, start + n + 1, dtype=torch.int64, device=device)

    def srl(z, k):  # logical shift right on int64 bit patterns
        return (z >> k) & ((1 << (64 - k)) - 1)

    def s64(v):
        return v - (1 << 64) if v >= (1 << 63) else v

    z = i * s64(GOLD) + s64(seed)
    z = (z ^ srl(z, 30)) * s64(M1)
    z = (z ^ srl(z, 27)) * s64(M2)
    z = z ^ srl(z, 31)
    return z


def normal_torch(seed: int, n: int, device="cuda", chunk: int = 1 << 26, start: int = 0):
    """Same bits as normal(seed, n, start); generated on the device in chunks."""
    import torch
    out = torch.empty(n, dtype=torch.float64, device=device)
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        z = _torch_splitmix(seed, 2 * (start + s), 2 * m, device)
        u = (((z >> 11) & ((1 << 53) - 1)).to(torch.float64)) * (2.0 ** -53)
        u1, u2 = u[0::2], u[1::2]
        out[s:s + m] = torch.sqrt(-2.0 * torch.log1p(-u1)) * torch.cos(2.0 * math.pi * u2)
    return out


def uniform_torch(seed: int, n: int, lo=0.0, hi=1.0, device="cuda", chunk: int = 1 << 26):
    import torch
    out = torch.empty(n, dtype=torch.float64, device=device)
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        z = _torch_splitmix(seed, s, m, device)
        u = (((z >> 11) & ((1 << 53) - 1)).to(torch.float64)) * (2.0 ** -53)
        out[s:s + m] = lo + (hi - lo) * u
    return out


# ---------------------------------------------------------------------------- C1: fused view + map + reduce
def c1_inputs(dtype: str = "f64", n: int = 1 << 20):
    if dtype == "s32":
        x = randint(seed_of(1, 0), n, -1000, 1000).astype(np.int32)
        y = randint(seed_of(1, 1), n, -1000, 1000).astype(np.int32)
    else:
        x = uniform(seed_of(1, 0), n, -1.0, 1.0)
        y = uniform(seed_of(1, 1), n, -1.0, 1.0)
    return x, y


def c1_tree(xm, ym, side: int = 1024):
    """r = morph-reduce 'sum (morph+ (morph-map sq xs) ys) '(1), with
    xs = slice(transpose(reshape(x, side x side), (1 0)), (0 0), (side side), (1 2))."""
    def view(m):
        return morph_slice(morph_transpose(morph_reshape(m, (side, side)), (1, 0)), (0, 0), (side, side), (1, 2))
    xs, ys = view(xm), view(ym)
    return morph_reduce("sum", morph_add(morph_map(lambda a: a * a, xs), ys), (1,))


# ---------------------------------------------------------------------------- C2: polyphase filter bank
BRANCHES, TAPS = 64, 16
PROTO = BRANCHES * TAPS


def c2_prototype() -> np.ndarray:
    """1024-tap Hamming-windowed sinc, cutoff 1/64, computed in f64, cast to f32."""
    n = np.arange(PROTO, dtype=np.float64)
    fc = 1.0 / BRANCHES
    w = 0.54 - 0.46 * np.cos(2.0 * np.pi * n / (PROTO - 1))
    h = w * 2.0 * fc * np.sinc(2.0 * fc * (n - (PROTO - 1) / 2.0))
    return h.astype(np.float32)


def c2_signal(sig: int, length: int) -> np.ndarray:
    """N(0,1) noise + 4 unit sinusoids at seeded normalised frequencies in (0, 0.5)."""
    x = normal(seed_of(2, 2 * sig + 16), length)
    p = uniform(seed_of(2, 2 * sig + 17), 8)
    t = np.arange(length, dtype=np.float64)
    for q in range(4):
        f, ph = 0.5 * p[2 * q], 2.0 * np.pi * p[2 * q + 1]
        x = x + np.sin(2.0 * np.pi * f * t + ph)
    return x.astype(np.float32)


def c2_signals_torch(batch: int, length: int, device="cuda", first: int = 0):
    """The same signals generated on the device (f32, (batch, length))."""
    import torch
    out = torch.empty((batch, length), dtype=torch.float32, device=device)
    t = torch.arange(length, dtype=torch.float64, device=device)
    for b in range(batch):
        s = first + b
        x = normal_torch(seed_of(2, 2 * s + 16), length, device)
        p = uniform(seed_of(2, 2 * s + 17), 8)
        for q in range(4):
            f, ph = 0.5 * p[2 * q], 2.0 * np.pi * p[2 * q + 1]
            x = x + torch.sin(2.0 * np.pi * f * t + ph)
        out[b] = x.to(torch.float32)
    return out


def c2_frames(length: int) -> int:
    return 1 + (length - PROTO) // BRANCHES


def c2_tree(xm, hm):
    """The filter-bank morphism tree: im2col of (B,1,1,L) with kernel (1,1024),
    stride (1,64) -> (B,1024,F); reshape (B,16,64,F); transpose (0 3 1 2)
    -> (B,F,16,64); times h (16,64); sum over taps -> (B,F,64)."""
    B, L = xm.shape[0], xm.shape[-1]
    F = c2_frames(L)
    x4 = morph_reshape(xm, (B, 1, 1, L))
    col = im2col_morph(x4, (1, PROTO), (1, BRANCHES), 0)
    win = morph_transpose(morph_reshape(col, (B, TAPS, BRANCHES, F)), (0, 3, 1, 2))
    h2 = morph_reshape(hm, (TAPS, BRANCHES))
    return morph_reduce("sum", morph_mul(win, h2), (2,))


# ---------------------------------------------------------------------------- C5: linear regression
def c5_inputs(n: int, d: int = 256):
    X = normal(seed_of(5, 0), n * d).reshape(n, d)
    wt = normal(seed_of(5, 1), d)
    y = X @ wt + 0.01 * normal(seed_of(5, 2), n)
    return X, y, wt


def c5_inputs_torch(n: int, d: int = 256, device="cuda"):
    import torch
    X = normal_torch(seed_of(5, 0), n * d, device).view(n, d)
    wt = torch.from_numpy(normal(seed_of(5, 1), d)).to(device)
    y = X @ wt + 0.01 * normal_torch(seed_of(5, 2), n, device)
    return X, y, wt


def c5_shard_torch(n: int, d: int = 256, shard: int = 0, device="cuda"):
    """Rows [shard*n, (shard+1)*n) of the config-5 data on the device: X
    (n, d) and y (n, 1), y = X w_true + 0.01 noise with the shared w_true."""
    import torch
    X = normal_torch(seed_of(5, 0), n * d, device, start=shard * n * d).view(n, d)
    wt = torch.from_numpy(normal(seed_of(5, 1), d)).to(device)
    y = X @ wt + 0.01 * normal_torch(seed_of(5, 2), n, device, start=shard * n)
    return X, y.view(n, 1)


# ---------------------------------------------------------------------------- device entry points (torch tensors)
def _ptr(t) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


def _stream(stream=None) -> C.c_void_p:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _dev(t):
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError("expected a contiguous CUDA tensor")
    return t


def window_fir(x, h, out, hop: int = BRANCHES, taps: int = TAPS, branches: int = BRANCHES, stream=None):
    """out[b, f, m] = sum_t h[t*M + m] * x[b, f*hop + t*M + m] (f32, ordered)."""
    _dev(x), _dev(h), _dev(out)
    B, L = x.shape
    F = out.shape[1]
    A.call("amc_window_fir_f32", _ptr(x), B, L, F, hop, taps, branches, _ptr(h), _ptr(out), _stream(stream))


def linreg_partials_count(rows: int, d: int) -> int:
    n = C.c_int32()
    A.call("amc_linreg_partials_count", rows, d, C.byref(n))
    return n.value


def linreg_partials(X, y, w, partials, n_total: int, stream=None):
    A.call("amc_linreg_partials", _ptr(_dev(X)), _ptr(_dev(y)), _ptr(_dev(w)), X.shape[0], X.shape[1], n_total,
           _ptr(_dev(partials)), _stream(stream))


def linreg_reduce(partials, n_partials: int, d: int, grad_loss, stream=None):
    A.call("amc_linreg_reduce", _ptr(partials), n_partials, d, _ptr(grad_loss), _stream(stream))


def linreg_update(w, grad_loss, n_total: int, lr: float, loss_out=None, stream=None):
    A.call("amc_linreg_update", _ptr(w), _ptr(grad_loss), w.shape[0], n_total, lr,
           _ptr(loss_out) if loss_out is not None else C.c_void_p(0), _stream(stream))


def attention_fwd(q, k, v, o, lse, scale: float, stream=None):
    *lead, n, dk = q.shape
    blocks = int(np.prod(lead)) if lead else 1
    A.call("amc_attention_fwd_f32", _ptr(_dev(q)), _ptr(_dev(k)), _ptr(_dev(v)), _ptr(_dev(o)), _ptr(_dev(lse)),
           blocks, n, dk, v.shape[-1], scale, _stream(stream))


def attention_bwd(q, k, v, o, do, lse, dq, dk_, dv, scale: float, stream=None):
    *lead, n, dk = q.shape
    blocks = int(np.prod(lead)) if lead else 1
    A.call("amc_attention_bwd_f32", _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(do), _ptr(lse), _ptr(dq), _ptr(dk_),
           _ptr(dv), blocks, n, dk, v.shape[-1], scale, _stream(stream))


def conv2d_fwd(x, w, y, stride: int = 1, pad: int = 1, stream=None):
    N, Cc, H, W = x.shape
    K, _, KH, KW = w.shape
    A.call("amc_conv2d_fwd_f32", _ptr(_dev(x)), _ptr(_dev(w)), _ptr(_dev(y)), N, Cc, H, W, K, KH, KW, stride, stride,
           pad, pad, _stream(stream))


def conv2d_dgrad(dy, w, dx, stride: int = 1, pad: int = 1, stream=None):
    N, Cc, H, W = dx.shape
    K, _, KH, KW = w.shape
    A.call("amc_conv2d_dgrad_f32", _ptr(_dev(dy)), _ptr(_dev(w)), _ptr(_dev(dx)), N, Cc, H, W, K, KH, KW, stride,
           stride, pad, pad, _stream(stream))


def conv2d_wgrad(x, dy, dw, stride: int = 1, pad: int = 1, stream=None):
    N, Cc, H, W = x.shape
    K, _, KH, KW = dw.shape
    A.call("amc_conv2d_wgrad_f32", _ptr(_dev(x)), _ptr(_dev(dy)), _ptr(_dev(dw)), N, Cc, H, W, K, KH, KW, stride,
           stride, pad, pad, _stream(stream))


def c1_inputs_morph(dtype="f64", n=1 << 20):
    x, y = c1_inputs(dtype, n)
    return morph_from_numpy(x, dtype), morph_from_numpy(y, dtype)


def tc_peak_tf32(iters: int = 4000, n: int = 256, warps: int = 1, a_tmem: bool = False, stream=None) -> float:
    """TFLOP/s reached by back-to-back tcgen05 kind::tf32 products of M=128,
    N=n from `warps` issuing threads per SM (amc_tc_peak_tf32), with A read
    from shared memory or, if `a_tmem`, from tensor memory.  The default
    shape gives the dense TF32 peak, the roofline denominator of the
    tensor-core kernels."""
    out = C.c_double(0.0)
    A.call("amc_tc_peak_tf32", n, warps, int(bool(a_tmem)), iters, C.byref(out), _stream(stream))
    return out.value


# ---------------------------------------------------------------------------- C5 through the public SSA path
class LinregSSA:
    """Config 5 as a user writes it: the MSE loss of a linear model built
    from variables (grad.scm's var-* constructors), compiled to a joint
    forward + reverse-mode SSA program (morphism-to-ssa, ssa-vjp) and run by
    ssa-realize/ctx with buffer reuse: one traced step, finalize, then each
    step replays the compiled plan in the context's arena and updates the
    parameter in place, w <- w - lr * dw (the plain gradient step of
    example-09, realized as a morphism over the gradient's arena buffer).

    X (rows, d) and y (rows, 1) are concrete arrays (host or device
    resident); w0 is (d,).  On the device the planner runs the program's
    forward GEMV and gradient GEMV as one pass over X (the GEMV pair of the
    row-pass kernels).  `grad_hook(dw_concrete)` runs between the replay and
    the update (a multi-GPU caller sums the gradient over the row shards
    there).  At most `max_steps` steps are recorded."""

    def __init__(self, X, y, w0, lr: float, stream=None, max_steps: int = 4096, grad_hook=None):
        from .grad import make_var, var_matmul, var_mean, var_mul, var_sub
        from .morph import Concrete, morph_from_numpy
        from .ssa import morphism_to_ssa, ssa_constant_id, ssa_loss_binding_val, ssa_vjp
        self.X = X if isinstance(X, Concrete) else morph_from_numpy(np.asarray(X, dtype=np.float64))
        rows, d = self.X.shape
        self.y = y if isinstance(y, Concrete) else morph_from_numpy(np.asarray(y, dtype=np.float64).reshape(rows, 1))
        self.rows, self.d, self.lr = rows, d, float(lr)
        self.w = morph_from_numpy(np.asarray(w0, dtype=np.float64).reshape(d, 1))
        wv = make_var(self.w, True)
        r = var_sub(var_matmul(make_var(self.X), wv), make_var(self.y))
        fwd = morphism_to_ssa(var_mean(var_mul(r, r)))
        self.prog = ssa_vjp(fwd, [ssa_constant_id(fwd, self.w)], ssa_loss_binding_val(fwd))
        self.ctx = None
        self.stream = stream
        self.max_steps = max_steps
        self.grad_hook = grad_hook
        self.steps = 0
        self._update = None
        self._losses = None
        self.trace_stats = None

    def _apply(self, dw, loss) -> None:
        """w <- w - lr * dw on the device, into w's own buffer, and the
        step's loss copied into the device-side loss record."""
        from .morph import morph_from_numpy, morph_mul, morph_sub
        from .realize import Plan, device_buffer_of
        if self.steps >= self.max_steps:
            raise ValueError(f"LinregSSA: more than max_steps={self.max_steps} steps")
        if self.grad_hook is not None:
            self.grad_hook(dw)
        wbuf = device_buffer_of(self.w)
        if self._update is None:
            # planned once over the arena buffer of dw, which every replay rewrites
            self._update = Plan(morph_sub(self.w, morph_mul(morph_from_numpy(np.array([self.lr])), dw)))
            self._update_out = self._update.result()._dev
        self._update.execute(self.stream)
        st = C.c_void_p(self.stream or 0)     # the replay's stream (0: the library's stream)
        A.call("amc_buf_copy_async", wbuf.handle, 0, self._update_out.handle, 0, 8 * self.d, st)
        A.call("amc_buf_copy_async", self._losses.handle, 8 * self.steps, loss._dev.handle, 8 * loss.offset, 8, st)
        self.w._data = None        # the host copy is stale; .data downloads the device value
        self.steps += 1

    def trace(self) -> None:
        """The first step: ssa-realize/ctx in trace mode (allocations
        recorded, outputs pinned), the update, then finalize-context!."""
        from .context import context_stats, finalize_context, make_morphism_context
        from .realize import DeviceBuffer, device_buffer_of
        from .ssa import ssa_realize_ctx
        self.ctx = make_morphism_context()
        loss, dw = ssa_realize_ctx(self.ctx, self.prog)
        if self.grad_hook is not None:
            self.grad_hook(dw)
        w_new = np.ascontiguousarray(self.w.values().reshape(-1) - self.lr * np.asarray(dw.values()).reshape(-1))
        wbuf = device_buffer_of(self.w)
        A.call("amc_buf_upload", wbuf.handle, w_new.ctypes.data_as(C.c_void_p), w_new.nbytes, 0)
        self.w._data = None
        self._losses = DeviceBuffer.create("f64", self.max_steps)
        l0 = np.asarray(loss.values(), dtype=np.float64).reshape(-1)[:1].copy()
        A.call("amc_buf_upload", self._losses.handle, l0.ctypes.data_as(C.c_void_p), 8, 0)
        self.trace_stats = context_stats(self.ctx)
        finalize_context(self.ctx)
        self.steps = 1

    def step(self) -> None:
        """One replayed step: reset-context!, the compiled SSA plan, the
        in-place update.  Allocates nothing after the first replay."""
        from .context import reset_context
        from .ssa import ssa_realize_ctx
        reset_context(self.ctx)
        loss, dw = ssa_realize_ctx(self.ctx, self.prog, stream=self.stream)
        self._apply(dw, loss)

    def replay_launches(self) -> int:
        """Kernel launches of one replayed step: the compiled SSA plan and the
        update (the copies are not kernels)."""
        plan = self.prog.__dict__.get("_replay", {}).get(self.ctx.handle, (None,))[0]
        n = plan.stats()["launches"] if plan is not None else 0
        return n + (self._update.stats()["launches"] if self._update is not None else 0)

    def losses(self) -> np.ndarray:
        """The loss of every step so far (the traced step first)."""
        return self._losses.download()[: self.steps].copy() if self._losses is not None else np.zeros(0)

    def weights(self) -> np.ndarray:
        return np.asarray(self.w.values()).reshape(-1)
