"""Bias-free linear layer in the compute dtype with fp32 master weights.

``y = x @ W^T`` runs in bf16 on CUDA (fp32 accumulation); the weight gradient
is produced directly in fp32 (``dW = dy^T x``) so fp32 master parameters need
no extra cast pass.  When the weight's ``.grad`` is a managed fp32 buffer, ``dW`` is accumulated
into it inside the GEMM.  The bf16 copy of each weight is cached and refreshed
only when the parameter's version counter changes (i.e. after an optimizer
step), so each weight is cast once per step, not once per micro-batch.
On CPU the layer computes in fp32 (reference path for tests).
"""
from __future__ import annotations

import torch

from . import gemm
from ..parallel import param_ready as _ready

# Parameters carrying this attribute (set by the data-parallel gradient
# synchroniser, whose ``zero_grad`` zeroes their ``.grad`` buffers every step)
# receive weight gradients by in-GEMM accumulation into ``.grad`` instead of
# through autograd.  ``torch.autograd.grad`` therefore sees no gradient for them.
ACCUMULATE_ATTR = "_ro_accumulate_grad"
# Optional callable on such parameters, invoked once the in-GEMM accumulation
# for the current backward pass has been issued (gradient bucketing).
READY_ATTR = "_ro_grad_ready"
# Optional callable ``route(gy2, x2) -> bool`` on such parameters: when it
# returns True it has computed dW = gy^T x itself and delivered it elsewhere
# (the reduce-to-owner transport: the GEMM stores its tiles straight into the
# layer owner's receive slot over NVLink), so nothing is added locally.
ROUTE_ATTR = "_ro_grad_route"


def managed_grad(param):
    """The parameter's fp32 ``.grad`` buffer when kernels may add into it directly, else None."""
    buf = param.grad
    if (getattr(param, ACCUMULATE_ATTR, False) and buf is not None and buf.is_cuda
            and buf.dtype == torch.float32 and buf.is_contiguous()):
        return buf
    return None


def report_ready(param):
    """Tell the gradient synchroniser that ``param``'s gradient for this backward is final."""
    ready = getattr(param, READY_ATTR, None)
    if ready is not None:
        ready(param)


def accumulate_weight_grad(weight, buf, gy2, x2):
    """dW = gy^T x into the managed buffer ``buf`` (or routed, see ROUTE_ATTR); reports ready."""
    route = getattr(weight, ROUTE_ATTR, None)
    if route is None or not route(gy2, x2):
        gemm.matmul_tn_accumulate_(buf, gy2, x2)
    report_ready(weight)


def weight_grad(weight, gy2, x2, needed):
    """dW = gy^T x: added inside the GEMM into a managed ``.grad`` (reported ready, returns
    None), else returned for autograd to accumulate."""
    if not needed:
        return None
    buf = managed_grad(weight)
    if buf is not None:
        accumulate_weight_grad(weight, buf, gy2, x2)
        return None
    return gemm.matmul_tn(gy2, x2, out_dtype=weight.dtype)


class _WeightCache:
    __slots__ = ("version", "tensor", "data_ptr")

    def __init__(self):
        self.version = -1
        self.tensor = None
        self.data_ptr = 0


# While a CUDA graph of the forward/backward is being captured, every cast is
# recorded into the graph (the weights change between replays), written into
# the cache's persistent tensor; the graph object keeps those tensors alive.
_CAPTURE = {"active": False, "keep": []}


def capture_casts(active: bool, keep=None):
    _CAPTURE["active"] = bool(active)
    _CAPTURE["keep"] = keep if keep is not None else []


def _captured_cast(weight, dtype, cache, transpose):
    src = weight.detach().t() if transpose else weight.detach()
    if cache.tensor is None or cache.tensor.shape != src.shape or cache.tensor.dtype != dtype:
        cache.tensor = torch.empty(src.shape, device=weight.device, dtype=dtype)
    cache.tensor.copy_(src)
    cache.version = -1  # eager use after capture recasts (and replaces the tensor)
    cache.data_ptr = weight.data_ptr()
    _CAPTURE["keep"].append(cache.tensor)
    return cache.tensor


def cached_cast(weight: torch.Tensor, dtype: torch.dtype, cache: _WeightCache) -> torch.Tensor:
    if weight.dtype == dtype:
        return weight.detach()
    if _CAPTURE["active"]:
        return _captured_cast(weight, dtype, cache, False)
    version = weight._version
    if (cache.tensor is None or cache.version != version or cache.data_ptr != weight.data_ptr()
            or cache.tensor.dtype != dtype):
        cache.tensor = weight.detach().to(dtype)
        cache.version = version
        cache.data_ptr = weight.data_ptr()
    return cache.tensor


def cached_cast_t(weight: torch.Tensor, dtype: torch.dtype, cache: _WeightCache) -> torch.Tensor:
    """``weight.T`` in ``dtype``, contiguous, refreshed when the weight's version changes."""
    if _CAPTURE["active"]:
        return _captured_cast(weight, dtype, cache, True)
    version = weight._version
    if (cache.tensor is None or cache.version != version or cache.data_ptr != weight.data_ptr()
            or cache.tensor.dtype != dtype):
        # one transposing, converting copy (no intermediate)
        src = weight.detach().t()
        cache.tensor = torch.empty(src.shape, device=weight.device, dtype=dtype).copy_(src)
        cache.version = version
        cache.data_ptr = weight.data_ptr()
    return cache.tensor


class _LinearFunction(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, w_compute):
        ctx.weight = weight
        x2 = x.reshape(-1, x.shape[-1])
        if x2.dtype != w_compute.dtype:
            x2 = x2.to(w_compute.dtype)
        y = gemm.matmul_nt(x2, w_compute)
        ctx.save_for_backward(x2, w_compute)
        ctx.in_shape = x.shape
        ctx.x_dtype = x.dtype
        ctx.w_dtype = weight.dtype
        return y.reshape(*x.shape[:-1], w_compute.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, w = ctx.saved_tensors
        g2 = gy.reshape(-1, gy.shape[-1])
        if g2.dtype != w.dtype:
            g2 = g2.to(w.dtype)
        gx = gw = None
        if ctx.needs_input_grad[0]:
            gx = gemm.matmul_nn(g2, w).reshape(ctx.in_shape)
            if gx.dtype != ctx.x_dtype:
                gx = gx.to(ctx.x_dtype)
        if ctx.needs_input_grad[1]:
            buf = ctx.weight.grad
            if (getattr(ctx.weight, ACCUMULATE_ATTR, False) and buf is not None and buf.is_cuda
                    and buf.dtype == torch.float32 and buf.is_contiguous()):
                # dW accumulates in the GEMM (beta = 1) straight into the
                # parameter's gradient buffer; autograd then has nothing to add.
                accumulate_weight_grad(ctx.weight, buf, g2, x2)
            else:
                gw = gemm.matmul_tn(g2, x2, out_dtype=ctx.w_dtype)
        return gx, gw, None


class Linear(torch.nn.Linear):
    """``nn.Linear`` (no bias) whose CUDA forward runs in ``compute_dtype``.

    The parameter is the usual ``weight`` so state-dict keys match the
    reference model (training/train.py:48-162).
    """

    def __init__(self, in_features, out_features, bias=False, device=None, dtype=None):
        if bias:
            raise ValueError("the reference architecture uses bias-free linear layers")
        super().__init__(in_features, out_features, bias=False, device=device, dtype=dtype)
        self._cache = _WeightCache()
        self.compute_dtype = torch.bfloat16

    def forward(self, x):
        if _ready.pending():
            _ready.wait(self.weight)
        if not x.is_cuda or self.compute_dtype == self.weight.dtype:
            if x.dtype != self.weight.dtype:
                x = x.to(self.weight.dtype)
            return torch.nn.functional.linear(x, self.weight)
        w = cached_cast(self.weight, self.compute_dtype, self._cache)
        return _LinearFunction.apply(x, self.weight, w)
