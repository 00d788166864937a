"""The reference's asynchronous-runtime API, on CUDA streams.

Reference: async_rt/__init__.py:1-6 (is_asyncrt_enabled), async_rt/runtime.py
(RUNTIME, AsyncRunMode, AsyncModeStart/End, AsyncSync) and
async_rt/async_ops.py:55-222 (MyMul, MyAdd, MyTanh, MySiLU,
ApplyRotaryComplexFn and the kernel helpers).

The reference imitates a stream on CPU cores: a dispatch mode hands the hot ops
to a C++ worker thread, and RUNTIME.sync() waits for that thread to drain.  On
a GPU every harp op is already enqueued on the current CUDA stream, so this
module keeps the API with stream semantics:

  RUNTIME.sync()        wait for the current CUDA stream (nothing to wait for
                        without CUDA); RUNTIME.shutdown() and bind() have no
                        worker to act on
  AsyncRunMode          a dispatch mode that runs every op as called (ops are
                        asynchronous on the stream already)
  AsyncModeStart / AsyncModeEnd
                        identity autograd functions that set
                        AsyncRunMode.mode_enable as the reference's do (End
                        and Start's backward also wait for the stream)
  AsyncSync(x, fwd, bwd) identity; waits for the stream in the forward and/or
                        backward when the flag is True
  is_asyncrt_enabled()  ASYNC_RUNTIME_ENABLE=1

Whole training steps get the reference's "enqueue, don't wait" effect from CUDA
graphs instead (harp_b200.trainer.Trainer with cuda_graph=True).
"""
from __future__ import annotations

import os

import torch
from torch.utils._python_dispatch import TorchDispatchMode

from ..ops import functional as Fn
from ..ops.modules import ApplyRotaryComplexFn, MySiLU, MyTanh  # noqa: F401  (reference names)


def is_asyncrt_enabled() -> bool:
    return os.environ.get("ASYNC_RUNTIME_ENABLE", "0") == "1"


class StreamRuntime:
    """RUNTIME: the handle the reference's trainer and models call."""

    def __init__(self):
        self.rank = int(os.environ.get("RANK", os.environ.get("OMPI_COMM_WORLD_RANK", "0")))
        # read by the reference's trainer around forward/backward; activation
        # offload here is TrainConfig.offload_activations
        self.offloader_enable = False

    def sync(self):
        if torch.cuda.is_available() and torch.cuda.is_initialized():
            torch.cuda.current_stream().synchronize()

    def shutdown(self):
        """No worker thread to stop."""

    def bind(self, core_id):
        """No worker thread to pin (the reference pins its op worker to a core)."""


RUNTIME = StreamRuntime()


class AsyncRunMode(TorchDispatchMode):
    mode_enable = False

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        return func(*args, **(kwargs or {}))


class AsyncModeStart(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        AsyncRunMode.mode_enable = True
        return x

    @staticmethod
    def backward(ctx, g):
        AsyncRunMode.mode_enable = False
        RUNTIME.sync()
        return g


class AsyncModeEnd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        AsyncRunMode.mode_enable = False
        RUNTIME.sync()
        return x

    @staticmethod
    def backward(ctx, g):
        AsyncRunMode.mode_enable = True
        return g


class AsyncSync(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, forward_sync, backward_sync):
        if forward_sync is True:
            RUNTIME.sync()
        ctx.backward_sync = backward_sync
        return x

    @staticmethod
    def backward(ctx, g):
        if ctx.backward_sync is True:
            RUNTIME.sync()
        return g, None, None


# ---------------------------------------------------------------------------
# broadcasting elementwise autograd functions (async_ops.py:55-122)
# ---------------------------------------------------------------------------
class MyMul(torch.autograd.Function):
    """a * b with broadcasting; each gradient is summed back to its input's shape."""

    @staticmethod
    def forward(ctx, a, b):
        ctx.save_for_backward(a, b)
        return _binary(a, b, mul=True)

    @staticmethod
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        ga = (g * b).sum_to_size(a.shape) if ctx.needs_input_grad[0] else None
        gb = (g * a).sum_to_size(b.shape) if ctx.needs_input_grad[1] else None
        return ga, gb


class MyAdd(torch.autograd.Function):
    """a + b with broadcasting; `a` may be a Python number (no gradient)."""

    @staticmethod
    def forward(ctx, a, b):
        ctx.a_shape = a.shape if isinstance(a, torch.Tensor) else None
        ctx.b_shape = b.shape
        if ctx.a_shape is None:
            return torch.add(b, a)
        return _binary(a, b, mul=False)

    @staticmethod
    def backward(ctx, g):
        ga = g.sum_to_size(ctx.a_shape) if ctx.a_shape is not None and ctx.needs_input_grad[0] else None
        gb = g.sum_to_size(ctx.b_shape) if ctx.needs_input_grad[1] else None
        return ga, gb


def _same_bf16(a, b, out=None) -> bool:
    ts = (a, b) if out is None else (a, b, out)
    return (all(isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous()
                for t in ts) and a.shape == b.shape and (out is None or out.shape == a.shape))


def _binary(a, b, mul: bool):
    if _same_bf16(a, b):
        out = torch.empty_like(a)
        (torch.ops.async_op.mul_out if mul else torch.ops.async_op.add_out)(a, b, out)
        return out
    out = torch.empty(torch.broadcast_shapes(a.shape, b.shape), dtype=a.dtype, device=a.device)
    return torch.mul(a, b, out=out) if mul else torch.add(a, b, out=out)


# ---------------------------------------------------------------------------
# kernel helpers (async_ops.py:181-222): write into the caller's output
# ---------------------------------------------------------------------------
def mm_kernel(output, input, weight, bias):
    """output = input @ weight^T + bias."""
    if input.is_cuda:
        torch.ops.xhpops.kp_linear_forward(input, weight, bias, output)
        return
    x2 = input.reshape(-1, input.shape[-1])
    output.copy_(Fn.gemm(x2, weight, bias=bias).view(output.shape))


def mm_backward_kernel(grad_input, grad_output_flat, inputx, weight, grad_weight, grad_bias):
    """grad_input = dY W, grad_weight = dY^T X, grad_bias = column sums of dY."""
    if grad_output_flat.is_cuda:
        torch.ops.xhpops.kp_linear_backward(grad_output_flat, inputx, weight, grad_input, grad_weight, grad_bias)
        return
    dy = grad_output_flat.reshape(-1, grad_output_flat.shape[-1])
    x2 = inputx.reshape(-1, inputx.shape[-1])
    dx, dw, db = Fn.linear_bwd(dy, x2, weight, need_bias=grad_bias is not None)
    grad_input.copy_(dx.view(grad_input.shape))
    grad_weight.copy_(dw)
    if grad_bias is not None:
        grad_bias.copy_(db)


def silu_kernel(output, input):
    if input.is_cuda:
        torch.ops.async_op.silu_out(input, output)
    else:
        output.copy_(Fn.silu(input))


def silu_backward_kernel(grad_input, grad_output, input):
    if input.is_cuda:
        torch.ops.async_op.silu_backward_out(grad_output, input, grad_input)
    else:
        grad_input.copy_(Fn.silu_bwd(grad_output, input))


def mul_kernel(output, input_a, input_b):
    torch.mul(input_a, input_b, out=output)


def add_kernel(output, input_a, input_b):
    torch.add(input_a, input_b, out=output)


def mul_fast(output, input_a, input_b):
    """Same-shape product on the harp elementwise kernel (bf16 CUDA tensors)."""
    if _same_bf16(input_a, input_b, output):
        torch.ops.async_op.mul_out(input_a, input_b, output)
    else:
        torch.mul(input_a, input_b, out=output)


def add_fast(output, input_a, input_b):
    """Same-shape sum on the harp elementwise kernel (bf16 CUDA tensors)."""
    if _same_bf16(input_a, input_b, output):
        torch.ops.async_op.add_out(input_a, input_b, output)
    else:
        torch.add(input_a, input_b, out=output)
