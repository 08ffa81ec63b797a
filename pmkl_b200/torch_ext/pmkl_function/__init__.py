"""Autograd wrapper around ``pmkl_pytorch_ext`` -- the reference's public
Python API for fused self-attention, kept name for name
(``pmkl_pytorch_ext/pmkl_function/__init__.py:12-33``):

    out, out_m, out_l = fused_self_attention(q, k, v, is_casual, debug=False)

Differences from the reference, all deliberate:

* CUDA tensors run the B200 kernels whatever ``debug`` is (the reference
  raises ``NotImplementedError`` unless the tensors are on the CPU and
  ``debug`` is true, ``__init__.py:15-18``);
* CPU tensors raise ``NotImplementedError``: this build has no CPU path;
* the backward runs the B200 backward kernels on CUDA tensors (the
  reference's raises ``NotImplementedError`` for any non-CPU tensor,
  ``__init__.py:27-31``).  Like the reference it ignores the gradients
  arriving for ``out_m`` and ``out_l``;
* strided q, k, v (e.g. ``[B, S, H, D]`` tensors viewed as ``[B, H, S, D]``)
  are read in place by the forward; the backward gets contiguous copies.
"""
import torch
from torch.autograd import Function

import pmkl_pytorch_ext

__all__ = [
    'fused_self_attention',
]


class fused_self_attention_(Function):
    @staticmethod
    def forward(q, k, v, is_casual, debug=False):
        if q.is_cuda:
            return pmkl_pytorch_ext.fused_self_attention_fw(q, k, v, is_casual)
        raise NotImplementedError("pmkl_b200 runs on CUDA tensors only (no CPU path)")

    @staticmethod
    def setup_context(ctx, inputs, output):
        q, k, v, is_casual, debug = inputs
        out, out_m, out_l = output
        ctx.save_for_backward(q, k, v, torch.BoolTensor([is_casual]), torch.BoolTensor([debug]), out_m, out_l)

    @staticmethod
    def backward(ctx, grad_output, grad_m, grad_l):
        q, k, v, is_casual, debug, out_m, out_l = ctx.saved_tensors
        # The forward reads strided inputs in place; the backward kernels take
        # contiguous ones (as the reference's does, fused_self_attention.cpp:179).
        q, k, v = (t.contiguous() for t in (q, k, v))
        dq, dk, dv = pmkl_pytorch_ext.fused_self_attention_bw(
            grad_output, q, k, v, out_m, out_l, is_casual.item())
        return dq, dk, dv, None, None


fused_self_attention = fused_self_attention_.apply
