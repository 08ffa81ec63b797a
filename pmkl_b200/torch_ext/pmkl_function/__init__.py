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
  are read in place by the forward and the backward, and the gradients come
  back in their inputs' layout.

One addition without a reference counterpart:

    out, out_m, out_l = fused_self_attention_ex(q, k, v, is_causal, scale=0.0)

takes k, v with fewer heads than q (grouped-query / multi-query attention:
query head h reads K/V head h // (H // H_kv)) and an explicit score scale
(<= 0: 1/sqrt(D)); its backward returns dk, dv with k's and v's head count,
each the sum over the query heads that read it.
"""
import torch
from torch.autograd import Function

import pmkl_pytorch_ext

__all__ = [
    'fused_self_attention',
    'fused_self_attention_ex',
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
        # Strided q, k, v and grad_output are read in place (the reference
        # makes them contiguous, fused_self_attention.cpp:179).
        dq, dk, dv = pmkl_pytorch_ext.fused_self_attention_bw(
            grad_output, q, k, v, out_m, out_l, is_casual.item())
        return dq, dk, dv, None, None


fused_self_attention = fused_self_attention_.apply


class fused_self_attention_ex_(Function):
    """Grouped-query form with an explicit score scale; see the module text."""

    @staticmethod
    def forward(q, k, v, is_causal, scale=0.0):
        if q.is_cuda:
            return pmkl_pytorch_ext.fused_self_attention_fw_ex(q, k, v, is_causal, False, 0, scale)
        raise NotImplementedError("pmkl_b200 runs on CUDA tensors only (no CPU path)")

    @staticmethod
    def setup_context(ctx, inputs, output):
        q, k, v, is_causal, scale = inputs
        out, out_m, out_l = output
        ctx.is_causal = bool(is_causal)
        ctx.scale = float(scale)
        ctx.save_for_backward(q, k, v, out_m, out_l)

    @staticmethod
    def backward(ctx, grad_output, grad_m, grad_l):
        q, k, v, out_m, out_l = ctx.saved_tensors
        dq, dk, dv = pmkl_pytorch_ext.fused_self_attention_bw_ex(
            grad_output, q, k, v, out_m, out_l, ctx.is_causal, 0, ctx.scale)
        return dq, dk, dv, None, None


fused_self_attention_ex = fused_self_attention_ex_.apply
