"""The attention entry points as PyTorch custom operators (torch.library).

`torch.ops.mosaic_b200.attn_func` and `torch.ops.mosaic_b200.sparse_attn` wrap
mosaic_attn_func (primitives.py:54-59) and mosaic_sparse_attn (ops.py:557-566)
with a fake (meta) implementation that only describes the output, so graph
capture (torch.compile, torch.export, CUDA-graph trees of mode="reduce-overhead",
which the reference's inference script uses, inference.py:473) can trace a model
around them without running them: the ops stay opaque nodes that call the CUDA
library at run time. Eagerly, `mosaic_attn_func` / `mosaic_sparse_attn` call the
library directly and route through these ops only while being compiled, which
keeps the dispatcher's overhead out of eager calls.

For training graphs, `torch.ops.mosaic_b200.sparse_attn_fwd` (output and lse,
ops.mosaic_attn_fwd, ops.py:137-176) carries an autograd formula that calls
`torch.ops.mosaic_b200.sparse_attn_bwd` (ops.mosaic_attn_bwd, ops.py:436-507);
mosaic_sparse_attn routes through it while being compiled when an input needs a
gradient.
"""
from typing import Optional, Tuple

import torch
from torch.library import custom_op, register_autograd, register_fake

__all__ = ["attn_func", "sparse_attn", "sparse_attn_fwd", "sparse_attn_bwd"]


@custom_op("mosaic_b200::attn_func", mutates_args=(), device_types="cuda")
def attn_func(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, weight_ba_cmp_slc: Optional[torch.Tensor],
              block_attn_size: int, sparse_block_size: int, sparse_block_count: int, block_attn_only: bool,
              no_compression: bool) -> torch.Tensor:
    from .primitives import _mosaic_attn_func_eager

    return _mosaic_attn_func_eager(q, k, v, weight_ba_cmp_slc, block_attn_size, sparse_block_size,
                                   sparse_block_count, block_attn_only, no_compression)


@register_fake("mosaic_b200::attn_func")
def _attn_func_fake(q, k, v, weight_ba_cmp_slc, block_attn_size, sparse_block_size, sparse_block_count,
                    block_attn_only, no_compression):
    return q.new_empty(q.shape)


@custom_op("mosaic_b200::sparse_attn", mutates_args=(), device_types="cuda")
def sparse_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_indices: torch.Tensor, block_size: int,
                softmax_scale: float) -> torch.Tensor:
    from .ops import _sparse_fwd

    out, _ = _sparse_fwd(q, k, v, block_indices, block_size, softmax_scale, want_lse=False)
    return out.to(q.dtype)


@register_fake("mosaic_b200::sparse_attn")
def _sparse_attn_fake(q, k, v, block_indices, block_size, softmax_scale):
    return q.new_empty(q.shape)


@custom_op("mosaic_b200::sparse_attn_fwd", mutates_args=(), device_types="cuda")
def sparse_attn_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block_indices: torch.Tensor,
                    block_size: int, softmax_scale: float) -> Tuple[torch.Tensor, torch.Tensor]:
    from .ops import _sparse_fwd

    out, lse = _sparse_fwd(q, k, v, block_indices, block_size, softmax_scale, want_lse=True)
    return out.to(q.dtype), lse


@register_fake("mosaic_b200::sparse_attn_fwd")
def _sparse_attn_fwd_fake(q, k, v, block_indices, block_size, softmax_scale):
    return q.new_empty(q.shape), q.new_empty(q.shape[:3], dtype=torch.float32)


@custom_op("mosaic_b200::sparse_attn_bwd", mutates_args=(), device_types="cuda")
def sparse_attn_bwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, lse: torch.Tensor,
                    grad_out: torch.Tensor, block_indices: torch.Tensor, block_size: int,
                    softmax_scale: float) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    from .ops import mosaic_attn_bwd

    dq, dk, dv = mosaic_attn_bwd(q, k, v, out, lse, grad_out, softmax_scale, block_indices, block_size)
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


@register_fake("mosaic_b200::sparse_attn_bwd")
def _sparse_attn_bwd_fake(q, k, v, out, lse, grad_out, block_indices, block_size, softmax_scale):
    return q.new_empty(q.shape), k.new_empty(k.shape), v.new_empty(v.shape)


def _sparse_attn_fwd_setup(ctx, inputs, output):
    q, k, v, block_indices, block_size, softmax_scale = inputs
    out, lse = output
    ctx.save_for_backward(q, k, v, out, lse, block_indices)
    ctx.block_size = block_size
    ctx.softmax_scale = softmax_scale


def _sparse_attn_fwd_backward(ctx, grad_out, grad_lse):
    q, k, v, out, lse, block_indices = ctx.saved_tensors
    dq, dk, dv = torch.ops.mosaic_b200.sparse_attn_bwd(q, k, v, out, lse, grad_out.contiguous(), block_indices,
                                                        ctx.block_size, ctx.softmax_scale)
    return dq, dk, dv, None, None, None


register_autograd("mosaic_b200::sparse_attn_fwd", _sparse_attn_fwd_backward, setup_context=_sparse_attn_fwd_setup)
