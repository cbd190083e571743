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
"""
from typing import Optional

import torch
from torch.library import custom_op, register_fake

__all__ = ["attn_func", "sparse_attn"]


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
