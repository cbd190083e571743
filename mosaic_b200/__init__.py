"""mosaic_b200: B200-native (sm_100a) block-sparse attention of Mosaic.

Public API (same signatures as the reference's ops.py / primitives.py):
    mosaic_sparse_attn(q, k, v, block_indices, block_size, softmax_scale=None)
        (differentiable in q, k, v; mosaic_attn_fwd / mosaic_attn_bwd are its halves)
    mosaic_attn_func(q, k, v, weight_ba_cmp_slc, block_attn_size, sparse_block_size,
                     sparse_block_count, block_attn_only, no_compression=False)
    attn_topk(q, k, block_count), block_attention(q, k, v, block_size)
    MosaicAttention(config, block_attn_only, no_compression=False)   # primitives.py:139-209
        (the whole attention block: fused projections + RoPE + gates, attention, to_o)
    CrossAttentionInterpolate(config)                                 # primitives.py:228-284
    MosaicBlock(config, block_attn_only, no_compression=False)        # primitives.py:212-229
        (attention block + fused FFN: norm2, w13 with noise / SiLU / product, w2 + residual)
    MosaicSwiGLU(dim, hidden_dim, noise_dim)                          # primitives.py:92-106
plus get_healpix_grid / rope_tables for the RoPE tables, `ensemble` for
member-sharded multi-GPU runs and `streaming.StreamedAttention` for host-resident
batches with their PCIe copies overlapped with the attention.
"""
from . import attention
from .attention import MosaicAttention
from . import interp
from .interp import CrossAttentionInterpolate
from . import updown
from . import ffn
from .ffn import MosaicBlock, MosaicSwiGLU
from .updown import HEALPixDownsample, HEALPixUpsample
from .healpix import get_healpix_grid, healpix_rope_tables, pix2ang_nest, rope_tables
from .ops import mosaic_attn_bwd, mosaic_attn_fwd, mosaic_sparse_attn, mosaic_sparse_attn_with_lse
from .primitives import attn_topk, block_attention, block_pool, cmp_attention, mosaic_attn_func

__all__ = [
    "mosaic_sparse_attn", "mosaic_sparse_attn_with_lse", "mosaic_attn_fwd", "mosaic_attn_bwd", "mosaic_attn_func", "attn_topk", "block_attention",
    "block_pool", "cmp_attention", "MosaicAttention", "CrossAttentionInterpolate", "MosaicBlock", "MosaicSwiGLU", "HEALPixDownsample", "HEALPixUpsample", "get_healpix_grid", "healpix_rope_tables", "pix2ang_nest", "rope_tables",
]
