"""Drop-in for primitives.MosaicAttention (primitives.py:139-209): the whole attention
block of a Mosaic layer on libmosaic_b200.so.

    x [S, B, dim] --mosaic_attn_qkv_proj-->  q (RoPE), k (RoPE), v, strategy gates
                  --mosaic_bsa_fwd-------->  block-sparse attention (local + compressed
                                             + selected, gated combine)
                  --mosaic_attn_out_proj-->  to_o, back to [S, B, dim]

The module has the reference's constructor, submodule names and buffers (`to_q`,
`to_k`, `to_v`, `to_o`, `to_strategy_combine_mlp`, `q_rope` / `k_rope` with
`cos_freqs` / `sin_freqs` and `initialize_rope`), so a reference state dict loads
into it and `primitives.MosaicAttention = mosaic_b200.MosaicAttention` swaps it in.
The projections run as one tcgen05 GEMM whose epilogue applies the RoPE, the gate
softmax and the layout changes (rearranges) of the reference's forward.

It serves inference: the fused projections have no backward, so a forward that
would need gradients for the module's weights or its input raises (wrap inference
in torch.no_grad() / torch.inference_mode(), as the reference's rollout does).
"""
import torch
import torch.nn as nn

from . import _lib
from .healpix import rope_tables
from .ops import _ptr, _require_cuda, _stream_ptr
from .primitives import mosaic_attn_func

__all__ = ["RoPE", "MosaicAttention", "qkv_projection", "out_projection"]


class RoPE(nn.Module):
    """Same buffers and initialiser as the reference's RoPE (primitives.py:108-135);
    forward applies the rotation with torch (the attention block itself never calls
    it: the projection epilogue rotates q and k)."""

    def __init__(self, dim, theta=10000):
        super().__init__()
        assert dim % 2 == 0
        self.dim = dim
        self.theta = theta
        self.register_buffer("cos_freqs", None, persistent=True)
        self.register_buffer("sin_freqs", None, persistent=True)

    def initialize_rope(self, positions):
        cos, sin = rope_tables(positions.float().cpu(), self.dim, float(self.theta))
        dev = positions.device
        self.register_buffer("cos_freqs", cos.to(dev), persistent=True)
        self.register_buffer("sin_freqs", sin.to(dev), persistent=True)

    def forward(self, x):
        cos = self.cos_freqs.unsqueeze(0).unsqueeze(2).repeat_interleave(2, dim=-1)
        sin = self.sin_freqs.unsqueeze(0).unsqueeze(2).repeat_interleave(2, dim=-1)
        xf = x.float()
        rot = torch.stack((-xf[..., 1::2], xf[..., 0::2]), dim=-1).flatten(-2)
        return (xf * cos + rot * sin).to(x.dtype)


def _bf16c(t):
    t = t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)
    return t.contiguous()


def qkv_projection(x, w_qkvg, num_q_heads, num_kv_heads, rope_cos=None, rope_sin=None, with_gates=True,
                   status=None):
    """q, k, v ([B, S, H, 64] bf16, q and k rotated when the tables are given) and the
    strategy gates ([3, B, S, Hq] bf16, or None) of x [S, B, dim] through
    mosaic_attn_qkv_proj; w_qkvg = cat(to_q, to_k, to_v[, to_strategy_combine_mlp])
    weights."""
    _require_cuda(x, w_qkvg)
    S, B, dim = x.shape
    Hq, Hk = int(num_q_heads), int(num_kv_heads)
    n = (Hq + 2 * Hk) * 64 + (3 * Hq if with_gates else 0)
    if tuple(w_qkvg.shape) != (n, dim):
        raise ValueError(f"w_qkvg must be [{n}, {dim}], got {tuple(w_qkvg.shape)}")
    xb, wb = _bf16c(x), _bf16c(w_qkvg)
    dev = x.device
    q = torch.empty(B, S, Hq, 64, dtype=torch.bfloat16, device=dev)
    k = torch.empty(B, S, Hk, 64, dtype=torch.bfloat16, device=dev)
    v = torch.empty(B, S, Hk, 64, dtype=torch.bfloat16, device=dev)
    g = torch.empty(3, B, S, Hq, dtype=torch.bfloat16, device=dev) if with_gates else None
    cos = rope_cos.float().contiguous() if rope_cos is not None else None
    sin = rope_sin.float().contiguous() if rope_sin is not None else None
    lib = _lib.load()
    with torch.cuda.device(dev):
        rc = lib.mosaic_attn_qkv_proj(_ptr(xb), _ptr(wb), _ptr(cos), _ptr(sin), _ptr(q), _ptr(k), _ptr(v), _ptr(g),
                                      _ptr(status), S, B, dim, Hq, Hk, 64, _stream_ptr(dev))
    _lib.check("mosaic_attn_qkv_proj", rc)
    return q, k, v, g


def out_projection(attn, w_o, status=None, residual=None):
    """rearrange(attn, 'b s h d -> s b (h d)') @ w_o^T through mosaic_attn_out_proj:
    attn [B, S, Hq, 64] -> [S, B, dim] bf16; with `residual` [S, B, dim] (bf16 or fp16)
    the result is residual + that in the residual's dtype (mosaic_attn_out_proj_residual)."""
    _require_cuda(attn, w_o)
    B, S, Hq, D = attn.shape
    dim = w_o.shape[0]
    if tuple(w_o.shape) != (dim, Hq * D):
        raise ValueError(f"w_o must be [dim, {Hq * D}], got {tuple(w_o.shape)}")
    ab, wb = _bf16c(attn), _bf16c(w_o)
    out = torch.empty(S, B, dim, dtype=torch.bfloat16, device=attn.device)
    lib = _lib.load()
    with torch.cuda.device(attn.device):
        if residual is None:
            rc = lib.mosaic_attn_out_proj(_ptr(ab), _ptr(wb), _ptr(out), _ptr(status), S, B, dim, Hq, D,
                                          _stream_ptr(attn.device))
        else:
            if residual.dtype not in (torch.bfloat16, torch.float16):
                raise TypeError(f"residual must be bf16 or fp16, got {residual.dtype}")
            rb = residual.contiguous()
            if tuple(rb.shape) != (S, B, dim):
                raise ValueError(f"residual must be [{S}, {B}, {dim}], got {tuple(rb.shape)}")
            out = torch.empty_like(rb)
            dt = _lib.MOSAIC_DTYPE_F16 if rb.dtype == torch.float16 else _lib.MOSAIC_DTYPE_BF16
            rc = lib.mosaic_attn_out_proj_residual(_ptr(ab), _ptr(wb), _ptr(rb), _ptr(out), _ptr(status), S, B, dim,
                                                   Hq, D, dt, _stream_ptr(attn.device))
    _lib.check("mosaic_attn_out_proj" if residual is None else "mosaic_attn_out_proj_residual", rc)
    return out


class MosaicAttention(nn.Module):
    """primitives.MosaicAttention (primitives.py:139-209) with the same constructor
    (`config` fields num_heads, gqa_ratio, dim, qkv_compress_ratio, rope, rope_theta,
    block_attn_size, sparse_block_size, sparse_block_count) and parameters."""

    def __init__(self, config, block_attn_only: bool, no_compression: bool = False):
        super().__init__()
        self.block_attn_only = block_attn_only
        self.no_compression = no_compression
        self.block_attn_size = config.block_attn_size
        self.sparse_block_size = config.sparse_block_size
        self.sparse_block_count = config.sparse_block_count
        q_heads = config.num_heads
        kv_heads = q_heads // config.gqa_ratio
        dim = config.dim
        head_dim = int(dim // q_heads // config.qkv_compress_ratio)
        self.q_heads, self.kv_heads, self.head_dim = q_heads, kv_heads, head_dim
        self.to_q = nn.Linear(dim, q_heads * head_dim, bias=False)
        self.to_k = nn.Linear(dim, kv_heads * head_dim, bias=False)
        self.to_v = nn.Linear(dim, kv_heads * head_dim, bias=False)
        self.to_o = nn.Linear(q_heads * head_dim, dim, bias=False)
        self.q_rope = RoPE(head_dim, config.rope_theta) if config.rope else None
        self.k_rope = RoPE(head_dim, config.rope_theta) if config.rope else None
        self.to_strategy_combine_mlp = None if block_attn_only else nn.Linear(dim, 3 * q_heads, bias=False)

    def _w_qkvg(self):
        """cat(to_q, to_k, to_v[, gate]) weights in bf16, rebuilt only when a weight changes
        (another tensor, or an in-place update, which bumps its version counter)."""
        ws = [self.to_q.weight, self.to_k.weight, self.to_v.weight]
        if self.to_strategy_combine_mlp is not None:
            ws.append(self.to_strategy_combine_mlp.weight)
        key = tuple((w.data_ptr(), w._version, w.dtype, w.device) for w in ws)
        if getattr(self, "_w_qkvg_key", None) != key:
            self._w_qkvg_cache = torch.cat([w.detach().to(torch.bfloat16) for w in ws], dim=0)
            self._w_qkvg_key = key
        return self._w_qkvg_cache

    def _check_rope_tables(self):
        """q_rope and k_rope must hold the same tables (the projection epilogue applies one
        pair to both); compared once per version of the tables, so that the forward is
        free of host synchronisation afterwards (and can be captured in a CUDA graph)."""
        ts = (self.q_rope.cos_freqs, self.q_rope.sin_freqs, self.k_rope.cos_freqs, self.k_rope.sin_freqs)
        key = tuple((t.data_ptr(), t._version) for t in ts)
        if getattr(self, "_rope_key", None) != key:
            if not (torch.equal(ts[0], ts[2]) and torch.equal(ts[1], ts[3])):
                raise ValueError("q_rope and k_rope must hold the same tables (both come from the same grid)")
            self._rope_key = key

    def forward(self, x, residual=None):
        """The block's attention on x [S, B, dim]; with `residual` (a bf16 or fp16 [S, B, dim]
        tensor, mosaic_b200.MosaicBlock passes the stream before norm1) it returns
        residual + attention(x) in the residual's dtype, the add done in the output
        projection's epilogue."""
        if torch.is_grad_enabled() and (x.requires_grad or any(p_.requires_grad for p_ in self.parameters())):
            raise NotImplementedError(
                "mosaic_b200.MosaicAttention serves inference (the fused projections have no backward); "
                "run it under torch.no_grad() or torch.inference_mode()")
        rope = self.q_rope is not None
        if rope and self.q_rope.cos_freqs is None:
            raise ValueError("RoPE tables not initialised (call q_rope/k_rope.initialize_rope)")
        if rope:
            self._check_rope_tables()
        with_gates = not self.block_attn_only
        q, k, v, g = qkv_projection(
            x, self._w_qkvg(), self.q_heads, self.kv_heads,
            self.q_rope.cos_freqs if rope else None, self.q_rope.sin_freqs if rope else None, with_gates)
        out = mosaic_attn_func(q, k, v, g, self.block_attn_size, self.sparse_block_size, self.sparse_block_count,
                               self.block_attn_only, self.no_compression)
        if residual is not None:
            return out_projection(out, self.to_o.weight, residual=residual)
        return out_projection(out, self.to_o.weight).to(x.dtype)
