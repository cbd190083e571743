"""Drop-in for the attention functions of the reference's primitives module.

`mosaic_attn_func`, `attn_topk` and `block_attention` keep the signatures of
primitives.py:54-59, :35-36 and :28; they run on libmosaic_b200.so:

    mosaic_attn_func  -> mosaic_bsa_fwd: (a) RoPE/pool, coarse attention,
                         (b) block scores + top-k, (c) fused local + selected
                         attention with the gated combine in the epilogue
    attn_topk         -> mosaic_block_pool is not needed (inputs are pooled) ->
                         mosaic_attn_topk
    block_attention   -> mosaic_block_attn_fwd

`mosaic_attn_func` additionally accepts `rope_tables=(cos, sin)` (fp32
[N, head_dim // 2], see healpix.rope_tables): q and k are then taken
UN-rotated and the library applies the 2D RoPE of RoPE.forward
(primitives.py:132-135) inside the pooling kernel, saving the separate RoPE
passes of MosaicAttention.forward (primitives.py:193-195).
"""
import ctypes

import torch

from . import _lib
from .ops import (HEAD_DIM, _act, _check_qkv, _ptr, _require_cuda, _stream_ptr, act_dtype, dtype_code,
                  mosaic_sparse_attn, pad_head_dim)

__all__ = ["mosaic_attn_func", "attn_topk", "block_attention", "block_pool", "cmp_attention", "bsa_attend",
           "mosaic_sparse_attn"]

COMBINE_GATED, COMBINE_NO_CMP, COMBINE_NO_SLC = 0, 1, 2


def _gates(weight_ba_cmp_slc, B, N, Hq, dt):
    w = weight_ba_cmp_slc
    if w.dim() == 5:
        if w.shape[-1] != 1:
            raise ValueError("weight_ba_cmp_slc must be [3, B, N, Hq, 1]")
        w = w[..., 0]
    if tuple(w.shape) != (3, B, N, Hq):
        raise ValueError(f"weight_ba_cmp_slc must be [3, {B}, {N}, {Hq}, 1], got {tuple(weight_ba_cmp_slc.shape)}")
    return _act(w, dt)


def mosaic_attn_func(q, k, v, weight_ba_cmp_slc, block_attn_size, sparse_block_size, sparse_block_count,
                     block_attn_only, no_compression=False, *, rope_tables=None, return_block_indices=False,
                     status=None):
    """Mosaic block-sparse attention forward (primitives.py:54-89).

    o = w0 * o_ba + w1 * o_cmp + w2 * o_slc with
      o_ba  = attention inside windows of block_attn_size tokens,
      o_cmp = attention over mean-pooled blocks of sparse_block_size tokens, repeated,
      o_slc = attention over the sparse_block_count blocks of highest pooled score.
    `block_attn_only` returns o_ba; `no_compression` drops o_cmp and renormalises
    (w0, w2); sparse_block_count == 0 drops o_slc and renormalises (w0, w1).
    fp16 inputs (the reference's dtype under fp16 autocast) run natively in fp16,
    with the pooled means and the top-k scores rounded to fp16 as the reference's
    attn_topk does then; other dtypes run in bf16. The result has q's dtype.
    Under torch.compile the call becomes the opaque custom op
    torch.ops.mosaic_b200.attn_func (see torch_ops.py).
    """
    if (torch.compiler.is_compiling() and rope_tables is None and not return_block_indices and status is None):
        from . import torch_ops  # noqa: F401  (registers the op)

        return torch.ops.mosaic_b200.attn_func(q, k, v, weight_ba_cmp_slc, int(block_attn_size),
                                               int(sparse_block_size), int(sparse_block_count),
                                               bool(block_attn_only), bool(no_compression))
    return _mosaic_attn_func_eager(q, k, v, weight_ba_cmp_slc, block_attn_size, sparse_block_size,
                                   sparse_block_count, block_attn_only, no_compression, rope_tables=rope_tables,
                                   return_block_indices=return_block_indices, status=status)


def _mosaic_attn_func_eager(q, k, v, weight_ba_cmp_slc, block_attn_size, sparse_block_size, sparse_block_count,
                            block_attn_only, no_compression=False, *, rope_tables=None, return_block_indices=False,
                            status=None):
    _require_cuda(q, k, v)
    _check_qkv(q, k, v)
    D0 = q.shape[-1]  # head_dim below 64: zero-padded to 64 (pad_head_dim), scale of D0
    if D0 != HEAD_DIM:
        if rope_tables is not None:
            raise ValueError("rope_tables needs head_dim 64; rotate q and k before the call for other head dims")
        q, k, v = pad_head_dim(q, k, v)
    B, N, Hq, D = q.shape
    Hk = k.shape[2]
    out_dtype = q.dtype
    lib = _lib.load()
    dt = act_dtype(q)
    qb, kb, vb = _act(q, dt), _act(k, dt), _act(v, dt)
    gates = None
    if not block_attn_only:
        _require_cuda(weight_ba_cmp_slc)
        gates = _gates(weight_ba_cmp_slc, B, N, Hq, dt)
    cos = sin = None
    if rope_tables is not None:
        cos, sin = rope_tables
        _require_cuda(cos, sin)
        if tuple(cos.shape) != (N, D // 2) or tuple(sin.shape) != (N, D // 2):
            raise ValueError(f"rope tables must be [{N}, {D // 2}]")
        cos = cos.float().contiguous()
        sin = sin.float().contiguous()
    bs = int(sparse_block_size) if sparse_block_size else 64
    K = 0 if block_attn_only else int(sparse_block_count)
    if not block_attn_only and K > N // bs:
        raise ValueError(f"sparse_block_count {K} exceeds the number of blocks {N // bs}")
    out = torch.empty(B, N, Hq, D, dtype=dt, device=q.device)
    want_idx = return_block_indices and not block_attn_only and K > 0
    idx = torch.empty(B, N // bs, Hk, K, dtype=torch.int64, device=q.device) if want_idx else None
    ws_bytes = lib.mosaic_bsa_workspace_bytes(B, N, Hq, Hk, D, bs, K, int(cos is not None))
    need_ws = (not block_attn_only) or cos is not None
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device) if need_ws else None

    args = _lib.MosaicBsaArgs()
    args.q, args.k, args.v = qb.data_ptr(), kb.data_ptr(), vb.data_ptr()
    args.gates = gates.data_ptr() if gates is not None else None
    args.rope_cos = cos.data_ptr() if cos is not None else None
    args.rope_sin = sin.data_ptr() if sin is not None else None
    args.out = out.data_ptr()
    args.block_indices = idx.data_ptr() if idx is not None else None
    args.workspace = ws.data_ptr() if ws is not None else None
    args.workspace_bytes = ws.numel() if ws is not None else 0
    args.status = status.data_ptr() if status is not None else None
    args.batch, args.seq_len, args.num_q_heads, args.num_kv_heads, args.head_dim = B, N, Hq, Hk, D
    args.block_attn_size = int(block_attn_size)
    args.sparse_block_size = bs
    args.sparse_block_count = K
    args.block_attn_only = int(bool(block_attn_only))
    args.no_compression = int(bool(no_compression))
    args.softmax_scale = float(D0 ** -0.5)
    args.dtype = dtype_code(dt)
    with torch.cuda.device(q.device):
        rc = lib.mosaic_bsa_fwd(ctypes.byref(args), _stream_ptr(q.device))
    _lib.check("mosaic_bsa_fwd", rc)
    if D0 != HEAD_DIM:
        out = out[..., :D0].contiguous()
    out = out.to(out_dtype)
    return (out, idx) if return_block_indices else out


@torch.no_grad()
def attn_topk(q, k, block_count):
    """Top-k block selection on pooled q/k (primitives.py:35-51): int64 [B, nb, Hk, K].
    Scores are rounded to fp16 for fp16 inputs and to bf16 otherwise."""
    _require_cuda(q, k)
    B, nb, Hq, D = q.shape
    Hk = k.shape[2]
    if k.shape[0] != B or k.shape[1] != nb or k.shape[3] != D or Hq % Hk != 0:
        raise ValueError("attn_topk: q [B, nb, Hq, D] and k [B, nb, Hk, D] do not match")
    if block_count > nb:
        raise ValueError(f"block_count {block_count} exceeds the number of blocks {nb}")
    lib = _lib.load()
    dt = act_dtype(q)
    qb, kb = _act(q, dt), _act(k, dt)
    idx = torch.empty(B, nb, Hk, int(block_count), dtype=torch.int64, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib.mosaic_attn_topk(_ptr(qb), _ptr(kb), _ptr(idx), B, nb, Hq, Hk, D, int(block_count), dtype_code(dt),
                                  _stream_ptr(q.device))
    _lib.check("mosaic_attn_topk", rc)
    return idx


def block_attention(q, k, v, block_size, status=None):
    """Full attention inside each window of block_size tokens (primitives.py:28-32)."""
    _require_cuda(q, k, v)
    _check_qkv(q, k, v)
    D0 = q.shape[-1]  # head_dim below 64: zero-padded to 64 (pad_head_dim), scale of D0
    if D0 != HEAD_DIM:
        if rope_tables is not None:
            raise ValueError("rope_tables needs head_dim 64; rotate q and k before the call for other head dims")
        q, k, v = pad_head_dim(q, k, v)
    B, N, Hq, D = q.shape
    Hk = k.shape[2]
    if N % block_size != 0:
        raise ValueError(f"seq_len {N} is not a multiple of block_size {block_size}")
    lib = _lib.load()
    dt = act_dtype(q)
    qb, kb, vb = _act(q, dt), _act(k, dt), _act(v, dt)
    out = torch.empty(B, N, Hq, D, dtype=dt, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib.mosaic_block_attn_fwd(_ptr(qb), _ptr(kb), _ptr(vb), _ptr(out), _ptr(status), B, N, Hq, Hk, D,
                                       int(block_size), float(D ** -0.5), dtype_code(dt), _stream_ptr(q.device))
    _lib.check("mosaic_block_attn_fwd", rc)
    return out.to(q.dtype)


def block_pool(q, k, v, block_size, rope_tables=None):
    """Mean-pool q, k, v over blocks (primitives.py:65-66,76), optionally after RoPE.

    Returns (q_cmp, k_cmp, v_cmp) or, with rope_tables, (q_cmp, k_cmp, v_cmp, q_rot, k_rot)."""
    _require_cuda(q, k, v)
    _check_qkv(q, k, v)
    D0 = q.shape[-1]  # head_dim below 64: zero-padded to 64 (pad_head_dim), scale of D0
    if D0 != HEAD_DIM:
        if rope_tables is not None:
            raise ValueError("rope_tables needs head_dim 64; rotate q and k before the call for other head dims")
        q, k, v = pad_head_dim(q, k, v)
    B, N, Hq, D = q.shape
    Hk = k.shape[2]
    if N % block_size != 0:
        raise ValueError(f"seq_len {N} is not a multiple of block_size {block_size}")
    nb = N // block_size
    lib = _lib.load()
    dt = act_dtype(q)
    qb, kb, vb = _act(q, dt), _act(k, dt), _act(v, dt)
    dev = q.device
    q_cmp = torch.empty(B, nb, Hq, D, dtype=dt, device=dev)
    k_cmp = torch.empty(B, nb, Hk, D, dtype=dt, device=dev)
    v_cmp = torch.empty(B, nb, Hk, D, dtype=dt, device=dev)
    cos = sin = q_rot = k_rot = None
    if rope_tables is not None:
        cos, sin = (t.float().contiguous() for t in rope_tables)
        q_rot = torch.empty_like(qb)
        k_rot = torch.empty_like(kb)
    with torch.cuda.device(dev):
        rc = lib.mosaic_block_pool(_ptr(qb), _ptr(kb), _ptr(vb), _ptr(cos), _ptr(sin), _ptr(q_rot), _ptr(k_rot),
                                   _ptr(q_cmp), _ptr(k_cmp), _ptr(v_cmp), B, N, Hq, Hk, D, int(block_size),
                                   dtype_code(dt), _stream_ptr(dev))
    _lib.check("mosaic_block_pool", rc)
    if rope_tables is not None:
        return q_cmp, k_cmp, v_cmp, q_rot, k_rot
    return q_cmp, k_cmp, v_cmp


def cmp_attention(q_cmp, k_cmp, v_cmp, status=None):
    """Attention over the pooled blocks: flash_attn_func(q_cmp, k_cmp, v_cmp) of primitives.py:77."""
    _require_cuda(q_cmp, k_cmp, v_cmp)
    _check_qkv(q_cmp, k_cmp, v_cmp)
    B, nb, Hq, D = q_cmp.shape
    Hk = k_cmp.shape[2]
    lib = _lib.load()
    dt = act_dtype(q_cmp)
    qb, kb, vb = _act(q_cmp, dt), _act(k_cmp, dt), _act(v_cmp, dt)
    out = torch.empty(B, nb, Hq, D, dtype=dt, device=q_cmp.device)
    with torch.cuda.device(q_cmp.device):
        rc = lib.mosaic_cmp_attn_fwd(_ptr(qb), _ptr(kb), _ptr(vb), _ptr(out), _ptr(status), B, nb, Hq, Hk, D,
                                     float(D ** -0.5), dtype_code(dt), _stream_ptr(q_cmp.device))
    _lib.check("mosaic_cmp_attn_fwd", rc)
    return out.to(q_cmp.dtype)


def bsa_attend(q, k, v, block_indices, weight_ba_cmp_slc, o_cmp, block_attn_size, sparse_block_size,
               sparse_block_count, combine=COMBINE_GATED, status=None):
    """The fused attention stage alone (kernel (c) of mosaic_attn_func): local window
    + selected blocks `block_indices` + gated combine with the pooled coarse
    attention `o_cmp` [B, N // sparse_block_size, Hq, D]."""
    _require_cuda(q, k, v)
    _check_qkv(q, k, v)
    D0 = q.shape[-1]  # head_dim below 64: zero-padded to 64 (pad_head_dim), scale of D0
    if D0 != HEAD_DIM:
        if rope_tables is not None:
            raise ValueError("rope_tables needs head_dim 64; rotate q and k before the call for other head dims")
        q, k, v = pad_head_dim(q, k, v)
    B, N, Hq, D = q.shape
    Hk = k.shape[2]
    lib = _lib.load()
    dt = act_dtype(q)
    qb, kb, vb = _act(q, dt), _act(k, dt), _act(v, dt)
    gates = _gates(weight_ba_cmp_slc, B, N, Hq, dt)
    idx = block_indices.to(torch.int64).contiguous() if block_indices is not None else None
    oc = _act(o_cmp, dt) if o_cmp is not None else None
    out = torch.empty(B, N, Hq, D, dtype=dt, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib.mosaic_bsa_attend_fwd(_ptr(qb), _ptr(kb), _ptr(vb), _ptr(idx), _ptr(gates), _ptr(oc), _ptr(out),
                                       _ptr(status), B, N, Hq, Hk, D, int(block_attn_size), int(sparse_block_size),
                                       int(sparse_block_count), int(combine), float(D ** -0.5), dtype_code(dt),
                                       _stream_ptr(q.device))
    _lib.check("mosaic_bsa_attend_fwd", rc)
    return out.to(q.dtype)
