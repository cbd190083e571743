"""Drop-in for the reference's ops module (ops.py): `mosaic_sparse_attn`.

Same call signature and semantics as ops.mosaic_sparse_attn (ops.py:557-566):
q [B, N, Hq, D], k/v [B, N, Hk, D], block_indices int64 [B, N // block_size, Hk, K];
query n of q head j attends to the K*block_size keys of blocks
block_indices[b, n // block_size, j // (Hq // Hk), :] of kv head j // (Hq // Hk)
with softmax scale `softmax_scale` (default D ** -0.5). The tensor-core operands
are fp16 when q is fp16 (the reference's dtype under fp16 autocast) and bf16
otherwise (like the reference kernel, which casts to bf16, ops.py:92,115-116),
always with fp32 accumulation; the result is returned in q's dtype (ops.py:538).

The work runs in `mosaic_sparse_attn_fwd` (and, for gradients,
`mosaic_sparse_attn_bwd`) of libmosaic_b200.so on the current CUDA stream.
There is no CPU path: CPU tensors raise, as the reference's Triton kernel would.
"""
import ctypes

import torch

from . import _lib

__all__ = ["mosaic_sparse_attn", "mosaic_sparse_attn_with_lse", "mosaic_attn_fwd", "mosaic_attn_bwd",
           "MosaicAttnFunction"]


def _stream_ptr(device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _require_cuda(*tensors):
    for t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError("mosaic_b200 ops need CUDA tensors (there is no CPU implementation)")
    dev = tensors[0].device
    for t in tensors[1:]:
        if t.device != dev:
            raise ValueError("all tensors must be on the same CUDA device")


def _bf16(t):
    t = t if t.dtype == torch.bfloat16 else t.to(torch.bfloat16)
    return t.contiguous()


def act_dtype(t):
    """The 16-bit type a forward call computes in: fp16 when `t` (q) is fp16, else bf16."""
    return torch.float16 if t.dtype == torch.float16 else torch.bfloat16


def dtype_code(dt):
    """The C ABI's code (MOSAIC_DTYPE_*) for an activation type from act_dtype."""
    return _lib.MOSAIC_DTYPE_F16 if dt == torch.float16 else _lib.MOSAIC_DTYPE_BF16


def _act(t, dt):
    t = t if t.dtype == dt else t.to(dt)
    return t.contiguous()


def _check_qkv(q, k, v):
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError("q, k, v must be [batch, seq_len, heads, head_dim]")
    if k.shape != v.shape or q.shape[0] != k.shape[0] or q.shape[1] != k.shape[1] or q.shape[3] != k.shape[3]:
        raise ValueError(f"inconsistent q/k/v shapes {tuple(q.shape)} {tuple(k.shape)} {tuple(v.shape)}")
    if q.shape[2] % k.shape[2] != 0:
        raise ValueError("num_q_heads must be a multiple of num_kv_heads")


def status_buffer(device):
    """A zeroed device int32 status word for the C ABI's optional `status` argument."""
    return torch.zeros(1, dtype=torch.int32, device=device)


def check_status(status):
    """Synchronising read of a status word; raises on any device-side fault bit."""
    s = int(status.item())
    if s & _lib.MOSAIC_STATUS_TIMEOUT:
        raise RuntimeError("mosaic_b200: a kernel pipeline wait timed out (results are invalid)")
    if s & _lib.MOSAIC_STATUS_BAD_INDEX:
        raise RuntimeError("mosaic_b200: block index outside [0, seq_len // block_size)")
    return s


def _sparse_fwd(q, k, v, block_indices, block_size, softmax_scale, want_lse, status=None):
    _require_cuda(q, k, v, block_indices)
    _check_qkv(q, k, v)
    B, N, Hq, D = q.shape
    Hk = k.shape[2]
    if block_indices.dim() != 4 or tuple(block_indices.shape[:3]) != (B, N // block_size, Hk):
        raise ValueError(f"block_indices must be [B, N // block_size, Hk, K], got {tuple(block_indices.shape)}")
    lib = _lib.load()
    dt = act_dtype(q)
    qb, kb, vb = _act(q, dt), _act(k, dt), _act(v, dt)
    idx = block_indices.to(torch.int64).contiguous()
    out = torch.empty(B, N, Hq, D, dtype=dt, device=q.device)
    lse = torch.empty(B, N, Hq, dtype=torch.float32, device=q.device) if want_lse else None
    with torch.cuda.device(q.device):
        rc = lib.mosaic_sparse_attn_fwd(
            _ptr(qb), _ptr(kb), _ptr(vb), _ptr(idx), _ptr(out), _ptr(lse), _ptr(status),
            B, N, Hq, Hk, D, int(block_size), int(idx.shape[-1]), float(softmax_scale), dtype_code(dt),
            _stream_ptr(q.device))
    _lib.check("mosaic_sparse_attn_fwd", rc)
    return out, lse


def mosaic_attn_fwd(q, k, v, block_indices, block_size, softmax_scale, status=None):
    """ops.mosaic_attn_fwd (ops.py:137-176): (output in the activation type of q (fp16 or
    bf16), lse fp32 [B, N, Hq] in log2 units)."""
    return _sparse_fwd(q, k, v, block_indices, block_size, softmax_scale, want_lse=True, status=status)


def mosaic_attn_bwd(q, k, v, output, lse, grad_o, softmax_scale, block_indices, block_size, status=None):
    """ops.mosaic_attn_bwd (ops.py:436-507): (grad_q, grad_k, grad_v), bf16, through
    `mosaic_sparse_attn_bwd` of libmosaic_b200.so on the current stream.

    `output` and `lse` are the forward's (mosaic_attn_fwd). grad_q counts a block
    selected twice twice, as the forward does; grad_k / grad_v take each selecting
    query block once, like the reference's boolean block mask (ops.py:277-297).
    Keys of blocks that no query block selected get zero gradients."""
    _require_cuda(q, k, v, output, lse, grad_o, block_indices)
    _check_qkv(q, k, v)
    B, N, Hq, D = q.shape
    Hk = k.shape[2]
    if output.shape != q.shape or grad_o.shape != q.shape:
        raise ValueError("output and grad_o must have q's shape")
    if tuple(lse.shape) != (B, N, Hq):
        raise ValueError(f"lse must be [B, N, Hq], got {tuple(lse.shape)}")
    if block_indices.dim() != 4 or tuple(block_indices.shape[:3]) != (B, N // block_size, Hk):
        raise ValueError(f"block_indices must be [B, N // block_size, Hk, K], got {tuple(block_indices.shape)}")
    lib = _lib.load()
    qb, kb, vb, ob, gb = _bf16(q), _bf16(k), _bf16(v), _bf16(output), _bf16(grad_o)
    lse32 = lse.to(torch.float32).contiguous()
    idx = block_indices.to(torch.int64).contiguous()
    K = int(idx.shape[-1])
    grad_q = torch.empty(B, N, Hq, D, dtype=torch.bfloat16, device=q.device)
    grad_k = torch.empty(B, N, Hk, D, dtype=torch.bfloat16, device=q.device)
    grad_v = torch.empty(B, N, Hk, D, dtype=torch.bfloat16, device=q.device)
    nbytes = lib.mosaic_sparse_attn_bwd_workspace_bytes(B, N, Hq, Hk, D, int(block_size), K)
    ws = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib.mosaic_sparse_attn_bwd(
            _ptr(qb), _ptr(kb), _ptr(vb), _ptr(ob), _ptr(gb), _ptr(lse32), _ptr(idx),
            _ptr(grad_q), _ptr(grad_k), _ptr(grad_v), _ptr(ws), ws.numel(), _ptr(status),
            B, N, Hq, Hk, D, int(block_size), K, float(softmax_scale), _stream_ptr(q.device))
    _lib.check("mosaic_sparse_attn_bwd", rc)
    return grad_q, grad_k, grad_v


class MosaicAttnFunction(torch.autograd.Function):
    """ops.MosaicAttnFunction (ops.py:510-554). The forward keeps (q, k, v, output,
    lse, block_indices) only when an input needs a gradient; the backward returns
    the gradients in the inputs' dtypes."""

    @staticmethod
    def forward(ctx, q, k, v, block_indices, block_size, softmax_scale):
        need_grad = any(ctx.needs_input_grad[:3])
        out, lse = _sparse_fwd(q, k, v, block_indices, block_size, softmax_scale, want_lse=need_grad)
        if need_grad:
            ctx.save_for_backward(q, k, v, out, lse, block_indices)
            ctx.block_size = block_size
            ctx.softmax_scale = softmax_scale
        return out.to(q.dtype)

    @staticmethod
    def backward(ctx, grad_o):
        q, k, v, out, lse, block_indices = ctx.saved_tensors
        dq, dk, dv = mosaic_attn_bwd(q, k, v, out, lse, grad_o, ctx.softmax_scale, block_indices, ctx.block_size)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None, None


HEAD_DIM = 64  # the kernels' head dimension


def pad_head_dim(*ts):
    """Zero-pads the last (head) dimension of [B, N, H, d] tensors up to 64 for d < 64:
    zero columns add nothing to q.k, to the pooled means or to the top-k scores, and the
    output's padded columns are zero, so a head_dim below 64 (the reference's kernel takes
    any feature_dim, ops.py:25-60) runs on the 64-wide kernels with the softmax scale of
    the original d. Raises for d > 64."""
    d = ts[0].shape[-1]
    if d > HEAD_DIM:
        raise ValueError(f"head_dim {d} is not supported (at most {HEAD_DIM})")
    if d == HEAD_DIM:
        return ts
    return tuple(torch.nn.functional.pad(t, (0, HEAD_DIM - d)) for t in ts)


def mosaic_sparse_attn(q, k, v, block_indices, block_size, softmax_scale=None):
    """Selected-block attention (ops.py:557-566), differentiable in q, k, v. Under
    torch.compile the call becomes the opaque custom op torch.ops.mosaic_b200.sparse_attn
    (or sparse_attn_fwd, which has an autograd formula, when an input needs a gradient).
    head_dim 64, or less (zero-padded to 64, see pad_head_dim)."""
    softmax_scale = q.shape[-1] ** -0.5 if softmax_scale is None else softmax_scale
    d = q.shape[-1]
    if d != HEAD_DIM:
        q, k, v = pad_head_dim(q, k, v)
        return mosaic_sparse_attn(q, k, v, block_indices, block_size, softmax_scale)[..., :d].contiguous()
    if torch.compiler.is_compiling():
        from . import torch_ops  # noqa: F401  (registers the op)

        if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
            return torch.ops.mosaic_b200.sparse_attn_fwd(q, k, v, block_indices, int(block_size),
                                                         float(softmax_scale))[0]
        return torch.ops.mosaic_b200.sparse_attn(q, k, v, block_indices, int(block_size), float(softmax_scale))
    return MosaicAttnFunction.apply(q, k, v, block_indices, block_size, softmax_scale)


def mosaic_sparse_attn_with_lse(q, k, v, block_indices, block_size, softmax_scale=None, status=None):
    """Like mosaic_sparse_attn, also returning the log-sum-exp in log2 units
    (fp32 [B, N, Hq]), the second output of ops.mosaic_attn_fwd (ops.py:176)."""
    softmax_scale = q.shape[-1] ** -0.5 if softmax_scale is None else softmax_scale
    d = q.shape[-1]
    qp, kp, vp = pad_head_dim(q, k, v)
    out, lse = _sparse_fwd(qp, kp, vp, block_indices, block_size, softmax_scale, want_lse=True, status=status)
    return out[..., :d].contiguous().to(q.dtype), lse
