"""ctypes binding of libmosaic_b200.so (the C ABI declared in include/mosaic_b200.h).

The library is the only compute path of this package: when it is missing or
cannot be loaded, every op raises instead of falling back to anything else.
"""
import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmosaic_b200.so")

MOSAIC_OK = 0
MOSAIC_ERR_INVALID_ARGUMENT = 1
MOSAIC_ERR_UNSUPPORTED = 2
MOSAIC_ERR_WORKSPACE = 3
MOSAIC_ERR_CUDA = 4

MOSAIC_STATUS_TIMEOUT = 1
MOSAIC_STATUS_BAD_INDEX = 2

MOSAIC_DTYPE_BF16 = 0
MOSAIC_DTYPE_F16 = 1

# Every symbol include/mosaic_b200.h declares, with its ctypes signature.
_vp, _i, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t


class MosaicBsaArgs(ctypes.Structure):
    """Mirror of `MosaicBsaArgs` in include/mosaic_b200.h (field order matters)."""

    _fields_ = [
        ("q", _vp), ("k", _vp), ("v", _vp), ("gates", _vp),
        ("rope_cos", _vp), ("rope_sin", _vp),
        ("out", _vp), ("block_indices", _vp),
        ("workspace", _vp), ("workspace_bytes", _sz),
        ("status", _vp),
        ("batch", _i), ("seq_len", _i), ("num_q_heads", _i), ("num_kv_heads", _i), ("head_dim", _i),
        ("block_attn_size", _i), ("sparse_block_size", _i), ("sparse_block_count", _i),
        ("block_attn_only", _i), ("no_compression", _i),
        ("softmax_scale", _f),
        ("dtype", _i),
    ]


SIGNATURES = {
    "mosaic_abi_version": ([], _i),
    "mosaic_error_string": ([_i], ctypes.c_char_p),
    "mosaic_selftest_wait_timeout": ([_vp, _vp, _i, _vp], _i),
    "mosaic_bsa_workspace_bytes": ([_i, _i, _i, _i, _i, _i, _i, _i], _sz),
    "mosaic_bsa_fwd": ([ctypes.POINTER(MosaicBsaArgs), _vp], _i),
    "mosaic_bsa_fwd_noalloc": ([ctypes.POINTER(MosaicBsaArgs), _vp], _i),
    "mosaic_bsa_attend_fwd": ([_vp] * 8 + [_i] * 9 + [_f, _i, _vp], _i),
    "mosaic_sparse_attn_fwd": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _i, _vp], _i),
    "mosaic_block_attn_fwd": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _i, _vp], _i),
    "mosaic_block_pool": ([_vp] * 10 + [_i] * 7 + [_vp], _i),
    "mosaic_cmp_attn_fwd": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _i, _vp], _i),
    "mosaic_attn_topk": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp], _i),
    "mosaic_sparse_attn_bwd_workspace_bytes": ([_i] * 7, _sz),
    "mosaic_sparse_attn_bwd": ([_vp] * 10 + [_vp, _sz, _vp] + [_i] * 7 + [_f, _vp], _i),
    "mosaic_attn_qkv_proj": ([_vp] * 9 + [_i] * 6 + [_vp], _i),
    "mosaic_attn_out_proj": ([_vp] * 4 + [_i] * 5 + [_vp], _i),
    "mosaic_linear": ([_vp] * 5 + [_i] * 3 + [_vp], _i),
    "mosaic_linear_residual": ([_vp] * 6 + [_i] * 4 + [_vp], _i),
    "mosaic_attn_out_proj_residual": ([_vp] * 5 + [_i] * 6 + [_vp], _i),
    "mosaic_rms_norm": ([_vp, _vp, _vp, _i, _i, _f, _i, _vp], _i),
    "mosaic_ffn_swiglu": ([_vp] * 6 + [_i] * 4 + [_vp], _i),
    "mosaic_row_rms": ([_vp, _vp, _i, _i, _f, _vp], _i),
    "mosaic_interp_attend": ([_vp] * 6 + [_i] * 6 + [_f, _vp], _i),
    "mosaic_interp_attend_tiled": ([_vp] * 11 + [_i] * 8 + [_f, _vp], _i),
    "mosaic_healpix_downsample": ([_vp] * 6 + [_i] * 5 + [_f, _vp], _i),
    "mosaic_healpix_upsample": ([_vp] * 7 + [_i] * 5 + [_f, _vp], _i),
}

EXPECTED_ABI_VERSION = 2

_lib = None


class MosaicError(RuntimeError):
    """A mosaic_b200 C-ABI call returned a non-zero code."""

    def __init__(self, fn, code):
        self.code = code
        super().__init__(f"{fn} failed with code {code}: {error_string(code)}")


def load():
    """Load (once) and return the C-ABI library; raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"mosaic_b200: {LIB_PATH} is missing; build it with `python -m mosaic_b200.build` "
            "(there is no fallback implementation)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (argtypes, restype) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = restype
    if lib.mosaic_abi_version() != EXPECTED_ABI_VERSION:
        raise RuntimeError("mosaic_b200: library ABI version mismatch; rebuild it")
    _lib = lib
    return lib


def error_string(code):
    try:
        return load().mosaic_error_string(code).decode()
    except Exception:  # pragma: no cover - only when the library itself is unusable
        return "unknown"


def check(fn_name, code):
    if code != MOSAIC_OK:
        raise MosaicError(fn_name, code)
