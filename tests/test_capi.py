"""The C-ABI library: it loads without a GPU, exports every symbol that
include/mosaic_b200.h declares, and rejects bad arguments on the host (before any
CUDA call, so these run on a CPU-only machine)."""
import ctypes
import os
import re

import pytest

from mosaic_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mosaic_b200.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mosaic_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for n in ("mosaic_bsa_fwd", "mosaic_sparse_attn_fwd", "mosaic_block_attn_fwd", "mosaic_attn_topk",
              "mosaic_block_pool", "mosaic_cmp_attn_fwd", "mosaic_bsa_workspace_bytes"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def declared_arg_counts():
    """{function: number of parameters} from the header's MOSAIC_API declarations."""
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for name, params in re.findall(r"MOSAIC_API[^;(]*?\b(mosaic_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", src, flags=re.S):
        params = params.strip()
        out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_ctypes_signatures_match_the_header_arity():
    counts = declared_arg_counts()
    assert set(counts) == set(declared_functions())
    for name, n in counts.items():
        assert len(_lib.SIGNATURES[name][0]) == n, (name, n, len(_lib.SIGNATURES[name][0]))


def test_abi_version_and_error_strings():
    lib = _lib.load()
    assert lib.mosaic_abi_version() == _lib.EXPECTED_ABI_VERSION
    for code in range(5):
        assert lib.mosaic_error_string(code)
    assert b"unknown" in lib.mosaic_error_string(99)


def test_struct_layout_matches_header():
    # the Python mirror must have the header's field order
    src = open(HEADER).read()
    body = src[src.index("typedef struct MosaicBsaArgs"): src.index("} MosaicBsaArgs;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = re.findall(r"\b(\w+);", body)
    assert [f for f, _ in _lib.MosaicBsaArgs._fields_] == fields


def test_workspace_size():
    lib = _lib.load()
    b = lib.mosaic_bsa_workspace_bytes(1, 49152, 12, 3, 64, 64, 24, 0)
    nb = 49152 // 64
    expect = nb * 12 * 128 * 2 + nb * 3 * 128 * 2 + nb * 3 * 24 * 8
    assert expect <= b <= expect + 5 * 256
    assert lib.mosaic_bsa_workspace_bytes(1, 49152, 12, 3, 64, 64, 24, 1) > b + 49152 * 15 * 128 - 1


FAKE = ctypes.c_void_p(0x10000)  # 16-byte aligned, never dereferenced: validation fails first


def _sparse(**kw):
    a = dict(q=FAKE, k=FAKE, v=FAKE, idx=FAKE, out=FAKE, lse=None, status=None, B=1, N=1024, Hq=8, Hk=2, D=64,
             bs=64, K=4, scale=0.0, dtype=_lib.MOSAIC_DTYPE_BF16)
    a.update(kw)
    return _lib.load().mosaic_sparse_attn_fwd(a["q"], a["k"], a["v"], a["idx"], a["out"], a["lse"], a["status"],
                                             a["B"], a["N"], a["Hq"], a["Hk"], a["D"], a["bs"], a["K"],
                                             a["scale"], a["dtype"], None)


@pytest.mark.parametrize("kw,code", [
    (dict(q=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(idx=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(k=ctypes.c_void_p(0x10008)), _lib.MOSAIC_ERR_INVALID_ARGUMENT),  # misaligned
    (dict(D=128), _lib.MOSAIC_ERR_UNSUPPORTED),
    (dict(Hq=7, Hk=2), _lib.MOSAIC_ERR_INVALID_ARGUMENT),     # not a multiple
    (dict(bs=32), _lib.MOSAIC_ERR_UNSUPPORTED),
    (dict(N=1000), _lib.MOSAIC_ERR_INVALID_ARGUMENT),         # N % bs
    (dict(K=0), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(B=-1), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(dtype=2), _lib.MOSAIC_ERR_INVALID_ARGUMENT),        # neither bf16 nor fp16
])
def test_sparse_attn_rejects_bad_arguments(kw, code):
    assert _sparse(**kw) == code


def test_empty_inputs_are_a_no_op():
    assert _sparse(B=0) == _lib.MOSAIC_OK
    assert _sparse(N=0) == _lib.MOSAIC_OK


def _bsa(**kw):
    a = _lib.MosaicBsaArgs()
    a.q = a.k = a.v = a.gates = a.out = 0x10000
    a.workspace, a.workspace_bytes = 0x20000, 1 << 40
    a.batch, a.seq_len, a.num_q_heads, a.num_kv_heads, a.head_dim = 1, 3072, 4, 1, 64
    a.block_attn_size, a.sparse_block_size, a.sparse_block_count = 1024, 64, 8
    for k, v in kw.items():
        setattr(a, k, v)
    return _lib.load().mosaic_bsa_fwd(ctypes.byref(a), None)


@pytest.mark.parametrize("kw,code", [
    (dict(gates=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(block_attn_size=1000), _lib.MOSAIC_ERR_INVALID_ARGUMENT),     # N % bas
    (dict(sparse_block_count=49), _lib.MOSAIC_ERR_INVALID_ARGUMENT),    # K > nb
    (dict(sparse_block_count=0, no_compression=1), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(workspace=None), _lib.MOSAIC_ERR_WORKSPACE),
    (dict(workspace_bytes=16), _lib.MOSAIC_ERR_WORKSPACE),
    (dict(rope_cos=0x10000), _lib.MOSAIC_ERR_INVALID_ARGUMENT),         # cos without sin
    (dict(head_dim=32), _lib.MOSAIC_ERR_UNSUPPORTED),
    (dict(num_q_heads=16), _lib.MOSAIC_ERR_UNSUPPORTED),     # top-k with G = 16
    (dict(num_q_heads=27), _lib.MOSAIC_ERR_UNSUPPORTED),     # top-k with G = 9
    (dict(num_q_heads=6, num_kv_heads=4), _lib.MOSAIC_ERR_INVALID_ARGUMENT),  # not a multiple
    (dict(dtype=-1), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
])
def test_bsa_rejects_bad_arguments(kw, code):
    assert _bsa(**kw) == code


def test_bsa_null_args():
    assert _lib.load().mosaic_bsa_fwd(None, None) == _lib.MOSAIC_ERR_INVALID_ARGUMENT


def test_topk_rejects_bad_arguments():
    lib = _lib.load()
    bf16, f16 = _lib.MOSAIC_DTYPE_BF16, _lib.MOSAIC_DTYPE_F16
    assert lib.mosaic_attn_topk(FAKE, FAKE, FAKE, 1, 48, 4, 1, 64, 49, bf16, None) == _lib.MOSAIC_ERR_INVALID_ARGUMENT
    assert lib.mosaic_attn_topk(FAKE, FAKE, FAKE, 1, 48, 4, 1, 64, 129, f16, None) != _lib.MOSAIC_OK
    assert lib.mosaic_attn_topk(FAKE, FAKE, FAKE, 1, 48, 4, 1, 64, 0, f16, None) == _lib.MOSAIC_OK
    assert lib.mosaic_attn_topk(FAKE, FAKE, FAKE, 1, 48, 4, 1, 64, 8, 7, None) == _lib.MOSAIC_ERR_INVALID_ARGUMENT
    for hq in (9, 16):  # G outside 1 to 8
        assert lib.mosaic_attn_topk(FAKE, FAKE, FAKE, 1, 48, hq, 1, 64, 8, bf16, None) == _lib.MOSAIC_ERR_UNSUPPORTED


def _sparse_bwd(**kw):
    a = dict(q=FAKE, k=FAKE, v=FAKE, out=FAKE, go=FAKE, lse=FAKE, idx=FAKE, dq=FAKE, dk=FAKE, dv=FAKE,
             ws=ctypes.c_void_p(0x100000), ws_bytes=1 << 30, status=None, B=1, N=1024, Hq=8, Hk=2, D=64, bs=64,
             K=4, scale=0.0)
    a.update(kw)
    return _lib.load().mosaic_sparse_attn_bwd(
        a["q"], a["k"], a["v"], a["out"], a["go"], a["lse"], a["idx"], a["dq"], a["dk"], a["dv"], a["ws"],
        a["ws_bytes"], a["status"], a["B"], a["N"], a["Hq"], a["Hk"], a["D"], a["bs"], a["K"], a["scale"], None)


def test_sparse_bwd_workspace_size():
    lib = _lib.load()
    B, N, Hq, Hk, bs, K = 2, 4096, 8, 2, 64, 16
    b = lib.mosaic_sparse_attn_bwd_workspace_bytes(B, N, Hq, Hk, 64, bs, K)
    nkb = N // bs
    # D (fp32 per row and head) + counts, cursors, offsets, two list copies, per-tile union sizes
    expect = B * N * Hq * 4 + B * Hk * (3 * nkb + 1 + 2 * nkb * K) * 4 + B * Hk * (N // 128) * 4
    assert expect <= b <= expect + 7 * 256
    assert lib.mosaic_sparse_attn_bwd_workspace_bytes(-1, N, Hq, Hk, 64, bs, K) == 0


@pytest.mark.parametrize("kw,code", [
    (dict(q=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(lse=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(go=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(dv=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(dk=ctypes.c_void_p(0x10008)), _lib.MOSAIC_ERR_INVALID_ARGUMENT),  # misaligned
    (dict(D=128), _lib.MOSAIC_ERR_UNSUPPORTED),
    (dict(Hq=7, Hk=2), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(bs=32), _lib.MOSAIC_ERR_UNSUPPORTED),
    (dict(N=1000), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(K=0), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(K=1025), _lib.MOSAIC_ERR_UNSUPPORTED),
    (dict(ws=None), _lib.MOSAIC_ERR_WORKSPACE),
    (dict(ws_bytes=1024), _lib.MOSAIC_ERR_WORKSPACE),
    (dict(ws=ctypes.c_void_p(0x100010)), _lib.MOSAIC_ERR_WORKSPACE),  # not 256-aligned
])
def test_sparse_bwd_rejects_bad_arguments(kw, code):
    assert _sparse_bwd(**kw) == code


def test_sparse_bwd_empty_inputs_are_a_no_op():
    assert _sparse_bwd(B=0) == _lib.MOSAIC_OK
    assert _sparse_bwd(N=0) == _lib.MOSAIC_OK


def _qkv(**kw):
    a = dict(x=FAKE, w=FAKE, cos=None, sin=None, q=FAKE, k=FAKE, v=FAKE, g=FAKE, status=None, S=3072, B=1, dim=768,
             Hq=12, Hk=3, D=64)
    a.update(kw)
    return _lib.load().mosaic_attn_qkv_proj(a["x"], a["w"], a["cos"], a["sin"], a["q"], a["k"], a["v"], a["g"],
                                            a["status"], a["S"], a["B"], a["dim"], a["Hq"], a["Hk"], a["D"], None)


@pytest.mark.parametrize("kw,code", [
    (dict(x=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(v=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(q=ctypes.c_void_p(0x10008)), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(cos=FAKE), _lib.MOSAIC_ERR_INVALID_ARGUMENT),          # cos without sin
    (dict(D=128), _lib.MOSAIC_ERR_UNSUPPORTED),
    (dict(dim=760), _lib.MOSAIC_ERR_UNSUPPORTED),
    (dict(Hq=24, Hk=6), _lib.MOSAIC_ERR_UNSUPPORTED),           # 3 Hq gate columns > 64
    (dict(S=-1), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
])
def test_qkv_proj_rejects_bad_arguments(kw, code):
    assert _qkv(**kw) == code


def test_qkv_proj_without_gates_allows_more_heads_and_empty_is_noop():
    assert _qkv(S=0) == _lib.MOSAIC_OK and _qkv(B=0) == _lib.MOSAIC_OK
    assert _qkv(Hq=24, Hk=6, g=None, S=0) == _lib.MOSAIC_OK


@pytest.mark.parametrize("kw,code", [
    (dict(attn=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(out=ctypes.c_void_p(0x10008)), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(D=32), _lib.MOSAIC_ERR_UNSUPPORTED),
    (dict(dim=770), _lib.MOSAIC_ERR_UNSUPPORTED),
])
def test_out_proj_rejects_bad_arguments(kw, code):
    a = dict(attn=FAKE, w=FAKE, out=FAKE, S=3072, B=1, dim=768, Hq=12, D=64)
    a.update(kw)
    rc = _lib.load().mosaic_attn_out_proj(a["attn"], a["w"], a["out"], None, a["S"], a["B"], a["dim"], a["Hq"],
                                          a["D"], None)
    assert rc == code


@pytest.mark.parametrize("kw,code", [
    (dict(kv=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(nbr=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(out=ctypes.c_void_p(0x10008)), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(H=8), _lib.MOSAIC_ERR_UNSUPPORTED),          # head_dim 96
    (dict(dim=640, H=10), _lib.MOSAIC_ERR_UNSUPPORTED),  # dim not a multiple of 256
    (dict(k=0), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(S_from=0), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
])
def test_interp_attend_rejects_bad_arguments(kw, code):
    a = dict(kv=FAKE, nbr=FAKE, rel=FAKE, wq=FAKE, out=FAKE, S_to=49152, S_from=29040, B=1, dim=768, H=12, k=24)
    a.update(kw)
    rc = _lib.load().mosaic_interp_attend(a["kv"], a["nbr"], a["rel"], a["wq"], a["out"], None, a["S_to"],
                                          a["S_from"], a["B"], a["dim"], a["H"], a["k"], 0.0, None)
    assert rc == code


def test_linear_and_rms_reject_bad_arguments():
    lib = _lib.load()
    assert lib.mosaic_linear(FAKE, FAKE, FAKE, None, None, 100, 100, 64, None) == _lib.MOSAIC_ERR_UNSUPPORTED
    # widths that end inside a 32-column chunk: the epilogue stores whole chunks
    assert lib.mosaic_linear(FAKE, FAKE, FAKE, None, None, 100, 128, 40, None) == _lib.MOSAIC_ERR_UNSUPPORTED
    assert lib.mosaic_linear(None, FAKE, FAKE, None, None, 100, 128, 64, None) == _lib.MOSAIC_ERR_INVALID_ARGUMENT
    assert lib.mosaic_linear(FAKE, FAKE, FAKE, None, None, 0, 128, 64, None) == _lib.MOSAIC_OK
    assert lib.mosaic_row_rms(FAKE, FAKE, 10, 100, 1e-6, None) == _lib.MOSAIC_ERR_UNSUPPORTED
    assert lib.mosaic_row_rms(FAKE, None, 10, 128, 1e-6, None) == _lib.MOSAIC_ERR_INVALID_ARGUMENT


def _updown_call(kind, **kw):
    a = dict(x=ctypes.c_void_p(0x10000), sc=ctypes.c_void_p(0x20000), w=ctypes.c_void_p(0x30000),
             pos=ctypes.c_void_p(0x40000), nw=None, out=ctypes.c_void_p(0x50000),
             n=192, F=4, B=1, c_in=768, c_out=1024, eps=1e-2)
    a.update(kw)
    lib = _lib.load()
    if kind == "down":
        return lib.mosaic_healpix_downsample(a["x"], a["w"], a["pos"], a["nw"], a["out"], None, a["n"], a["F"],
                                             a["B"], a["c_in"], a["c_out"], a["eps"], None)
    return lib.mosaic_healpix_upsample(a["x"], a["sc"], a["w"], a["pos"], a["nw"], a["out"], None, a["n"],
                                       a["F"], a["B"], a["c_in"], a["c_out"], a["eps"], None)


@pytest.mark.parametrize("kind", ["down", "up"])
@pytest.mark.parametrize("kw,code", [
    (dict(c_in=96), _lib.MOSAIC_ERR_UNSUPPORTED),     # not a multiple of 64
    (dict(c_out=640 + 64), _lib.MOSAIC_ERR_UNSUPPORTED),  # not a multiple of 128
    (dict(n=-1), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(F=0), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(eps=-1.0), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(pos=None), _lib.MOSAIC_ERR_INVALID_ARGUMENT),
    (dict(out=ctypes.c_void_p(0x50008)), _lib.MOSAIC_ERR_INVALID_ARGUMENT),  # misaligned
    (dict(n=0), _lib.MOSAIC_OK),                      # empty: nothing to do, no CUDA call
])
def test_healpix_updown_rejects_bad_arguments(kind, kw, code):
    assert _updown_call(kind, **kw) == code
