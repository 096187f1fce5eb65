"""Argument checks at the C-ABI boundary, on the CPU: the additions to the reference interface
return nonzero and leave a message in attn_last_error() for arguments they cannot take, before
touching the GPU (the reference's functions are void and have no error channel; these report)."""

import ctypes

import pytest

import gpu_helpers  # noqa: F401  (puts the package on sys.path)
from gpu_helpers import load_pkg_and_lib


@pytest.fixture(scope="module")
def pl():
    return load_pkg_and_lib()


@pytest.fixture()
def buf():
    # host addresses the checks may see but never dereference
    b = (ctypes.c_char * 4096)()
    base = (ctypes.addressof(b) + 255) & ~255
    return b, base


def _err(pkg, lib):
    msg = pkg.last_error(lib)
    lib.attn_clear_error()
    return msg


def test_noalloc_rejects_bad_arguments(pl, buf):
    pkg, lib = pl
    _, p = buf
    f, sc = lib.attention_decode_gqa_noalloc, ctypes.c_float(pkg.SCALE)
    lib.attn_clear_error()
    assert f(None, p, p, 64, pkg.ATTN_KV_BF16, p, 8, sc, None) != 0
    assert "NULL" in _err(pkg, lib)
    assert f(p, p, p, 64, 7, p, 8, sc, None) != 0
    assert "kv_dtype" in _err(pkg, lib)
    assert f(p, p, p, 64, pkg.ATTN_KV_BF16, p, 0, sc, None) != 0
    assert "kv_len" in _err(pkg, lib)
    assert f(p, p, p, 64, pkg.ATTN_KV_BF16, p, 65, sc, None) != 0
    assert "kv_len" in _err(pkg, lib)
    assert f(p, p + 4, p, 64, pkg.ATTN_KV_BF16, p, 8, sc, None) != 0
    assert "aligned" in _err(pkg, lib)
    # the query and output are read and written with 16-byte vectors: refused on the host
    assert f(p + 4, p, p, 64, pkg.ATTN_KV_BF16, p, 8, sc, None) != 0
    assert "aligned" in _err(pkg, lib)
    assert f(p, p, p, 64, pkg.ATTN_KV_BF16, p + 8, 8, sc, None) != 0
    assert "aligned" in _err(pkg, lib)


def test_heads_to_tokens_rejects_bad_arguments(pl, buf):
    pkg, lib = pl
    _, p = buf
    lib.attn_clear_error()
    assert lib.attn_heads_to_tokens(p, p, 16, 5) != 0
    assert "element type" in _err(pkg, lib)
    assert lib.attn_heads_to_tokens(p, p, -1, pkg.ATTN_DT_F32) != 0
    assert _err(pkg, lib)
    assert lib.attn_heads_to_tokens(None, p, 16, pkg.ATTN_DT_F32) != 0
    assert _err(pkg, lib)
    assert lib.attn_heads_to_tokens(p, p, 0, pkg.ATTN_DT_F32) == 0  # nothing to do
    assert not _err(pkg, lib)


def test_batched_decode_rejects_bad_arguments(pl, buf):
    pkg, lib = pl
    _, p = buf
    sc = ctypes.c_float(pkg.SCALE)
    lib.attn_clear_error()
    assert lib.attention_decode_gqa_batched(p, p, p, p, 0, 0, sc) != 0
    assert "batch" in _err(pkg, lib)
    assert lib.attention_decode_gqa_batched(p, None, p, p, 2, 0, sc) != 0
    assert _err(pkg, lib)


def test_head_range_is_checked(pl, buf):
    pkg, lib = pl
    _, p = buf
    sc = ctypes.c_float(pkg.SCALE)
    lib.attn_clear_error()
    for kvh0, n in ((7, 2), (-1, 1), (0, 0), (0, 9)):
        assert lib.attention_decode_append_gqa_heads(p, p, p, None, p, 0, sc, kvh0, n) != 0
        assert "KV heads" in _err(pkg, lib)


def test_gather_requires_setup(pl):
    pkg, lib = pl
    lib.attn_clear_error()
    assert lib.attn_gather_init(2, 2) != 0  # rank outside [0, world)
    assert _err(pkg, lib)
    assert lib.attn_gather_init(0, 9) != 0  # more ranks than the exchange holds
    assert _err(pkg, lib)


def test_wait_limit_and_reserve_reject_bad_arguments(pl):
    pkg, lib = pl
    lib.attn_clear_error()
    assert lib.attn_set_wait_limit_ns(10) != 0  # below 1 us: refused before any CUDA call
    assert "below" in _err(pkg, lib)
    assert lib.attn_workspace_reserve(-1, 0, 0) != 0
    assert "negative" in _err(pkg, lib)


def test_shard_init_rejects_bad_arguments(pl):
    import ctypes as C
    pkg, lib = pl
    cb = pkg.ALLGATHER_FN(lambda s, r, n, u: 0)
    p = C.cast(cb, C.c_void_p)
    lib.attn_clear_error()
    assert lib.attn_shard_init(0, 3, 0, p, None) != 0  # 3 ranks do not divide the 8 KV heads
    assert "nranks" in _err(pkg, lib)
    assert lib.attn_shard_init(2, 2, 0, p, None) != 0
    assert "rank" in _err(pkg, lib)
    assert lib.attn_shard_init(0, 2, 0, None, None) != 0  # no exchange callback
    assert "callback" in _err(pkg, lib)
    assert lib.attn_shard_heads(None, None) != 0  # nothing set up
    assert "attn_shard_init" in _err(pkg, lib)
