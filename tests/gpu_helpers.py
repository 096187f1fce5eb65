"""Helpers for the GPU tests: device buffers through torch, raw-pointer copies through
the CUDA runtime torch already loaded, and cache set-up through the C-ABI."""

import ctypes

import numpy as np

# Parity bar of the FP32 path against the reference (max-abs, rel-L2).
TOL_MAX, TOL_REL = 2e-3, 1e-3
# BF16 KV path against the FP32 reference, for K/V ~ N(0, 1): one bf16 rounding of K and V
# (relative 2^-9) moves a single-row output by up to ~3 * 2^-9; averaging over rows
# shrinks it.
TOL_BF16_MAX, TOL_BF16_REL = 1.5e-2, 6e-3

_cudart = None


def cudart():
    global _cudart
    if _cudart is None:
        import torch  # noqa: F401  (loads libcudart)
        _cudart = ctypes.CDLL("libcudart.so.12")
        _cudart.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    return _cudart


def d2h(ptr, shape, dtype=np.float32):
    """Copy a raw device buffer into a new numpy array."""
    out = np.empty(shape, dtype=dtype)
    rc = cudart().cudaMemcpy(out.ctypes.data, ptr, out.nbytes, 2)
    assert rc == 0, f"cudaMemcpy D2H failed: {rc}"
    return out


def vp(x):
    """c_void_p of a numpy array (host) or torch tensor (device)."""
    if isinstance(x, np.ndarray):
        assert x.flags["C_CONTIGUOUS"]
        return ctypes.c_void_p(x.ctypes.data)
    return ctypes.c_void_p(x.data_ptr())


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def check(pkg, lib, what):
    pkg.check(lib, what)


def new_cache(pkg, lib, max_seq, dtype):
    lib.attn_clear_error()
    h = lib.kv_cache_alloc_ex(max_seq, dtype)
    assert h, pkg.last_error(lib)
    return h


def fill_layer(pkg, lib, h, layer, k_rows, v_rows):
    """Write token-major rows [n,8,128] at rows 0..n-1 of `layer` (host path), restoring
    seq_len afterwards."""
    cs = pkg.cache_struct(h)
    saved = cs.seq_len
    cs.seq_len = 0
    lib.kv_cache_append_prefill(h, layer, vp(k_rows), vp(v_rows), k_rows.shape[0])
    cs.seq_len = saved
    check(pkg, lib, "fill_layer")


def bf16_round(a):
    """Round fp32 to the nearest bf16 (ties to even), back in fp32."""
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).float().numpy()


def head_first(rows):
    """token-major [n,8,128] -> head-first [8,n,128]."""
    return np.ascontiguousarray(rows.transpose(1, 0, 2))


def load_pkg_and_lib():
    """The package (from the repository) and its loaded library, for child processes that run
    outside the pytest fixtures."""
    import conftest
    pkg = conftest.load_pkg()
    return pkg, pkg.load_attention_lib()
