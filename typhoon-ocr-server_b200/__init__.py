"""B200-native GQA attention for the typhoon-ocr-server text decoder.

The product is the C-ABI shared library ``libtyphoon_attn.so`` built from ``csrc/``
(see ``include/*.h`` for the interface).  This module is the Python view of it, in the
style of the reference's ctypes binding (decoder.py:77-158 ``load_decoder_lib``):
``load_attention_lib()`` loads the library and declares every entry point's types.

There is no fallback: if the library is missing or cannot be loaded, loading raises.
"""

import ctypes
import os
from pathlib import Path

# Qwen3-VL 2B constants (decoder.py:28-41 of the reference)
HIDDEN_DIM = 2048
KV_DIM = 1024
NUM_Q_HEADS = 16
NUM_KV_HEADS = 8
HEAD_DIM = 128
NUM_LAYERS = 28
SCALE = 0.08838834764831843  # 1/sqrt(128), kernel/decoder.c:28
RMS_EPS = 1e-6
MROPE_SECTIONS = (24, 20, 20)
MROPE_THETA = 5000000.0

ATTN_KV_F32 = 0
ATTN_KV_BF16 = 1
ATTN_DT_F32 = 0
ATTN_DT_BF16 = 1

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libtyphoon_attn.so"


class KVHead(ctypes.Structure):
    _fields_ = [("k", ctypes.c_void_p), ("v", ctypes.c_void_p)]


class KVLayer(ctypes.Structure):
    _fields_ = [("heads", KVHead * NUM_KV_HEADS)]


class KVCache(ctypes.Structure):
    """Byte-for-byte the reference struct (kernel/kv_cache.h:11-26)."""

    _fields_ = [
        ("layers", KVLayer * NUM_LAYERS),
        ("seq_len", ctypes.c_int),
        ("max_seq_len", ctypes.c_int),
        ("rope_offset", ctypes.c_int),
    ]


class DecoderScratch(ctypes.Structure):
    """Byte-for-byte the reference struct (kernel/scratch.h:17-34): token-major activations
    (page-locked host memory here), then the head-major slots, which are device memory here."""

    _fields_ = [(name, ctypes.c_void_p) for name in (
        "residual", "q", "k", "v", "attn", "gate", "up", "mlp", "q_hm", "k_hm", "v_hm", "o_hm", "qkv_fused",
        "gate_up_fused")]


_F32P = ctypes.POINTER(ctypes.c_float)
_VP = ctypes.c_void_p


def build(verbose: bool = False) -> Path:
    """Compile the library for sm_100a with the package Makefile (nvcc + gcc)."""
    import subprocess

    env = dict(os.environ)
    env.setdefault("HOSTCC", "/usr/bin/gcc" if Path("/usr/bin/gcc").exists() else "gcc")
    r = subprocess.run(["make", "-j8", "-C", str(PKG_DIR), f"HOSTCC={env['HOSTCC']}"],
                       capture_output=True, text=True, env=env)
    if verbose or r.returncode != 0:
        print(r.stdout[-4000:], r.stderr[-4000:])
    if r.returncode != 0:
        raise RuntimeError("building libtyphoon_attn.so failed")
    return LIB_PATH


# Every exported entry point: name -> (restype, argtypes).
_SIGNATURES = {
    # kernel/attention.h:11-47
    "attention_decode_gqa": (None, [_VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_float]),
    "attention_prefill_gqa": (None, [_VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                     _VP, _VP, _VP, _VP]),
    "attention_chunked_prefill_gqa": (None, [_VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             ctypes.c_float]),
    # kernel/kv_cache.h:28-37
    "kv_cache_alloc": (_VP, [ctypes.c_int]),
    "kv_cache_free": (None, [_VP]),
    "kv_cache_clear": (None, [_VP]),
    "kv_cache_append": (None, [_VP, ctypes.c_int, _VP, _VP]),
    "kv_cache_append_prefill": (None, [_VP, ctypes.c_int, _VP, _VP, ctypes.c_int]),
    "kv_cache_advance": (None, [_VP, ctypes.c_int]),
    "kv_cache_k": (_VP, [_VP, ctypes.c_int, ctypes.c_int]),
    "kv_cache_v": (_VP, [_VP, ctypes.c_int, ctypes.c_int]),
    # kernel/scratch.h:36-37
    "decoder_scratch_alloc": (_VP, [ctypes.c_int]),
    "decoder_scratch_free": (None, [_VP]),
    # include/attn_ext.h (additions)
    "kv_cache_alloc_ex": (_VP, [ctypes.c_int, ctypes.c_int]),
    "kv_cache_dtype": (ctypes.c_int, [_VP]),
    "attn_last_error": (ctypes.c_char_p, []),
    "attn_clear_error": (None, []),
    "attn_set_stream": (None, [_VP]),
    "attn_sync": (ctypes.c_int, []),
    "attn_set_wait_limit_ns": (ctypes.c_int, [ctypes.c_ulonglong]),
    "attn_workspace_reserve": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "attention_decode_gqa_batched": (ctypes.c_int, [_VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_int,
                                                    ctypes.c_float]),
    "attention_prefill_fused_gqa": (ctypes.c_int, [_VP, _VP, _VP, ctypes.c_int, _VP, _VP, _VP, _VP, _VP, ctypes.c_int,
                                                   _VP, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float]),
    "attention_decode_append_gqa": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_float]),
    "attention_decode_gqa_noalloc": (ctypes.c_int, [_VP, _VP, _VP, ctypes.c_int, ctypes.c_int, _VP,
                                                    ctypes.c_int, ctypes.c_float, _VP]),
    "attention_prefill_fused_gqa_heads": (ctypes.c_int, [_VP, _VP, _VP, ctypes.c_int, _VP, _VP, _VP, _VP, _VP,
                                                         ctypes.c_int, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                                         ctypes.c_float, ctypes.c_int, ctypes.c_int]),
    "attention_decode_append_gqa_heads": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_float,
                                                         ctypes.c_int, ctypes.c_int]),
    "attn_heads_to_tokens": (ctypes.c_int, [_VP, _VP, ctypes.c_int, ctypes.c_int]),
    "attention_decode_append_fused_gqa": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, _VP, ctypes.c_int,
                                                         ctypes.c_float, ctypes.c_float]),
    "attn_gather_init": (ctypes.c_int, [ctypes.c_int, ctypes.c_int]),
    "attn_gather_handle": (ctypes.c_int, [_VP]),
    "attn_gather_connect": (ctypes.c_int, [_VP]),
    "attn_gather_close": (None, []),
    "attention_decode_append_gqa_gathered": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_float,
                                                            ctypes.c_int, ctypes.c_int]),
    "attn_shard_init": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_int, _VP, _VP]),
    "attn_shard_close": (None, []),
    "attn_shard_heads": (ctypes.c_int, [_VP, _VP]),
    "attention_prefill_fused_gqa_sharded": (ctypes.c_int, [_VP, _VP, _VP, ctypes.c_int, _VP, _VP, _VP, _VP, _VP,
                                                           ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                                           _VP]),
    "attention_decode_append_gqa_sharded": (ctypes.c_int, [_VP, _VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_float]),
}

# The all-gather callback of attn_shard_init: (send, recv, bytes, user) -> 0 on success.
ALLGATHER_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p)


def declared_symbols():
    """Names of the entry points this binding declares (all of include/*.h)."""
    return sorted(_SIGNATURES)


def load_attention_lib(path=None) -> ctypes.CDLL:
    """Load libtyphoon_attn.so and declare its entry points' types (no fallback)."""
    p = Path(path or os.environ.get("TYB_ATTN_LIB") or LIB_PATH)
    if not p.exists():
        raise FileNotFoundError(f"{p} is missing: run __graft_entry__.build() (nvcc for sm_100a)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def cache_struct(handle) -> KVCache:
    """The host-visible KVCache fields behind a handle (seq_len, rope_offset, pointers)."""
    return KVCache.from_address(handle)


def scratch_struct(handle) -> DecoderScratch:
    """The fields of a DecoderScratch handle from decoder_scratch_alloc."""
    return DecoderScratch.from_address(handle)


def last_error(lib) -> str:
    return (lib.attn_last_error() or b"").decode()


def check(lib, what="call"):
    """Raise if the calling thread's library error is set; clear it."""
    msg = last_error(lib)
    if msg:
        lib.attn_clear_error()
        raise RuntimeError(f"{what}: {msg}")
