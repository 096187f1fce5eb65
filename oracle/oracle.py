"""Python view of the oracle -- TEST INFRASTRUCTURE ONLY.

Two CPU implementations of the reference hot path, used only as checkers (tests/,
__graft_entry__.smoke, bench.py's CPU-baseline leg):

* ``Oracle``  -- liboracle.so, the C restatement in attn_oracle.c (always available once
  built; it travels with the repository snapshot).
* ``RefLib``  -- _ref/libref_attn.so, the reference's own kernel/attention.c,
  kernel/kv_cache.c and kernel/ops.c compiled unmodified for x86_64 (oracle/Makefile).
  Present only where it was built; ``RefLib.available()`` says so.

All arrays are numpy fp32 / int32, C-contiguous.
"""

import ctypes
import os
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_LIB = HERE / "liboracle.so"
REF_LIB = HERE / "_ref" / "libref_attn.so"
# The reference source tree, read only to compile oracle/_ref and by the boundary test that
# compiles its decoder.c: the TYB_REFERENCE_DIR environment variable, else the mount point
# used when this repository was built.  Nothing on a GPU box reads it.
REFERENCE_DIR = Path(os.environ.get("TYB_REFERENCE_DIR", "/root/reference"))


def reference_present():
    """True when the reference tree (its kernel/ sources) is readable here."""
    return (REFERENCE_DIR / "kernel" / "attention.c").exists()


HQ, HKV, D = 16, 8, 128
NUM_LAYERS = 28
THETA = 5000000.0
EPS = 1e-6

_VP = ctypes.c_void_p


def host_threads():
    """Cores this process may run on (its CPU affinity), at least 1."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def set_host_threads(n):
    """Thread count of later OpenMP parallel regions in the libraries here (both link the
    system libgomp).  Launchers such as torchrun export OMP_NUM_THREADS=1 to their workers;
    this overrides it for the calling thread.  Returns the count set, or 0 if libgomp is
    not loadable."""
    try:
        gomp = ctypes.CDLL("libgomp.so.1")
    except OSError:
        return 0
    gomp.omp_set_num_threads.argtypes = [ctypes.c_int]
    gomp.omp_set_num_threads(int(n))
    return int(n)


def _p(a):
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be C-contiguous"
    return a.ctypes.data_as(_VP)


def build():
    """liboracle.so, and oracle/_ref where the reference tree is present."""
    import subprocess
    target = "all" if reference_present() else "oracle"
    r = subprocess.run(["make", "-C", str(HERE), target, f"REF={REFERENCE_DIR}"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout[-3000:] + r.stderr[-3000:])


class Oracle:
    """The C restatement (attn_oracle.c)."""

    def __init__(self, path=ORACLE_LIB):
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        L.oracle_attention_prefill.argtypes = [_VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.oracle_attention_chunked_prefill.argtypes = [_VP, _VP, _VP, ctypes.c_int, _VP, ctypes.c_int,
                                                       ctypes.c_int, ctypes.c_float]
        L.oracle_attention_decode.argtypes = [_VP, _VP, _VP, ctypes.c_int, _VP, ctypes.c_int, ctypes.c_float]
        L.oracle_rmsnorm_rows.argtypes = [_VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.oracle_mrope_cos_sin_3d.argtypes = [_VP, _VP, _VP, ctypes.c_int, ctypes.c_float]
        L.oracle_mrope_table.argtypes = [_VP, _VP, ctypes.c_int, ctypes.c_float]
        L.oracle_rope_rows.argtypes = [_VP, ctypes.c_int, _VP, _VP]
        L.oracle_qk_norm_rope.argtypes = [_VP, _VP, _VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_float]

    def prefill(self, q, k, v, Sk=None, scale=0.08838834764831843):
        Sq = q.shape[0]
        out = np.zeros_like(q)
        self.lib.oracle_attention_prefill(_p(q), _p(k), _p(v), _p(out), Sq, Sq if Sk is None else Sk,
                                          ctypes.c_float(scale))
        return out

    def chunked_prefill(self, q, cache_k, cache_v, pos_offset, scale=0.08838834764831843):
        """cache_k/cache_v: one layer, head-first [8, max_seq, 128]."""
        out = np.zeros_like(q)
        self.lib.oracle_attention_chunked_prefill(_p(q), _p(cache_k), _p(cache_v), cache_k.shape[1], _p(out),
                                                  q.shape[0], pos_offset, ctypes.c_float(scale))
        return out

    def decode(self, q, cache_k, cache_v, kv_len, scale=0.08838834764831843):
        """q [16,128]; cache_k/cache_v one layer [8, max_seq, 128]."""
        out = np.zeros((HQ, D), dtype=np.float32)
        self.lib.oracle_attention_decode(_p(q), _p(cache_k), _p(cache_v), cache_k.shape[1], _p(out), kv_len,
                                         ctypes.c_float(scale))
        return out

    def rmsnorm_rows(self, x, w, eps=EPS):
        x2 = np.ascontiguousarray(x.reshape(-1, x.shape[-1]))
        out = np.empty_like(x2)
        self.lib.oracle_rmsnorm_rows(_p(out), _p(x2), _p(w), x2.shape[0], x2.shape[1], ctypes.c_float(eps))
        return out.reshape(x.shape)

    def mrope_cos_sin_3d(self, pos_ids, theta=THETA):
        pos_ids = np.ascontiguousarray(pos_ids, dtype=np.int32)
        S = pos_ids.shape[1]
        c = np.empty((S, D // 2), dtype=np.float32)
        s = np.empty((S, D // 2), dtype=np.float32)
        self.lib.oracle_mrope_cos_sin_3d(_p(c), _p(s), _p(pos_ids), S, ctypes.c_float(theta))
        return c, s

    def mrope_table(self, max_seq, theta=THETA):
        c = np.empty((max_seq, D // 2), dtype=np.float32)
        s = np.empty((max_seq, D // 2), dtype=np.float32)
        self.lib.oracle_mrope_table(_p(c), _p(s), max_seq, ctypes.c_float(theta))
        return c, s

    def qk_norm_rope(self, q, k, q_norm, k_norm, cos, sin, eps=EPS):
        q2, k2 = q.copy(), k.copy()
        self.lib.oracle_qk_norm_rope(_p(q2), _p(k2), _p(q_norm), _p(k_norm), _p(cos), _p(sin), q.shape[0],
                                     ctypes.c_float(eps))
        return q2, k2

    def rope_rows(self, x, cos_row, sin_row):
        x2 = np.ascontiguousarray(x, dtype=np.float32).copy()
        heads = x2.size // D
        self.lib.oracle_rope_rows(_p(x2), heads, _p(np.ascontiguousarray(cos_row)), _p(np.ascontiguousarray(sin_row)))
        return x2


class RefLib:
    """The reference's own CPU code (kernel/attention.c, kv_cache.c, ops.c) built here."""

    @staticmethod
    def available(path=REF_LIB):
        return Path(path).exists()

    def __init__(self, path=REF_LIB):
        self.lib = ctypes.CDLL(str(path))
        L = self.lib
        L.attention_prefill_gqa.argtypes = [_VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                            _VP, _VP, _VP, _VP]
        L.attention_decode_gqa.argtypes = [_VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.attention_chunked_prefill_gqa.argtypes = [_VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                    ctypes.c_float]
        L.kv_cache_alloc.restype = _VP
        L.kv_cache_alloc.argtypes = [ctypes.c_int]
        L.kv_cache_free.argtypes = [_VP]
        L.kv_cache_append.argtypes = [_VP, ctypes.c_int, _VP, _VP]
        L.kv_cache_append_prefill.argtypes = [_VP, ctypes.c_int, _VP, _VP, ctypes.c_int]
        L.kv_cache_advance.argtypes = [_VP, ctypes.c_int]
        L.kv_cache_k.restype = _VP
        L.kv_cache_k.argtypes = [_VP, ctypes.c_int, ctypes.c_int]
        L.kv_cache_v.restype = _VP
        L.kv_cache_v.argtypes = [_VP, ctypes.c_int, ctypes.c_int]
        L.rmsnorm_seq_f32.argtypes = [_VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        L.mrope_build_cos_sin_3d.argtypes = [_VP, _VP, _VP, ctypes.c_int, ctypes.c_int, _VP, _VP]
        L.mrope_precompute.argtypes = [_VP, _VP, ctypes.c_int, ctypes.c_int, _VP, _VP]
        L.mrope_apply_seq_3d.argtypes = [_VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.mrope_apply.argtypes = [_VP, _VP, _VP, _VP, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        self._sections = (ctypes.c_int * 3)(24, 20, 20)
        self._theta = (ctypes.c_float * 3)(THETA, THETA, THETA)

    def prefill(self, q, k, v, Sk=None, scale=0.08838834764831843):
        Sq = q.shape[0]
        out = np.zeros_like(q)
        self.lib.attention_prefill_gqa(_p(q), _p(k), _p(v), _p(out), Sq, Sq if Sk is None else Sk,
                                       ctypes.c_float(scale), None, None, None, None)
        return out

    def _cache_with_rows(self, k_rows, v_rows, layer, max_seq):
        """A reference KVCache with token-major rows [n, 8, 128] at rows 0..n-1 of `layer`."""
        c = self.lib.kv_cache_alloc(max_seq)
        if not c:
            raise MemoryError("reference kv_cache_alloc failed")
        n = k_rows.shape[0]
        self.lib.kv_cache_append_prefill(c, layer, _p(k_rows), _p(v_rows), n)
        return c

    def decode(self, q, k_rows, v_rows, kv_len, layer=0, max_seq=None, scale=0.08838834764831843):
        """Attention of q [16,128] over token-major rows k_rows/v_rows [n,8,128] (n >= kv_len)."""
        max_seq = max_seq or k_rows.shape[0]
        c = self._cache_with_rows(k_rows, v_rows, layer, max_seq)
        try:
            out = np.zeros((HQ, D), dtype=np.float32)
            self.lib.attention_decode_gqa(_p(q), c, _p(out), layer, kv_len, ctypes.c_float(scale))
        finally:
            self.lib.kv_cache_free(c)
        return out

    def chunked_prefill(self, q, k_rows, v_rows, pos_offset, layer=0, scale=0.08838834764831843):
        """q [chunk,16,128] at positions pos_offset..; K/V rows 0..pos_offset+chunk-1 token-major."""
        c = self._cache_with_rows(k_rows, v_rows, layer, k_rows.shape[0])
        try:
            out = np.zeros_like(q)
            self.lib.attention_chunked_prefill_gqa(_p(q), c, _p(out), layer, q.shape[0], pos_offset,
                                                   ctypes.c_float(scale))
        finally:
            self.lib.kv_cache_free(c)
        return out

    def rmsnorm_rows(self, x, w, eps=EPS):
        x2 = np.ascontiguousarray(x.reshape(-1, x.shape[-1])).copy()
        self.lib.rmsnorm_seq_f32(_p(x2), _p(x2), _p(w), x2.shape[0], x2.shape[1], ctypes.c_float(eps))
        return x2.reshape(x.shape)

    def mrope_cos_sin_3d(self, pos_ids):
        pos_ids = np.ascontiguousarray(pos_ids, dtype=np.int32)
        S = pos_ids.shape[1]
        c = np.empty((S, D // 2), dtype=np.float32)
        s = np.empty((S, D // 2), dtype=np.float32)
        self.lib.mrope_build_cos_sin_3d(_p(c), _p(s), _p(pos_ids), S, D, self._sections, self._theta)
        return c, s

    def mrope_table(self, max_seq):
        c = np.empty((max_seq, D // 2), dtype=np.float32)
        s = np.empty((max_seq, D // 2), dtype=np.float32)
        self.lib.mrope_precompute(_p(c), _p(s), max_seq, D, self._sections, self._theta)
        return c, s

    def qk_norm_rope(self, q, k, q_norm, k_norm, cos, sin, eps=EPS):
        """kernel/decoder.c:73-87 for PREFILL_3D mode, through the reference's own ops."""
        S = q.shape[0]
        q2, k2 = q.copy(), k.copy()
        self.lib.rmsnorm_seq_f32(_p(q2), _p(q2), _p(q_norm), S * HQ, D, ctypes.c_float(eps))
        self.lib.rmsnorm_seq_f32(_p(k2), _p(k2), _p(k_norm), S * HKV, D, ctypes.c_float(eps))
        self.lib.mrope_apply_seq_3d(_p(q2), _p(k2), _p(cos), _p(sin), HQ, HKV, D, S)
        return q2, k2

    def rope_decode(self, q, k, cos_tab, sin_tab, pos):
        """kernel/decoder.c:79-83: one token at table position `pos`."""
        q2, k2 = np.ascontiguousarray(q).copy(), np.ascontiguousarray(k).copy()
        self.lib.mrope_apply(_p(q2), _p(k2), _p(cos_tab), _p(sin_tab), HQ, HKV, D, pos)
        return q2, k2


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
