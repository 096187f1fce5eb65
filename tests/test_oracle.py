"""The oracle is pinned before it is trusted (CPU only).

1. The C restatement reproduces every golden vector; those were produced by the
   reference's own kernel/attention.c, kv_cache.c and ops.c (tests/golden/make_golden.py).
2. Where the reference build is present (oracle/_ref), restatement and reference agree
   exactly on seeded inputs across the edge cases the reference's loops have: one
   token, tile boundaries (32 query rows, 256 key columns), ragged tails, Sk < Sq,
   decode at kv_len 1, chunked prefill with offsets.
"""

import numpy as np
import pytest

from oracle import max_abs

TOL = 1e-6  # same algorithm, same flags: expected bit-exact; this allows libm drift


def test_golden_prefill_chain(oracle, golden):
    g = golden("prefill_s36.npz")
    cos, sin = oracle.mrope_cos_sin_3d(g["pos"])
    assert max_abs(cos, g["cos"]) <= TOL and max_abs(sin, g["sin"]) <= TOL
    q, k = oracle.qk_norm_rope(g["q_raw"], g["k_raw"], g["q_norm"], g["k_norm"], g["cos"], g["sin"])
    assert max_abs(q, g["q"]) <= TOL and max_abs(k, g["k"]) <= TOL
    out = oracle.prefill(g["q"], g["k"], g["v"])
    assert max_abs(out, g["out"]) <= TOL


def test_golden_chunked(oracle, golden):
    g = golden("chunked_c20_off37.npz")
    ck = np.ascontiguousarray(g["k_rows"].transpose(1, 0, 2))
    cv = np.ascontiguousarray(g["v_rows"].transpose(1, 0, 2))
    out = oracle.chunked_prefill(g["q"], ck, cv, int(g["pos_offset"]))
    assert max_abs(out, g["out"]) <= TOL


def test_golden_decode(oracle, golden):
    g = golden("decode_kv45.npz")
    qn = oracle.rmsnorm_rows(g["q_raw"], g["q_norm"])
    kn = oracle.rmsnorm_rows(g["k_raw"], g["k_norm"])
    q = oracle.rope_rows(qn, g["cos_row"], g["sin_row"])
    k = oracle.rope_rows(kn, g["cos_row"], g["sin_row"])
    assert max_abs(q, g["q"]) <= TOL and max_abs(k, g["k_new"]) <= TOL
    ct, st = oracle.mrope_table(int(g["rope_pos"]) + 1)
    assert max_abs(ct[-1], g["cos_row"]) <= TOL and max_abs(st[-1], g["sin_row"]) <= TOL
    ck = np.ascontiguousarray(g["k_rows"].transpose(1, 0, 2))
    cv = np.ascontiguousarray(g["v_rows"].transpose(1, 0, 2))
    out = oracle.decode(g["q"], ck, cv, g["k_rows"].shape[0])
    assert max_abs(out, g["out"]) <= TOL


@pytest.mark.parametrize("S,Sk", [(1, 1), (2, 2), (31, 31), (32, 32), (33, 33), (255, 255), (257, 257),
                                  (300, 300), (40, 20), (64, 100)])
def test_prefill_matches_reference(oracle, ref, S, Sk):
    rng = np.random.default_rng(S * 7 + Sk)
    q = rng.standard_normal((S, 16, 128), dtype=np.float32)
    n = max(S, Sk)
    k = rng.standard_normal((n, 8, 128), dtype=np.float32)
    v = rng.standard_normal((n, 8, 128), dtype=np.float32)
    assert max_abs(oracle.prefill(q, k, v, Sk), ref.prefill(q, k, v, Sk)) <= TOL


@pytest.mark.parametrize("kv_len", [1, 2, 17, 256, 257, 1500])
def test_decode_matches_reference(oracle, ref, kv_len):
    rng = np.random.default_rng(kv_len)
    q = rng.standard_normal((16, 128), dtype=np.float32)
    k = rng.standard_normal((kv_len + 3, 8, 128), dtype=np.float32)
    v = rng.standard_normal((kv_len + 3, 8, 128), dtype=np.float32)
    ck = np.ascontiguousarray(k.transpose(1, 0, 2))
    cv = np.ascontiguousarray(v.transpose(1, 0, 2))
    assert max_abs(oracle.decode(q, ck, cv, kv_len), ref.decode(q, k, v, kv_len)) <= TOL


@pytest.mark.parametrize("chunk,off", [(1, 0), (1, 99), (32, 0), (33, 256), (70, 31)])
def test_chunked_matches_reference(oracle, ref, chunk, off):
    rng = np.random.default_rng(chunk * 1000 + off)
    n = off + chunk
    q = rng.standard_normal((chunk, 16, 128), dtype=np.float32)
    k = rng.standard_normal((n, 8, 128), dtype=np.float32)
    v = rng.standard_normal((n, 8, 128), dtype=np.float32)
    ck = np.ascontiguousarray(k.transpose(1, 0, 2))
    cv = np.ascontiguousarray(v.transpose(1, 0, 2))
    assert max_abs(oracle.chunked_prefill(q, ck, cv, off), ref.chunked_prefill(q, k, v, off)) <= TOL


def test_norm_rope_matches_reference(oracle, ref, pkg):
    import importlib
    wl = importlib.import_module(pkg.__name__ + ".workloads")
    pos = wl.mrope_positions(5, 7, 9)
    rng = np.random.default_rng(3)
    q, k, _ = wl.qkv(rng, pos.shape[1])
    qn, kn = wl.norm_weights(rng)
    c1, s1 = oracle.mrope_cos_sin_3d(pos)
    c2, s2 = ref.mrope_cos_sin_3d(pos)
    assert max_abs(c1, c2) <= TOL and max_abs(s1, s2) <= TOL
    a = oracle.qk_norm_rope(q, k, qn, kn, c1, s1)
    b = ref.qk_norm_rope(q, k, qn, kn, c2, s2)
    assert max_abs(a[0], b[0]) <= TOL and max_abs(a[1], b[1]) <= TOL


def test_planted_mistake_is_caught(oracle, golden):
    """A checker that cannot fail proves nothing: perturb one input element on the CPU
    and the oracle's output must leave the golden tolerance."""
    g = golden("prefill_s36.npz")
    q = g["q"].copy()
    q[5, 3, 7] += 0.5
    assert max_abs(oracle.prefill(q, g["k"], g["v"]), g["out"]) > 1e-3
