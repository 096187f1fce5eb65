"""Regenerate the golden vectors in this folder from the REFERENCE's own code.

The reference (typhoon-ocr-server) ships no tests or golden vectors, so these are made
by running its kernel/attention.c, kernel/kv_cache.c and kernel/ops.c -- compiled
unmodified by oracle/Makefile into oracle/_ref/libref_attn.so -- on small seeded
inputs.  The chain mirrors kernel/decoder.c:73-117 for one layer: raw Q/K -> per-head
RMSNorm (q_norm/k_norm) -> M-RoPE (3-D positions) -> KV append -> attention.

Run from the repository root (needs the reference tree to build oracle/_ref):
    python tests/golden/make_golden.py
"""

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))

from oracle import RefLib  # noqa: E402

OUT = Path(__file__).resolve().parent
SEED = 20240501


def positions(n_vis_h, n_vis_w, n_text):
    n_vis = n_vis_h * n_vis_w
    pos = np.zeros((3, n_vis + n_text), dtype=np.int32)
    rows, cols = np.divmod(np.arange(n_vis, dtype=np.int32), n_vis_w)
    pos[1, :n_vis], pos[2, :n_vis] = rows, cols
    pos[:, n_vis:] = max(n_vis_h, n_vis_w) + np.arange(n_text, dtype=np.int32)
    return pos


def main():
    ref = RefLib()
    rng = np.random.default_rng(SEED)
    f32 = np.float32

    # 1. Pre-attention chain + prefill, S = 36 (one full 32-row tile and a ragged one).
    pos = positions(4, 6, 12)  # 24 vision tokens on a 4x6 grid, then 12 text tokens
    S = pos.shape[1]
    q_raw = (0.5 * rng.standard_normal((S, 16, 128))).astype(f32)
    k_raw = (0.5 * rng.standard_normal((S, 8, 128))).astype(f32)
    v = (0.5 * rng.standard_normal((S, 8, 128))).astype(f32)
    q_norm = (1 + 0.02 * rng.standard_normal(128)).astype(f32)
    k_norm = (1 + 0.02 * rng.standard_normal(128)).astype(f32)
    cos, sin = ref.mrope_cos_sin_3d(pos)
    q, k = ref.qk_norm_rope(q_raw, k_raw, q_norm, k_norm, cos, sin)
    out = ref.prefill(q, k, v)
    np.savez_compressed(OUT / "prefill_s36.npz", pos=pos, q_raw=q_raw, k_raw=k_raw, v=v, q_norm=q_norm,
                        k_norm=k_norm, cos=cos, sin=sin, q=q, k=k, out=out)

    # 2. Chunked prefill from the cache: 20 query tokens at positions 37..56 over 57 rows.
    off, chunk = 37, 20
    qc = rng.standard_normal((chunk, 16, 128)).astype(f32)
    kc = rng.standard_normal((off + chunk, 8, 128)).astype(f32)
    vc = rng.standard_normal((off + chunk, 8, 128)).astype(f32)
    outc = ref.chunked_prefill(qc, kc, vc, off)
    np.savez_compressed(OUT / "chunked_c20_off37.npz", q=qc, k_rows=kc, v_rows=vc, pos_offset=np.int32(off),
                        out=outc)

    # 3. Decode: one token over kv_len = 45 rows; decode-mode RoPE at table position 288.
    kv_len = 45
    qd_raw = (0.5 * rng.standard_normal((16, 128))).astype(f32)
    kd_raw = (0.5 * rng.standard_normal((8, 128))).astype(f32)
    kr = rng.standard_normal((kv_len, 8, 128)).astype(f32)
    vr = rng.standard_normal((kv_len, 8, 128)).astype(f32)
    cos_tab, sin_tab = ref.mrope_table(300)
    qd = ref.rmsnorm_rows(qd_raw, q_norm)
    kd = ref.rmsnorm_rows(kd_raw, k_norm)
    qd, kd = ref.rope_decode(qd, kd, cos_tab, sin_tab, 288)
    kr[kv_len - 1] = kd  # the appended row is the new token's normed, roped key
    outd = ref.decode(qd, kr, vr, kv_len)
    np.savez_compressed(OUT / "decode_kv45.npz", q_raw=qd_raw, k_raw=kd_raw, q_norm=q_norm, k_norm=k_norm,
                        rope_pos=np.int32(288), cos_row=cos_tab[288], sin_row=sin_tab[288], q=qd, k_new=kd,
                        k_rows=kr, v_rows=vr, out=outd)
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
