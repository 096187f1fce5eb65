"""Seeded synthetic workloads for the GQA attention path.

The reference publishes no dataset or benchmark suite for this path, so every input is
synthetic, with the shapes and value distributions the five benchmark configurations
name.  Random draws use numpy ``default_rng(seed)`` in a fixed order, stated per
function, so the same seed gives the same tensors everywhere.

Positions follow Qwen3-VL's multimodal RoPE indexing: vision tokens of an h x w merged
grid get (t, h, w) = (0, row, col) in row-major order; the text tokens after them get
sequential positions starting at max(previous) + 1, equal in all three sections.  (The
reference obtains these from HF ``get_rope_index``, decoder.py:405-416.)
"""

import numpy as np

NUM_Q_HEADS = 16
NUM_KV_HEADS = 8
HEAD_DIM = 128


def mrope_positions(grid_h: int, grid_w: int, n_text: int) -> np.ndarray:
    """int32 [3, grid_h*grid_w + n_text]: vision grid then sequential text positions."""
    n_vis = grid_h * grid_w
    pos = np.zeros((3, n_vis + n_text), dtype=np.int32)
    rows, cols = np.divmod(np.arange(n_vis, dtype=np.int32), grid_w)
    pos[0, :n_vis] = 0
    pos[1, :n_vis] = rows
    pos[2, :n_vis] = cols
    start = int(max(grid_h, grid_w)) if n_vis else 0  # max(t, h, w) + 1
    pos[:, n_vis:] = start + np.arange(n_text, dtype=np.int32)[None, :]
    return pos


def qkv(rng, S: int, sigma: float = 0.5):
    """q [S,16,128], k [S,8,128], v [S,8,128] fp32 ~ sigma * N(0,1), drawn q, k, v."""
    q = (sigma * rng.standard_normal((S, NUM_Q_HEADS, HEAD_DIM), dtype=np.float32)).astype(np.float32)
    k = (sigma * rng.standard_normal((S, NUM_KV_HEADS, HEAD_DIM), dtype=np.float32)).astype(np.float32)
    v = (sigma * rng.standard_normal((S, NUM_KV_HEADS, HEAD_DIM), dtype=np.float32)).astype(np.float32)
    return q, k, v


def norm_weights(rng):
    """q_norm, k_norm [128] fp32 ~ 1 + 0.02 * N(0,1), drawn q_norm then k_norm."""
    qn = (1.0 + 0.02 * rng.standard_normal(HEAD_DIM, dtype=np.float32)).astype(np.float32)
    kn = (1.0 + 0.02 * rng.standard_normal(HEAD_DIM, dtype=np.float32)).astype(np.float32)
    return qn, kn


def config1(seed: int = 0, n_decode: int = 256):
    """Config 1: one layer, 1,024-token prefill (768 vision tokens on a 24x32 grid + 256
    text tokens) then `n_decode` decode steps.  Draw order: Q, K, V, q_norm, k_norm, then
    per decode step q, k, v ([1,16,128], [1,8,128], [1,8,128])."""
    rng = np.random.default_rng(seed)
    pos = mrope_positions(24, 32, 256)
    S = pos.shape[1]
    q, k, v = qkv(rng, S)
    qn, kn = norm_weights(rng)
    steps = [qkv(rng, 1) for _ in range(n_decode)]
    return dict(q=q, k=k, v=v, q_norm=qn, k_norm=kn, pos=pos, decode=steps,
                rope_offset=int(pos.max()) + 1)


def config3_positions():
    """Config 3: 4,096 tokens = 3,600 vision tokens (60x60 grid) + 496 text tokens."""
    return mrope_positions(60, 60, 496)


def config5_positions():
    """Config 5: 32,768 tokens = 30,000 vision tokens (150x200 grid) + 2,768 text tokens."""
    return mrope_positions(150, 200, 2768)


def config4_kv_lens(n_seq: int = 512, seed: int = 0, lo: int = 1024, hi: int = 8192):
    """Config 4: ragged KV lengths ~ U[lo, hi] (inclusive), seeded."""
    rng = np.random.default_rng(seed)
    return rng.integers(lo, hi + 1, size=n_seq, dtype=np.int64).astype(np.int32)
