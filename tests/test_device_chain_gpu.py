"""One decode step of a small decoder kept on the device from end to end: per layer the Q/K/V
projections of the hidden state (torch GEMMs on the library stream) feed the decode call
directly, its [16][128] output stays on the device and is consumed by the O-projection GEMM plus
the residual (the handoff of kernel/decoder.c:121-124, with the projections standing in for the
reference's INT8 GEMMs), and the next layer's projections read that result -- no host
synchronisation between layers.  The decode kernels may start before their producer finishes
(programmatic dependent launch, L2 prefetch of q and of the new row before their dependency
wait), so this checks that every input is read after the kernel that wrote it.

Forms: attention_decode_append_fused_gqa (raw q/k, RMSNorm + M-RoPE in the decode kernel, BF16
cache) and attention_decode_append_gqa (q/k normalised and rotated by torch, FP32 cache).  The
final hidden state is compared with the same chain on the CPU (numpy GEMMs, the oracle's norm,
rotation and decode over the rows the cache holds) at the FP32 bar."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_helpers import TOL_MAX, TOL_REL, d2h, fill_layer, new_cache, vp
from oracle import max_abs, rel_l2

pytestmark = pytest.mark.gpu
SCALE = ctypes.c_float(0.08838834764831843)
EPS = 1e-6
LAYERS = 4
N0 = 1500  # rows already in the cache
HID = 2048


def _weights(rng):
    s = 1.0 / np.sqrt(HID)
    return [dict(wq=(s * rng.standard_normal((HID, 2048))).astype(np.float32),
                 wk=(s * rng.standard_normal((HID, 1024))).astype(np.float32),
                 wv=(s * rng.standard_normal((HID, 1024))).astype(np.float32),
                 wo=(s * rng.standard_normal((2048, HID))).astype(np.float32),
                 qn=(1 + 0.02 * rng.standard_normal(128)).astype(np.float32),
                 kn=(1 + 0.02 * rng.standard_normal(128)).astype(np.float32)) for _ in range(LAYERS)]


@pytest.mark.parametrize("form", ["fused_qk", "append"])
def test_device_resident_decode_chain(pkg, lib, oracle, form):
    torch.backends.cuda.matmul.allow_tf32 = False
    rng = np.random.default_rng(31 if form == "fused_qk" else 32)
    W = _weights(rng)
    dtype = pkg.ATTN_KV_BF16 if form == "fused_qk" else pkg.ATTN_KV_F32
    h = new_cache(pkg, lib, N0 + 4, dtype)
    cs = pkg.cache_struct(h)
    pos = N0 + 7  # the token's position (all three M-RoPE sections equal for text)
    cos, sin = oracle.mrope_table(pos + 1)
    cos_r, sin_r = np.ascontiguousarray(cos[pos]), np.ascontiguousarray(sin[pos])
    hid0 = rng.standard_normal(HID).astype(np.float32)
    stream = torch.cuda.Stream()
    lib.attn_set_stream(ctypes.c_void_p(stream.cuda_stream))
    try:
        for layer in range(LAYERS):
            k_old = rng.standard_normal((N0, 8, 128), dtype=np.float32)
            v_old = rng.standard_normal((N0, 8, 128), dtype=np.float32)
            fill_layer(pkg, lib, h, layer, k_old, v_old)
        cs.seq_len = N0
        torch.cuda.synchronize()
        dW = [{k: torch.from_numpy(v).cuda() for k, v in w.items()} for w in W]
        dcos, dsin = torch.from_numpy(cos_r).cuda(), torch.from_numpy(sin_r).cuda()
        with torch.cuda.stream(stream):
            hid = torch.from_numpy(hid0).cuda()
            for layer in range(LAYERS):
                w = dW[layer]
                q = (hid @ w["wq"]).view(16, 128)
                k = (hid @ w["wk"]).view(8, 128)
                v = (hid @ w["wv"]).view(8, 128)
                out = torch.empty((16, 128), device="cuda")
                if form == "fused_qk":
                    rc = lib.attention_decode_append_fused_gqa(vp(q), vp(k), vp(v), vp(w["qn"]), vp(w["kn"]), vp(dcos),
                                                               vp(dsin), h, vp(out), layer, SCALE, ctypes.c_float(EPS))
                else:
                    def norm_rope(x, wn):
                        y = x * torch.rsqrt((x * x).mean(-1, keepdim=True) + EPS) * wn
                        y1, y2 = y[:, :64], y[:, 64:]
                        return torch.cat([y1 * dcos - y2 * dsin, y2 * dcos + y1 * dsin], -1).contiguous()
                    # named, so they stay allocated until the call has queued its kernel
                    qr_d, kr_d, v_d = norm_rope(q, w["qn"]), norm_rope(k, w["kn"]), v.contiguous()
                    rc = lib.attention_decode_append_gqa(vp(qr_d), vp(kr_d), vp(v_d), h, vp(out), layer, SCALE)
                assert rc == 0, pkg.last_error(lib)
                hid = hid + out.view(-1) @ w["wo"]  # the O-projection reads the output on the device
        assert lib.attn_sync() == 0, pkg.last_error(lib)
        stream.synchronize()
        got = hid.cpu().numpy()
        # the rows the cache holds (the appended ones included), for the CPU chain
        rows = []
        for layer in range(LAYERS):
            if dtype == pkg.ATTN_KV_BF16:
                f = lambda p: (d2h(p, (8, N0 + 4, 128), np.uint16).astype(np.uint32) << 16).view(np.float32)  # noqa: E731
            else:
                f = lambda p: d2h(p, (8, N0 + 4, 128))  # noqa: E731
            rows.append((f(lib.kv_cache_k(h, layer, 0)), f(lib.kv_cache_v(h, layer, 0))))
    finally:
        lib.attn_set_stream(None)
        lib.kv_cache_free(h)
    hid = hid0.copy()
    for layer in range(LAYERS):
        w = W[layer]
        q = (hid @ w["wq"]).reshape(1, 16, 128).astype(np.float32)
        k = (hid @ w["wk"]).reshape(1, 8, 128).astype(np.float32)
        qr, _ = oracle.qk_norm_rope(q, k, w["qn"], w["kn"], cos_r[None], sin_r[None])
        kc, vc = rows[layer]
        att = oracle.decode(np.ascontiguousarray(qr[0]), kc, vc, N0 + 1)
        hid = hid + att.reshape(-1) @ w["wo"]
    print(f"{form}: max {max_abs(got, hid):.3e} rel {rel_l2(got, hid):.3e}; "
          f"attention part rel {rel_l2(got - hid0, hid - hid0):.3e}")
    assert max_abs(got, hid) <= TOL_MAX and rel_l2(got, hid) <= TOL_REL
    # the layers' contributions alone (a stale input would change them wholesale)
    assert rel_l2(got - hid0, hid - hid0) <= TOL_REL
