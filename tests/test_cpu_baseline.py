"""The timed CPU port of the reference's decode step (``oracle/cpu_baseline.py``): its pieces compute what
the oracle computes (so the timed work is the reference's arithmetic, not something cheaper), and both
timing entry points run whole steps at a small shape."""

import numpy as np
import torch

from oracle import attention as oatt
from oracle import linear as olin
from oracle import cpu_baseline as cb


def test_port_linear_is_dequantize_then_matmul():
    g = torch.Generator().manual_seed(0)
    q, s = cb._rand_codes(g, 48, 64)
    x = torch.randn((5, 64), generator=g)
    got = cb._qlinear(x, (q, s)).numpy()
    want = olin.i8_linear(x.numpy(), q.numpy(), s[:, 0].numpy())
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5)


def test_port_layer_attention_matches_oracle_sdpa():
    """One layer step: the attention inside it over the grown cache equals the oracle's decode SDPA."""
    layer = cb.LlamaLayerPort(64, 4, 2, 16, 96, batch=3, ctx=20)
    k0, v0 = layer.k.clone(), layer.v.clone()
    h = torch.randn((3, 64), generator=torch.Generator().manual_seed(1))
    B, D = 3, 16
    x = cb._rms(h, layer.n1, layer.eps)
    q = layer._rope(cb._qlinear(x, layer.wq).view(B, 1, 4, D).transpose(1, 2))
    k = layer._rope(cb._qlinear(x, layer.wk).view(B, 1, 2, D).transpose(1, 2))
    v = cb._qlinear(x, layer.wv).view(B, 1, 2, D).transpose(1, 2)
    kk, vv = torch.cat([k0, k], 2), torch.cat([v0, v], 2)
    att = torch.nn.functional.scaled_dot_product_attention(q, kk, vv, enable_gqa=True)
    for b in range(B):
        want = oatt.sdpa_decode(q[b, :, 0].numpy(), kk[b].numpy(), vv[b].numpy(),
                                1.0 / np.sqrt(D))
        np.testing.assert_allclose(att[b, :, 0].numpy(), want, rtol=1e-4, atol=1e-5)
    out = layer.step(h)
    assert out.shape == (3, 64) and torch.isfinite(out).all()
    assert layer.k.shape == k0.shape  # the cache length is held fixed across repeated samples


def test_port_timing_entry_points_run():
    r = cb.measure_steps(64, 4, 2, 16, 96, 200, layers=3, batch=2, ctx=20, budget_s=1.0, max_steps=2)
    assert 1 <= r["steps"] <= 2 and r["step_s"] > 0 and r["threads"] >= 1
    m = cb.measure(64, 4, 2, 16, 96, 200, layers=3, batch=2, ctx=20, budget_s=0.5)
    assert m["layers_timed"] >= 2 and m["step_s"] > 0
