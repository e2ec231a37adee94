"""Fused ReLU + dropout of the GCN hidden layer (tcc_relu_dropout_forward /
_backward) against a numpy restatement of the same counter-based draw: the
kept elements, the outputs and the gradients are bit-exact."""
import ctypes as C

import numpy as np
import pytest
import torch

from tcc_b200 import _lib as L
from tcc_b200 import gcn

pytestmark = pytest.mark.gpu

M64 = np.uint64(0xFFFFFFFFFFFFFFFF)


def kept(seed, n, p):
    """keep(seed, i): SplitMix64 finaliser of seed + (i + 1) * golden, top 32
    bits >= ceil(p * 2^32) (numpy uint64 arithmetic wraps like the device)."""
    with np.errstate(over="ignore"):
        i = np.arange(n, dtype=np.uint64)
        z = np.uint64(seed) + (i + np.uint64(1)) * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    thresh = min(int(np.ceil(p * 4294967296.0)), 0xFFFFFFFF)
    return (z >> np.uint64(32)) >= np.uint64(thresh)


@pytest.mark.parametrize("p", [0.5, 0.1, 0.0])
def test_relu_dropout_matches_restatement(gpu, p):
    n = 1 << 20
    gen = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(n, generator=gen, device="cuda")
    seed = 123456789
    out = torch.empty_like(x)
    st = L.lib().tcc_relu_dropout_forward(C.c_void_p(x.data_ptr()), C.c_void_p(out.data_ptr()),
                                          n, p, seed, None)
    assert st == L.TCC_OK
    xh = x.cpu().numpy()
    k = kept(seed, n, p)
    scale = np.float32(1.0) / (np.float32(1.0) - np.float32(p))  # as the device computes it
    want = np.where((xh > 0) & k, xh * scale, np.float32(0)).astype(np.float32)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    if p > 0:
        assert abs(k.mean() - (1 - p)) < 0.005
    g = torch.randn(n, generator=gen, device="cuda")
    gi = torch.empty_like(g)
    st = L.lib().tcc_relu_dropout_backward(C.c_void_p(g.data_ptr()), C.c_void_p(out.data_ptr()),
                                           C.c_void_p(gi.data_ptr()), n, p, None)
    assert st == L.TCC_OK
    gw = np.where(want > 0, g.cpu().numpy() * scale, np.float32(0)).astype(np.float32)
    np.testing.assert_array_equal(gi.cpu().numpy(), gw)


def test_relu_dropout_autograd(gpu):
    gen = torch.Generator(device="cuda").manual_seed(6)
    x = torch.randn((1000, 256), generator=gen, device="cuda", requires_grad=True)
    y = gcn.relu_dropout(x, 0.5, seed=42)
    y2 = gcn.relu_dropout(x, 0.5, seed=42)
    assert torch.equal(y, y2)  # the draw depends only on (seed, index)
    y3 = gcn.relu_dropout(x, 0.5, seed=43)
    assert not torch.equal(y, y3)
    w = torch.randn((1000, 256), generator=gen, device="cuda")
    (y * w).sum().backward()
    mask = (y.detach() > 0).float()
    assert torch.equal(x.grad, w * mask * 2.0)
    assert torch.equal(gcn.relu_dropout(x, 0.5, 1, training=False), torch.relu(x))
