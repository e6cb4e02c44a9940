"""Host side of the fused convolution epilogue (no GPU): which dense modules
after a sparse convolution SparseSequential folds into its store, and the
BatchNorm fold itself (reference: SparseSequential applies them to
x.features one by one, trispconv/pytorch/modules.py:320-329)."""
import torch
import torch.nn as nn

import trispconv_b200.pytorch as spconv
from trispconv_b200 import _lib as L
from trispconv_b200.pytorch import modules as M


def _bn(c, seed=0):
    g = torch.Generator().manual_seed(seed)
    bn = nn.BatchNorm1d(c, eps=1e-3)
    with torch.no_grad():
        bn.weight.copy_(torch.rand(c, generator=g) + 0.5)
        bn.bias.copy_(torch.randn(c, generator=g) * 0.1)
        bn.running_mean.copy_(torch.randn(c, generator=g) * 0.2)
        bn.running_var.copy_(torch.rand(c, generator=g) + 0.3)
    return bn.eval()


def test_fold_matches_batchnorm_of_conv_plus_bias():
    conv = spconv.SubMConv3d(8, 16, 3)
    with torch.no_grad():
        conv.bias.normal_()
    bn = _bn(16)
    scale, shift = M._fold_bn(bn, conv, torch.device("cpu"))
    acc = torch.randn(100, 16)
    want = bn(acc + conv.bias)
    torch.testing.assert_close(acc * scale + shift, want, rtol=1e-5, atol=1e-5)


def test_fusion_patterns():
    conv = spconv.SubMConv3d(8, 16, 3)
    cases = [
        ([conv, nn.ReLU()], 1, True),
        ([conv, _bn(16), nn.ReLU()], 2, L.ACT_RELU),
        ([conv, _bn(16)], 1, L.ACT_NONE),
        ([conv, nn.LeakyReLU(0.1)], 1, L.ACT_LEAKY_RELU),
        ([conv, _bn(16), nn.SiLU()], 2, L.ACT_SILU),
        ([conv, _bn(16).train(), nn.ReLU()], 0, False),   # batch statistics: not a fixed affine map
        ([conv, _bn(8)], 0, False),                       # wrong channel count
        ([conv, nn.Tanh()], 0, False),
        ([conv], 0, False),
    ]
    for mods, n, what in cases:
        seq = spconv.SparseSequential(*mods)
        got_n, post = seq._fusion(list(seq.children()), 0)
        assert got_n == n, mods
        if what is True or what is False:
            assert post is what, mods
        else:
            assert isinstance(post, M.Epilogue) and post.act == what, mods
    seq = spconv.SparseSequential(conv, nn.LeakyReLU(0.2))
    assert seq._fusion(list(seq.children()), 0)[1].alpha == 0.2
    # a BatchNorm that comes first in the chain is not after a conv: nothing fuses
    seq = spconv.SparseSequential(_bn(8), conv)
    assert seq._fusion(list(seq.children()), 0) == (0, False)


def test_fold_cache_follows_in_place_updates():
    conv = spconv.SubMConv3d(8, 16, 3)
    bn = _bn(16)
    seq = spconv.SparseSequential(conv, bn)
    mods = list(seq.children())
    _, e1 = seq._fusion(mods, 0)
    _, e2 = seq._fusion(mods, 0)
    assert e1.scale is e2.scale  # cached
    with torch.no_grad():
        bn.running_var.mul_(2.0)
    _, e3 = seq._fusion(mods, 0)
    assert e3.scale is not e1.scale
    torch.testing.assert_close(e3.scale, M._fold_bn(bn, conv, torch.device("cpu"))[0])
    assert not torch.allclose(e3.scale, e1.scale)
