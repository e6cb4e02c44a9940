"""Host-side behaviour of the drop-in API (no GPU): constructors, errors,
weight layout, SparseConvTensor container semantics.  Mirrors the
reference's tests/test_tensor.py and the ctor checks of modules.py:46-51."""
import numpy as np
import pytest
import torch
import torch.nn as nn

import trispconv_b200.pytorch as spconv
from trispconv_b200.pytorch.indices import IndiceData, _output_spatial_shape, _to3
from trispconv_b200.pytorch.weight import normalize_spconv_weight
from trispconv_b200.testing.synthetic import generate_sparse_data, sparse_data_to_tensors


def make_sparse(B=1, N=8, C=4, D=8, H=8, W=8):
    coords = torch.randint(0, min(D, H, W), (N, 3), dtype=torch.int32)
    indices = torch.cat([torch.zeros(N, 1, dtype=torch.int32), coords], dim=1)
    return spconv.SparseConvTensor(torch.randn(N, C), indices, [D, H, W], B)


def test_exports():
    for name in ["SparseConvTensor", "SparseConvolution", "SubMConv3d", "SparseConv3d",
                 "SparseInverseConv3d", "SparseSequential", "SparseModule", "ConvAlgo"]:
        assert hasattr(spconv, name)
    assert [a.name for a in spconv.ConvAlgo] == ["Native", "MaskImplicitGemm", "MaskSplitImplicitGemm"]


def test_tensor_construction_and_replace():
    x = make_sparse()
    assert x.features.shape == (8, 4) and x.indices.shape == (8, 4)
    assert x.spatial_shape == [8, 8, 8] and x.batch_size == 1
    y = x.replace_feature(torch.ones(8, 4))
    assert y.indices is x.indices and y.indice_dict is x.indice_dict
    assert not torch.equal(x.features, y.features)
    with pytest.raises(AttributeError):
        x.features = torch.zeros(8, 4)
    assert x.find_indice_pair(None) is None and x.find_indice_pair("nope") is None


def test_tensor_asserts_int32():
    with pytest.raises(AssertionError):
        spconv.SparseConvTensor(torch.randn(3, 2), torch.zeros(3, 4, dtype=torch.int64), [4, 4, 4], 1)
    with pytest.raises(AssertionError):
        spconv.SparseConvTensor(torch.randn(3), torch.zeros(3, 4, dtype=torch.int32), [4, 4, 4], 1)


def test_dense_host_tensor_raises():
    """dense() runs on the GPU only (tsc_to_dense); CPU tensors are refused
    like at every other entry point, not scattered on the host."""
    x = make_sparse(B=2, N=10, C=3, D=4, H=5, W=6)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        x.dense()
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        x.dense(channels_first=False)


def test_ctor_errors():
    with pytest.raises(NotImplementedError):
        spconv.SparseConvolution(2, 4, 4, 3)
    with pytest.raises(NotImplementedError):
        spconv.SparseConvolution(3, 4, 4, 3, groups=2)
    with pytest.raises(NotImplementedError):
        spconv.SparseConvolution(3, 4, 4, 3, transposed=True)
    spconv.SparseConvolution(3, 4, 4, 3, transposed=True, inverse=True)


def test_module_parameters_krsc():
    m = spconv.SubMConv3d(4, 8, 3, stride=2, padding=1, indice_key="k", algo=spconv.ConvAlgo.Native)
    assert m.weight.shape == (8, 3, 3, 3, 4) and m.bias.shape == (8,)
    assert m.stride == (1, 1, 1) and m.padding == (0, 0, 0)
    s = spconv.SparseConv3d(4, 8, (3, 1, 1), stride=(2, 1, 1), bias=False)
    assert s.weight.shape == (8, 3, 1, 1, 4) and s.bias is None
    assert set(s.state_dict()) == {"weight"}
    inv = spconv.SparseInverseConv3d(8, 4, 3, indice_key="k")
    assert inv.inverse and not inv.subm
    # kaiming-uniform bound sqrt(6 / fan_in)
    bound = np.sqrt(6.0 / (27 * 4))
    assert float(m.weight.abs().max()) <= bound + 1e-6


def test_weight_normalizer():
    w = torch.randn(8, 3, 3, 3, 4)
    n = normalize_spconv_weight(w, (3, 3, 3), 4, 8)
    assert n.shape == (27, 4, 8)
    assert torch.equal(n, w.reshape(8, 27, 4).permute(1, 2, 0))
    w1 = torch.randn(6, 1, 1, 1, 5)
    n1 = normalize_spconv_weight(w1, (1, 1, 1), 5, 6)
    assert torch.equal(n1[0], w1.reshape(30).view(5, 6))  # spconv 1x1x1 quirk
    assert torch.equal(normalize_spconv_weight(w1.reshape(6, 5), (1, 1, 1), 5, 6), n1)
    assert normalize_spconv_weight(n, (3, 3, 3), 4, 8) is not None
    with pytest.raises(ValueError):
        normalize_spconv_weight(torch.randn(2, 2), (3, 3, 3), 4, 8)


def test_krsc_checkpoint_tensors_load_and_normalize():
    """KRSC checkpoint tensors of a decoder upsample block (the shapes of
    the reference's checkpoint test, tests/test_anigen_weights.py, drawn at
    random here) load into the modules by state_dict and normalise to
    (K, C_in, C_out), the 1x1x1 inverse conv through the flat quirk."""
    torch.manual_seed(3)
    blocks = {
        "inv3": (spconv.SparseInverseConv3d(768, 192, 3, indice_key="u0"), (192, 3, 3, 3, 768)),
        "subm3": (spconv.SubMConv3d(192, 192, 3), (192, 3, 3, 3, 192)),
        "inv1": (spconv.SparseInverseConv3d(768, 192, 1, indice_key="u1"), (192, 1, 1, 1, 768)),
    }
    for name, (m, shape) in blocks.items():
        assert tuple(m.weight.shape) == shape, name
        sd = {"weight": torch.randn(shape), "bias": torch.randn(192)}
        m.load_state_dict(sd)
        assert torch.equal(m.weight.data, sd["weight"]) and torch.equal(m.bias.data, sd["bias"])
        K = shape[1] * shape[2] * shape[3]
        n = normalize_spconv_weight(m.weight.data, shape[1:4], shape[4], shape[0])
        assert n.shape == (K, shape[4], shape[0]), name
    with pytest.raises(RuntimeError):  # a transposed (K, C_in, C_out) tensor is not a KRSC parameter
        blocks["subm3"][0].load_state_dict({"weight": torch.randn(27, 192, 192), "bias": torch.randn(192)})


def test_kernel_weight_views_match_normalizer():
    """The conv kernel reads the KRSC parameter in place; check that the
    layouts it is handed address exactly normalize_spconv_weight's values."""
    for ks in [(3, 3, 3), (1, 1, 1), (3, 1, 1), (2, 2, 2)]:
        m = spconv.SparseConv3d(5, 7, ks)
        K = int(np.prod(ks))
        w, layout = m._kernel_weight(K)
        ref = m._get_weight()
        if layout == 1:  # KRSC (Cout, K, Cin): element (k, c, n) = w[n, k, c]
            got = w.reshape(7, K, 5).permute(1, 2, 0)
        else:
            got = w.reshape(K, 5, 7)
        assert torch.equal(got, ref), ks
    m = spconv.SparseInverseConv3d(5, 7, 3)
    w, layout = m._kernel_weight(1)
    assert layout == 0 and torch.equal(w, m._get_weight()[:1])
    with pytest.raises(IndexError):
        spconv.SubMConv3d(5, 7, 1)._kernel_weight(27)


def test_helpers():
    assert _to3(3) == (3, 3, 3) and _to3([1, 2, 3]) == (1, 2, 3)
    assert _output_spatial_shape((8, 8, 8), (3, 3, 3), (2, 2, 2), (1, 1, 1), (1, 1, 1)) == (4, 4, 4)
    assert _output_spatial_shape((41, 1600, 1408), (3, 3, 3), (2, 2, 2), (1, 1, 1), (1, 1, 1)) == (21, 800, 704)


def test_indice_data_fields():
    d = IndiceData(torch.zeros(0, 4, dtype=torch.int32), [torch.zeros(0, dtype=torch.long)],
                   [torch.zeros(0, dtype=torch.long)], torch.zeros(1, dtype=torch.long),
                   torch.zeros(0, 4, dtype=torch.int32), (4, 4, 4), (4, 4, 4), (1, 1, 1), (1, 1, 1),
                   (0, 0, 0), (1, 1, 1), True)
    assert d.subm and d.kernel_size == (1, 1, 1) and len(d.pairs_in) == 1 and d.pair_num.shape == (1,)


def test_host_tensors_rejected():
    """No CPU fallback: the conv path refuses host tensors loudly."""
    x = make_sparse(C=4)
    with pytest.raises(RuntimeError, match="CUDA"):
        spconv.SubMConv3d(4, 4, 3)(x)
    with pytest.raises(RuntimeError, match="CUDA"):
        spconv.SparseSequential(spconv.SparseConv3d(4, 4, 3, stride=2), nn.ReLU())(x)


def test_generate_sparse_data_roundtrip():
    d = generate_sparse_data([5, 6, 7], [20, 30], 3, seed=1)
    f, dense, idx = sparse_data_to_tensors(d)
    assert idx.dtype == torch.int32 and idx.shape == (50, 4)
    assert torch.equal(dense[idx[:, 0].long(), :, idx[:, 1].long(), idx[:, 2].long(), idx[:, 3].long()], f)
    for b in range(2):
        sel = idx[idx[:, 0] == b]
        assert len(torch.unique(sel, dim=0)) == len(sel)


def test_sequential_dict_and_kwargs():
    seq = spconv.SparseSequential({"a": nn.ReLU(), "b": nn.Identity()})
    assert list(dict(seq.named_children())) == ["a", "b"]
    seq2 = spconv.SparseSequential(nn.ReLU(), extra=nn.Identity())
    assert list(dict(seq2.named_children())) == ["0", "extra"]
    x = make_sparse()
    y = spconv.SparseSequential(nn.ReLU())(x)
    assert (y.features >= 0).all() and y.indices is x.indices
