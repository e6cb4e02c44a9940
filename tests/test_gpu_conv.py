"""Convolution parity on the GPU.

* spconv-2.x golden fixtures through the modules (the reference's
  tests/test_vs_spconv.py:51-145, same tolerance 1e-4),
* dense conv3d comparisons (the reference's tests/test_vs_dense.py cases,
  fp32 torch reference with TF32 off, 1e-4),
* fp16 / bf16 against the fp32 oracle (scale-relative 1e-2),
* SparseSequential ReLU fusion, hand-built IndiceData, duplicates.
"""
import numpy as np
import pytest
import torch
import torch.nn as nn

import oracle
import trispconv_b200.pytorch as spconv
from golden_util import fixture_value, load_npz, spconv_fixture_names
from gpu_util import assert_close_rel, np_
from trispconv_b200.pytorch.functional import sparse_conv_forward
from trispconv_b200.pytorch.indices import IndiceData
from trispconv_b200.testing.synthetic import generate_sparse_data, sparse_data_to_tensors

pytestmark = pytest.mark.gpu


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _sort_by_key(f, i, shape):
    enc = oracle.encode_coords(i, *shape)
    o = np.argsort(enc, kind="stable")
    return f[o], i[o]


@pytest.mark.parametrize("name", spconv_fixture_names())
def test_vs_spconv_golden(cuda, name):
    fix = load_npz(name)
    ct = str(fix["conv_type"])
    cin, cout, k = int(fixture_value(fix, "C_in")), int(fixture_value(fix, "C_out")), int(fixture_value(fix, "kernel_size"))
    s, p, d = (int(fixture_value(fix, n)) for n in ("stride", "padding", "dilation"))
    bias = fixture_value(fix, "bias")
    B = int(fixture_value(fix, "batch_size"))
    use_bias = bias is not None
    with torch.no_grad():
        if ct in ("subm", "strided"):
            m = (spconv.SubMConv3d(cin, cout, k, dilation=d, bias=use_bias) if ct == "subm" else
                 spconv.SparseConv3d(cin, cout, k, stride=s, padding=p, dilation=d, bias=use_bias)).to(cuda)
            m.weight.copy_(_t(fix["weight"], cuda))
            if use_bias:
                m.bias.copy_(_t(bias, cuda))
            x = spconv.SparseConvTensor(_t(fix["features"], cuda), _t(fix["indices"], cuda),
                                        [int(v) for v in fix["spatial_shape"]], B)
            y = m(x)
        else:
            down = spconv.SparseConv3d(int(fixture_value(fix, "down_C_in")), int(fixture_value(fix, "down_C_out")),
                                       k, stride=s, padding=p, bias=False, indice_key="down").to(cuda)
            down.weight.copy_(_t(fix["down_weight"], cuda))
            xd = spconv.SparseConvTensor(_t(fix["down_in_features"], cuda), _t(fix["down_in_indices"], cuda),
                                         [int(v) for v in fix["down_in_spatial_shape"]], B)
            x_down = down(xd)
            shp = list(x_down.spatial_shape)
            ref_sorted = np.argsort(oracle.encode_coords(fix["indices"], *shp), kind="stable")
            ours_sorted = np.argsort(oracle.encode_coords(np_(x_down.indices), *shp), kind="stable")
            perm = np.empty(len(ours_sorted), dtype=np.int64)
            perm[ours_sorted] = np.arange(len(ours_sorted))
            feats = fix["features"][ref_sorted][perm]
            m = spconv.SparseInverseConv3d(cin, cout, k, bias=use_bias, indice_key="down").to(cuda)
            m.weight.copy_(_t(fix["weight"], cuda))
            if use_bias:
                m.bias.copy_(_t(bias, cuda))
            y = m(spconv.SparseConvTensor(_t(feats, cuda), x_down.indices, shp, B, indice_dict=x_down.indice_dict))
    f, i = _sort_by_key(np_(y.features), np_(y.indices), y.spatial_shape)
    assert np.array_equal(i, fix["out_indices"])
    np.testing.assert_allclose(f, fix["out_features"], rtol=1e-4, atol=1e-4)


STRIDED_CASES = [pytest.param(bs, k, s, p, d, id=f"bs{bs}-k{k}-s{s}-p{p}-d{d}")
                 for bs in [1, 2] for k in [2, 3] for s in [1, 2] for p in [0, 1] for d in [1, 2]
                 if not (s > 1 and d > 1)]
SUBM_CASES = [pytest.param(bs, k, d, id=f"bs{bs}-k{k}-d{d}") for bs in [1, 2] for k in [1, 3] for d in [1, 2]]
SHAPE = [19, 18, 17]


@pytest.mark.parametrize("batch_size,ksize,stride,padding,dilation", STRIDED_CASES)
def test_sparseconv3d_vs_dense(cuda, batch_size, ksize, stride, padding, dilation):
    seed = 17 * batch_size + 5 * ksize + 3 * stride + 7 * padding + dilation
    f, dense, idx = sparse_data_to_tensors(generate_sparse_data(SHAPE, [300] * batch_size, 16, seed=seed), cuda)
    w = torch.from_numpy(np.random.default_rng(seed).uniform(-1, 1, (16, ksize, ksize, ksize, 16)).astype(np.float32))
    m = spconv.SparseConv3d(16, 16, ksize, stride=stride, padding=padding, dilation=dilation, bias=False).to(cuda)
    with torch.no_grad():
        m.weight.copy_(w)
    y = m(spconv.SparseConvTensor(f, idx, SHAPE, batch_size))
    ref = nn.functional.conv3d(dense, w.permute(0, 4, 1, 2, 3).to(cuda), stride=stride, padding=padding,
                               dilation=dilation)
    got = y.dense()
    assert got.shape == ref.shape
    o = y.indices.long()
    torch.testing.assert_close(got[o[:, 0], :, o[:, 1], o[:, 2], o[:, 3]],
                               ref[o[:, 0], :, o[:, 1], o[:, 2], o[:, 3]], rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("batch_size,ksize,dilation", SUBM_CASES)
def test_submconv3d_vs_dense(cuda, batch_size, ksize, dilation):
    seed = 31 * batch_size + 7 * ksize + dilation
    f, dense, idx = sparse_data_to_tensors(generate_sparse_data(SHAPE, [300] * batch_size, 16, seed=seed), cuda)
    w = torch.from_numpy(np.random.default_rng(seed).uniform(-1, 1, (16, ksize, ksize, ksize, 16)).astype(np.float32))
    m = spconv.SubMConv3d(16, 16, ksize, dilation=dilation, bias=False).to(cuda)
    with torch.no_grad():
        m.weight.copy_(w)
    y = m(spconv.SparseConvTensor(f, idx, SHAPE, batch_size))
    if ksize == 1:  # spconv 1x1x1: features @ weight.view(C_in, C_out)
        ref = f @ w.reshape(16 * 16).view(16, 16).to(cuda)
    else:
        pad = dilation * (ksize // 2)
        out = nn.functional.conv3d(dense, w.permute(0, 4, 1, 2, 3).to(cuda), padding=pad, dilation=dilation)
        i = idx.long()
        ref = out[i[:, 0], :, i[:, 1], i[:, 2], i[:, 3]]
    torch.testing.assert_close(y.features, ref, rtol=1e-4, atol=1e-4)
    assert torch.equal(y.indices, idx)


def test_strided_full_block_vs_dense(cuda):
    """reference tests/test_indices_strided.py:31-61 (all 10^3 voxels active)."""
    torch.manual_seed(10)
    z, y_, x_ = torch.meshgrid(torch.arange(10), torch.arange(10), torch.arange(10), indexing="ij")
    idx = torch.stack([torch.zeros(1000, dtype=torch.long), z.reshape(-1), y_.reshape(-1), x_.reshape(-1)], 1).int()
    f = torch.randn(1000, 4)
    w = torch.randn(8, 3, 3, 3, 4)
    b = torch.randn(8)
    m = spconv.SparseConv3d(4, 8, 3, stride=2, padding=1).to(cuda)
    with torch.no_grad():
        m.weight.copy_(w)
        m.bias.copy_(b)
    y = m(spconv.SparseConvTensor(f.to(cuda), idx.to(cuda), [10, 10, 10], 1))
    dense = torch.zeros(1, 4, 10, 10, 10)
    dense[0, :, idx[:, 1].long(), idx[:, 2].long(), idx[:, 3].long()] = f.t()
    ref = nn.functional.conv3d(dense, w.permute(0, 4, 1, 2, 3), b, stride=2, padding=1)
    o = y.indices.long().cpu()
    torch.testing.assert_close(y.features.cpu(), ref[o[:, 0], :, o[:, 1], o[:, 2], o[:, 3]], rtol=1e-4, atol=1e-4)
    assert y.spatial_shape == [5, 5, 5]


def test_inverse_restores_coords_and_key_errors(cuda):
    torch.manual_seed(13)
    coords = torch.randint(0, 8, (20, 3), dtype=torch.int32)
    idx = torch.cat([torch.zeros(20, 1, dtype=torch.int32), coords], 1).to(cuda)
    down = spconv.SparseConv3d(4, 8, 3, stride=2, padding=1, bias=False, indice_key="down1").to(cuda)
    up = spconv.SparseInverseConv3d(8, 4, 3, bias=False, indice_key="down1").to(cuda)
    x = spconv.SparseConvTensor(torch.randn(20, 4, device=cuda), idx, [8, 8, 8], 1)
    y = down(x)
    assert "down1" in y.indice_dict and y.spatial_shape == [4, 4, 4]
    z = up(y)
    # with duplicate coordinates every row still participates (k3 s2 p1)
    assert torch.equal(z.indices, x.indices) and z.spatial_shape == [8, 8, 8] and z.features.shape == (20, 4)
    with pytest.raises(KeyError):
        spconv.SparseInverseConv3d(4, 4, 3, indice_key="missing").to(cuda)(x)
    with pytest.raises(ValueError):
        spconv.SparseInverseConv3d(4, 4, 3).to(cuda)(x)


def test_inverse_1x1x1_quirk(cuda):
    """modules.py:162-173: a 1x1x1 forward makes the inverse a plain matmul in
    the inverse input's space."""
    idx = torch.tensor([[0, 2, 2, 2], [0, 0, 2, 4], [0, 4, 4, 0]], dtype=torch.int32, device=cuda)
    down = spconv.SparseConv3d(4, 6, 1, stride=2, bias=False, indice_key="k1").to(cuda)
    up = spconv.SparseInverseConv3d(6, 5, 1, indice_key="k1").to(cuda)
    y = down(spconv.SparseConvTensor(torch.randn(3, 4, device=cuda), idx, [6, 6, 6], 1))
    assert y.indices.shape == (3, 4)
    z = up(y)
    assert z.indices is y.indices and z.spatial_shape == y.spatial_shape
    ref = y.features @ up._get_weight()[0] + up.bias
    torch.testing.assert_close(z.features, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("cin,cout", [(4, 16), (16, 16), (32, 64), (64, 64), (96, 40), (128, 128)])
def test_low_precision_vs_fp32_oracle(cuda, dtype, cin, cout):
    rng = np.random.default_rng(cin * 131 + cout)
    shape = (24, 24, 24)
    n = 3000
    cells = rng.choice(np.prod(shape), n, replace=False)
    z, y, x = np.unravel_index(cells, shape)
    idx = np.stack([np.zeros(n), z, y, x], 1).astype(np.int32)
    f = rng.standard_normal((n, cin)).astype(np.float32)
    w = (rng.standard_normal((cout, 3, 3, 3, cin)) / np.sqrt(27 * cin)).astype(np.float32)
    b = rng.standard_normal(cout).astype(np.float32) * 0.1
    np_dt = np.float16 if dtype == torch.float16 else np.float32
    for kind in ("subm", "spconv"):
        spec = dict(type=kind, cin=cin, cout=cout, ksize=3, stride=2, padding=1, dilation=1, key=None,
                    weight=w, bias=b)
        m = (spconv.SubMConv3d(cin, cout, 3) if kind == "subm" else
             spconv.SparseConv3d(cin, cout, 3, stride=2, padding=1)).to(cuda)
        with torch.no_grad():
            m.weight.copy_(torch.from_numpy(w))
            m.bias.copy_(torch.from_numpy(b))
        m = m.to(dtype)
        xt = spconv.SparseConvTensor(torch.from_numpy(f).to(cuda, dtype), torch.from_numpy(idx).to(cuda), shape, 1)
        yt = m(xt)
        assert yt.features.dtype == dtype
        ref = oracle.network.conv_layer(oracle.network.OracleTensor(f.astype(np_dt).astype(np.float32), idx, shape, 1), spec)
        assert np.array_equal(np_(yt.indices), ref.indices)
        assert_close_rel(np_(yt.features.float()), ref.features, 1e-2, f"{kind} {dtype}", dtype=dtype)


def test_sequential_relu_fusion_matches_unfused(cuda, monkeypatch):
    import trispconv_b200.pytorch.modules as M

    rng = np.random.default_rng(9)
    f, _, idx = sparse_data_to_tensors(generate_sparse_data([12, 12, 12], [200, 150], 8, seed=3), cuda)
    seq = spconv.SparseSequential(spconv.SubMConv3d(8, 16, 3, indice_key="a"), nn.ReLU(),
                                  spconv.SparseConv3d(16, 8, 3, stride=2, padding=1), nn.ReLU(inplace=True),
                                  nn.BatchNorm1d(8), nn.ReLU()).to(cuda).eval()
    x = spconv.SparseConvTensor(f, idx, [12, 12, 12], 2)
    fused = seq(x)
    monkeypatch.setattr(M, "FUSE_RELU", False)
    unfused = seq(spconv.SparseConvTensor(f, idx, [12, 12, 12], 2))
    assert torch.equal(fused.indices, unfused.indices)
    torch.testing.assert_close(fused.features, unfused.features, rtol=0, atol=0)
    assert (fused.features >= 0).all()
    del rng


def test_hand_built_indice_data(cuda):
    """IndiceData assembled from explicit pair lists (no device map)."""
    rng = np.random.default_rng(11)
    idx = np.unique(rng.integers(0, 6, (60, 3)), axis=0)
    idx = np.concatenate([np.zeros((len(idx), 1), int), idx], 1).astype(np.int32)
    ref = oracle.subm_pairs(idx, (6, 6, 6), 1, 3)
    dev_pairs_in = [torch.from_numpy(p).to(cuda) for p in ref.pairs_in]
    dev_pairs_out = [torch.from_numpy(p).to(cuda) for p in ref.pairs_out]
    it = torch.from_numpy(idx).to(cuda)
    d = IndiceData(it, dev_pairs_in, dev_pairs_out, torch.from_numpy(ref.pair_num), it, (6, 6, 6), (6, 6, 6),
                   (3, 3, 3), (1, 1, 1), (0, 0, 0), (1, 1, 1), True)
    f = rng.standard_normal((len(idx), 5)).astype(np.float32)
    w = rng.standard_normal((27, 5, 7)).astype(np.float32)
    out = sparse_conv_forward(torch.from_numpy(f).to(cuda), torch.from_numpy(w).to(cuda), None, d, len(idx))
    exp = oracle.conv_forward(f, w, None, ref.pairs_in, ref.pairs_out, len(idx))
    np.testing.assert_allclose(np_(out), exp, rtol=1e-4, atol=1e-4)
    # repeated output ids inside one offset accumulate like index_add_
    d2 = IndiceData(it, [torch.tensor([0, 1], device=cuda)], [torch.tensor([2, 2], device=cuda)],
                    torch.tensor([2]), it, (6, 6, 6), (6, 6, 6), (1, 1, 1), (1, 1, 1), (0, 0, 0), (1, 1, 1), True)
    out2 = sparse_conv_forward(torch.from_numpy(f).to(cuda), torch.from_numpy(w[:1]).to(cuda), None, d2, 3)
    np.testing.assert_allclose(np_(out2)[2], (f[0] + f[1]) @ w[0], rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(np_(out2)[:2], 0, atol=0)


def test_duplicate_coordinates_strided_conv(cuda):
    """Duplicate input coordinates: every duplicate contributes (index_add_
    semantics), handled by the overflow list of the gather map."""
    rng = np.random.default_rng(12)
    base = rng.integers(0, 8, (50, 3))
    idx = np.concatenate([base, base[:20], base[:5]])
    idx = np.concatenate([np.zeros((len(idx), 1), int), idx], 1).astype(np.int32)
    idx = idx[rng.permutation(len(idx))]
    f = rng.standard_normal((len(idx), 6)).astype(np.float32)
    w = (rng.standard_normal((9, 3, 3, 3, 6)) * 0.3).astype(np.float32)
    spec = dict(type="spconv", cin=6, cout=9, ksize=3, stride=2, padding=1, dilation=1, key=None, weight=w, bias=None)
    ref = oracle.network.conv_layer(oracle.network.OracleTensor(f, idx, (8, 8, 8), 1), spec)
    m = spconv.SparseConv3d(6, 9, 3, stride=2, padding=1, bias=False).to(cuda)
    with torch.no_grad():
        m.weight.copy_(torch.from_numpy(w))
    y = m(spconv.SparseConvTensor(torch.from_numpy(f).to(cuda), torch.from_numpy(idx).to(cuda), [8, 8, 8], 1))
    assert np.array_equal(np_(y.indices), ref.indices)
    np.testing.assert_allclose(np_(y.features), ref.features, rtol=1e-4, atol=1e-4)


def test_dense_matches_host_scatter(cuda):
    f, dense, idx = sparse_data_to_tensors(generate_sparse_data([5, 6, 7], [20, 30], 3, seed=2), cuda)
    x = spconv.SparseConvTensor(f, idx, [5, 6, 7], 2)
    torch.testing.assert_close(x.dense(), dense, rtol=0, atol=0)
    torch.testing.assert_close(x.dense(channels_first=False), dense.permute(0, 2, 3, 4, 1), rtol=0, atol=0)
    bad = idx.clone()
    bad[0, 2] = 99
    with pytest.raises(AssertionError):
        spconv.SparseConvTensor(f, bad, [5, 6, 7], 2).dense()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("cin,cout,ks", [(4, 16, 3), (12, 8, 3), (16, 32, 3), (32, 32, 2), (64, 64, 3),
                                         (96, 136, 3), (128, 256, 3), (64, 24, 1), (20, 16, 3)])
def test_tensor_core_matches_cuda_core_kernel(cuda, dtype, cin, cout, ks):
    """Same inputs through the mma.sync kernel and the fp32-FFMA kernel
    (TRISPCONV_B200_FORCE_SIMT path): both accumulate in fp32, so they agree
    to within fp32 summation-order differences before the final rounding."""
    from trispconv_b200.pytorch import functional as Fn

    rng = np.random.default_rng(cin + 7 * cout + ks)
    shape = (20, 20, 20)
    n = 2500
    cells = rng.choice(np.prod(shape), n, replace=False)
    z, y, x = np.unravel_index(cells, shape)
    idx = torch.from_numpy(np.stack([np.zeros(n), z, y, x], 1).astype(np.int32)).to(cuda)
    f = torch.from_numpy(rng.standard_normal((n, cin)).astype(np.float32)).to(cuda, dtype)
    for kind in ("subm", "spconv"):
        m = (spconv.SubMConv3d(cin, cout, ks) if kind == "subm" else
             spconv.SparseConv3d(cin, cout, ks, stride=2, padding=1)).to(cuda, dtype)
        x_ = spconv.SparseConvTensor(f, idx, shape, 1)
        a = m(x_)
        Fn.set_force_simt(True)
        try:
            b = m(spconv.SparseConvTensor(f, idx, shape, 1))
        finally:
            Fn.set_force_simt(False)
        assert torch.equal(a.indices, b.indices)
        scale = b.features.float().abs().max().item()
        err = (a.features.float() - b.features.float()).abs().max().item()
        ulp = 2 ** -7 if dtype == torch.bfloat16 else 2 ** -10
        assert err <= 2 * ulp * max(scale, 1e-3), (kind, err, scale)


@pytest.mark.parametrize("cin,cout", [(4, 16), (16, 16), (16, 32), (32, 32), (32, 64), (8, 24)])
def test_mma_resident_weights_match_streamed_weights(cuda, cin, cout):
    """The persistent mma.sync kernel with resident weights gives the same
    bits as the kernel that streams the weights per tile."""
    from trispconv_b200 import _lib as L
    from trispconv_b200.pytorch.indices import generate_subm_indice_pairs

    rng = np.random.default_rng(cin * 100 + cout)
    shape = (40, 80, 80)
    n = 60_000
    cells = rng.choice(int(np.prod(shape)), n, replace=False)
    z, y, x = np.unravel_index(cells, shape)
    idx = torch.from_numpy(np.stack([np.zeros(n), z, y, x], 1).astype(np.int32)).to(cuda)
    km = generate_subm_indice_pairs(idx, shape, 1, 3)._kmap
    f = torch.from_numpy(rng.standard_normal((n, cin)).astype(np.float32)).to(cuda).half()
    w = (torch.randn(cout, 3, 3, 3, cin, device=cuda) * 0.1).half()
    b = torch.randn(cout, device=cuda).half()
    outs = []
    for extra in (L.CONV_NO_RG, L.CONV_NO_RG | L.CONV_NO_RESIDENT_W):
        out = torch.empty(n, cout, dtype=torch.half, device=cuda)
        rc = L.load().tsc_conv_forward(f.data_ptr(), L.DTYPE_CODE[torch.float16], n, cin, w.data_ptr(), L.W_KRSC,
                                       b.data_ptr(), km.gather.data_ptr(), None, 27, n, cout, None, 0,
                                       km.meta.data_ptr(), out.data_ptr(), L.CONV_RELU | extra,
                                       L.status_word(cuda).data_ptr(), None, L.stream_ptr(cuda))
        L.check(rc, "tsc_conv_forward")
        outs.append(out)
    torch.cuda.synchronize()
    L.check_device_status(cuda)
    assert torch.equal(outs[0], outs[1])
