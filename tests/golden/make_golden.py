"""Generates the golden fixtures under tests/golden/ from the reference.

Run in a container where the reference (mrpulford/trispconv, pure Python)
is importable:

    python tests/golden/make_golden.py --reference /path/to/trispconv

Writes
  spconv_<tag>.npz     the reference's nine spconv-2.x golden fixtures
                       (tests/fixtures/spconv_golden_*.pt), converted to numpy
  ref_<case>.npz       small seeded cases run through the reference itself:
                       inputs, per-offset pair lists, out_indices, features
  ref_digests.json     SHA-256 digests of every kernel map (pair lists,
                       pair_num, out_indices) the reference builds for the
                       full-size benchmark configurations 1-5, so the GPU
                       tests can check bit-exactness at full size without
                       shipping the tables

The GPU box never runs this script; it only reads the files it wrote.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

from golden_util import kmap_digest  # noqa: E402


def _np(t):
    return t.detach().cpu().numpy() if hasattr(t, "detach") else np.asarray(t)


def convert_spconv_fixtures(ref_root: Path) -> None:
    import torch

    for p in sorted((ref_root / "tests" / "fixtures").glob("spconv_golden_*.pt")):
        fix = torch.load(p, map_location="cpu", weights_only=True)
        out = {}
        for k, v in fix.items():
            if v is None:
                out[k] = np.array([], dtype=np.float32)
                out[k + "__none"] = np.array(1)
            elif hasattr(v, "numpy"):
                out[k] = v.numpy()
            elif isinstance(v, str):
                out[k] = np.array(v)
            else:
                out[k] = np.asarray(v)
        tag = p.stem.replace("spconv_golden_", "")
        np.savez_compressed(HERE / f"spconv_{tag}.npz", **out)
        print("wrote", f"spconv_{tag}.npz")


def _pack_pairs(data):
    pin = [_np(p).astype(np.int64) for p in data.pairs_in]
    pout = [_np(p).astype(np.int64) for p in data.pairs_out]
    offsets = np.cumsum([0] + [len(p) for p in pin]).astype(np.int64)
    cat_in = np.concatenate(pin) if pin else np.empty(0, np.int64)
    cat_out = np.concatenate(pout) if pout else np.empty(0, np.int64)
    return cat_in, cat_out, offsets


SMALL_CASES = [
    # name, kind, batch, shape, n_per_sample, ksize, stride, padding, dilation, dup
    ("subm_k3", "subm", 2, (10, 11, 12), 120, 3, 1, 0, 1, False),
    ("subm_k3_d2", "subm", 1, (9, 9, 9), 150, 3, 1, 0, 2, False),
    ("subm_k1", "subm", 1, (8, 8, 8), 60, 1, 1, 0, 1, False),
    ("subm_k2", "subm", 2, (7, 8, 9), 90, 2, 1, 0, 1, False),
    ("subm_k311", "subm", 1, (6, 10, 10), 100, (3, 1, 1), 1, 0, 1, False),
    ("subm_dup", "subm", 1, (6, 6, 6), 80, 3, 1, 0, 1, True),
    ("strided_s2p1k3", "strided", 2, (12, 12, 12), 150, 3, 2, 1, 1, False),
    ("strided_s2p0k2", "strided", 2, (12, 13, 11), 150, 2, 2, 0, 1, False),
    ("strided_s1k2", "strided", 1, (9, 9, 9), 100, 2, 1, 0, 1, False),
    ("strided_s1k3d2", "strided", 1, (10, 10, 10), 120, 3, 1, 1, 2, False),
    ("strided_second4", "strided", 2, (11, 20, 18), 200, 3, 2, (0, 1, 1), 1, False),
    ("strided_k311s211", "strided", 2, (5, 12, 12), 150, (3, 1, 1), (2, 1, 1), 0, 1, False),
    ("strided_dup", "strided", 1, (8, 8, 8), 120, 3, 2, 1, 1, True),
    ("strided_sparse_p0", "strided", 1, (9, 9, 9), 5, 3, 2, 0, 1, False),
]


def _small_input(rng, batch, shape, n, dup):
    rows = []
    for b in range(batch):
        cells = rng.choice(int(np.prod(shape)), size=n, replace=dup)
        z, y, x = np.unravel_index(cells, shape)
        rows.append(np.stack([np.full(n, b), z, y, x], axis=1))
    idx = np.concatenate(rows).astype(np.int32)
    return idx[rng.permutation(len(idx))]


def small_cases() -> None:
    import torch
    from trispconv.pytorch import indices as R
    from trispconv.pytorch.functional import sparse_conv_forward
    from trispconv.pytorch.weight import normalize_spconv_weight

    rng = np.random.default_rng(20261201)
    for name, kind, B, shape, n, ks, st, pd, dl, dup in SMALL_CASES:
        idx = _small_input(rng, B, shape, n, dup)
        t_idx = torch.from_numpy(idx)
        if kind == "subm":
            data = R.generate_subm_indice_pairs(t_idx, shape, B, ks, dl)
        else:
            data = R.generate_strided_indice_pairs(t_idx, shape, B, ks, st, pd, dl)
        k3 = R._to3(ks)
        K = int(np.prod(k3))
        cin, cout = 8, 12
        feats = rng.standard_normal((len(idx), cin)).astype(np.float32)
        w = rng.standard_normal((cout, *k3, cin)).astype(np.float32) * 0.2
        bias = rng.standard_normal(cout).astype(np.float32) * 0.1
        wi = normalize_spconv_weight(torch.from_numpy(w), k3, cin, cout)
        n_out = len(data.out_indices)
        out = sparse_conv_forward(torch.from_numpy(feats), wi, torch.from_numpy(bias), data, n_out)
        cat_in, cat_out, offsets = _pack_pairs(data)
        rec = dict(kind=np.array(kind), batch=np.array(B), shape=np.array(shape), ksize=np.array(k3),
                   stride=np.array(R._to3(st)), padding=np.array(R._to3(pd)), dilation=np.array(R._to3(dl)),
                   indices=idx, features=feats, weight=w, bias=bias, out_indices=_np(data.out_indices),
                   pairs_in=cat_in, pairs_out=cat_out, offsets=offsets, pair_num=_np(data.pair_num),
                   out_features=_np(out), out_spatial_shape=np.array(data.output_spatial_shape))
        if kind == "strided":
            # inverse of this strided map, through the reference module
            import trispconv.pytorch as rsp

            down = rsp.SparseConv3d(cin, cout, ks, stride=st, padding=pd, dilation=dl, bias=False,
                                    indice_key="d")
            down.weight.data.copy_(torch.from_numpy(w))
            x = rsp.SparseConvTensor(torch.from_numpy(feats), t_idx, list(shape), B)
            y = down(x)
            up = rsp.SparseInverseConv3d(cout, cin, ks, bias=True, indice_key="d")
            w_up = rng.standard_normal((cin, *k3, cout)).astype(np.float32) * 0.2
            b_up = rng.standard_normal(cin).astype(np.float32) * 0.1
            up.weight.data.copy_(torch.from_numpy(w_up))
            up.bias.data.copy_(torch.from_numpy(b_up))
            inv_feats = rng.standard_normal((len(y.indices), cout)).astype(np.float32)
            z = up(y.replace_feature(torch.from_numpy(inv_feats)))
            rec.update(inv_weight=w_up, inv_bias=b_up, inv_features=inv_feats, inv_out_indices=_np(z.indices),
                       inv_out_features=_np(z.features), down_out_features=_np(y.features))
        np.savez_compressed(HERE / f"ref_{name}.npz", **rec)
        print("wrote", f"ref_{name}.npz", "pairs", int(data.pair_num.sum()), "n_out", n_out)


def _capture_network_kmaps(workload) -> list:
    """Runs the workload's layer list through the reference modules with
    1-channel features (kernel maps do not depend on features) and records
    the IndiceData every convolution uses, in layer order."""
    import torch
    import trispconv.pytorch as rsp
    import trispconv.pytorch.modules as rmod

    captured = []
    orig = rmod.sparse_conv_forward

    def spy(features, weight, bias, indice_data, n_out):
        captured.append(indice_data)
        return orig(features, weight, bias, indice_data, n_out)

    rmod.sparse_conv_forward = spy
    try:
        x = rsp.SparseConvTensor(torch.zeros(len(workload.indices), 1),
                                 torch.from_numpy(workload.indices), workload.spatial_shape,
                                 workload.batch_size)
        stack = []
        with torch.no_grad():
            for spec in workload.layers:
                t = spec["type"]
                if t == "push":
                    stack.append(x)
                    continue
                if t == "cat_pop":
                    stack.pop()
                    continue
                if t == "relu":
                    continue
                if t == "subm":
                    m = rsp.SubMConv3d(1, 1, spec["ksize"], dilation=spec["dilation"], bias=False,
                                       indice_key=spec["key"])
                elif t == "spconv":
                    m = rsp.SparseConv3d(1, 1, spec["ksize"], stride=spec["stride"], padding=spec["padding"],
                                         dilation=spec["dilation"], bias=False, indice_key=spec["key"])
                else:
                    m = rsp.SparseInverseConv3d(1, 1, spec["ksize"], bias=False, indice_key=spec["key"])
                x = m(x)
    finally:
        rmod.sparse_conv_forward = orig
    return captured


def config_digests() -> None:
    from trispconv_b200.testing import synthetic as syn

    out = {}
    for name, make in [("config1", syn.config1), ("config2", syn.config2), ("config3", syn.config3),
                       ("config4", syn.config4), ("config5", lambda: syn.config5(64))]:
        wl = make()
        datas = _capture_network_kmaps(wl)
        digests = []
        for d in datas:
            digests.append(dict(digest=kmap_digest(d.pairs_in, d.pairs_out, d.pair_num, _np(d.out_indices)),
                                n_out=int(len(d.out_indices)), pairs=int(d.pair_num.sum())))
        out[name] = dict(n_voxels=int(wl.n_voxels), layers=digests,
                         input_sha256=hashlib.sha256(wl.indices.tobytes()).hexdigest())
        print(name, wl.n_voxels, [(x["n_out"], x["pairs"]) for x in digests])
    (HERE / "ref_digests.json").write_text(json.dumps(out, indent=1))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="checkout of the reference (mrpulford/trispconv)")
    ap.add_argument("--skip-configs", action="store_true")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref))
    convert_spconv_fixtures(ref)
    small_cases()
    if not args.skip_configs:
        config_digests()


if __name__ == "__main__":
    main()
