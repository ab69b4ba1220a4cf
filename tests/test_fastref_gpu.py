"""The fp-mode face (trixium_b200.fastref.HybridRef: matmul of an entry over X [T, cols], proj of
(role, layer) with the image's Hadamard rotation and K-segments; model/fastref.py:95-140) against the
reference's own HybridRef on the reference-made image tokens_hybrid_t5_kseg.img.gz
(tests/golden/fastref_hybrid_t5_kseg.npz): every output within 1e-3 of its row's scale (fp32 sums in
another order), for numpy and device inputs."""
import gzip
import os
import shutil

import numpy as np
import pytest
import torch

from conftest import GOLDEN, load

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.fixture(scope="module")
def ref(tmp_path_factory):
    from trixium_b200 import bons, fastref
    p = tmp_path_factory.mktemp("img") / "img"
    with gzip.open(os.path.join(GOLDEN, "tokens_hybrid_t5_kseg.img.gz"), "rb") as src, open(p, "wb") as dst:
        shutil.copyfileobj(src, dst)
    return fastref.HybridRef(bons.BONSImage(str(p)))


def _err(got, want):
    scale = np.maximum(np.abs(want).max(axis=1, keepdims=True), 1e-30)
    return float((np.abs(np.asarray(got, dtype=np.float64) - want) / scale).max())


def test_proj_and_matmul_match_reference(ref):
    d = load(os.path.join(GOLDEN, "fastref_hybrid_t5_kseg.npz"))
    assert ref.B > 0  # the image carries the rotated basis
    for i in range(int(d["n"])):
        role, l, X = int(d[f"proj{i}_role"]), int(d[f"proj{i}_layer"]), d[f"proj{i}_X"]
        assert _err(ref.proj(role, l, X), d[f"proj{i}_Y"]) < TOL, i
        e = ref.img.matvec_entries(role, l)[0]
        assert _err(ref.matmul(e, X), d[f"proj{i}_M"]) < TOL, i
        Yd = ref.proj(role, l, torch.from_numpy(X).cuda())
        assert Yd.is_cuda and _err(Yd.cpu().numpy(), d[f"proj{i}_Y"]) < TOL, i


def test_fp_rows_equal_single_row_launches(ref):
    """Rows of one launch equal the one-row entry (trx_matvec_fp) bit for bit, with and without the
    residual add."""
    from trixium_b200 import ops
    t = ref._tensor(ref.img.matvec_entries(11, 0)[0])
    rng = np.random.default_rng(3)
    X = torch.from_numpy(rng.standard_normal((9, t.cols)).astype(np.float32)).cuda()
    R = torch.from_numpy(rng.standard_normal((9, t.rows)).astype(np.float32)).cuda()
    Y = ops.matvec_fp_rows(ref.ctx, t, X).cpu().numpy()
    Yr = ops.matvec_fp_rows(ref.ctx, t, X, resid=R).cpu().numpy()
    for i in range(9):
        y1 = ops.matvec_fp(ref.ctx, t, X[i].contiguous()).cpu().numpy()
        assert np.array_equal(Y[i].view(np.uint32), y1.view(np.uint32)), i
        assert np.array_equal(Yr[i].view(np.uint32), (R[i].cpu().numpy() + y1).view(np.uint32)), i
