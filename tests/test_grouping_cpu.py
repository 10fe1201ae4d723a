"""SA grouping on the host: the oracle pinned to the reference's own outputs
(tests/golden/grouping.npz: compat.gather_operation / grouping_operation and
the grouping of tests/test_pointnet2_e2e.py:40-44, with gradients), the
reference's torch path kept for CPU tensors, and argument checks."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from mps_pointops import compat, grouping
from oracle import oracle as O


def test_oracle_matches_reference_gather():
    c = golden("grouping")["gather"]
    got = O.group_points(c["features"], c["idx"][..., None])[..., 0]
    np.testing.assert_array_equal(got, c["out"])


@pytest.mark.parametrize("case", ["qg_r0.15", "qg_r0.4"])
def test_oracle_matches_reference_query_and_group(case):
    c = golden("grouping")[case]
    radius, nsample = float(c["meta"][0]), int(c["meta"][1])
    out, idx = O.query_and_group(c["xyz"], c["new_xyz"], c["features"], radius, nsample)
    np.testing.assert_array_equal(idx, c["idx"])
    np.testing.assert_array_equal(out, c["out"])
    gx, gq, gf = O.query_and_group_backward(c["grad_out"], idx, c["xyz"].shape[1])
    np.testing.assert_allclose(gx, c["grad_xyz"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(gq, c["grad_new_xyz"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(gf, c["grad_features"], rtol=1e-5, atol=1e-5)


def test_cpu_tensors_keep_the_reference_gather():
    # For CPU tensors (and dtypes other than float32) gather/grouping are the
    # reference's own torch gather, gradients included.
    c = golden("grouping")["qg_r0.4"]
    f = torch.from_numpy(c["features"]).requires_grad_()
    idx = torch.from_numpy(c["idx"])
    out = compat.grouping_operation(f, idx)
    np.testing.assert_array_equal(out.detach().numpy(), c["out"][:, 3:])
    out.backward(torch.from_numpy(c["grad_out"][:, 3:]))
    np.testing.assert_allclose(f.grad.numpy(), c["grad_features"], rtol=1e-5, atol=1e-5)
    g = golden("grouping")["gather"]
    got = compat.gather_operation(torch.from_numpy(g["features"]).double(),
                                  torch.from_numpy(g["idx"]))
    assert got.dtype == torch.float64
    np.testing.assert_array_equal(got.float().numpy(), g["out"])


def test_query_and_group_argument_checks():
    x = torch.rand(1, 10, 3)
    with pytest.raises(ValueError, match="Cannot have not features"):
        grouping.query_and_group(x, x[:, :2], None, 0.5, 4, use_xyz=False)
    with pytest.raises(ValueError, match="shapes"):
        grouping.query_and_group(x[..., :2], x[:, :2], None, 0.5, 4)
    with pytest.raises(ValueError, match="features must have shape"):
        grouping.query_and_group(x, x[:, :2], torch.rand(1, 4, 9), 0.5, 4)
    with pytest.raises(ValueError, match="radius"):
        grouping.query_and_group(x, x[:, :2], None, -1.0, 4)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        grouping.query_and_group(x, x[:, :2], None, 0.5, 4)
    with pytest.raises(ValueError, match="Cannot have not features"):
        grouping.QueryAndGroup(0.5, 4, use_xyz=False)(x, x[:, :2])


def test_group_all_matches_pointnet2_ops_layout():
    x = torch.rand(2, 7, 3)
    f = torch.rand(2, 4, 7)
    out = grouping.GroupAll()(x, None, f)
    assert out.shape == (2, 7, 1, 7)
    assert torch.equal(out[:, :3, 0], x.transpose(1, 2))
    assert torch.equal(out[:, 3:, 0], f)
    assert torch.equal(grouping.GroupAll(use_xyz=False)(x, None, f), f.unsqueeze(2))
    assert torch.equal(grouping.GroupAll()(x, None), x.transpose(1, 2).unsqueeze(2))
