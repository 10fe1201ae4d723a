"""End-to-end selections on B200: the PointNet++ SSG segmentation fixture of
gamzerA/mps-pointops (docs/parity/pointnet2-segmentation-*.npz, all 12
FPS / ball-query / three_nn selection arrays) and BASELINE config 1."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from mps_pointops import compat, knn
from mps_pointops.pointnet2 import three_nn

pytestmark = pytest.mark.gpu


def test_segmentation_fixture_selections(cuda_device):
    g = golden("pointnet2_segmentation")
    xyz = [torch.from_numpy(g["xyz"]).to(cuda_device)]
    sels = []
    for npoint, radius in [(1024, 0.1), (256, 0.2), (64, 0.4), (16, 0.8)]:
        s = compat.furthest_point_sample(xyz[-1], npoint)
        new = compat.gather_operation(xyz[-1].transpose(1, 2).contiguous(), s)
        new = new.transpose(1, 2).contiguous()
        sels += [s, compat.ball_query(radius, 32, xyz[-1], new)]
        xyz.append(new)
    for i in range(4):
        sels.append(three_nn(xyz[3 - i], xyz[4 - i])[1])
    keys = sorted(k for k in g if k.startswith("selection"))
    for key, got in zip(keys, sels):
        np.testing.assert_array_equal(got.cpu().numpy(), g[key], err_msg=key)


def test_config1_pipeline(cuda_device):
    c = golden("config1")
    xyz = torch.from_numpy(c["xyz"]).to(cuda_device)
    idx = compat.furthest_point_sample(xyz, 1024)
    np.testing.assert_array_equal(idx.cpu().numpy(), c["fps_idx"])
    centres = compat.gather_operation(xyz.transpose(1, 2).contiguous(), idx).transpose(1, 2)
    centres = centres.contiguous()
    np.testing.assert_array_equal(centres.cpu().numpy(), c["centres"])
    np.testing.assert_array_equal(compat.ball_query(0.2, 32, xyz, centres).cpu().numpy(),
                                  c["ball_query_idx"])
    d, i = knn(centres, xyz, 16)
    np.testing.assert_array_equal(i.cpu().numpy(), c["knn_idx"])
    np.testing.assert_allclose(d.cpu().numpy(), c["knn_dist"], rtol=1e-6, atol=0)
    d, i = three_nn(xyz, centres)
    np.testing.assert_array_equal(i.cpu().numpy(), c["three_nn_idx"])
    np.testing.assert_allclose(d.cpu().numpy(), c["three_nn_dist"], rtol=1e-6, atol=0)
