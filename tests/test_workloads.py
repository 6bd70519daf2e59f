"""The device-side shell generator (used for the 2.58M-voxel config-5b
volume) returns exactly the numpy generator's coordinates: same seeded draws,
same float64 operations, same lexicographic order."""
import numpy as np
import pytest
import torch

import workloads


@pytest.mark.parametrize("res,seed,thickness", [(64, 0, 1.5), (64, 7, 1.5), (96, 1, 1.5), (128, 3, 4.0)])
def test_shell_device_equals_numpy_on_cpu(res, seed, thickness):
    a = workloads.ellipsoid_shell(res, seed, thickness=thickness)
    b = workloads.ellipsoid_shell_device(res, seed, thickness=thickness, device="cpu")
    assert np.array_equal(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize("res,seed,thickness", [(64, 0, 1.5), (256, 0, 1.5), (256, 2, 4.0)])
def test_shell_device_equals_numpy_on_gpu(res, seed, thickness):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    a = workloads.ellipsoid_shell(res, seed, thickness=thickness)
    b = workloads.ellipsoid_shell_device(res, seed, thickness=thickness, device="cuda")
    assert np.array_equal(a, b)
