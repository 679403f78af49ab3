"""Sinkhorn CUDA path vs the CPU oracle (and the reference's golden outputs)."""

import os

import numpy as np
import pytest
import torch

import oracle
from ascendc_kernel_b200 import sinkhorn as sk

pytestmark = pytest.mark.gpu

TOL = 2e-6  # fp32 op order mirrors the reference; exp may differ by an ulp


def test_golden_full_shape(golden_dir, cuda_device):
    g = np.load(os.path.join(golden_dir, "sinkhorn.npz"))
    x = torch.from_numpy(g["full_x"]).to(cuda_device)
    y = sk.ModelNew()(x).cpu().numpy()
    assert np.abs(y - g["full_y"]).max() < TOL
    assert np.abs(y - oracle.sinkhorn(g["full_x"])).max() < TOL


def test_golden_other_repeat_eps(golden_dir, cuda_device):
    g = np.load(os.path.join(golden_dir, "sinkhorn.npz"))
    x = torch.from_numpy(g["small_x"]).to(cuda_device)
    m = sk.ModelNew(int(g["small_repeat"]), float(g["small_eps"]))
    y = m(x).cpu().numpy()
    assert np.abs(y - g["small_y"]).max() < TOL


@pytest.mark.parametrize("shape", [(1, 1, 4, 4), (3, 37, 4, 4), (1, 100003, 4, 4)])
@pytest.mark.parametrize("repeat", [1, 10, 20])
def test_random_shapes_vs_oracle(cuda_device, shape, repeat):
    torch.manual_seed(repeat)
    x = torch.randn(*shape) * 4
    y = sk.sinkhorn(x.to(cuda_device), repeat, 1e-6).cpu().numpy()
    want = oracle.sinkhorn(x.numpy(), repeat, 1e-6)
    assert np.abs(y - want).max() < TOL * 4


def test_in_place_output(cuda_device):
    torch.manual_seed(0)
    x = torch.randn(1, 1024, 4, 4, device=cuda_device)
    want = sk.sinkhorn(x.clone())
    got = sk.sinkhorn(x, out=x)
    assert torch.equal(got, want)


def test_reference_interface(cuda_device):
    torch.manual_seed(42)
    m = sk.ModelNew(*sk.get_init_inputs())
    (x,) = sk.get_inputs()
    y = m(x.to(cuda_device))
    assert y.shape == x.shape and y.dtype == torch.float32
    # columns sum to ~1 after the final column normalisation
    assert torch.allclose(y.sum(-2), torch.ones_like(y.sum(-2)), atol=1e-4)
