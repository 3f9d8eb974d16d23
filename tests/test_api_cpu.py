"""CPU tests of the host-side API logic (argument checks, registry)."""
import pytest
import torch

import efficient_linear_assignment_b200 as ela


def test_shape_multiple_of_8_is_enforced():
    with pytest.raises(ValueError, match="multiples of 8"):
        ela.linear_assignment(torch.rand(2, 10, 16))


def test_unknown_backend():
    with pytest.raises(ValueError, match="not available"):
        ela.linear_assignment(torch.rand(1, 8, 8), backend="nope")


def test_cpu_tensor_has_no_fallback():
    with pytest.raises(RuntimeError, match="CUDA"):
        ela.linear_assignment(torch.rand(1, 8, 8))


def test_registry_names():
    for name in ("b200", "cuda", "cpp", "torch"):
        assert ela.BACKENDS[name] is ela.AuctionB200


def test_epsilon_validation():
    with pytest.raises(ValueError):
        ela.solve(torch.rand(1, 8, 8), epsilon=0.0)
    with pytest.raises(ValueError):
        ela.solve(torch.rand(1, 8, 8), epsilon=[])
