"""CPU tests of the padding helpers (reference src/efficient_linear_assignment/utils.py)."""
import torch

import efficient_linear_assignment_b200 as ela


def test_get_pad_size():
    assert [ela.get_pad_size(n) for n in (8, 9, 15, 16, 1)] == [0, 7, 1, 0, 7]


def test_pad_input_blocks():
    c = torch.rand(2, 5, 11)
    p, shape = ela.pad_input(c)
    assert shape == (2, 5, 11) and p.shape == (2, 8, 16)
    assert torch.equal(p[:, :5, :11], c)
    assert (p[:, :5, 11:] == 1e9).all() and (p[:, 5:, :11] == 1e9).all()
    assert (p[:, 5:, 11:] == 0).all()


def test_pad_input_rows_only_keeps_large_cost():
    c = torch.rand(1, 5, 8)
    p, _ = ela.pad_input(c)
    assert p.shape == (1, 8, 8) and (p[:, 5:, :] == 1e9).all()


def test_no_padding_is_identity_and_unpad():
    c = torch.rand(1, 8, 16)
    p, shape = ela.pad_input(c)
    assert p is c
    idx = torch.arange(16).view(1, 16)
    assert torch.equal(ela.unpad_result(idx, (1, 5, 16)), idx[:, :5])


def test_pad_to_shape():
    t = torch.ones(2, 3)
    out = ela.pad_to_shape(t, (4, 5), value=-1.0)
    assert out.shape == (4, 5) and out[3, 4] == -1.0 and out[0, 0] == 1.0
