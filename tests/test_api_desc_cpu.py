"""The lean call path packs st_tensor / st_exec descriptors with struct; its
bytes must be exactly those of the ctypes structures the C ABI declares."""
import ctypes

import pytest
import torch

from sptiles_b200 import _native as N
from sptiles_b200 import api


@pytest.mark.parametrize("make", [
    lambda: torch.randn(3, 5),
    lambda: torch.randn(3, 5)[:, 1:4],
    lambda: torch.randn(6, 4).t(),
    lambda: torch.randn(9),
    lambda: torch.randn(9)[::3],
    lambda: torch.empty(0, 4),
    lambda: torch.empty(0),
    lambda: torch.randn(4, 4, dtype=torch.float16),
    lambda: torch.randn(4, 4).to(torch.bfloat16),
], ids=["dense", "cols", "transposed", "vec", "strided_vec", "empty2d", "empty1d", "f16", "bf16"])
def test_tensor_descriptor_bytes_match_ctypes(make):
    t = make()
    assert api._desc(t) == bytes(api.tensor_view(t))


def test_descriptor_rejects_what_tensor_view_rejects():
    for t in (torch.zeros(2, 2, 2), torch.zeros(4, dtype=torch.int64)):
        with pytest.raises(ValueError):
            api.tensor_view(t)
        with pytest.raises(ValueError):
            api._desc(t)


def test_exec_descriptor_layout_matches_ctypes():
    ex = N.StExec()
    ex.stream, ex.device, ex.flags, ex.timeout_ms = 0x7F00DEAD0000, 3, 0, 60000
    assert api._EXEC_DESC.pack(0x7F00DEAD0000, 3, 0, 60000, 0, 0) == bytes(ex)
    assert api._EXEC_DESC.size == ctypes.sizeof(N.StExec)
