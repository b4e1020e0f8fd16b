"""Host-side checks of paged.BatchDecoder (no GPU): the argument and capacity errors
it raises before any device work.  A stand-in cache object supplies the pool's
geometry; the decoder's plan handle is created and destroyed through the C ABI,
which touches no device for an unbuilt plan."""

from __future__ import annotations

import pytest
import torch

import paged


class _Geometry:
    """The attributes BatchDecoder reads from a PagedKVCache before planning."""
    num_layers = 2
    page_size = 16


def test_rejects_mismatched_layers_and_rows():
    bt = torch.zeros((3, 4), dtype=torch.int32)
    with pytest.raises(ValueError):
        paged.BatchDecoder(_Geometry(), [object()], bt, 8, [0, 0, 0])        # 1 of 2 layers
    with pytest.raises(ValueError):
        paged.BatchDecoder(_Geometry(), [object(), object()], bt, 8, [0] * 4)  # 4 seqs, 3 rows
    with pytest.raises(ValueError):
        paged.BatchDecoder(_Geometry(), [object(), object()], bt[0], 8, [0])   # not 2-D


def test_capacity_and_batch_shape_checked_before_planning():
    bt = torch.zeros((3, 4), dtype=torch.int32)          # 4 pages of 16: 64 positions per row
    dec = paged.BatchDecoder(_Geometry(), [object(), object()], bt, 8, [10, 64, 0])
    assert dec.capacity == 64
    with pytest.raises(ValueError):
        dec.step(torch.zeros((2, 16), dtype=torch.float16))   # one token per sequence (3)
    with pytest.raises(IndexError):
        dec.step(torch.zeros((3, 16), dtype=torch.float16))   # row 1 is full
    with pytest.raises(IndexError):
        dec.prefill(0, torch.zeros((55, 16), dtype=torch.float16))   # 10 + 55 > 64
    x = torch.zeros((0, 16), dtype=torch.float16)
    assert dec.prefill(2, x) is x                             # empty chunk: nothing to run
    assert list(dec.ctx) == [10, 64, 0]
    dec.close()
