"""Host logic of the GPT-2 forward that needs no GPU: how it reads a logits tensor's layout."""

from __future__ import annotations

import pytest


def test_logits_row_pitch():
    """The LM head's row pitch from a logits tensor's strides: contiguous rows, rows on
    128-byte lines (GPT2.new_logits' layout), and the layouts it refuses."""
    torch = pytest.importorskip("torch")
    from ppy_b200 import runtime
    from ppy_b200.gpt2 import GPT2

    pitch = GPT2._row_pitch
    assert pitch(torch.empty(2, 4, 50257), 2, 4, 50257, "cpu") == 50257
    assert pitch(torch.empty(2, 4, 50272)[:, :, :50257], 2, 4, 50257, "cpu") == 50272
    assert pitch(torch.empty(1, 4, 64)[:, :, :10], 1, 4, 10, "cpu") == 64  # one sequence
    refused = [torch.empty(2, 5, 50272)[:, :4, :50257],  # rows unevenly spaced
               torch.empty(2, 4, 50257, 2)[..., 0],      # vocabulary not unit-stride
               torch.empty(2, 4, 50257, dtype=torch.float64),
               torch.empty(2, 4, 50256)]
    for logits in refused:
        with pytest.raises(runtime.B200Error):
            pitch(logits, 2, 4, 50257, "cpu")
    with pytest.raises(runtime.B200Error):  # host memory where the GPU writes
        pitch(torch.empty(2, 4, 50257), 2, 4, 50257)
