"""CPU: frame sizes other than 518 x 518.

* ``qvggt_b200.frames.crop_size`` follows the reference loader's rule
  (``qvggt/inference/io.py:50-100``): width 518, height rounded to a multiple
  of 14, centre-cropped to 518; "pad" keeps the longer side at 518.
* The DINOv2 position table resampled to the frame's patch grid (the product's
  set-up, ``frames.interpolate_position_table``) against an independent
  restatement of separable antialiased bicubic resampling in the oracle.
"""
import pytest
import torch

from oracle import model as om
from qvggt_b200 import frames


@pytest.mark.parametrize("hw,expect", [((518, 518), (518, 518, 518, 518)), ((480, 640), (392, 518, 392, 518)),
                                       ((1080, 1920), (294, 518, 294, 518)), ((900, 600), (784, 518, 518, 518)),
                                       ((100, 3000), (14, 518, 14, 518))])
def test_crop_rule(hw, expect):
    assert frames.crop_size(*hw) == expect


def test_pad_rule():
    assert frames.crop_size(900, 600, mode="pad") == (518, 350, 518, 518)
    assert frames.crop_size(480, 640, mode="pad") == (392, 518, 518, 518)
    with pytest.raises(ValueError):
        frames.crop_size(10, 10, mode="stretch")


@pytest.mark.parametrize("rows,cols", [(37, 37), (28, 37), (21, 37), (1, 37), (37, 20), (40, 37)])
def test_position_table_matches_oracle(rows, cols):
    g = torch.Generator().manual_seed(rows * 100 + cols)
    pe = (torch.randn(1 + 37 * 37, 64, generator=g) * 0.02).half()
    got = frames.interpolate_position_table(pe, rows, cols)
    ref = om.interpolate_pos_embed(pe, rows, cols)
    assert got.shape == (1 + rows * cols, 64)
    assert torch.equal(got[0], pe[0].float())
    assert (got - ref).abs().max().item() <= 1e-6 * max(1.0, ref.abs().max().item() * 50)


def test_token_table_layout():
    pe = torch.arange((1 + 9) * 2, dtype=torch.float32).reshape(10, 2)
    t = frames.token_position_table(pe, 3, 3, n_special=5)
    assert t.shape == (14, 2) and t.dtype == torch.float16
    assert torch.equal(t[0], pe[0].half()) and not t[1:5].any() and torch.equal(t[5:], pe[1:].half())
