"""Host logic of the two decoder kinds (CPU): the kind a descriptor tensor selects, the variant's scene
shapes and initialisation, and the gradient buffer laid out for either width."""
import pytest
import torch

from flare_b200 import dp
from flare_b200.renderer import DECODER_GRID_SH, DECODER_LUT_PE, DECODERS, decoder_kind
from flare_b200.scene import GRID_COND_DIM, GRID_RES, GRID_SIZE, make_scene


def test_decoder_kind_from_descriptor_width():
    assert decoder_kind(torch.zeros(5, 96, dtype=torch.float16)) == DECODER_LUT_PE
    assert decoder_kind(torch.zeros(5, 32, dtype=torch.float16)) == DECODER_GRID_SH
    for bad in (torch.zeros(5, 64), torch.zeros(96)):
        with pytest.raises(ValueError):
            decoder_kind(bad)
    assert DECODERS[DECODER_LUT_PE] == (96, 13154) and DECODERS[DECODER_GRID_SH] == (GRID_COND_DIM, GRID_SIZE)


def test_grid_table_layout():
    # 8 levels of floor(4 * 1.5^l) vertices per side, each under the 2^16-entry table (row-major, unhashed)
    assert GRID_RES == (4, 6, 9, 13, 20, 30, 45, 68)
    assert all(r * r < 2 ** 16 for r in GRID_RES)
    assert GRID_SIZE == 2 * sum(r * r for r in GRID_RES) == 16502


def test_grid_sh_scene_shapes_and_weights():
    sc = make_scene(100, 3, decoder="grid_sh")
    assert sc.cond.shape == (100, 32) and sc.cond.dtype == torch.float16
    assert sc.features.shape == (GRID_SIZE,)
    assert float(sc.features.abs().max()) <= 0.1
    assert sc.A1.shape == (64, 128) and sc.A1.dtype == torch.float16
    assert torch.count_nonzero(sc.A1[:, 64:]) == 0          # the unused half of W1
    bound = (6.0 / (64 + 64)) ** 0.5                         # Xavier over the 64 real inputs
    assert float(sc.A1[:, :64].float().abs().max()) <= bound * 1.001
    # the reference decoder's scene is unchanged by the option (same seed, same tensors)
    a, b = make_scene(100, 3), make_scene(100, 3, decoder="lut_pe")
    assert all(torch.equal(getattr(a, k), getattr(b, k)) for k in a.__dict__)
    with pytest.raises(ValueError):
        make_scene(10, 0, decoder="hash")


@pytest.mark.parametrize("cdim,nfeat", [(96, 13154), (32, 16502)])
def test_grad_buffer_for_either_decoder(cdim, nfeat):
    g = dp.GradBuffer(37, True, "cpu", cdim, nfeat)
    assert g["cond"].shape == (37, cdim) and g["features"].shape == (nfeat,)
    assert all(v.data_ptr() % 64 == 0 for v in g.views.values())  # vector reductions need aligned segments
