"""Half-precision shapes outside the tensor-core kernels' range (head_dim other than 64 / 128,
or a route block that is not a multiple of 128) run the CUDA-core kernels, several times
slower; the operator says so once per shape instead of falling off that cliff quietly.  The
check is host logic and needs no GPU."""

import warnings

import pytest
import torch

from ultrametric import block_list as bl


@pytest.fixture(autouse=True)
def _fresh_registry():
    saved = set(bl._SIMT_WARNED)
    bl._SIMT_WARNED.clear()
    yield
    bl._SIMT_WARNED.clear()
    bl._SIMT_WARNED.update(saved)


@pytest.mark.parametrize("dtype,D,RB", [(torch.bfloat16, 96, 128), (torch.float16, 128, 64),
                                        (torch.bfloat16, 256, 256)])
def test_warns_once_per_shape(dtype, D, RB):
    with pytest.warns(RuntimeWarning, match="CUDA-core"):
        bl._warn_if_simt(dtype, D, RB)
    with warnings.catch_warnings():
        warnings.simplefilter("error")
        bl._warn_if_simt(dtype, D, RB)  # the same shape again: silent


@pytest.mark.parametrize("dtype,D,RB", [(torch.bfloat16, 128, 128), (torch.float16, 64, 256),
                                        (torch.float32, 96, 64)])
def test_silent_on_tensor_core_shapes_and_fp32(dtype, D, RB):
    with warnings.catch_warnings():
        warnings.simplefilter("error")
        bl._warn_if_simt(dtype, D, RB)
