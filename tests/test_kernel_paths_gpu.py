"""The shapes meant for the tcgen05 kernels must run on them (no silent hand-off to the
CUDA-core kernels), and the device status word must stay clear (no bounded wait gave up).
Kernel names are read from the torch profiler's CUDA activity."""

import pytest
import torch
from torch.profiler import ProfilerActivity, profile

from helpers import random_router, randn
from ultrametric import _native, block_list_attention, build_block_lists, ultrametric_decode

pytestmark = pytest.mark.gpu
DEV = "cuda"


def kernel_names(fn):
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]


@pytest.mark.parametrize("D,dtype", [(128, torch.bfloat16), (64, torch.float16)])
def test_forward_uses_tcgen05_kernel(D, dtype):
    gen = torch.Generator().manual_seed(1)
    q, k, v = (randn((1, 4, 512, D), gen).to(dtype).to(DEV) for _ in range(3))
    bl = build_block_lists(random_router(1, 4, 4, 4, 2).to(DEV), 1, is_causal=True, arity=2)
    names = kernel_names(lambda: block_list_attention(q, k, v, bl, route_block=128, is_causal=True))
    assert any("fwd_sm100_kernel" in n for n in names), names
    assert not any("simt" in n for n in names), names
    assert _native.read_device_status() == 0


@pytest.mark.parametrize("D,deterministic", [(128, False), (128, True), (64, False)])
def test_backward_uses_tcgen05_kernels(D, deterministic):
    """head_dim 128 runs the fused single-pass kernel unless deterministic sums are asked
    for; the two-kernel path (dQ, dK/dV) serves deterministic=True and head_dim 64."""
    gen = torch.Generator().manual_seed(2)
    q, k, v = (randn((1, 4, 512, D), gen).bfloat16().to(DEV).requires_grad_(True) for _ in range(3))
    bl = build_block_lists(random_router(1, 4, 4, 4, 2).to(DEV), 1, is_causal=True, sink_block=True, arity=2)
    out = block_list_attention(q, k, v, bl, route_block=128, is_causal=True, deterministic=deterministic)
    g = torch.ones_like(out)
    names = kernel_names(lambda: out.backward(g))
    if D == 128 and not deterministic:
        assert any("bwd_fused_sm100_kernel" in n for n in names), names
        assert not any("bwd_dq_sm100_kernel" in n for n in names), names
    else:
        assert any("bwd_dq_sm100_kernel" in n for n in names), names
        assert any("bwd_dkdv_sm100_kernel" in n for n in names), names
    assert not any("simt" in n for n in names), names
    assert _native.read_device_status() == 0


def test_fp32_uses_cuda_core_kernel():
    gen = torch.Generator().manual_seed(1)
    q, k, v = (randn((1, 2, 256, 64), gen).to(DEV) for _ in range(3))
    bl = build_block_lists(random_router(1, 2, 2, 4, 2).to(DEV), 1, arity=2)
    names = kernel_names(lambda: block_list_attention(q, k, v, bl, route_block=128))
    assert any("fwd_simt_kernel" in n for n in names), names


def test_builder_and_decode_kernels_run():
    r = random_router(1, 2, 64, 6, 2).to(DEV)
    names = kernel_names(lambda: build_block_lists(r, 2, arity=2))
    assert any("build_lists_kernel" in n for n in names), names
    B, H, Hkv, D, page = 2, 8, 2, 128, 64
    gen = torch.Generator().manual_seed(0)
    q = randn((B, H, D), gen).bfloat16().to(DEV)
    kc = randn((8, Hkv, page, D), gen).bfloat16().to(DEV)
    bt = torch.arange(8, dtype=torch.int32, device=DEV).view(2, 4)
    ctx = torch.tensor([200, 256], dtype=torch.int32, device=DEV)
    ri = torch.zeros(8, H, 3, dtype=torch.int32, device=DEV)
    qri = torch.zeros(B, H, 3, dtype=torch.int32, device=DEV)
    names = kernel_names(lambda: ultrametric_decode(q, kc, kc, bt, ctx, ri, qri, 2))
    for k in ("decode_init_kernel", "decode_select_kernel", "decode_stream_kernel",
              "decode_unit_combine_kernel"):
        assert any(k in n for n in names), names
    assert not any("decode_split_kernel" in n for n in names), names
    assert _native.read_device_status() == 0


def test_decode_general_path_for_other_shapes():
    """fp32 caches (and page sizes other than 16, 32 or a multiple of 64) take the general
    split-K kernel."""
    B, H, Hkv, D, page = 2, 4, 2, 64, 48
    gen = torch.Generator().manual_seed(0)
    q = randn((B, H, D), gen).to(DEV)
    kc = randn((6, Hkv, page, D), gen).to(DEV)
    bt = torch.arange(6, dtype=torch.int32, device=DEV).view(2, 3)
    ctx = torch.tensor([100, 144], dtype=torch.int32, device=DEV)
    ri = torch.zeros(6, H, 3, dtype=torch.int32, device=DEV)
    qri = torch.zeros(B, H, 3, dtype=torch.int32, device=DEV)
    for dt in (torch.float32, torch.bfloat16):
        names = kernel_names(lambda: ultrametric_decode(q.to(dt), kc.to(dt), kc.to(dt), bt, ctx, ri,
                                                        qri, 2))
        assert any("decode_split_kernel" in n for n in names), (dt, names)
        assert not any("decode_stream_kernel" in n for n in names), (dt, names)
    assert _native.read_device_status() == 0
