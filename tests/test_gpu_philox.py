"""Bit-exact reproduction of torch's CUDA Philox normal stream (the reference controller's
torch.randn(..., generator=cuda_generator) draws, ds_mezo/controller.py:184-191)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _layout():
    p = torch.cuda.get_device_properties(0)
    return p.multi_processor_count, p.max_threads_per_multi_processor


@pytest.mark.parametrize("n", [1, 7, 256, 1000, 4096, 32768, 303104, 303105, 1212416, 1212417, 1212417 * 3 + 5])
@pytest.mark.parametrize("seed,pre", [(0, 0), (1234567, 3), (2 ** 40 + 17, 1)])
def test_randn_stream_bit_exact(n, seed, pre):
    from dsmezo_b200 import _lib
    sm, mt = _layout()
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    for _ in range(pre):                       # earlier draws move the offset
        torch.randn(1000 + 4096 * _, device=DEV, generator=g)
    off = g.get_offset()
    want = torch.randn(n, device=DEV, generator=g)
    advance = g.get_offset() - off
    assert advance == _lib.lib().dsmz_randn_offset_increment(n, sm, mt)
    got = torch.empty(n, device=DEV)
    _lib.check(_lib.lib().dsmz_randn(got.data_ptr(), n, g.initial_seed(), off, sm, mt,
                                     torch.cuda.current_stream().cuda_stream), "randn")
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))


def test_two_dim_draw_matches_flat():
    from dsmezo_b200 import _lib
    sm, mt = _layout()
    g = torch.Generator(device=DEV)
    g.manual_seed(5)
    off = g.get_offset()
    want = torch.randn(18944, 64, device=DEV, generator=g)
    got = torch.empty(18944 * 64, device=DEV)
    _lib.check(_lib.lib().dsmz_randn(got.data_ptr(), got.numel(), 5, off, sm, mt,
                                     torch.cuda.current_stream().cuda_stream), "randn")
    torch.cuda.synchronize()
    assert torch.equal(got.view(18944, 64), want)
