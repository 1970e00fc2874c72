"""The tensor-parallel exchange cells of ``mt_w4a16_linear_packed_tp`` on one GPU.

A world of two ranks is emulated on a single device by giving both ranks the same (local)
receive area, so the consumer side can be exercised without a second GPU and without any
peer mapping. Cells are 64-bit ``flag << 32 | bf16 pair`` elements written here from the
host side of the test:

* all cells fresh: the kernel sums the two ranks' rows in fp32, rounds to bf16 and gives the
  same bits as the plain entry point fed that bf16 sum;
* rank 1's cells never written (a dead peer): the poll gives up at its deadline, the call
  returns (no hang), and the library's error word reads 2.
"""
import time

import numpy as np
import pytest
import torch

from moss_tts._runtime import native, synthetic
from moss_tts._runtime.weights import Projection

pytestmark = pytest.mark.gpu

N, K = 256, 512


def _cells(x: torch.Tensor, flag: int) -> torch.Tensor:
    """bf16 [K] -> int64 [K / 2] cells {flag << 32 | bf16 pair}."""
    pairs = x.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return pairs | (flag << 32)


@pytest.fixture(scope="module")
def setup(cuda_device):
    dev = cuda_device
    rng = np.random.Generator(np.random.PCG64(91))
    p = Projection.from_host(synthetic.quantized(rng, N, K), dev)
    norm = (torch.randn(K, device=dev) * 0.02 + 1).to(torch.bfloat16)
    ws = torch.zeros(native.w4a16_packed_size(N, K, True, 0)[1], device=dev, dtype=torch.uint8)
    return dev, p, norm, ws


def _tp_call(dev, p, norm, ws, recv, epoch, y):
    d = native.TpExchange()
    d.recv[0] = d.recv[1] = recv.data_ptr()  # both ranks' areas are this device's buffer
    d.epoch = epoch.data_ptr()
    d.world, d.rank, d.in_slot, d.out_slot, d.slot_elems = 2, 0, 0, -1, K
    import ctypes
    native.call("mt_w4a16_linear_packed_tp", None, None, norm.data_ptr(), 1e-6, None, p.packed_tiles().data_ptr(),
                1, y.data_ptr(), N, K, native.LINEAR_NORM, ws.data_ptr(), ctypes.byref(d), 0,
                torch.cuda.current_stream(dev).cuda_stream)


def test_exchange_sums_fresh_cells_like_the_plain_call(setup):
    dev, p, norm, ws = setup
    native.error_word(clear=True)
    x0 = torch.randn(K, device=dev).to(torch.bfloat16)
    x1 = torch.randn(K, device=dev).to(torch.bfloat16)
    epoch = torch.tensor([5], device=dev, dtype=torch.long)
    recv = torch.stack([_cells(x0, 5), _cells(x1, 5)])  # [slot 0][rank][K / 2]
    y_tp = torch.empty(N, device=dev, dtype=torch.bfloat16)
    _tp_call(dev, p, norm, ws, recv, epoch, y_tp)
    x = (x0.float() + x1.float()).to(torch.bfloat16)
    y = torch.empty_like(y_tp)
    native.call("mt_w4a16_linear_packed", x.data_ptr(), None, norm.data_ptr(), 1e-6, None,
                p.packed_tiles().data_ptr(), 1, y.data_ptr(), N, K, native.LINEAR_NORM, ws.data_ptr(), 0,
                torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    assert native.error_word(clear=True) == 0
    assert torch.equal(y_tp, y)


def test_exchange_gives_up_on_a_silent_peer(setup):
    dev, p, norm, ws = setup
    native.error_word(clear=True)
    x0 = torch.randn(K, device=dev).to(torch.bfloat16)
    epoch = torch.tensor([7], device=dev, dtype=torch.long)
    recv = torch.stack([_cells(x0, 7), _cells(x0, 6)])  # rank 1 still holds the previous step's flag
    y = torch.empty(N, device=dev, dtype=torch.bfloat16)
    try:
        t0 = time.perf_counter()
        _tp_call(dev, p, norm, ws, recv, epoch, y)
        torch.cuda.synchronize(dev)
        elapsed = time.perf_counter() - t0
        word = native.error_word()
    finally:
        native.error_word(clear=True)  # later calls give up at once while the word is 2
    print(f"silent peer: call returned after {elapsed * 1e3:.1f} ms, error word {word}")
    assert word == 2
    assert elapsed < 3.0  # one 1 s deadline for the whole kernel, not one per cell
