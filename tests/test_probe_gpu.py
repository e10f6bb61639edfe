"""w4_read_probe on the GPU: it runs, reads, and leaves the sink alone on a zero buffer."""
import pytest
import torch

from xe2x2_b200 import _lib as L, ops


@pytest.mark.gpu
def test_read_probe_runs_and_writes_nothing_on_zeros():
    dev = torch.device("cuda:0")
    buf = torch.zeros(64 << 20, dtype=torch.uint8, device=dev)
    sink = torch.full((1,), 7, dtype=torch.int32, device=dev)
    for _ in range(3):
        L.call("w4_read_probe", ops._p(buf), buf.numel(), ops._p(sink), ops._stream(dev))
    torch.cuda.synchronize()
    assert int(sink.item()) == 7
    assert L.lib().w4_check_device_status() == L.W4_OK
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    L.call("w4_read_probe", ops._p(buf), buf.numel(), ops._p(sink), ops._stream(dev))
    e1.record()
    torch.cuda.synchronize()
    gbs = buf.numel() / (e0.elapsed_time(e1) * 1e6)
    assert 500 < gbs < 12000, gbs  # a real HBM read, not an empty launch
