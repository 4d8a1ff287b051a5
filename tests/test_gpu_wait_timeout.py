"""Failure detection on the GPU without a fault. The kernels' one device-side
wait (the table's bulk copy into shared memory) is bounded. A self-test
kernel waits on an mbarrier that nothing completes: it must give up after
its poll limit and report AIB_STATUS_WAIT_TIMEOUT in the status word the host
reads. The context stays usable: a decode right after it is bit-exact."""
import pytest
import torch

from afterimage_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("polls", [1, 4096])
def test_bounded_wait_gives_up_and_reports_the_timeout(polls):
    L = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    assert L.aib_selftest_wait_timeout(polls, status.data_ptr(), stream.cuda_stream) == _lib.AIB_OK
    b.record(stream)
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.STATUS_WAIT_TIMEOUT
    assert a.elapsed_time(b) < 10_000.0  # ms: the wait ends on its own


def test_context_survives_a_timed_out_wait():
    from afterimage_b200.runtime.compressed_store import compress_layer, decompress_layer_gpu
    L = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert L.aib_selftest_wait_timeout(64, status.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    W = (torch.randn(256, 320, generator=torch.Generator().manual_seed(3)) * 0.02).to(torch.bfloat16)
    out = decompress_layer_gpu(compress_layer(W, chunk_size=128), device="cuda")
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.STATUS_WAIT_TIMEOUT
    assert torch.equal(out.cpu().view(torch.int16), W.view(torch.int16))
