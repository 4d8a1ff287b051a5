"""One-shot NVLink all-reduce (csrc/allreduce.cu, runtime/allreduce.py).

Host-side validation runs without a GPU. On one GPU: a single-rank group
is a copy, and a two-rank group whose second rank never arrives (its words
never land) gives up within its poll limit with AIB_STATUS_PEER_TIMEOUT,
leaving the context usable. On two GPUs (one process each, NCCL for the
handle exchange): sums bit-identical to an explicit rank-order fp32 sum of
the gathered inputs on every rank, across sizes, repeated calls and CUDA
graph replays, and within fp32 rounding of torch.distributed.all_reduce."""
import ctypes
import socket

import pytest
import torch
import torch.multiprocessing as mp

from afterimage_b200 import _lib


def _group(bufs, rank, world, max_floats):
    g = _lib.ArGroup()
    for i, b in enumerate(bufs):
        g.buffers[i] = b
    g.rank, g.world, g.max_floats = rank, world, max_floats
    return g


def test_host_validation_without_a_gpu():
    L = _lib.load()
    assert L.aib_allreduce_oneshot_f32(None, None, None, 4, 10, None, None) == _lib.AIB_EINVAL
    g = _group([256, 512], 0, 9, 100)
    assert L.aib_allreduce_oneshot_f32(ctypes.byref(g), None, None, 4, 10, None, None) == _lib.AIB_EINVAL
    assert b"world" in L.aib_last_error()
    g = _group([256, 512], 2, 2, 100)
    assert L.aib_allreduce_oneshot_f32(ctypes.byref(g), None, None, 4, 10, None, None) == _lib.AIB_EINVAL
    g = _group([256, 512], 0, 2, 100)
    assert L.aib_allreduce_oneshot_f32(ctypes.byref(g), None, None, 101, 10, None, None) == _lib.AIB_EINVAL
    assert b"max_floats" in L.aib_last_error()
    assert L.aib_allreduce_oneshot_f32(ctypes.byref(g), None, None, 8, 0, None, None) == _lib.AIB_EINVAL
    assert L.aib_allreduce_oneshot_f32(ctypes.byref(g), None, None, 0, 10, None, None) == _lib.AIB_OK
    g = _group([256, 0], 0, 2, 100)
    assert L.aib_allreduce_oneshot_f32(ctypes.byref(g), 4096, 4096, 8, 10, None, None) == _lib.AIB_EINVAL
    assert b"rank 1" in L.aib_last_error()
    g = _group([256, 100], 0, 2, 100)
    assert L.aib_allreduce_oneshot_f32(ctypes.byref(g), 4096, 4096, 8, 10, None, None) == _lib.AIB_EINVAL


def test_buffer_size_and_grid():
    L = _lib.load()
    assert L.aib_ar_buffer_bytes(1) == 4096 + 2 * 8 * 8
    assert L.aib_ar_buffer_bytes(1 << 16) == 4096 + 128 * (1 << 16)
    assert [L.aib_ar_ctas(n) for n in (0, 1, 1024, 1025, 5120, 1 << 20, 1 << 30)] == [0, 1, 1, 2, 5, 64, 64]


def test_cpu_decoder_keeps_its_collective():
    """A CPU rank (the gloo host-logic tests) never builds the NVLink path."""
    from afterimage_b200.runtime.tp_decoder import TPDecoder
    dec = TPDecoder.__new__(TPDecoder)
    dec.world, dec.device, dec.allreducer = 2, torch.device("cpu"), None
    dec.use_oneshot_allreduce()
    assert dec.allreducer is None


@pytest.mark.gpu
def test_single_rank_is_a_copy_and_in_place_works():
    from afterimage_b200.runtime import _device
    L = _lib.load()
    dev = torch.device("cuda", 0)
    buf = ctypes.c_void_p()
    _lib.check(L.aib_ar_alloc(1 << 16, ctypes.byref(buf)))
    try:
        g = _group([buf.value], 0, 1, 1 << 16)
        for n in (1, 3, 4, 4096, 5121, 1 << 16):
            x = torch.randn(n, device=dev)
            out = torch.empty_like(x)
            _lib.check(L.aib_allreduce_oneshot_f32(ctypes.byref(g), x.data_ptr(), out.data_ptr(), n, 1 << 20,
                                                   _device.status_word(dev).data_ptr(), _device.stream_ptr(dev)))
            ref = x.clone()
            _lib.check(L.aib_allreduce_oneshot_f32(ctypes.byref(g), x.data_ptr(), x.data_ptr(), n, 1 << 20,
                                                   _device.status_word(dev).data_ptr(), _device.stream_ptr(dev)))
            torch.cuda.synchronize()
            _device.check_status(dev)
            assert torch.equal(out, ref) and torch.equal(x, ref)
    finally:
        torch.cuda.synchronize()
        _lib.check(L.aib_ar_free(buf))


@pytest.mark.gpu
def test_a_peer_that_never_arrives_times_out_with_a_status():
    """Rank 1's buffer is this rank's own, and nothing writes rank 1's
    words: the one kernel's bounded wait gives up (no second launch waits on
    it)."""
    from afterimage_b200.runtime import _device
    L = _lib.load()
    dev = torch.device("cuda", 0)
    buf = ctypes.c_void_p()
    _lib.check(L.aib_ar_alloc(4096, ctypes.byref(buf)))
    try:
        g = _group([buf.value, buf.value], 0, 2, 4096)
        x = torch.ones(4096, device=dev)
        out = torch.full_like(x, 7.0)
        _device.check_status(dev)
        _lib.check(L.aib_allreduce_oneshot_f32(ctypes.byref(g), x.data_ptr(), out.data_ptr(), 4096, 2000,
                                               _device.status_word(dev).data_ptr(), _device.stream_ptr(dev)))
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="gave up waiting for a peer"):
            _device.check_status(dev)
        assert torch.equal(out, torch.full_like(x, 7.0))   # out untouched
        # the context is healthy: an ordinary kernel runs and the status is clear
        y = (x * 2).sum()
        torch.cuda.synchronize()
        assert float(y) == 8192.0
        _device.check_status(dev)
    finally:
        torch.cuda.synchronize()
        _lib.check(L.aib_ar_free(buf))


def _ordered_sum(x, world):
    parts = [torch.empty_like(x) for _ in range(world)]
    torch.distributed.all_gather(parts, x)
    want = parts[0].clone()
    for p in parts[1:]:
        want = want + p
    return want


def _rank_main(rank, world, port, q):
    import datetime
    import os
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=120), device_id=dev)
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.allreduce import OneShotAllReduce
    ar = None
    try:
        ar = OneShotAllReduce(None, dev, 1 << 20)
        results = []
        g = torch.Generator(device=dev)
        sizes = [1, 3, 4, 5120, 5121, 17 * 5120, 1 << 20, 5120, 4096, 1 << 20]
        for call, n in enumerate(sizes):
            g.manual_seed(1000 * call + rank)
            x = torch.randn(n, device=dev, generator=g) * (rank + 1)
            want = _ordered_sum(x, world)
            nccl = x.clone()
            torch.distributed.all_reduce(nccl)
            got = ar(x.clone())
            torch.cuda.synchronize()
            results.append((n, bool(torch.equal(got, want)),
                            float((got - nccl).abs().max()), float(nccl.abs().max())))
        # in a CUDA graph: capture three calls, replay with new inputs
        n = 5120
        xs = [torch.zeros(n, device=dev) for _ in range(3)]
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            ar(xs[0])  # warm on the capture stream
        torch.cuda.synchronize()
        torch.distributed.barrier()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for t in xs:
                ar(t)
        torch.cuda.synchronize()
        torch.distributed.barrier()
        graph_ok = []
        for rep in range(3):
            ins = []
            for i, t in enumerate(xs):
                g.manual_seed(77 + 10 * rep + i + 1000 * rank)
                v = torch.randn(n, device=dev, generator=g)
                t.copy_(v)
                ins.append(v)
            torch.cuda.synchronize()
            torch.distributed.barrier()
            graph.replay()
            torch.cuda.synchronize()
            for t, v in zip(xs, ins):
                graph_ok.append(bool(torch.equal(t, _ordered_sum(v, world))))
        del graph
        torch.cuda.synchronize()
        _device.check_status(dev)
        q.put((rank, results, graph_ok))
    finally:
        if ar is not None:
            ar.close()
        torch.distributed.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_bit_identical_to_rank_order_sum():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = sorted([q.get(timeout=300) for _ in range(2)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, results, graph_ok in got:
        for n, exact, diff_nccl, scale in results:
            assert exact, (rank, n)
            assert diff_nccl <= 1e-6 * max(scale, 1.0), (rank, n, diff_nccl)
        assert all(graph_ok) and len(graph_ok) == 9


def test_loader_rejects_an_unknown_collective(tmp_path):
    """load_tp_decoder validates `collective` before building anything."""
    from afterimage_b200.runtime.tp_decoder import load_tp_decoder
    (tmp_path / "manifest.json").write_text('{"tensors": {}}')
    with pytest.raises(ValueError, match="collective"):
        load_tp_decoder(tmp_path, None, 1, 0, None, "cpu", resident="decoded", collective="mpi")
