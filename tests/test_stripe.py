"""Striped device layout of a compressed stream (aib_stripe_layout /
aib_stripe_stream) and the decode kernel reading it.

The layout is this library's own (the reference reads each chunk where the
encoder wrote it, huffman_chunked.py:180-206); what must hold is that a
striped stream decodes to exactly what the reference layout decodes to, for
every mode, chunk size, element range and chunk sub-range, and that a
corrupt group table raises like corrupt chunk offsets do. The layout helpers
restated here in numpy are test infrastructure."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O


def _layout_np(nbs: np.ndarray) -> np.ndarray:
    """group_base: region g starts at sum over earlier groups of
    32 * max(ceil(nbytes / 16)) over the group's chunks."""
    n = nbs.shape[0]
    rows = [int(((nbs[g:g + 32].astype(np.int64) + 15) // 16).max(initial=0)) for g in range(0, n, 32)]
    return np.concatenate([[0], np.cumsum(np.asarray(rows, dtype=np.int64) * 32)]).astype(np.int64)


def _stripe_np(packed: np.ndarray, offs: np.ndarray, nbs: np.ndarray, base: np.ndarray) -> np.ndarray:
    out = np.zeros(int(base[-1]) * 16, dtype=np.uint8)
    for c in range(nbs.shape[0]):
        g, col = divmod(c, 32)
        data = packed[int(offs[c]):int(offs[c]) + int(nbs[c])]
        for i in range(0, data.shape[0], 16):
            blk = (int(base[g]) + col + 32 * (i // 16)) * 16
            piece = data[i:i + 16]
            out[blk:blk + piece.shape[0]] = piece
    return out


# ---------------------------------------------------------------- host side

@pytest.mark.parametrize("n", [0, 1, 31, 32, 33, 95, 1000])
def test_stripe_layout_matches_numpy(n):
    from afterimage_b200.runtime import _device
    rng = np.random.default_rng(n)
    nbs = rng.integers(0, 700, size=n).astype(np.int32)
    if n > 3:
        nbs[3] = 0   # an empty chunk
    assert np.array_equal(_device.stripe_layout(nbs), _layout_np(nbs))


def test_stripe_layout_rejects_negative_counts():
    from afterimage_b200.runtime import _device
    with pytest.raises(ValueError, match="negative byte count"):
        _device.stripe_layout(np.array([4, -1, 5], np.int32))


def test_striped_addresses_give_back_every_chunk():
    """The kernel's address rule (chunk c's block j at 16 x (group_base[c / 32]
    + c mod 32 + 32 j)) applied to the numpy striping returns each chunk's
    bytes, followed by zeros up to its region's row count."""
    from afterimage_b200.runtime.compressed_store import compress_layer
    g = torch.Generator().manual_seed(5)
    W = (torch.randn(70, 333, generator=g) * 0.02).to(torch.bfloat16)
    e = compress_layer(W, chunk_size=100).encoded
    packed, offs, nbs = np.asarray(e.packed), np.asarray(e.chunk_offsets), np.asarray(e.chunk_nbytes)
    base = _layout_np(nbs)
    st = _stripe_np(packed, offs, nbs, base)
    for c in range(nbs.shape[0]):
        grp = c // 32
        rows = (int(base[grp + 1]) - int(base[grp])) // 32
        got = np.concatenate([st[(int(base[grp]) + c % 32 + 32 * j) * 16:][:16] for j in range(rows)])
        n = int(nbs[c])
        assert np.array_equal(got[:n], packed[offs[c]:offs[c] + n])
        assert not got[n:].any()


@pytest.mark.parametrize("chunk_size", [1, 5, 100, 1024])
def test_host_striping_matches_numpy(chunk_size):
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.compressed_store import compress_layer
    g = torch.Generator().manual_seed(chunk_size + 77)
    W = (torch.randn(37, 411, generator=g) * 0.02).to(torch.bfloat16)
    e = compress_layer(W, chunk_size=chunk_size).encoded
    packed, offs, nbs = np.asarray(e.packed), np.asarray(e.chunk_offsets), np.asarray(e.chunk_nbytes)
    got, base = _device.stripe_host(packed, offs, nbs)
    assert np.array_equal(base, _layout_np(nbs))
    assert np.array_equal(got, _stripe_np(packed, offs, nbs, base))
    if nbs.shape[0] >= 70:
        # a chunk sub-range with its own offset base (chunks [32, 70))
        sub, sbase = _device.stripe_host(packed[offs[32]:], offs[32:70], nbs[32:70], int(offs[32]))
        assert np.array_equal(sub, _stripe_np(packed, offs[32:70], nbs[32:70], sbase))


def test_host_striping_rejects_a_chunk_outside_the_stream():
    from afterimage_b200.runtime import _device
    packed = np.arange(100, dtype=np.uint8)
    with pytest.raises(ValueError, match="does not fit"):
        _device.stripe_host(packed, np.array([0, 90], np.int32), np.array([40, 20], np.int32))


def test_striped_descriptor_validation_without_a_gpu():
    from afterimage_b200 import _lib
    L = _lib.load()
    buf = (ctypes.c_uint8 * 64)()
    addr = (ctypes.addressof(buf) + 15) // 16 * 16
    d = _lib.StreamDesc()
    d.packed, d.packed_capacity, d.packed_nbytes = addr, 32, 32
    d.chunk_nbytes = d.tables = d.sym_lut = d.len_lut = d.out = d.sign_mantissa = addr
    d.stripe_base = addr
    d.chunk_size, d.max_bits, d.n_symbols, d.elem_begin, d.elem_end = 16, 8, 4096, 1024, 2048
    d.chunk_base = 16   # not a multiple of 32
    assert L.aib_decode_bf16(ctypes.byref(d), None, None) == _lib.AIB_EINVAL
    assert b"multiple of 32" in L.aib_last_error()
    # the fused GEMV takes only the reference layout
    g = _lib.GemvDesc()
    g.stream = d
    g.stream.chunk_base = 0
    g.stream.elem_begin, g.stream.elem_end = 0, 1024
    g.cols, g.x, g.partial, g.y = 64, addr, addr, addr
    assert L.aib_decode_gemv_bf16_batch(ctypes.byref(g), 1, None, None) == _lib.AIB_EINVAL
    assert b"reference layout" in L.aib_last_error()
    assert L.aib_stripe_stream(addr, 16, 0, addr, addr, 5, 1, addr, addr, 16, None, None) == _lib.AIB_EINVAL


# ---------------------------------------------------------------- device

def _resident(enc, dev, c0=0, c1=None, striped=True):
    from afterimage_b200.runtime import _device
    ds = _device.upload_stream(enc, dev, c0, c1)
    if striped:
        c1 = enc.n_chunks if c1 is None else c1
        ds = _device.stripe_stream(ds, np.asarray(enc.chunk_nbytes)[c0:c1], dev)
    return ds


@pytest.mark.gpu
@pytest.mark.parametrize("chunk_size", [5, 100, 1024])
def test_stripe_stream_matches_numpy(chunk_size):
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.compressed_store import compress_layer
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(chunk_size)
    W = (torch.randn(200, 517, generator=g) * 0.02).to(torch.bfloat16)
    e = compress_layer(W, chunk_size=chunk_size).encoded
    ds = _resident(e, dev)
    torch.cuda.synchronize()
    packed, offs, nbs = np.asarray(e.packed), np.asarray(e.chunk_offsets), np.asarray(e.chunk_nbytes)
    want = _stripe_np(packed, offs, nbs, _layout_np(nbs))
    assert ds.nbytes == want.shape[0]
    assert np.array_equal(_device.stripe_host(packed, offs, nbs)[0], want)
    assert np.array_equal(ds.packed[:ds.nbytes].cpu().numpy(), want)


@pytest.mark.gpu
@pytest.mark.parametrize("chunk_size", [1, 5, 8, 31, 64, 333, 1024, 4096])
@pytest.mark.parametrize("mode", ["bf16", "u8", "i32"])
def test_striped_decode_equals_oracle(chunk_size, mode):
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.gpu_decode_v2 import prepare_decode_tables
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(300 + chunk_size)
    W = (torch.randn(517, 389, generator=g) * 0.02).to(torch.bfloat16)
    layer = compress_layer(W, chunk_size=chunk_size)
    e = layer.encoded
    t = prepare_decode_tables(e, dev)
    ds = _resident(e, dev)
    sm = layer.sign_mantissa.reshape(-1).to(dev)
    exps = O.decode_chunked(e)
    n = int(e.n_symbols)
    rng = np.random.default_rng(chunk_size)
    ranges = [(0, n)] + [tuple(sorted(rng.integers(0, n + 1, 2))) for _ in range(3)]
    for e0, e1 in ranges:
        e0, e1 = int(e0), int(e1)
        if mode == "bf16":
            out = torch.empty(max(e1 - e0, 1), dtype=torch.int16, device=dev)
            d = _device.make_desc(ds, t, e, e0, e1, out, sm[e0:])
            _device.call("aib_decode_bf16", d, dev)
            want = O.recombine(exps[e0:e1], layer.sign_mantissa.numpy().reshape(-1)[e0:e1]).view(np.int16)
        else:
            out = torch.empty(max(e1 - e0, 1), dtype=torch.uint8 if mode == "u8" else torch.int32, device=dev)
            d = _device.make_desc(ds, t, e, e0, e1, out)
            _device.call("aib_decode_exponents_u8" if mode == "u8" else "aib_decode_exponents_i32", d, dev)
            want = exps[e0:e1].astype(np.uint8 if mode == "u8" else np.int32)
        torch.cuda.synchronize()
        _device.check_status(dev)
        assert np.array_equal(out[:e1 - e0].cpu().numpy(), want), (e0, e1)


@pytest.mark.gpu
@pytest.mark.parametrize("c0,c1", [(32, 96), (64, 65), (0, 31), (96, 160)])
def test_striped_chunk_subrange_equals_oracle(c0, c1):
    """A stream uploaded for chunks [c0, c1) only (chunk_base = c0, a multiple
    of 32), as the tensor-parallel shards and the sliced paths keep them."""
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.gpu_decode_v2 import prepare_decode_tables
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(c0 * 7 + c1)
    W = (torch.randn(160, 256, generator=g) * 0.02).to(torch.bfloat16)
    layer = compress_layer(W, chunk_size=256)
    e = layer.encoded
    t = prepare_decode_tables(e, dev)
    ds = _resident(e, dev, c0, c1)
    e0, e1 = c0 * 256 + 3, c1 * 256 - 5
    out = torch.empty(e1 - e0, dtype=torch.uint8, device=dev)
    _device.call("aib_decode_exponents_u8", _device.make_desc(ds, t, e, e0, e1, out), dev)
    torch.cuda.synchronize()
    _device.check_status(dev)
    assert np.array_equal(out.cpu().numpy(), O.decode_chunked(e)[e0:e1])


@pytest.mark.gpu
@pytest.mark.parametrize("chunk_size", [16, 1024])
def test_striped_non_prefix_lut_reads_zeros_past_the_chunk_end(chunk_size):
    """Past a chunk's end the striped layout holds zero padding or the next
    group's bytes; the exact slow path must still see zeros there
    (huffman_chunked.py:225-231)."""
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.gpu_decode_v2 import prepare_decode_tables
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(chunk_size + 1)
    W = (torch.randn(64, 512, generator=g) * 0.02).to(torch.bfloat16)
    e = compress_layer(W, chunk_size=chunk_size).encoded
    sym = (np.arange(1 << int(e.max_bits), dtype=np.int64) & 0xFF).astype(np.int32)
    bad = type(e)(**{**e.__dict__, "sym_lut": sym})
    t = prepare_decode_tables(bad, dev)
    ds = _resident(bad, dev)
    out = torch.empty(int(e.n_symbols), dtype=torch.uint8, device=dev)
    _device.call("aib_decode_exponents_u8", _device.make_desc(ds, t, bad, 0, int(e.n_symbols), out), dev)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), O.decode_chunked(bad))


@pytest.mark.gpu
def test_corrupt_group_table_raises_and_context_survives():
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.gpu_decode_v2 import prepare_decode_tables
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(9)
    W = (torch.randn(256, 512, generator=g) * 0.02).to(torch.bfloat16)
    e = compress_layer(W, chunk_size=256).encoded
    t = prepare_decode_tables(e, dev)
    ds = _resident(e, dev)
    good_base = ds.stripe_base.clone()
    n = int(e.n_symbols)
    out = torch.empty(n, dtype=torch.uint8, device=dev)
    for bad in (10 ** 12, -5, int(good_base[-1].item())):
        ds.stripe_base.copy_(good_base)
        ds.stripe_base[2] = bad
        _device.call("aib_decode_exponents_u8", _device.make_desc(ds, t, e, 0, n, out), dev)
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="corrupt offsets"):
            _device.check_status(dev)
    ds.stripe_base.copy_(good_base)
    _device.call("aib_decode_exponents_u8", _device.make_desc(ds, t, e, 0, n, out), dev)
    torch.cuda.synchronize()
    _device.check_status(dev)
    assert np.array_equal(out.cpu().numpy(), O.decode_chunked(e))


@pytest.mark.gpu
def test_layer_decoder_striped_batch_equals_reference_layout():
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.layer_decode import LayerDecoder, upload_layer
    dev = torch.device("cuda", 0)
    shapes = [(1024, 4096), (256, 4096), (4096, 1000), (17, 3), (3072, 1024)]
    chunks = [1024, 1024, 640, 7, 1088]
    Ws = []
    for i, s in enumerate(shapes):
        g = torch.Generator().manual_seed(40 + i)
        Ws.append((torch.randn(*s, generator=g) * 0.02).to(torch.bfloat16))
    layers = [compress_layer(W, chunk_size=c) for W, c in zip(Ws, chunks)]
    dec = LayerDecoder(dev)
    outs = dec.decode([upload_layer(lay, dev, striped=True) for lay in layers])
    torch.cuda.synchronize()
    _device.check_status(dev)
    assert dec.launches == 1
    for W, o in zip(Ws, outs):
        assert torch.equal(o.cpu().view(torch.int16), W.view(torch.int16))
