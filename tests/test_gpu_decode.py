"""GPU parity: the sm_100a decode kernels (through the C ABI, via the
reference-shaped Python entry points) against the golden vectors the
reference produced and against the CPU oracle. Integer work: bit-exact."""
import ctypes
import hashlib

import numpy as np
import pytest
import torch

import golden_cases as G
from oracle import oracle as O

pytestmark = pytest.mark.gpu

EXP = [c["name"] for c in G.cases("exponents")]
BF16 = [c["name"] for c in G.cases("bf16")]


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).reshape(-1).numpy()


def _layer(name):
    from afterimage_b200.runtime.compressed_store import CompressedLayer
    from afterimage_b200.runtime.huffman_chunked import ChunkedEncoded
    c = G.case(name)
    e = G.enc(name)
    enc = ChunkedEncoded(packed=e.packed, chunk_offsets=e.chunk_offsets, chunk_nbytes=e.chunk_nbytes,
                         sym_lut=e.sym_lut, len_lut=e.len_lut, max_bits=e.max_bits,
                         chunk_size=e.chunk_size, n_symbols=e.n_symbols, shape=e.shape)
    return CompressedLayer(sign_mantissa=torch.from_numpy(G.arr(name, "sign_mantissa").copy()),
                           encoded=enc, shape=tuple(c["shape"]))


@pytest.mark.parametrize("name", EXP)
def test_decode_gpu_v2_matches_reference_golden(name):
    from afterimage_b200.runtime.gpu_decode_v2 import decode_gpu_v2
    e = G.enc(name)
    got = decode_gpu_v2(e).cpu().numpy()
    assert got.dtype == np.uint8 and got.shape == (e.n_symbols,)
    assert np.array_equal(got, G.arr(name, "decoded"))


@pytest.mark.parametrize("name", EXP)
def test_decode_gpu_int32_matches_reference_golden(name):
    from afterimage_b200.runtime.gpu_decode import decode_gpu
    e = G.enc(name)
    got = decode_gpu(e).cpu().numpy()
    assert got.dtype == np.int32
    assert np.array_equal(got, G.arr(name, "decoded").astype(np.int32))


@pytest.mark.parametrize("block_chunks", [1, 4, 32, 128, 256])
def test_block_chunks_values_all_decode_identically(block_chunks):
    from afterimage_b200.runtime.gpu_decode_v2 import decode_gpu_v2
    e = G.enc("v2_block_sizes_64")
    got = decode_gpu_v2(e, block_chunks=block_chunks).cpu().numpy()
    assert np.array_equal(got, G.arr("v2_block_sizes_64", "decoded"))


@pytest.mark.parametrize("name", BF16)
def test_decompress_layer_matches_reference_recon(name):
    from afterimage_b200.runtime.compressed_store import decompress_layer_gpu
    layer = _layer(name)
    out = decompress_layer_gpu(layer)
    assert out.dtype == torch.bfloat16 and tuple(out.shape) == tuple(G.case(name)["shape"])
    assert np.array_equal(_bits(out), G.arr(name, "recon_bits"))


@pytest.mark.parametrize("name", ["store_128x512", "rows_200x256", "sliced_512x512", "work_chunks_37x59",
                                  "special_bits_cs5"])
@pytest.mark.parametrize("slice_elems", [7, 97, 1 << 12, 1 << 17])
def test_sliced_decompress_is_bit_identical(name, slice_elems):
    from afterimage_b200.runtime.compressed_store import decompress_layer_gpu
    layer = _layer(name)
    out = decompress_layer_gpu(layer, max_slice_elems=slice_elems, reuse_decode_tables=True)
    assert np.array_equal(_bits(out), G.arr(name, "weight_bits"))


@pytest.mark.parametrize("name", [n for n in BF16 if G.has(n, "rows_bits")])
def test_decompress_rows_matches_reference_rows(name):
    from afterimage_b200.runtime.compressed_store import decompress_rows_gpu
    c = G.case(name)
    r0, r1 = c["rows"]
    out = decompress_rows_gpu(_layer(name), r0, r1)
    assert tuple(out.shape) == (r1 - r0, c["shape"][1])
    assert np.array_equal(_bits(out), G.arr(name, "rows_bits"))


def test_rows_every_window_matches_full_decode():
    from afterimage_b200.runtime.compressed_store import decompress_layer_gpu, decompress_rows_gpu
    layer = _layer("rows_200x256")
    full = _bits(decompress_layer_gpu(layer)).reshape(200, 256)
    for r0, r1 in [(0, 1), (0, 200), (3, 4), (7, 9), (199, 200), (150, 260), (-5, 2), (50, 50)]:
        got = decompress_rows_gpu(layer, r0, r1)
        a, b = max(0, r0), min(200, r1)
        assert np.array_equal(_bits(got).reshape(-1, 256) if b > a else np.zeros((0, 256), np.int16),
                              full[a:b])


def test_rows_requires_2d():
    from afterimage_b200.runtime.compressed_store import decompress_rows_gpu
    layer = _layer("store_128x512")
    layer.shape = (128 * 512,)
    with pytest.raises(ValueError):
        decompress_rows_gpu(layer, 0, 1)


# --- oracle comparisons on seeded inputs (product encoder -> GPU vs oracle) ---

@pytest.mark.parametrize("chunk_size", [1, 5, 8, 31, 64, 100, 333, 512, 1000, 1024, 2048, 4096])
def test_gpu_matches_oracle_across_chunk_sizes(chunk_size):
    from afterimage_b200.runtime.compressed_store import compress_layer, decompress_layer_gpu
    g = torch.Generator().manual_seed(1000 + chunk_size)
    W = (torch.randn(517, 389, generator=g) * 0.02).to(torch.bfloat16)
    layer = compress_layer(W, chunk_size=chunk_size)
    got = _bits(decompress_layer_gpu(layer))
    ref = O.decompress(layer.encoded, layer.sign_mantissa.numpy()).view(np.int16)
    assert np.array_equal(got, ref)
    assert np.array_equal(got, _bits(W))


@pytest.mark.parametrize("max_bits", [1, 2, 4, 6, 8, 10, 11, 12, 13, 14, 16])
def test_gpu_matches_oracle_across_code_lengths(max_bits):
    """max_bits below, at and above the kernel's 12-bit first-level table,
    with package-merge limiting a wide skewed alphabet."""
    from afterimage_b200.runtime.gpu_decode_v2 import decode_gpu_v2
    from afterimage_b200.runtime.huffman_chunked import encode_chunked
    rng = np.random.default_rng(max_bits)
    k = 200
    p = 0.5 ** np.arange(k, dtype=np.float64)  # geometric: natural depth ~ k
    p /= p.sum()
    data = rng.choice(256, size=300_000, p=np.concatenate([p, np.zeros(56)]))
    enc = encode_chunked(data.astype(np.uint8), chunk_size=1024, max_bits=max_bits)
    assert enc.max_bits <= max_bits
    got = decode_gpu_v2(enc).cpu().numpy()
    assert np.array_equal(got, O.decode_chunked(enc))
    if (1 << max_bits) >= len(np.unique(data)):
        # a limit too small for the alphabet makes the reference encoder
        # itself lossy; GPU == oracle above still holds there
        assert np.array_equal(got, data.astype(np.uint8))


def test_gpu_matches_oracle_uniform_full_alphabet():
    from afterimage_b200.runtime.gpu_decode_v2 import decode_gpu_v2
    from afterimage_b200.runtime.huffman_chunked import encode_chunked
    data = np.random.default_rng(7).integers(0, 256, size=1_000_003).astype(np.uint8)
    enc = encode_chunked(data, chunk_size=777)
    assert np.array_equal(decode_gpu_v2(enc).cpu().numpy(), data)


@pytest.mark.parametrize("scale", [1e-6, 1e-3, 0.02, 1.0, 1e4])
def test_gpu_bf16_scales_and_specials(scale):
    from afterimage_b200.runtime.compressed_store import compress_layer, decompress_layer_gpu
    g = torch.Generator().manual_seed(int(scale * 1000) % 9973)
    W = (torch.randn(300, 1024, generator=g) * scale).to(torch.bfloat16)
    W.view(-1)[:6] = torch.tensor([0.0, -0.0, float("inf"), float("-inf"), float("nan"), 1e-40],
                                  dtype=torch.bfloat16)
    layer = compress_layer(W, chunk_size=1024)
    assert np.array_equal(_bits(decompress_layer_gpu(layer)), _bits(W))


def test_config1_recipe_encoder_digests_and_gpu_roundtrip():
    """The single-tensor round-trip case (4096x4096, seed 0) at full size: product encoder == reference encoder
    (sha256 of every array), GPU decode == input, bit for bit."""
    from afterimage_b200.runtime.compressed_store import compress_layer, decompress_layer_gpu
    c = G.case("config1_4096x4096")
    torch.manual_seed(c["seed"])
    W = (torch.randn(*c["shape"]) * c["scale"]).to(torch.bfloat16)
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    assert sha(W.view(torch.int16).numpy()) == c["sha256"]["weight_bits"], "torch RNG drifted"
    layer = compress_layer(W, chunk_size=c["chunk_size_arg"])
    enc = layer.encoded
    assert sha(enc.packed) == c["sha256"]["packed"]
    assert sha(enc.chunk_offsets) == c["sha256"]["chunk_offsets"]
    assert sha(enc.chunk_nbytes) == c["sha256"]["chunk_nbytes"]
    assert sha(enc.sym_lut) == c["sha256"]["sym_lut"]
    assert sha(enc.len_lut) == c["sha256"]["len_lut"]
    assert sha(layer.sign_mantissa.numpy()) == c["sha256"]["sign_mantissa"]
    assert enc.max_bits == c["max_bits"]
    out = decompress_layer_gpu(layer)
    assert torch.equal(out.cpu().view(torch.int16), W.view(torch.int16))


def test_nondefault_stream_and_special_bit_patterns():
    from afterimage_b200.runtime.compressed_store import compress_layer, decompress_layer_gpu
    bits = torch.tensor([0, -32768, 32640, -128, 32705, -63, 1, 127, 128,
                         16256, -16512, 32767], dtype=torch.int16).reshape(3, 4)
    layer = compress_layer(bits.view(torch.bfloat16), chunk_size=5)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        output = decompress_layer_gpu(layer, max_slice_elems=7, reuse_decode_tables=True)
    stream.synchronize()
    assert torch.equal(output.cpu().view(torch.int16), bits)


@pytest.mark.parametrize("slice_elems", [97, 1 << 20])
def test_tables_prepared_once_per_tensor_and_tensor_local(monkeypatch, slice_elems):
    from afterimage_b200.runtime import gpu_decode_v2 as gd
    from afterimage_b200.runtime.compressed_store import compress_layer, decompress_layer_gpu
    original = gd.prepare_decode_tables
    seen = []

    def prepare(enc, device="cuda"):
        seen.append(id(enc))
        return original(enc, device)

    monkeypatch.setattr(gd, "prepare_decode_tables", prepare)
    for seed, scale in [(1, .01), (2, 10.)]:
        torch.manual_seed(seed)
        weight = (torch.randn(31, 59) * scale).to(torch.bfloat16)
        layer = compress_layer(weight, chunk_size=31)
        before = len(seen)
        output = decompress_layer_gpu(layer, max_slice_elems=slice_elems, reuse_decode_tables=True)
        assert torch.equal(output.cpu().view(torch.int16), weight.view(torch.int16))
        assert len(seen) - before == 1


@pytest.mark.parametrize("value", [0, -1, 3])
def test_rejects_invalid_block_width_before_allocating(value):
    from afterimage_b200.runtime.gpu_decode_v2 import decode_gpu_v2
    with pytest.raises(ValueError, match="power of 2"):
        decode_gpu_v2(None, block_chunks=value)


def test_tables_reused_across_calls_stream_ordered():
    from afterimage_b200.runtime.gpu_decode_v2 import decode_gpu_v2, prepare_decode_tables
    e = G.enc("real_bf16_128x4096")
    t = prepare_decode_tables(e)
    a = decode_gpu_v2(e, tables=t, synchronize=False)
    b = decode_gpu_v2(e, tables=t, synchronize=False)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert np.array_equal(a.cpu().numpy(), G.arr("real_bf16_128x4096", "decoded"))


def test_tables_unpack_and_plain_pairs_work_as_in_the_reference():
    """prepare_decode_tables unpacks to (sym_lut, len_lut) as the reference's
    does (gpu_decode_v2.py:71-76, :98), and decode_gpu_v2 also takes such a
    plain pair -- int32 lengths included -- building the table block itself."""
    from afterimage_b200.runtime.gpu_decode_v2 import decode_gpu_v2, prepare_decode_tables
    e = G.enc("real_bf16_128x4096")
    sym, ln = prepare_decode_tables(e)
    got = decode_gpu_v2(e, tables=(sym, ln.to(torch.int32)))
    assert np.array_equal(got.cpu().numpy(), G.arr("real_bf16_128x4096", "decoded"))
    with pytest.raises(TypeError):
        decode_gpu_v2(e, tables=(sym,))


def test_cpu_device_raises_no_fallback():
    from afterimage_b200.runtime.compressed_store import decompress_layer_gpu
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        decompress_layer_gpu(_layer("store_128x512"), device="cpu")


# --- failure handling: host-side validation and the device status word ---

def test_corrupt_chunk_offsets_raise_instead_of_reading_out_of_bounds():
    from afterimage_b200.runtime.gpu_decode_v2 import decode_gpu_v2
    e = G.enc("real_bf16_128x4096")
    bad = G.Enc(**{**e.__dict__})
    offs = e.chunk_offsets.copy()
    offs[5] = 10 ** 9          # far past the end of packed
    offs[9] = -400
    bad.chunk_offsets = offs
    with pytest.raises(RuntimeError, match="corrupt offsets"):
        decode_gpu_v2(bad)
    # the context is still healthy afterwards
    assert np.array_equal(decode_gpu_v2(e).cpu().numpy(), G.arr("real_bf16_128x4096", "decoded"))


def test_corrupt_offsets_raise_through_the_layer_and_rows_entry_points():
    """The engine's main entry points read the status word on their
    synchronising path (the reference syncs there, gpu_decode_v2.py:115-116)."""
    from afterimage_b200.runtime.compressed_store import decompress_layer_gpu, decompress_rows_gpu
    good = _layer("sliced_512x512")
    e = good.encoded
    offs = np.asarray(e.chunk_offsets).copy()
    offs[3] = 10 ** 9
    offs[7] = -400
    bad = type(good)(sign_mantissa=good.sign_mantissa, shape=good.shape,
                     encoded=type(e)(**{**e.__dict__, "chunk_offsets": offs}))
    with pytest.raises(RuntimeError, match="corrupt offsets"):
        decompress_layer_gpu(bad, device="cuda")
    with pytest.raises(RuntimeError, match="corrupt offsets"):
        decompress_layer_gpu(bad, device="cuda", max_slice_elems=4096)   # sliced path too
    with pytest.raises(RuntimeError, match="corrupt offsets"):
        decompress_rows_gpu(bad, 0, 16, device="cuda")
    # stream-ordered table reuse does not synchronise; the error surfaces at the next check
    from afterimage_b200.runtime import _device
    decompress_layer_gpu(bad, device="cuda", reuse_decode_tables=True)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="corrupt offsets"):
        _device.check_status(torch.device("cuda", torch.cuda.current_device()))
    # the context and the status word are healthy afterwards
    assert np.array_equal(_bits(decompress_layer_gpu(good, device="cuda")), G.arr("sliced_512x512", "recon_bits"))


def _decode_unbounded(enc) -> np.ndarray:
    """The reader WITHOUT the chunk-end bound (refills from the bytes that
    follow the chunk), to show that a case depends on that bound."""
    packed = np.asarray(enc.packed)
    mb, cs = int(enc.max_bits), int(enc.chunk_size)
    out = np.zeros(enc.n_chunks * cs, dtype=np.uint8)
    for c in range(enc.n_chunks):
        pos, buf, nbits = int(enc.chunk_offsets[c]), 0, 0
        for i in range(cs):
            while nbits < mb:
                buf |= (int(packed[pos]) if pos < packed.shape[0] else 0) << (24 - nbits)
                pos += 1
                nbits += 8
            w = (buf >> (32 - mb)) & ((1 << mb) - 1)
            out[c * cs + i] = int(enc.sym_lut[w]) & 0xFF
            n = int(enc.len_lut[w])
            buf = (buf << n) & 0xFFFFFFFF
            nbits -= n
    return out[:enc.n_symbols]


@pytest.mark.parametrize("chunk_size", [16, 64, 1024])
def test_non_prefix_lut_reads_zeros_past_the_chunk_end(chunk_size):
    """A LUT whose symbol depends on every bit of the window (sym = window &
    0xFF, lengths from the real code): at each chunk's last codes the window
    reaches past the chunk's bytes into the next chunk's (non-zero) bytes.
    The reference reader shifts in zeros there (huffman_chunked.py:225-231),
    and so must the exact slow path."""
    from afterimage_b200.runtime.compressed_store import compress_layer, decompress_layer_gpu
    from afterimage_b200.runtime.gpu_decode_v2 import decode_gpu_v2
    g = torch.Generator().manual_seed(chunk_size)
    W = (torch.randn(64, 256, generator=g) * 0.02).to(torch.bfloat16)
    layer = compress_layer(W, chunk_size=chunk_size)
    e = layer.encoded
    sym = (np.arange(1 << int(e.max_bits), dtype=np.int64) & 0xFF).astype(np.int32)
    bad = type(e)(**{**e.__dict__, "sym_lut": sym})
    want = O.decode_chunked(bad)
    # the case really reads past chunk ends: the same LUT over unbounded windows differs
    assert not np.array_equal(_decode_unbounded(bad), want)
    got = decode_gpu_v2(bad).cpu().numpy()
    assert np.array_equal(got, want)
    blayer = type(layer)(sign_mantissa=layer.sign_mantissa, encoded=bad, shape=layer.shape)
    bits = _bits(decompress_layer_gpu(blayer, device="cuda"))
    assert np.array_equal(bits.view(np.uint16), O.recombine(want.astype(np.uint8), layer.sign_mantissa.numpy()))


def test_non_prefix_lut_is_flagged_and_decoded_exactly_by_the_slow_path():
    """A LUT that is not a prefix-code table (entries not replicated across
    their code's windows): the tables flag it and every lookup goes through
    the reference LUT, so the GPU still equals the oracle symbol for symbol."""
    from afterimage_b200 import _lib
    from afterimage_b200.runtime.gpu_decode_v2 import decode_gpu_v2, prepare_decode_tables
    e = G.enc("chunked_roundtrip")
    bad = G.Enc(**{**e.__dict__})
    sym = e.sym_lut.copy()
    sym[1] = (int(sym[1]) + 1) % 256   # breaks replication of window 0's code
    bad.sym_lut = sym
    t = prepare_decode_tables(bad)
    flags = ctypes.c_int32(0)
    L = _lib.load()
    _lib.check(L.aib_tables_flags(t.block.data_ptr(), ctypes.addressof(flags),
                                  torch.cuda.current_stream().cuda_stream))
    assert flags.value & _lib.STATUS_LUT_NOT_PREFIX
    got = decode_gpu_v2(bad, tables=t).cpu().numpy()
    assert np.array_equal(got, O.decode_chunked(bad))


def test_bad_descriptor_rejected_on_host():
    from afterimage_b200 import _lib
    L = _lib.load()
    d = _lib.StreamDesc()
    d.chunk_size, d.max_bits, d.n_symbols, d.elem_end = 16, 8, 100, 100
    d.packed = 1   # misaligned
    assert L.aib_decode_bf16(ctypes.byref(d), None, None) == _lib.AIB_EINVAL
    assert b"16-byte" in L.aib_last_error()


# --- direct C-ABI use: batch of tensors in one launch ---

@pytest.mark.parametrize("sizes", [(1024, 1024, 1024, 7, 1024),      # mixed: per-job loop choice
                                   (1024,) * 5,                       # all default: specialised loop
                                   (640, 1088, 64, 7, 2176),          # none default: general loop
                                   (1024, 640, 1024, 1088, 1024)])    # a TP-ready layer's mix
def test_batch_entry_point_decodes_several_tensors_in_one_launch(sizes):
    from afterimage_b200 import _lib
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.gpu_decode_v2 import prepare_decode_tables
    dev = torch.device("cuda", 0)
    shapes = [(1024, 4096), (256, 4096), (4096, 1000), (17, 3), (3072, 1024)]
    Ws, keep, descs = [], [], (_lib.StreamDesc * len(shapes))()
    for i, s in enumerate(shapes):
        g = torch.Generator().manual_seed(i)
        W = (torch.randn(*s, generator=g) * (0.02 * (i + 1))).to(torch.bfloat16)
        layer = compress_layer(W, chunk_size=sizes[i])
        t = prepare_decode_tables(layer.encoded, dev)
        ds = _device.upload_stream(layer.encoded, dev)
        sm = layer.sign_mantissa.to(dev)
        out = torch.empty(W.numel(), dtype=torch.bfloat16, device=dev)
        descs[i] = _device.make_desc(ds, t, layer.encoded, 0, W.numel(), out, sm)
        Ws.append(W)
        keep.append((t, ds, sm, out))
    L = _lib.load()
    st = _device.status_word(dev)
    _lib.check(L.aib_decode_bf16_batch(descs, len(shapes), st.data_ptr(),
                                       torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    for W, (_, _, _, out) in zip(Ws, keep):
        assert torch.equal(out.cpu().view(torch.int16), W.reshape(-1).view(torch.int16))


def test_recombine_entry_point_matches_oracle():
    from afterimage_b200.runtime.compressed_store import recombine_exponent_and_sign_mantissa
    rng = np.random.default_rng(3)
    e = rng.integers(0, 256, 100_001).astype(np.uint8)
    sm = rng.integers(0, 256, 100_001).astype(np.uint8)
    got = recombine_exponent_and_sign_mantissa(e, sm, (100_001,), "cuda")
    assert np.array_equal(_bits(got).view(np.uint16), O.recombine(e, sm))
    # unaligned views take the scalar path
    got2 = recombine_exponent_and_sign_mantissa(torch.from_numpy(e)[1:], torch.from_numpy(sm)[1:],
                                                (100_000,), "cuda")
    assert np.array_equal(_bits(got2).view(np.uint16), O.recombine(e[1:], sm[1:]))


@pytest.mark.parametrize("max_ctas", [1, 3, 7, 100])
def test_batch_decode_on_capped_ctas_is_bit_exact(max_ctas):
    """aib_decode_bf16_batch_ctas: the same batch on at most max_ctas CTAs
    (each job keeps at least one; its warps loop over more chunk groups)."""
    from afterimage_b200.runtime import _device
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.layer_decode import LayerDecoder, upload_layer
    dev = torch.device("cuda", 0)
    shapes, chunks = [(512, 2048), (64, 2048), (2048, 640), (9, 5)], [1024, 1024, 640, 3]
    Ws = []
    for i, s in enumerate(shapes):
        g = torch.Generator().manual_seed(70 + i)
        Ws.append((torch.randn(*s, generator=g) * 0.02).to(torch.bfloat16))
    resident = [upload_layer(compress_layer(W, chunk_size=c), dev, striped=(i % 2 == 0))
                for i, (W, c) in enumerate(zip(Ws, chunks))]
    dec = LayerDecoder(dev, max_ctas=max_ctas)
    outs = dec.decode(resident)
    torch.cuda.synchronize()
    _device.check_status(dev)
    assert dec.launches == 1
    for W, o in zip(Ws, outs):
        assert torch.equal(o.cpu().view(torch.int16), W.view(torch.int16))
