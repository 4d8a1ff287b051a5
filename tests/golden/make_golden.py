"""Generates the golden fixtures in this directory by running the REFERENCE
implementation (Afterimage 0.3.0's own encoder and decoders).

Run where a checkout of the reference is available:

    python tests/golden/make_golden.py /path/to/afterimage-checkout
    (or set AFTERIMAGE_REF to that path)

It imports the reference read-only (no bytecode written, numba cache
redirected to a temp dir) and writes:

  cases.npz        -- every small case: the reference's encoder output
                      (packed / chunk_offsets / chunk_nbytes / sym_lut /
                      len_lut / max_bits / chunk_size / n_symbols / shape),
                      the reference decoders' outputs and, for weight cases,
                      sign_mantissa and the reconstructed bf16 bits.
  manifest.json    -- case list with metadata; large cases (config-1 size)
                      are recorded as a recipe plus sha256 digests of the
                      reference encoder's arrays, so a test can regenerate
                      the input with torch's seeded CPU generator, encode it
                      with the product encoder and compare digests.

The inputs mirror the reference's own hot-path tests (tests/test_huffman.py,
test_huffman_chunked.py, test_gpu_decode.py, test_gpu_decode_v2.py,
test_cpu_decode.py, test_compressed_store.py, test_sliced_decompress.py,
test_decode_table_reuse.py) plus the benchmark's config-1 tensor.
"""
from __future__ import annotations

import hashlib
import json
import os
import pathlib
import sys
import tempfile

os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba_golden_"))
sys.dont_write_bytecode = True

_ref_arg = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AFTERIMAGE_REF")
if not _ref_arg:
    raise SystemExit("usage: make_golden.py <path to an Afterimage checkout> (or set AFTERIMAGE_REF)")
REF = pathlib.Path(_ref_arg)
sys.path.insert(0, str(REF))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from afterimage.runtime import compressed_store as cs  # noqa: E402
from afterimage.runtime import cpu_decode  # noqa: E402
from afterimage.runtime import huffman_chunked as hc  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def bf16_exponents(W: torch.Tensor) -> torch.Tensor:
    bits = W.contiguous().view(torch.int16).to(torch.int32) & 0xFFFF
    return ((bits >> 7) & 0xFF).flatten()


arrays: dict[str, np.ndarray] = {}
manifest: dict = {"generator": "tests/golden/make_golden.py",
                  "reference": "afterimage-llm 0.3.0 (afterimage/runtime)",
                  "torch": torch.__version__, "numpy": np.__version__,
                  "cases": []}


def put_enc(name: str, enc) -> dict:
    arrays[f"{name}/packed"] = np.asarray(enc.packed, dtype=np.uint8)
    arrays[f"{name}/chunk_offsets"] = np.asarray(enc.chunk_offsets, dtype=np.int32)
    arrays[f"{name}/chunk_nbytes"] = np.asarray(enc.chunk_nbytes, dtype=np.int32)
    arrays[f"{name}/sym_lut"] = np.asarray(enc.sym_lut, dtype=np.int32)
    arrays[f"{name}/len_lut"] = np.asarray(enc.len_lut, dtype=np.int8)
    return {"max_bits": int(enc.max_bits), "chunk_size": int(enc.chunk_size),
            "n_symbols": int(enc.n_symbols), "enc_shape": list(enc.shape),
            "n_chunks": int(enc.n_chunks)}


def exp_case(name: str, symbols: torch.Tensor, chunk_size: int, max_bits: int = 16,
             note: str = ""):
    """Exponent-stream case: reference encode_chunked + both CPU decoders."""
    enc = hc.encode_chunked(symbols, chunk_size=chunk_size, max_bits=max_bits)
    meta = {"name": name, "kind": "exponents", "chunk_size_arg": chunk_size,
            "max_bits_arg": max_bits, "note": note}
    meta.update(put_enc(name, enc))
    sym_np = symbols.flatten().cpu().numpy()
    arrays[f"{name}/symbols"] = sym_np.astype(np.uint8)  # every symbol is < 256
    arrays[f"{name}/symbols_dtype_uint8"] = np.array([symbols.dtype == torch.uint8])
    ref = hc.decode_chunked_cpu_reference(enc)
    assert np.array_equal(ref, sym_np)
    arrays[f"{name}/decoded"] = ref.astype(np.uint8)
    if enc.n_chunks:
        # full chunk_size output per chunk, padding symbols included
        arrays[f"{name}/numba_full"] = cpu_decode.decode_chunks_numba(enc)
    manifest["cases"].append(meta)


def weight_case(name: str, W: torch.Tensor, chunk_size: int = 1024,
                work_chunk_elems: int = 1 << 24, rows: tuple | None = None,
                slices: tuple = (), note: str = ""):
    """BF16 weight case: reference compress_layer + CPU reference decompress,
    plus the numba-backed sliced/rows paths where asked."""
    layer = cs.compress_layer(W, chunk_size=chunk_size, work_chunk_elems=work_chunk_elems)
    meta = {"name": name, "kind": "bf16", "shape": list(W.shape),
            "chunk_size_arg": chunk_size, "compressed_bytes": int(layer.compressed_bytes),
            "original_bytes": int(layer.original_bytes), "note": note}
    meta.update(put_enc(name, layer.encoded))
    arrays[f"{name}/weight_bits"] = W.contiguous().view(torch.int16).flatten().numpy().copy()
    arrays[f"{name}/sign_mantissa"] = layer.sign_mantissa.numpy().copy()
    recon = cs.decompress_layer_cpu_reference(layer)
    assert torch.equal(recon.view(torch.int16), W.view(torch.int16))
    arrays[f"{name}/recon_bits"] = recon.contiguous().view(torch.int16).flatten().numpy().copy()
    if rows is not None:
        r0, r1 = rows
        got = cs.decompress_rows_gpu(layer, r0, r1, device="cpu")
        arrays[f"{name}/rows_bits"] = got.contiguous().view(torch.int16).flatten().numpy().copy()
        meta["rows"] = [r0, r1]
    meta["slices"] = []
    for s in slices:
        got = cs.decompress_layer_gpu(layer, device="cpu", max_slice_elems=s)
        assert torch.equal(got.view(torch.int16), W.view(torch.int16))
        meta["slices"].append(int(s))
    manifest["cases"].append(meta)


def hash_case(name: str, seed: int, shape: tuple, scale: float, chunk_size: int,
              note: str = ""):
    """Large case kept as a recipe + digests of the reference's arrays."""
    torch.manual_seed(seed)
    W = (torch.randn(*shape) * scale).to(torch.bfloat16)
    layer = cs.compress_layer(W, chunk_size=chunk_size)
    enc = layer.encoded
    recon = cs.decompress_layer_gpu(layer, device="cpu")
    assert torch.equal(recon.view(torch.int16), W.view(torch.int16))
    manifest["cases"].append({
        "name": name, "kind": "bf16_recipe", "seed": seed, "shape": list(shape),
        "scale": scale, "chunk_size_arg": chunk_size, "note": note,
        "max_bits": int(enc.max_bits), "chunk_size": int(enc.chunk_size),
        "n_symbols": int(enc.n_symbols), "n_chunks": int(enc.n_chunks),
        "compressed_bytes": int(layer.compressed_bytes),
        "distinct_symbols": len(set(enc.sym_lut[enc.len_lut > 0].tolist())),
        "sha256": {
            "weight_bits": sha(W.contiguous().view(torch.int16).numpy()),
            "sign_mantissa": sha(layer.sign_mantissa.numpy()),
            "packed": sha(enc.packed), "chunk_offsets": sha(enc.chunk_offsets.astype(np.int32)),
            "chunk_nbytes": sha(enc.chunk_nbytes.astype(np.int32)),
            "sym_lut": sha(enc.sym_lut.astype(np.int32)),
            "len_lut": sha(enc.len_lut.astype(np.int8)),
        },
        "packed_nbytes": int(enc.packed.nbytes),
    })


def main():
    # --- exponent streams (test_huffman_chunked.py, test_gpu_decode*.py) ---
    torch.manual_seed(0)
    exp_case("chunked_roundtrip", torch.randint(100, 140, (10000,)), 256)
    torch.manual_seed(10)
    exp_case("uint8_input", torch.randint(0, 256, (4099,), dtype=torch.uint8), 127)
    torch.manual_seed(1)
    exp_case("nondividing_300", torch.randint(100, 140, (10007,)), 300)
    torch.manual_seed(2)
    exp_case("full_alphabet_128", torch.randint(0, 256, (5000,)), 128)
    torch.manual_seed(3)
    exp_case("reader_margin_64", torch.randint(0, 256, (3000,)), 64)
    torch.manual_seed(4)
    exp_case("real_bf16_128x4096", bf16_exponents((torch.randn(128, 4096) * 0.02).to(torch.bfloat16)), 512)
    torch.manual_seed(5)
    exp_case("tiny_chunks_16", torch.randint(50, 80, (2000,)), 16)
    torch.manual_seed(0)
    exp_case("v2_block_sizes_64", torch.randint(100, 140, (20000,)), 64)
    torch.manual_seed(1)
    exp_case("v2_masked_tail_100", torch.randint(0, 256, (7777,)), 100)
    torch.manual_seed(0)
    exp_case("v1_skewed_64", torch.randint(100, 140, (2000,)), 64)
    torch.manual_seed(1)
    exp_case("v1_uniform_256", torch.randint(0, 256, (8000,)), 256)
    torch.manual_seed(3)
    e = torch.randint(50, 90, (10000,))
    for c in (32, 128, 512, 1024):
        exp_case(f"v1_chunk_{c}", e, c)
    torch.manual_seed(4)
    exp_case("v1_nondividing_333", torch.randint(0, 200, (7777,)), 333)
    exp_case("single_symbol", torch.full((5000,), 42, dtype=torch.int64), 256)
    exp_case("two_symbol_skew", torch.from_numpy(
        np.random.default_rng(5).choice([10, 200], size=6000, p=[0.99, 0.01])), 256)
    for seed in range(8):
        rng = np.random.default_rng(seed)
        k = rng.integers(2, 200)
        probs = rng.dirichlet(np.ones(k) * rng.uniform(0.1, 3.0))
        data = rng.choice(k, size=rng.integers(2000, 8000), p=probs)
        exp_case(f"dirichlet_{seed}", torch.from_numpy(data.astype(np.int64)), 256)
    # Fibonacci-weighted alphabet: natural Huffman depth > 16, so the
    # reference's package-merge length limiting is exercised.
    fib = [1, 1]
    while len(fib) < 26:
        fib.append(fib[-1] + fib[-2])
    fib_data = np.concatenate([np.full(f, 60 + i, dtype=np.int64) for i, f in enumerate(fib)])
    np.random.default_rng(11).shuffle(fib_data)
    exp_case("fibonacci_limit16", torch.from_numpy(fib_data), 1024)
    exp_case("fibonacci_limit6", torch.from_numpy(fib_data[:20000]), 512, max_bits=6)
    for c, mb in ((32, 8), (1024, 8), (128, 12), (1024, 12)):
        torch.manual_seed(100 + c + mb)
        w = (torch.randn(80_000) * 0.02).to(torch.bfloat16)
        bits = w.view(torch.int16).to(torch.int32) & 0xFFFF
        exp_case(f"maxbits_{mb}_cs{c}", (bits >> 7) & 0xFF, c, max_bits=mb)
    exp_case("empty", torch.zeros(0, dtype=torch.int64), 1024)
    exp_case("one_symbol_total", torch.tensor([127], dtype=torch.int64), 1024)
    exp_case("fewer_than_chunk", torch.randint(120, 124, (700,)), 1024)

    # --- bf16 weights (test_compressed_store.py, test_sliced_decompress.py,
    #     test_decode_table_reuse.py) ---
    torch.manual_seed(0)
    weight_case("store_128x512", (torch.randn(128, 512) * 0.02).to(torch.bfloat16), 256)
    torch.manual_seed(40)
    weight_case("work_chunks_37x59", (torch.randn(37, 59) * 0.02).to(torch.bfloat16), 31,
                work_chunk_elems=17)
    torch.manual_seed(1)
    for scale in (0.001, 0.02, 0.5, 3.0):
        weight_case(f"scale_{scale}", (torch.randn(64, 256) * scale).to(torch.bfloat16))
    weight_case("special_values", torch.tensor(
        [0.0, -0.0, 1.0, -1.0, 1e-30, -1e-30, 1e30, -1e30, 3.14159],
        dtype=torch.bfloat16).reshape(3, 3), 9)
    torch.manual_seed(3)
    for shape in ((1, 100), (100, 1), (7, 13)):
        weight_case("shape_%dx%d" % shape, (torch.randn(*shape) * 0.02).to(torch.bfloat16), 512)
    bits = torch.tensor([0, -32768, 32640, -128, 32705, -63, 1, 127, 128,
                         16256, -16512, 32767], dtype=torch.int16).reshape(3, 4)
    weight_case("special_bits_cs5", bits.view(torch.bfloat16), 5)
    for seed, scale in ((1, .01), (2, 10.)):
        torch.manual_seed(seed)
        weight_case(f"table_reuse_{seed}", (torch.randn(31, 59) * scale).to(torch.bfloat16), 31)
    torch.manual_seed(22)
    weight_case("rows_200x256", (torch.randn(200, 256) * 0.02).to(torch.bfloat16), 64,
                rows=(30, 90))
    torch.manual_seed(21)
    weight_case("sliced_512x512", (torch.randn(512, 512) * 0.02).to(torch.bfloat16), 1024,
                slices=(1 << 30, 1 << 17), rows=(100, 333))
    weight_case("all_zero", torch.zeros(64, 64, dtype=torch.bfloat16), 1024)

    # --- large cases as recipes + digests ---
    hash_case("config1_4096x4096", 0, (4096, 4096), 0.02, 1024,
              note="BASELINE config 1: 4096x4096 N(0,0.02) seed 0, chunk_size 1024")
    hash_case("sliced_4096x512", 1, (4096, 512), 0.02, 1024,
              note="test_sliced_decompress.py::test_sliced_gpu_decompress_matches_unsliced_bit_exact")
    hash_case("v2_real_512x4096", 2, (512, 4096), 0.02, 512,
              note="test_gpu_decode_v2.py::test_real_bf16_exponent_distribution (exponent stream)")

    np.savez_compressed(OUT / "cases.npz", **arrays)
    (OUT / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print("wrote %d cases, %d arrays, %.1f KB" % (
        len(manifest["cases"]), len(arrays), (OUT / "cases.npz").stat().st_size / 1024))


if __name__ == "__main__":
    main()
