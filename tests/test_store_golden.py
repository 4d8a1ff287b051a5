"""The offline compressor against the reference's own output
(tests/golden/ref_store/, written by make_store_golden.py with the
reference's compress_model_to_disk): on the same checkpoint, untied and
tied, this package writes a byte-identical weights.bin and the same
manifest, so either engine reads either store. Every stored tensor then
decodes through the oracle to the checkpoint's exact bits."""
import hashlib
import json
import pathlib
import shutil

import numpy as np
import pytest
import torch
from safetensors.torch import load_file, save_file

from oracle import oracle as O
from afterimage_b200.runtime.binstore import BinaryWeightReader
from afterimage_b200.runtime.huffman_chunked import ChunkedEncoded
from afterimage_b200.runtime.streaming_engine import EngineConfig, _raw_tensor, compress_model_to_disk

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden" / "ref_store"
DIGESTS = json.loads((GOLDEN / "digests.json").read_text())


def _snapshot(dst: pathlib.Path, tag: str) -> dict:
    dst.mkdir(parents=True)
    sd = load_file(str(GOLDEN / "model.safetensors"))
    if tag == "tied":
        sd.pop("lm_head.weight")
    save_file(sd, str(dst / "model.safetensors"))
    shutil.copy(GOLDEN / ("config_%s.json" % tag), dst / "config.json")
    return sd


@pytest.mark.parametrize("tag", ["untied", "tied"])
def test_store_is_byte_identical_to_the_reference(tmp_path, tag):
    sd = _snapshot(tmp_path / "snap", tag)
    store = tmp_path / "store"
    m = compress_model_to_disk(DIGESTS["model_id"], store, config=EngineConfig(chunk_size=DIGESTS["chunk_size"]),
                               progress_every=0, source_dir=str(tmp_path / "snap"))
    ref_manifest = json.loads((GOLDEN / ("manifest_%s.json" % tag)).read_text())
    assert json.loads((store / "manifest.json").read_text()) == ref_manifest
    assert m["tensors"].keys() == ref_manifest["tensors"].keys()
    blob = (store / "weights.bin").read_bytes()
    assert len(blob) == DIGESTS[tag]["bytes"]
    assert hashlib.sha256(blob).hexdigest() == DIGESTS[tag]["sha256"]

    # the reference's manifest, read through this package's reader and decoded
    # by the oracle, gives back the checkpoint's bits
    with BinaryWeightReader(store / "weights.bin") as reader:
        for key, meta in ref_manifest["tensors"].items():
            want = sd[key].view(torch.int16).numpy().reshape(-1)
            blobs = {n: reader.read(ref) for n, ref in meta["blobs"].items()}
            if not meta["compressed"]:
                got = _raw_tensor(meta, blobs["raw"]).view(torch.int16).reshape(-1).numpy()
                assert np.array_equal(got, want), key
                continue
            enc = ChunkedEncoded(packed=blobs["packed"], chunk_offsets=blobs["chunk_offsets"],
                                 chunk_nbytes=blobs["chunk_nbytes"], sym_lut=blobs["sym_lut"],
                                 len_lut=blobs["len_lut"], max_bits=int(meta["max_bits"]),
                                 chunk_size=int(meta["chunk_size"]), n_symbols=int(meta["n_symbols"]),
                                 shape=(int(meta["n_symbols"]),))
            got = O.decompress(enc, blobs["sign_mantissa"]).view(np.int16)
            assert np.array_equal(got.reshape(-1), want), key
    assert ("lm_head.weight" in ref_manifest["tensors"]) == (tag == "untied")
