"""Offline compression and store checks that need no GPU: the store layout
follows the reference's per-tensor rules (streaming_engine.py:158-253,
:362-427), every compressed tensor round-trips through the oracle, and the
engine refuses bad stores before touching a device."""
import json
import shutil

import numpy as np
import pytest
import torch

from test_streaming_engine_gpu import _store, _tiny
from oracle import oracle as O
from afterimage_b200.runtime.binstore import BinaryWeightReader
from afterimage_b200.runtime.huffman_chunked import ChunkedEncoded


@pytest.fixture(scope="module")
def untied_store(tmp_path_factory):
    tmp = tmp_path_factory.mktemp("store")
    cfg, model = _tiny(tie=False, seed=1)
    snap, store, manifest = _store(tmp, cfg, model, "u")
    return cfg, model, snap, store, manifest


def test_store_layout_matches_reference_rules(untied_store):
    cfg, model, snap, store, m = untied_store
    assert m["schema_version"] == 2 and m["tied"] is False
    t = m["tensors"]
    assert t["model.embed_tokens.weight"]["row_gather"] is True
    assert t["model.embed_tokens.weight"]["hidden_size"] == cfg.hidden_size
    assert t["model.layers.0.mlp.gate_proj.weight"]["compressed"] is True
    assert t["model.layers.0.self_attn.k_proj.weight"]["compressed"] is False  # 160x320 <= 65536
    assert t["model.layers.0.input_layernorm.weight"]["dtype"] == "torch.bfloat16"
    assert set(t["model.layers.0.mlp.gate_proj.weight"]["blobs"]) == {
        "sign_mantissa", "packed", "chunk_offsets", "chunk_nbytes", "sym_lut", "len_lut"}
    assert m["total_orig_bytes"] == sum(v["orig_bytes"] for v in t.values())


def test_every_stored_tensor_round_trips_through_the_oracle(untied_store):
    cfg, model, snap, store, m = untied_store
    sd = model.state_dict()
    with BinaryWeightReader(store / "weights.bin") as r:
        for key, meta in m["tensors"].items():
            blobs = {n: r.read(ref, verify=True) for n, ref in meta["blobs"].items()}
            want = sd[key].view(torch.int16).reshape(-1).numpy()
            if meta.get("compressed"):
                n = meta["n_symbols"]
                enc = ChunkedEncoded(packed=blobs["packed"], chunk_offsets=blobs["chunk_offsets"],
                                     chunk_nbytes=blobs["chunk_nbytes"], sym_lut=blobs["sym_lut"],
                                     len_lut=blobs["len_lut"], max_bits=meta["max_bits"],
                                     chunk_size=meta["chunk_size"], n_symbols=n, shape=(n,))
                got = O.decompress(enc, blobs["sign_mantissa"]).view(np.int16)
            elif meta.get("row_gather"):
                got = blobs["raw"].reshape(-1)
            else:
                got = torch.from_numpy(blobs["raw"]).to(torch.bfloat16).view(torch.int16).reshape(-1).numpy()
            assert np.array_equal(got, want), key


def test_engine_rejects_bad_schema_and_truncated_store_before_any_device_use(untied_store, tmp_path):
    from afterimage_b200.runtime.streaming_engine import StreamingLosslessModel
    cfg, model, snap, store, _ = untied_store
    bad = tmp_path / "bad"
    shutil.copytree(store, bad)
    m = json.loads((bad / "manifest.json").read_text())
    m["schema_version"] = 1
    (bad / "manifest.json").write_text(json.dumps(m))
    with pytest.raises(RuntimeError, match="schema_version"):
        StreamingLosslessModel(str(snap), bad)
    m["schema_version"] = 2
    (bad / "manifest.json").write_text(json.dumps(m))
    with open(bad / "weights.bin", "r+b") as f:
        f.truncate(100)
    with pytest.raises(RuntimeError, match="truncated"):
        StreamingLosslessModel(str(snap), bad)


def test_engine_config_validation():
    """The reference's rules (config.py:412-511) for the fields this engine
    keeps, including the decode and read knobs that change no values."""
    from afterimage_b200.runtime.streaming_engine import EngineConfig
    for bad in (dict(chunk_size=0), dict(max_bits=17), dict(io_prefetch_depth=-1),
                dict(ram_tier_format="x"), dict(vram_tier_format="y"), dict(ram_budget_gb=1.0),
                dict(block_chunks=24), dict(storage_read_policy="x"), dict(storage_extent_max_bytes=0),
                dict(storage_extent_max_gap_bytes=-1), dict(max_context=16), dict(max_context=0, vram_budget_gb=1.0),
                dict(vram_safety_margin_gb=0.5), dict(vram_safety_margin_gb=-1.0, vram_budget_gb=1.0),
                dict(empty_cache_every=-1), dict(require_pinned_ram=True),
                dict(require_pinned_ram=True, vram_budget_gb=1.0, ram_budget_gb=1.0, ram_tier_format="compressed"),
                dict(placement_policy="nope"), dict(placement_policy="critical_path", vram_budget_gb=1.0)):
        with pytest.raises(ValueError):
            EngineConfig(**bad)
    EngineConfig(block_chunks=128, storage_read_policy="tensor_extents", vram_budget_gb=2.0,
                 vram_safety_margin_gb=0.25, max_context=512, empty_cache_every=8, progress=True,
                 ram_budget_gb=1.0, require_pinned_ram=True)


@pytest.mark.parametrize("policy", ["per_blob", "tensor_extents", "coalesced_extents"])
def test_read_policies_change_reads_not_bytes(untied_store, policy):
    """storage_read_policy: one read per stored array, per tensor, or per
    group of adjacent tensors -- the arrays are the same every time."""
    import types
    from afterimage_b200.runtime.streaming_engine import EngineConfig, StreamingLosslessModel, StreamStats
    cfg, model, snap, store, m = untied_store
    keys = [k for k in m["tensors"] if k.startswith("model.layers.0.")]  # one layer: contiguous in the file
    blobs = sum(len(m["tensors"][k]["blobs"]) for k in keys)
    eng = types.SimpleNamespace(manifest=m, config=EngineConfig(storage_read_policy=policy), stats=StreamStats())
    ref = types.SimpleNamespace(manifest=m, config=EngineConfig(storage_read_policy="per_blob"), stats=StreamStats())
    with BinaryWeightReader(store / "weights.bin") as r:
        got = StreamingLosslessModel._read_arrays(eng, keys, r, False)
        want = StreamingLosslessModel._read_arrays(ref, keys, r, False)
    calls = eng.stats.storage_read_calls
    assert calls == {"per_blob": blobs, "tensor_extents": len(keys), "coalesced_extents": 1}[policy]
    for k in keys:
        for name in want[k]:
            assert np.array_equal(np.asarray(got[k][name]), np.asarray(want[k][name])), (k, name)


def test_compress_calls_control_per_tensor_and_cancels(tmp_path):
    """compress_model_to_disk keeps the reference's parameters: `control`
    (a pause/cancel hook with checkpoint()) runs before each tensor, and an
    exception from it stops the write; `max_workers` is checked."""
    from afterimage_b200.runtime.streaming_engine import EngineConfig, compress_model_to_disk

    class Control:
        def __init__(self, cancel_at=None):
            self.calls, self.cancel_at = 0, cancel_at

        def checkpoint(self):
            self.calls += 1
            if self.cancel_at is not None and self.calls >= self.cancel_at:
                raise KeyboardInterrupt("cancelled")

    cfg, model = _tiny(tie=False, seed=4)
    snap, store, m = _store(tmp_path, cfg, model, "c")
    ctl = Control()
    m2 = compress_model_to_disk("tiny", tmp_path / "again", EngineConfig(chunk_size=256), 0, 2, ctl, str(snap))
    assert ctl.calls == len(m2["tensors"]) == len(m["tensors"])
    assert (tmp_path / "again" / "weights.bin").read_bytes() == (store / "weights.bin").read_bytes()
    with pytest.raises(KeyboardInterrupt):
        compress_model_to_disk("tiny", tmp_path / "cancelled", EngineConfig(chunk_size=256), control=Control(3),
                               source_dir=str(snap))
    assert not (tmp_path / "cancelled" / "manifest.json").exists()
    with pytest.raises(ValueError, match="max_workers"):
        compress_model_to_disk("tiny", tmp_path / "bad", max_workers=0, source_dir=str(snap))


def test_engine_config_contract_round_trip_and_fingerprint():
    """is_lossless / exactness_contract / describe / to_dict / from_dict /
    fingerprint as in the reference (config.py:575-628), for the modes this
    package builds."""
    from afterimage_b200.runtime.config import EngineConfig
    cfg = EngineConfig()
    assert cfg.quantize is None and cfg.is_lossless and cfg.exactness_contract == "reference_execution_equivalent"
    assert cfg.describe() == "LOSSLESS (bit-exact output) | residency: legacy fixed policy"
    chunked = EngineConfig(lm_head_slice_rows=4096, vram_budget_gb=4.0, ram_budget_gb=2.0, io_prefetch_depth=2)
    assert not chunked.is_lossless and chunked.exactness_contract == "approximate"
    assert chunked.describe() == ("LOSSY: lm_head_slice_rows=4096 -- output is NOT bit-exact | residency: "
                                  "VRAM 4.00 GB + RAM 2.00 GB | io_prefetch_depth=2")
    again = EngineConfig.from_dict(chunked.to_dict())
    assert again == chunked and again.fingerprint() == chunked.fingerprint() != cfg.fingerprint()
    assert len(cfg.fingerprint()) == 16 and int(cfg.fingerprint(), 16) >= 0
    with pytest.raises(ValueError, match="unknown EngineConfig fields: draft_mode"):
        EngineConfig.from_dict({**cfg.to_dict(), "draft_mode": "model"})
    for bad in (dict(spec_k=0), dict(quantize="q8")):
        with pytest.raises(ValueError):
            EngineConfig(**bad)


def test_progress_lines_only_when_asked(capsys):
    """EngineConfig.progress: one stderr line per generated token, ended by
    a newline; silent otherwise."""
    import time
    import types
    from afterimage_b200.runtime.streaming_engine import EngineConfig, StreamingLosslessModel
    quiet = types.SimpleNamespace(config=EngineConfig())
    loud = types.SimpleNamespace(config=EngineConfig(progress=True))
    t0 = time.perf_counter()
    StreamingLosslessModel._progress(quiet, 1, 3, t0)
    assert capsys.readouterr().err == ""
    for i in (1, 2, 3):
        StreamingLosslessModel._progress(loud, i, 3, t0)
    StreamingLosslessModel._progress(loud, None, 3, t0)
    err = capsys.readouterr().err
    assert err.count("[afterimage_b200] token") == 3 and "token 3/3" in err and err.endswith("\n")
