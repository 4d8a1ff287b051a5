"""Generates tests/golden/ref_store/ by running the REFERENCE's offline
compressor (afterimage/runtime/streaming_engine.py compress_model_to_disk)
on a small seeded Qwen3-shaped checkpoint, untied and tied.

Usage: python tests/golden/make_store_golden.py <path to an Afterimage checkout>
       (or set AFTERIMAGE_REF)

Written files:
  model.safetensors            the checkpoint (the tied variant is the same
                               tensors without lm_head.weight)
  config_untied.json / config_tied.json
  manifest_untied.json / manifest_tied.json   the reference's manifests
  digests.json                 sha256 and size of the reference's weights.bin
                               for each variant

The reference is imported read-only (no bytecode written, numba cache in a
temp dir) and run with one worker.
"""
from __future__ import annotations

import hashlib
import json
import os
import pathlib
import shutil
import sys
import tempfile

os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba_store_golden_"))
sys.dont_write_bytecode = True

import torch  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent / "ref_store"
CHUNK_SIZE = 256
SHAPE = dict(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=2,
             num_key_value_heads=1, head_dim=32, max_position_embeddings=64)


def checkpoint():
    from transformers import AutoModelForCausalLM, Qwen3Config
    torch.manual_seed(5)
    model = AutoModelForCausalLM.from_config(Qwen3Config(**SHAPE, tie_word_embeddings=False), dtype=torch.bfloat16)
    with torch.no_grad():
        for p in model.parameters():
            if p.dim() == 2:
                p.normal_(0, 0.02)
    return {k: v.contiguous() for k, v in model.state_dict().items()}


def snapshot(dst: pathlib.Path, tie: bool) -> None:
    """A checkpoint directory for one variant, from the committed files."""
    dst.mkdir(parents=True, exist_ok=True)
    shutil.copy(OUT / "model.safetensors", dst / "model.safetensors")
    if tie:
        from safetensors.torch import load_file, save_file
        sd = load_file(str(dst / "model.safetensors"))
        sd.pop("lm_head.weight")
        save_file(sd, str(dst / "model.safetensors"))
    shutil.copy(OUT / ("config_%s.json" % ("tied" if tie else "untied")), dst / "config.json")


def main() -> None:
    from safetensors.torch import save_file
    from transformers import Qwen3Config
    root = pathlib.Path(sys.argv[1] if len(sys.argv) > 1 else os.environ["AFTERIMAGE_REF"])
    sys.path.insert(0, str(root))
    from afterimage.runtime import streaming_engine as ref
    OUT.mkdir(exist_ok=True)
    save_file(checkpoint(), str(OUT / "model.safetensors"))
    digests = {}
    with tempfile.TemporaryDirectory() as tmp:
        for tie in (False, True):
            tag = "tied" if tie else "untied"
            (OUT / ("config_%s.json" % tag)).write_text(
                Qwen3Config(**SHAPE, tie_word_embeddings=tie).to_json_string())
            snap = pathlib.Path(tmp) / ("snap_" + tag)
            snapshot(snap, tie)
            store = pathlib.Path(tmp) / ("store_" + tag)
            ref.compress_model_to_disk("golden/tiny-qwen3", store, config=ref.EngineConfig(chunk_size=CHUNK_SIZE),
                                       progress_every=10 ** 9, source_dir=str(snap), max_workers=1)
            shutil.copy(store / "manifest.json", OUT / ("manifest_%s.json" % tag))
            blob = (store / "weights.bin").read_bytes()
            digests[tag] = {"sha256": hashlib.sha256(blob).hexdigest(), "bytes": len(blob)}
    (OUT / "digests.json").write_text(json.dumps({"chunk_size": CHUNK_SIZE, "model_id": "golden/tiny-qwen3",
                                                  **digests}, indent=1))
    print("wrote", OUT, digests)


if __name__ == "__main__":
    main()
