"""Generates tests/golden/engine_tokens_qwen3-0.6b.npz by running the
REFERENCE's own engine (afterimage/runtime/streaming_engine.py
StreamingLosslessModel, device="cpu": numba decode, transformers forward) on
the benchmark's Qwen3-0.6B-shaped configuration.

Usage: python tests/golden/make_engine_tokens_golden.py <path to an Afterimage checkout>
       (or set AFTERIMAGE_REF)

Inputs (the same as bench.py's tokens runs of this shape):
  * weights: bench.synthetic_checkpoint(cfg, seed 14) generated on the CPU
    (N(0, 0.02) matrices, unit norm weights), so a GPU box regenerates the
    very same tensors;
  * store: the reference's compress_model_to_disk, chunk_size 1024;
  * prompt: 64 ids from torch.randint(0, vocab, generator seed 64);
  * run: generate_greedy(prompt, 4) under a 1 GB VRAM budget setting.

Written arrays:
  prompt          int64 [64]
  tokens          int64 [4]       the reference's greedy tokens
  logits_bits     int16 [4, vocab] last-position BF16 logits of each step
  top2_margin     float32 [4]     top-1 minus top-2 logit of each step
  weight_sha256   bench.checkpoint_digest of the checkpoint (the test checks
                  that it regenerated the same weights)

The reference is imported read-only (no bytecode written, numba cache in a
temp dir).
"""
from __future__ import annotations

import os
import pathlib
import shutil
import sys
import tempfile

os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba_engine_golden_"))
sys.dont_write_bytecode = True

import numpy as np  # noqa: E402
import torch  # noqa: E402

REPO = pathlib.Path(__file__).resolve().parents[2]
OUT = pathlib.Path(__file__).resolve().parent / "engine_tokens_qwen3-0.6b.npz"
MODEL = "qwen3-0.6b"


def main() -> None:
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AFTERIMAGE_REF")
    if not ref:
        raise SystemExit("usage: make_engine_tokens_golden.py <Afterimage checkout>")
    sys.path.insert(0, str(REPO))
    import bench
    from safetensors.torch import save_file
    cfg, prompt_len, new_tokens, budget, _ = bench.model_config(MODEL)
    root = pathlib.Path(tempfile.mkdtemp(prefix="engine_golden_"))
    try:
        snap = root / "snapshot"
        snap.mkdir()
        items = list(bench.synthetic_checkpoint(cfg, bench.TOKENS_WEIGHT_SEED, torch.device("cpu")))
        digest = bench.checkpoint_digest(items)
        save_file({k: v.contiguous() for k, v in items}, str(snap / "model.safetensors"))
        del items
        cfg.save_pretrained(snap)
        sys.path.insert(0, str(pathlib.Path(ref).resolve()))
        from afterimage.runtime import streaming_engine as R
        model_id = "synthetic/%s-shape" % MODEL
        R.compress_model_to_disk(model_id, root / "store", config=R.EngineConfig(chunk_size=1024),
                                 progress_every=10 ** 9, source_dir=str(snap))
        prompt = torch.randint(0, cfg.vocab_size, (1, prompt_len), generator=torch.Generator().manual_seed(bench.TOKENS_PROMPT_SEED))
        eng = R.StreamingLosslessModel(model_id, root / "store", device="cpu",
                                       config=R.EngineConfig(vram_budget_gb=budget), source_dir=str(snap))
        steps = []
        inner = eng.forward_logits

        def recording(*a, **kw):
            out = inner(*a, **kw)
            steps.append(out[0, -1].detach().clone())
            return out
        eng.forward_logits = recording
        seq = eng.generate_greedy(prompt, new_tokens)
        tokens = seq[0, prompt_len:].numpy().astype(np.int64)
        logits = torch.stack(steps)
        assert logits.dtype == torch.bfloat16 and logits.shape == (new_tokens, cfg.vocab_size)
        top = torch.topk(logits.float(), 2, dim=-1).values
        np.savez_compressed(OUT, prompt=prompt[0].numpy().astype(np.int64), tokens=tokens,
                            logits_bits=logits.view(torch.int16).numpy(),
                            top2_margin=(top[:, 0] - top[:, 1]).numpy().astype(np.float32),
                            weight_sha256=np.array(digest))
        print("wrote", OUT, "tokens", tokens.tolist(), "margins", (top[:, 0] - top[:, 1]).tolist())
    finally:
        shutil.rmtree(root, ignore_errors=True)


if __name__ == "__main__":
    main()
