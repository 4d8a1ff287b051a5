"""REFERENCE ENGINE ON THE HOST CPU -- a baseline measurement, never part of
the product path and never run on a GPU box (the reference checkout is not
there).

Greedy tokens/s of the reference's own StreamingLosslessModel with
device="cpu" (numba decode, transformers forward) on one of the benchmark's
decoder shapes. The checkpoint is random N(0, 0.02) BF16 weights of that
shape, generated on the CPU with the same seeds as bench.py's tokens runs.
It is compressed by the reference's compress_model_to_disk and decoded under
the configuration's VRAM budget setting. The prompt is uniform ids; the
forced greedy tokens are the configuration's count.

Usage (in a container that has an Afterimage checkout):

    python tests/golden/measure_ref_engine_tokens_cpu.py <path to the checkout> [--model qwen3-0.6b]

Prints one JSON line: tokens/s, s/token, torch threads, compression time.
The reference is imported read-only (no bytecode written, numba cache in a
temp dir).
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import shutil
import sys
import tempfile
import time

os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
os.environ.setdefault("NUMBA_CACHE_DIR", tempfile.mkdtemp(prefix="numba_ref_engine_"))
sys.dont_write_bytecode = True

import torch  # noqa: E402

REPO = pathlib.Path(__file__).resolve().parents[2]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("checkout")
    ap.add_argument("--model", default="qwen3-0.6b")
    args = ap.parse_args()
    sys.path.insert(0, str(REPO))
    import bench
    from safetensors.torch import save_file
    cfg, prompt_len, new_tokens, budget, label = bench.model_config(args.model)
    root = pathlib.Path(tempfile.mkdtemp(prefix="ref_engine_cpu_"))
    try:
        snap = root / "snapshot"
        snap.mkdir()
        sd = dict(bench.synthetic_checkpoint(cfg, 14, torch.device("cpu")))
        if getattr(cfg, "tie_word_embeddings", False):
            sd.pop("lm_head.weight", None)
        save_file({k: v.contiguous() for k, v in sd.items()}, str(snap / "model.safetensors"))
        del sd
        cfg.save_pretrained(snap)
        sys.path.insert(0, str(pathlib.Path(args.checkout).resolve()))
        from afterimage.runtime import streaming_engine as ref
        model_id = "synthetic/%s-shape" % args.model
        t0 = time.perf_counter()
        ref.compress_model_to_disk(model_id, root / "store", config=ref.EngineConfig(chunk_size=1024),
                                   progress_every=10 ** 9, source_dir=str(snap))
        compress_s = time.perf_counter() - t0
        prompt = torch.randint(0, cfg.vocab_size, (1, prompt_len), generator=torch.Generator().manual_seed(64))
        eng = ref.StreamingLosslessModel(model_id, root / "store", device="cpu",
                                         config=ref.EngineConfig(vram_budget_gb=budget), source_dir=str(snap))
        eng.generate_greedy(prompt, 1)  # warm: numba JIT, allocator
        t0 = time.perf_counter()
        eng.generate_greedy(prompt, new_tokens)
        dt = time.perf_counter() - t0
        print(json.dumps({"impl": "reference engine, device=cpu", "model": label, "prompt_tokens": prompt_len,
                          "new_tokens": new_tokens, "vram_budget_gb": budget,
                          "tokens_per_s": round(new_tokens / dt, 4), "s_per_token": round(dt / new_tokens, 3),
                          "torch_threads": torch.get_num_threads(), "compress_s": round(compress_s, 1)}),
              flush=True)
    finally:
        shutil.rmtree(root, ignore_errors=True)


if __name__ == "__main__":
    main()
