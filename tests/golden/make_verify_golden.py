"""Generates tests/golden/verify_cases.pt by running the REFERENCE's
speculative-verification helpers (afterimage/runtime/verify.py:
sample_categorical, temperature_probs, speculative_sample_step) on seeded
inputs: float32 and bfloat16 logits, temperatures at, below and above zero,
chains where the draft equals the target, disagrees with it, or dominates
it everywhere, each with its own seeded CPU generator.

Usage: python tests/golden/make_verify_golden.py <path to an Afterimage checkout>
       (or set AFTERIMAGE_REF)

The reference module imports only torch; it is loaded read-only from its
file (no bytecode written).
"""
from __future__ import annotations

import importlib.util
import os
import pathlib
import sys

sys.dont_write_bytecode = True

import torch  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent / "verify_cases.pt"
VOCAB = 48
TEMPS = (0.0, -1.0, 0.5, 1.0, 1.7)
DTYPES = (torch.float32, torch.bfloat16)


def load_reference(root: pathlib.Path):
    path = root / "afterimage" / "runtime" / "verify.py"
    spec = importlib.util.spec_from_file_location("afterimage_ref_verify", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def logits(seed: int, dtype, scale: float = 3.0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(VOCAB, generator=g) * scale).to(dtype)


def one_hot(i: int, dtype) -> torch.Tensor:
    p = torch.zeros(VOCAB, dtype=dtype)
    p[i] = 1.0
    return p


def chain(ref, kind: str, k: int, seed: int, dtype, temp: float):
    """Draft/target distributions for a k-token chain, the draft tokens
    (sampled from the draft with its own generator) and the bonus
    distribution."""
    if kind == "equal":
        draft = [ref.temperature_probs(logits(seed + i, dtype), temp) for i in range(k)]
        target = [d.clone() for d in draft]
    elif kind == "disagree":
        draft = [ref.temperature_probs(logits(seed + i, dtype), temp) for i in range(k)]
        target = [ref.temperature_probs(logits(seed + 100 + i, dtype), temp) for i in range(k)]
    elif kind == "certain_reject":
        # the draft always proposes token 0, which the target never emits
        draft = [one_hot(0, dtype) for _ in range(k)]
        target = [one_hot(1 + i, dtype) for i in range(k)]
    elif kind == "draft_dominates":
        # target mass sits on the draft token only as a fraction: q >= p everywhere
        draft = [one_hot(3, dtype) for _ in range(k)]
        target = [torch.full((VOCAB,), 0.0, dtype=dtype) for _ in range(k)]
        for t in target:
            t[3] = 0.25
            t[5] = 0.75
    else:
        raise ValueError(kind)
    gd = torch.Generator().manual_seed(seed + 7)
    tokens = [ref.sample_categorical(d, gd) for d in draft]
    bonus = ref.temperature_probs(logits(seed + 200, dtype), temp)
    return draft, target, tokens, bonus


def main() -> None:
    root = pathlib.Path(sys.argv[1] if len(sys.argv) > 1 else os.environ["AFTERIMAGE_REF"])
    ref = load_reference(root)
    cases = {"temperature_probs": [], "sample_categorical": [], "speculative_sample_step": []}
    for dtype in DTYPES:
        for temp in TEMPS:
            for seed in (1, 2, 3):
                x = logits(seed, dtype)
                cases["temperature_probs"].append({"logits": x, "temperature": temp,
                                                   "probs": ref.temperature_probs(x, temp)})
    for dtype in DTYPES:
        for seed in range(6):
            p = ref.temperature_probs(logits(seed + 40, dtype), 1.0)
            g = torch.Generator().manual_seed(seed)
            cases["sample_categorical"].append({"probs": p, "seed": seed,
                                                "tokens": [ref.sample_categorical(p, g) for _ in range(4)]})
    for dtype in DTYPES:
        for temp in (0.0, 0.7, 1.0):
            for kind in ("equal", "disagree", "certain_reject", "draft_dominates"):
                for k in (1, 3, 5):
                    for seed in (11, 12):
                        draft, target, tokens, bonus = chain(ref, kind, k, seed, dtype, temp)
                        g = torch.Generator().manual_seed(seed + 1000)
                        out, n = ref.speculative_sample_step(draft, target, tokens, bonus, g)
                        cases["speculative_sample_step"].append({
                            "kind": kind, "temperature": temp, "seed": seed + 1000, "draft_probs": draft,
                            "target_probs": target, "draft_tokens": tokens, "bonus": bonus,
                            "tokens": out, "n_accepted": n})
    torch.save(cases, OUT)
    print("wrote %s: %s" % (OUT, {k: len(v) for k, v in cases.items()}))


if __name__ == "__main__":
    main()
