"""The speculative-verification helpers against the reference's own outputs
(tests/golden/verify_cases.pt, written by make_verify_golden.py from the
reference's afterimage/runtime/verify.py): same probabilities bit for bit
and in the same dtype, and the same sampled tokens and accepted counts from
the same seeded CPU generator."""
import pathlib

import pytest
import torch

from afterimage_b200.runtime.verify import sample_categorical, speculative_sample_step, temperature_probs

CASES = torch.load(pathlib.Path(__file__).resolve().parent / "golden" / "verify_cases.pt", weights_only=False)


@pytest.mark.parametrize("i", range(len(CASES["temperature_probs"])))
def test_temperature_probs_matches_reference(i):
    c = CASES["temperature_probs"][i]
    got = temperature_probs(c["logits"], c["temperature"])
    assert got.dtype == c["probs"].dtype
    assert torch.equal(got, c["probs"])


@pytest.mark.parametrize("i", range(len(CASES["sample_categorical"])))
def test_sample_categorical_matches_reference(i):
    c = CASES["sample_categorical"][i]
    g = torch.Generator().manual_seed(c["seed"])
    assert [sample_categorical(c["probs"], g) for _ in range(len(c["tokens"]))] == c["tokens"]


@pytest.mark.parametrize("i", range(len(CASES["speculative_sample_step"])))
def test_speculative_sample_step_matches_reference(i):
    c = CASES["speculative_sample_step"][i]
    g = torch.Generator().manual_seed(c["seed"])
    tokens, n = speculative_sample_step(c["draft_probs"], c["target_probs"], c["draft_tokens"], c["bonus"], g)
    assert (tokens, n) == (c["tokens"], c["n_accepted"]), c["kind"]
    assert len(tokens) == n + 1


def test_fixture_covers_every_chain_kind_and_dtype():
    kinds = {c["kind"] for c in CASES["speculative_sample_step"]}
    assert kinds == {"equal", "disagree", "certain_reject", "draft_dominates"}
    dtypes = {c["logits"].dtype for c in CASES["temperature_probs"]}
    assert dtypes == {torch.float32, torch.bfloat16}
    # the chains reach both outcomes: a full accept (bonus) and an early rejection
    ns = {(c["n_accepted"] == len(c["draft_tokens"])) for c in CASES["speculative_sample_step"]}
    assert ns == {True, False}
