"""bench.py host logic on the CPU: the reference arm's JSON line (it times
the oracle port of the reference's CPU decoder, so it runs without a GPU)
and the decoder configurations the tokens/s measurements build."""
import io
import json
import contextlib

import pytest

import bench


def test_reference_arm_prints_the_contract_line():
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        rc = bench.main(["--impl", "reference", "--steps", "1", "--warmup", "3",
                         "--workload", "config1-4096x4096"])
    assert rc == 0
    line = json.loads(out.getvalue().strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == "GB/s"
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["config"]["workload"] == "config1-4096x4096"
    # same workload description as our arm: the whole workload is decoded every step
    assert line["config"] == bench.bench_config(bench.argparse.Namespace(workload="config1-4096x4096", layers=2),
                                                bench.WORKLOADS["config1-4096x4096"],
                                                line["config"]["algorithmic_bytes_per_step"], 1)
    assert "whole config1-4096x4096 workload" in line["cpu_baseline"]["sample"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


@pytest.mark.parametrize("name", sorted(bench.MODELS))
def test_model_configurations(name):
    cfg, prompt, new, budget, label = bench.model_config(name)
    assert prompt > 0 and new > 0 and budget > 0 and label
    assert cfg.num_attention_heads % cfg.num_key_value_heads == 0
    # every shape shards at TP 8: KV heads and the vocabulary split evenly
    assert cfg.num_key_value_heads % 8 == 0 and cfg.vocab_size % 8 == 0
    assert cfg.tie_word_embeddings == (name == "qwen3-0.6b")


def test_tp_store_chunk_size():
    assert bench.tp_store_chunk_size(8) == 256
    assert bench.tp_store_chunk_size(1) == bench.tp_store_chunk_size(2) == bench.tp_store_chunk_size(4) == 1024


def test_cpu_baseline_reports_all_threads_and_one_thread():
    spec = bench.WORKLOADS["config1-4096x4096"]
    layers = bench.make_layers(spec, 3, "cpu", bench.WORKLOAD_CHUNKS.get("config1-4096x4096"))
    cpu = bench.cpu_baseline(layers, max_seconds=0.5)
    assert cpu["kind"] == "port" and cpu["value"] > 0 and cpu["cores"] >= 1
    one = cpu["single_thread"]
    assert one["cores"] == 1 and one["value"] > 0 and one["sample"].endswith("4096x4096 tensor")


def test_reference_engine_token_fixture_is_consistent():
    """tests/golden/engine_tokens_qwen3-0.6b.npz (the reference engine's own
    greedy run): its tokens are the argmax of its recorded logits, its
    margins the top-2 gaps, and its prompt the benchmark's seeded prompt."""
    import numpy as np
    import pathlib
    import torch
    g = np.load(pathlib.Path(__file__).resolve().parent / "golden" / "engine_tokens_qwen3-0.6b.npz")
    cfg, P, N, _, _ = bench.model_config("qwen3-0.6b")
    logits = torch.from_numpy(g["logits_bits"]).view(torch.bfloat16).float()
    assert logits.shape == (N, cfg.vocab_size)
    assert g["tokens"].tolist() == logits.argmax(-1).tolist()
    top = torch.topk(logits, 2, dim=-1).values
    assert np.allclose(g["top2_margin"], (top[:, 0] - top[:, 1]).numpy())
    prompt = torch.randint(0, cfg.vocab_size, (1, P), generator=torch.Generator().manual_seed(bench.TOKENS_PROMPT_SEED))
    assert g["prompt"].tolist() == prompt[0].tolist()
