"""Benchmark: bit-exact BF16 weight decode throughput on B200.

Workload ("qwen3-14b-layer"): one decoder layer of the Qwen3-14B shape
(q/k/v/o/gate/up/down = 330.3 M BF16 weights, random N(0, 0.02), seeded),
compressed with this package's encoder (byte-identical to the reference's
compress_layer, chunk_size 1024). A step decodes every tensor of one layer
back to bit-exact BF16 with ONE kernel launch. `--layers` distinct layers
are resident and used round-robin; each step reads ~0.45 GB and writes
0.66 GB, far above the 126 MB L2, so no L2 flush is needed.

  value  GB/s of algorithmic bytes (sign/mantissa + packed stream + chunk
         offsets + first-level codebook + BF16 written) with the compressed
         layer resident in HBM, whole job (sum over ranks, max-over-ranks time)
  e2e    same metric through the public layer-decode API with the
         compressed layer in pinned HOST memory: every step uploads it
         (packed, offsets, byte counts, sign/mantissa, LUTs), rebuilds the
         decode tables, decodes, and reads back the 4-byte status word.

Multi-GPU: one process per GPU; every rank decodes its own layers (the
decode has no exchange step), so scaling is weak and the data path has no
collective. `--impl reference` times the reference's CPU decode path (the
oracle port of its numba decoder + recombine, all host threads) on the same
workload and metric.

The same line carries the tokens/s half of the metric: greedy decoding of a
random-init decoder of the `--model` shape (Qwen3-0.6B, Llama-3-8B,
Qwen3-14B by default, or Mistral-Small-24B) through the tensor-parallel
decoder at the run's N (streamed from host memory, streamed under the
configuration's per-rank VRAM budget, compressed-resident eager and
graphed), and with `--tokens` through the transformers-driven engine.
"""
from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

QWEN3_14B_LAYER = [("q_proj", 5120, 5120), ("k_proj", 1024, 5120), ("v_proj", 1024, 5120),
                   ("o_proj", 5120, 5120), ("gate_proj", 17408, 5120), ("up_proj", 17408, 5120),
                   ("down_proj", 5120, 17408)]
CONFIG1 = [("w", 4096, 4096)]
WORKLOADS = {"qwen3-14b-layer": QWEN3_14B_LAYER, "config1-4096x4096": CONFIG1,
             "qwen3-14b-layer-tp8": QWEN3_14B_LAYER}
# per-tensor chunk sizes where a workload differs from the reference default
# (a store written with write_store(tp_row_chunks=8): row-parallel tensors in
# whole chunks of every rank's columns)
WORKLOAD_CHUNKS = {"qwen3-14b-layer-tp8": {"o_proj": 640, "down_proj": 1088}}
FAST_TABLE_BYTES = 4096 * 8
# the benchmark's decoder shapes (random-init weights in every measurement)
QWEN3_06B = dict(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                 num_attention_heads=16, num_key_value_heads=8, head_dim=128, rope_theta=1e6,
                 tie_word_embeddings=True, max_position_embeddings=4096)
QWEN3_14B = dict(vocab_size=151936, hidden_size=5120, intermediate_size=17408, num_hidden_layers=40,
                 num_attention_heads=40, num_key_value_heads=8, head_dim=128, rope_theta=1e6,
                 tie_word_embeddings=False, max_position_embeddings=4096)
LLAMA3_8B = dict(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32,
                 num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=500000.0,
                 tie_word_embeddings=False, max_position_embeddings=8192)
MISTRAL_24B = dict(vocab_size=131072, hidden_size=5120, intermediate_size=32768, num_hidden_layers=40,
                   num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=1e8,
                   tie_word_embeddings=False, max_position_embeddings=8192)
# the benchmark's decoder configurations: config class, shape, prompt length, forced greedy
# tokens and the VRAM budget of its streamed run
MODELS = {
    "qwen3-0.6b": ("Qwen3Config", QWEN3_06B, 64, 4, 1.0, "Qwen3-0.6B shape"),
    "llama3-8b": ("LlamaConfig", LLAMA3_8B, 128, 8, 4.0, "Llama-3-8B shape"),
    "qwen3-14b": ("Qwen3Config", QWEN3_14B, 64, 4, 4.0, "Qwen3-14B shape"),
    "mistral-24b": ("MistralConfig", MISTRAL_24B, 256, 4, 8.0, "Mistral-Small-24B shape"),
}
METRIC = "bit-exact BF16 weight decode GB/s"
# host -> device copy rate assumed only when link_rates() cannot measure it (no CUDA)
PCIE_GBS_FALLBACK = 55.0


def env_int(name, default):
    v = os.environ.get(name)
    return int(v) if v not in (None, "") else default


def algorithmic_bytes(layers) -> int:
    """sign_mantissa (n) + packed (its bytes) + chunk offsets (4/chunk)
    + codebook bytes read (the 32 KiB first-level table per tensor)
    + BF16 written (2n)."""
    total = 0
    for layer in layers:
        enc = layer.encoded
        n = int(enc.n_symbols)
        total += n + int(np.asarray(enc.packed).nbytes) + 4 * int(enc.n_chunks) + FAST_TABLE_BYTES + 2 * n
    return total


def make_layers(spec, seed: int, device, chunks: dict | None = None, keep_source: bool = False):
    """The workload's tensors, random N(0, 0.02) BF16 (seeded), compressed.
    With keep_source, also returns each tensor's BF16 source on `device`
    (what the bit-exact gate compares the decoded layer with)."""
    from afterimage_b200.runtime.compressed_store import compress_layer
    g = torch.Generator(device=device).manual_seed(seed)
    out, src = [], []
    for i, (name, rows, cols) in enumerate(spec):
        W = (torch.randn(rows, cols, generator=g, device=device) * 0.02).to(torch.bfloat16)
        out.append(compress_layer(W.cpu(), chunk_size=(chunks or {}).get(name, 1024)))
        if keep_source:
            src.append(W)
        del W
    return (out, src) if keep_source else out


def bit_exact_gate(decoder, descs, outs, sources, layers: list[int]) -> None:
    """Decodes each listed resident layer with one launch and compares every
    tensor with its BF16 source bit for bit (raises on a mismatch or a
    device status error)."""
    from afterimage_b200.runtime import _device
    for i in layers:
        for o in outs:
            o.fill_(float("nan"))
        decoder.launch(descs[i], len(outs))
        torch.cuda.synchronize(decoder.device)
        _device.check_status(decoder.device)
        check_outputs(outs, sources[i], "layer %d" % i)


def check_outputs(outs, source, what: str) -> None:
    for o, w in zip(outs, source):
        if not torch.equal(o.view(torch.int16), w.view(torch.int16)):
            bad = int((o.view(torch.int16) != w.view(torch.int16)).sum())
            raise AssertionError("decoded %s differs from its source in %d of %d weights" % (what, bad, w.numel()))


class Clocks:
    """nvidia-smi sampler for the timed region (the recipe's clocks line)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = pathlib.Path(tempfile.gettempdir()) / f"aib_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "200"], stdout=self.fh,
                                         stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        try:
            self.path.unlink()
        except OSError:
            pass
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, STREAM-style copy)"
    return 6650.0, "fallback (6.65 TB/s, earlier measurement on this pool)"


def profile_traffic(workload: str):
    """DRAM bytes per decode launch from the committed ncu summary, if any."""
    p = ROOT / "profiles" / f"decode_bf16_{workload}.json"
    if p.exists():
        try:
            return json.loads(p.read_text()).get("dram_bytes_per_launch")
        except (ValueError, OSError):
            return None
    return None


def cpu_baseline(layers, max_seconds: float = 12.0) -> dict:
    """The reference's CPU decode (oracle port of decode_chunks_numba +
    _recombine), all host threads, over a bounded sample: whole tensors of
    the workload, repeated until ~max_seconds."""
    from oracle import oracle as O
    threads = O.max_threads()
    sample = layers[:]
    # warm-up on the smallest tensor (thread pool spin-up)
    small = min(sample, key=lambda layer: int(layer.encoded.n_symbols))
    O.decompress(small.encoded, small.sign_mantissa.numpy(), threads)
    done_bytes = 0
    t0 = time.perf_counter()
    reps = 0
    names = []
    while True:
        for layer in sample:
            O.decompress(layer.encoded, layer.sign_mantissa.numpy(), threads)
            done_bytes += algorithmic_bytes([layer])
            if reps == 0:
                names.append(tuple(layer.shape))
        reps += 1
        if time.perf_counter() - t0 > max_seconds:
            break
    dt = time.perf_counter() - t0
    # one thread: best of 3 passes over the first tensor
    one = sample[0]
    best = min(_timed(lambda: O.decompress(one.encoded, one.sign_mantissa.numpy(), 1)) for _ in range(3))
    return {"value": done_bytes / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{reps} pass(es) over the workload's {len(sample)} tensors "
                      f"({sum(int(l.encoded.n_symbols) for l in sample) / 1e6:.1f} M weights), "
                      f"{dt:.1f} s, OpenMP over chunks (restates cpu_decode.py:67-113 + compressed_store.py:94-114)",
            "single_thread": {"value": round(algorithmic_bytes([one]) / best / 1e9, 4), "unit": "GB/s", "cores": 1,
                              "sample": "best of 3 passes over the %s tensor" % "x".join(map(str, one.shape))}}


def _timed(fn) -> float:
    t0 = time.perf_counter()
    fn()
    return time.perf_counter() - t0


def synthetic_checkpoint(hf_cfg, seed: int, device):
    """(key, bf16 tensor) pairs of a random-init model in checkpoint order
    (embedding and head first): N(0, 0.02) matrices, unit norm weights,
    generated on the GPU and handed over one at a time."""
    from transformers import AutoModelForCausalLM
    with torch.device("meta"):
        meta = AutoModelForCausalLM.from_config(hf_cfg, dtype=torch.bfloat16)
    names = [(n, tuple(p.shape)) for n, p in meta.named_parameters()]
    if getattr(hf_cfg, "tie_word_embeddings", False):
        names = [(n, s) for n, s in names if n != "lm_head.weight"]
    big = ("embed_tokens.weight", "lm_head.weight")
    names = [x for x in names if x[0].endswith(big)] + [x for x in names if not x[0].endswith(big)]
    g = torch.Generator(device=device).manual_seed(seed)
    for name, shape in names:
        if len(shape) == 2:
            t = (torch.randn(shape, generator=g, device=device) * 0.02).to(torch.bfloat16)
        else:
            t = torch.ones(shape, dtype=torch.bfloat16, device=device)
        yield name, t.cpu()


# seeds of the tokens/s runs: the random-init checkpoint and the prompt
# (tests/golden/engine_tokens_qwen3-0.6b.npz records the reference engine on these)
TOKENS_WEIGHT_SEED = 14
TOKENS_PROMPT_SEED = 64


def checkpoint_digest(items) -> str:
    """sha256 over (name, BF16 bits) of every tensor, in checkpoint order."""
    import hashlib
    h = hashlib.sha256()
    for name, t in items:
        h.update(name.encode())
        h.update(t.contiguous().view(torch.int16).numpy().tobytes())
    return h.hexdigest()


def model_config(name: str):
    import transformers
    cls, shape, prompt, new, budget, label = MODELS[name]
    return getattr(transformers, cls)(**shape), prompt, new, budget, label


def run_tokens(args, dev) -> dict:
    """tokens/s of greedy decoding on the --model shape (default the Qwen3-14B
    shape, the benchmark's streamed 14B configuration) through the
    transformers-driven engine: the compressed store streamed under the
    configuration's VRAM budget (4 GB for 14B), the whole model
    compressed-resident in HBM, and, for the 14B shape, draft speculation
    with a Qwen3-0.6B-shaped draft at temperature 0 (token-identical to
    greedy)."""
    import shutil
    from transformers import AutoModelForCausalLM, Qwen3Config
    from afterimage_b200.runtime.streaming_engine import EngineConfig, StreamingLosslessModel, write_store
    root = pathlib.Path(tempfile.mkdtemp(prefix="aib_tokens_", dir="/dev/shm" if os.path.isdir("/dev/shm") else None))
    try:
        cfg, P, new_default, budget, label = model_config(args.model)
        new_tokens = args.new_tokens or new_default
        args = argparse.Namespace(**{**vars(args), "new_tokens": new_tokens})
        tied = bool(getattr(cfg, "tie_word_embeddings", False))
        t0 = time.perf_counter()
        m = write_store(synthetic_checkpoint(cfg, 14, dev), root / args.model, EngineConfig(chunk_size=1024),
                        tied=tied, model_id="synthetic/%s-shape" % args.model, progress_every=0)
        build_s = time.perf_counter() - t0
        gen = torch.Generator().manual_seed(64)
        prompt = torch.randint(0, cfg.vocab_size, (1, P), generator=gen)
        out = {"model": label + ", random N(0,0.02)", "params_orig_gb": round(m["total_orig_bytes"] / 1e9, 2),
               "store_gb": round(m["total_comp_bytes"] / 1e9, 2), "ratio": round(m["ratio"], 4),
               "store_build_s": round(build_s, 1), "prompt_tokens": P, "new_tokens": args.new_tokens}
        ref_tokens = None
        for name, ecfg in (("streamed_%gGB" % budget, EngineConfig(vram_budget_gb=budget, io_prefetch_depth=4,
                                                                   lm_head_slice_rows=0 if tied else 16384)),
                           ("resident_compressed", EngineConfig(vram_budget_gb=100.0, vram_tier_format="compressed"))):
            torch.cuda.empty_cache()
            torch.cuda.reset_peak_memory_stats(dev)
            harness = torch.cuda.memory_allocated(dev)  # the harness's own buffers, not the engine's
            with StreamingLosslessModel("synthetic/%s-shape" % args.model, root / args.model, device=str(dev),
                                        config=ecfg, hf_config=cfg) as eng:
                eng.generate_greedy(prompt, 2)  # warm: prompt pass and one single-token step
                eng.stats.reset()
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                seq = eng.generate_greedy(prompt, args.new_tokens)
                torch.cuda.synchronize()
                dt = time.perf_counter() - t0
                st = eng.stats
                out[name] = {"tokens_per_s": round(args.new_tokens / dt, 3), "s_per_token": round(dt / args.new_tokens, 4),
                             "bytes_read_gb": round(st.bytes_read / 1e9, 2), "h2d_gb": round(st.h2d_bytes / 1e9, 2),
                             "decode_launches": st.decode_launches, "prefetch_hits": st.prefetch_hits,
                             "prefetch_misses": st.prefetch_misses,
                             "io_s": round(st.io_seconds, 3), "h2d_enqueue_s": round(st.h2d_seconds, 3),
                             "decode_enqueue_s": round(st.decode_seconds, 3),
                             "vram_budget_gb": ecfg.vram_budget_gb,
                             "peak_vram_gb": round((torch.cuda.max_memory_allocated(dev) - harness) / 1e9, 2),
                             "harness_vram_gb": round(harness / 1e9, 2)}
                if ref_tokens is None:
                    ref_tokens = seq
                else:
                    out[name]["tokens_equal_streamed"] = bool(torch.equal(seq.cpu(), ref_tokens.cpu()))
                if name == "resident_compressed" and args.model == "qwen3-14b":
                    dcfg = Qwen3Config(**QWEN3_06B)
                    draft = AutoModelForCausalLM.from_config(dcfg, dtype=torch.bfloat16).to(dev).eval()
                    eng.generate_speculative(prompt, 1, draft, k=8, temperature=0.0)
                    eng.stats.reset()
                    torch.cuda.synchronize()
                    t0 = time.perf_counter()
                    spec = eng.generate_speculative(prompt, args.new_tokens, draft, k=8, temperature=0.0)
                    torch.cuda.synchronize()
                    dt = time.perf_counter() - t0
                    same = bool(torch.equal(spec.cpu(), ref_tokens.cpu()))
                    info = {"tokens_per_s": round(args.new_tokens / dt, 3), "k": 8, "sweeps": eng.stats.spec_sweeps,
                            "accepted_from_draft": eng.stats.spec_accepted_tokens, "tokens_equal_greedy": same,
                            "note": "random-init draft and target rarely agree; speculation checks correctness here"}
                    if not same:
                        # greedy decoded with a KV cache (M=1 projections); the verification sweep recomputes
                        # the whole sequence (M=prompt+k), so BF16 rounding differs: report the first
                        # divergent position and the top-2 logit margin the greedy run had there
                        a, b = spec[0].cpu().tolist(), ref_tokens[0].cpu().tolist()
                        pos = next(i for i in range(len(a)) if a[i] != b[i])
                        lg = eng.forward_logits(ref_tokens[:, :pos], use_cache=False)[0, -1].float()
                        top = torch.topk(lg, 2).values
                        info.update(first_divergence=pos - prompt.shape[1],
                                    top2_margin_at_divergence=round(float(top[0] - top[1]), 5))
                    out["speculative_draft_0.6B"] = info
                    del draft
            torch.cuda.empty_cache()
            torch.cuda.reset_peak_memory_stats(dev)
        return out
    finally:
        shutil.rmtree(root, ignore_errors=True)


def _shared_tmpdir(world: int, rank: int, prefix: str) -> pathlib.Path:
    root = None
    if rank == 0:
        root = tempfile.mkdtemp(prefix=prefix, dir="/dev/shm" if os.path.isdir("/dev/shm") else None)
    if world > 1:
        box = [root]
        torch.distributed.broadcast_object_list(box, src=0)
        root = box[0]
    return pathlib.Path(root)


def _max_over_ranks(v: float, world: int, dev) -> float:
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int) -> None:
    if world > 1:
        torch.distributed.barrier()


def link_rates(world: int, rank: int, dev, nbytes: int = 1 << 30) -> dict:
    """Measured link rates on this box, CUDA events, max time over ranks:
      pcie_h2d_gbps / pcie_d2h_gbps: one pinned 1 GiB copy per rank, every
        rank at once (as the streamed decoder's ranks copy), per-rank rate;
      nvlink_p2p_gbps (world >= 2): rank 0 sends 1 GiB to rank 1 over NCCL's
        peer-to-peer path (NVLink through NVSwitch), one direction."""
    host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = {}
    for name, dst, src in (("pcie_h2d_gbps", buf, host), ("pcie_d2h_gbps", host, buf)):
        dst.copy_(src, non_blocking=True)  # warm
        torch.cuda.synchronize()
        _barrier(world)
        a.record()
        dst.copy_(src, non_blocking=True)
        b.record()
        torch.cuda.synchronize()
        ms = _max_over_ranks(a.elapsed_time(b), world, dev)
        out[name] = round(nbytes / (ms / 1e3) / 1e9, 2)
    del host
    if world >= 2:
        ms = 0.0
        for it in range(2):  # the first transfer sets up the peer connection
            _barrier(world)
            if rank in (0, 1):
                a.record()
                if rank == 0:
                    torch.distributed.send(buf, 1)
                else:
                    torch.distributed.recv(buf, 0)
                b.record()
                torch.cuda.synchronize()
                ms = a.elapsed_time(b)
            ms = _max_over_ranks(ms if rank in (0, 1) else 0.0, world, dev)
        out["nvlink_p2p_gbps"] = round(nbytes / (ms / 1e3) / 1e9, 2)
    del buf
    torch.cuda.empty_cache()
    out["bytes"] = nbytes
    return out


def allreduce_probe(world: int, dev, hidden: int, count: int, links: dict | None = None) -> dict | None:
    """The per-block exchange of tensor-parallel decoding: `count`
    back-to-back all-reduces of one token's fp32 row-parallel partial sums
    (hidden floats), through NCCL and through the one-shot NVLink kernel the
    decoder uses (runtime/allreduce.py). Each is timed eagerly and as one
    captured CUDA graph of the `count` calls (as the graphed decode step runs
    them: no host launch cost), CUDA events, max over ranks. Latency-bound at
    this size: the bus rate is far below the link rate."""
    if world < 2:
        return None
    from afterimage_b200.runtime.allreduce import OneShotAllReduce
    x = torch.randn(hidden, device=dev)
    ar = OneShotAllReduce(None, dev, hidden)
    nbytes = hidden * 4
    out = {"all_reduces_per_token": count, "bytes_each": nbytes}
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    side = torch.cuda.Stream(dev)
    for name, fn in (("nccl", lambda: torch.distributed.all_reduce(x)), ("oneshot", lambda: ar(x))):
        for _ in range(20):
            fn()
        torch.cuda.synchronize()
        _barrier(world)
        a.record()
        for _ in range(count):
            fn()
        b.record()
        torch.cuda.synchronize()
        eager_ms = _max_over_ranks(a.elapsed_time(b), world, dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            fn()  # warm on the capture stream
        torch.cuda.synchronize()
        _barrier(world)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            for _ in range(count):
                fn()
        torch.cuda.synchronize()
        _barrier(world)
        graph.replay()  # warm
        torch.cuda.synchronize()
        _barrier(world)
        a.record()
        graph.replay()
        b.record()
        torch.cuda.synchronize()
        graph_ms = _max_over_ranks(a.elapsed_time(b), world, dev)
        del graph  # graphs holding NCCL calls go before the process group
        torch.cuda.synchronize()
        per_us = graph_ms * 1e3 / count
        out[name] = {"us_each_graphed": round(per_us, 2), "ms_per_token_graphed": round(graph_ms, 3),
                     "us_each_eager": round(eager_ms * 1e3 / count, 2),
                     "bus_gbps_graphed": round(2 * (world - 1) / world * nbytes / (per_us * 1e-6) / 1e9, 3)}
    _barrier(world)
    ar.close()
    if links and links.get("nvlink_p2p_gbps"):
        out["nvlink_p2p_gbps_measured"] = links["nvlink_p2p_gbps"]
    out["note"] = "one token's fp32 partial sums per all-reduce: latency-bound, far below the link rate"
    return out


def tp_store_chunk_size(world: int) -> int:
    """Chunk size of the store written for a TP degree. A chunk is decoded
    serially by one lane, so a rank's small layer shard is latency-bound on
    its chunk length. Measured on B200 for one TP-8 rank's 14B layer: 85 us
    at 1024 symbols, 75 at 512, 52 at 256. A whole layer is fastest at the
    reference's 1024 (270 us; 350 at 256)."""
    return 256 if world >= 8 else 1024


def run_tp_tokens(args, world: int, rank: int, dev) -> dict:
    """Greedy tokens/s of the --model shape (default Qwen3-14B, the benchmark's 14B configuration) through
    the tensor-parallel decoder on `world` GPUs (one rank per GPU; world=1
    is a single GPU): every rank decodes only its own column/row shards of
    every layer, one all-reduce after o_proj and after down_proj (the
    one-shot NVLink kernel; NCCL for sums above its buffer).
      streamed:            compressed shards in page-locked host memory,
                           copied to the GPU one layer at a time (the layer
                           streamer over PCIe; device memory stays a few GB);
      streamed_<B>GB_per_rank: the same under the configuration's per-rank
                           VRAM budget (the planner keeps what fits resident);
      compressed_resident: compressed shards resident in HBM, decoded per
                           layer per forward, the next layer's decode
                           overlapping this layer's projections.
    Timed: prompt (P uniform ids, 64 for 14B) + new_tokens greedy tokens, CUDA events,
    max over ranks. The store is written once (rank 0, TP-ready chunking)."""
    from afterimage_b200.runtime.streaming_engine import EngineConfig, write_store
    from afterimage_b200.runtime.tp_decoder import KVCache, load_tp_decoder, timeline_summary, _mark
    import shutil
    cfg, P, new_default, budget, label = model_config(args.model)
    args = argparse.Namespace(**{**vars(args), "new_tokens": args.new_tokens or new_default})
    tied = bool(getattr(cfg, "tie_word_embeddings", False))
    root = _shared_tmpdir(world, rank, "aib_tp_")
    store = root / (args.model + "-tp8")
    out = {"model": label + ", random N(0,0.02)", "tp": world, "prompt_tokens": P,
           "new_tokens": args.new_tokens}
    try:
        if rank == 0:
            from afterimage_b200.runtime.streaming_engine import tp_chunk_size
            cs = tp_store_chunk_size(world)
            t0 = time.perf_counter()
            m = write_store(synthetic_checkpoint(cfg, 14, dev), store, EngineConfig(chunk_size=cs), tied=tied,
                            model_id="synthetic/%s-shape" % args.model, progress_every=0, tp_row_chunks=8)
            out.update(store_gb=round(m["total_comp_bytes"] / 1e9, 2), ratio=round(m["ratio"], 4),
                       store_build_s=round(time.perf_counter() - t0, 1),
                       store_chunking="chunk_size %d; o_proj %d, down_proj %d (whole chunks per rank up to TP 8)"
                       % (cs, tp_chunk_size(cfg.hidden_size, 8, cs), tp_chunk_size(cfg.intermediate_size, 8, cs)))
        draft = None
        if args.model == "qwen3-14b":
            # the configuration's draft: a Qwen3-0.6B-shaped decoder (same vocabulary), decoded
            # and resident on every rank, sharded like the target
            dstore = root / "qwen3-0.6b-draft"
            if rank == 0:
                dcfg = model_config("qwen3-0.6b")[0]
                write_store(synthetic_checkpoint(dcfg, 15, torch.device("cpu")), dstore,
                            EngineConfig(chunk_size=1024), tied=True, model_id="synthetic/qwen3-0.6b-draft",
                            progress_every=0)
            _barrier(world)
            draft = load_tp_decoder(dstore, model_config("qwen3-0.6b")[0], world, rank, None, dev,
                                    resident="decoded")
        _barrier(world)
        prompt = torch.randint(0, cfg.vocab_size, (1, P), generator=torch.Generator().manual_seed(64))
        links = link_rates(world, rank, dev)
        seqs = {}
        modes = (("streamed", "streamed", {}),
                 ("streamed_%gGB_per_rank" % budget, "streamed",
                  {"vram_budget_gb": budget, "max_context": P + args.new_tokens + 8}),
                 ("compressed_resident", "compressed", {"overlap": True}))
        wanted = set((getattr(args, "tp_modes", None) or "streamed,streamed_budget,compressed_resident").split(","))
        modes = [m for m in modes if (m[0] if not m[0].startswith("streamed_") else "streamed_budget") in wanted]
        for name, resident, kw in modes:
            harness = torch.cuda.memory_allocated(dev)  # the harness's own buffers, not the decoder's
            t0 = time.perf_counter()
            dec = load_tp_decoder(store, cfg, world, rank, None, dev, resident=resident, **kw)
            torch.cuda.synchronize()
            load_s = _max_over_ranks(time.perf_counter() - t0, world, dev)
            # warm: the prompt pass and one single-token step (kernels load lazily on first
            # launch; tables, allocator, NCCL)
            dec.generate_greedy(prompt, 2)
            torch.cuda.synchronize()
            torch.cuda.reset_peak_memory_stats(dev)
            _barrier(world)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            seq = dec.generate_greedy(prompt, args.new_tokens)
            b.record()
            torch.cuda.synchronize()
            ms = _max_over_ranks(a.elapsed_time(b), world, dev)
            peak = _max_over_ranks((torch.cuda.max_memory_allocated(dev) - harness) / 1e9, world, dev)
            seqs[name] = seq.cpu()
            # one single-token forward with the event timeline (after the timed region)
            cache = KVCache(dec.n_layers, dec.nkv, dec.hd, P + 16, dec.device)
            dec.forward(prompt, cache)
            torch.cuda.synchronize()
            dec.timeline = []
            base = _mark(torch.cuda.current_stream(dev))
            dec.forward(seq[:, P:P + 1], cache)
            torch.cuda.synchronize()
            tl = timeline_summary(dec.timeline, base)
            dec.timeline = None
            events = tl.pop("events")
            step_ms = _max_over_ranks(tl["span_ms"], world, dev)
            dbytes = dec.decode_bytes_per_forward()
            dec_ms = tl.get("decode_busy_ms", 0.0)
            peak_hbm, _ = measured_peak()
            info = {"tokens_per_s": round(args.new_tokens / (ms / 1e3), 3),
                    "s_per_token": round(ms / 1e3 / args.new_tokens, 4), "load_s": round(load_s, 1),
                    "peak_vram_gb_per_rank": round(peak, 2),
                    "harness_vram_gb_rank0": round(harness / 1e9, 2),
                    "decode_step_ms": round(step_ms, 3), "timeline_rank0": tl,
                    "decode_bytes_per_forward_per_rank": dbytes,
                    "decode_gbps_in_step": round(dbytes / (dec_ms / 1e3) / 1e9, 1) if dec_ms else None,
                    "decode_hbm_frac": round(dbytes / (dec_ms / 1e3) / 1e9 / peak_hbm, 4) if dec_ms else None}
            # the terms that bound one single-token forward on this rank: PCIe for the
            # streamed bytes, HBM for the decode, HBM for the projections reading the
            # decoded BF16 weights; the largest is the tokens/s roofline
            pcie_gbs = links.get("pcie_h2d_gbps") or PCIE_GBS_FALLBACK
            terms = {"pcie_ms": round(dec.h2d_bytes_per_forward() / pcie_gbs / 1e6, 3),
                     "decode_hbm_ms": round(dbytes / peak_hbm / 1e6, 3),
                     "projection_hbm_ms": round(2 * dec.weights_per_forward() / peak_hbm / 1e6, 3)}
            # the decode and the projections share HBM, so their times add; PCIe is a
            # separate link that overlaps them
            terms["hbm_ms"] = round(terms["decode_hbm_ms"] + terms["projection_hbm_ms"], 3)
            bound = "pcie_ms" if terms["pcie_ms"] >= terms["hbm_ms"] else "hbm_ms"
            info["roofline_terms"] = dict(terms, bound=bound, pcie_gbs=pcie_gbs, hbm_gbs=peak_hbm,
                                          step_ms=round(step_ms, 3),
                                          frac_of_bound=round(terms[bound] / step_ms, 4) if step_ms else None)
            if resident != "streamed":
                # the single-token step captured once as a CUDA graph and replayed per token
                dec.generate_greedy_graphed(prompt, args.new_tokens)  # warm + capture
                torch.cuda.synchronize()
                _barrier(world)
                a.record()
                gseq = dec.generate_greedy_graphed(prompt, args.new_tokens)
                b.record()
                torch.cuda.synchronize()
                gms = _max_over_ranks(a.elapsed_time(b), world, dev)
                # the captured step alone (prefill excluded): 32 more replays
                _barrier(world)
                a.record()
                k = dec.replay_steps(32)
                b.record()
                torch.cuda.synchronize()
                sms = _max_over_ranks(a.elapsed_time(b) / max(k, 1), world, dev)
                info["graphed"] = {"tokens_per_s": round(args.new_tokens / (gms / 1e3), 3),
                                   "s_per_token": round(gms / 1e3 / args.new_tokens, 4),
                                   "tokens_equal_eager": bool(torch.equal(gseq.cpu(), seqs[name])),
                                   "step_ms": round(sms, 3), "step_tokens_per_s": round(1e3 / sms, 2),
                                   "frac_of_bound": round(terms[bound] / sms, 4) if sms else None,
                                   "note": "tokens_per_s includes the %d-token prompt pass (a captured graph " % P +
                                           "too); step_ms is one replay of the captured single-token step"}
                dec.release_graphs()
            if draft is not None and name in ("streamed", "compressed_resident"):
                info["speculative_draft_0.6B"] = _time_speculative(dec, draft, prompt, args.new_tokens,
                                                                  seqs[name], world, dev)
            if getattr(dec, "budget_plan", None):
                info["budget_plan"] = dec.budget_plan
            if resident == "streamed":
                hb = dec.h2d_bytes_per_forward()
                up = tl.get("upload_busy_ms", 0.0)
                info.update(h2d_bytes_per_forward_per_rank=hb,
                            h2d_gbps_in_step=round(hb / (up / 1e3) / 1e9, 1) if up else None)
            if tl.get("allreduce_busy_ms") is not None and tl.get("span_ms"):
                info["allreduce_share_of_step"] = round(tl["allreduce_busy_ms"] / tl["span_ms"], 4)
            info["collective"] = "oneshot NVLink all-reduce" if dec.allreducer is not None else \
                ("none" if world == 1 else "NCCL all-reduce")
            dec.close()  # collective when the one-shot all-reduce is in use
            if rank == 0 and name == "compressed_resident":
                (root / "timeline_events.json").write_text(json.dumps(events))
            out[name] = info
            del dec, cache
            torch.cuda.empty_cache()
        ref_seq = next(iter(seqs.values()))
        out["tokens_equal_across_modes"] = all(bool(torch.equal(v, ref_seq)) for v in seqs.values())
        try:
            out["all_reduce"] = allreduce_probe(world, dev, cfg.hidden_size, 2 * cfg.num_hidden_layers, links)
        except Exception as exc:  # reported; the tokens/s figures above stand
            out["all_reduce"] = {"error": "%s: %s" % (type(exc).__name__, exc)}
        out["links"] = links
        if draft is not None:
            draft.close()
        return out
    finally:
        _barrier(world)
        if rank == 0:
            shutil.rmtree(root, ignore_errors=True)


def _time_speculative(dec, draft, prompt, new_tokens: int, greedy, world: int, dev, k: int = 4) -> dict:
    """Draft/target speculation at temperature 0 (TPDecoder.generate_speculative:
    k proposals from the Qwen3-0.6B-shaped draft, one (k+1)-token target forward
    per sweep), timed like greedy decoding: prompt pass + new_tokens, CUDA
    events, max over ranks. Random-init draft and target rarely agree, so
    this measures the sweep cost and checks the tokens against greedy."""
    dec.generate_speculative(prompt, 1, draft, k=k)  # warm: draft prompt path, (k+1)-token forward
    torch.cuda.synchronize()
    _barrier(world)
    st = {}
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    seq = dec.generate_speculative(prompt, new_tokens, draft, k=k, stats=st)
    b.record()
    torch.cuda.synchronize()
    ms = _max_over_ranks(a.elapsed_time(b), world, dev)
    same = bool(torch.equal(seq.cpu(), greedy))
    out = {"tokens_per_s": round(new_tokens / (ms / 1e3), 3), "s_per_token": round(ms / 1e3 / new_tokens, 4),
           "k": k, "sweeps": st.get("sweeps"), "accepted_from_draft": st.get("accepted_from_draft"),
           "tokens_equal_greedy": same, "temperature": 0.0,
           "note": "random-init draft and target rarely agree: about one token per target sweep"}
    if not same:
        # greedy decoding ran the fused single-token step, verification the (k+1)-token
        # torch math: report where they part and the target's top-2 margin there
        P = prompt.shape[1]
        a_, b_ = seq[0].tolist(), greedy[0].tolist()
        pos = next(i for i in range(len(a_)) if a_[i] != b_[i])
        lg = dec.forward(greedy[:, :pos].to(dev))[-1].float()
        top = torch.topk(lg, 2).values
        out.update(first_divergence=pos - P, top2_margin_at_divergence=round(float(top[0] - top[1]), 5))
    return out


def _timed_ms(fn, dev, reps: int = 50) -> float:
    for _ in range(5):
        fn()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b) / reps


def projections_compare(spec, chunks: dict, dev) -> dict:
    """One layer's single-token projections (the seven tensors): one batched
    decode launch followed by F.linear per tensor (cuBLAS), against the fused
    decode -> GEMV kernel (per dependent launch group, and all tensors in one
    launch)."""
    import torch.nn.functional as F
    from afterimage_b200.runtime.compressed_store import compress_layer
    from afterimage_b200.runtime.decode_gemv import GemvBatch, gemv_desc
    from afterimage_b200.runtime.layer_decode import LayerDecoder, upload_layer
    from afterimage_b200.runtime import _device
    g = torch.Generator(device=dev).manual_seed(7)
    res = []
    for name, r, c in spec:
        W = (torch.randn(r, c, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        res.append(upload_layer(compress_layer(W.cpu(), chunk_size=chunks.get(name, 1024)), dev))
    outs = [torch.empty(r, c, dtype=torch.bfloat16, device=dev) for _, r, c in spec]
    dec = LayerDecoder(dev)
    descs = dec.descriptors(res, outs)
    xs = [torch.randn(c, device=dev, generator=g).to(torch.bfloat16) for _, _, c in spec]
    ys = [torch.empty(r, dtype=torch.bfloat16, device=dev) for _, r, _ in spec]
    parts = [torch.empty(r * c // int(rr.encoded.chunk_size), dtype=torch.float32, device=dev)
             for rr, (_, r, c) in zip(res, spec)]
    gd = [gemv_desc(rr.stream, rr.tables, rr.encoded, 0, r * c, rr.sign_mantissa, c, x, p, y)
          for rr, (_, r, c), x, p, y in zip(res, spec, xs, parts, ys)]
    names = [n for n, _, _ in spec]
    groups = [[names.index(n) for n in grp if n in names]
              for grp in (("q_proj", "k_proj", "v_proj"), ("o_proj",), ("gate_proj", "up_proj"), ("down_proj",))]
    batches = [GemvBatch([gd[i] for i in grp], dev) for grp in groups if grp]
    one = GemvBatch(gd, dev)
    t_dec = _timed_ms(lambda: dec.launch(descs, len(spec)), dev)
    t_lin = _timed_ms(lambda: [F.linear(x[None], o) for x, o in zip(xs, outs)], dev)
    t_groups = _timed_ms(lambda: [bt.launch() for bt in batches], dev)
    t_one = _timed_ms(one.launch, dev)
    _device.check_status(dev)
    return {"weights": sum(r * c for _, r, c in spec), "decode_ms": round(t_dec, 4), "linear_ms": round(t_lin, 4),
            "unfused_ms": round(t_dec + t_lin, 4), "fused_4_launches_ms": round(t_groups, 4),
            "fused_one_launch_ms": round(t_one, 4)}


def projections_kernels(dev) -> list:
    """The dense projections of a decoded Qwen3-14B layer (joined q/k/v, o,
    joined gate/up, down) and the vocabulary head, through cuBLAS (F.linear)
    and through this package's kernels: the BF16 GEMV (csrc/gemv.cu) for 1
    and 5 tokens, the tcgen05 tensor-core GEMM (csrc/gemm_tc.cu) for 16 and
    64 tokens. Several distinct weights per shape are used round-robin so the
    L2 does not hold them; GB/s counts weights + activations + outputs."""
    import torch.nn.functional as F
    from afterimage_b200.runtime import tp_ops
    peak, _ = measured_peak()
    shapes = {"qkv": (7168, 5120), "o": (5120, 5120), "gate_up": (34816, 5120), "down": (5120, 17408),
              "head": (151936, 5120)}
    out = []
    for m in (1, 5, 16, 64):
        own = tp_ops.gemv if m <= 8 else tp_ops.gemm_tc
        for name, (n, k) in shapes.items():
            ws = [(torch.randn(n, k, device=dev) * 0.02).to(torch.bfloat16)
                  for _ in range(max(2, int(4e8 // (n * k * 2)) + 1))]
            x = torch.randn(m, k, device=dev).to(torch.bfloat16)
            it = [0]

            def cub():
                it[0] += 1
                return F.linear(x, ws[it[0] % len(ws)])

            def mine():
                it[0] += 1
                return own(x, ws[it[0] % len(ws)])
            tc, to = _timed_ms(cub, dev), _timed_ms(mine, dev)
            nb = n * k * 2 + m * k * 2 + m * n * 2
            out.append({"tokens": m, "projection": name, "n": n, "k": k,
                        "kernel": "gemv" if m <= 8 else "tcgen05 gemm", "cublas_ms": round(tc, 4),
                        "own_ms": round(to, 4), "own_gbps": round(nb / to / 1e6, 1),
                        "own_frac_of_hbm": round(nb / to / 1e6 / peak, 3),
                        "cublas_frac_of_hbm": round(nb / tc / 1e6 / peak, 3)})
            del ws
    return out


def run_projections(dev) -> int:
    """`bench.py --projections`: one JSON line per case (not the benchmark line)."""
    layer = QWEN3_14B_LAYER
    rank8 = [("q_proj", 640, 5120), ("k_proj", 128, 5120), ("v_proj", 128, 5120), ("o_proj", 5120, 640),
             ("gate_proj", 2176, 5120), ("up_proj", 2176, 5120), ("down_proj", 5120, 1088)]
    tp = {"o_proj": 640, "down_proj": 1088}
    for name, spec, chunks in (("qwen3-14b-layer", layer, {}), ("qwen3-14b-layer-tp8-chunks", layer, tp),
                               ("qwen3-14b-rank-of-tp8", rank8, tp)):
        print(json.dumps({"case": "decode->gemv " + name, **projections_compare(spec, chunks, dev)}), flush=True)
    for row in projections_kernels(dev):
        print(json.dumps(row), flush=True)
    return 0


def bench_config(args, spec, step_bytes: int, world: int) -> dict:
    """The workload description both arms print (same keys and values)."""
    return {"workload": args.workload, "tensors": [n for n, _, _ in spec],
            "layer_weights": sum(r * c for _, r, c in spec),
            "chunk_size": {"default": 1024, **WORKLOAD_CHUNKS.get(args.workload, {})},
            "distinct_resident_layers": args.layers, "l2": "inputs > L2 (no flush needed)",
            "algorithmic_bytes_per_step": step_bytes, "parallelism": f"replica{world}"}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                             timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def run_reference(args, world, rank):
    """The reference arm: its CPU decode path (the oracle port of
    decode_chunks_numba + _recombine, all host threads) on the host cores,
    over the same workload as our arm: every step decodes the whole layer."""
    if rank != 0:
        return 0
    spec = WORKLOADS[args.workload]
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    layers = make_layers(spec, 1234, dev, WORKLOAD_CHUNKS.get(args.workload))
    nbytes = algorithmic_bytes(layers)
    from oracle import oracle as O
    threads = O.max_threads()
    for _ in range(args.warmup):
        for layer in layers:
            O.decompress(layer.encoded, layer.sign_mantissa.numpy(), threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for layer in layers:
            O.decompress(layer.encoded, layer.sign_mantissa.numpy(), threads)
    dt = time.perf_counter() - t0
    v = nbytes * args.steps / dt / 1e9
    sample = ("the whole %s workload (%d tensors, %.1f M weights) per step; oracle port of the reference "
              "CPU decoder" % (args.workload, len(spec), sum(r * c for _, r, c in spec) / 1e6))
    line = {"metric": METRIC, "value": round(v, 4), "unit": "GB/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic", "config": bench_config(args, spec, int(nbytes), world),
            "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="qwen3-14b-layer", choices=sorted(WORKLOADS))
    ap.add_argument("--layers", type=int, default=2, help="distinct resident layers used round-robin")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--layout", default="striped", choices=["striped", "reference"],
                    help="device layout of the resident streams: striped (aib_stripe_stream, coalesced "
                         "stream copies) or the reference's back-to-back chunks")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--tokens", action="store_true",
                    help="also measure greedy tokens/s through the engine on the --model shape "
                         "(the default Qwen3-14B shape builds a ~20 GB store)")
    ap.add_argument("--new-tokens", type=int, default=None,
                    help="greedy tokens per generation (default: the model configuration's)")
    ap.add_argument("--model", default="qwen3-14b", choices=sorted(MODELS),
                    help="decoder configuration of the tokens/s measurements")
    ap.add_argument("--projections", action="store_true",
                    help="instead of the benchmark: time one layer's projections (decode + cuBLAS, fused "
                         "decode->GEMV, this package's GEMV and tensor-core GEMM against cuBLAS)")
    ap.add_argument("--tp-modes", default=None,
                    help="comma list of tensor-parallel tokens/s modes to run (streamed, streamed_budget, "
                         "compressed_resident; default all)")
    ap.add_argument("--tp-tokens-only", action="store_true",
                    help="run only the tensor-parallel tokens/s measurement of --model and print its JSON line")
    ap.add_argument("--no-tp-tokens", action="store_true",
                    help="skip the tensor-parallel tokens/s measurement (its store of the --model shape "
                         "is written to /dev/shm)")
    args = ap.parse_args(argv)
    args.warmup = max(3, args.warmup)

    world, rank, local = dist_setup()
    if args.impl == "reference":
        rc = run_reference(args, world, rank)
        if world > 1:
            torch.distributed.destroy_process_group()
        return rc

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.projections:
        rc = run_projections(dev) if rank == 0 else 0
        if world > 1:
            torch.distributed.destroy_process_group()
        return rc
    if args.tp_tokens_only:
        t = run_tp_tokens(args, world, rank, dev)
        if rank == 0:
            print(json.dumps({"tokens_%s_tp" % args.model.replace("-", "_").replace(".", ""): t}), flush=True)
        if world > 1:
            torch.distributed.destroy_process_group()
        return 0
    from afterimage_b200.runtime import layer_decode as LD
    from afterimage_b200.runtime import _device

    spec = WORKLOADS[args.workload]
    made = [make_layers(spec, 1000 * rank + i + 1, dev, WORKLOAD_CHUNKS.get(args.workload), keep_source=True)
            for i in range(args.layers)]
    host_layers = [h for h, _ in made]
    sources = [s for _, s in made]  # BF16 source of every resident layer, on the device
    del made
    resident = [[LD.upload_layer(t, dev, striped=args.layout == "striped") for t in layer]
                for layer in host_layers]
    stream_bytes = sum(int(np.asarray(t.encoded.packed).nbytes) for t in host_layers[0])
    resident_stream_bytes = sum(r.stream.nbytes for r in resident[0])
    outs = [torch.empty(r, c, dtype=torch.bfloat16, device=dev) for _, r, c in spec]
    decoder = LD.LayerDecoder(dev)
    descs = [decoder.descriptors(res, outs) for res in resident]
    step_bytes = [algorithmic_bytes(layer) for layer in host_layers]
    torch.cuda.synchronize()

    # correctness gate before timing: every tensor of every resident layer bit-exact
    bit_exact_gate(decoder, descs, outs, sources, list(range(args.layers)))

    stream = torch.cuda.current_stream(dev)
    for i in range(args.warmup):
        decoder.launch(descs[i % args.layers], len(spec))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with Clocks(torch.cuda.current_device()) as clk:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        total_bytes = 0
        for i in range(args.steps):
            ev[i][0].record(stream)
            decoder.launch(descs[i % args.layers], len(spec))
            ev[i][1].record(stream)
            total_bytes += step_bytes[i % args.layers]
        t_end.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
    clocks = clk.summary()
    elapsed_ms = t_start.elapsed_time(t_end)
    launch_ms = [a.elapsed_time(b) for a, b in ev]
    _device.check_status(dev)
    # after the timed loop: the last timed launch's output, then every layer again
    check_outputs(outs, sources[(args.steps - 1) % args.layers], "layer of the last timed step")
    bit_exact_gate(decoder, descs, outs, sources, list(range(args.layers)))
    parity = "bit-exact: every tensor of the %d resident layers equals its BF16 source before and after " \
             "the timed loop, and the last timed launch's output was checked" % args.layers
    del sources
    t = torch.tensor([elapsed_ms], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    max_ms = float(t.item())
    value = total_bytes * world / (max_ms / 1e3) / 1e9
    avg_launch_ms = sum(launch_ms) / len(launch_ms)
    per_launch_bytes = total_bytes / args.steps
    achieved = per_launch_bytes / (avg_launch_ms / 1e3) / 1e9
    peak, peak_src = measured_peak()

    # ---- end to end through the public API with pinned host buffers --------
    e2e = None
    if not args.no_e2e:
        pinned = [LD.pin_layer(t) for t in host_layers[0]]
        h2d = sum(int(np.asarray(p.encoded.packed).nbytes) + int(np.asarray(p.encoded.chunk_offsets).nbytes)
                  + int(np.asarray(p.encoded.chunk_nbytes).nbytes) + int(p.sign_mantissa.numel())
                  + int(np.asarray(p.encoded.sym_lut).nbytes) + int(np.asarray(p.encoded.len_lut).nbytes)
                  for p in pinned)
        status_host = torch.empty(1, dtype=torch.int32, pin_memory=True)
        for _ in range(2):
            decoder.decode_host(pinned)
        torch.cuda.synchronize()
        if world > 1:
            torch.distributed.barrier()
        s0 = torch.cuda.Event(enable_timing=True)
        s1 = torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(args.e2e_steps):
            decoder.decode_host(pinned)
            status_host.copy_(_device.status_word(dev), non_blocking=True)
            stream.synchronize()
        s1.record(stream)
        torch.cuda.synchronize()
        te = torch.tensor([s0.elapsed_time(s1)], dtype=torch.float64, device=dev)
        if world > 1:
            torch.distributed.all_reduce(te, op=torch.distributed.ReduceOp.MAX)
        e2e_v = step_bytes[0] * args.e2e_steps * world / (float(te.item()) / 1e3) / 1e9
        e2e = {"value": round(e2e_v, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
               "ms_per_step": round(float(te.item()) / args.e2e_steps, 3),
               "path": "LayerDecoder.decode_host on pinned host layers (upload, tables, one batched decode, status D2H)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(host_layers[0])
    tokens = tp_tokens = None
    if not args.no_tp_tokens or args.tokens:
        del resident, descs, outs
        torch.cuda.empty_cache()
    if not args.no_tp_tokens:
        try:
            tp_tokens = run_tp_tokens(args, world, rank, dev)
        except Exception as exc:  # reported in the line; the decode measurement above stands
            tp_tokens = {"error": "%s: %s" % (type(exc).__name__, exc)}
    if args.tokens and rank == 0:
        tokens = run_tokens(args, dev)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(max_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic: random N(0,0.02) BF16 weights, seeded, encoded by afterimage_b200 (reference-identical)",
            "config": bench_config(args, spec, int(step_bytes[0]), world),
            "gpu_launches": args.steps * (-(-len(spec) // 16)),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src,
                         "traffic": profile_traffic(args.workload),
                         "kernel": "aib::decode_kernel<0> (fused decode + recombine)",
                         "stream_layout": args.layout,
                         "resident_stream_bytes_vs_reference": round(resident_stream_bytes / stream_bytes, 4),
                         "avg_launch_ms": round(avg_launch_ms, 5)},
            "parity": parity,
            "clocks": clocks,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        if tp_tokens is not None:
            line["tokens_%s_tp" % args.model.replace("-", "_").replace(".", "")] = tp_tokens
        if tokens is not None:
            line["tokens_per_s_%s" % args.model.replace("-", "_").replace(".", "")] = tokens
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
