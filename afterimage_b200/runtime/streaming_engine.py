"""Layer-streaming execution of a compressed BF16 model -- the hot path of
the reference's afterimage/runtime/streaming_engine.py, rebuilt around the
batched sm_100a decoder.

Kept (reference file:line): the store format -- `weights.bin` plus a
schema-v2 `manifest.json` (compress_model_to_disk :256-428, per-tensor
compression rules :158-253); store integrity checks :843-871; residency
tiers from the planner :904-1043; row-gathered untied embeddings
:1232-1271; resident materialisation with weight re-tying :1273-1456;
transformers-driven forward with per-layer load/free hooks :1743-1915;
forward_logits :2154-2212; generate_greedy :2385-2429; draft-model
generate_speculative :2488-2575.

What the B200 build does differently on the per-layer path:
  * a prefetch thread reads a layer's compressed blobs straight into a
    page-locked slot (no pageable copy), `io_prefetch_depth` layers ahead;
  * the host->device copies run on a copy stream, ordered before the
    decode by a CUDA event, so they overlap the previous layer's compute;
  * every streamed tensor of the layer is decoded by ONE kernel launch
    (aib_decode_bf16_batch) into fresh BF16 parameters;
  * decode tables are built once per tensor and stay on the device;
  * nothing synchronises the device per layer: buffers are returned to the
    caching allocator in stream order.
Extra tier: `vram_tier_format="compressed"` keeps VRAM-tier decoder-layer
tensors in their compressed form in HBM and decodes them per layer -- ~1.5x
more model per GB of HBM at the cost of one decode per use.
"""
from __future__ import annotations

import concurrent.futures
import dataclasses
import json
import pathlib
import sys
import threading
import time

import numpy as np
import torch

from . import _device
from . import gpu_decode_v2 as _gd
from .binstore import BinaryWeightReader, BinaryWeightWriter, PinnedBuffer, blobref_to_dict
from .compressed_store import decompress_rows_gpu, CompressedLayer, compress_layer, decompress_layer_gpu
from .huffman_chunked import ChunkedEncoded
from .layer_decode import LayerDecoder, ResidentLayer, upload_layer
from .verify import sample_categorical, speculative_sample_step, temperature_probs

CURRENT_SCHEMA_VERSION = 2
_BIG_TENSOR_SUFFIXES = ("embed_tokens.weight", "lm_head.weight")
_COMPRESSED_BLOBS = ("sign_mantissa", "packed", "chunk_offsets", "chunk_nbytes", "sym_lut", "len_lut")


@dataclasses.dataclass
class EngineConfig:
    """The codec and streaming fields of the reference's EngineConfig
    (afterimage/runtime/config.py:360-410), plus B200 additions."""
    chunk_size: int = 1024
    max_bits: int = 16
    force_raw_storage: bool = False
    decode_slice_elems: int = 1 << 25
    reuse_decode_tables: bool = True
    vram_budget_gb: float | None = None
    ram_budget_gb: float | None = None
    ram_tier_format: str = "decoded"        # "decoded" | "compressed"
    vram_tier_format: str = "decoded"       # "decoded" | "compressed" (decoded per use from HBM)
    io_prefetch_depth: int = 1
    io_threads: int = 8                     # concurrent positional reads of the pinned prefetch slots
    storage_extent_max_gap_bytes: int = 0
    storage_extent_max_bytes: int = 1 << 28
    direct_io: bool = False
    max_context: int | None = None
    vram_cap_gb: float | None = None
    spec_k: int = 8
    lm_head_slice_rows: int = 0             # reference config: rows of lm_head per block, 0 = whole
    max_inflight_layers: int = 2            # streamed layers whose device buffers may be alive at once
    # further reference fields on this path (config.py:362-406)
    block_chunks: int = 32                  # validated like the reference; the CUDA grouping is fixed at 32
    vram_safety_margin_gb: float = 0.0      # extra non-residency reserve inside vram_budget_gb
    storage_read_policy: str = "coalesced_extents"  # "per_blob" | "coalesced_extents" | "tensor_extents"
    empty_cache_every: int = 0              # release cached device blocks every N layer frees; 0 never
    progress: bool = False                  # print generation progress to stderr
    require_pinned_ram: bool = False        # a failed pin of the decoded RAM tier always raises here
    placement_policy: str = "traffic_density"  # the planner's ranking; profiled ones are out of scope
    quantize: str | None = None             # lossless only: the reference's lossy "q8" is not built here

    def __post_init__(self):
        if self.chunk_size < 1:
            raise ValueError("chunk_size must be >= 1")
        if not 1 <= self.max_bits <= 16:
            raise ValueError("max_bits must be in [1, 16]")
        if self.decode_slice_elems < 1:
            raise ValueError("decode_slice_elems must be positive")
        if self.io_prefetch_depth < 0:
            raise ValueError("io_prefetch_depth must be >= 0")
        if self.io_threads < 1:
            raise ValueError("io_threads must be >= 1")
        if self.lm_head_slice_rows < 0:
            raise ValueError("lm_head_slice_rows must be >= 0")
        if self.max_inflight_layers < 1:
            raise ValueError("max_inflight_layers must be >= 1")
        if self.ram_tier_format not in ("decoded", "compressed"):
            raise ValueError("ram_tier_format must be 'decoded' or 'compressed'")
        if self.vram_tier_format not in ("decoded", "compressed"):
            raise ValueError("vram_tier_format must be 'decoded' or 'compressed'")
        if self.ram_budget_gb is not None and self.vram_budget_gb is None:
            raise ValueError("ram_budget_gb requires vram_budget_gb (the planner decides both tiers)")
        if self.block_chunks & (self.block_chunks - 1) != 0:
            raise ValueError("block_chunks must be a power of 2, got %d" % self.block_chunks)
        if self.storage_read_policy not in ("per_blob", "coalesced_extents", "tensor_extents"):
            raise ValueError("storage_read_policy must be 'per_blob', 'coalesced_extents' or 'tensor_extents', "
                             "got %r" % (self.storage_read_policy,))
        if self.storage_extent_max_bytes < 1:
            raise ValueError("storage_extent_max_bytes must be positive")
        if self.storage_extent_max_gap_bytes < 0:
            raise ValueError("storage_extent_max_gap_bytes must be non-negative")
        if self.max_context is not None and self.max_context < 1:
            raise ValueError("max_context must be >= 1, got %d" % self.max_context)
        if self.max_context is not None and self.vram_budget_gb is None:
            raise ValueError("max_context requires vram_budget_gb (the KV reserve is part of the plan)")
        if self.vram_safety_margin_gb < 0:
            raise ValueError("vram_safety_margin_gb must be non-negative")
        if self.vram_safety_margin_gb and self.vram_budget_gb is None:
            raise ValueError("vram_safety_margin_gb requires vram_budget_gb")
        if self.empty_cache_every < 0:
            raise ValueError("empty_cache_every must be >= 0")
        if self.require_pinned_ram and self.ram_budget_gb is None:
            raise ValueError("require_pinned_ram requires ram_budget_gb")
        if self.require_pinned_ram and self.ram_tier_format != "decoded":
            raise ValueError("require_pinned_ram requires ram_tier_format='decoded'")
        if self.placement_policy not in ("traffic_density", "profiled_knapsack", "critical_path",
                                         "replay_cem", "replay_qubo", "replay_extent_qubo"):
            raise ValueError("unknown placement_policy %r" % (self.placement_policy,))
        if self.placement_policy in ("profiled_knapsack", "critical_path"):
            raise ValueError("placement_policy=%r requires critical_path_profile with measured per-tensor "
                             "costs, which this package does not build" % self.placement_policy)
        if self.placement_policy != "traffic_density":
            raise ValueError("placement_policy=%r requires replay_plan_state from calibration traces, which "
                             "this package does not build" % self.placement_policy)
        if self.spec_k < 1:
            raise ValueError("spec_k must be >= 1, got %d" % self.spec_k)
        if self.quantize is not None:
            raise ValueError("quantize must be None (lossless); the reference's lossy %r mode is not built "
                             "in this package" % (self.quantize,))

    @property
    def uses_tiered_residency(self) -> bool:
        return self.vram_budget_gb is not None

    @property
    def is_lossless(self) -> bool:
        """Bit-identical output (reference config.py:575-580): false only
        with a chunked head, whose row blocks change the matmul's
        reduction order."""
        return self.quantize is None and self.lm_head_slice_rows == 0

    @property
    def exactness_contract(self) -> str:
        """The strongest claim this configuration supports (reference
        config.py:587-595, for the modes built here)."""
        return "approximate" if not self.is_lossless else "reference_execution_equivalent"

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)

    @classmethod
    def from_dict(cls, values: dict) -> "EngineConfig":
        """Rejects unknown fields, as the reference does (config.py:601-606)."""
        names = {f.name for f in dataclasses.fields(cls)}
        unknown = sorted(set(values) - names)
        if unknown:
            raise ValueError("unknown EngineConfig fields: %s" % ", ".join(unknown))
        return cls(**values)

    def fingerprint(self) -> str:
        """16 hex digits of the SHA-256 of the sorted-key JSON of every field."""
        import hashlib
        payload = json.dumps(self.to_dict(), sort_keys=True, separators=(",", ":"))
        return hashlib.sha256(payload.encode("utf-8")).hexdigest()[:16]

    def describe(self) -> str:
        """One line: exactness and residency (reference config.py:612-628)."""
        lossless = ("LOSSLESS (bit-exact output)" if self.is_lossless else
                    "LOSSY: lm_head_slice_rows=%d -- output is NOT bit-exact" % self.lm_head_slice_rows)
        if not self.uses_tiered_residency:
            return lossless + " | residency: legacy fixed policy"
        return "%s | residency: VRAM %.2f GB%s | io_prefetch_depth=%d" % (
            lossless, self.vram_budget_gb, (" + RAM %.2f GB" % self.ram_budget_gb) if self.ram_budget_gb else "",
            self.io_prefetch_depth)


@dataclasses.dataclass
class StreamStats:
    io_seconds: float = 0.0
    decode_seconds: float = 0.0
    h2d_seconds: float = 0.0
    compute_seconds: float = 0.0
    target_seconds: float = 0.0
    draft_seconds: float = 0.0
    bytes_read: int = 0
    h2d_bytes: int = 0
    storage_read_calls: int = 0
    layer_loads: int = 0
    decode_launches: int = 0
    prefetch_hits: int = 0
    prefetch_misses: int = 0
    spec_sweeps: int = 0
    spec_accepted_tokens: int = 0

    def reset(self) -> None:
        for f in dataclasses.fields(self):
            setattr(self, f.name, f.default)


# ---------------------------------------------------------------------------
# offline compression
# ---------------------------------------------------------------------------

def _weight_shards(snapshot: pathlib.Path) -> list[pathlib.Path]:
    index = snapshot / "model.safetensors.index.json"
    if index.exists():
        files = sorted(set(json.loads(index.read_text())["weight_map"].values()))
        return [snapshot / f for f in files]
    single = snapshot / "model.safetensors"
    if single.exists():
        return [single]
    return sorted(p for p in snapshot.glob("*.safetensors") if not p.name.startswith("consolidated"))


def _resolve_snapshot(model_id: str, source_dir, revision=None) -> pathlib.Path:
    if source_dir is not None:
        return pathlib.Path(source_dir)
    if pathlib.Path(model_id).is_dir():
        return pathlib.Path(model_id)
    from huggingface_hub import snapshot_download
    return pathlib.Path(snapshot_download(model_id, revision=revision,
                                          ignore_patterns=["consolidated*.safetensors"]))


def compress_one_tensor(key: str, W: torch.Tensor, cfg: EngineConfig, row_gather: bool = False) -> dict:
    """Storage decision and arrays for one tensor (reference
    streaming_engine.py:158-253): row-gathered embeddings raw int16,
    2-D BF16 tensors above 65536 elements compressed, everything else raw
    (float32 for non-BF16 / small tensors, int16 bit patterns when raw
    storage is forced on a BF16 matrix)."""
    orig = W.numel() * W.element_size()
    if row_gather:
        if W.dtype != torch.bfloat16 or W.dim() != 2:
            raise ValueError("row-gather storage needs a 2-D bf16 table, got %s %s for %s"
                             % (W.dtype, tuple(W.shape), key))
        return {"key": key, "kind": "row_gather", "shape": list(W.shape), "hidden_size": int(W.shape[1]),
                "orig_bytes": orig, "comp_bytes": orig,
                "arrays": {"raw": W.contiguous().view(torch.int16).numpy()}}
    if W.dtype == torch.bfloat16 and W.dim() == 2 and W.numel() > 65536 and not cfg.force_raw_storage:
        layer = compress_layer(W, chunk_size=cfg.chunk_size, max_bits=cfg.max_bits)
        e = layer.encoded
        return {"key": key, "kind": "compressed", "shape": list(W.shape), "max_bits": int(e.max_bits),
                "n_symbols": int(e.n_symbols), "chunk_size": int(e.chunk_size), "orig_bytes": orig,
                "comp_bytes": layer.compressed_bytes,
                "arrays": {"sign_mantissa": layer.sign_mantissa.numpy(), "packed": e.packed,
                           "chunk_offsets": e.chunk_offsets, "chunk_nbytes": e.chunk_nbytes,
                           "sym_lut": e.sym_lut, "len_lut": e.len_lut}}
    if cfg.force_raw_storage and W.dtype == torch.bfloat16:
        return {"key": key, "kind": "raw", "shape": list(W.shape), "dtype": "bfloat16", "orig_bytes": orig,
                "comp_bytes": orig, "arrays": {"raw": W.contiguous().view(torch.int16).numpy()}}
    return {"key": key, "kind": "raw", "shape": list(W.shape), "dtype": str(W.dtype), "orig_bytes": orig,
            "comp_bytes": orig, "arrays": {"raw": W.to(torch.float32).numpy()}}


def tp_chunk_size(in_features: int, parts: int, chunk_size: int) -> int:
    """Chunk size for a row-parallel tensor split `parts` ways by columns:
    a divisor of in_features/parts, so that every rank's column range is
    whole chunks, chosen to keep chunks about as long as the default (a
    kernel lane decodes one chunk: far fewer, longer chunks would leave the
    GPU idle). Preferred: the multiple of 64 nearest to chunk_size within
    [chunk_size/2, 2*chunk_size] (64-symbol multiples take the decoder's
    vectorised merge); else the largest divisor <= chunk_size, if at least
    a quarter of it. A segment no longer than chunk_size is one chunk.
    Keeps `chunk_size` when the columns do not divide or nothing fits."""
    if parts < 1 or in_features % parts:
        return chunk_size
    seg = in_features // parts
    if seg % chunk_size == 0:
        return chunk_size
    if seg <= chunk_size:
        return seg
    divs = [d for d in range(1, min(seg, 2 * chunk_size) + 1) if seg % d == 0]
    v64 = [d for d in divs if d % 64 == 0 and chunk_size // 2 <= d <= 2 * chunk_size]
    if v64:
        return min(v64, key=lambda d: (abs(d - chunk_size), -d))
    best = max((d for d in divs if d <= chunk_size), default=1)
    return best if 4 * best >= chunk_size else chunk_size


def write_store(items, out_dir, config: EngineConfig | None = None, *, tied: bool, model_id: str = "",
                revision: str | None = None, progress_every: int = 50, total: int | None = None,
                tp_row_chunks: int | None = None, control=None) -> dict:
    """Writes a compressed store from an iterable of (key, tensor) pairs:
    `weights.bin` + schema-v2 `manifest.json` (reference
    streaming_engine.py:345-427). The untied embedding is stored raw and
    row-addressable; each tensor is released after it is written.

    tp_row_chunks=P makes the store tensor-parallel ready: the row-parallel
    projections (o_proj, down_proj) use a chunk_size that divides
    in_features / P (`tp_chunk_size`), so each of P (or any divisor of P)
    ranks owns whole chunks of every row. The format is unchanged
    (chunk_size is per tensor).

    `control` (anything with a checkpoint() method, like the reference's
    JobControl) is called before each tensor is written: a pause/cancel
    boundary, as in the reference."""
    cfg = config or EngineConfig()
    out_dir = pathlib.Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    row_gather_key = None if tied else "model.embed_tokens.weight"
    manifest = {"schema_version": CURRENT_SCHEMA_VERSION, "model_id": model_id, "revision": revision,
                "quantize": None, "chunk_size": cfg.chunk_size, "force_raw_storage": cfg.force_raw_storage,
                "tied": tied, "tensors": {}, "expert_slices": {}}
    total_orig = total_comp = 0
    with BinaryWeightWriter(out_dir / "weights.bin") as writer:
        for n, (key, W) in enumerate(items, 1):
            if control is not None:
                control.checkpoint()
            tcfg = cfg
            if tp_row_chunks and W.dim() == 2 and key.endswith(("o_proj.weight", "down_proj.weight")):
                cs = tp_chunk_size(int(W.shape[1]), int(tp_row_chunks), cfg.chunk_size)
                if cs != cfg.chunk_size:
                    tcfg = dataclasses.replace(cfg, chunk_size=cs)
            res = compress_one_tensor(key, W, tcfg, row_gather=(key == row_gather_key))
            del W
            entry = {"orig_bytes": res["orig_bytes"], "comp_bytes": res["comp_bytes"], "shape": res["shape"],
                     "blobs": {name: blobref_to_dict(writer.write(arr)) for name, arr in res["arrays"].items()}}
            if res["kind"] == "compressed":
                entry.update(compressed=True, max_bits=res["max_bits"], n_symbols=res["n_symbols"],
                             chunk_size=res["chunk_size"])
            elif res["kind"] == "row_gather":
                entry.update(compressed=False, row_gather=True, hidden_size=res["hidden_size"], dtype="bfloat16")
            else:
                entry.update(compressed=False, dtype=res["dtype"])
            manifest["tensors"][key] = entry
            total_orig += res["orig_bytes"]
            total_comp += res["comp_bytes"]
            del res
            if progress_every and n % progress_every == 0:
                print("  [%d/%s] %.2f GB -> %.2f GB" % (n, total or "?", total_orig / 1e9, total_comp / 1e9),
                      flush=True)
    manifest["total_orig_bytes"] = total_orig
    manifest["total_comp_bytes"] = total_comp
    manifest["ratio"] = total_orig / max(total_comp, 1)
    (out_dir / "manifest.json").write_text(json.dumps(manifest, indent=2), encoding="utf-8", newline="\n")
    return manifest


def compress_model_to_disk(model_id: str, out_dir, config: EngineConfig | None = None, progress_every: int = 50,
                           max_workers: int | None = None, control=None, source_dir=None,
                           revision: str | None = None, hf_config=None) -> dict:
    """safetensors -> one `weights.bin` + `manifest.json` (schema v2),
    readable by the reference engine and by this one (reference
    streaming_engine.py:256-428; same parameters). The encoder is
    multi-threaded C++, so tensors are compressed in-process in checkpoint
    order (embedding and head first, as the reference writes them):
    `max_workers`, the reference's process-pool size, is validated and
    otherwise unused. `control.checkpoint()` runs before each tensor."""
    from safetensors import safe_open

    if max_workers is not None and max_workers < 1:
        raise ValueError("max_workers must be >= 1")

    snap = _resolve_snapshot(model_id, source_dir, revision)
    shards = _weight_shards(snap)
    if not shards:
        raise FileNotFoundError("no .safetensors in " + str(snap))
    if hf_config is None:
        from transformers import AutoConfig
        hf_config = AutoConfig.from_pretrained(snap, trust_remote_code=False)
    tasks = []
    for shard in shards:
        with safe_open(str(shard), framework="pt", device="cpu") as f:
            tasks.extend((str(shard), key) for key in f.keys())
    tasks = ([t for t in tasks if t[1].endswith(_BIG_TENSOR_SUFFIXES)]
             + [t for t in tasks if not t[1].endswith(_BIG_TENSOR_SUFFIXES)])

    def items():
        for shard, key in tasks:
            with safe_open(shard, framework="pt", device="cpu") as f:
                yield key, f.get_tensor(key)

    return write_store(items(), out_dir, config, tied=bool(getattr(hf_config, "tie_word_embeddings", False)),
                       model_id=model_id, revision=revision, progress_every=progress_every, total=len(tasks),
                       control=control)


# ---------------------------------------------------------------------------
# online engine
# ---------------------------------------------------------------------------

def layer_working_set(manifest: dict) -> int:
    """Device bytes one streamed decoder layer holds while it runs: its
    compressed upload plus its decoded weights (upper bound: every tensor of
    the layer streamed; a layer is decoded by one launch)."""
    per: dict[int, int] = {}
    for key, meta in manifest["tensors"].items():
        if key.startswith("model.layers.") and not meta.get("row_gather"):
            i = int(key.split(".")[2])
            per[i] = per.get(i, 0) + int(meta["orig_bytes"]) + int(meta.get("comp_bytes", 0))
    return max(per.values(), default=0)


def engine_headroom_bytes(manifest: dict, cfg: EngineConfig, stream_only: dict | None = None,
                          activation_slack_bytes: int | None = None) -> int:
    """VRAM the streaming engine keeps free of resident tensors: the larger
    of the biggest tensor it materialises and `max_inflight_layers` streamed
    layers, plus decode scratch and activations."""
    from .vram_planner import DEFAULT_ACTIVATION_SLACK_BYTES, decode_scratch_bytes
    stream_only = stream_only or {}
    largest = 0
    for key, meta in manifest["tensors"].items():
        if not meta.get("row_gather"):
            largest = max(largest, int(stream_only.get(key, meta["orig_bytes"])))
    slack = DEFAULT_ACTIVATION_SLACK_BYTES if activation_slack_bytes is None else activation_slack_bytes
    return (max(largest, cfg.max_inflight_layers * layer_working_set(manifest))
            + decode_scratch_bytes(cfg.decode_slice_elems) + slack)


def _split_key(root: torch.nn.Module, key: str):
    mod_path, _, name = key.rpartition(".")
    return (root.get_submodule(mod_path) if mod_path else root), name


def _set_param(root: torch.nn.Module, key: str, value: torch.Tensor) -> None:
    mod, name = _split_key(root, key)
    if name in mod._parameters:
        mod._parameters[name] = torch.nn.Parameter(value, requires_grad=False)
    else:
        mod._buffers[name] = value


def _to_meta(root: torch.nn.Module, key: str) -> None:
    mod, name = _split_key(root, key)
    cur = mod._parameters.get(name)
    if cur is not None:
        mod._parameters[name] = torch.nn.Parameter(torch.empty(cur.shape, dtype=cur.dtype, device="meta"),
                                                   requires_grad=False)


def _encoded_from_arrays(meta: dict, arrays: dict) -> CompressedLayer:
    n = int(meta["n_symbols"])
    enc = ChunkedEncoded(packed=arrays["packed"], chunk_offsets=arrays["chunk_offsets"],
                         chunk_nbytes=arrays["chunk_nbytes"], sym_lut=arrays["sym_lut"], len_lut=arrays["len_lut"],
                         max_bits=int(meta["max_bits"]), chunk_size=int(meta["chunk_size"]), n_symbols=n,
                         shape=(n,))
    sm = arrays["sign_mantissa"]
    sm_t = sm if isinstance(sm, torch.Tensor) else torch.from_numpy(np.asarray(sm))
    return CompressedLayer(sign_mantissa=sm_t, encoded=enc, shape=tuple(meta["shape"]))


def _raw_tensor(meta: dict, raw) -> torch.Tensor:
    t = raw if isinstance(raw, torch.Tensor) else torch.from_numpy(np.asarray(raw))
    dt = meta.get("dtype", "bfloat16")
    if t.dtype == torch.int16 and "bfloat16" in dt:
        return t.view(torch.bfloat16)
    if "bfloat16" in dt:
        return t.to(torch.bfloat16)
    if "float16" in dt:
        return t.to(torch.float16)
    return t


class RowGatherEmbedding(torch.nn.Module):
    """Embedding whose table stays in the store: each forward reads only the
    rows of the requested token ids (reference streaming_engine.py:1232-1271)."""

    def __init__(self, engine: "StreamingLosslessModel", meta: dict, padding_idx=None):
        super().__init__()
        ref = meta["blobs"]["raw"]
        self._engine = engine
        self._offset = int(ref["offset"])
        self.hidden = int(meta["hidden_size"])
        self.num_embeddings = int(meta["shape"][0])
        self.padding_idx = padding_idx

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        eng = self._engine
        t0 = time.perf_counter()
        flat = input_ids.reshape(-1).detach().cpu().numpy()
        with eng._reader_lock:
            rows = eng._reader.read_rows(self._offset, flat, self.hidden * 2, "int16")
        eng.stats.bytes_read += rows.nbytes
        eng.stats.io_seconds += time.perf_counter() - t0
        t = torch.from_numpy(np.ascontiguousarray(rows)).view(torch.bfloat16)
        return t.to(eng.device, non_blocking=False).view(*input_ids.shape, self.hidden)


class StreamingLosslessModel:
    """Layer-at-a-time execution from a compressed store."""

    CHUNKED_HEAD_KEY = "lm_head.weight"

    def __init__(self, model_id: str, store_dir, device: str = "cuda", config: EngineConfig | None = None,
                 control=None, source_dir=None, hf_config=None):
        from transformers import AutoConfig, AutoModelForCausalLM

        self.config = config or EngineConfig()
        self.control = control      # pause/cancel boundary once per layer load (checkpoint()), as the reference
        self.store = pathlib.Path(store_dir)
        self.manifest = json.loads((self.store / "manifest.json").read_text())
        self._check_store_integrity()
        self.device = _device.cuda_device(device)
        self.stats = StreamStats()
        self._reader = BinaryWeightReader(self.store / "weights.bin", direct=self.config.direct_io)
        self._reader_lock = threading.Lock()

        if hf_config is None:
            hf_config = AutoConfig.from_pretrained(source_dir if source_dir is not None else model_id,
                                                   trust_remote_code=False)
        self.hf_cfg = hf_config
        with torch.device("meta"):
            self.model = AutoModelForCausalLM.from_config(hf_config, dtype=torch.bfloat16)
        self.model.eval()
        self.layers = self.model.model.layers
        self.n_layers = len(self.layers)
        self._layer_keys = [self._layer_param_keys(i) for i in range(self.n_layers)]

        if self.config.vram_cap_gb is not None:
            total = torch.cuda.get_device_properties(self.device).total_memory
            torch.cuda.set_per_process_memory_fraction(min(1.0, self.config.vram_cap_gb * 1e9 / total),
                                                       self.device)
        self._tier = self._compute_tier_assignment()
        self._decoder = LayerDecoder(self.device)
        self._copy_stream = torch.cuda.Stream(self.device)
        self._tables: dict[str, _gd.DecodeTables] = {}      # per-tensor decode tables, built once
        self._ram_cache: dict = {}                          # key -> pinned BF16 tensor or pinned arrays
        self._vram_compressed: dict[str, ResidentLayer] = {}
        self._kv_cache = None

        depth = self.config.io_prefetch_depth
        self._prefetch = depth > 0
        self._slots = [PinnedBuffer() for _ in range(depth + 1)] if self._prefetch else [PinnedBuffer()]
        self._slot_free = [None] * len(self._slots)          # CUDA event: H2D from the slot finished
        self._slot_readers = [BinaryWeightReader(self.store / "weights.bin", direct=self.config.direct_io,
                                                 threads=self.config.io_threads)
                              for _ in self._slots]
        self._pool = concurrent.futures.ThreadPoolExecutor(max_workers=max(1, depth), thread_name_prefix="aib-io")
        self._futures: dict[int, concurrent.futures.Future] = {}
        self._inflight: list = []   # (layer, compute-stream event after its forward), oldest first
        self._head_future = None
        self._frees = 0             # layer frees, for empty_cache_every
        self._head_reader = None
        self._head_buf = None
        if self._chunked_head_rows():
            self._head_reader = BinaryWeightReader(self.store / "weights.bin", direct=self.config.direct_io,
                                                   threads=self.config.io_threads)
            self._head_buf = PinnedBuffer()

        self._materialize_resident()
        self._install_hooks()

    # -- store -------------------------------------------------------------
    def _check_store_integrity(self) -> None:
        version = self.manifest.get("schema_version")
        if version != CURRENT_SCHEMA_VERSION:
            raise RuntimeError("store at %s has schema_version=%r, this code expects %d -- re-run "
                               "compress_model_to_disk" % (self.store, version, CURRENT_SCHEMA_VERSION))
        weights = self.store / "weights.bin"
        if not weights.exists():
            raise RuntimeError("no weights.bin found at %s" % self.store)
        need = 0
        for meta in self.manifest["tensors"].values():
            for ref in meta.get("blobs", {}).values():
                need = max(need, ref["offset"] + ref["nbytes"])
        have = weights.stat().st_size
        if have < need:
            raise RuntimeError("weights.bin at %s is truncated: manifest references bytes up to offset %d but "
                               "the file is only %d bytes -- the store is incomplete or was corrupted; "
                               "recompress it" % (weights, need, have))

    def _layer_param_keys(self, idx: int) -> list[str]:
        layer = self.layers[idx]
        keys = []
        for pname, _ in layer.named_parameters():
            key = "model.layers.%d.%s" % (idx, pname)
            if key in self.manifest["tensors"]:
                keys.append(key)
        return keys

    def _chunked_head_rows(self) -> int:
        """Rows of lm_head per block, or 0 when chunking is off or does not
        apply: a tied head has no tensor of its own and a raw-stored head no
        chunk ranges (reference streaming_engine.py:877-892)."""
        if self.config.lm_head_slice_rows <= 0:
            return 0
        meta = self.manifest["tensors"].get(self.CHUNKED_HEAD_KEY)
        if not meta or not meta.get("compressed") or len(meta["shape"]) != 2:
            return 0
        return self.config.lm_head_slice_rows

    def _stream_only_overrides(self) -> dict:
        """{key: bytes live at once} for tensors computed in blocks and never
        held whole (reference :894-902)."""
        step = self._chunked_head_rows()
        if not step:
            return {}
        rows, cols = self.manifest["tensors"][self.CHUNKED_HEAD_KEY]["shape"]
        return {self.CHUNKED_HEAD_KEY: min(step, rows) * cols * 2}

    def _compute_tier_assignment(self) -> dict[str, str]:
        """key -> "vram" | "ram" | "disk" | "row_gather" (reference
        streaming_engine.py:904-1043): without a budget every decoder-layer
        tensor streams and everything else is resident; with one, the
        planner ranks all tensors. A chunked head always streams.

        The headroom given to the planner is this engine's working set: the
        largest tensor it materialises, or `max_inflight_layers` streamed
        layers (each a compressed upload plus its decoded weights, since a
        layer is decoded by one launch), whichever is larger, plus decode
        scratch and activations -- so the budget bounds the measured peak."""
        cfg = self.config
        tiers = {k: "row_gather" for k, m in self.manifest["tensors"].items() if m.get("row_gather")}
        chunked = self.CHUNKED_HEAD_KEY if self._chunked_head_rows() else None
        if chunked:
            tiers[chunked] = "disk"
        if not cfg.uses_tiered_residency:
            for key in self.manifest["tensors"]:
                tiers.setdefault(key, "disk" if key.startswith("model.layers.") else "vram")
            return tiers
        from .vram_planner import DEFAULT_ACTIVATION_SLACK_BYTES, kv_cache_bytes_per_token, plan_from_manifest
        slack = DEFAULT_ACTIVATION_SLACK_BYTES
        if cfg.max_context is not None:
            slack += kv_cache_bytes_per_token(self.hf_cfg) * cfg.max_context
        stream_only = self._stream_only_overrides()
        headroom = (engine_headroom_bytes(self.manifest, cfg, stream_only, slack)
                    + int(cfg.vram_safety_margin_gb * 1e9))
        plan = plan_from_manifest(self.manifest, vram_budget_gb=cfg.vram_budget_gb,
                                  ram_budget_gb=cfg.ram_budget_gb or 0.0, stream_only=stream_only,
                                  vram_headroom_bytes=headroom, placement_policy=cfg.placement_policy)
        if not plan.feasible:
            raise RuntimeError("VRAM budget is infeasible: " + plan.reason)
        self.plan = plan
        for k in plan.vram_keys:
            tiers[k] = "vram"
        for k in plan.ram_keys:
            tiers[k] = "ram"
        for k in plan.disk_keys:
            tiers[k] = "disk"
        return tiers

    def tier_of(self, key: str) -> str:
        return self._tier.get(key, "disk")

    def _read_arrays(self, keys: list[str], reader: BinaryWeightReader, pinned) -> dict[str, dict]:
        """Every blob of `keys` in one read_many call, merged into extents as
        storage_read_policy says: "per_blob" one read per stored array,
        "tensor_extents" adjacent arrays of one tensor, "coalesced_extents"
        adjacent arrays of all of them (within the gap / extent bounds). The
        policy changes the reads, never the bytes."""
        cfg = self.config
        named = [(k, name, ref) for k in keys for name, ref in self.manifest["tensors"][k]["blobs"].items()]
        per_blob = cfg.storage_read_policy == "per_blob"
        t0 = time.perf_counter()
        arrays, calls, nbytes = reader.read_many([r for _, _, r in named],
                                                 max_gap_bytes=0 if per_blob else cfg.storage_extent_max_gap_bytes,
                                                 max_extent_bytes=1 if per_blob else cfg.storage_extent_max_bytes,
                                                 pinned=pinned,
                                                 groups=[k for k, _, _ in named]
                                                 if cfg.storage_read_policy == "tensor_extents" else None)
        out: dict[str, dict] = {k: {} for k in keys}
        for (k, name, _), a in zip(named, arrays):
            out[k][name] = a
        self.stats.io_seconds += time.perf_counter() - t0
        self.stats.storage_read_calls += calls
        self.stats.bytes_read += nbytes
        return out

    def _tables_for(self, key: str, enc: ChunkedEncoded) -> _gd.DecodeTables:
        t = self._tables.get(key)
        if t is None:
            t = _gd.prepare_decode_tables(enc, self.device)
            self._tables[key] = t
        return t

    # -- residency -----------------------------------------------------------
    def _decode_whole(self, key: str, arrays: dict) -> torch.Tensor:
        meta = self.manifest["tensors"][key]
        if not meta["compressed"]:
            return _raw_tensor(meta, arrays["raw"]).reshape(meta["shape"]).to(self.device)
        return decompress_layer_gpu(_encoded_from_arrays(meta, arrays), device=self.device,
                                    max_slice_elems=self.config.decode_slice_elems,
                                    reuse_decode_tables=self.config.reuse_decode_tables)

    def _materialize_resident(self) -> None:
        """VRAM / RAM tiers once, then re-tie the head to the embedding
        where the checkpoint stores only one (reference :1273-1456)."""
        embed_key = "model.embed_tokens.weight"
        row_gather = self._tier.get(embed_key) == "row_gather"
        missing = []
        for name, mod in self.model.named_modules():
            if row_gather and name == "model.embed_tokens":
                continue
            nonpersistent = getattr(mod, "_non_persistent_buffers_set", set())
            items = list(mod.named_parameters(recurse=False)) + [
                (b, t) for b, t in mod.named_buffers(recurse=False) if b not in nonpersistent]
            for pname, _ in items:
                key = (name + "." + pname) if name else pname
                if key not in self.manifest["tensors"]:
                    missing.append(key)
                    continue
                tier = self.tier_of(key)
                meta = self.manifest["tensors"][key]
                if tier in ("disk", "row_gather"):
                    continue
                arrays = self._read_arrays([key], self._reader, pinned=False)[key]
                if tier == "vram":
                    if (self.config.vram_tier_format == "compressed" and meta["compressed"]
                            and key.startswith("model.layers.")):
                        self._vram_compressed[key] = upload_layer(_encoded_from_arrays(meta, arrays), self.device)
                    else:
                        _set_param(self.model, key, self._decode_whole(key, arrays))
                else:  # ram
                    if self.config.ram_tier_format == "compressed" and meta["compressed"]:
                        from .layer_decode import pin_layer
                        self._ram_cache[key] = pin_layer(_encoded_from_arrays(meta, arrays))
                    else:
                        self._ram_cache[key] = self._decode_whole(key, arrays).to("cpu").pin_memory()
        # rotary tables are non-persistent buffers built at init: rebuild on the device
        lm = self.model.model
        if getattr(lm, "rotary_emb", None) is not None:
            lm.rotary_emb = type(lm.rotary_emb)(config=self.hf_cfg, device=self.device)
        tied = bool(getattr(self.hf_cfg, "tie_word_embeddings", False))
        if tied and "lm_head.weight" in missing:
            self.model.lm_head.weight = self.model.model.embed_tokens.weight
            missing.remove("lm_head.weight")
        if row_gather:
            if embed_key in missing:
                missing.remove(embed_key)
            old = self.model.model.embed_tokens
            self.model.model.embed_tokens = RowGatherEmbedding(self, self.manifest["tensors"][embed_key],
                                                               getattr(old, "padding_idx", None))
        if missing:
            raise RuntimeError("resident parameters with no source in the store and no tying rule to cover "
                               "them: " + ", ".join(missing[:8]))
        torch.cuda.synchronize(self.device)
        self.stats.reset()

    # -- per-layer streaming ---------------------------------------------------
    def _disk_keys(self, idx: int) -> list[str]:
        return [k for k in self._layer_keys[idx] if self.tier_of(k) == "disk"]

    def _start_prefetch(self, idx: int) -> None:
        if not self._prefetch or idx >= self.n_layers or idx in self._futures:
            return
        keys = self._disk_keys(idx)
        if not keys:
            return
        slot = idx % len(self._slots)
        ev = self._slot_free[slot]
        if ev is not None:
            ev.synchronize()  # the slot's previous upload has left host memory
            self._slot_free[slot] = None
        self._futures[idx] = self._pool.submit(self._read_arrays, keys, self._slot_readers[slot], self._slots[slot])

    def _fetch_layer(self, idx: int) -> tuple[dict, int]:
        keys = self._disk_keys(idx)
        slot = idx % len(self._slots)
        fut = self._futures.pop(idx, None)
        if fut is None:
            self.stats.prefetch_misses += 1 if self._prefetch else 0
            ev = self._slot_free[slot]
            if ev is not None:
                ev.synchronize()
                self._slot_free[slot] = None
            arrays = self._read_arrays(keys, self._slot_readers[slot], self._slots[slot]) if keys else {}
        else:
            if fut.done():
                self.stats.prefetch_hits += 1
            else:
                self.stats.prefetch_misses += 1
            arrays = fut.result()
        return arrays, slot

    def _upload_on_copy_stream(self, layers: dict[str, CompressedLayer]) -> tuple[dict[str, ResidentLayer], torch.cuda.Event]:
        compute = torch.cuda.current_stream(self.device)
        resident = {}
        with torch.cuda.stream(self._copy_stream):
            for key, layer in layers.items():
                enc = layer.encoded
                n = int(np.asarray(enc.packed).shape[0])
                cap = max(16, (n + 15) // 16 * 16)
                packed = torch.empty(cap, dtype=torch.uint8, device=self.device)
                packed[:n].copy_(torch.from_numpy(np.asarray(enc.packed)), non_blocking=True)
                offs = torch.from_numpy(np.asarray(enc.chunk_offsets)).to(self.device, non_blocking=True)
                nbs = torch.from_numpy(np.asarray(enc.chunk_nbytes)).to(self.device, non_blocking=True)
                sm_src = layer.sign_mantissa
                sm_src = sm_src if isinstance(sm_src, torch.Tensor) else torch.from_numpy(np.asarray(sm_src))
                sm = sm_src.reshape(-1).to(self.device, non_blocking=True)
                for t in (packed, offs, nbs, sm):
                    t.record_stream(compute)
                self.stats.h2d_bytes += cap + offs.numel() * 8 + sm.numel()
                ds = _device.DeviceStream(packed=packed, nbytes=n, capacity=cap, offset_base=0, offsets=offs,
                                          chunk_nbytes=nbs, chunk_base=0)
                resident[key] = ResidentLayer(stream=ds, sign_mantissa=sm, tables=None, encoded=enc,
                                              shape=tuple(layer.shape))
            done = torch.cuda.Event()
            done.record(self._copy_stream)
        return resident, done

    def _decode_into_params(self, module_root: torch.nn.Module, items: dict[str, ResidentLayer]) -> None:
        """One batched decode launch; fresh BF16 tensors become the params."""
        keys = list(items)
        outs = [torch.empty(items[k].shape, dtype=torch.bfloat16, device=self.device) for k in keys]
        res = [items[k] for k in keys]
        t0 = time.perf_counter()
        self._decoder.decode(res, outs)
        self.stats.decode_seconds += time.perf_counter() - t0
        self.stats.decode_launches += (len(keys) + 15) // 16
        for k, o in zip(keys, outs):
            _set_param(module_root, k, o)

    def _bound_inflight(self, keep: int) -> None:
        """Waits until at most `keep` earlier streamed layers can still hold
        device buffers (the host otherwise runs layers ahead of the GPU and
        their uploads and decoded weights pile up past the VRAM budget)."""
        while len(self._inflight) > keep:
            _, ev = self._inflight.pop(0)
            ev.synchronize()

    def _streams(self, idx: int) -> bool:
        """Whether layer idx brings weights over PCIe (disk or RAM tier)."""
        return any(self.tier_of(k) in ("disk", "ram") for k in self._layer_keys[idx])

    def _load_layer(self, idx: int) -> None:
        if self.control is not None:
            self.control.checkpoint()
        if self._streams(idx):
            self._bound_inflight(self.config.max_inflight_layers - 1)
        compute = torch.cuda.current_stream(self.device)
        arrays, slot = self._fetch_layer(idx)
        for ahead in range(1, self.config.io_prefetch_depth + 1):
            self._start_prefetch(idx + ahead)
        if idx == max(0, self.n_layers - 2):
            self._start_head_prefetch()
        to_decode: dict[str, ResidentLayer] = {}
        streamed = {k: _encoded_from_arrays(self.manifest["tensors"][k], a)
                    for k, a in arrays.items() if self.manifest["tensors"][k]["compressed"]}
        for k in self._layer_keys[idx]:
            tier = self.tier_of(k)
            if tier == "ram":
                cached = self._ram_cache[k]
                if isinstance(cached, CompressedLayer):
                    streamed[k] = cached
                else:
                    _set_param(self.model, k, cached.to(self.device, non_blocking=True))
            elif tier == "vram" and k in self._vram_compressed:
                to_decode[k] = self._vram_compressed[k]
            elif tier == "disk" and not self.manifest["tensors"][k]["compressed"]:
                _set_param(self.model, k, _raw_tensor(self.manifest["tensors"][k], arrays[k]["raw"])
                           .reshape(self.manifest["tensors"][k]["shape"]).to(self.device))
        if streamed:
            t0 = time.perf_counter()
            uploaded, done = self._upload_on_copy_stream(streamed)
            self.stats.h2d_seconds += time.perf_counter() - t0
            compute.wait_event(done)
            if arrays:
                self._slot_free[slot] = done
            for k, r in uploaded.items():
                r.tables = self._tables_for(k, r.encoded)
            to_decode.update(uploaded)
        for k, r in to_decode.items():
            if r.tables is None:
                r.tables = self._tables_for(k, r.encoded)
        if to_decode:
            self._decode_into_params(self.model, to_decode)
        self.stats.layer_loads += 1

    def _free_layer(self, idx: int) -> None:
        if self._streams(idx):
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self._inflight.append((idx, ev))
        for k in self._layer_keys[idx]:
            if self.tier_of(k) == "vram" and k not in self._vram_compressed:
                continue
            _to_meta(self.model, k)
        self._frees += 1
        every = self.config.empty_cache_every
        if every and self._frees % every == 0:
            torch.cuda.empty_cache()

    def _install_hooks(self) -> None:
        """transformers drives the stack (masks, rotary, cache); hooks only
        bring each layer's weights in before it runs and drop them after."""
        def make_pre(i):
            def pre(module, args, kwargs):
                self._load_layer(i)
            return pre

        def make_post(i):
            def post(module, args, kwargs, output):
                self._free_layer(i)
                return output
            return post

        for i, layer in enumerate(self.layers):
            layer.register_forward_pre_hook(make_pre(i), with_kwargs=True)
            layer.register_forward_hook(make_post(i), with_kwargs=True)
        self._install_streamed_module_hooks()

    def _load_whole(self, key: str) -> torch.Tensor:
        """One disk- or RAM-tier tensor outside the decoder layers, whole on
        the device for one use: decoded from the store, from its compressed
        pinned copy, or copied from its pinned BF16 copy."""
        if self.tier_of(key) == "ram":
            cached = self._ram_cache[key]
            if isinstance(cached, CompressedLayer):
                return decompress_layer_gpu(cached, device=self.device,
                                            max_slice_elems=self.config.decode_slice_elems,
                                            reuse_decode_tables=self.config.reuse_decode_tables)
            return cached.to(self.device, non_blocking=True)
        return self._decode_whole(key, self._read_arrays([key], self._reader, pinned=False)[key])

    def _install_streamed_module_hooks(self) -> None:
        """Non-layer tensors that the plan leaves on disk or in host RAM (e.g.
        lm_head, or a tied embedding, at a small budget) are loaded just
        before their module runs and dropped after it (reference
        streaming_engine.py:1952-2091).

        A tied checkpoint stores only the embedding. When that streams, the
        embedding module's post-hook swaps its parameter for a fresh meta
        placeholder, so lm_head cannot share it: the head loads the same
        stored tensor again for its own live range. (A meta weight given to
        F.linear does not raise; it yields uninitialised logits.)"""
        groups: dict[str, list[str]] = {}
        chunked = self.CHUNKED_HEAD_KEY if self._chunked_head_rows() else None
        for key, tier in self._tier.items():
            if tier in ("disk", "ram") and not key.startswith("model.layers.") and key != chunked:
                groups.setdefault(key.rpartition(".")[0], []).append(key)
        embed_key = "model.embed_tokens.weight"
        if (bool(getattr(self.hf_cfg, "tie_word_embeddings", False))
                and "lm_head.weight" not in self.manifest["tensors"]
                and self._tier.get(embed_key) in ("disk", "ram")):
            groups.setdefault("lm_head", []).append(("lm_head.weight", embed_key))
        for mod_name, keys in groups.items():
            mod = self.model.get_submodule(mod_name)
            pairs = [k if isinstance(k, tuple) else (k, k) for k in keys]

            def pre(module, args, pairs=pairs):
                self._bound_inflight(0)
                for dst, src in pairs:
                    _set_param(self.model, dst, self._load_whole(src))

            def post(module, args, output, pairs=pairs):
                for dst, _ in pairs:
                    _to_meta(self.model, dst)
                return output
            mod.register_forward_pre_hook(pre)
            mod.register_forward_hook(post)
        if chunked:
            self._install_chunked_lm_head()

    def _start_head_prefetch(self) -> None:
        """The chunked head's compressed bytes are read into their own
        page-locked buffer while the last layers run (its block uploads
        then copy by DMA). Its uploads finish before the head returns, so
        the buffer is free again for the next forward."""
        if self._head_reader is None or self._head_future is not None:
            return
        self._head_future = self._pool.submit(self._read_arrays, [self.CHUNKED_HEAD_KEY], self._head_reader,
                                              self._head_buf)

    def _install_chunked_lm_head(self) -> None:
        """Logits in row blocks instead of a materialised lm_head (reference
        streaming_engine.py:2271-2334): logits[..., a:b] = x @ W[a:b].T, each
        block decoded from its chunk range by decompress_rows_gpu, so only
        one block's weights are live. The compressed bytes are read once per
        forward; the result is the same matmul in pieces."""
        step = self._chunked_head_rows()
        key = self.CHUNKED_HEAD_KEY
        meta = self.manifest["tensors"][key]
        rows = int(meta["shape"][0])

        def forward(x: torch.Tensor) -> torch.Tensor:
            self._bound_inflight(0)
            fut, self._head_future = self._head_future, None
            arrays = (fut.result() if fut is not None
                      else self._read_arrays([key], self._head_reader, self._head_buf))[key]
            layer = _encoded_from_arrays(meta, arrays)
            parts = []
            for r0 in range(0, rows, step):
                t0 = time.perf_counter()
                W = decompress_rows_gpu(layer, r0, min(rows, r0 + step), device=self.device)
                self.stats.decode_seconds += time.perf_counter() - t0
                parts.append(torch.nn.functional.linear(x, W))
                del W
            return torch.cat(parts, dim=-1)

        self.model.lm_head.forward = forward

    # -- inference --------------------------------------------------------------
    @torch.no_grad()
    def forward_logits(self, input_ids: torch.Tensor, use_cache: bool = False) -> torch.Tensor:
        t0 = time.perf_counter()
        io0, dec0, h2d0 = self.stats.io_seconds, self.stats.decode_seconds, self.stats.h2d_seconds
        for ahead in range(self.config.io_prefetch_depth):
            self._start_prefetch(ahead)
        input_ids = input_ids.to(self.device)
        if use_cache:
            out = self.model(input_ids=input_ids, use_cache=True, past_key_values=self._kv_cache)
            self._kv_cache = out.past_key_values
        else:
            out = self.model(input_ids=input_ids, use_cache=False)
        torch.cuda.synchronize(self.device)
        # the decodes of this forward were stream-ordered; a corrupt stream raises here
        _device.check_status(self.device)
        wall = time.perf_counter() - t0
        self.stats.compute_seconds += max(0.0, wall - (self.stats.io_seconds - io0)
                                          - (self.stats.decode_seconds - dec0) - (self.stats.h2d_seconds - h2d0))
        self.stats.target_seconds += wall
        return out.logits

    @torch.no_grad()
    def generate_greedy(self, input_ids: torch.Tensor, max_new_tokens: int, use_cache: bool = True,
                        on_token=None, stop_token_ids=()) -> torch.Tensor:
        seq = input_ids.to(self.device)
        self._kv_cache = None
        step = seq
        t0 = time.perf_counter()
        for i in range(max_new_tokens):
            logits = self.forward_logits(step, use_cache=use_cache)
            nxt = logits[:, -1, :].argmax(dim=-1, keepdim=True)
            seq = torch.cat([seq, nxt], dim=1)
            step = nxt if use_cache else seq
            tok = int(nxt.item())
            self._progress(i + 1, max_new_tokens, t0)
            if on_token is not None:
                on_token(tok)
            if tok in stop_token_ids:
                break
        self._progress(None, max_new_tokens, t0)
        return seq

    def _progress(self, done: int | None, total: int, t0: float) -> None:
        """One stderr line per generated token when config.progress is set
        (done=None ends the line)."""
        if not self.config.progress:
            return
        if done is None:
            sys.stderr.write("\n")
        else:
            dt = time.perf_counter() - t0
            sys.stderr.write("\r[afterimage_b200] token %d/%d, %.2f s/token" % (done, total, dt / done))
        sys.stderr.flush()

    @torch.no_grad()
    def generate_speculative(self, input_ids: torch.Tensor, max_new_tokens: int, draft_model, k: int | None = None,
                             temperature: float = 1.0, generator: torch.Generator | None = None) -> torch.Tensor:
        """Draft/verify speculation (reference :2488-2575): a resident draft
        proposes k tokens, one target sweep scores the chain, and
        speculative_sample_step accepts a prefix plus one token. At
        temperature <= 0 the output equals generate_greedy's."""
        k = k or self.config.spec_k
        draft_vocab = getattr(draft_model.config, "vocab_size", None)
        target_vocab = self.model.lm_head.weight.shape[0]
        if draft_vocab is not None and draft_vocab != target_vocab:
            raise ValueError("draft_model's vocabulary (%d) does not match this model's (%d)"
                             % (draft_vocab, target_vocab))
        seq = input_ids.to(self.device)
        self._kv_cache = None
        produced = 0
        while produced < max_new_tokens:
            step_k = min(k, max_new_tokens - produced)
            t0 = time.perf_counter()
            draft_seq, draft_tokens, draft_probs = seq, [], []
            for _ in range(step_k):
                dl = draft_model(input_ids=draft_seq).logits[0, -1, :]
                p = temperature_probs(dl, temperature)
                tok = sample_categorical(p, generator)
                draft_tokens.append(tok)
                draft_probs.append(p)
                draft_seq = torch.cat([draft_seq, torch.tensor([[tok]], device=self.device)], dim=1)
            self.stats.draft_seconds += time.perf_counter() - t0
            base = seq.shape[1] - 1
            tl = self.forward_logits(draft_seq, use_cache=False)[0]
            target_probs = [temperature_probs(tl[base + i], temperature) for i in range(step_k)]
            bonus = temperature_probs(tl[base + step_k], temperature)
            accepted, n_draft = speculative_sample_step(draft_probs, target_probs, draft_tokens, bonus, generator)
            seq = torch.cat([seq, torch.tensor([accepted], device=self.device)], dim=1)
            produced += len(accepted)
            self.stats.spec_sweeps += 1
            self.stats.spec_accepted_tokens += n_draft
        return seq[:, :input_ids.shape[1] + max_new_tokens]

    # -- lifetime ---------------------------------------------------------------
    def quiesce_prefetch(self) -> None:
        """Waits for every background read this engine started and drops its
        result (reference streaming_engine.py:647-666): afterwards no reader
        touches the store until the next forward, e.g. before a caller drops
        the OS page cache. The next forward reads what it needs again."""
        pending = list(self._futures.values())
        if self._head_future is not None:
            pending.append(self._head_future)
        concurrent.futures.wait(pending)
        self._futures.clear()
        self._head_future = None

    def close(self) -> None:
        for fut in self._futures.values():
            fut.cancel()
        self._futures.clear()
        self._pool.shutdown(wait=True)
        for r in [self._reader] + self._slot_readers + ([self._head_reader] if self._head_reader else []):
            r.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


def load_draft_model(model_id: str = "Qwen/Qwen3-0.6B", device: str = "cuda"):
    """A small, fully resident BF16 model for generate_speculative's draft
    step (reference streaming_engine.py:2734-2748). It must share the
    target's vocabulary; it is loaded the ordinary way, not streamed."""
    from transformers import AutoModelForCausalLM
    m = AutoModelForCausalLM.from_pretrained(model_id, dtype=torch.bfloat16)
    m.to(device)
    m.eval()
    return m
