"""Three-tier residency planner (VRAM / pinned RAM / disk) -- drop-in for
the reference's afterimage/runtime/vram_planner.py (TensorInfo :115-131,
TierPlan :134-196, decode_scratch_bytes :252-263, plan_tiers :266-402,
plan_from_manifest :414-466, kv_cache_bytes_per_token :216-249).

The ranking is the reference's: every tensor is worth
uses * comp_bytes / orig_bytes of bus traffic avoided per byte of residency
(`value_density`), filled greedily into VRAM then RAM; row-gathered tensors
are excluded; stream-only tensors always stream and reserve only their
materialised block. Plans are identical to the reference's for the same
inputs and the same per-element decode scratch.

What changes is the decode-scratch model. The reference decoder holds, per
element of a slice, a uint8 exponent plus int16 temporaries for the
recombine (10 bytes with slack). The fused decoder here writes BF16 straight
from the compressed stream, so a slice only needs its inputs on the device:
one sign/mantissa byte plus the slice's share of the packed exponent stream
(at most ~1 byte) -- 2 bytes per element. Lower scratch is what lowers the
minimum feasible VRAM budget.
"""
from __future__ import annotations

import dataclasses

# bytes of transient device memory per element of one decode slice
DECODE_SCRATCH_BYTES_PER_ELEM = 2
DEFAULT_SCRATCH_BYTES = 512 * 1024 * 1024
DEFAULT_ACTIVATION_SLACK_BYTES = 128 * 1024 * 1024


@dataclasses.dataclass
class TensorCost:
    """Measured per-tensor costs (the fields plan_from_manifest reads from
    a critical-path profile)."""
    key: str
    read_s: float = 0.0
    decode_s: float = 0.0
    transfer_s: float = 0.0
    counterfactual_s: float = 0.0
    observations: int = 0


@dataclasses.dataclass
class CriticalPathProfile:
    tensors: dict


@dataclasses.dataclass
class TensorInfo:
    key: str
    orig_bytes: int
    comp_bytes: int
    is_layer_weight: bool
    row_gather: bool = False
    uses: int = 1
    stream_only: bool = False
    materialize_override: int | None = None
    profiled_value_s: float = 0.0
    critical_value_s: float = 0.0
    profiled_observed: bool = False
    critical_observed: bool = False

    @property
    def materialize_bytes(self) -> int:
        """Peak bytes this tensor forces live at once (one block for a
        stream-only tensor, else the whole tensor)."""
        return self.materialize_override or self.orig_bytes

    @property
    def value_density(self) -> float:
        return (self.uses * self.comp_bytes) / max(self.orig_bytes, 1)

    def placement_density(self, policy: str) -> float:
        if policy == "traffic_density":
            return self.value_density
        if policy == "profiled_knapsack":
            if self.profiled_observed:
                return (self.uses * self.profiled_value_s) / max(self.orig_bytes, 1)
            return self.value_density
        if policy == "critical_path":
            if self.critical_observed:
                return (self.uses * self.critical_value_s) / max(self.orig_bytes, 1)
            return self.value_density
        raise ValueError("unknown placement policy %r" % policy)


@dataclasses.dataclass
class TierPlan:
    vram_budget_bytes: int
    ram_budget_bytes: int
    vram_headroom_bytes: int
    vram_keys: list
    ram_keys: list
    disk_keys: list
    row_gather_keys: list
    vram_bytes: int
    ram_bytes: int
    disk_bytes_per_token: int
    feasible: bool
    reason: str

    @property
    def vram_budget_gb(self) -> float:
        return self.vram_budget_bytes / 1e9

    @property
    def ram_budget_gb(self) -> float:
        return self.ram_budget_bytes / 1e9

    @property
    def vram_gb(self) -> float:
        return self.vram_bytes / 1e9

    @property
    def ram_gb(self) -> float:
        return self.ram_bytes / 1e9

    @property
    def disk_gb_per_token(self) -> float:
        return self.disk_bytes_per_token / 1e9

    def tier_of(self, key: str) -> str:
        if key in self.vram_keys:
            return "vram"
        if key in self.ram_keys:
            return "ram"
        if key in self.row_gather_keys:
            return "row_gather"
        return "disk"

    def describe(self) -> str:
        out = ["Tier plan -- VRAM %.2f GB / RAM %.2f GB budget:" % (self.vram_budget_gb, self.ram_budget_gb),
               "  vram tier           : %.2f GB across %d tensors" % (self.vram_gb, len(self.vram_keys)),
               "  ram  tier           : %.2f GB across %d tensors" % (self.ram_gb, len(self.ram_keys)),
               "  disk tier (streamed): %.2f GB/token across %d tensors"
               % (self.disk_gb_per_token, len(self.disk_keys))]
        if self.row_gather_keys:
            out.append("  row-gather (excluded): %d tensors" % len(self.row_gather_keys))
        out.append("  vram headroom        : %.2f GB" % (self.vram_headroom_bytes / 1e9))
        out.append("  feasible             : %s" % self.feasible)
        if not self.feasible:
            out.append("  reason               : " + self.reason)
        return "\n".join(out)


def decode_scratch_bytes(decode_slice_elems: int) -> int:
    """Transient VRAM one decode slice needs (reference :252-263, with this
    decoder's per-element scratch)."""
    return decode_slice_elems * DECODE_SCRATCH_BYTES_PER_ELEM


def kv_cache_bytes_per_token(hf_cfg, dtype_bytes: int = 2) -> int:
    """KV-cache bytes per token: 2 (K and V) x layers x kv_heads x head_dim
    x dtype bytes (reference :216-249)."""
    layers = getattr(hf_cfg, "num_hidden_layers", None)
    heads = getattr(hf_cfg, "num_attention_heads", None)
    if layers is None or heads is None:
        raise ValueError("hf_cfg is missing num_hidden_layers/num_attention_heads -- "
                         "can't estimate KV cache size for this architecture")
    kv_heads = getattr(hf_cfg, "num_key_value_heads", None) or heads
    head_dim = getattr(hf_cfg, "head_dim", None)
    if not head_dim:
        hidden = getattr(hf_cfg, "hidden_size", None)
        if not hidden:
            raise ValueError("hf_cfg has neither head_dim nor hidden_size -- can't estimate "
                             "KV cache size for this architecture")
        head_dim = hidden // heads
    return 2 * layers * kv_heads * head_dim * dtype_bytes


def _infeasible(vram_budget, ram_budget, headroom, tensors, row_gather_keys, reason) -> TierPlan:
    return TierPlan(vram_budget, ram_budget, headroom, [], [], [t.key for t in tensors], row_gather_keys,
                    0, 0, sum(t.comp_bytes for t in tensors), False, reason)


def plan_tiers(tensors, vram_budget_gb: float, ram_budget_gb: float = 0.0,
               vram_headroom_bytes: int = None, scratch_bytes: int = None,
               decode_slice_elems: int = None,
               activation_slack_bytes: int = DEFAULT_ACTIVATION_SLACK_BYTES,
               pin_layer_weights: bool = False, forced_ram_keys=(),
               placement_policy: str = "traffic_density") -> TierPlan:
    """VRAM / RAM / disk assignment for the given budgets (reference
    :266-402). Headroom defaults to the largest materialised tensor plus
    decode scratch plus activation slack; a budget below it is refused up
    front with a reason that names the decode_slice_elems lever."""
    if scratch_bytes is None:
        scratch_bytes = (decode_scratch_bytes(decode_slice_elems) if decode_slice_elems is not None
                         else DEFAULT_SCRATCH_BYTES) + activation_slack_bytes
    eligible = [t for t in tensors if not t.row_gather]
    row_gather_keys = [t.key for t in tensors if t.row_gather]
    forced = set(forced_ram_keys)
    by_key = {t.key: t for t in eligible}
    unknown = forced - set(by_key)
    if unknown:
        raise ValueError("forced RAM keys are not placement candidates: %s" % ", ".join(sorted(unknown)))
    forced_stream = {k for k in forced if by_key[k].stream_only}
    if forced_stream:
        raise ValueError("stream-only tensors cannot be forced into RAM: %s" % ", ".join(sorted(forced_stream)))

    vram_budget = int(vram_budget_gb * 1e9)
    ram_budget = int(ram_budget_gb * 1e9)
    if not eligible:
        return TierPlan(vram_budget, ram_budget, 0, [], [], [], row_gather_keys, 0, 0, 0, True, "")

    largest = max(t.materialize_bytes for t in eligible)
    if vram_headroom_bytes is None:
        vram_headroom_bytes = largest + scratch_bytes
    available = vram_budget - vram_headroom_bytes
    if available < 0:
        return _infeasible(
            vram_budget, ram_budget, vram_headroom_bytes, eligible, row_gather_keys,
            "vram_budget %.2f GB is below the %.2f GB needed just to materialize the largest "
            "eligible tensor (%.2f GB) plus decode scratch and activations (%.2f GB). Lowering "
            "decode_slice_elems shrinks the scratch term and lowers this floor."
            % (vram_budget / 1e9, vram_headroom_bytes / 1e9, largest / 1e9,
               (vram_headroom_bytes - largest) / 1e9))

    streamed = [t for t in eligible if t.stream_only]
    pinned_ram = [by_key[k] for k in sorted(forced)]
    pinned_ram_bytes = sum(t.orig_bytes for t in pinned_ram)
    if pinned_ram_bytes > ram_budget:
        return _infeasible(
            vram_budget, ram_budget, vram_headroom_bytes, eligible, row_gather_keys,
            "forced RAM tensors need %.2f GB, above the %.2f GB RAM budget"
            % (pinned_ram_bytes / 1e9, ram_budget / 1e9))

    candidates = [t for t in eligible if not t.stream_only and t.key not in forced]
    # stable sort, highest traffic avoided per byte first
    ranked = sorted(candidates, key=lambda t: t.placement_density(placement_policy), reverse=True)
    if pin_layer_weights:
        ranked = [t for t in ranked if t.is_layer_weight] + [t for t in ranked if not t.is_layer_weight]

    vram_keys, vram_used, left = [], 0, []
    for t in ranked:
        if vram_used + t.orig_bytes <= available:
            vram_keys.append(t.key)
            vram_used += t.orig_bytes
        else:
            left.append(t)
    ram_keys = [t.key for t in pinned_ram]
    ram_used = pinned_ram_bytes
    disk_keys = [t.key for t in streamed]
    for t in left:
        if ram_used + t.orig_bytes <= ram_budget:
            ram_keys.append(t.key)
            ram_used += t.orig_bytes
        else:
            disk_keys.append(t.key)
    on_disk = set(disk_keys)
    return TierPlan(vram_budget, ram_budget, vram_headroom_bytes, vram_keys, ram_keys, disk_keys,
                    row_gather_keys, vram_used, ram_used,
                    sum(t.comp_bytes for t in eligible if t.key in on_disk), True, "")


def _layer_index(key: str):
    if not key.startswith("model.layers."):
        return None
    try:
        return int(key.split(".")[2])
    except (IndexError, ValueError):
        return None


def plan_from_manifest(manifest: dict, vram_budget_gb: float, ram_budget_gb: float = 0.0,
                       draft_layer_indices=None, draft_uses: int = 1, stream_only: dict | None = None,
                       critical_path_profile=None, placement_policy: str = "traffic_density",
                       **kw) -> TierPlan:
    """Tier plan straight from a compressed store's manifest (reference
    :414-466): draft layers count `draft_uses` times, stream-only tensors
    reserve only their block, profile costs feed the profiled policies."""
    hot = set(draft_layer_indices) if draft_layer_indices else set()
    stream_only = stream_only or {}
    prof = getattr(critical_path_profile, "tensors", None) if critical_path_profile is not None else None

    def measured(key: str, field: str) -> float:
        cost = prof.get(key) if prof is not None else None
        return float(getattr(cost, field)) if cost is not None else 0.0

    infos = []
    for key, meta in manifest["tensors"].items():
        seen = prof is not None and key in prof
        infos.append(TensorInfo(
            key=key, orig_bytes=meta["orig_bytes"], comp_bytes=meta["comp_bytes"],
            is_layer_weight=key.startswith("model.layers."), row_gather=bool(meta.get("row_gather")),
            uses=draft_uses if _layer_index(key) in hot else 1, stream_only=key in stream_only,
            materialize_override=stream_only.get(key),
            profiled_value_s=measured(key, "read_s") + measured(key, "decode_s") + measured(key, "transfer_s"),
            critical_value_s=measured(key, "counterfactual_s"),
            profiled_observed=seen, critical_observed=seen))
    return plan_tiers(infos, vram_budget_gb, ram_budget_gb, placement_policy=placement_policy, **kw)
