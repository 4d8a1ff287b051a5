"""Residency planner: field-for-field parity with plans the reference
planner produced (tests/golden/planner_cases.json), plus the reference's own
behavioural tests (afterimage tests/test_vram_planner.py), with the
decode-scratch numbers restated for the fused decoder's 2 bytes/element."""
import json
import pathlib
import types

import pytest

from afterimage_b200.runtime import vram_planner as vp
from afterimage_b200.runtime.vram_planner import (
    CriticalPathProfile, TensorCost, TensorInfo, kv_cache_bytes_per_token, plan_from_manifest, plan_tiers,
)

GOLDEN = json.loads((pathlib.Path(__file__).parent / "golden" / "planner_cases.json").read_text())


def _plan_dict(p):
    return {k: getattr(p, k) for k in GOLDEN["cases"][0]["plan"]}


@pytest.mark.parametrize("i", range(len(GOLDEN["cases"])))
def test_plans_match_reference_planner(i, monkeypatch):
    monkeypatch.setattr(vp, "DECODE_SCRATCH_BYTES_PER_ELEM", GOLDEN["decode_scratch_bytes_per_elem"])
    c = GOLDEN["cases"][i]
    kw = dict(c["kwargs"])
    if c["kind"] == "plan_tiers":
        if "forced_ram_keys" in kw:
            kw["forced_ram_keys"] = set(kw["forced_ram_keys"])
        got = plan_tiers([TensorInfo(**t) for t in c["tensors"]], **kw)
    else:
        if c["profile"] is not None:
            kw["critical_path_profile"] = CriticalPathProfile(
                {k: TensorCost(k, **v) for k, v in c["profile"].items()})
        got = plan_from_manifest(c["manifest"], **kw)
    assert _plan_dict(got) == c["plan"]


def _t(key, orig_mb, comp_mb, layer=True, row_gather=False, uses=1):
    return TensorInfo(key, int(orig_mb * 1e6), int(comp_mb * 1e6), layer, row_gather, uses)


def test_everything_fits_in_vram_when_budget_is_ample():
    plan = plan_tiers([_t("a", 100, 70), _t("b", 100, 70)], vram_budget_gb=10.0)
    assert plan.feasible and set(plan.vram_keys) == {"a", "b"}
    assert plan.ram_keys == [] and plan.disk_keys == [] and plan.disk_bytes_per_token == 0


def test_infeasible_when_vram_budget_below_largest_tensor_headroom():
    plan = plan_tiers([_t("big", 2000, 1400)], vram_budget_gb=1.0)
    assert not plan.feasible and "largest eligible tensor" in plan.reason and plan.vram_keys == []


def test_least_compressible_tensors_fill_vram_first():
    plan = plan_tiers([_t("sparse", 100, 40), _t("dense", 100, 98)], vram_budget_gb=0.7,
                      scratch_bytes=int(500e6))
    assert plan.vram_keys == ["dense"] and plan.disk_keys == ["sparse"]


def test_ram_tier_catches_what_vram_could_not_hold():
    plan = plan_tiers([_t("a", 100, 90), _t("b", 100, 60), _t("c", 100, 30)], vram_budget_gb=0.7,
                      ram_budget_gb=0.15, scratch_bytes=int(500e6))
    assert (plan.vram_keys, plan.ram_keys, plan.disk_keys) == (["a"], ["b"], ["c"])
    assert plan.disk_bytes_per_token == int(30e6)


def test_forced_ram_overlay_and_its_budget_check():
    head, layer = _t("lm_head.weight", 100, 40, layer=False), _t("layer", 100, 90)
    plan = plan_tiers([head, layer], vram_budget_gb=0.7, ram_budget_gb=0.1, scratch_bytes=int(500e6),
                      forced_ram_keys={"lm_head.weight"})
    assert plan.ram_keys == ["lm_head.weight"] and plan.vram_keys == ["layer"]
    small = plan_tiers([head], vram_budget_gb=0.7, ram_budget_gb=0.05, scratch_bytes=int(500e6),
                       forced_ram_keys={"lm_head.weight"})
    assert not small.feasible and "forced RAM tensors need" in small.reason
    with pytest.raises(ValueError):
        plan_tiers([head], vram_budget_gb=1.0, forced_ram_keys={"nope"})


def test_row_gather_tensors_are_excluded_from_every_tier():
    embed = _t("embed", 1560, 1560, layer=False, row_gather=True)
    plan = plan_tiers([_t("normal", 100, 90), embed], vram_budget_gb=10.0, ram_budget_gb=10.0)
    assert embed.key not in plan.vram_keys + plan.ram_keys + plan.disk_keys
    assert plan.row_gather_keys == ["embed"] and plan.tier_of("embed") == "row_gather"


def test_budgets_are_monotone_in_disk_traffic():
    ts = [_t("a", 100, 90), _t("b", 100, 60), _t("c", 100, 30)]
    prev = None
    for gb in [0.7, 0.8, 0.9, 1.5]:
        d = plan_tiers(ts, vram_budget_gb=gb, scratch_bytes=int(500e6)).disk_bytes_per_token
        assert prev is None or d <= prev
        prev = d
    prev = None
    for ram in [0.0, 0.1, 0.2, 1.0]:
        d = plan_tiers(ts, vram_budget_gb=0.7, ram_budget_gb=ram, scratch_bytes=int(500e6)).disk_bytes_per_token
        assert prev is None or d <= prev
        prev = d


def test_fused_decoder_scratch_lowers_the_feasibility_floor():
    """A 1.56 GB lm_head with 2^25-element slices: the reference decoder's
    10 B/element scratch (335 MB) does not fit 1.9 GB; the fused decoder's
    2 B/element (67 MB) does."""
    ts = [_t("lm_head", 1556, 1100, layer=False), _t("layer", 27, 18)]
    assert plan_tiers(ts, vram_budget_gb=1.9, decode_slice_elems=1 << 25).feasible
    assert vp.decode_scratch_bytes(1 << 25) == 2 * (1 << 25)
    assert not plan_tiers(ts, vram_budget_gb=1.7, decode_slice_elems=1 << 25).feasible
    assert plan_tiers(ts, vram_budget_gb=1.7, decode_slice_elems=1 << 22).feasible


def test_explicit_scratch_overrides_and_reason_names_the_lever():
    plan = plan_tiers([_t("a", 100, 90)], vram_budget_gb=0.7, scratch_bytes=int(500e6))
    assert plan.vram_headroom_bytes == int(100e6) + int(500e6)
    bad = plan_tiers([_t("big", 2000, 1400)], vram_budget_gb=1.0, decode_slice_elems=1 << 25)
    assert not bad.feasible and "decode_slice_elems" in bad.reason


def test_uses_scale_density_and_flip_ranking():
    assert TensorInfo("a", 100, 50, True).uses == 1
    assert _t("b", 100, 50, uses=9).value_density == pytest.approx(9 * _t("a", 100, 50).value_density)
    plan = plan_tiers([_t("layer.30", 100, 50), _t("layer.0", 100, 50, uses=9)], vram_budget_gb=0.7,
                      scratch_bytes=int(500e6))
    assert plan.vram_keys == ["layer.0"] and plan.disk_keys == ["layer.30"]


def test_plan_from_manifest_draft_and_row_gather():
    manifest = {"tensors": {
        "model.embed_tokens.weight": {"orig_bytes": int(1.56e9), "comp_bytes": int(1.56e9), "row_gather": True},
        "model.layers.0.mlp.down_proj.weight": {"orig_bytes": int(27e6), "comp_bytes": int(18e6)},
        "lm_head.weight": {"orig_bytes": int(1.56e9), "comp_bytes": int(1.1e9)}}}
    plan = plan_from_manifest(manifest, vram_budget_gb=3.0)
    assert plan.feasible and plan.row_gather_keys == ["model.embed_tokens.weight"]
    m2 = {"tensors": {f"model.layers.{i}.mlp.down_proj.weight": {"orig_bytes": int(50e6), "comp_bytes": int(25e6)}
                      for i in (0, 1, 30)}}
    d = plan_from_manifest(m2, vram_budget_gb=0.15, scratch_bytes=int(50e6), draft_layer_indices=[0, 1],
                           draft_uses=9)
    assert d.vram_keys[0].startswith(("model.layers.0.", "model.layers.1."))
    assert "model.layers.30.mlp.down_proj.weight" in d.disk_keys


def test_critical_path_policy_preserves_observed_zero_value():
    manifest = {"tensors": {"off_path": {"orig_bytes": int(50e6), "comp_bytes": int(49e6)},
                            "critical": {"orig_bytes": int(50e6), "comp_bytes": int(10e6)}}}
    profile = CriticalPathProfile({"off_path": TensorCost("off_path", counterfactual_s=0.0, observations=1),
                                   "critical": TensorCost("critical", counterfactual_s=2.0, observations=1)})
    plan = plan_from_manifest(manifest, vram_budget_gb=0.15, scratch_bytes=int(50e6),
                              critical_path_profile=profile, placement_policy="critical_path")
    assert plan.vram_keys == ["critical"]


def test_stream_only_and_materialize_override():
    head = TensorInfo("lm_head.weight", int(1556e6), int(1100e6), False, stream_only=True,
                      materialize_override=int(84e6))
    plan = plan_tiers([head, _t("layer", 100, 90)], vram_budget_gb=5.0, scratch_bytes=int(50e6))
    assert "lm_head.weight" in plan.disk_keys and "layer" in plan.vram_keys
    assert plan.disk_bytes_per_token == int(1100e6)
    p2 = plan_tiers([head, _t("layer", 27, 18)], vram_budget_gb=0.4, scratch_bytes=int(50e6))
    assert p2.feasible and p2.vram_headroom_bytes == int(84e6) + int(50e6)
    assert TensorInfo("a", 100, 50, True).materialize_bytes == 100


def test_kv_cache_bytes_per_token():
    ns = types.SimpleNamespace
    assert kv_cache_bytes_per_token(ns(num_hidden_layers=40, num_attention_heads=40, num_key_value_heads=8,
                                       head_dim=128)) == 163840
    assert kv_cache_bytes_per_token(ns(num_hidden_layers=12, num_attention_heads=12, head_dim=64)) == 2 * 12 * 12 * 64 * 2
    assert kv_cache_bytes_per_token(ns(num_hidden_layers=12, num_attention_heads=12, num_key_value_heads=4,
                                       hidden_size=768)) == 2 * 12 * 4 * 64 * 2
    with pytest.raises(ValueError, match="num_hidden_layers"):
        kv_cache_bytes_per_token(ns(num_attention_heads=12))
    with pytest.raises(ValueError, match="head_dim"):
        kv_cache_bytes_per_token(ns(num_hidden_layers=12, num_attention_heads=12))


def test_describe_and_tier_of():
    plan = plan_tiers([_t("big", 4000, 3000)], vram_budget_gb=1.0)
    assert "Tier plan" in plan.describe() and "feasible             : False" in plan.describe()
    p = plan_tiers([_t("a", 100, 90)], vram_budget_gb=0.05, scratch_bytes=int(1e6))
    assert p.tier_of("a") == "disk" and p.tier_of("nonexistent") == "disk"
