"""Generates tests/golden/planner_cases.json by running the REFERENCE
residency planner (afterimage/runtime/vram_planner.py) on seeded random
scenarios: tensor lists with mixed compressibility, row-gather and
stream-only tensors, draft layers, forced-RAM overlays, budgets that are
feasible and infeasible, every placement policy.

Usage: python tests/golden/make_planner_golden.py <path to an Afterimage checkout>
       (or set AFTERIMAGE_REF)

The reference planner runs with its own decode-scratch constant
(10 bytes/element); the product test sets the same constant so the plans
must match field for field.
"""
from __future__ import annotations

import json
import os
import pathlib
import random
import sys
import types

sys.dont_write_bytecode = True
_ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AFTERIMAGE_REF")
if not _ref:
    raise SystemExit("usage: make_planner_golden.py <path to an Afterimage checkout> (or set AFTERIMAGE_REF)")
sys.path.insert(0, str(pathlib.Path(_ref)))

from afterimage.runtime import vram_planner as vp  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent / "planner_cases.json"


def plan_dict(p) -> dict:
    return {k: getattr(p, k) for k in ("vram_budget_bytes", "ram_budget_bytes", "vram_headroom_bytes",
                                         "vram_keys", "ram_keys", "disk_keys", "row_gather_keys",
                                         "vram_bytes", "ram_bytes", "disk_bytes_per_token", "feasible",
                                         "reason")}


def main():
    rng = random.Random(20261201)
    cases = []
    for i in range(120):
        n = rng.randint(1, 30)
        tensors = []
        for j in range(n):
            orig = rng.choice([rng.randint(1, 400), rng.randint(400, 3000)]) * 10 ** 6
            comp = int(orig * rng.uniform(0.3, 1.05))
            key = rng.choice([f"model.layers.{rng.randint(0, 40)}.mlp.p{j}.weight", f"t{j}",
                              f"lm_head{j}.weight"])
            tensors.append({"key": key + f"#{j}", "orig_bytes": orig, "comp_bytes": comp,
                            "is_layer_weight": key.startswith("model.layers."),
                            "row_gather": rng.random() < 0.08, "uses": rng.choice([1, 1, 1, 3, 9]),
                            "stream_only": rng.random() < 0.08,
                            "materialize_override": rng.choice([None, rng.randint(1, 200) * 10 ** 6]),
                            "profiled_value_s": rng.random(), "critical_value_s": rng.random(),
                            "profiled_observed": rng.random() < 0.5, "critical_observed": rng.random() < 0.5})
        kw = {"vram_budget_gb": rng.choice([0.2, 0.5, 1.0, 2.0, 4.0, 8.0, 30.0]),
              "ram_budget_gb": rng.choice([0.0, 0.5, 2.0, 10.0])}
        mode = rng.choice(["scratch", "slice", "default", "headroom"])
        if mode == "scratch":
            kw["scratch_bytes"] = rng.randint(1, 600) * 10 ** 6
        elif mode == "slice":
            kw["decode_slice_elems"] = rng.choice([100, 1 << 20, 1 << 22, 1 << 25])
            kw["activation_slack_bytes"] = rng.choice([0, 20 * 10 ** 6, 128 * 1024 * 1024])
        elif mode == "headroom":
            kw["vram_headroom_bytes"] = rng.randint(0, 2000) * 10 ** 6
        kw["pin_layer_weights"] = rng.random() < 0.2
        kw["placement_policy"] = rng.choice(["traffic_density", "profiled_knapsack", "critical_path"])
        eligible = [t for t in tensors if not t["row_gather"] and not t["stream_only"]]
        if eligible and rng.random() < 0.2:
            kw["forced_ram_keys"] = [rng.choice(eligible)["key"]]
        infos = [vp.TensorInfo(**t) for t in tensors]
        call = dict(kw)
        if "forced_ram_keys" in call:
            call["forced_ram_keys"] = set(call["forced_ram_keys"])
        try:
            out = plan_dict(vp.plan_tiers(infos, **call))
            err = None
        except ValueError as e:
            out, err = None, str(e)
        cases.append({"kind": "plan_tiers", "tensors": tensors, "kwargs": kw, "plan": out, "error": err})

    for i in range(40):
        n = rng.randint(1, 25)
        manifest = {"tensors": {}}
        for j in range(n):
            key = rng.choice([f"model.layers.{rng.randint(0, 30)}.self_attn.q{j}.weight", f"lm_head.w{j}",
                              f"model.embed_tokens.w{j}"])
            orig = rng.randint(1, 2000) * 10 ** 6
            meta = {"orig_bytes": orig, "comp_bytes": int(orig * rng.uniform(0.4, 1.0))}
            if rng.random() < 0.1:
                meta["row_gather"] = True
            manifest["tensors"][key] = meta
        keys = list(manifest["tensors"])
        kw = {"vram_budget_gb": rng.choice([0.5, 1.0, 3.0, 8.0]), "ram_budget_gb": rng.choice([0.0, 1.0, 5.0]),
              "scratch_bytes": rng.randint(1, 500) * 10 ** 6}
        if rng.random() < 0.5:
            kw["draft_layer_indices"] = sorted(rng.sample(range(31), 3))
            kw["draft_uses"] = rng.choice([3, 9])
        if rng.random() < 0.3:
            k = rng.choice(keys)
            if not manifest["tensors"][k].get("row_gather"):
                kw["stream_only"] = {k: rng.randint(1, 100) * 10 ** 6}
        profile = None
        if rng.random() < 0.4:
            kw["placement_policy"] = rng.choice(["profiled_knapsack", "critical_path"])
            profile = {k: {"read_s": rng.random(), "decode_s": rng.random(), "transfer_s": rng.random(),
                           "counterfactual_s": rng.choice([0.0, rng.random()])}
                       for k in rng.sample(keys, max(1, len(keys) // 2))}
        call = dict(kw)
        if profile is not None:
            call["critical_path_profile"] = types.SimpleNamespace(
                tensors={k: types.SimpleNamespace(**v) for k, v in profile.items()})
        out = plan_dict(vp.plan_from_manifest(manifest, **call))
        cases.append({"kind": "plan_from_manifest", "manifest": manifest, "kwargs": kw, "profile": profile,
                      "plan": out, "error": None})

    OUT.write_text(json.dumps({"generator": "tests/golden/make_planner_golden.py",
                               "decode_scratch_bytes_per_elem": vp.DECODE_SCRATCH_BYTES_PER_ELEM,
                               "cases": cases}) + "\n")
    print("wrote", len(cases), "planner cases,", OUT.stat().st_size // 1024, "KB")


if __name__ == "__main__":
    main()
