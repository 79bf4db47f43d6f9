"""Run the golden cases through the numpy oracle (test helper)."""
from __future__ import annotations

import numpy as np

from oracle import packed_ref as orc


def oracle_layer_for(case: dict) -> orc.OracleLayer:
    layer = orc.OracleLayer(case["levels"], case["page"], case["k_group"], case["v_group"], 2)
    for k, v in case["commits"]:
        layer.append(np.asarray(k, np.float32), np.asarray(v, np.float32))
    return layer


def layer_arrays(layer: orc.OracleLayer) -> dict:
    out = {}
    if layer.hist_k is not None:
        for code in (0, 1, 2):
            for name in ("code", "scale", "min"):
                out[f"k{code}_{name}"] = layer.hist_k[code][name]
        out["k3_value"] = layer.hist_k[3]["value"]
        for name in ("code", "scale", "min"):
            out[f"v_{name}"] = layer.hist_v[name]
    return out


def run_case(case: dict) -> dict:
    layer = oracle_layer_for(case)
    out = layer_arrays(layer)
    out["deq_k"], out["deq_v"] = layer.dequantize()
    out["hist_len"] = np.array(layer.hist_len)
    out["tail_len"] = np.array(layer.tail_len)
    out["attn"] = orc.reference_attention(layer, case["query"], case["key_new"], case["value_new"], case["scaling"])
    return out


def small_case(golden: dict, name: str, dtype: str = "float32") -> dict:
    commits = []
    i = 0
    while f"{name}_commit{i}_k" in golden:
        commits.append((golden[f"{name}_commit{i}_k"], golden[f"{name}_commit{i}_v"]))
        i += 1
    levels = golden[f"{name}_levels"]
    n_kv, d = levels.shape
    q = golden[f"{name}_query"]
    page = 64
    return {"dtype": dtype, "n_q": q.shape[0], "n_kv": n_kv, "head_dim": d, "page": page, "k_group": page,
            "v_group": d, "levels": levels, "commits": commits, "query": q,
            "key_new": golden[f"{name}_key_new"], "value_new": golden[f"{name}_value_new"],
            "scaling": {"cuda": 64 ** -0.5, "mixed": 0.125}[name]}
