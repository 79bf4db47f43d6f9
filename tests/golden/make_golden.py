"""Generate the golden fixtures by running the REFERENCE implementation.

Run from the repository root, in a checkout where the GASSFY/Logitfill sources
are importable (``--reference-src``, default ``$LOGITFILL_REFERENCE_SRC``):

    python tests/golden/make_golden.py --reference-src <logitfill>/src

It imports ``logitfill.packed`` (``layout.py``, ``cache.py``, ``reference.py``)
read-only and runs, on CPU:

* the reference's own unit-test inputs (``tests/test_logitfill_offline.py``
  127-145 and 187-219), regenerated with the same torch seeds;
* a small mixed-tier GQA case;
* BASELINE config 0 and ragged variants of it (``cases.py``);
* a packer corner-case page (``cases.pack_edge_page``).

For each it stores the packed history exactly as the reference stores it
(codes, scale/min bytes, FP16 tier, Value codes/scale/min), the dequantized
round trip, and ``reference_attention`` evaluated with an fp32 query (so the
reference returns fp32).  Small cases are stored whole; config-0 cases store
SHA-256 digests of the large arrays plus the full attention output.

Nothing at test time imports the reference: the fixtures written here are
what ``tests/test_oracle_golden.py`` pins the oracle against.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE))

import cases  # noqa: E402


def _np(t):
    import torch

    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.detach().cpu().numpy()


def _manager_arrays(layer) -> dict:
    out = {}
    if layer.hist_k is not None:
        for code in (0, 1, 2):
            for name in ("code", "scale", "min"):
                out[f"k{code}_{name}"] = _np(layer.hist_k[code][name])
        out["k3_value"] = _np(layer.hist_k[3]["value"])
        for name in ("code", "scale", "min"):
            out[f"v_{name}"] = _np(layer.hist_v[name])
    return out


def run_case(ref, torch, case: dict) -> dict:
    from logitfill.packed.cache import PackedKVManager
    from logitfill.packed.reference import reference_attention

    dt = {"bfloat16": torch.bfloat16, "float32": torch.float32}[case["dtype"]]
    manager = PackedKVManager(
        levels=[torch.as_tensor(case["levels"], dtype=torch.int64)], n_q=case["n_q"], n_kv=case["n_kv"],
        head_dim=case["head_dim"], page_size=case["page"], k_group_size=case["k_group"],
        v_group_size=case["v_group"], bit_v=2, device="cpu")
    for k, v in case["commits"]:
        manager.commit(0, torch.as_tensor(k)[None].to(dt), torch.as_tensor(v)[None].to(dt))
    layer = manager.layers[0]
    out = _manager_arrays(layer)
    kd, vd = layer.dequantize()
    out["deq_k"], out["deq_v"] = _np(kd), _np(vd)
    out["hist_len"] = np.array(layer.hist_len)
    out["tail_len"] = np.array(layer.tail_len)
    q = torch.as_tensor(case["query"])[None].float()
    kn = torch.as_tensor(case["key_new"])[None].to(dt)
    vn = torch.as_tensor(case["value_new"])[None].to(dt)
    out["attn"] = _np(reference_attention(manager, 0, q, kn, vn, case["scaling"]))[0]
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("LOGITFILL_REFERENCE_SRC"))
    args = ap.parse_args()
    if not args.reference_src:
        raise SystemExit("pass --reference-src <GASSFY/Logitfill>/src")
    sys.path.insert(0, args.reference_src)
    import torch
    import logitfill.packed.layout as ref

    small = {}
    # tests/test_logitfill_offline.py:127-145 -- layout round trip, all INT2, group 8.
    torch.manual_seed(0)
    page = torch.randn(2, 16, 8)
    levels = torch.zeros(2, 8, dtype=torch.int64)
    built = ref.tier_tables(levels)
    table = built["tiers"]
    table["tier"] = built["tier"]
    pk = ref.quantize_key_page(page, table, group_size=8)
    pv = ref.quantize_value_page(page, bits=2, group_size=8)
    small["layout_page"] = page.numpy()
    for name in ("code", "scale", "min"):
        small[f"layout_k0_{name}"] = _np(pk[0][name])
        small[f"layout_v_{name}"] = _np(pv[name])
    small["layout_deq_k"] = _np(ref.dequantize_key(16, table, pk, group_size=8))
    small["layout_deq_v"] = _np(ref.dequantize_value(pv, 16, 8, bits=2, group_size=8))

    # tests/test_logitfill_offline.py:187-219 -- kernel-vs-dense shape (CPU generator).
    torch.manual_seed(0)
    lv = torch.randint(0, 4, (1, 64))
    key, value = torch.randn(1, 1, 64, 64), torch.randn(1, 1, 64, 64)
    query, nk, nv = torch.randn(1, 1, 1, 64), torch.randn(1, 1, 1, 64), torch.randn(1, 1, 1, 64)
    cuda_case = {"dtype": "float32", "n_q": 1, "n_kv": 1, "head_dim": 64, "page": 64, "k_group": 64,
                 "v_group": 64, "levels": lv.numpy(), "commits": [(key[0].numpy(), value[0].numpy())],
                 "query": query[0].numpy(), "key_new": nk[0].numpy(), "value_new": nv[0].numpy(),
                 "scaling": 64 ** -0.5}

    # Mixed tiers, GQA 2, D 64, two pages plus a 10-token tail, fp32 inputs, 3 commits.
    rng = np.random.default_rng(11)
    mk = rng.standard_normal((3, 138, 64), dtype=np.float32)
    mv = rng.standard_normal((3, 138, 64), dtype=np.float32)
    mk[:, :, 5] *= 10.0
    mixed_case = {"dtype": "float32", "n_q": 6, "n_kv": 3, "head_dim": 64, "page": 64, "k_group": 64,
                  "v_group": 64, "levels": rng.integers(0, 4, size=(3, 64)),
                  "commits": [(mk[:, :50], mv[:, :50]), (mk[:, 50:100], mv[:, 50:100]), (mk[:, 100:], mv[:, 100:])],
                  "query": rng.standard_normal((6, 1, 64), dtype=np.float32),
                  "key_new": rng.standard_normal((3, 1, 64), dtype=np.float32),
                  "value_new": rng.standard_normal((3, 1, 64), dtype=np.float32), "scaling": 0.125}

    for name, case in (("cuda", cuda_case), ("mixed", mixed_case)):
        res = run_case(ref, torch, case)
        for key_, arr in res.items():
            small[f"{name}_{key_}"] = arr
        small[f"{name}_levels"] = np.asarray(case["levels"])
        small[f"{name}_query"] = case["query"]
        small[f"{name}_key_new"] = case["key_new"]
        small[f"{name}_value_new"] = case["value_new"]
        for i, (k, v) in enumerate(case["commits"]):
            small[f"{name}_commit{i}_k"] = k
            small[f"{name}_commit{i}_v"] = v

    # Packer corner cases (inputs rebuilt from cases.pack_edge_page).
    edge = cases.pack_edge_page()
    built = ref.tier_tables(torch.as_tensor(edge["levels"], dtype=torch.int64))
    table = built["tiers"]
    table["tier"] = built["tier"]
    kt = torch.as_tensor(edge["k"]).to(torch.bfloat16)
    vt = torch.as_tensor(edge["v"]).to(torch.bfloat16)
    pk = ref.quantize_key_page(kt, table, 128)
    pv = ref.quantize_value_page(vt, 2, 128)
    small["edge_input_sha"] = np.array([cases.sha(edge["k"]), cases.sha(edge["v"])])
    for code in (0, 1, 2):
        for name in ("code", "scale", "min"):
            small[f"edge_k{code}_{name}"] = _np(pk[code][name])
    small["edge_k3_value"] = _np(pk[3]["value"])
    for name in ("code", "scale", "min"):
        small[f"edge_v_{name}"] = _np(pv[name])
    np.savez_compressed(HERE / "golden_small.npz", **small)

    big = {}
    for name, (hist, tail) in cases.CONFIG0_VARIANTS.items():
        case = cases.config0_like(hist, tail)
        big[f"{name}_input_sha"] = np.array([cases.sha(case["levels"]), cases.sha(case["query"])]
                                            + [cases.sha(k) for k, _ in case["commits"]]
                                            + [cases.sha(v) for _, v in case["commits"]])
        res = run_case(ref, torch, case)
        for key_, arr in res.items():
            if key_ in ("attn", "hist_len", "tail_len"):
                big[f"{name}_{key_}"] = arr
            else:
                big[f"{name}_{key_}_sha"] = np.array(cases.sha(arr))
    np.savez_compressed(HERE / "golden_config0.npz", **big)
    print("wrote", HERE / "golden_small.npz", HERE / "golden_config0.npz")


if __name__ == "__main__":
    main()
