"""Helpers shared by the GPU parity tests: build the CUDA store from a case,
read its reference-shaped views back, and compare with the oracle."""
from __future__ import annotations

import numpy as np
import torch

from logitfill_b200.packed import PackedKVManager

TORCH_DT = {"bfloat16": torch.bfloat16, "float32": torch.float32, "float16": torch.float16}
ATOL = 2e-3       # max-abs bound on attention outputs
MIN_COS = 0.9999  # cosine bound on attention outputs


def manager_for(case: dict, device="cuda", capacity=None) -> PackedKVManager:
    dt = TORCH_DT[case["dtype"]]
    mgr = PackedKVManager(levels=[torch.as_tensor(case["levels"], dtype=torch.int64)], n_q=case["n_q"],
                          n_kv=case["n_kv"], head_dim=case["head_dim"], page_size=case["page"],
                          k_group_size=case["k_group"], v_group_size=case["v_group"], bit_v=2, device=device,
                          **({} if capacity is None else {"capacity": capacity}))
    for k, v in case["commits"]:
        mgr.commit(0, torch.as_tensor(k)[None].to(device=device, dtype=dt),
                   torch.as_tensor(v)[None].to(device=device, dtype=dt))
    return mgr


def store_arrays(layer) -> dict:
    out = {}
    if layer.hist_k is not None:
        hk, hv = layer.hist_k, layer.hist_v
        for code in (0, 1, 2):
            for name in ("code", "scale", "min"):
                out[f"k{code}_{name}"] = hk[code][name].cpu().numpy()
        out["k3_value"] = hk[3]["value"].cpu().numpy()
        for name in ("code", "scale", "min"):
            out[f"v_{name}"] = hv[name].cpu().numpy()
    return out


def bit_equal(a, b) -> bool:
    a, b = np.ascontiguousarray(a), np.ascontiguousarray(b)
    return a.shape == b.shape and a.dtype == b.dtype and np.array_equal(a.view(np.uint8), b.view(np.uint8))


def attention_close(got: np.ndarray, want: np.ndarray, atol: float = ATOL, min_cos: float = MIN_COS):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    err = float(np.max(np.abs(got - want))) if got.size else 0.0
    cos = float(np.dot(got, want) / (np.linalg.norm(got) * np.linalg.norm(want) + 1e-30))
    return err <= atol and cos >= min_cos, err, cos
