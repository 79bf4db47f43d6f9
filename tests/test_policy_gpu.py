"""A policy directory written by the reference's own policy code
(``tests/golden/policy_ref``, made by ``tests/golden/make_policy_fixture.py``
with ``build_policy(...).save(...)`` of ``src/logitfill/allocators/policy.py``)
loaded through ``DeepSeekQwenKVAdapter.load_policy`` and decoded through.

The adapter installs the policy's per-layer Key tier maps; their device tier
tables are built once and shared by the packed store (the store's layout
holds the very same tables object).  A tiny Qwen2 of the policy's shape
decodes teacher-forced tokens across page boundaries; every decode call is
checked against the oracle on the same inputs and every layer's packed
history must equal the oracle's bit for bit.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from logitfill_b200.adapter import DeepSeekQwenKVAdapter
from logitfill_b200.policy import TierTables, policy_tables
from oracle import packed_ref as orc
from tests.gpu_cases import ATOL, MIN_COS, bit_equal, store_arrays
from tests.oracle_runner import layer_arrays
from tests.qwen_cases import CheckedManager, OracleManager, adapter_logits, tiny_qwen2

pytestmark = pytest.mark.gpu
POLICY = Path(__file__).resolve().parent / "golden" / "policy_ref"


def test_decode_through_reference_written_policy():
    layers, n_q, n_kv, D, page = 2, 4, 2, 128, 128
    model = tiny_qwen2(n_q=n_q, n_kv=n_kv, head_dim=D, layers=layers, vocab=256, seed=7, device="cuda",
                       dtype=torch.float32, attn="sdpa")
    a = DeepSeekQwenKVAdapter(model).attach()
    policy = a.load_policy(POLICY)
    assert policy.levels.shape == (layers, n_kv, D) and policy.metadata["target_bit"] == 2.5
    tables = policy_tables(policy, "cuda")
    real = a.packed_manager()
    for i in range(layers):
        lay = real.cache.layers[i].layout
        assert lay.tables is tables[i] is TierTables.get(policy.levels[i], "cuda")  # built once, shared
        ref = orc.tier_tables(policy.levels[i])
        for t in range(4):
            for key in ("index", "count", "local"):
                assert np.array_equal(lay.table[t][key].cpu().numpy(), ref[t][key]), (i, t, key)
    levels = [policy.levels[i] for i in range(layers)]
    checked = CheckedManager(real, OracleManager(levels, n_q, n_kv, D, page, page, D))
    a._packed = checked
    ids = torch.randint(0, 256, (1, 300), generator=torch.Generator().manual_seed(7)).cuda()
    adapter_logits(model, a, ids, 140)
    real.cache.check_status()
    err, cos = checked.worst
    assert err <= ATOL and cos >= MIN_COS, (err, cos)
    for i in range(layers):
        got, want = store_arrays(real.layers[i]), layer_arrays(checked.oracle.layers[i].layer)
        for key in want:
            assert bit_equal(got[key], want[key]), (i, key)
