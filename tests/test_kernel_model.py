"""CPU check of the tensor-core kernel's fixed-point scheme (tests/kernel_model.py).

The decode kernel multiplies integer codes by 31-bit (QK, four limbs) and
23-bit (PV, three limbs) fixed point on the INT8 tensor cores.  The numpy
model of that arithmetic must stay inside the decode tolerance against the
oracle with a wide margin (observed ~2e-5 max-abs), also for sharp attention
(large scores), and narrower fixed point must not."""
from __future__ import annotations

import numpy as np
import pytest

from logitfill_b200.synthetic import synthetic_kv, synthetic_levels
from oracle import packed_ref as orc
from tests.gpu_cases import attention_close
from tests.kernel_model import model_attention


def _case(target_bit: float, T: int, seed: int = 1):
    levels = synthetic_levels(1, 4, 128, target_bit, seed=seed)[0]
    k, v = synthetic_kv(1, 4, T + 40, 128, seed=seed, layer=0)
    k, v = k[0].float().numpy(), v[0].float().numpy()
    store = orc.OracleLayer(levels, 128, 128, 128, 2)
    store.append(k[:, :T + 37], v[:, :T + 37])
    q = orc.bf16_to_f32(orc.f32_to_bf16_bits(np.random.default_rng(seed).standard_normal((28, 1, 128))))
    want = orc.reference_attention(store, q, k[:, T + 37:T + 38], v[:, T + 37:T + 38], 128 ** -0.5)[:, 0]
    return store, q[:, 0], k[:, T + 37:T + 38], v[:, T + 37:T + 38], want


@pytest.mark.parametrize("target_bit", [2.5, 4.0])
def test_kernel_fixed_point_within_tolerance(target_bit):
    store, q, kn, vn, want = _case(target_bit, 2048)
    got = model_attention(store, q, kn, vn, 128 ** -0.5)
    ok, err, cos = attention_close(got, want, atol=5e-4)  # 4x tighter than the decode bound
    assert ok, (err, cos)


@pytest.mark.parametrize("q_scale", [1.0, 3.0, 6.0])
def test_sharp_attention_within_tolerance(q_scale):
    """Scaled queries make the softmax sharp and the scores large; the QK
    rounding error grows with the score magnitude.  21-bit QK fixed point
    (three limbs) leaves the 2e-3 bound at the largest scale; 29 bits keep a
    20x margin."""
    store, q, kn, vn, _ = _case(2.5, 1024)
    q = q * q_scale
    want = orc.reference_attention(store, q[:, None], kn, vn, 128 ** -0.5)[:, 0]
    ok, err, cos = attention_close(model_attention(store, q, kn, vn, 128 ** -0.5), want, atol=1e-4)
    assert ok, (err, cos)
    if q_scale == 6.0:
        assert not attention_close(model_attention(store, q, kn, vn, 128 ** -0.5, qk_bits=21), want)[0]


def test_narrow_fixed_point_would_fail():
    store, q, kn, vn, want = _case(3.0, 2048)
    ok_qk, _, _ = attention_close(model_attention(store, q, kn, vn, 128 ** -0.5, qk_bits=14), want)
    err_pv = attention_close(model_attention(store, q, kn, vn, 128 ** -0.5, pv_bits=16), want)[1]
    assert not ok_qk
    assert err_pv > 5e-5
