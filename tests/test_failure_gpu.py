"""Failure detection on the GPU without a GPU fault.

Every mbarrier wait of the decode kernels is bounded; on expiry the kernel
records LF_ERR_DEVICE_TIMEOUT in a device status word, stops waiting and
returns, so the context stays usable.  lf_selftest_wait runs that same wait on
a barrier nothing arrives on (a flag that is never set): the test checks that
it gives up after its limit, reports the timeout through the status word, and
that decode attention still runs and matches the oracle afterwards.  The
host side of the report (PackedKVCache.check_status) raises on it.
"""
from __future__ import annotations

import time

import pytest
import torch

from logitfill_b200 import _lib
from tests.golden import cases
from tests.gpu_cases import attention_close, manager_for
from tests.oracle_runner import run_case

pytestmark = pytest.mark.gpu


def _selftest(limit_ns: int, arrive: bool) -> tuple[int, float]:
    status = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.check(_lib.lib().lf_selftest_wait(_lib.ptr(status), limit_ns, int(arrive), _lib.stream_handle(status.device)),
               "lf_selftest_wait")
    torch.cuda.synchronize()
    return int(status.item()), time.perf_counter() - t0


def test_completed_phase_passes():
    status, _ = _selftest(50_000_000, arrive=True)
    assert status == _lib.LF_OK


def test_wait_expires_reports_timeout_and_context_survives():
    limit = 20_000_000  # 20 ms
    status, elapsed = _selftest(limit, arrive=False)
    assert status == _lib.LF_ERR_DEVICE_TIMEOUT
    assert elapsed >= limit * 1e-9
    assert elapsed < 5.0
    # The context is still usable: a decode call runs and matches the oracle.
    case = cases.config0_like(256, 5)
    want = run_case(case)["attn"]
    mgr = manager_for(case)
    q = torch.as_tensor(case["query"])[None].to("cuda", torch.float32)
    kn = torch.as_tensor(case["key_new"])[None].to("cuda", torch.bfloat16)
    vn = torch.as_tensor(case["value_new"])[None].to("cuda", torch.bfloat16)
    from logitfill_b200.packed.attention import packed_attention
    out = packed_attention(mgr, 0, q, kn, vn, case["scaling"])
    ok, err, cos = attention_close(out[0].cpu().numpy(), want)
    assert ok, (err, cos)


def test_cache_status_word_raises_on_device_timeout():
    case = cases.config0_like(256, 5)
    mgr = manager_for(case)
    mgr.cache.check_status()  # clean
    mgr.cache.status.fill_(_lib.LF_ERR_DEVICE_TIMEOUT)
    with pytest.raises(RuntimeError, match="timed out"):
        mgr.cache.check_status()
