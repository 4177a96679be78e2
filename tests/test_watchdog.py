"""Bounded-wait watchdog: every device wait gives up after a limit, records a
role code in the context's status word and lets the kernel return, so the
host gets SPKV2_ERR_DEVICE_STATUS instead of a hung GPU.  The probe makes a
wait run out on purpose (an mbarrier nothing completes); no fault, trap or
unbounded loop is involved, and the context keeps working afterwards."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import compile_pair, seeded_input

pytestmark = pytest.mark.gpu

SPKV2_ERR_DEVICE_STATUS = -47


def test_watchdog_probe_reports_and_context_stays_usable(gpu):
    from spinnv2_b200.runtime import Runtime

    spk = compile_pair("lenet5", 1, targets=("cuda_b200",))["cuda_b200"]
    x = seeded_input((1, 1, 28, 28), "uniform")
    with Runtime(spk, device=0) as rt:
        before = rt.run(x)[0]
        rc, code = rt.watchdog_probe(2000)  # 2 ms limit
        assert rc == SPKV2_ERR_DEVICE_STATUS
        assert code == 9 and rt.lib.spkv2_cuda_last_device_code(rt.ctx) == 9
        after = rt.run(x)[0]  # the status word was cleared; the context still runs
        np.testing.assert_array_equal(before, after)
        rc2, _ = rt.watchdog_probe(1000)
        assert rc2 == SPKV2_ERR_DEVICE_STATUS
        np.testing.assert_array_equal(rt.run(x)[0], before)


def test_watchdog_probe_rejects_bad_limits(gpu):
    from spinnv2_b200.runtime import Runtime

    spk = compile_pair("lenet5", 1, targets=("cuda_b200",))["cuda_b200"]
    with Runtime(spk, device=0) as rt:
        assert rt.watchdog_probe(0)[0] == -1
        assert rt.watchdog_probe(3_000_000)[0] == -1
