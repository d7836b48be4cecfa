"""Failure detection without a GPU fault: every device-side wait in this
library is bounded; when the budget runs out the kernel records a code in the
context's status word and returns, and the host reports ITTS_ETIMEOUT. The
self-test makes one such wait run out on purpose (a barrier nothing completes)
and checks that the status arrives and that the context keeps working."""
from __future__ import annotations

import numpy as np
import pytest

import itts_cfm
import workloads as W

pytestmark = pytest.mark.gpu


def test_bounded_wait_expires_and_context_survives(ctx_unit, rng):
    rc, msg = ctx_unit.selftest_timeout(2_000_000)  # about 1 ms at 1.9 GHz
    assert rc == itts_cfm.ITTS_ETIMEOUT, (rc, msg)
    assert "bounded wait" in msg and "6" in msg, msg
    # The status word was cleared on the way out: normal work runs and matches
    # a run from before the self-test bit for bit.
    u = W.utterance(rng, 24, 4)
    a = ctx_unit.run(u.noise, u.prompt, u.cond, u.style, 2, 0.7)
    rc2, _ = ctx_unit.selftest_timeout(1_000_000)
    assert rc2 == itts_cfm.ITTS_ETIMEOUT
    b = ctx_unit.run(u.noise, u.prompt, u.cond, u.style, 2, 0.7)
    assert np.isfinite(a).all() and np.array_equal(a, b)


def test_selftest_rejects_bad_budget(ctx_unit):
    rc, msg = ctx_unit.selftest_timeout(10)
    assert rc == itts_cfm.ITTS_EINVAL_SHAPE and "budget" in msg
