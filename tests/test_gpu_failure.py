"""Failure detection without a GPU fault: the expert-parallel exchange kernel, run against a stand-in peer (a second
region of this GPU's own memory) that never takes part, gives up after its bounded wait and the call returns
KTMOE_ERR_KERNEL, as a forward whose peer rank stopped does; the context keeps working afterwards."""

import time

import numpy as np
import pytest

from tritify_b200 import _native

pytestmark = pytest.mark.gpu


def test_a_silent_peer_ends_the_wait_with_an_error(ctx):
    t0 = time.monotonic()
    status = ctx.check_wait_expiry()
    waited = time.monotonic() - t0
    assert status == _native.ERR_KERNEL
    assert 1.5 < waited < 60  # the wait's limit is 2 s of the GPU's global timer
    assert b"bounded wait" in _native.lib().ktmoe_last_error(ctx.handle)
    # the error word was cleared and the context still computes
    assert list(ctx.linear(np.array([1, 2], np.int32), np.array([3, 4], np.int32), 1, 1, 2)) == [11]
    assert ctx.check_wait_expiry() == _native.ERR_KERNEL  # and detects it again
