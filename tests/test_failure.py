"""Failure detection without a GPU fault: the bounded device wait that every kernel uses gives up,
records the timeout and returns; the host reads CWX_ETIMEOUT and the context keeps working. Bad
arguments come back as CWX_EINVAL before any device work."""

import numpy as np
import pytest

from coachwhip_b200 import CwxError, _lib

torch = pytest.importorskip("torch")


@pytest.mark.gpu
def test_bounded_wait_times_out_and_context_stays_usable():
    from coachwhip_b200.moe import route

    ctx = _lib.ctx(0)
    st = torch.cuda.current_stream().cuda_stream
    _lib.status(0)
    _lib.check(_lib.lib().cwx_ctx_check_wait(ctx, 2000, st))  # a 2 ms wait that nothing ends
    with pytest.raises(CwxError) as e:
        _lib.status(0)
    assert e.value.code == _lib.ETIMEOUT
    assert "gave up" in str(e.value)
    # the status was cleared and the context still computes
    logits = torch.tensor([[0.1, 3.0, 2.0, -1.0, 1.0]], device="cuda")
    ids, w = route(logits, 3, True)
    _lib.status(0)
    assert ids.cpu().tolist() == [[1, 2, 4]]


def test_check_wait_rejects_bad_limits_before_device_work():
    # argument checks come first: no device call is made, so this runs without a GPU
    assert _lib.lib().cwx_ctx_check_wait(None, 10, None) == _lib.EINVAL
