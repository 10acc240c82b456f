"""Failure detection without a GPU fault: a device-side bounded wait that
cannot complete must give up, be reported by spock_sync as SPOCK_ERR_TIMEOUT,
and leave the context usable for the next call."""
import numpy as np
import pytest
import torch

import oracle
import spock_b200
from tests.golden.gen import chunk_inputs
from tests.util import max_rel

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_recovers(cuda_ok):
    ctx = spock_b200.Context.get(0)
    ctx.selftest_wait_timeout(polls=64)
    with pytest.raises(spock_b200.SpockError) as e:
        ctx.sync()
    assert e.value.code == spock_b200.SPOCK_ERR_TIMEOUT
    ctx.sync()  # the error word was cleared
    # the context and the device still work
    q, k, v, g, b = chunk_inputs(2, 70, seed=4, batch=1)
    dev = torch.device("cuda", 0)
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    out, st = spock_b200.chunk_prefill(T(q), T(k), T(v), T(g), T(b))
    ctx.sync()
    ro, rs = oracle.chunk_rule(q[0], k[0], v[0], g[0], b[0])
    assert max_rel(out.cpu().numpy()[0], ro) <= 1e-3 and max_rel(st.cpu().numpy()[0], rs) <= 1e-3


def test_model_session_reports_timeouts_on_its_context(cuda_ok):
    """A model session created on a context shares the context's error word:
    a bounded wait that gives up is reported by spock_model_sync (and would be
    by spock_sync), then cleared."""
    ctx = spock_b200.Context.get(0)
    m = spock_b200.Model(num_layers=4, vocab=1024, max_batch=1, max_seq=16, ctx=ctx)
    try:
        ctx.selftest_wait_timeout(polls=64)
        with pytest.raises(spock_b200.SpockError) as e:
            m.sync()
        assert e.value.code == spock_b200.SPOCK_ERR_TIMEOUT
        m.sync()
        ctx.sync()
    finally:
        m.close()
