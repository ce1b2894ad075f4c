"""Failure detection without a GPU fault.  Every device-side wait of the
library is bounded; when one runs out the kernel records an error code,
stops and returns, the call reports GTMOE_ETIMEOUT, and the CUDA context
stays usable.  gtmoe_bounded_wait_selftest runs that bounded wait on an
mbarrier nothing completes (no fault, no hang: the wait gives up after about
two seconds); a forward afterwards must still match the oracle."""
import time

import pytest

from gotransformers_b200 import _lib
from gpu_helpers import TOL, gpu_moe, rel_l2
from moe_cases import make_case
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_reports_and_the_context_survives():
    L = _lib.lib()
    t0 = time.perf_counter()
    rc = L.gtmoe_bounded_wait_selftest(0)
    dt = time.perf_counter() - t0
    msg = L.gtmoe_last_error().decode()
    assert rc == -6, (rc, msg)  # GTMOE_ETIMEOUT
    assert "gave up" in msg
    assert dt >= 1.5  # the wait ran to its limit
    spec, x, ids = make_case(T=64, d=128, h=128, n_shared=1, n_routed=8, k=2, precision=O.INT8, seed=71)
    m = gpu_moe(spec)
    out = m.forward(x, ids)
    ref = O.moe_forward(spec, x, ids, threads=4)
    assert rel_l2(out, ref["out"]) <= TOL[O.INT8]
    m.close()
