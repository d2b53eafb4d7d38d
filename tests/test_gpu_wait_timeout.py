"""Every device wait in the kernels is bounded: it gives up after a time
limit, records an error in the pass's status word and lets its CTA stop, so
a pass that cannot finish fails with an error instead of hanging the GPU.
Here one wait is made to run out on purpose, without a fault: the next
pass's first fused FFN launch waits for an activation band one count beyond
what its up tiles deliver, with a limit of about half a millisecond
(omg_engine_arm_wait_timeout). The call must raise the engine's
wait-timeout error, and the same engine must then evaluate the request with
the same bits as before."""
import dataclasses

import numpy as np
import pytest

from grande_b200 import synth
from grande_b200._lib import OmgError
from grande_b200.engine import Want

pytestmark = pytest.mark.gpu


def test_a_wait_that_runs_out_fails_the_pass_and_the_engine_recovers(device):
    shape = dataclasses.replace(synth.CONFIGS["e2b-q4"], layers=2, global_every=2)
    req = synth.request(shape, seed=5)
    eng = synth.build_engine(shape, shape.tokens() + 64, shape.branches, device=device)
    try:
        before = eng.evaluate(req.prefix, req.branches, Want.HIDDEN)
        eng.evict_resident()
        eng.arm_wait_timeout(1 << 20)
        with pytest.raises(OmgError, match="gave up waiting"):
            eng.evaluate(req.prefix, req.branches, Want.HIDDEN)
        eng.evict_resident()
        after = eng.evaluate(req.prefix, req.branches, Want.HIDDEN)
        for a, b in zip(before, after):
            assert np.array_equal(a.rows, b.rows)
        with pytest.raises(OmgError, match="positive"):
            eng.arm_wait_timeout(0)
    finally:
        eng.close()
