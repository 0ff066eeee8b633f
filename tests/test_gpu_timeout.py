"""The attention kernel's bounded pipeline waits, made to run out.

b2_debug_withhold_q makes the tcgen05 attention kernel skip its Q load, so
the MMA issuer's wait for Q (and, behind it, the softmax warps' waits for S
and the producers' waits for free ring slots) can never complete.  Each wait
gives up after its time budget (about 2^31 cycles, ~1 s): the CTA records
(1 << 8 | site) in the device status word, waits for the loads it issued,
frees TMEM and returns.  The test checks that status, that the Python
wrapper raises, and that the context still computes correct results after.
Only one small CTA pair is launched, and nothing is left in flight when the
kernel returns: no GPU fault or hang is involved.
"""
import pytest
import torch

import pisa_oracle as oracle
from gpu_util import DEV

pytestmark = pytest.mark.gpu


def test_pipeline_wait_timeout_is_reported_and_recovered():
    import b200_pisa
    from b200_pisa import _lib

    q, k, v = oracle.generic_inputs(1, 128, 77)
    qd, kd, vd = (x.to(DEV) for x in (q, k, v))
    _lib.read_status()  # clear
    _lib.check(_lib.LIB.b2_debug_withhold_q(1))
    try:
        b200_pisa.forward(qd, kd, vd, exact_blocks=1)
        torch.cuda.synchronize()
    finally:
        _lib.check(_lib.LIB.b2_debug_withhold_q(0))
    assert _lib.last_kernel() == "tcgen05"
    with pytest.raises(_lib.PipelineTimeout) as info:
        _lib.check_status()
    assert info.value.status >> 8 == 1
    # the first wait to run out: Q (3), S for the softmax (8), a K/V ring slot (1, 13)
    assert info.value.site in (1, 3, 8, 13), hex(info.value.status)
    # the context is intact: the next call is correct and reports no timeout
    got = b200_pisa.forward(qd, kd, vd, exact_blocks=1).cpu().float()
    _lib.check_status()
    exp, _ = oracle.hyd_forward(q, k, v, 1)
    torch.testing.assert_close(got, exp.float(), atol=5e-2, rtol=5e-2)
