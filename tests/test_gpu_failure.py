"""Failure detection on the GPU without a fault: the bounded mbarrier wait
that every pipelined kernel here uses runs out on a barrier nothing arrives
on (paro_selftest_wait_timeout: one thread, no copy in flight), sets bit 1
of the device error word, and the kernel returns.  The host reads the word,
the operator workspaces are reset, and the context stays usable: the next
linear gives the same bits as before."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_timed_out_wait_reports_and_context_survives():
    import alpamayo_b200.ops as ops
    from alpamayo_b200 import _native
    from alpamayo_b200 import synthetic as syn
    L = _native.capi()
    layer = syn.make_layer(512, 1024, seed=3, checkpoint=False)
    x = syn.make_activations(4, 1024, seed=4)
    run = lambda: ops.linear_w4a8(x, layer["rot_table"], layer["cs_vec"], layer["packed"], 512, None, True,  # noqa: E731
                                  torch.float32)
    before = run()
    assert ops.device_error_word() == 0
    st = L.paro_selftest_wait_timeout(2_000_000, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, L.paro_status_string(st)
    torch.cuda.synchronize()
    assert ops.device_error_word() & 1            # the wait ran out and said so
    assert ops.device_error_word() == 0           # the read cleared it
    after = run()
    torch.cuda.synchronize()
    assert torch.equal(before, after)             # the context and the workspaces are intact
    assert ops.device_error_word() == 0
