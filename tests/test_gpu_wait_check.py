"""The device-side failure path, run on purpose without faulting or hanging the GPU.

st_check_device_wait runs one warp that waits, with the helpers the GEMM
kernels use for their bounded waits, on an mbarrier nothing arrives on
(kind 0) or a flag nothing sets (kind 1).  After its limit the kernel
records its abort code in the device's error word and returns.  The host
must report ST_ERR_DEVICE_ABORT (Python: DeviceAbort) at the next bounded
wait, clear the word, and keep the context usable.
"""
import ctypes

import pytest
import torch

import sptiles_b200 as st
from sptiles_b200 import _native as N

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
CODES = {0: 0x1F0, 1: 0x1F1}


def check_wait(kind, limit_us, flags):
    ex = N.StExec(None, 0, flags, 10000, None, 0)
    return N.lib().st_check_device_wait(st.context(0), kind, limit_us, ctypes.byref(ex))


def add_still_works():
    a = torch.arange(4096, dtype=torch.float32, device=DEV)
    c = st.vector_add(a, a)
    torch.cuda.synchronize()
    assert torch.equal(c, 2 * a)


@pytest.mark.parametrize("kind", [0, 1])
def test_wait_that_runs_out_is_reported_and_cleared(kind):
    rc = check_wait(kind, 2000, N.ST_EXEC_SYNC)
    assert rc == N.ST_ERR_DEVICE_ABORT
    assert f"(code {CODES[kind]})" in N.last_error()
    st.sync(0)  # the word was cleared by the report
    add_still_works()


@pytest.mark.parametrize("kind", [0, 1])
def test_asynchronous_call_reports_at_the_next_host_wait(kind):
    assert check_wait(kind, 1000, 0) == N.ST_OK  # queued, not waited for
    with pytest.raises(st.DeviceAbort, match=f"code {CODES[kind]}"):
        st.sync(0)
    st.sync(0)
    add_still_works()
