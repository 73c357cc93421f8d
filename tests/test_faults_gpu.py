"""Failure detection on the GPU without a fault: a device wait on a flag that nothing sets runs out after its time
limit, records an error word the host reads, and returns -- the context stays usable."""
import time

import pytest
import torch

from faster_yoco_b200 import ops
from faster_yoco_b200.utils.faults import DeviceStatus

pytestmark = pytest.mark.gpu


def _gemm_still_works():
    a = torch.randn(256, 128, device="cuda", dtype=torch.bfloat16)
    b = torch.randn(192, 128, device="cuda", dtype=torch.bfloat16)
    c = torch.empty(256, 192, device="cuda", dtype=torch.bfloat16)
    ops._C().gemm(a, b, c, False, False, None)
    ref = a.float() @ b.float().T
    assert ((c.float() - ref).abs().max() / ref.abs().max()).item() < 1e-2


def test_arrival_wait_times_out_and_context_survives():
    C = ops._C()
    st = DeviceStatus.native()
    st.clear()
    arrive = torch.zeros(64, dtype=torch.int32, device="cuda")      # nobody ever adds to it
    expected = torch.zeros_like(arrive)
    t0 = time.time()
    C.wait_arrivals(arrive, expected, 5, 1)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert st.value() == (1 << 16) | 305, hex(st.value())           # peer timeout at site 300 + bucket
    assert 1.0 < dt < 60.0
    with pytest.raises(RuntimeError, match="peer flag wait timed out"):
        st.raise_if_set()
    st.clear()
    _gemm_still_works()
    assert st.value() == 0


def test_flag_barrier_with_missing_peer_times_out():
    C = ops._C()
    st = DeviceStatus.native()
    st.clear()
    mine = torch.zeros(64 * 8, dtype=torch.int32, device="cuda")
    absent_peer = torch.zeros_like(mine)                              # a "peer" that never arrives
    counters = torch.zeros(65, dtype=torch.int32, device="cuda")
    C.flag_barrier([mine.data_ptr(), absent_peer.data_ptr()], mine, counters, 0, 3)
    torch.cuda.synchronize()
    assert st.value() == (1 << 16) | 203, hex(st.value())
    assert int(absent_peer[3 * 8 + 0].item()) == 1                   # our arrival was published to the peer
    st.clear()
    _gemm_still_works()
