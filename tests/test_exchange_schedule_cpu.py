"""Host logic of the exchange schedule: the measured per-GPU-count choice behind overlap / transport "auto", and
which exchange the optimizer step runs for the parameters under each overlap form (CPU, fake peer transport)."""
import torch

from faster_yoco_b200.config import OptimConfig, build_args
from faster_yoco_b200.models.yoco import YOCO
from faster_yoco_b200.parallel.zero import FlatParams, ZeroOptimizer


def test_exchange_schedule_auto_and_explicit():
    """The measured exchange schedule behind overlap / transport "auto", and explicit values passed through."""
    from faster_yoco_b200.parallel.zero import AUTO_SCHEDULE, exchange_schedule
    for world, (ov, tr) in AUTO_SCHEDULE.items():
        assert exchange_schedule(world, "fused") == (ov, tr)
        assert exchange_schedule(world, "nccl") == (False, "sm")        # the library path has no peer pushes
    assert exchange_schedule(1, "fused") == (False, "sm")
    assert exchange_schedule(2, "fused", "0", "auto")[0] is False
    assert exchange_schedule(8, "fused", "1", "ce") == (True, "ce")
    assert exchange_schedule(8, "fused", "grads", "ce") == ("grads", "ce")
    assert exchange_schedule(2, "fused", "auto", "pull") == (False, "pull")   # pull carries its own all-gather
    assert exchange_schedule(2, "fused", "auto", "gemm") == (False, "gemm")


class _FakeBuckets:
    """The parts of PeerComm the optimizer step consults, recording the parameter exchanges it asks for."""

    def __init__(self, params_mode):
        self.buckets = ([], [])
        self.params_mode = params_mode
        self.calls = []

    def all_gather(self, *a, **k):
        self.calls.append("all_gather")


def test_parameter_exchange_follows_the_overlap_form():
    torch.manual_seed(0)
    model = YOCO(build_args("yoco_tiny", max_seq_len=64))
    fp = FlatParams(model.named_parameters(), 2, 0, "cpu", dtype=torch.float32)
    zero = ZeroOptimizer(fp, OptimConfig(), comm="fused")
    # overlap 1: the parameters leave per bucket ahead of the next forward, so the step itself sends nothing
    zero.p2p = _FakeBuckets("bucketed")
    zero.all_gather_params()
    assert zero.p2p.calls == []
    # overlap "grads": only the gradients were bucketed; the step sends the parameters (on the GPU the fused
    # Adam + push kernel does it, elsewhere the all-gather after Adam)
    zero.p2p = _FakeBuckets("fused")
    zero.all_gather_params()
    assert zero.p2p.calls == ["all_gather"]
