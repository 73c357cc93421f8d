"""2-GPU data parallelism: the NVLink peer-memory collectives (fused reduce-to-owner, all-gather, mailbox
all-reduce; serial, overlapped with kernel pushes, overlapped with copy-engine pushes, and the latter inside the
whole-update CUDA graph; gradients overlapped with parameters by the fused Adam + push) against the NCCL path on the
same training run."""
import os

import pytest
import torch

from faster_yoco_b200.utils import dist_checks
from faster_yoco_b200.utils.launch import run_ranks

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def test_fused_p2p_matches_nccl(tmp_path):
    run_ranks(dist_checks.fused_vs_nccl_gpu, 2, str(tmp_path), 4, backend="nccl", timeout_s=300)
    r = torch.load(os.path.join(tmp_path, "fused_vs_nccl.pt"))
    for name in ("fused", "fused_serial", "fused_ce", "fused_ce_graph", "fused_serial_two_pass", "fused_grads_ce",
                 "fused_grads_sm_graph"):
        assert r[name]["status"] == 0 and r["nccl"]["status"] == 0
        for a, b in zip(r[name]["losses"], r["nccl"]["losses"]):
            assert abs(a - b) / abs(b) < 2e-3, (name, r[name]["losses"], r["nccl"]["losses"])
        pf, pn = r[name]["params"], r["nccl"]["params"]
        assert ((pf - pn).abs().max() / pn.abs().max()).item() < 2e-2, name
    # the overlapped and the serial peer-memory paths reduce in the same order; what differs run to run is only the
    # order of the fp32 atomics of the attention dQ accumulation
    for name in ("fused", "fused_ce", "fused_ce_graph", "fused_serial_two_pass", "fused_grads_ce",
                 "fused_grads_sm_graph"):
        for a, b in zip(r[name]["losses"], r["fused_serial"]["losses"]):
            assert abs(a - b) / abs(b) < 2e-4, (name, r[name]["losses"], r["fused_serial"]["losses"])
        pf, ps = r[name]["params"], r["fused_serial"]["params"]
        assert ((pf - ps).abs().max() / ps.abs().max()).item() < 1e-2, name


@pytest.mark.parametrize("chunk", [0, 1 << 14])
def test_gemm_gather_two_ranks(tmp_path, chunk):
    """The all-gather fused into the consumer GEMM over real peer replicas (2 GPUs)."""
    run_ranks(dist_checks.gemm_gather_gpu, 2, str(tmp_path), chunk, backend="nccl", timeout_s=180)
    for r in range(2):
        res = torch.load(os.path.join(tmp_path, f"gemm_gather_{r}.pt"))
        assert res["status"] == 0 and res["ok"], res
        assert res["err"] < 1e-2, res
