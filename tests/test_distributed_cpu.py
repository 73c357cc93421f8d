"""ZeRO data parallelism on CPU ranks (gloo, world_size 2): equivalence with single-process training,
checkpoint/resume (world-size independent optimizer state) and host-injected failure detection."""
import os
import time

import pytest
import torch

from faster_yoco_b200.parallel.zero import greedy_partition
from faster_yoco_b200.utils import dist_checks
from faster_yoco_b200.utils.launch import run_ranks


def test_greedy_partition_is_oss_rule():
    # next parameter to the rank with the smallest running total, ties to the lowest rank
    assert greedy_partition([10, 10, 5, 5, 1], 2) == [0, 1, 0, 1, 0]
    assert greedy_partition([100, 1, 1, 1], 3) == [0, 1, 2, 1]


@pytest.mark.parametrize("partition,chunk,sharding", [("even", None, "os"), ("cyclic", 1024, "os"),
                                                      ("even", None, "none")])
def test_zero_ws2_matches_single_process(tmp_path, partition, chunk, sharding):
    """ZeRO-1 (contiguous and block-cyclic owner maps) and unsharded data parallelism (--zero-sharding none)."""
    steps = 3
    run_ranks(dist_checks.zero_matches_single, 2, str(tmp_path), steps, partition, chunk, sharding)
    got = torch.load(os.path.join(tmp_path, f"ws2_{partition}_{sharding}.pt"))
    assert got["num_updates"] == steps
    ref = dist_checks.single_reference(str(tmp_path), 2, steps)
    for k, v in ref.items():
        assert torch.allclose(got["sd"][k].float(), v.float(), atol=2e-5, rtol=1e-4), k


@pytest.mark.parametrize("partition,resume_partition", [("even", "even"), ("cyclic", "cyclic"),
                                                        ("cyclic", "even"), ("greedy", "cyclic"),
                                                        ("even", "greedy")])
def test_checkpoint_resume_matches_uninterrupted(tmp_path, partition, resume_partition):
    run_ranks(dist_checks.checkpoint_resume, 2, str(tmp_path), 4, 2, partition, 1024, resume_partition)
    r = torch.load(os.path.join(tmp_path, "resume.pt"))
    assert r["n2"] == r["n3"] == 4
    for k, v in r["straight"].items():
        assert torch.allclose(r["resumed"][k].float(), v.float(), atol=1e-6, rtol=1e-5), k
    ck = torch.load(os.path.join(tmp_path, "ckpt.pt"))
    assert any(k.startswith("decoder.model.self_decoder.layers.0.mixer.q_proj") for k in ck["model"])
    assert "self_decoder.layers.0.mixer.q_proj.weight" in ck["last_optimizer_state"]["exp_avg"]


def test_injected_rank_failure_does_not_hang(tmp_path):
    t0 = time.time()
    with pytest.raises(RuntimeError):
        run_ranks(dist_checks.rank_fails_before_collective, 2, str(tmp_path), timeout_s=20)
    assert time.time() - t0 < 150


def test_exchange_free_measurement_mode(tmp_path):
    run_ranks(dist_checks.exchange_free_steps, 2, str(tmp_path), 2)
    r = torch.load(os.path.join(tmp_path, "noexchange.pt"))
    assert r["diverged"] and r["changed"] and r["loss"] == r["loss"]


def test_tensor_x_data_parallel_training_matches_single_process(tmp_path):
    """TP 2 x DP 2 on 4 gloo ranks: every slice ends where the matching slice of single-process training (same
    global batch, same initial weights) ends, and the clipped norm is the global one."""
    from faster_yoco_b200.models.yoco import shard_state_dict
    steps = 3
    model, tr = dist_checks._tiny_trainer(torch.device("cpu"))
    full0 = {k: v.detach().clone() for k, v in model.state_dict().items()}
    run_ranks(dist_checks.tp_dp_matches_single, 4, str(tmp_path), steps, full0, timeout_s=240)
    ref, ref_norm = dist_checks.single_reference(str(tmp_path), 2, steps, with_norm=True)
    for r in range(2):
        saved = torch.load(os.path.join(tmp_path, f"tp{r}.pt"))
        assert abs(saved["gnorm"] - ref_norm) <= 1e-5 * ref_norm, (saved["gnorm"], ref_norm)
        got = saved["sd"]
        want = shard_state_dict(ref, 2, r)
        assert set(got) == set(want)
        for k, v in want.items():
            assert torch.allclose(got[k].float(), v.float(), atol=2e-5, rtol=1e-4), k


def test_single_node_detection(monkeypatch):
    from faster_yoco_b200.parallel import dist as D
    monkeypatch.delenv("LOCAL_WORLD_SIZE", raising=False)
    assert D.single_node()
    monkeypatch.setenv("WORLD_SIZE", "16")
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "8")
    assert not D.single_node()
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "16")
    assert D.single_node()
