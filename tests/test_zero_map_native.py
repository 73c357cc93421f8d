"""The owner-map arithmetic of the sm_100a kernels (csrc/common/zero_map.cuh), compiled for the host with nvcc and
run on sampled flat indices, against the Python owner map of FlatParams (which the gloo training tests validate):
owner, local index, the round trip back to the flat index, and the owner-scatter destination (own slot, or owner
o's staging slot for this rank at the local index)."""
import os
import shutil
import subprocess

import pytest

from faster_yoco_b200.parallel.zero import FlatParams

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "faster_yoco_b200", "csrc")


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available")
    exe = str(tmp_path_factory.mktemp("zm") / "zero_map_check")
    subprocess.run([nvcc, "-O2", "-std=c++17", "-I" + CSRC, os.path.join(HERE, "native", "zero_map_check.cu"),
                    "-o", exe], check=True, capture_output=True)
    return exe


def _flat(world, rank, chunk):
    import torch
    m = torch.nn.ModuleDict({"a": torch.nn.Linear(48, 200, bias=False), "b": torch.nn.Linear(200, 96, bias=False),
                             "n": torch.nn.LayerNorm(96, bias=False)})
    return FlatParams(m.named_parameters(), world, rank, "cpu", partition="cyclic" if chunk else "even", chunk=chunk)


@pytest.mark.parametrize("world,chunk", [(2, 0), (4, 0), (3, 64), (8, 128)])
def test_kernel_owner_map_matches_python(checker, world, chunk):
    rank = world - 1
    fp = _flat(world, rank, chunk)
    n = world * fp.seg
    out = subprocess.run([checker, str(world), str(fp.seg), str(fp.chunk), str(rank), "0", str(min(n, 4000)),
                          str(max(1, n // 4000))], check=True, capture_output=True, text=True).stdout.split("\n")
    rows = [list(map(int, l.split())) for l in out if l.strip()]
    assert len(rows) > 100
    own_base, seg = 15 << 40, fp.seg
    for x, o, loc, back, dst in rows:
        assert o == fp.owner_of(x) and loc == fp.local_of(x), (x, o, loc)
        assert back == x
        want = own_base + 2 * x if o == rank else ((o + 1) << 40) + 2 * (rank * seg + loc)
        assert dst == want, (x, o, dst, want)
