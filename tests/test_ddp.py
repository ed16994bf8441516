"""Data-parallel training across real processes.

CPU: two gloo ranks (backend cpustaging) must agree with each other and with a
single process that sees both ranks' data.  GPU (needs >= 2 devices): the fused
NVLink path must track the NCCL baseline.
"""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(backend, world, tmp_path, steps=3, timeout=240, env_extra=None):
    tag = "_".join(f"{k}{v}" for k, v in sorted((env_extra or {}).items()))
    out = str(tmp_path / f"{backend}_{world}{tag}.json")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", "-m", "oxidizr_b200.parallel.selftest",
           "--backend", backend, "--steps", str(steps), "--out", out]
    env = dict(os.environ, PYTHONPATH=REPO, NCCL_NVLS_ENABLE="0", OMP_NUM_THREADS="1", **(env_extra or {}))
    r = subprocess.run(["timeout", "-k", "30", str(timeout)] + cmd, cwd=REPO, env=env, capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return json.load(open(out))


def test_gloo_ddp_two_ranks(tmp_path):
    res = _run("cpustaging", 2, tmp_path)
    assert len(res["losses"]) == 3
    assert all(l == l for l in res["losses"])
    assert res["losses"][-1] < res["losses"][0] + 0.5


@pytest.mark.gpu
def test_fused_ddp_matches_nccl(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    a = _run("nccl", 2, tmp_path, steps=4)
    b = _run("fused", 2, tmp_path, steps=4)
    for la, lb in zip(a["losses"], b["losses"]):
        assert abs(la - lb) < 2e-2 * abs(la), (a["losses"], b["losses"])
    for na, nb in zip(a["grad_norms"], b["grad_norms"]):
        assert abs(na - nb) < 5e-2 * abs(na) + 1e-3, (a["grad_norms"], b["grad_norms"])


def _multicast_ok() -> bool:
    from oxidizr_b200.parallel.fused_ar import multicast_supported
    return multicast_supported(torch.device("cuda", 0))


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["pull", "push", "nvls"])
def test_sharded_transports_agree(tmp_path, mode):
    """The NVLink transports (P2P pull / push, NVLS multicast) against the same
    sharded algorithm over NCCL: the same losses, norms and replicas."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    if mode == "nvls" and not _multicast_ok():
        pytest.skip("no multicast support on these GPUs")
    a = _run("nccl_sharded", 2, tmp_path, steps=4)
    b = _run("fused", 2, tmp_path, steps=4, env_extra={"OXI_AR_MODE": mode})
    for la, lb in zip(a["losses"], b["losses"]):
        assert abs(la - lb) < 1e-2 * abs(la), (a["losses"], b["losses"])
    for na, nb in zip(a["grad_norms"], b["grad_norms"]):
        assert abs(na - nb) < 3e-2 * abs(na) + 1e-3, (a["grad_norms"], b["grad_norms"])


@pytest.mark.gpu
def test_peer_wait_gives_up_and_reports():
    """A peer flag that nobody sets: the norm exchange stops waiting after its
    limit, records the peer-timeout status and disables the update (coef 0),
    and the device stays usable afterwards.  Runs as one kernel on one GPU."""
    import time
    from oxidizr_b200.ops._C import ext, read_status, status
    dev = torch.device("cuda", 0)
    read_status(dev)
    pad = torch.zeros(ext().pad_words(), dtype=torch.int32, device=dev)
    # a two-rank job whose "peer" pad is our own: rank 0 posts its flag, rank 1's never comes
    table = torch.tensor([pad.data_ptr(), pad.data_ptr()], dtype=torch.int64, device=dev)
    sumsq = torch.ones(1, device=dev)
    coef = torch.full((1,), 7.0, device=dev)
    norm = torch.zeros(1, device=dev)
    t0 = time.time()
    ext().norm_exchange(table, pad, 0, 2, 1, sumsq, 1.0, coef, norm, status(dev), int(0.2e9))
    torch.cuda.synchronize(dev)
    dt = time.time() - t0
    assert read_status(dev) == 2  # OXI_ERR_TIMEOUT_PEER
    assert coef.item() == 0.0 and norm.isnan().item()
    assert dt < 5.0
    x = torch.randn(1000, device=dev)
    assert abs((x * 2).sum().item() - 2 * x.sum().item()) < 1e-2
