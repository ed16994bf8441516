"""Expert parallelism: the sharded MoE layer (E/W experts per rank) against the
whole layer, across real processes.

CPU: gloo ranks exchanging rows with all-to-all.  GPU (>= 2 devices): the
NVLink dispatch/combine kernels and the NCCL all-to-all baseline.
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


def _run(tmp_path, device, backend, world=2, extra=(), timeout=240):
    out = str(tmp_path / f"ep_{device}_{backend}_{world}.json")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", "-m", "oxidizr_b200.parallel.ep_selftest",
           "--device", device, "--backend", backend, "--out", out, *extra]
    env = dict(os.environ, PYTHONPATH=REPO, NCCL_NVLS_ENABLE="0", OMP_NUM_THREADS="1")
    r = subprocess.run(["timeout", "-k", "30", str(timeout)] + cmd, cwd=REPO, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return json.load(open(out))


def test_ep_gloo_matches_whole_layer(tmp_path):
    res = _run(tmp_path, "cpu", "nccl")
    for e in res["errors"]:
        assert e["max_over_ranks"] < 1e-5, e


@pytest.mark.gpu
@pytest.mark.parametrize("backend", ["nvlink", "nccl"])
@pytest.mark.parametrize("shape", [("300", "8", "2", "256", "128", ""), ("1000", "16", "4", "512", "256", ""),
                                   ("700", "16", "4", "512", "256", "--two-layers")])
def test_ep_gpu_matches_whole_layer(tmp_path, backend, shape):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    T, E, k, H, I, extra = shape
    res = _run(tmp_path, "cuda", backend,
               extra=("--tokens", T, "--experts", E, "--topk", k, "--hidden", H, "--inter", I)
               + ((extra,) if extra else ()))
    for e in res["errors"]:
        assert e["y"] < 2e-2 and e["dx"] < 3e-2 and e["router"] < 5e-2, e
        assert e["w_gu"] < 3e-2 and e["w_down"] < 3e-2, e
        assert not e.get("skipped"), e
    assert res.get("regrows", 0) == 0


@pytest.mark.gpu
def test_ep_over_capacity_skips_then_regrows(tmp_path):
    """Receive buffers that start too small: the first step's layers run over capacity on
    the device, are skipped on every rank and flag the step (the optimizer would skip its
    update); the host regrows the buffers before the next step, which matches the whole
    layer.  No host read of the routing counts happens inside a step."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = _run(tmp_path, "cuda", "nvlink",
               extra=("--tokens", "1000", "--experts", "16", "--topk", "4", "--hidden", "512", "--inter", "256",
                      "--steps", "3", "--initial-rows", "256"))
    first = [e for e in res["errors"] if e["step"] == 0]
    later = [e for e in res["errors"] if e["step"] > 0]
    assert first and all(e["skipped"] for e in first), first
    assert res["regrows"] == 1
    for e in later:
        assert not e["skipped"], e
        assert e["y"] < 2e-2 and e["dx"] < 3e-2 and e["router"] < 5e-2, e
        assert e["w_gu"] < 3e-2 and e["w_down"] < 3e-2, e
