"""Roofline arithmetic of the data-parallel step benchmark (parallel/commbench.py) and
the expert-parallel layer benchmark (parallel/epbench.py), on CPU: the byte and FLOP
counts against hand calculations for the configurations the profiles quote."""
import pytest


def test_sharded_step_roofline_counts():
    from oxidizr_b200.parallel.commbench import NVLINK_GBS, roofline_ms
    N = 1_280_000_000
    # W = 2: HBM = 10N + 2N + 4N/2 + 28N/2 + 2N = 30N bytes; P2P NVLink out 4N/2 = 2N
    r = roofline_ms(N, 2, "pull", 6458.0)
    assert r["hbm_ms"] == pytest.approx(30 * N / 6458e9 * 1e3, rel=1e-3)
    assert r["nvlink_ms"] == pytest.approx(2 * N / (NVLINK_GBS * 1e9) * 1e3, rel=1e-3)
    assert r["bound"] == "hbm" and r["roofline_ms"] == r["hbm_ms"]
    # W = 8: HBM = 14N + 32N/8 = 18N; P2P out 4N * 7/8 = 3.5N; NVLS out 2N + 2N/8 = 2.25N
    p8 = roofline_ms(N, 8, "pull", 6549.4)
    n8 = roofline_ms(N, 8, "nvls", 6549.4)
    assert p8["hbm_ms"] == pytest.approx(18 * N / 6549.4e9 * 1e3, rel=1e-3)
    assert p8["nvlink_ms"] == pytest.approx(3.5 * N / 770e9 * 1e3, rel=1e-3)
    assert n8["nvlink_ms"] == pytest.approx(2.25 * N / 770e9 * 1e3, rel=1e-3)
    assert p8["bound"] == n8["bound"] == "nvlink"
    assert n8["roofline_ms"] < p8["roofline_ms"]


def test_expert_parallel_phase_rooflines():
    from oxidizr_b200.parallel.epbench import phase_rooflines
    H, I, peak = 2048, 1024, 1324.7e12
    rows_out, rows_in, rows_local = 114_562, 116_235, 132_745
    r = phase_rooflines(rows_out, rows_in, rows_local, H, I, peak)
    link = 116_235 * 2 * H / 770e9 * 1e3  # the larger direction, bf16 rows
    assert r["send_fwd"] == pytest.approx(link) and r["send_bwd"] == pytest.approx(link)
    assert r["gemm_gu"] == pytest.approx(2 * rows_local * H * 2 * I / peak * 1e3)
    # the fused return phases are bounded by the slower of the GEMM and the transfer
    assert r["gemm_down_ret"] == pytest.approx(max(2 * rows_local * I * H / peak * 1e3, link))
    assert r["gemm_dx_ret"] == pytest.approx(max(2 * rows_local * 2 * I * H / peak * 1e3, link))
    assert r["gemm_wgrad"] == pytest.approx(2 * rows_local * H * 3 * I / peak * 1e3)
    # the figures quoted in the 8-GPU profile
    assert round(r["send_fwd"], 3) == 0.618 and round(r["gemm_gu"], 3) == 0.841
