"""Model FLOPs per token (oxidizr_b200/utils/flops.py) against hand counts of the bench configs."""
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)


def test_llama_flops_per_token_by_hand():
    import bench
    from oxidizr_b200.utils.flops import flops_per_token
    m = bench.bench_config("llama").model
    H, L, nh, kv, I, V, S = 2048, 16, 16, 8, 5632, 128354, 2048
    hd = H // nh
    attn = H * (nh * hd + 2 * kv * hd) + nh * hd * H
    mlp = 3 * H * I
    params = L * (attn + mlp) + V * H          # the embedding is a gather, lm_head a matmul
    scores = L * 3.0 * S * nh * 2 * hd         # causal half of QK^T and PV, forward + backward
    assert abs(flops_per_token(m) - (6.0 * params + scores)) < 1.0
    assert 6.4e9 < flops_per_token(m) < 6.6e9


def test_mamba3_scan_counted_once():
    import bench
    from oxidizr_b200.utils.flops import _mamba2
    m = bench.bench_config("mamba3").model
    p, scan = _mamba2(m, True)
    hs, P, N, C, R = 32, 64, 128, 256, 4
    assert scan == 3.0 * hs * (C * (N + P * R) + 4 * N * P * R)
    assert p > 0
