"""The chunked restatements of the SSD scans against the sequential recurrence
(CPU, fp64).  The sequential recurrence is the ground truth: the reference's
own chunked code pairs the diagonal with ``C_l . B_l`` (mamba2.rs:523-536,
mamba3.rs:803-811) and the Mamba3 inter-chunk state with B_t
(mamba3.rs:709-712); those two quirks are reproduced only under
``compat: reference``, and must differ from the recurrence."""
import torch

from oxidizr_b200.ops import reference as R


def _inputs(b=2, S=21, H=3, P=4, N=5, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(b, S, H, P, generator=g, dtype=torch.float64)
    dt = torch.rand(b, S, H, generator=g, dtype=torch.float64) * 0.4 + 0.05
    A = -(torch.rand(H, generator=g, dtype=torch.float64) * 2 + 0.1)
    Bm = torch.randn(b, S, H, N, generator=g, dtype=torch.float64)
    Cm = torch.randn(b, S, H, N, generator=g, dtype=torch.float64)
    lam = torch.rand(b, S, H, generator=g, dtype=torch.float64)
    return x, dt, A, Bm, Cm, lam


def _rel(a, b):
    return ((a - b).norm() / b.norm()).item()


def test_ssd_chunked_equals_sequential():
    x, dt, A, Bm, Cm, _ = _inputs()
    seq = R.ssd_sequential(x, dt, A, Bm, Cm)
    for chunk in (4, 8, 21, 32):  # S = 21: a ragged last chunk, one chunk, a chunk longer than S
        assert _rel(R.ssd_chunked(x, dt, A, Bm, Cm, chunk), seq) < 1e-12, chunk


def test_ssd_diag_only_g_is_not_the_recurrence():
    x, dt, A, Bm, Cm, _ = _inputs()
    seq = R.ssd_sequential(x, dt, A, Bm, Cm)
    assert _rel(R.ssd_chunked(x, dt, A, Bm, Cm, 8, diag_only_g=True), seq) > 1e-2


def test_mamba3_chunked_equals_sequential():
    x, dt, A, Bm, Cm, lam = _inputs(seed=1)
    seq = R.mamba3_sequential(x, dt, A, Bm, Cm, lam)
    for chunk in (4, 8, 21, 32):
        assert _rel(R.mamba3_scan(x, dt, A, Bm, Cm, lam, chunk), seq) < 1e-12, chunk


def test_mamba3_compat_pairing_is_not_the_recurrence():
    x, dt, A, Bm, Cm, lam = _inputs(seed=1)
    seq = R.mamba3_sequential(x, dt, A, Bm, Cm, lam)
    # one chunk: no inter-chunk state, the quirk does not show
    assert _rel(R.mamba3_scan(x, dt, A, Bm, Cm, lam, 32, compat=True), seq) < 1e-12
    # several chunks: it does
    assert _rel(R.mamba3_scan(x, dt, A, Bm, Cm, lam, 4, compat=True), seq) > 1e-3


def test_mamba3_shifted_state_identity():
    """The single-term form run on the tensor cores: K_t = a_t K_{t-1} + (gamma_t + c_t) u_t with
    c_t = (1 - lam_{t+1}) dt_{t+1} (c_{S-1} = 0), y_t = C_t K_t - c_t <B_t, C_t> x_t, equals the
    two-term trapezoidal recurrence exactly."""
    x, dt, A, Bm, Cm, lam = _inputs(seed=2)
    w = (1 - lam) * dt
    c = torch.cat([w[:, 1:], torch.zeros_like(w[:, :1])], 1)
    gp = lam * dt + c
    # ssd_sequential adds dt_t u_t: feed x scaled by gp / dt to get gp_t u_t
    yk = R.ssd_sequential(x * (gp / dt)[..., None], dt, A, Bm, Cm)
    y = yk - (c * (Bm * Cm).sum(-1))[..., None] * x
    assert _rel(y, R.mamba3_sequential(x, dt, A, Bm, Cm, lam)) < 1e-12


def test_selective_scan_clamp_only_in_compat():
    """Mamba1: without the clamp the scan is the plain linear recurrence; with A > 0 (the
    reference's sign) the state grows and the +-30 clamp changes the result."""
    g = torch.Generator().manual_seed(3)
    b, S, D, N = 1, 40, 6, 4
    u = torch.randn(b, S, D, generator=g, dtype=torch.float64) * 3
    delta = torch.rand(b, S, D, generator=g, dtype=torch.float64)
    Bm = torch.randn(b, S, N, generator=g, dtype=torch.float64)
    Cm = torch.randn(b, S, N, generator=g, dtype=torch.float64)
    A_neg = -torch.rand(D, N, generator=g, dtype=torch.float64)
    a = R.selective_scan(u, delta, A_neg, Bm, Cm)
    # linear recurrence by hand
    h = torch.zeros(b, D, N, dtype=torch.float64)
    ys = []
    for t in range(S):
        h = torch.exp(delta[:, t, :, None] * A_neg) * h + delta[:, t, :, None] * u[:, t, :, None] * Bm[:, t, None]
        ys.append((h * Cm[:, t, None]).sum(-1))
    assert _rel(a, torch.stack(ys, 1)) < 1e-12
    A_pos = torch.rand(D, N, generator=g, dtype=torch.float64) + 0.5
    free = R.selective_scan(u, delta, A_pos, Bm, Cm)
    clamped = R.selective_scan(u, delta, A_pos, Bm, Cm, clamp=30.0)
    assert _rel(clamped, free) > 1e-3
