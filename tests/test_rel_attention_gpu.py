"""p2cu_rel_attention: the encoder's relative-position self-attention as one tensor-core kernel (attn_rel_tc.cu).

The truth is the reference's self_attention core (csrc/encoder.c:471-528 with combine_softmax at :425-447) in float64
on the same inputs: Q + bias_u and Q + bias_v rounded to fp32 as the reference adds them, then AC = Q_u K^T,
BD = Q_v P^T over the window's 2T - 1 positions, scores (AC[i][j] + BD[i][T - 1 - i + j]) / sqrt(128), a softmax per
row and the context S V, per head, the heads concatenated. The kernel computes every product in the three-part tf32
split (about fp32 accuracy) with an online softmax, so it is held to a tolerance, written below, not to bits. The
argument checks run on the CPU (no device call is made before they pass).
"""
import ctypes as C

import numpy as np
import pytest

D, H, DH = 1024, 8, 128
# |kernel - float64 truth| <= TOL * max |V| * max(1, max |score| / 4) over a window's outputs: the fp32-class error
# of the split products (a score's absolute error grows with its size, and a probability's relative error is that
# absolute error) and of the softmax; scores of these N(0, 1)-like inputs stay below 4
TOL = 2e-5


def _truth(qkv, P, bu, bv, Ts, Tmax):
    out = np.zeros((sum(Ts), D), np.float64)
    smax = []
    scale = np.float64(np.float32(1.0) / np.sqrt(np.float32(DH)))
    r0 = 0
    for T in Ts:
        i = np.arange(T)
        sm = 0.0
        idx = (T - 1 - i)[:, None] + i[None, :]
        for h in range(H):
            sl = slice(h * DH, (h + 1) * DH)
            Q = qkv[r0:r0 + T, sl]
            K = qkv[r0:r0 + T, D + h * DH:D + (h + 1) * DH].astype(np.float64)
            V = qkv[r0:r0 + T, 2 * D + h * DH:2 * D + (h + 1) * DH].astype(np.float64)
            Qu = (Q + bu[sl]).astype(np.float64)   # fp32 additions, as the reference's gather_heads
            Qv = (Q + bv[sl]).astype(np.float64)
            Pw = P[Tmax - T:Tmax + T - 1, sl].astype(np.float64)
            ac = Qu @ K.T
            bd = Qv @ Pw.T
            s = (ac + np.take_along_axis(bd, idx, axis=1)) * scale
            sm = max(sm, float(np.abs(s).max()))
            s -= s.max(axis=1, keepdims=True)
            e = np.exp(s)
            out[r0:r0 + T, sl] = (e / e.sum(axis=1, keepdims=True)) @ V
        smax.append(sm)
        r0 += T
    return out, smax


def _inputs(Ts, Tmax, seed, pattern=None):
    rng = np.random.default_rng(seed)
    R = sum(Ts)
    qkv = (0.5 * rng.standard_normal((R, 3 * D))).astype(np.float32)
    P = (0.5 * rng.standard_normal((2 * Tmax - 1, D))).astype(np.float32)
    bu = (0.1 * rng.standard_normal(D)).astype(np.float32)
    bv = (0.1 * rng.standard_normal(D)).astype(np.float32)
    if pattern is not None:
        # scores that climb (or fall) steadily along the keys: Q = 0, bias_u = 4 u for a unit vector u, K_j = j/4 u
        # (or (T - 1 - j)/4 u), so a score grows by 5.7 per 64-key chunk and the online softmax's reference (slack
        # 16) moves every third chunk when they rise
        u = rng.standard_normal(DH).astype(np.float32)
        u /= np.linalg.norm(u)
        qkv[:, :D] = 0.0
        bu[:] = np.tile(4.0 * u, H)
        r0 = 0
        for T in Ts:
            j = np.arange(T, dtype=np.float32)
            steep = (j / 4.0) if pattern == "rising" else ((T - 1 - j) / 4.0)
            qkv[r0:r0 + T, D:2 * D] = np.tile(steep[:, None] * u[None, :], (1, H))
            r0 += T
    return qkv, P, bu, bv


def _run(pkg, Ts, Tmax, qkv, P, bu, bv):
    import torch
    dev = torch.device("cuda:0")
    L = pkg.lib()
    Tarr = (C.c_int * len(Ts))(*Ts)
    nws = L.p2cu_rel_attention_ws_bytes(len(Ts), Tarr)
    assert nws > 0
    t = {k: torch.from_numpy(v).to(dev) for k, v in dict(qkv=qkv, P=P, bu=bu, bv=bv).items()}
    out = torch.full((sum(Ts), D), float("nan"), dtype=torch.float32, device=dev)
    ws = torch.empty(nws, dtype=torch.uint8, device=dev)
    pkg.check(L.p2cu_rel_attention(t["qkv"].data_ptr(), t["P"].data_ptr(), t["bu"].data_ptr(), t["bv"].data_ptr(),
                                   Tarr, len(Ts), Tmax, out.data_ptr(), ws.data_ptr(), nws, None))
    pkg.check_device()
    return out.cpu().numpy()


def _check(got, truth, qkv, Ts):
    want, smax = truth
    assert np.isfinite(got).all()
    r0 = 0
    for T, sm in zip(Ts, smax):
        vmax = float(np.abs(qkv[r0:r0 + T, 2 * D:]).max())
        err = float(np.abs(got[r0:r0 + T] - want[r0:r0 + T]).max())
        print(f"T={T}: max |err| {err:.3g}, max |V| {vmax:.3g}, max |score| {sm:.3g}")
        assert err <= TOL * vmax * max(1.0, sm / 4.0), (T, err, vmax, sm)
        r0 += T


@pytest.mark.gpu
@pytest.mark.parametrize("Ts,Tmax", [
    ([1, 64, 65, 127, 128, 129, 200], 200),   # one frame; one chunk exactly; a chunk and one; the query-tile edges
    ([375, 438, 300], 438),                   # config-3 lengths (25 - 35 s windows)
    ([512, 100], 512),                        # the longest window the kernel takes beside a short one
    ([38], 38),                               # config 4 (3 s)
])
def test_rel_attention_matches_float64(pkg, cuda, Ts, Tmax):
    qkv, P, bu, bv = _inputs(Ts, Tmax, seed=sum(Ts))
    got = _run(pkg, Ts, Tmax, qkv, P, bu, bv)
    _check(got, _truth(qkv, P, bu, bv, Ts, Tmax), qkv, Ts)


@pytest.mark.gpu
@pytest.mark.parametrize("pattern", ["rising", "falling"])
def test_rel_attention_online_softmax_moves(pkg, cuda, pattern):
    """Scores that rise along the keys past the kernel's slack (the running reference moves and the context is
    rescaled), and scores that fall (it never moves)."""
    Ts, Tmax = [512, 300], 512
    qkv, P, bu, bv = _inputs(Ts, Tmax, seed=3, pattern=pattern)
    got = _run(pkg, Ts, Tmax, qkv, P, bu, bv)
    _check(got, _truth(qkv, P, bu, bv, Ts, Tmax), qkv, Ts)


@pytest.mark.gpu
def test_rel_attention_rows_outside_windows_untouched(pkg, cuda):
    """The kernel writes exactly the windows' rows: a buffer longer than the windows keeps its tail."""
    import torch
    Ts, Tmax = [130, 70], 130
    qkv, P, bu, bv = _inputs(Ts, Tmax, seed=11)
    L = pkg.lib()
    Tarr = (C.c_int * 2)(*Ts)
    nws = L.p2cu_rel_attention_ws_bytes(2, Tarr)
    dev = torch.device("cuda:0")
    out = torch.full((sum(Ts) + 16, D), 7.0, dtype=torch.float32, device=dev)
    ws = torch.empty(nws, dtype=torch.uint8, device=dev)
    t = [torch.from_numpy(a).to(dev) for a in (qkv, P, bu, bv)]
    pkg.check(L.p2cu_rel_attention(*(x.data_ptr() for x in t), Tarr, 2, Tmax, out.data_ptr(), ws.data_ptr(), nws,
                                   None))
    pkg.check_device()
    o = out.cpu().numpy()
    assert (o[sum(Ts):] == 7.0).all()
    _check(o[:sum(Ts)], _truth(qkv, P, bu, bv, Ts, Tmax), qkv, Ts)


def test_rel_attention_argument_errors(pkg):
    """Shapes the kernel does not take are refused before any device call."""
    L = pkg.lib()
    fake = 1 << 20   # 16-byte aligned, never dereferenced: every case fails its checks first
    T1 = (C.c_int * 1)(600)
    assert L.p2cu_rel_attention(fake, fake, fake, fake, T1, 1, 600, fake, fake, 1 << 20, None) == pkg.P2CU_EUNSUPPORTED
    T2 = (C.c_int * 2)(100, 120)
    assert L.p2cu_rel_attention(fake, fake, fake, fake, T2, 2, 110, fake, fake, 1 << 20, None) == pkg.P2CU_EINVAL
    assert L.p2cu_rel_attention(fake + 4, fake, fake, fake, T2, 2, 120, fake, fake, 1 << 20, None) == pkg.P2CU_EINVAL
    assert L.p2cu_rel_attention(fake, fake, fake, fake, T2, 2, 120, fake, fake, 8, None) == pkg.P2CU_EINVAL
    assert L.p2cu_rel_attention(None, fake, fake, fake, T2, 2, 120, fake, fake, 1 << 20, None) == pkg.P2CU_EINVAL
    T0 = (C.c_int * 1)(0)
    assert L.p2cu_rel_attention_ws_bytes(1, T0) == 0
    assert L.p2cu_rel_attention(fake, fake, fake, fake, T0, 1, 10, fake, fake, 1 << 20, None) == pkg.P2CU_EINVAL
    assert L.p2cu_rel_attention(fake, fake, fake, fake, T2, 0, 120, fake, fake, 0, None) == 0
