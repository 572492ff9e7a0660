"""Parity of the sm_100a GEMMs with the CPU oracle, through the device C ABI (include/p2cuda.h).

int8 / int8w: the int32 sums are compared directly (exposed through the epilogue with unit scales) and the fp32
outputs bit for bit against the restatement, which runs the reference's epilogue in the reference's order.
exact: bit for bit against the restatement, which is itself bit for bit the reference library (tests/test_oracle.py).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# (M, K, N, alpha, beta): config 0, the block's shapes at T = 375 (the positional projection at 2T - 1 rows),
# the short-utterance regime (T = 38) and ragged edges.
SHAPES = [
    (375, 1024, 4096, 1.0, 0.0),
    (375, 4096, 1024, 0.5, 1.0),
    (375, 1024, 3072, 1.0, 0.0),
    (749, 1024, 1024, 1.0, 0.0),
    (375, 1024, 1024, 1.0, 1.0),
    (375, 1024, 2048, 1.0, 0.0),
    (38, 1024, 4096, 1.0, 0.0),
    (1, 1024, 128, 1.0, 0.0),
    (129, 2048, 256, 1.0, 1.0),
    (200, 1040, 384, 1.0, 0.0),     # K not a multiple of 128: the last stage reads zero-filled rows
    (64, 4096, 128, 0.5, 0.5),      # beta outside {0, 1}: C scaled first
]


def _run_fvb(pkg, torch, cuda, w, A, mode, alpha, beta, C0, codes=False):
    from phonon2_b200.device import DeviceFiveValue
    M, K = A.shape
    N = w["N"]
    B = DeviceFiveValue(w, cuda, codes=codes)
    A_d = torch.from_numpy(A).to(cuda)
    C_d = torch.from_numpy(C0.copy()).to(cuda)
    nws = max(pkg.workspace_bytes(M, N, K, mode), 16)
    ws = torch.empty(nws, dtype=torch.uint8, device=cuda)
    pkg.sgemm_fvb(M, N, K, alpha, A_d.data_ptr(), K, B.struct, mode, beta, C_d.data_ptr(), N, ws.data_ptr(), nws)
    pkg.check_device()
    return C_d.cpu().numpy()


def _bits_equal(a, b):
    return np.array_equal(np.ascontiguousarray(a).view(np.uint32), np.ascontiguousarray(b).view(np.uint32))


def _report(got, want):
    bad = np.argwhere(got.view(np.uint32) != want.view(np.uint32))
    if len(bad) == 0:
        return "equal"
    i = tuple(bad[0])
    return f"{len(bad)} of {got.size} differ; first {i}: got {got[i]!r} want {want[i]!r}"


@pytest.mark.parametrize("mode", ["int8w", "int8"])
@pytest.mark.parametrize("M,K,N,alpha,beta", SHAPES)
def test_five_value_int8_modes_bitwise(pkg, orc, synth, cuda, mode, M, K, N, alpha, beta):
    import torch
    w = synth.five_value(K, N, seed=M + K + N)
    A = synth.activations(M, K, seed=M * 3 + 1)
    C0 = np.random.default_rng(7).standard_normal((M, N)).astype(np.float32)
    got = _run_fvb(pkg, torch, cuda, w, A, pkg.MODES[mode], alpha, beta, C0)
    want = orc.sgemm_i8(A, mode, C0.copy(), w=w, alpha=alpha, beta=beta)
    assert _bits_equal(got, want), _report(got, want)


@pytest.mark.parametrize("M,K,N,alpha,beta", SHAPES[:2] + SHAPES[6:9])
def test_five_value_exact_bitwise(pkg, orc, synth, cuda, M, K, N, alpha, beta):
    import torch
    w = synth.five_value(K, N, seed=M + 2 * K + N)
    A = synth.activations(M, K, seed=M * 5 + 2)
    C0 = np.random.default_rng(8).standard_normal((M, N)).astype(np.float32)
    got = _run_fvb(pkg, torch, cuda, w, A, pkg.EXACT, alpha, beta, C0)
    want = orc.gemm_exact(A, C0.copy(), w=w, alpha=alpha, beta=beta)
    assert _bits_equal(got, want), _report(got, want)


@pytest.mark.parametrize("K", [1024, 4096, 640])
def test_int32_accumulators_bitwise(pkg, orc, synth, cuda, K):
    """The int32 sums, read through the int8 epilogue with unit row scales: lo = hi = 1 gives f = accS exactly,
    lo = 0, hi = 1 gives f = accT exactly (all sums are below 2^24, so the conversions are exact)."""
    import torch
    from phonon2_b200.device import DeviceFiveValue
    M, N = 300, 256
    w = synth.five_value(K, N, seed=K + 1)
    q, _ = orc.quant_rows(synth.activations(M, K, seed=4))
    accS, accT = orc.acc_blocks(q, "int8", w=w)
    q_d = torch.from_numpy(q).to(cuda)
    ones = torch.ones(M, dtype=torch.float32, device=cuda)
    for plane, (lo, hi), want_blocks in (("S", (1.0, 1.0), accS), ("T", (0.0, 1.0), accT)):
        ww = dict(w, lo=np.full(N, lo, np.float32), hi=np.full(N, hi, np.float32))
        B = DeviceFiveValue(ww, cuda)
        C_d = torch.zeros((M, N), dtype=torch.float32, device=cuda)
        nws = max(pkg.q8a_workspace_bytes(M, N, K), 16)
        ws = torch.empty(nws, dtype=torch.uint8, device=cuda)
        pkg.sgemm_fvb_q8a(M, N, K, 1.0, q_d.data_ptr(), ones.data_ptr(), B.struct, pkg.INT8, 0.0, C_d.data_ptr(), N,
                          ws.data_ptr(), nws)
        pkg.check_device()
        got = C_d.cpu().numpy().astype(np.int64)
        want = want_blocks.astype(np.int64).sum(axis=0)   # blocks summed in fp32 exactly (integers below 2^24)
        assert np.array_equal(got, want), f"plane {plane}: {np.count_nonzero(got != want)} sums differ"


@pytest.mark.parametrize("M,K,N", [(375, 1024, 4096), (38, 4096, 1024), (130, 1024, 384)])
def test_cached_codes_equal_planes(pkg, orc, synth, cuda, M, K, N):
    """int8w from pre-expanded codes (one MMA plane, the code cache) equals int8w from the planes, bit for bit."""
    import torch
    from phonon2_b200.device import DeviceFiveValue
    w = synth.five_value(K, N, seed=3)
    B = DeviceFiveValue(w, cuda, codes=True)
    torch.cuda.synchronize()
    assert np.array_equal(B.codes.cpu().numpy(), orc.fv_codes(w))
    A = synth.activations(M, K, seed=5)
    got = _run_fvb(pkg, torch, cuda, w, A, pkg.INT8W, 1.0, 0.0, np.zeros((M, N), np.float32), codes=True)
    want = orc.sgemm_i8(A, "int8w", np.zeros((M, N), np.float32), w=w)
    assert _bits_equal(got, want), _report(got, want)


@pytest.mark.parametrize("mode", ["int8", "exact"])
@pytest.mark.parametrize("M,K,N", [(375, 4096, 1024), (375, 1024, 640), (3, 4096, 1024)])
def test_int8_table_bitwise(pkg, orc, synth, cuda, mode, M, K, N):
    """The int8-table weights (subsampling.linear 4096 -> 1024, the projector 1024 -> 640)."""
    import torch
    t = synth.int8_table(K, N, seed=6)
    A = synth.activations(M, K, seed=7)
    A_d = torch.from_numpy(A).to(cuda)
    B_d = torch.from_numpy(t["q8"]).to(cuda)
    s_d = torch.from_numpy(t["scales"]).to(cuda)
    C_d = torch.zeros((M, N), dtype=torch.float32, device=cuda)
    m = pkg.MODES[mode]
    nws = max(pkg.workspace_bytes(M, N, K, m), 16)
    ws = torch.empty(nws, dtype=torch.uint8, device=cuda)
    pkg.sgemm_q8b(M, N, K, 1.0, A_d.data_ptr(), K, B_d.data_ptr(), s_d.data_ptr(), N, m, 0.0, C_d.data_ptr(), N,
                  ws.data_ptr(), nws)
    pkg.check_device()
    got = C_d.cpu().numpy()
    if mode == "exact":
        want = orc.gemm_exact(A, np.zeros((M, N), np.float32), q8=t)
    else:
        want = orc.sgemm_i8(A, "q8b", np.zeros((M, N), np.float32), q8=t)
    assert _bits_equal(got, want), _report(got, want)


@pytest.mark.parametrize("M,K", [(1, 16), (375, 1024), (749, 4096), (33, 1000)])
def test_quantiser_bitwise(pkg, orc, cuda, M, K):
    import torch
    rng = np.random.default_rng(M)
    A = (rng.standard_normal((M, K)) * rng.uniform(0.001, 50, (M, 1))).astype(np.float32)
    A[0, : min(4, K)] = 0.0
    A_d = torch.from_numpy(A).to(cuda)
    q_d = torch.empty((M, K), dtype=torch.int8, device=cuda)
    s_d = torch.empty(M, dtype=torch.float32, device=cuda)
    pkg.quant_rows(A_d.data_ptr(), M, K, K, q_d.data_ptr(), s_d.data_ptr())
    pkg.check_device()
    q, s = orc.quant_rows(A)
    assert np.array_equal(q_d.cpu().numpy(), q)
    assert _bits_equal(s_d.cpu().numpy(), s)


@pytest.mark.parametrize("K", [20, 1000, 1002, 1024, 4100])
def test_quantiser_edge_rows_bitwise(pkg, orc, synth, cuda, K):
    """Rows at the quantiser's edges (synth.quantiser_edge_rows): values whose reciprocal and division roundings
    differ, in the 16-wide body and in the K % 16 tail that the reference divides (csrc/blas.c:1139-1143); a row whose
    1 / scale overflows (the conversion saturates, NaN gives 0); zeros; ties. The register path (K % 4 == 0,
    K <= 4096) and the strided path (K = 1002, 4100)."""
    import torch
    A = np.concatenate([synth.quantiser_edge_rows(K, seed=K), synth.activations(9, K, seed=K + 1)])
    M = A.shape[0]
    A_d = torch.from_numpy(A).to(cuda)
    q_d = torch.empty((M, K), dtype=torch.int8, device=cuda)
    s_d = torch.empty(M, dtype=torch.float32, device=cuda)
    pkg.quant_rows(A_d.data_ptr(), M, K, K, q_d.data_ptr(), s_d.data_ptr())
    pkg.check_device()
    q, s = orc.quant_rows(A)
    assert np.array_equal(q_d.cpu().numpy(), q)
    assert _bits_equal(s_d.cpu().numpy(), s)


# Shapes the reference's int8 path takes but the tensor-core kernels do not (N % 128 != 0, K % 16 != 0): the SIMT
# kernel, bit for bit.
RAGGED = [(13, 1028, 48, 1.0, 0.0), (77, 2056, 144, 0.5, 1.0), (130, 1024, 80, 1.0, 0.5), (3, 100, 16, 1.0, 0.0),
          (40, 1000, 256, 1.0, 1.0)]


@pytest.mark.parametrize("mode", ["int8w", "int8"])
@pytest.mark.parametrize("M,K,N,alpha,beta", RAGGED)
def test_ragged_shapes_bitwise(pkg, orc, synth, cuda, mode, M, K, N, alpha, beta):
    import torch
    w = synth.five_value(K, N, seed=M + K + N)
    A = np.concatenate([synth.quantiser_edge_rows(K, seed=K)[:M], synth.activations(max(M - 8, 0), K, seed=M)])[:M]
    C0 = np.random.default_rng(9).standard_normal((M, N)).astype(np.float32)
    got = _run_fvb(pkg, torch, cuda, w, A, pkg.MODES[mode], alpha, beta, C0)
    want = orc.sgemm_i8(A, mode, C0.copy(), w=w, alpha=alpha, beta=beta)
    assert _bits_equal(got, want), _report(got, want)
    if mode == "int8w":   # from the code cache
        got = _run_fvb(pkg, torch, cuda, w, A, pkg.INT8W, alpha, beta, C0, codes=True)
        assert _bits_equal(got, want), _report(got, want)


@pytest.mark.parametrize("M,K,N", [(13, 1028, 48), (33, 1000, 640)])
def test_ragged_int8_table_bitwise(pkg, orc, synth, cuda, M, K, N):
    import torch
    t = synth.int8_table(K, N, seed=3)
    A = synth.activations(M, K, seed=4)
    A_d = torch.from_numpy(A).to(cuda)
    B_d = torch.from_numpy(t["q8"]).to(cuda)
    s_d = torch.from_numpy(t["scales"]).to(cuda)
    C_d = torch.zeros((M, N), dtype=torch.float32, device=cuda)
    nws = max(pkg.workspace_bytes(M, N, K, pkg.INT8), 16)
    ws = torch.empty(nws, dtype=torch.uint8, device=cuda)
    pkg.sgemm_q8b(M, N, K, 1.0, A_d.data_ptr(), K, B_d.data_ptr(), s_d.data_ptr(), N, pkg.INT8, 0.0, C_d.data_ptr(),
                  N, ws.data_ptr(), nws)
    pkg.check_device()
    want = orc.sgemm_i8(A, "q8b", np.zeros((M, N), np.float32), q8=t)
    assert _bits_equal(C_d.cpu().numpy(), want), _report(C_d.cpu().numpy(), want)


@pytest.mark.parametrize("mode", ["int8w", "int8"])
def test_k_not_whole_quads_takes_the_exact_path(pkg, orc, synth, cuda, mode):
    """The reference quantises only rows of whole quads: with K % 4 != 0 its p2_sgemm_fvb runs the exact path
    (csrc/blas.c:1490-1498), and so does this one."""
    import torch
    M, K, N = 21, 1022, 128
    w = synth.five_value(K, N, seed=5)
    A = synth.activations(M, K, seed=6)
    C0 = np.random.default_rng(7).standard_normal((M, N)).astype(np.float32)
    got = _run_fvb(pkg, torch, cuda, w, A, pkg.MODES[mode], 1.0, 0.5, C0)
    want = orc.gemm_exact(A, C0.copy(), w=w, alpha=1.0, beta=0.5)
    assert _bits_equal(got, want), _report(got, want)


@pytest.mark.parametrize("tA,tB", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(375, 375, 128), (48, 749, 128), (100, 128, 375), (5, 7, 3)])
def test_fp32_sgemm(pkg, orc, cuda, tA, tB, M, N, K):
    """p2_sgemm on the device: NN bit for bit the reference (one FMA chain per output); the transposed forms run one
    chain per output too, against the reference's lane-split reductions within 1e-5 relative."""
    import torch
    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((K, M) if tA else (M, K)).astype(np.float32)
    B = rng.standard_normal((N, K) if tB else (K, N)).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    A_d, B_d = torch.from_numpy(A).to(cuda), torch.from_numpy(B).to(cuda)
    C_d = torch.from_numpy(C0.copy()).to(cuda)
    pkg.sgemm(tA, tB, M, N, K, 0.5, A_d.data_ptr(), A.shape[1], B_d.data_ptr(), B.shape[1], 1.0, C_d.data_ptr(), N)
    pkg.check_device()
    got = C_d.cpu().numpy()
    want = orc.ref_sgemm(tA, tB, A, B, C0.copy(), alpha=0.5, beta=1.0) if orc.ref_available() else None
    ref64 = 0.5 * ((A.T if tA else A).astype(np.float64) @ (B.T if tB else B).astype(np.float64)) + C0
    scale = 0.5 * (np.abs(A.T if tA else A).astype(np.float64) @ np.abs(B.T if tB else B)) + np.abs(C0)
    assert (np.abs(got - ref64) / scale).max() < 1e-5
    if want is not None and tA == 0 and tB == 0 and N % 16 == 0:
        assert _bits_equal(got, want), _report(got, want)


def test_contract_errors(pkg, orc, synth, cuda):
    import torch
    from phonon2_b200.device import DeviceFiveValue
    w = synth.five_value(256, 144, seed=1)                  # N % 16 == 0 but not % 128: no tensor-core tile
    B = DeviceFiveValue(w, cuda)
    A = synth.activations(8, 256, seed=2)
    A_d = torch.from_numpy(A).to(cuda)
    C_d = torch.zeros((8, 144), device=cuda)
    ws = torch.empty(1 << 16, dtype=torch.uint8, device=cuda)
    # the reference takes this shape, and so does the SIMT kernel
    pkg.sgemm_fvb(8, 144, 256, 1.0, A_d.data_ptr(), 256, B.struct, pkg.INT8W, 0.0, C_d.data_ptr(), 144,
                  ws.data_ptr(), ws.numel())
    pkg.check_device()
    assert _bits_equal(C_d.cpu().numpy(), orc.sgemm_i8(A, "int8w", np.zeros((8, 144), np.float32), w=w))
    with pytest.raises(pkg.Error) as e:                     # N not a multiple of 16, as the reference refuses it
        pkg.sgemm_fvb(8, 136, 256, 1.0, A_d.data_ptr(), 256, B.struct, pkg.INT8W, 0.0, C_d.data_ptr(), 144,
                      ws.data_ptr(), ws.numel())
    assert e.value.code == pkg.P2CU_EINVAL
    with pytest.raises(pkg.Error) as e:                     # workspace too small
        pkg.sgemm_fvb(8, 144, 256, 1.0, A_d.data_ptr(), 256, B.struct, pkg.INT8W, 0.0, C_d.data_ptr(), 144,
                      ws.data_ptr(), 10)
    assert e.value.code == pkg.P2CU_EINVAL
    with pytest.raises(pkg.Error) as e:                     # weight shape disagrees with the call
        pkg.sgemm_fvb(8, 144, 128, 1.0, A_d.data_ptr(), 256, B.struct, pkg.EXACT, 0.0, C_d.data_ptr(), 144,
                      ws.data_ptr(), ws.numel())
    assert e.value.code == pkg.P2CU_EINVAL
    pkg.check_device()


TILE_CHILD = r"""
import json, sys
import numpy as np
sys.path.insert(0, {root!r})
import __graft_entry__ as ge
import torch
pkg, orc = ge.load_package(), ge.load_oracle()
from phonon2_b200 import synth
from phonon2_b200.device import DeviceFiveValue
dev = torch.device("cuda:0")
res = []
for (M, K, N, mode, beta, codes) in [(375, 1024, 1024, "int8w", 1.0, False), (300, 2048, 512, "int8", 0.0, False),
                                     (130, 1024, 768, "int8w", 0.0, True), (375, 1024, 512, "int8", 1.0, False)]:
    w = synth.five_value(K, N, seed=M + N)
    A = synth.activations(M, K, seed=K)
    C0 = np.random.default_rng(1).standard_normal((M, N)).astype(np.float32)
    B = DeviceFiveValue(w, dev, codes=codes)
    A_d, C_d = torch.from_numpy(A).to(dev), torch.from_numpy(C0.copy()).to(dev)
    m = pkg.MODES[mode]
    nws = max(pkg.workspace_bytes(M, N, K, m), 16)
    ws = torch.empty(nws, dtype=torch.uint8, device=dev)
    pkg.sgemm_fvb(M, N, K, 1.0, A_d.data_ptr(), K, B.struct, m, beta, C_d.data_ptr(), N, ws.data_ptr(), nws)
    pkg.check_device()
    got = C_d.cpu().numpy()
    want = orc.sgemm_i8(A, mode, C0.copy(), w=w, beta=beta)
    res.append(bool(np.array_equal(got.view(np.uint32), want.view(np.uint32))))
print(json.dumps(res))
"""


@pytest.mark.parametrize("tile", ["64", "128", "256"])
def test_every_tile_width_bitwise(cuda, tile):
    """The same GEMMs with each tile width forced (P2CU_TILE_N, read once per process: a child each)."""
    import json
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = str(Path(__file__).resolve().parents[1])
    env = dict(os.environ, P2CU_TILE_N=tile)
    out = subprocess.run([sys.executable, "-c", TILE_CHILD.format(root=root)], env=env, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr[-3000:]
    assert json.loads(out.stdout.strip().splitlines()[-1]) == [True] * 4


PERSIST_CHILD = r"""
import json, sys
import numpy as np
sys.path.insert(0, {root!r})
import __graft_entry__ as ge
import torch
pkg, orc = ge.load_package(), ge.load_oracle()
from phonon2_b200 import synth
from phonon2_b200.device import DeviceFiveValue
dev = torch.device("cuda:0")
res = []
cases = [(2500, 1024, 4096, "int8w", 1.0, 0.0, False), (2500, 4096, 1024, "int8w", 0.5, 1.0, False),
         (1300, 1024, 2048, "int8", 1.0, 1.0, False), (2500, 1024, 3072, "int8w", 1.0, 0.0, True),
         (640, 2048, 1024, "int8", 1.0, 0.0, False), (375, 1024, 1024, "int8w", 1.0, 1.0, False)]
for (M, K, N, mode, alpha, beta, codes) in cases:
    w = synth.five_value(K, N, seed=M + N)
    A = synth.activations(M, K, seed=K)
    C0 = np.random.default_rng(1).standard_normal((M, N)).astype(np.float32)
    B = DeviceFiveValue(w, dev, codes=codes)
    A_d, C_d = torch.from_numpy(A).to(dev), torch.from_numpy(C0.copy()).to(dev)
    m = pkg.MODES[mode]
    nws = max(pkg.workspace_bytes(M, N, K, m), 16)
    ws = torch.empty(nws, dtype=torch.uint8, device=dev)
    pkg.sgemm_fvb(M, N, K, alpha, A_d.data_ptr(), K, B.struct, m, beta, C_d.data_ptr(), N, ws.data_ptr(), nws)
    pkg.check_device()
    want = orc.sgemm_i8(A, mode, C0.copy(), w=w, alpha=alpha, beta=beta)
    res.append(bool(np.array_equal(C_d.cpu().numpy().view(np.uint32), want.view(np.uint32))))
# an int8 table (q8b) through the same kernel
M, K, N = 2000, 4096, 1024
t = synth.int8_table(K, N, seed=3)
A = synth.activations(M, K, seed=4)
A_d = torch.from_numpy(A).to(dev)
C_d = torch.zeros((M, N), dtype=torch.float32, device=dev)
q8, sc = torch.from_numpy(t["q8"]).to(dev), torch.from_numpy(t["scales"]).to(dev)
nws = pkg.workspace_bytes(M, N, K, pkg.INT8)
ws = torch.empty(nws, dtype=torch.uint8, device=dev)
pkg.sgemm_q8b(M, N, K, 1.0, A_d.data_ptr(), K, q8.data_ptr(), sc.data_ptr(), N, pkg.INT8, 0.0, C_d.data_ptr(), N,
              ws.data_ptr(), nws)
pkg.check_device()
want = orc.sgemm_i8(A, "q8b", np.zeros((M, N), np.float32), q8=t)
res.append(bool(np.array_equal(C_d.cpu().numpy().view(np.uint32), want.view(np.uint32))))
print(json.dumps(res))
"""


@pytest.mark.parametrize("persist,tile,pair", [("1", "128", ""), ("1", "256", ""), ("1", "64", ""), ("", "", ""),
                                               ("", "", "1")])
def test_persistent_kernel_bitwise(cuda, persist, tile, pair):
    """The persistent GEMM (many tiles; forced with P2CU_PERSIST=1 for every shape, including few-tile ones, or chosen
    by tile count) and the CTA-pair GEMM (P2CU_PAIR=1: every int8w / int8-table shape with N % 256 == 0, including
    M = 375, whose last pair tile has no rows in its odd CTA) against the restatement, bit for bit: every mode,
    beta 0 / 1 / alpha 1/2, K > 1024 through the workspace slices, the code cache and an int8 table."""
    import json
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = str(Path(__file__).resolve().parents[1])
    env = dict(os.environ)
    env.pop("P2CU_PERSIST", None)
    env.pop("P2CU_TILE_N", None)
    env.pop("P2CU_PAIR", None)
    if pair:
        env["P2CU_PAIR"] = pair
    if persist:
        env["P2CU_PERSIST"] = persist
    if tile:
        env["P2CU_TILE_N"] = tile
    out = subprocess.run([sys.executable, "-c", PERSIST_CHILD.format(root=root)], env=env, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-3000:]
    assert json.loads(out.stdout.strip().splitlines()[-1]) == [True] * 7


def test_device_wait_timeout_is_reported_and_the_context_survives(pkg, orc, synth, cuda):
    """Failure detection without a fault: a kernel waits, through the GEMM kernels' own bounded wait, on a barrier
    that nothing completes; the wait gives up after 4096 polls, the kernel records code 1 (DEV_TIMEOUT_FULL) in the
    device error word and returns; p2cu_check_device reports it as P2CU_EDEVICE and clears the word; the next GEMM on
    the same context is still bit for bit the oracle's."""
    import ctypes as C
    import torch
    secs = C.c_double()
    rc = pkg.lib().p2cu_probe_wait_timeout(4096, C.byref(secs))
    assert rc == pkg.P2CU_EDEVICE, pkg.last_error()
    assert "device error code 1" in pkg.last_error()
    assert 0.0 < secs.value < 2.0
    pkg.check_device()   # cleared
    M, K, N = 77, 1024, 256
    w = synth.five_value(K, N, seed=1)
    A = synth.activations(M, K, seed=2)
    got = _run_fvb(pkg, torch, cuda, w, A, pkg.INT8W, 1.0, 0.0, np.zeros((M, N), np.float32))
    assert _bits_equal(got, orc.sgemm_i8(A, "int8w", np.zeros((M, N), np.float32), w=w))
