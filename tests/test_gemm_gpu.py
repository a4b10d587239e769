"""GPU parity: tcgen05 dot_general GEMM (bf16) and the exact f32 projection."""
import numpy as np
import pytest
import torch

from tests._util import from_np_bf16, rel_err, to_np_bf16

pytestmark = pytest.mark.gpu
TOL = 2e-2  # bf16 outputs, fp32 accumulate


def _inputs(orc, batch, M, N, K, b_nk=False, seed=42):
    a = orc.to_bf16(orc.uniform("gemm_a", (batch, M, K), seed=seed))
    b = orc.to_bf16(orc.uniform("gemm_b", (batch, N, K) if b_nk else (batch, K, N), seed=seed))
    return a, b


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (200, 296, 136), (1, 8, 8), (129, 264, 72),
                                   (256, 512, 1024), (384, 40, 520), (17, 1000, 16)])
def test_gemm_bf16_full_parity(rb, orc, M, N, K):
    a, b = _inputs(orc, 1, M, N, K)
    c = rb.gemm(from_np_bf16(a[0]), from_np_bf16(b[0]))
    ref_f, ref_b = orc.gemm_bf16_rows(a[0], b[0], 0, M)
    got = orc.bf16_to_f32(to_np_bf16(c))
    assert rel_err(got, ref_f) <= TOL
    # bf16 store of an fp32 sum: agree with the oracle's rounding almost everywhere
    assert np.mean(to_np_bf16(c) == ref_b) > 0.95


@pytest.mark.parametrize("layout", ["kn", "nk"])
def test_gemm_bf16_batched_layouts(rb, orc, layout):
    batch, M, N, K = 3, 130, 264, 200
    nk = layout == "nk"
    a, b = _inputs(orc, batch, M, N, K, b_nk=nk)
    c = rb.gemm(from_np_bf16(a), from_np_bf16(b), b_layout=rb.B_NK if nk else rb.B_KN)
    got = orc.bf16_to_f32(to_np_bf16(c))
    for i in range(batch):
        ref_f, _ = orc.gemm_bf16_rows(a[i], b[i], 0, M, b_kn=not nk)
        assert rel_err(got[i], ref_f) <= TOL


def test_gemm_bf16_strided_views(rb, orc):
    # leading dimensions larger than the logical extents
    a, b = _inputs(orc, 1, 192, 320, 256)
    A = torch.zeros(192, 264, dtype=torch.bfloat16, device="cuda")
    A[:, :256] = from_np_bf16(a[0])
    B = torch.zeros(256, 336, dtype=torch.bfloat16, device="cuda")
    B[:, :320] = from_np_bf16(b[0])
    C = torch.full((192, 328), 7.0, dtype=torch.bfloat16, device="cuda")
    rb.gemm(A[:, :256], B[:, :320], out=C[:, :320])
    ref_f, _ = orc.gemm_bf16_rows(a[0], b[0], 0, 192)
    got = orc.bf16_to_f32(to_np_bf16(C))
    assert rel_err(got[:, :320], ref_f) <= TOL
    assert np.all(got[:, 320:] == 7.0)  # nothing written outside C's extent


def test_gemm_bf16_1024_sampled_and_deterministic(rb, orc):
    M = N = K = 1024
    a, b = _inputs(orc, 1, M, N, K)
    A, B = from_np_bf16(a[0]), from_np_bf16(b[0])
    c1 = rb.gemm(A, B)
    c2 = rb.gemm(A, B)
    assert torch.equal(c1.view(torch.int16), c2.view(torch.int16))
    rng = np.random.default_rng(0)
    ii, jj = rng.integers(0, M, 4096), rng.integers(0, N, 4096)
    ref = orc.gemm_bf16_samples(a[0], b[0], ii, jj)
    got = orc.bf16_to_f32(to_np_bf16(c1))[ii, jj]
    assert rel_err(got, ref) <= TOL
    # secondary check against torch fp32
    t = (A.float() @ B.float()).cpu().numpy()
    assert rel_err(orc.bf16_to_f32(to_np_bf16(c1)), t) <= TOL


def test_gemm_k_zero_gives_zeros(rb):
    A = torch.empty(64, 0, dtype=torch.bfloat16, device="cuda")
    B = torch.empty(0, 64, dtype=torch.bfloat16, device="cuda")
    C = torch.full((64, 64), 3.0, dtype=torch.bfloat16, device="cuda")
    rb.gemm(A, B, out=C)
    assert torch.all(C == 0)


def test_gemm_rejects_misaligned(rb):
    A = torch.zeros(64, 36, dtype=torch.bfloat16, device="cuda")
    B = torch.zeros(36, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(rb.RemoraError) as e:
        rb.gemm(A[:, :30], B[:30])  # K = 30 is not a multiple of 8
    assert e.value.code == rb.ERR_INVALID
    B2 = torch.zeros(32, 300, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(rb.RemoraError):
        rb.gemm(A[:, :32], B2)  # N = 300 breaks the 16-byte row rule of TMA


def test_run_test_gemm_full_size(rb):
    rep = rb.run_test("gemm", iters=2, warmup=1)  # 8192^3, 4096 sampled outputs
    assert rep["passed"] and rep["checked"] == 4096 and rep["max_rel_err"] <= TOL


def test_run_test_gemm_batched(rb):
    rep = rb.run_test("gemm", config="batched", iters=2, warmup=1)
    assert rep["passed"] and rep["checked"] == 4096


@pytest.mark.parametrize("M,N,K", [(512, 768, 768), (37, 53, 101)])
def test_gemm_f32_exact_bit_identical(rb, orc, M, N, K):
    a = orc.normal("x", (M, K))
    b = orc.normal("bias", (K, N))
    ref = orc.gemm_f32(a, b)
    got = rb.gemm_f32_exact(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_run_test_projection_known_answer(rb):
    rep = rb.run_test("projection")
    assert rep["passed"] and rep["max_abs_err"] == 0.0
