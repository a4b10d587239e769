"""GPU parity: the elementwise attention epilogue against the oracle."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_run_test_elementwise_known_answer(rb):
    rep = rb.run_test("elementwise", iters=3, warmup=1)
    assert rep["passed"] and rep["checked"] == 512 * 768 and rep["max_abs_err"] == 0.0


@pytest.mark.parametrize("rows,d", [(512, 768), (33, 7), (1, 4), (0, 768), (1000, 6)])
def test_relu_bias_bit_exact(rb, orc, rows, d):
    x = orc.normal("x", (rows, d))
    b = orc.normal("bias", (d,))
    ref = orc.relu_bias(x, b)
    out = rb.relu_bias(torch.from_numpy(x).cuda(), torch.from_numpy(b).cuda())
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_relu_bias_special_values(rb, orc):
    x = np.array([[np.nan, -1.0, -0.0, 2.0, np.inf, -np.inf, 1e-45, -1e-45]], np.float32)
    b = np.zeros(8, np.float32)
    ref = orc.relu_bias(x, b)
    out = rb.relu_bias(torch.from_numpy(x).cuda(), torch.from_numpy(b).cuda()).cpu().numpy()
    assert np.array_equal(np.isnan(out), np.isnan(ref))
    m = ~np.isnan(ref)
    assert np.array_equal(out[m].view(np.uint32), ref[m].view(np.uint32))


@pytest.mark.parametrize("n", [8 * 128 * 128, 1, 4099, 1 << 20])
def test_scale_add_exp_parity(rb, orc, n):
    s = orc.normal("scores", (n,))
    b = orc.normal("bias", (n,))
    ref = orc.scale_add_exp(s, b, 0.125)
    out = rb.scale_add_exp(torch.from_numpy(s).cuda(), torch.from_numpy(b).cuda(), 0.125)
    got = out.cpu().numpy()
    assert np.max(np.abs(got - ref) / np.abs(ref)) <= 1e-5  # f32 elementwise tolerance: 1e-5 relative


def test_scale_add_exp_unaligned_views(rb, orc):
    s = torch.from_numpy(orc.normal("scores", (1027,))).cuda()
    b = torch.from_numpy(orc.normal("bias", (1027,))).cuda()
    out = torch.empty(1030, device="cuda")
    rb.scale_add_exp(s[1:], b[1:], 0.125, out=out[2:1028])
    ref = orc.scale_add_exp(s[1:].cpu().numpy(), b[1:].cpu().numpy(), 0.125)
    got = out[2:1028].cpu().numpy()
    assert np.max(np.abs(got - ref) / np.abs(ref)) <= 1e-5


def test_run_test_chain_config(rb):
    rep = rb.run_test("elementwise_chain", iters=5, warmup=2)
    assert rep["passed"] and rep["checked"] == 8 * 128 * 128 and rep["max_rel_err"] <= 1e-5


def test_fill_matches_oracle_generator(rb, orc):
    key = orc.stream_key("moe_x")
    t = torch.empty(100_000, device="cuda")
    rb.fill_normal(t, key)
    ref = orc.normal("moe_x", (100_000,))
    got = t.cpu().numpy()
    # double-precision log/cos may differ in the last bit between libm and
    # CUDA; after rounding to f32 the draws agree to within 1 ulp
    assert np.max(np.abs(got - ref)) <= 2.5e-7 * np.max(np.abs(ref))
    tb = torch.empty(100_000, dtype=torch.bfloat16, device="cuda")
    rb.fill_uniform(tb, orc.stream_key("gemm_a"))
    refb = orc.to_bf16(orc.uniform("gemm_a", (100_000,)))
    from tests._util import to_np_bf16

    assert np.mean(to_np_bf16(tb) == refb) > 0.999
