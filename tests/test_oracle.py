"""CPU tests of the oracle: generator, known answers, golden vectors."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_generator_c_matches_numpy(orc):
    for name in ("x", "gemm_a", "moe_wd"):
        key = orc.stream_key(name)
        assert np.array_equal(orc.normal(name, (5000,)), orc.normal_np(key, 5000))
        assert np.array_equal(orc.uniform(name, (5000,)), orc.uniform_np(key, 5000, -1.0, 1.0))


def test_generator_distribution(orc):
    z = orc.normal("scores", (1 << 18,))
    assert abs(float(z.mean())) < 0.01 and abs(float(z.std()) - 1.0) < 0.01
    u = orc.uniform("gemm_a", (1 << 18,))
    assert u.min() >= -1.0 and u.max() <= 1.0 and abs(float(u.mean())) < 0.01


def test_bf16_rounding_rne(orc):
    f = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, 1e-40, np.inf, -0.0], np.float32)
    b = orc.to_bf16(f)
    # 1 + 2^-8 is a tie -> even (1.0); 1 + 3*2^-8 is a tie -> up (1 + 2^-6).
    assert b[0] == 0x3F80 and b[1] == 0x3F80 and b[2] == 0x3F82
    assert orc.bf16_to_f32(b)[3] == -2.5
    assert b[6] == 0x7F80 and b[7] == 0x8000
    nan = orc.to_bf16(np.array([np.nan], np.float32))
    assert np.isnan(orc.bf16_to_f32(nan)[0])


def test_known_answer_elementwise(orc):
    """x = 1, bias = -0.5 -> 0.5 (compiler/gpu_tests.cpp:53-56, cpu_tests.cpp:26-58)."""
    ka = np.load(os.path.join(GOLDEN, "known_answers.npz"))
    x = np.ones((1, 512, 768), np.float32)
    out = orc.relu_bias(x, np.full(768, -0.5, np.float32))
    assert np.all(out == ka["elementwise"])


def test_relu_bias_maximumf_semantics(orc):
    x = np.array([[np.nan, -1.0, -0.0, 2.0]], np.float32)
    out = orc.relu_bias(x, np.zeros(4, np.float32))
    assert np.isnan(out[0, 0]) and out[0, 1] == 0.0 and out[0, 3] == 2.0
    assert out[0, 2] == 0.0 and not np.signbit(out[0, 2])


def test_known_answer_projection(orc):
    """x = 1, w = 1/768 -> fl(sum) (cpu_tests.cpp:65-97 prints it as 1.0)."""
    ka = np.load(os.path.join(GOLDEN, "known_answers.npz"))
    out = orc.gemm_f32(np.ones((512, 768), np.float32), np.full((768, 768), 1 / 768, np.float32))
    assert np.all(out == ka["projection"])
    assert abs(float(ka["projection"]) - 1.0) < 1e-5


def test_moe_mini_against_numpy_reference(orc):
    """The reference's MoE check: seed-42 mini dims, atol 1e-4
    (scripts/export/export_mixtral_layer.py:154-235)."""
    z = np.load(os.path.join(GOLDEN, "moe_mini_seed42.npz"))
    idx, w = orc.router_topk(z["tokens"], z["router"], 2)
    assert np.array_equal(idx, z["idx"])
    np.testing.assert_allclose(w, z["w"], atol=1e-6)
    out = orc.moe_f32(z["tokens"], z["router"], z["w_gate"], z["w_up"], z["w_down"], 2)
    assert np.abs(out - z["out"]).max() < 1e-4


def test_oracle_small_regression(orc):
    z = np.load(os.path.join(GOLDEN, "oracle_small.npz"))
    idx, w, lg = orc.router_topk(z["moe_x"], z["moe_wr"], 2, return_logits=True)
    assert np.array_equal(idx, z["idx"]) and np.array_equal(lg, z["logits"])
    assert np.array_equal(w, z["w"])
    counts, offsets, perm, inv = orc.dispatch(idx, 8)
    for a, n in ((counts, "counts"), (offsets, "offsets"), (perm, "perm"), (inv, "inv")):
        assert np.array_equal(a, z[n]), n
    gf, gb = orc.gemm_bf16_rows(z["gemm_a"], z["gemm_b"], 0, 40)
    assert np.array_equal(gf, z["gemm_f32"]) and np.array_equal(gb, z["gemm_bf16"])
    att = orc.attention_rows(z["attn_q"], z["attn_k"], z["attn_v"], np.arange(80))
    assert np.array_equal(att, z["attn_out"])
    *_, out = orc.moe_layer_bf16(z["moe_x"], z["moe_wr"], z["moe_wg"], z["moe_wu"], z["moe_wd"], 2)
    assert np.array_equal(out, z["moe_out"])


def test_gemm_bf16_matches_float64(orc):
    a = orc.to_bf16(orc.uniform("gemm_a", (33, 200)))
    b = orc.to_bf16(orc.uniform("gemm_b", (200, 45)))
    ref = orc.bf16_to_f32(a).astype(np.float64) @ orc.bf16_to_f32(b).astype(np.float64)
    gf, gb = orc.gemm_bf16_rows(a, b, 0, 33)
    assert np.abs(gf - ref).max() < 1e-4
    bt = np.ascontiguousarray(b.T)
    gf2, _ = orc.gemm_bf16_rows(a, bt, 0, 33, b_kn=False)
    assert np.array_equal(gf, gf2)
    s = orc.gemm_bf16_samples(a, b, np.array([0, 5, 32]), np.array([0, 44, 7]))
    assert np.array_equal(s, gf[[0, 5, 32], [0, 44, 7]])


def test_attention_matches_dense_float64(orc):
    S, Dh = 50, 32
    q = orc.to_bf16(orc.normal("attn_q", (S, Dh)))
    k = orc.to_bf16(orc.normal("attn_k", (S, Dh)))
    v = orc.to_bf16(orc.normal("attn_v", (S, Dh)))
    qf, kf, vf = (orc.bf16_to_f32(t).astype(np.float64) for t in (q, k, v))
    s = qf @ kf.T / np.sqrt(Dh)
    s[np.triu_indices(S, 1)] = -np.inf
    p = np.exp(s - s.max(1, keepdims=True))
    ref = (p / p.sum(1, keepdims=True)) @ vf
    out = orc.attention_rows(q, k, v, np.arange(S), causal=True)
    assert np.abs(out - ref).max() < 1e-5


def test_topk_tie_and_nan_rules(orc):
    # ties -> lower index; NaN ranks above every number
    x = np.array([[1.0]], np.float32)  # D = 1, so the logits are wr's row
    wr = np.array([[0.5, 2.0, 2.0, 0.5]], np.float32)
    idx, _ = orc.router_topk(x, wr, 3)
    assert idx.tolist() == [[1, 2, 0]]
    wr2 = np.array([[0.5, np.nan, 2.0, 0.5]], np.float32).reshape(1, 4)
    idx2, _ = orc.router_topk(x, wr2, 2)
    assert idx2.tolist() == [[1, 2]]


def test_dispatch_is_stable_by_expert(orc):
    idx = np.array([[2, 0], [0, 2], [1, 0], [2, 1]], np.int32)
    counts, offsets, perm, inv = orc.dispatch(idx, 3)
    assert counts.tolist() == [3, 2, 3]
    assert offsets.tolist() == [0, 3, 5, 8]
    assert perm.tolist() == [1, 2, 5, 4, 7, 0, 3, 6]
    assert np.array_equal(perm[inv], np.arange(8))
    with pytest.raises(ValueError):
        orc.dispatch(np.array([[3, 0]], np.int32), 3)
