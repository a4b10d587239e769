"""GPU parity: fused causal softmax attention against the oracle (fp64)."""
import numpy as np
import pytest
import torch

from tests._util import from_np_bf16, norm_err, to_np_bf16

pytestmark = pytest.mark.gpu
TOL = 2e-2  # bf16 outputs, normwise relative per (batch, head) block


def _qkv(orc, B, H, S, D=128, seed=42):
    q = orc.to_bf16(orc.normal("attn_q", (B, H, S, D), seed=seed))
    k = orc.to_bf16(orc.normal("attn_k", (B, H, S, D), seed=seed))
    v = orc.to_bf16(orc.normal("attn_v", (B, H, S, D), seed=seed))
    return q, k, v


def _check(orc, q, k, v, out, causal, rows=None):
    B, H, S, D = q.shape
    got = orc.bf16_to_f32(to_np_bf16(out))
    worst = 0.0
    for b in range(B):
        for h in range(H):
            rr = np.arange(S) if rows is None else rows
            ref = orc.attention_rows(q[b, h], k[b, h], v[b, h], rr, causal=causal)
            worst = max(worst, norm_err(got[b, h][rr], ref))
    return worst


@pytest.mark.parametrize("S,causal", [(256, True), (256, False), (512, True), (200, True),
                                      (100, False), (384, True), (640, False)])
def test_attention_full_parity(rb, orc, S, causal):
    q, k, v = _qkv(orc, 1, 2, S)
    out = rb.attention(from_np_bf16(q), from_np_bf16(k), from_np_bf16(v), causal=causal)
    assert _check(orc, q, k, v, out, causal) <= TOL


def test_attention_multi_head_batch_sampled(rb, orc):
    q, k, v = _qkv(orc, 2, 3, 1024)
    out = rb.attention(from_np_bf16(q), from_np_bf16(k), from_np_bf16(v), causal=True)
    rows = np.array([0, 1, 127, 128, 129, 255, 256, 511, 700, 1023])
    assert _check(orc, q, k, v, out, True, rows) <= TOL


def test_attention_large_logits_rescale(rb, orc):
    # scaled-up scores force the running-max rescale path
    q, k, v = _qkv(orc, 1, 1, 512)
    q = orc.to_bf16(orc.bf16_to_f32(q) * 4.0)
    out = rb.attention(from_np_bf16(q), from_np_bf16(k), from_np_bf16(v), causal=True)
    assert _check(orc, q, k, v, out, True) <= TOL


def test_attention_matches_torch_sdpa(rb, orc):
    q, k, v = _qkv(orc, 1, 4, 1024)
    Q, K, V = from_np_bf16(q), from_np_bf16(k), from_np_bf16(v)
    out = rb.attention(Q, K, V, causal=True)
    ref = torch.nn.functional.scaled_dot_product_attention(Q.float(), K.float(), V.float(),
                                                           is_causal=True)
    assert norm_err(out.float().cpu().numpy(), ref.cpu().numpy()) <= TOL


def test_attention_deterministic(rb, orc):
    q, k, v = _qkv(orc, 1, 2, 512)
    Q, K, V = from_np_bf16(q), from_np_bf16(k), from_np_bf16(v)
    a = rb.attention(Q, K, V)
    b = rb.attention(Q, K, V)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_attention_rejects_head_dim(rb):
    x = torch.zeros(1, 1, 128, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(rb.RemoraError):
        rb.attention(x, x, x)


def test_run_test_attention_full_size(rb):
    rep = rb.run_test("attention", iters=2, warmup=1)  # [4,32,4096,128] causal
    assert rep["passed"] and rep["checked"] == 64 * 128 and rep["max_rel_err"] <= TOL
