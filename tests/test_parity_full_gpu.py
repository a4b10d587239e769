"""GPU parity at the full benchmark shapes, checked against the oracle (not
against the library's own run_test self-check):

- dot_general bf16 8192^3 and the batched [8,4096,4096]^2 form: sampled
  outputs against the oracle's increasing-k fp32 loop nest;
- causal attention [4,32,4096,128]: sampled rows of sampled (batch, head)
  pairs against the fp64 oracle;
- the 65536-token, 64-expert, top-8 MoE layer (D 2048, F 1536): every
  routing index and the dispatch permutation bit-exact, 16 sampled tokens
  through the experts and the combine;
- the reference's own seed-42 MoE check (T=4, D=16, F=32, E=8, top-2,
  scripts/export/export_mixtral_layer.py:154-235) run through the library
  with the inputs rounded to bf16.

Inputs are generated on the device by the seeded generator and copied to the
host, so the oracle sees exactly the bits the kernels read."""
import os

import numpy as np
import pytest
import torch

from tests._util import from_np_bf16, norm_err, rel_err, to_np_bf16

pytestmark = pytest.mark.gpu
TOL = 2e-2  # bf16 outputs
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _filled(rb, orc, shape, name, kind="uniform", sigma=1.0):
    t = torch.empty(shape, dtype=torch.bfloat16, device="cuda")
    if kind == "uniform":
        rb.fill_uniform(t, orc.stream_key(name))
    else:
        rb.fill_normal(t, orc.stream_key(name), 0.0, sigma)
    return t


def test_gemm_8192_sampled_vs_oracle(rb, orc):
    n = 8192
    A = _filled(rb, orc, (n, n), "gemm_a")
    B = _filled(rb, orc, (n, n), "gemm_b")
    C = rb.gemm(A, B)
    torch.cuda.synchronize()
    a, b, c = to_np_bf16(A), to_np_bf16(B), to_np_bf16(C)
    rng = np.random.default_rng(8192)
    ii, jj = rng.integers(0, n, 4096), rng.integers(0, n, 4096)
    # corners and tile edges as well as random positions
    ii[:8] = [0, 0, n - 1, n - 1, 127, 128, 4095, 4096]
    jj[:8] = [0, n - 1, 0, n - 1, 255, 256, 4095, 4096]
    ref = orc.gemm_bf16_samples(a, b, ii, jj)
    got = orc.bf16_to_f32(c[ii, jj])
    assert rel_err(got, ref) <= TOL
    # the bf16 store of the fp32 sum agrees with the oracle's rounding almost everywhere
    assert np.mean(c[ii, jj] == orc.to_bf16(ref)) > 0.95


def test_gemm_batched_8x4096_sampled_vs_oracle(rb, orc):
    bt, n = 8, 4096
    A = _filled(rb, orc, (bt, n, n), "gemm_a")
    B = _filled(rb, orc, (bt, n, n), "gemm_b")
    C = rb.gemm(A, B)
    torch.cuda.synchronize()
    rng = np.random.default_rng(4096)
    for i in range(bt):
        a, b, c = to_np_bf16(A[i]), to_np_bf16(B[i]), to_np_bf16(C[i])
        ii, jj = rng.integers(0, n, 512), rng.integers(0, n, 512)
        ref = orc.gemm_bf16_samples(a, b, ii, jj)
        assert rel_err(orc.bf16_to_f32(c[ii, jj]), ref) <= TOL, f"batch {i}"


def test_attention_full_size_sampled_vs_oracle(rb, orc):
    """[4,32,4096,128] causal.  Tolerance: normwise max|g-r|/max|r| <= 2e-2
    per (batch, head) block.  The per-element relative error (floor
    1e-3*max|r|, the GEMM metric) is reported beside it and bounded loosely:
    P is rounded to bf16 for the second product, and an output element near
    a zero crossing of its weighted sum of V rows keeps that absolute error
    while its own magnitude vanishes -- a CPU emulation of exactly this
    rounding against the same fp64 oracle gives 0.15 on these inputs."""
    B, H, S, Dh = 4, 32, 4096, 128
    q = _filled(rb, orc, (B, H, S, Dh), "attn_q", "normal")
    k = _filled(rb, orc, (B, H, S, Dh), "attn_k", "normal")
    v = _filled(rb, orc, (B, H, S, Dh), "attn_v", "normal")
    o = rb.attention(q, k, v, causal=True)
    torch.cuda.synchronize()
    rng = np.random.default_rng(3)
    pairs = [(0, 0), (3, 31), (1, 7), (2, 20)] + [tuple(p) for p in
                                                   rng.integers(0, [B, H], (4, 2))]
    rows = np.concatenate([[0, 1, 127, 128, 255, 256, 2047, 4094, 4095],
                           rng.integers(0, S, 7)])
    worst_norm, worst_elem = 0.0, 0.0
    for b, h in pairs:
        ref = orc.attention_rows(to_np_bf16(q[b, h]), to_np_bf16(k[b, h]), to_np_bf16(v[b, h]),
                                 rows, causal=True)
        got = orc.bf16_to_f32(to_np_bf16(o[b, h]))[rows]
        worst_norm = max(worst_norm, norm_err(got, ref))
        worst_elem = max(worst_elem, rel_err(got, ref))
    print(f"attention [4,32,4096,128]: normwise {worst_norm:.2e}, per-element {worst_elem:.2e}")
    assert worst_norm <= TOL
    assert worst_elem <= 0.5


def test_moe_config5_layer_sampled(rb, orc):
    """T=65536, D=2048, F=1536, E=64, top-8 on one GPU: router indices and the
    dispatch permutation bit-exact over every token; 16 sampled tokens
    through the expert FFNs and the combine within 2e-2 (normwise)."""
    T, D, F, E, k = 65536, 2048, 1536, 64, 8
    x = _filled(rb, orc, (T, D), "moe_x", "normal")
    wr = _filled(rb, orc, (D, E), "moe_router", "normal", 0.02)
    wg = _filled(rb, orc, (E, D, F), "moe_wg", "normal", 0.02)
    wu = _filled(rb, orc, (E, D, F), "moe_wu", "normal", 0.02)
    wd = _filled(rb, orc, (E, F, D), "moe_wd", "normal", 0.02)
    out = rb.moe_layer(x, wr, wg, wu, wd, k=k)
    idx, _ = rb.moe_router_topk(x, wr, k)
    _, _, perm, _ = rb.moe_dispatch(idx, E)
    rb.synchronize_and_check()
    xh, wrh = to_np_bf16(x), to_np_bf16(wr)
    ridx, rw = orc.router_topk(xh, wrh, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    _, _, rperm, _ = orc.dispatch(ridx, E)
    assert np.array_equal(perm.cpu().numpy(), rperm)
    toks = np.random.default_rng(5).choice(T, 16, replace=False)
    toks[0], toks[1] = 0, T - 1
    ysel = np.empty((16 * k, D), np.uint16)
    for e in np.unique(ridx[toks]):
        sel_t, sel_j = np.nonzero(ridx[toks] == e)
        _, y, _ = orc.expert_ffn(xh[toks[sel_t]], to_np_bf16(wg[e]), to_np_bf16(wu[e]),
                                 to_np_bf16(wd[e]))
        ysel[sel_t * k + sel_j] = y
    ref = orc.combine(ysel, np.arange(16 * k, dtype=np.int32).reshape(16, k), rw[toks])
    got = orc.bf16_to_f32(to_np_bf16(out)[toks])
    assert norm_err(got, orc.bf16_to_f32(ref)) <= TOL


def test_moe_reference_seed42_fixture(rb, orc):
    """The reference's own MoE check (export_mixtral_layer.py:154-235: T=4,
    D=16, F=32, E=8, top-2, default_rng(42) inputs, f32 numpy output) run on
    the GPU with its inputs rounded to bf16.  The library's layer takes
    d_model in multiples of 32, so D is zero-padded to 32: the extra router
    rows, gate/up rows and down columns are 0, which leaves every logit,
    every expert activation and the first 16 output columns unchanged.
    Indices must match the fixture wherever the logit gaps that decide the
    top-2 exceed the worst change bf16 rounding of the inputs can cause;
    the outputs of those tokens must be within 2e-2 (normwise) of the
    fixture's f32 output."""
    z = np.load(os.path.join(GOLDEN, "moe_mini_seed42.npz"))
    T, D = z["tokens"].shape
    E, _, F = z["w_gate"].shape
    Dp = 32
    pad = lambda a, axis: np.concatenate(
        [a, np.zeros(a.shape[:axis] + (Dp - D,) + a.shape[axis + 1:], np.float32)], axis=axis)
    x = orc.to_bf16(pad(z["tokens"], 1))
    wr = orc.to_bf16(pad(z["router"], 0))
    wg = orc.to_bf16(pad(z["w_gate"], 1))
    wu = orc.to_bf16(pad(z["w_up"], 1))
    wd = orc.to_bf16(pad(z["w_down"], 2))
    args = [from_np_bf16(a) for a in (x, wr, wg, wu, wd)]
    out = rb.moe_layer(*args, k=2)
    idx, _ = rb.moe_router_topk(args[0], args[1], 2)
    rb.synchronize_and_check()
    idx = idx.cpu().numpy()
    got = orc.bf16_to_f32(to_np_bf16(out))[:, :D]
    assert np.all(to_np_bf16(out)[:, D:] == 0)
    lg = z["tokens"].astype(np.float64) @ z["router"].astype(np.float64)
    bound = 2 * 2.0 ** -8 * (np.abs(z["tokens"]) @ np.abs(z["router"])).max(axis=1)
    srt = np.sort(lg, axis=1)[:, ::-1]
    decided = (srt[:, 0] - srt[:, 1] > 2 * bound) & (srt[:, 1] - srt[:, 2] > 2 * bound)
    assert decided.sum() >= 3
    assert np.array_equal(idx[decided], z["idx"][decided])
    assert norm_err(got[decided], z["out"][decided]) <= TOL
