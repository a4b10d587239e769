"""GPU parity of the heterogeneous MoE layer (experts of different FFN widths,
mlir/stablehlo/heterogeneous_moe_layer.mlir:66-212) against the oracle:
router indices bit-exact, bf16 outputs within 2e-2."""
import numpy as np
import pytest
import torch

from tests._util import from_np_bf16, norm_err, rel_err, to_np_bf16

pytestmark = pytest.mark.gpu
TOL = 2e-2
REF_F = [14336, 14336, 8192, 8192, 4096, 4096, 2048, 2048]  # heterogeneous_moe_layer.mlir:8-16


def _weights(orc, D, F, seed_base=0):
    wg = [orc.to_bf16(orc.normal(32, (D, f), sigma=0.02, seed=1000 + seed_base + e))
          for e, f in enumerate(F)]
    wu = [orc.to_bf16(orc.normal(33, (D, f), sigma=0.02, seed=1000 + seed_base + e))
          for e, f in enumerate(F)]
    wd = [orc.to_bf16(orc.normal(34, (f, D), sigma=0.02, seed=1000 + seed_base + e))
          for e, f in enumerate(F)]
    return wg, wu, wd


def test_var_grouped_gemms_per_expert_widths(rb, orc):
    """Each expert's h columns [0, F_e) and its down GEMM over K = F_e, with
    one expert empty and rows of one expert spanning several row tiles."""
    D, F = 256, [512, 256, 128, 64, 384, 192]
    E, rows = len(F), 700
    xs = orc.to_bf16(orc.normal("moe_x", (rows, D)))
    wg, wu, wd = _weights(orc, D, F)
    offsets = np.array([0, 300, 300, 350, 480, 481, rows], np.int32)  # expert 1 empty
    off_t = torch.from_numpy(offsets).cuda()
    G = [from_np_bf16(a) for a in wg]
    U = [from_np_bf16(a) for a in wu]
    W = [from_np_bf16(a) for a in wd]
    h = rb.grouped_gemm_swiglu_var(from_np_bf16(xs), G, U, off_t)
    y = rb.grouped_gemm_var(h, W, off_t)
    rb.synchronize_and_check()
    hh, yy = to_np_bf16(h), orc.bf16_to_f32(to_np_bf16(y))
    for e in range(E):
        a, b = offsets[e], offsets[e + 1]
        if a == b:
            continue
        hr, _, _ = orc.expert_ffn(xs[a:b], wg[e], wu[e], wd[e])
        assert rel_err(orc.bf16_to_f32(hh[a:b, :F[e]]), orc.bf16_to_f32(hr)) <= TOL, f"h {e}"
        assert np.all(hh[a:b, F[e]:] == 0), f"h {e}: columns past F_e written"
        ref_y, _ = orc.gemm_bf16_rows(np.ascontiguousarray(hh[a:b, :F[e]]), wd[e], 0, b - a)
        assert rel_err(yy[a:b], ref_y) <= TOL, f"y {e}"


@pytest.mark.parametrize("T,D,F,k", [(300, 256, [512, 256, 128, 64, 384, 192], 2),
                                     (97, 128, [64, 128, 192, 64], 1)])
def test_hetero_layer_parity(rb, orc, T, D, F, k):
    E = len(F)
    x = orc.to_bf16(orc.normal("moe_x", (T, D)))
    wr = orc.to_bf16(orc.normal("moe_router", (D, E), sigma=0.02))
    wg, wu, wd = _weights(orc, D, F)
    out = rb.moe_hetero_layer(from_np_bf16(x), from_np_bf16(wr), [from_np_bf16(a) for a in wg],
                              [from_np_bf16(a) for a in wu], [from_np_bf16(a) for a in wd], k)
    rb.synchronize_and_check()
    _, _, ref = orc.moe_hetero_layer_bf16(x, wr, wg, wu, wd, k)
    assert norm_err(orc.bf16_to_f32(to_np_bf16(out)), orc.bf16_to_f32(ref)) <= TOL


def test_hetero_layer_reference_shape_sampled(rb, orc):
    """The program's own shape: T=512, D=4096, F = 14336 x2, 8192 x2, 4096 x2,
    2048 x2, top-1.  Router indices over every token bit-exact; 16 sampled
    tokens (and the first and last) through the experts within 2e-2."""
    T, D, E, k = 512, 4096, 8, 1
    dev = torch.device("cuda")
    x = rb.fill_normal(torch.empty(T, D, dtype=torch.bfloat16, device=dev), orc.stream_key("moe_x"))
    wr = rb.fill_normal(torch.empty(D, E, dtype=torch.bfloat16, device=dev),
                        orc.stream_key("moe_router"), 0.0, 0.02)
    ws = []
    for kind, shape in ((32, lambda f: (D, f)), (33, lambda f: (D, f)), (34, lambda f: (f, D))):
        ws.append([rb.fill_normal(torch.empty(shape(f), dtype=torch.bfloat16, device=dev),
                                  orc.stream_key(kind, seed=1000 + e), 0.0, 0.02)
                   for e, f in enumerate(REF_F)])
    out = rb.moe_hetero_layer(x, wr, *ws, k)
    idx, _ = rb.moe_router_topk(x, wr, k)
    rb.synchronize_and_check()
    xh, wrh = to_np_bf16(x), to_np_bf16(wr)
    ridx, _ = orc.router_topk(xh, wrh, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    toks = np.random.default_rng(9).choice(T, 16, replace=False)
    toks[0], toks[1] = 0, T - 1
    wl = [[to_np_bf16(w) for w in kind] for kind in ws]
    _, _, ref = orc.moe_hetero_layer_bf16(xh, wrh, *wl, k, tokens=toks)
    assert norm_err(orc.bf16_to_f32(to_np_bf16(out)[toks]), orc.bf16_to_f32(ref)) <= TOL
    assert len(np.unique(ridx)) >= 4  # several widths were exercised


def test_hetero_rejects_bad_widths(rb):
    x = torch.zeros(8, 64, dtype=torch.bfloat16, device="cuda")
    wr = torch.zeros(64, 2, dtype=torch.bfloat16, device="cuda")
    wg = [torch.zeros(64, 96, dtype=torch.bfloat16, device="cuda")] * 2  # 96 % 64 != 0
    wd = [torch.zeros(96, 64, dtype=torch.bfloat16, device="cuda")] * 2
    with pytest.raises((rb.RemoraError, ValueError)):
        rb.moe_hetero_layer(x, wr, wg, wg, wd, 1)


def test_run_test_moe_hetero(rb):
    rep = rb.run_test("moe", config="hetero", iters=2, warmup=1)
    assert rep["passed"] and rep["max_rel_err"] <= TOL and rep["checked"] > 0
