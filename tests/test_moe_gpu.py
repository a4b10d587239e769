"""GPU parity: MoE router / dispatch / grouped expert GEMMs / combine / layer.

Router top-k indices and the dispatch permutation must be bit-identical to
the oracle; bf16 outputs are within 2e-2."""
import numpy as np
import pytest
import torch

from tests._util import from_np_bf16, norm_err, rel_err, to_np_bf16

pytestmark = pytest.mark.gpu
TOL = 2e-2


def _moe_inputs(orc, T, D, F, E, seed=42):
    x = orc.to_bf16(orc.normal("moe_x", (T, D), seed=seed))
    wr = orc.to_bf16(orc.normal("moe_router", (D, E), sigma=0.02, seed=seed))
    wg = orc.to_bf16(orc.normal("moe_wg", (E, D, F), sigma=0.02, seed=seed))
    wu = orc.to_bf16(orc.normal("moe_wu", (E, D, F), sigma=0.02, seed=seed))
    wd = orc.to_bf16(orc.normal("moe_wd", (E, F, D), sigma=0.02, seed=seed))
    return x, wr, wg, wu, wd


@pytest.mark.parametrize("T,D,E,k", [(1000, 256, 8, 2), (333, 512, 64, 8), (77, 64, 6, 3),
                                     (4096, 1024, 16, 4), (5, 8, 2, 1), (130, 128, 256, 8),
                                     (2000, 512, 36, 4), (600, 256, 128, 8), (300, 96, 24, 16),
                                     (8192, 2048, 64, 8)])
def test_router_topk_bit_exact(rb, orc, T, D, E, k):
    x = orc.to_bf16(orc.normal("moe_x", (T, D)))
    wr = orc.to_bf16(orc.normal("moe_router", (D, E), sigma=0.02))
    idx, w = rb.moe_router_topk(from_np_bf16(x), from_np_bf16(wr), k)
    ridx, rw = orc.router_topk(x, wr, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_allclose(w.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)


def test_router_ties_choose_lower_expert(rb, orc):
    # identical router columns -> identical logits -> ties broken to the lower index
    T, D, E = 64, 32, 8
    x = orc.to_bf16(orc.normal("moe_x", (T, D)))
    col = orc.to_bf16(orc.normal("moe_router", (D, 1), sigma=0.02))
    wr = np.ascontiguousarray(np.repeat(col, E, axis=1))
    idx, _ = rb.moe_router_topk(from_np_bf16(x), from_np_bf16(wr), 3)
    ridx, _ = orc.router_topk(x, wr, 3)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert np.all(ridx == np.array([0, 1, 2]))


@pytest.mark.parametrize("T,D,E,k", [(8192, 4096, 8, 2), (65536, 2048, 64, 8)])
def test_router_full_size_bit_exact(rb, orc, T, D, E, k):
    """The two MoE configurations at full size: every index bit-exact."""
    x = orc.to_bf16(orc.normal("moe_x", (T, D)))
    wr = orc.to_bf16(orc.normal("moe_router", (D, E), sigma=0.02))
    idx, w = rb.moe_router_topk(from_np_bf16(x), from_np_bf16(wr), k)
    ridx, rw = orc.router_topk(x, wr, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    assert np.max(np.abs(w.cpu().numpy() - rw)) < 1e-6


@pytest.mark.parametrize("T,k,E,mode", [(1000, 2, 8, "uniform"), (65536, 8, 64, "uniform"),
                                        (100000, 8, 64, "skewed"), (70000, 16, 256, "uniform"),
                                        (3000, 2, 8, "one_expert"), (777, 4, 32, "skewed"),
                                        (1, 1, 4, "uniform"), (1024, 1, 3, "uniform")])
def test_dispatch_bit_exact(rb, orc, T, k, E, mode):
    rng = np.random.default_rng(T + k + E)
    if mode == "uniform":
        idx = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    elif mode == "one_expert":
        idx = np.tile(np.arange(k, dtype=np.int32), (T, 1))
    else:
        p = np.arange(1, E + 1, dtype=np.float64) ** 3
        idx = np.stack([rng.choice(E, k, replace=False, p=p / p.sum())
                        for _ in range(T)]).astype(np.int32)
    counts, offsets, perm, inv = rb.moe_dispatch(torch.from_numpy(idx).cuda(), E)
    rc, ro, rp, ri = orc.dispatch(idx, E)
    assert np.array_equal(counts.cpu().numpy(), rc)
    assert np.array_equal(offsets.cpu().numpy(), ro)
    assert np.array_equal(perm.cpu().numpy(), rp)
    assert np.array_equal(inv.cpu().numpy(), ri)


def test_dispatch_rejects_bad_expert_id(rb):
    idx = torch.tensor([[0, 1], [5, 2]], dtype=torch.int32, device="cuda")
    rb.moe_dispatch(idx, 4)
    with pytest.raises(rb.RemoraError) as e:
        rb.synchronize_and_check()
    assert e.value.code == rb.ERR_INVALID
    rb.synchronize_and_check()  # the error word was cleared


@pytest.mark.parametrize("T,D,E,k", [(500, 256, 8, 2), (300, 1000, 16, 5), (64, 2048, 64, 8),
                                     (40, 136, 32, 12), (7, 8, 4, 3)])
def test_gather_and_combine_bit_exact(rb, orc, T, D, E, k):
    x, wr, *_ = _moe_inputs(orc, T, D, 128, E)
    idx, w = orc.router_topk(x, wr, k)
    _, _, perm, inv = orc.dispatch(idx, E)
    xs = rb.moe_gather(from_np_bf16(x), torch.from_numpy(perm).cuda(), k)
    assert np.array_equal(to_np_bf16(xs), x[perm // k])
    xs2 = rb.moe_scatter(from_np_bf16(x), torch.from_numpy(inv).cuda(), k)
    assert np.array_equal(to_np_bf16(xs2), x[perm // k])
    y = orc.to_bf16(orc.normal("moe_wd", (T * k, D)))
    out = rb.moe_combine(from_np_bf16(y), torch.from_numpy(inv).cuda(), torch.from_numpy(w).cuda())
    assert np.array_equal(to_np_bf16(out), orc.combine(y, inv, w))


def _expert_rows(orc, x, wr, k, E):
    idx, w = orc.router_topk(x, wr, k)
    counts, offsets, perm, inv = orc.dispatch(idx, E)
    return idx, w, counts, offsets, perm, inv, x[perm // k]


@pytest.mark.parametrize("T,D,F,E,k", [(300, 256, 128, 8, 2), (64, 512, 384, 4, 2),
                                       (1000, 256, 256, 16, 4)])
def test_grouped_gemms_parity(rb, orc, T, D, F, E, k):
    x, wr, wg, wu, wd = _moe_inputs(orc, T, D, F, E)
    idx, w, counts, offsets, perm, inv, xs = _expert_rows(orc, x, wr, k, E)
    off_t = torch.from_numpy(offsets).cuda()
    h = rb.grouped_gemm_swiglu(from_np_bf16(xs), from_np_bf16(wg), from_np_bf16(wu), off_t)
    y = rb.grouped_gemm(h, from_np_bf16(wd), off_t)
    hg = orc.bf16_to_f32(to_np_bf16(h))
    yg = orc.bf16_to_f32(to_np_bf16(y))
    for e in range(E):
        a, b = offsets[e], offsets[e + 1]
        if a == b:
            continue
        hr, _, _ = orc.expert_ffn(xs[a:b], wg[e], wu[e], wd[e])
        assert rel_err(hg[a:b], orc.bf16_to_f32(hr)) <= TOL, f"h expert {e}"
        # the down GEMM checked on the GPU's own h (isolates the second GEMM)
        ref_y, _ = orc.gemm_bf16_rows(to_np_bf16(h)[a:b], wd[e], 0, b - a)
        assert rel_err(yg[a:b], ref_y) <= TOL, f"y expert {e}"


def test_grouped_gemm_empty_and_skewed_experts(rb, orc):
    # all rows on expert 2, experts 0, 1, 3 empty
    rows, D, F, E = 200, 256, 128, 4
    xs = orc.to_bf16(orc.normal("moe_x", (rows, D)))
    wg = orc.to_bf16(orc.normal("moe_wg", (E, D, F), sigma=0.02))
    wu = orc.to_bf16(orc.normal("moe_wu", (E, D, F), sigma=0.02))
    offsets = np.array([0, 0, 0, rows, rows], np.int32)
    h = rb.grouped_gemm_swiglu(from_np_bf16(xs), from_np_bf16(wg), from_np_bf16(wu),
                               torch.from_numpy(offsets).cuda())
    hr, _, _ = orc.expert_ffn(xs, wg[2], wu[2], np.zeros((F, D), np.uint16))
    assert rel_err(orc.bf16_to_f32(to_np_bf16(h)), orc.bf16_to_f32(hr)) <= TOL


@pytest.mark.parametrize("T,D,F,E,k", [(512, 256, 256, 8, 2), (256, 512, 128, 64, 8)])
def test_moe_layer_parity(rb, orc, T, D, F, E, k):
    x, wr, wg, wu, wd = _moe_inputs(orc, T, D, F, E)
    out = rb.moe_layer(*(from_np_bf16(a) for a in (x, wr, wg, wu, wd)), k=k)
    rb.synchronize_and_check()
    *_, ref = orc.moe_layer_bf16(x, wr, wg, wu, wd, k)
    got = orc.bf16_to_f32(to_np_bf16(out))
    r = orc.bf16_to_f32(ref)
    assert norm_err(got, r) <= TOL


@pytest.mark.parametrize("T,chunk", [(1000, 256), (777, 0), (4096, 1000), (8192, 512)])
def test_moe_layer_host_buffers_match_device_layer(rb, orc, T, chunk):
    """Tokens and output in pinned host memory, copied in chunks (a ragged
    last chunk; one chunk when chunk_tokens=0 covers T; from T >= 4 chunks the
    quarter- and half-size first and last chunks) overlapped with the layer:
    bit-identical to the device-buffer layer."""
    D, F, E, k = 256, 128, 16, 4
    x, wr, wg, wu, wd = _moe_inputs(orc, T, D, F, E)
    dev = [from_np_bf16(a) for a in (x, wr, wg, wu, wd)]
    ref = rb.moe_layer(*dev, k=k)
    x_host = dev[0].cpu().pin_memory()
    out = rb.moe_layer_host(x_host, *dev[1:], k=k, chunk_tokens=chunk)
    torch.cuda.current_stream().synchronize()
    rb.synchronize_and_check()
    assert torch.equal(out.view(torch.int16), ref.cpu().view(torch.int16))
    # a second call reuses the library's copy streams and events
    out2 = rb.moe_layer_host(x_host, *dev[1:], k=k, chunk_tokens=chunk)
    torch.cuda.current_stream().synchronize()
    assert torch.equal(out2.view(torch.int16), ref.cpu().view(torch.int16))


def test_moe_layer_deterministic(rb, orc):
    x, wr, wg, wu, wd = _moe_inputs(orc, 256, 256, 128, 8)
    args = [from_np_bf16(a) for a in (x, wr, wg, wu, wd)]
    a = rb.moe_layer(*args, k=2)
    b = rb.moe_layer(*args, k=2)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_moe_layer_config4_sampled(rb, orc):
    """T=8192, D=4096, F=14336, E=8, top-2 at full size: routing over all
    tokens bit-exact, 16 sampled tokens through the experts and combine."""
    T, D, F, E, k = 8192, 4096, 14336, 8, 2
    dev = torch.device("cuda")
    x = torch.empty(T, D, dtype=torch.bfloat16, device=dev)
    wr = torch.empty(D, E, dtype=torch.bfloat16, device=dev)
    wg = torch.empty(E, D, F, dtype=torch.bfloat16, device=dev)
    wu = torch.empty(E, D, F, dtype=torch.bfloat16, device=dev)
    wd = torch.empty(E, F, D, dtype=torch.bfloat16, device=dev)
    for t, name, sig in ((x, "moe_x", 1.0), (wr, "moe_router", 0.02), (wg, "moe_wg", 0.02),
                         (wu, "moe_wu", 0.02), (wd, "moe_wd", 0.02)):
        rb.fill_normal(t, orc.stream_key(name), 0.0, sig)
    out = rb.moe_layer(x, wr, wg, wu, wd, k=k)
    idx, _ = rb.moe_router_topk(x, wr, k)
    rb.synchronize_and_check()
    xh, wrh = to_np_bf16(x), to_np_bf16(wr)
    ridx, rw = orc.router_topk(xh, wrh, k)
    assert np.array_equal(idx.cpu().numpy(), ridx)
    toks = np.random.default_rng(1).choice(T, 16, replace=False)
    ref = np.empty((16, D), np.uint16)
    ysel = np.empty((16 * k, D), np.uint16)
    for j in range(k):
        for e in np.unique(ridx[toks, j]):
            sel = np.nonzero(ridx[toks, j] == e)[0]
            _, y, _ = orc.expert_ffn(xh[toks[sel]], to_np_bf16(wg[e]), to_np_bf16(wu[e]),
                                     to_np_bf16(wd[e]))
            ysel[sel * k + j] = y
    ref = orc.combine(ysel, np.arange(16 * k, dtype=np.int32).reshape(16, k), rw[toks])
    got = orc.bf16_to_f32(to_np_bf16(out)[toks])
    assert norm_err(got, orc.bf16_to_f32(ref)) <= TOL


def test_grouped_gemm_segments_match_expert_order(rb, orc):
    """Rows regrouped as (source rank, local expert) segments, the layout an
    expert-parallel rank receives, give the same rows bit for bit."""
    T, D, F, E, k, P = 600, 256, 256, 8, 2, 3
    x, wr, wg, wu, wd = _moe_inputs(orc, T, D, F, E)
    idx, w, counts, offsets, perm, inv, xs = _expert_rows(orc, x, wr, k, E)
    off_t = torch.from_numpy(offsets).cuda()
    Xs, Wg, Wu, Wd = (from_np_bf16(a) for a in (xs, wg, wu, wd))
    y_ref = to_np_bf16(rb.grouped_gemm(rb.grouped_gemm_swiglu(Xs, Wg, Wu, off_t), Wd, off_t))
    # split each expert's rows into P chunks ("sources"), order source-major
    order, seg_off, seg_exp = [], [0], []
    for src in range(P):
        for e in range(E):
            a, b = offsets[e], offsets[e + 1]
            chunk = np.arange(a, b)[src::P]
            order.extend(chunk.tolist())
            seg_off.append(seg_off[-1] + len(chunk))
            seg_exp.append(e)
    order = np.array(order)
    so = torch.tensor(seg_off, dtype=torch.int32, device="cuda")
    se = torch.tensor(seg_exp, dtype=torch.int32, device="cuda")
    h = rb.grouped_gemm_swiglu_segments(from_np_bf16(xs[order]), Wg, Wu, so, se)
    y = to_np_bf16(rb.grouped_gemm_segments(h, Wd, so, se))
    assert np.array_equal(y, y_ref[order])


def test_moe_layer_simple_moe_shape(rb, orc):
    """simple_moe.mlir:16 shapes (T=8, D=32, F=64, E=2, top-1): tiles wider
    than the matrices, column guards in the epilogues."""
    x, wr, wg, wu, wd = _moe_inputs(orc, 8, 32, 64, 2)
    out = rb.moe_layer(*(from_np_bf16(a) for a in (x, wr, wg, wu, wd)), k=1)
    rb.synchronize_and_check()
    *_, ref = orc.moe_layer_bf16(x, wr, wg, wu, wd, 1)
    assert norm_err(orc.bf16_to_f32(to_np_bf16(out)), orc.bf16_to_f32(ref)) <= TOL


@pytest.mark.parametrize("cfg", ["simple", "mixtral", "4"])
def test_run_test_moe_configs(rb, cfg):
    rep = rb.run_test("moe", config=cfg, iters=2, warmup=1)
    assert rep["passed"] and rep["max_rel_err"] <= TOL and rep["checked"] > 0
