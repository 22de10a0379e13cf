"""The resident MoE layer on the GPU against the oracle's composition of the
reference path (router -> top-k -> gate/up -> SwiGLU -> down -> route-ordered
sum -> shared expert).  Routing must match exactly; outputs within the 2e-3
relative-L2 contract (they land near 1e-6)."""
import numpy as np
import pytest
import torch

from warp_b200 import container as C

pytestmark = pytest.mark.gpu

TOL_FFN = 2e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _oracle_layer(oracle, layer, xs, K, renorm, with_shared, recs):
    bank = layer.bank
    booksT = bank.booksT.cpu().numpy()
    router = layer.router.cpu().numpy()
    sh = None
    if with_shared:
        sh = {k: (v.cpu().numpy().view(np.uint16) if k.endswith("_s") else v.cpu().numpy())
              if torch.is_tensor(v) else v for k, v in layer.shared.items()}
    sg = None if layer.shared_gate is None else layer.shared_gate.cpu().numpy()
    outs, idxs = [], []
    for x in xs:
        out, idx, w, acc = oracle.moe_layer(x, bank.hidden, bank.inter, bank.E, K, renorm,
                                            router, recs, booksT, sh, sg)
        outs.append(out)
        idxs.append(idx)
    return np.stack(outs), np.stack(idxs)


def _layer(hidden, inter, E, seed, shared, shared_gate, device, bits=4, group=32):
    from warp_b200 import synth
    bank = synth.random_bank(E, hidden, inter, seed, device=device)
    router = synth.router_matrix(E, hidden, seed + 1, device=device)
    sh = synth.shared_expert(hidden, inter, seed + 2, group=group, bits=bits,
                             device=device) if shared else None
    sg = (torch.randn(hidden, generator=torch.Generator(device=device).manual_seed(seed + 3),
                      device=device) * 0.02) if shared_gate else None
    return synth.SyntheticLayer(bank, router, sh, sg)


@pytest.mark.parametrize("tile", [True, False])
@pytest.mark.parametrize("hidden,inter,E,K,T,shared,gate", [
    (256, 128, 16, 4, 1, False, False),
    (256, 128, 16, 4, 3, True, False),
    (128, 96, 8, 2, 2, True, True),
    (384, 160, 8, 3, 1, True, False),         # partial chunks on both sides
    (2304, 1024, 32, 8, 1, True, False),      # config 1 geometry
])
def test_moe_layer_random_bank(cuda, oracle, hidden, inter, E, K, T, shared, gate, tile):
    layer = _layer(hidden, inter, E, hidden + E, shared, gate, cuda)
    recs = layer.host_records()
    moe = layer.moe(K, renorm=True, max_tokens=T, tile_bank=tile)
    gen = torch.Generator().manual_seed(hidden * 3 + T)
    x = torch.randn(T, hidden, generator=gen)
    x = x / x.pow(2).mean(-1, keepdim=True).add(1e-6).sqrt()          # RMSNorm'd
    out, idx, w = moe.forward(x.to(cuda), want_route=True)
    moe.status()
    want, widx = _oracle_layer(oracle, layer, x.numpy(), K, True, shared, recs)
    np.testing.assert_array_equal(idx.cpu().numpy(), widx)
    err = rel_l2(out.cpu().numpy(), want)
    assert err < TOL_FFN, err
    assert err < 1e-4, f"far above fp32 reordering noise: {err}"


def test_moe_layer_residual(cuda, oracle):
    layer = _layer(256, 128, 16, 7, True, False, cuda)
    moe = layer.moe(4, max_tokens=2)
    x = torch.randn(2, 256, generator=torch.Generator().manual_seed(1)).to(cuda)
    r = torch.randn(2, 256, generator=torch.Generator().manual_seed(2)).to(cuda)
    a = moe.forward(x)
    b = moe.forward(x, residual=r)
    torch.testing.assert_close(b, a + r, rtol=1e-6, atol=1e-6)


def test_config1_encoded(cuda, oracle):
    """Config 1: 32 routed experts N(0, 0.02) from seed 0, codebooks trained
    and every matrix encoded by the device port of waste_vq_encode; the codes
    of sampled experts must equal the oracle encoder's byte for byte, and the
    layer (top-8 softmax router, Q4 g32 shared expert) must match the oracle."""
    from warp_b200 import synth
    hidden, inter, E, K = 2304, 1024, 32, 8
    ws = []
    bank = synth.encoded_bank(E, hidden, inter, seed=0, device=cuda, weights_out=ws)
    # codes: re-encode sampled matrices with the CPU oracle's restatement of
    # quantize_vq + waste_vq_encode, using the same fp32 training books
    from warp_b200 import ops
    books32 = bank.books32.numpy()
    for e in (0, E - 1):
        rec = bank.record(e).cpu().numpy()
        hdr = C.parse_header(rec)
        for k, (M, N), off, soff in ((0, (inter, hidden), hdr["gate_off"], 0),
                                     (2, (hidden, inter), hdr["down_off"], 2 * inter)):
            Wk = ws[e][k].numpy()
            blk = rec[off:off + C.index_bytes(M, N)]
            codes, scales = oracle.quantize_vq(Wk, books32[3 * k:3 * k + 3])
            np.testing.assert_array_equal(C.unblock_indices(blk, M, N), codes)
            sc = np.frombuffer(rec[hdr["chan_corr_off"] + 2 * soff:][:2 * M].tobytes(),
                               np.uint16)
            np.testing.assert_array_equal(sc, scales)
            # the device dequant of the stored record equals the oracle's
            dq = ops.vq_dequant(torch.from_numpy(blk.copy()).to(cuda),
                                torch.from_numpy(sc.view(np.int16).copy()).to(cuda),
                                bank.books, M, N, 3 * k).cpu().numpy()
            want = oracle.vq_dequant(blk, sc, bank.books.cpu().numpy(), M, N, 3 * k)
            np.testing.assert_array_equal(dq.view(np.uint32), want.view(np.uint32))
            rel = np.linalg.norm(dq - Wk) / np.linalg.norm(Wk)
            assert rel < 0.5, rel                  # 3-bit RVQ reconstructs
    router = synth.router_matrix(E, hidden, 1, device=cuda)
    sh = synth.shared_expert(hidden, inter, 2, device=cuda)
    layer = synth.SyntheticLayer(bank, router, sh)
    recs = layer.host_records()
    moe = layer.moe(K)
    x = torch.randn(1, hidden, generator=torch.Generator().manual_seed(0))
    x = x / x.pow(2).mean(-1, keepdim=True).add(1e-6).sqrt()
    out, idx, w = moe.forward(x.to(cuda), want_route=True)
    want, widx = _oracle_layer(oracle, layer, x.numpy(), K, True, True, recs)
    np.testing.assert_array_equal(idx.cpu().numpy(), widx)
    assert rel_l2(out.cpu().numpy(), want) < TOL_FFN


def test_tiled_bank_marks_headers(cuda):
    """Re-tiling happens once: the headers carry the mark, a second layer on
    the same bank reuses it, and the gather results agree with the untiled
    path."""
    from warp_b200 import container as C
    layer = _layer(256, 128, 8, 3, True, False, cuda)
    plain = layer.bank.bank.clone()
    x = torch.randn(1, 256, generator=torch.Generator().manual_seed(5)).to(cuda)
    ref = synth_layer_with(layer, plain).moe(2, tile_bank=False).forward(x)
    m1 = layer.moe(2)
    h = C.parse_header(layer.bank.bank[:48].cpu().numpy())
    assert h["flags"] & 0x80
    a = m1.forward(x)
    m2 = layer.moe(2)                     # already tiled: no second transform
    b = m2.forward(x)
    torch.testing.assert_close(a, b, rtol=0, atol=0)
    torch.testing.assert_close(a, ref, rtol=1e-5, atol=1e-6)


def synth_layer_with(layer, bank_tensor):
    from warp_b200 import synth
    bk = layer.bank
    nb = synth.ExpertBank(bank_tensor, bk.rec_bytes, bk.books_f16, bk.hidden, bk.inter, bk.E)
    return synth.SyntheticLayer(nb, layer.router, layer.shared, layer.shared_gate)


@pytest.mark.parametrize("hidden,inter,E,K,T,weight", [
    (256, 128, 16, 4, 1, False),
    (384, 160, 8, 3, 3, True),
    (2304, 1024, 32, 8, 2, True),            # config 1 geometry
])
def test_block_forward(cuda, oracle, hidden, inter, E, K, T, weight):
    """warp_moe_block_forward: out = h + MoE(RMSNorm(h) * w).  It equals
    warp_rmsnorm followed by the layer with residual h, and the oracle's
    layer on the host-normalised input."""
    from warp_b200 import ops
    layer = _layer(hidden, inter, E, hidden + 3 * E, True, False, cuda)
    recs = layer.host_records()
    moe = layer.moe(K, max_tokens=T)
    gen = torch.Generator().manual_seed(hidden + T)
    h = torch.randn(T, hidden, generator=gen) * 3.0
    nw = (torch.rand(hidden, generator=gen) + 0.5) if weight else None
    hd = h.to(cuda)
    nwd = nw.to(cuda) if weight else None
    out = torch.empty_like(hd)
    got, idx, w = moe.forward_block(hd, out, norm_w=nwd, eps=1e-6, want_route=True)
    xn = ops.rmsnorm(hd, w=nwd, eps=1e-6)
    ref, ridx, rw = moe.forward(xn, residual=hd, want_route=True)
    moe.status()
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx.cpu().numpy())
    assert torch.equal(got, ref)
    # against the oracle on the host-normalised input
    hn = h.double()
    x = (hn / torch.sqrt(hn.pow(2).mean(-1, keepdim=True) + 1e-6)).float()
    if weight:
        x = x * nw
    want, widx = _oracle_layer(oracle, layer, x.numpy(), K, True, True, recs)
    np.testing.assert_array_equal(idx.cpu().numpy(), widx)
    assert rel_l2(got.cpu().numpy() - h.numpy(), want) < 1e-4


@pytest.mark.parametrize("func,bias,scale", [(0, True, 2.5), (2, False, 1.0), (1, True, 1.0)])
def test_moe_layer_router_of_moe_layer(cuda, oracle, func, bias, scale):
    """A layer with moe_layer's router (model.c:5466-5556): sigmoid /
    sqrt-softplus / softmax scores, the selection-only bias, renorm and
    routed_scale, an unscaled shared expert; routing exact against the
    oracle's layer, output within 1e-4."""
    hidden, inter, E, K, T = 512, 256, 32, 8, 2
    layer = _layer(hidden, inter, E, 91 + func, True, False, cuda)
    recs = layer.host_records()
    gen = torch.Generator().manual_seed(5 + func)
    b = (torch.randn(E, generator=gen) * 0.05) if bias else None
    moe = layer.moe(K, max_tokens=T, router_kind=1, score_func=func,
                    score_bias=None if b is None else b.to(cuda), routed_scale=scale)
    x = torch.randn(T, hidden, generator=gen)
    x = x / x.pow(2).mean(-1, keepdim=True).add(1e-6).sqrt()
    out, idx, w = moe.forward(x.to(cuda), want_route=True)
    moe.status()
    router = layer.router.cpu().numpy()
    booksT = layer.bank.booksT.cpu().numpy()
    sh = {k: (v.cpu().numpy().view(np.uint16) if k.endswith("_s") else v.cpu().numpy())
          if torch.is_tensor(v) else v for k, v in layer.shared.items()}
    route = dict(func=func, bias=None if b is None else b.numpy(), routed_scale=scale)
    for t in range(T):
        want, widx, ww, _ = oracle.moe_layer(x[t].numpy(), hidden, inter, E, K, True, router,
                                             recs, booksT, sh, None, route)
        np.testing.assert_array_equal(idx.cpu().numpy()[t], widx)
        assert rel_l2(out.cpu().numpy()[t], want) < 1e-4
