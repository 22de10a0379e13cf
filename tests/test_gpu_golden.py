"""The CUDA kernels against the golden vectors made by the reference's own
code (tests/golden/make_golden.py), through the C ABI.  Same bars as the
other GPU tests: bit-exact where the arithmetic allows it, 2e-5 relative L2
for the bandwidth kernels, the 2e-3 FFN contract for a whole layer."""
import hashlib
import json
import os
import sys

import numpy as np
import pytest
import torch

from warp_b200 import container as C

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
if GOLD not in sys.path:
    sys.path.insert(0, GOLD)
import make_golden as MG  # noqa: E402

TOL_KERNEL = 2e-5
TOL_FFN = 2e-3


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def load(name):
    z = np.load(os.path.join(GOLD, name))
    return z, json.loads(str(z["meta"]))


def dev(a, cuda):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    return torch.from_numpy(a.copy()).to(cuda)


def test_dequant_kimi_records(cuda, oracle):
    from warp_b200 import ops
    z, meta = load("kimi_tiny.npz")
    books, _ = oracle.books_decode(z["books_f16"])
    db = dev(books, cuda)
    for ei, rec in enumerate(z["records"]):
        h = C.parse_header(rec)
        sc = h["chan_corr_off"]
        for k, (off, (M, N)) in enumerate(zip(
                (h["gate_off"], h["up_off"], h["down_off"]),
                ((meta["inter"], meta["hidden"]), (meta["inter"], meta["hidden"]),
                 (meta["hidden"], meta["inter"])))):
            idx = rec[off:off + C.index_bytes(M, N)]
            scale = np.frombuffer(rec[sc:sc + 2 * M].tobytes(), np.uint16)
            sc += 2 * M
            got = ops.vq_dequant(dev(idx, cuda), dev(scale, cuda), db, M, N, 3 * k)
            assert sha(got.cpu().numpy()) == z["engine_sha"][ei][k]


def test_tables_and_apply(cuda, oracle):
    from warp_b200 import ops
    z, k = load("kernels_ref.npz")
    books_f16, x = MG.lut_inputs(k)
    _, booksT = oracle.books_decode(books_f16)
    for j, cb in enumerate((0, 3, 6)):
        lut = ops.vq_build_lut(dev(booksT, cuda), dev(x, cuda), cb)
        assert sha(lut.cpu().numpy()) == z["lut_sha"][j]
    idx, scale, lut = MG.rows_inputs(k)
    M = k["rows_M"]
    args = (dev(idx, cuda), dev(scale, cuda), dev(lut, cuda), M)
    y = ops.vq_apply(*args, ordered=True).cpu().numpy()
    np.testing.assert_array_equal(y.view(np.uint32), z["rows_y"].view(np.uint32))
    yf = ops.vq_apply(*args, ordered=False).cpu().numpy()
    assert rel_l2(yf, z["rows_y"]) < TOL_KERNEL


def test_encoder_rebuilds_convert_record(cuda):
    """The device encoder (waste_vq_encode) on convert.py's normalized
    vectors and trained books reproduces convert.py's record byte for byte."""
    from warp_b200 import ops
    z, cfg = load("convert_expert.npz")
    Ws = MG.convert_weights(cfg)
    assert [sha(W) for W in Ws] == list(z["w_sha"])
    books = z["books_f32"].reshape(3, 3, 256, 8)
    blocked, scales = [], []
    for k, W in enumerate(Ws):
        amax = np.maximum(np.abs(W).max(1, keepdims=True), np.float32(1e-8))
        X = (W / amax).astype(np.float32).reshape(-1, 8)
        codes = ops.vq_encode(dev(X, cuda), dev(books[k], cuda)).cpu().numpy()
        blocked.append(C.block_indices(codes, *W.shape))
        scales.append(amax.reshape(-1).astype(np.float16).view(np.uint16))
    rec = C.write_record(cfg["layer"], cfg["expert"], cfg["cb_base"], blocked, scales,
                         cfg["hidden"], cfg["inter"])
    assert rec == z["record"].tobytes()


def test_route(cuda):
    from warp_b200 import ops
    z, k = load("kernels_ref.npz")
    o = 0
    for E, K, renorm, logits in MG.route_inputs(k):
        idx, w = ops.qwen_moe_route(dev(logits, cuda).view(1, E), K, bool(renorm))
        np.testing.assert_array_equal(idx.cpu().numpy()[0], z["route_idx"][o:o + K])
        # indices bit-exact; the device sums the softmax as a tree, so weights
        # land within an ulp or two of the reference's serial sum
        np.testing.assert_allclose(w.cpu().numpy()[0], z["route_w"][o:o + K], rtol=4e-6)
        o += K


@pytest.mark.parametrize("bits", [4, 8])
def test_matvec(cuda, bits):
    from warp_b200 import ops
    z, k = load("kernels_ref.npz")
    W, ws, x, group, rowbytes = MG.mvq_inputs(k, bits)
    y = ops.mvq_matvec(dev(W, cuda), dev(ws, cuda), dev(x, cuda).view(1, -1), k["mvq_out"],
                       k["mvq_in"], group, bits, rowbytes).cpu().numpy()[0]
    assert rel_l2(y, z[f"mvq{bits}_portable"]) < TOL_KERNEL


def test_moe_layer(cuda, oracle):
    """The small layer the reference ran (router, experts_staged, shared
    expert) as a resident device layer."""
    from warp_b200 import ops
    z, k = load("kernels_ref.npz")
    books_f16, _codes, router, shared, x = MG.moe_inputs(k)
    books, booksT = oracle.books_decode(books_f16)
    recs = z["moe_records"]
    (gw, gs), (uw, us), (dw, ds) = shared
    sh = {"gate_w": dev(gw, cuda), "gate_s": dev(gs, cuda), "up_w": dev(uw, cuda),
          "up_s": dev(us, cuda), "down_w": dev(dw, cuda), "down_s": dev(ds, cuda),
          "inter": k["moe_si"], "group": 32, "bits": 4}
    layer = ops.MoELayer(dev(recs.reshape(-1), cuda), recs.shape[1], dev(books, cuda),
                         dev(booksT, cuda), dev(router, cuda), k["moe_hidden"],
                         k["moe_inter"], k["moe_E"], k["moe_K"], True, sh)
    try:
        out, idx, w = layer.forward(dev(x, cuda).view(1, -1), want_route=True)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(idx.cpu().numpy()[0], z["moe_idx"])
        # the device computes its own logits (another summation order), so the
        # weights agree to fp32 rounding rather than bit for bit
        np.testing.assert_allclose(w.cpu().numpy()[0], z["moe_w"], rtol=1e-5)
        want = z["moe_routed"] + z["moe_shared"]
        err = rel_l2(out.cpu().numpy()[0], want)
        assert err < TOL_FFN
        assert err < 1e-4
    finally:
        layer.close()
