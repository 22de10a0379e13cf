"""The oracle against golden vectors made by the reference's own code
(tests/golden/make_golden.py): the reference's Python tools and its C kernels
compiled from source.  These pins hold without the reference present."""
import hashlib
import json
import os
import sys

import numpy as np
import pytest

from warp_b200 import container as C

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
if GOLD not in sys.path:
    sys.path.insert(0, GOLD)
import make_golden as MG  # noqa: E402


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def load(name):
    z = np.load(os.path.join(GOLD, name))
    return z, json.loads(str(z["meta"]))


def check_inputs(got, want, what):
    assert list(got) == list(want), (
        f"{what}: regenerated inputs differ from the ones the fixture was made "
        "from (numpy stream change?); rerun tests/golden/make_golden.py")


def record_matrices(rec, hidden, inter):
    """(blocked idx, scale u16, M, N) of gate, up, down of one record."""
    h = C.parse_header(rec)
    assert h["magic"] == C.MAGIC_EXPERT and h["fmt"] == C.FMT_VQ3R
    out, sc = [], h["chan_corr_off"]
    for off, (M, N) in zip((h["gate_off"], h["up_off"], h["down_off"]),
                           ((inter, hidden), (inter, hidden), (hidden, inter))):
        out.append((rec[off:off + C.index_bytes(M, N)],
                    np.frombuffer(rec[sc:sc + 2 * M].tobytes(), np.uint16), M, N))
        sc += 2 * M
    return h, out


def test_kimi_ref_dequant(oracle):
    """Expert dequant of tools/kimi_ref.py on make_test_container's records.
    With the engine's codebook decode (subnormals flushed) the oracle is
    bit-exact; with kimi_ref's own torch decode (subnormals kept) too, and the
    two differ exactly at the recorded number of subnormal-hit weights."""
    z, meta = load("kimi_tiny.npz")
    books_engine, _ = oracle.books_decode(z["books_f16"])
    books_kimi = np.ascontiguousarray(z["books_f16"].view(np.float16).astype(np.float32))
    assert int(np.sum(books_engine != books_kimi)) > 0       # the fixture has subnormals
    for ei, rec in enumerate(z["records"]):
        h, mats = record_matrices(rec, meta["hidden"], meta["inter"])
        assert h["layer"] == meta["layer"] and h["expert_id"] == meta["experts"][ei]
        assert h["codebook_id"] == meta["cb_base"]
        for k, (idx, scale, M, N) in enumerate(mats):
            eng = oracle.vq_dequant(idx, scale, books_engine, M, N, 3 * k)
            assert sha(eng) == z["engine_sha"][ei][k]
            np.testing.assert_array_equal(eng.reshape(-1)[:16], z["engine_head"][ei][k])
            kim = oracle.vq_dequant(idx, scale, books_kimi, M, N, 3 * k)
            assert sha(kim) == z["kimi_sha"][ei][k]
            assert int(np.sum(eng.view(np.uint32) != kim.view(np.uint32))) == \
                z["subnormal_diffs"][ei][k]


def test_convert_expert_record(oracle):
    """tools/convert.py's record for one expert (trained books, native
    encoder, write_expert_record) equals the oracle's quantize_vq + block +
    record writer byte for byte; its Q4 g32 and Q8 per-row quantizers too."""
    z, cfg = load("convert_expert.npz")
    Ws = MG.convert_weights(cfg)
    check_inputs([sha(W) for W in Ws], z["w_sha"], "convert weights")
    books = z["books_f32"].reshape(3, 3, 256, 8)
    blocked, scales = [], []
    for k, W in enumerate(Ws):
        codes, s = oracle.quantize_vq(W, books[k])
        blocked.append(C.block_indices(codes, *W.shape))
        scales.append(s)
    rec = C.write_record(cfg["layer"], cfg["expert"], cfg["cb_base"], blocked, scales,
                         cfg["hidden"], cfg["inter"])
    want = z["record"].tobytes()
    assert len(rec) == len(want)
    assert rec[:C.HDR.size] == want[:C.HDR.size]
    assert rec == want
    q4, s4 = oracle.quant_q(Ws[0], 32, 4)
    assert [sha(q4), sha(s4)] == list(z["q4_sha"])
    q8, s8 = oracle.quant_q(Ws[0], cfg["hidden"], 8)
    assert [sha(q8), sha(s8)] == list(z["q8_sha"])


@pytest.fixture(scope="module")
def kern():
    return load("kernels_ref.npz")


def test_books_and_tables(oracle, kern):
    z, k = kern
    books_f16, x = MG.lut_inputs(k)
    check_inputs([sha(books_f16), sha(x)], z["lut_in_sha"], "table inputs")
    books, booksT = oracle.books_decode(books_f16)
    assert [sha(books), sha(booksT)] == list(z["books_sha"])
    for j, cb in enumerate((0, 3, 6)):
        lut = oracle.lut_build(booksT, x, cb)
        assert sha(lut) == z["lut_sha"][j]
        np.testing.assert_array_equal(lut.reshape(-1)[:16], z["lut_head"][j])


def test_vq_rows(oracle, kern):
    z, k = kern
    idx, scale, lut = MG.rows_inputs(k)
    check_inputs([sha(idx), sha(scale), sha(lut)], z["rows_in_sha"], "vq_rows inputs")
    y = oracle.vq_rows(idx, scale, lut, k["rows_M"])
    np.testing.assert_array_equal(y.view(np.uint32), z["rows_y"].view(np.uint32))


@pytest.mark.parametrize("bits", [4, 8])
def test_mvq_rows(oracle, kern, bits):
    z, k = kern
    W, ws, x, group, rowbytes = MG.mvq_inputs(k, bits)
    check_inputs([sha(W), sha(ws), sha(x)], z[f"mvq{bits}_in_sha"], "matvec inputs")
    y = oracle.mvq_rows(W, ws, x, k["mvq_out"], k["mvq_in"], group, bits, rowbytes)
    np.testing.assert_array_equal(y.view(np.uint32), z[f"mvq{bits}_portable"].view(np.uint32))
    # the AVX-512 slot uses FMA in another order
    simd = z[f"mvq{bits}_avx512"]
    np.testing.assert_allclose(y, simd, rtol=1e-4, atol=1e-5 * np.abs(simd).max())


def test_route(oracle, kern):
    z, k = kern
    cases = MG.route_inputs(k)
    check_inputs([sha(c[3]) for c in cases], z["route_in_sha"], "router inputs")
    o = 0
    for E, K, renorm, logits in cases:
        rc, idx, w = oracle.qwen_route(logits, K, renorm)
        assert rc == 0
        np.testing.assert_array_equal(idx, z["route_idx"][o:o + K])
        np.testing.assert_array_equal(w.view(np.uint32), z["route_w"][o:o + K].view(np.uint32))
        o += K


def test_moe_layer(oracle, kern):
    """A whole small layer: route and routed experts bit-exact against
    experts_staged; the shared expert (AVX-512 in the reference) within fp32
    rounding."""
    z, k = kern
    books_f16, codes, router, shared, x = MG.moe_inputs(k)
    check_inputs([sha(books_f16), sha(router), sha(x)] + [sha(a) for p in shared for a in p],
                 z["moe_in_sha"], "layer inputs")
    _, booksT = oracle.books_decode(books_f16)
    recs = [np.ascontiguousarray(r) for r in z["moe_records"]]
    (gw, gs), (uw, us), (dw, ds) = shared
    sh = dict(gate_w=gw, gate_s=gs, up_w=uw, up_s=us, down_w=dw, down_s=ds, group=32, bits=4,
              inter=k["moe_si"])
    out, idx, w, acc = oracle.moe_layer(x, k["moe_hidden"], k["moe_inter"], k["moe_E"],
                                        k["moe_K"], 1, router, recs, booksT, sh)
    np.testing.assert_array_equal(idx, z["moe_idx"])
    np.testing.assert_array_equal(w.view(np.uint32), z["moe_w"].view(np.uint32))
    np.testing.assert_array_equal(acc.view(np.uint32), z["moe_acc"].view(np.uint32))
    want = z["moe_routed"] + z["moe_shared"]
    np.testing.assert_allclose(out, want, rtol=1e-5, atol=1e-6 * np.abs(want).max())
