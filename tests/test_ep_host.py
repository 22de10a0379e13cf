"""The expert-parallel decomposition on CPU, world_size 2 over gloo.

Each rank computes its slots with the oracle: the unweighted outputs of the
routes it computes (mode 0: ep.owner of the expert; mode 1: ep.route_owner
of the route) and its column blocks of the shared expert's down projection
(ep.shared_block_span).  ep.EPLayer all-reduces the slots and combines them
(routes in route order, then the shared partials in block order).  The
result must equal the same decomposition computed by one process bit for
bit, on both ranks, and the oracle's whole layer to fp32 rounding.  The
CUDA kernels are exercised by the GPU tests.  This test covers the host
logic of the N > 1 path: ownership, the slot layout, the shared-expert
block split, the all-reduce and the combine order."""
import os
import socket

import numpy as np
import pytest
import torch

HIDDEN, INTER, E, K, SI, T = 128, 64, 8, 3, 64, 3


def _layer():
    from oracle import oracle as O
    from warp_b200 import container as C
    rng = np.random.default_rng(77)
    books_f16 = rng.uniform(-0.3, 0.3, (9, 256, 8)).astype(np.float16).view(np.uint16)
    _, booksT = O.books_decode(books_f16)
    recs = []
    for e in range(E):
        blocks = [rng.integers(0, 256, C.index_bytes(M, N), dtype=np.uint8)
                  for M, N in ((INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER))]
        scales = [rng.uniform(0.01, 0.05, n).astype(np.float16).view(np.uint16)
                  for n in (INTER, INTER, HIDDEN)]
        recs.append(np.frombuffer(C.write_record(0, e, 0, blocks, scales, HIDDEN, INTER),
                                  np.uint8).copy())
    router = (rng.standard_normal((E, HIDDEN)) * 0.1).astype(np.float32)
    sh = {"group": 32, "bits": 4, "inter": SI}
    for k, (M, N) in (("gate", (SI, HIDDEN)), ("up", (SI, HIDDEN)), ("down", (HIDDEN, SI))):
        W = (rng.standard_normal((M, N)) * 0.02).astype(np.float32)
        sh[k + "_w"], sh[k + "_s"] = O.quant_q(W, 32, 4)
    xs = rng.standard_normal((T, HIDDEN)).astype(np.float32)
    return O, booksT, recs, router, sh, xs


class OracleMoE:
    """The MoELayer interface EPLayer drives, computed by the oracle."""

    def __init__(self, rank, size, mode):
        from warp_b200 import ep
        self.O, self.booksT, self.recs, self.router, self.sh, _ = _layer()
        self.rank, self.size, self.mode = rank, size, mode
        self.hidden = HIDDEN
        self.nb = ep.shared_blocks(SI, 32)
        self.w = None

    def slots(self, T, device=None):
        return torch.zeros(T, K + self.nb, HIDDEN)

    def _shared_partial(self, x, b):
        """The down projection over column block b of silu(gate) * up."""
        O, sh = self.O, self.sh
        rb_h, rb_i = HIDDEN // 2, SI // 2
        a = O.mvq_rows(sh["gate_w"], sh["gate_s"], x, SI, HIDDEN, 32, 4, rb_h)
        u = O.mvq_rows(sh["up_w"], sh["up_s"], x, SI, HIDDEN, 32, 4, rb_h)
        h = O.swiglu(a, u)
        cpb = SI // self.nb
        W = sh["down_w"].reshape(HIDDEN, rb_i)[:, b * cpb // 2:(b + 1) * cpb // 2].copy()
        S = sh["down_s"].reshape(HIDDEN, SI // 32)[:, b * cpb // 32:(b + 1) * cpb // 32].copy()
        return O.mvq_rows(W, S, h[b * cpb:(b + 1) * cpb], HIDDEN, cpb, 32, 4, cpb // 2)

    def forward_ep(self, x, slots):
        from warp_b200 import ep
        xs = x.numpy()
        self.w = []
        for t in range(xs.shape[0]):
            _, idx, w, acc = self.O.moe_layer(xs[t], HIDDEN, INTER, E, K, 1, self.router,
                                              self.recs, self.booksT)
            self.w.append(w)
            for j in range(K):
                r = ep.owner(int(idx[j]), self.size) if self.mode == 0 else \
                    ep.route_owner(t * K + j, self.size)
                if r == self.rank:
                    slots[t, j] = torch.from_numpy(acc[j])
            b0, b1 = ep.shared_block_span(self.nb, self.rank, self.size)
            for b in range(b0, b1):
                slots[t, K + b] = torch.from_numpy(self._shared_partial(xs[t], b))

    def combine(self, slots, residual=None, out=None):
        s = slots.numpy()
        res = np.empty((s.shape[0], HIDDEN), np.float32)
        for t in range(s.shape[0]):
            acc = np.zeros(HIDDEN, np.float32)
            for j in range(K):
                acc = acc + np.float32(self.w[t][j]) * s[t, j]
            shp = np.zeros(HIDDEN, np.float32)
            for b in range(self.nb):
                shp = shp + s[t, K + b]
            res[t] = acc + np.float32(1.0) * shp
        return torch.from_numpy(res)


def _rank_main(rank, size, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=size)
        from warp_b200 import ep
        O, booksT, recs, router, sh, xs = _layer()
        for mode in (0, 1):
            layer = ep.EPLayer(OracleMoE(rank, size, mode))
            got = layer.forward(torch.from_numpy(xs)).numpy()
            # one process computing every slot: the same decomposition
            one = OracleMoE(0, 1, mode)
            slots = one.slots(T)
            one.forward_ep(torch.from_numpy(xs), slots)
            want1 = one.combine(slots).numpy()
            np.testing.assert_array_equal(got.view(np.uint32), want1.view(np.uint32))
            for t in range(T):
                want, _, _, _ = O.moe_layer(xs[t], HIDDEN, INTER, E, K, 1, router, recs,
                                            booksT, sh)
                np.testing.assert_allclose(got[t], want, rtol=1e-5, atol=1e-6)
        # every rank ends with the same slots: one contributor each
        dist.barrier()
        q.put((rank, "ok"))
    except Exception as exc:                       # reported to the parent
        q.put((rank, repr(exc)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ownership_and_block_split():
    from warp_b200 import ep
    for size in (1, 2, 3, 8):
        owned = [ep.owned_experts(256, r, size) for r in range(size)]
        assert sorted(sum(owned, [])) == list(range(256))
        assert all(ep.owner(e, size) == r for r in range(size) for e in owned[r])
        routes = [[q for q in range(8 * 3) if ep.route_owner(q, size) == r] for r in range(size)]
        assert sorted(sum(routes, [])) == list(range(24))
        assert max(map(len, routes)) - min(map(len, routes)) <= 1
        for nb in (1, 2, 4, 8):
            spans = [ep.shared_block_span(nb, r, size) for r in range(size)]
            assert spans[0][0] == 0 and spans[-1][1] == nb
            assert all(spans[r][1] == spans[r + 1][0] for r in range(size - 1))
    assert ep.shared_blocks(2048, 32) == 8 and ep.shared_blocks(64, 32) == 2
    assert ep.shared_blocks(96, 32) == 1
    with pytest.raises(ValueError):
        ep.owned_experts(4, 0, 8)


def test_two_ranks_match_one_layer():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
