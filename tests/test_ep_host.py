"""The expert-parallel decomposition on CPU, world_size 2 over gloo.

Each rank computes its slots with the oracle: its own experts' unweighted
outputs (ep.owner), its share of the shared expert (ep.shared_tokens).
ep.EPLayer all-reduces the slots and combines them in route order. The
result must equal the oracle's whole layer bit for bit on both ranks.
The CUDA kernels are exercised by the GPU tests. This test covers the host
logic of the N > 1 path: ownership, the slot layout, the shared-expert
token split, the all-reduce and the combine order."""
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

    def __init__(self, rank, size):
        self.O, self.booksT, self.recs, self.router, self.sh, _ = _layer()
        self.rank, self.size = rank, size
        self.hidden = HIDDEN
        self.w = None

    def slots(self, T, device=None):
        return torch.zeros(T, K + 1, HIDDEN)

    def _shared(self, x):
        O, sh = self.O, self.sh
        rb_h, rb_i = HIDDEN // 2, SI // 2
        a = O.mvq_rows(sh["gate_w"], sh["gate_s"], x, SI, HIDDEN, 32, 4, rb_h)
        b = O.mvq_rows(sh["up_w"], sh["up_s"], x, SI, HIDDEN, 32, 4, rb_h)
        return O.mvq_rows(sh["down_w"], sh["down_s"], O.swiglu(a, b), HIDDEN, SI, 32, 4, rb_i)

    def forward_ep(self, x, slots):
        from warp_b200 import ep
        xs = x.numpy()
        self.w = []
        for t in range(xs.shape[0]):
            _, idx, w, acc = self.O.moe_layer(xs[t], HIDDEN, INTER, E, K, 1, self.router,
                                              self.recs, self.booksT)
            self.w.append(w)
            for j in range(K):
                if ep.owner(int(idx[j]), self.size) == self.rank:
                    slots[t, j] = torch.from_numpy(acc[j])
        t0, t1 = ep.shared_tokens(xs.shape[0], self.rank, self.size)
        for t in range(t0, t1):
            slots[t, K] = torch.from_numpy(self._shared(xs[t]))

    def combine(self, slots, residual=None, out=None):
        s = slots.numpy()
        res = np.empty((s.shape[0], HIDDEN), np.float32)
        for t in range(s.shape[0]):
            acc = np.zeros(HIDDEN, np.float32)
            for j in range(K):
                acc = acc + np.float32(self.w[t][j]) * s[t, j]
            res[t] = acc + np.float32(1.0) * s[t, K]
        return torch.from_numpy(res)


def _rank_main(rank, size, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=size)
        from warp_b200 import ep
        O, booksT, recs, router, sh, xs = _layer()
        layer = ep.EPLayer(OracleMoE(rank, size))
        got = layer.forward(torch.from_numpy(xs)).numpy()
        for t in range(T):
            want, _, _, _ = O.moe_layer(xs[t], HIDDEN, INTER, E, K, 1, router, recs, booksT, sh)
            np.testing.assert_array_equal(got[t].view(np.uint32), want.view(np.uint32))
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


def test_ownership_and_token_split():
    from warp_b200 import ep
    for size in (1, 2, 3, 8):
        owned = [ep.owned_experts(256, r, size) for r in range(size)]
        assert sorted(sum(owned, [])) == list(range(256))
        assert all(ep.owner(e, size) == r for r in range(size) for e in owned[r])
        for T in (1, 3, 8, 17):
            spans = [ep.shared_tokens(T, r, size) for r in range(size)]
            assert spans[0][0] == 0 and spans[-1][1] == T
            assert all(spans[r][1] == spans[r + 1][0] for r in range(size - 1))
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
