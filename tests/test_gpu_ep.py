"""Expert parallelism on the GPU.

* G ranks emulated on one GPU. Each rank's layer holds only its experts
  (ep.owned_experts) and runs warp_moe_layer_forward_ep. The slots are
  summed, standing in for the all-reduce, and warp_moe_layer_combine
  finishes. The output, routing and weights equal warp_moe_layer_forward on
  the whole bank bit for bit.
* Two real ranks over NCCL (two GPUs or more): ep.EPLayer on each rank
  equals the whole layer on that rank, bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _build(hidden, inter, E, seed, device, experts=None, shared=True, gate=False):
    from warp_b200 import synth
    bank = synth.random_bank(E, hidden, inter, seed, device=device, experts=experts)
    router = synth.router_matrix(E, hidden, seed + 1, device=device)
    sh = synth.shared_expert(hidden, inter, seed + 2, device=device) if shared else None
    sg = (torch.randn(hidden, generator=torch.Generator(device=device).manual_seed(seed + 3),
                      device=device) * 0.02) if gate else None
    return synth.SyntheticLayer(bank, router, sh, sg)


@pytest.mark.parametrize("mode", [0, 1])
@pytest.mark.parametrize("hidden,inter,E,K,T,G,shared,gate", [
    (256, 128, 16, 4, 1, 2, True, False),
    (256, 128, 16, 4, 4, 4, True, True),
    (384, 160, 12, 3, 5, 3, True, False),        # partial chunks, uneven splits
    (256, 128, 16, 4, 3, 1, False, False),       # route-list mode covering every route
    (2304, 1024, 32, 8, 2, 8, True, False),      # config 1 geometry
    (2304, 1024, 32, 8, 1, 8, True, False),      # one token over eight ranks
])
def test_emulated_ranks_match_one_gpu(cuda, hidden, inter, E, K, T, G, shared, gate, mode):
    """G ranks on one GPU, in both splits: mode 0 (each rank's bank holds
    the experts it owns) and mode 1 (whole bank on every rank, routes
    dealt).  Every slot has one contributor, the shared expert's column
    blocks are spread over the ranks, and the combine equals the one-GPU
    layer bit for bit."""
    from warp_b200 import ep
    seed = hidden + E + G
    full = _build(hidden, inter, E, seed, cuda, shared=shared, gate=gate)
    moe = full.moe(K, max_tokens=T)
    x = torch.randn(T, hidden, generator=torch.Generator().manual_seed(seed)).to(cuda)
    res = torch.randn(T, hidden, generator=torch.Generator().manual_seed(seed + 1)).to(cuda)
    want, widx, ww = moe.forward(x, residual=res, want_route=True)
    nb = ep.shared_blocks(inter, 32) if shared else 0
    total = torch.zeros(T, K + nb, hidden, device=cuda)
    layers = []
    for r in range(G):
        experts = ep.owned_experts(E, r, G) if mode == 0 else None
        part = _build(hidden, inter, E, seed, cuda, experts=experts, shared=shared, gate=gate)
        m = part.moe(K, max_tokens=T, ep_rank=r, ep_size=G, ep_mode=mode)
        assert m.slots_per_token() == K + nb
        slots = torch.full((T, K + nb, hidden), float("nan"), device=cuda)
        idx, w = m.forward_ep(x, slots, want_route=True)
        assert torch.equal(idx, widx) and torch.equal(w, ww)
        # a rank writes every slot: its own values, zeros elsewhere
        if mode == 0:
            own = torch.tensor([[ep.owner(int(e), G) == r for e in row] for row in idx.cpu()],
                               device=cuda)
        else:
            own = torch.tensor([[ep.route_owner(t * K + j, G) == r for j in range(K)]
                                for t in range(T)], device=cuda)
        assert not torch.isnan(slots).any()
        assert (slots[:, :K][~own] == 0).all()
        if shared:
            b0, b1 = ep.shared_block_span(nb, r, G)
            other = [b for b in range(nb) if not b0 <= b < b1]
            if other:
                assert (slots[:, [K + b for b in other]] == 0).all()
        total += slots
        layers.append((part, m))
    got = layers[0][1].combine(total, residual=res)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    for _, m in layers:
        m.status()
        m.close()
    moe.close()


def test_forward_refuses_an_ep_layer(cuda):
    from warp_b200 import ep, ffi
    part = _build(256, 128, 16, 5, cuda, experts=ep.owned_experts(16, 1, 2))
    m = part.moe(4, ep_rank=1, ep_size=2)
    with pytest.raises(ffi.WarpError):
        m.forward(torch.zeros(1, 256, device=cuda))
    m.close()


def _nccl_rank(rank, size, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=size,
                                timeout=datetime.timedelta(seconds=60))
        from warp_b200 import ep
        hidden, inter, E, K, T = 512, 256, 16, 4, 2
        full = _build(hidden, inter, E, 9, dev)
        want = full.moe(K, max_tokens=T)
        part = _build(hidden, inter, E, 9, dev, experts=ep.owned_experts(E, rank, size))
        layer = ep.EPLayer(part.moe(K, max_tokens=T, ep_rank=rank, ep_size=size))
        whole = _build(hidden, inter, E, 9, dev)
        dealt = ep.EPLayer(whole.moe(K, max_tokens=T, ep_rank=rank, ep_size=size, ep_mode=1))
        x = torch.randn(T, hidden, generator=torch.Generator().manual_seed(3)).to(dev)
        got = layer.forward(x)
        got1 = dealt.forward(x)
        ref = want.forward(x)
        torch.cuda.synchronize()
        ok = torch.equal(got.view(torch.int32), ref.view(torch.int32)) and \
            torch.equal(got1.view(torch.int32), ref.view(torch.int32))
        dist.barrier()
        q.put((rank, "ok" if ok else "mismatch"))
    except Exception as exc:                        # reported to the parent
        q.put((rank, repr(exc)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_nccl_two_ranks(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_nccl_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert results == {0: "ok", 1: "ok"}, results
