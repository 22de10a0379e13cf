"""Seeded synthetic experts in the container layout, built on the device.

Two recipes, both producing real WEXP records and fp16 codebooks:

* ``encoded``: Gaussian weights N(0, std) from a seed, codebooks trained the
  way convert.py's convert_layer trains them (convert.py:1353-1365: up to 12
  sampled experts, 300k row-normalized vectors, residual k-means with 10 Lloyd
  iterations per stage, train_codebooks convert.py:745-762), and every matrix
  encoded by warp_vq_encode (the GPU port of waste_vq_encode, bit-exact) after
  quantize_vq's per-row amax normalization (convert.py:821-851).
* ``random``: codes, codebooks and scales drawn at random, the recipe of the
  reference's own tools/make_test_container.py (write_expert, :461-497;
  codebooks U(-0.3, 0.3), scales U(0.01, 0.05)).  The gather kernels cost the
  same whatever the codes are, which is why the throughput configs use it for
  containers far larger than anything the encoder should run on per bench.

Trunk/shared tensors are quantized with quantize_q4g / quantize_q8g
(convert.py:893-925), restated in torch (same ops, so the same bytes).
"""
import ctypes
import math

import numpy as np
import torch

from . import container as C

TRAIN_VECTORS = 300000
CB_SAMPLE = 12


# ------------------------------------------------------------ quantizers --

def assign(X, Cb, chunk=1 << 20):
    """Nearest centroid by the ||c||^2 - 2 x.c expansion (convert.py:766-775)."""
    cn = (Cb * Cb).sum(1)
    out = torch.empty(X.shape[0], dtype=torch.long, device=X.device)
    for s in range(0, X.shape[0], chunk):
        x = X[s:s + chunk]
        d = cn.unsqueeze(0) - 2.0 * (x @ Cb.T)
        out[s:s + chunk] = d.argmin(1)
    return out


def train_codebooks(X, n_stages, dev, iters=10, sample=TRAIN_VECTORS, seed=0,
                    entries=C.ENTRIES):
    """Residual k-means, one codebook per stage (convert.py:745-762)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    books = []
    resid = X[torch.randperm(X.shape[0], generator=g)[:sample]].to(dev)
    for _ in range(n_stages):
        Cb = resid[torch.randperm(resid.shape[0], generator=g)[:entries]].clone()
        for _ in range(iters):
            idx = assign(resid, Cb)
            for j in range(entries):
                m = idx == j
                if m.any():
                    Cb[j] = resid[m].mean(0)
        books.append(Cb)
        resid = resid - Cb[assign(resid, Cb)]
    return books


def quantize_q(W, group, bits):
    """quantize_q4g / quantize_q8g (convert.py:893-925) for [rows][N] with N a
    multiple of group -> (payload uint8 [rows][N*bits/8], scales fp16 bits as
    int16 [rows][N/group])."""
    X = W.float()
    rows, N = X.shape
    Xg = X.view(rows, -1, group)
    lim = 7.0 if bits == 4 else 127.0
    scale = Xg.abs().amax(-1, keepdim=True).clamp(min=1e-8) / lim
    if bits == 4:
        Q = torch.clamp(torch.round(Xg / scale), -8, 7).to(torch.int32).flatten()
        nib = (Q + 8).to(torch.uint8) & 0x0F
        packed = (nib[0::2] | (nib[1::2] << 4)).contiguous().view(rows, N // 2)
    else:
        packed = torch.clamp(torch.round(Xg / scale), -127, 127).to(torch.int8) \
            .view(torch.uint8).reshape(rows, N)
    s16 = scale.half().reshape(rows, -1).contiguous().view(torch.int16)
    return packed.contiguous(), s16


# ------------------------------------------------------------ VQ3R experts --

def _encode_matrix(W, books_f32):
    """quantize_vq: per-row amax scale, X = W/scale, residual codes."""
    from .ops import vq_encode
    scale = W.abs().amax(-1, keepdim=True).clamp(min=1e-8)
    X = (W / scale).reshape(-1, C.VEC).contiguous().float()
    codes = vq_encode(X, books_f32)
    return codes, scale.half().flatten()


def _block(codes, M, N):
    """block_indices on the device: [M*N/8][3] -> [ceil(M/64)*N/8*64*3]."""
    nv = N // C.VEC
    t = codes.view(M, nv, C.STAGES)
    pad = (-M) % C.BLOCK
    if pad:
        t = torch.cat([t, torch.zeros(pad, nv, C.STAGES, dtype=t.dtype, device=t.device)], 0)
    nb = t.shape[0] // C.BLOCK
    return t.view(nb, C.BLOCK, nv, C.STAGES).permute(0, 2, 1, 3).contiguous().view(-1)


def _header(layer, eid, cb_base, hidden, inter, crc=0):
    g, u, d, s, end, rec = C.record_layout(hidden, inter)
    return C.HDR.pack(C.MAGIC_EXPERT, layer, eid, C.FMT_VQ3R, 0, cb_base, 0, 0,
                      rec // C.ALIGN, g, u, d, s, crc, 0, 0)


class ExpertBank:
    """E expert records of one layer, resident on the device, plus the
    layer's nine codebooks (fp16 bits and decoded fp32)."""

    def __init__(self, bank, rec_bytes, books_f16, hidden, inter, n_experts, layer=0,
                 cb_base=0, ids=None):
        self.bank, self.rec_bytes = bank, rec_bytes
        self.hidden, self.inter, self.E = hidden, inter, n_experts
        # the expert ids of the records, in order (all E unless expert-parallel)
        self.ids = list(range(n_experts)) if ids is None else list(ids)
        self.layer, self.cb_base = layer, cb_base
        self.books_f16 = books_f16                  # torch int16 [9][256][8] (cpu)
        books, booksT = C.books_decode(books_f16.numpy().view(np.uint16))
        dev = bank.device
        self.books = torch.from_numpy(books).to(dev)
        self.booksT = torch.from_numpy(booksT).to(dev)

    def record(self, e):
        return self.bank[e * self.rec_bytes:(e + 1) * self.rec_bytes]

    def packed_bytes_per_expert(self):
        return C.packed_bytes_per_expert(self.hidden, self.inter)


def encoded_bank(n_experts, hidden, inter, seed, std=0.02, device="cuda", layer=0,
                 cb_base=0, gen_device="cpu", weights_out=None):
    """Gaussian experts encoded with trained codebooks (the cfg1 recipe).

    Weights come from torch.Generator(gen_device).manual_seed(seed), expert by
    expert, gate then up then down; weights_out (a list) receives them on the
    CPU when given (for oracle checks at small sizes)."""
    g, u, d, s, end, rec = C.record_layout(hidden, inter)
    gen = torch.Generator(device=gen_device).manual_seed(seed)
    shapes = [(inter, hidden), (inter, hidden), (hidden, inter)]

    def weights(e):
        return [torch.randn(M, N, generator=gen, device=gen_device) * std for M, N in shapes]

    # Codebooks: sample row-normalized vectors from up to CB_SAMPLE experts
    # (convert.py:1353-1365).  Weights are regenerated from the seed when the
    # bank is written, so every expert's draw is replayed in order.
    all_w = [weights(e) for e in range(n_experts)]
    sample_ids = list(range(0, n_experts, max(1, n_experts // CB_SAMPLE)))[:CB_SAMPLE]
    per = max(1, TRAIN_VECTORS // len(sample_ids))
    books32 = []
    for k in range(3):
        chunks = []
        for e in sample_ids:
            W = all_w[e][k]
            sc = W.abs().amax(-1, keepdim=True).clamp(min=1e-8)
            V = (W / sc).reshape(-1, C.VEC)
            gg = torch.Generator().manual_seed(1234 + e)
            chunks.append(V[torch.randperm(V.shape[0], generator=gg)[:per]].cpu())
        X = torch.cat(chunks)
        books32 += train_codebooks(X, C.STAGES, torch.device(device))
    books32 = [b.float() for b in books32]
    books_f16 = torch.stack([b.detach().cpu().half() for b in books32]).view(torch.int16)
    bank = torch.zeros(n_experts * rec, dtype=torch.uint8, device=device)
    for e in range(n_experts):
        W3 = all_w[e]
        if weights_out is not None:
            weights_out.append([w.cpu() for w in W3])
        blocks, scales = [], []
        for k, (M, N) in enumerate(shapes):
            Bk = torch.stack(books32[3 * k:3 * k + 3]).to(device).contiguous()
            codes, sc = _encode_matrix(W3[k].to(device), Bk)
            blocks.append(_block(codes, M, N))
            scales.append(sc.view(torch.uint8))
        r = bank[e * rec:(e + 1) * rec]
        body = torch.cat(blocks + scales)
        r[g:end] = body
        crc = _crc32(body)
        r[:C.HDR.size] = torch.frombuffer(bytearray(_header(layer, e, cb_base, hidden, inter, crc)),
                                          dtype=torch.uint8).to(device)
    eb = ExpertBank(bank, rec, books_f16, hidden, inter, n_experts, layer, cb_base)
    eb.books32 = torch.stack([b.cpu() for b in books32])    # the encoder's fp32 books
    return eb


def _crc32(t):
    import zlib
    return zlib.crc32(t.cpu().numpy().tobytes()) & 0xFFFFFFFF


def random_bank(n_experts, hidden, inter, seed, device="cuda", layer=0, cb_base=0,
                experts=None):
    """Random codes, codebooks U(-0.3, 0.3) and scales U(0.01, 0.05)
    (make_test_container.py:461-497, 1066-1090), generated on the device.
    Record checksums are left 0 (the engine checks them only on request).

    experts: the expert ids this bank holds, in order (default: all
    n_experts).  Each record depends only on (seed, expert id), so the bank of
    an expert-parallel rank holds exactly the records of the whole bank it
    owns."""
    g, u, d, s, end, rec = C.record_layout(hidden, inter)
    ids = list(range(n_experts)) if experts is None else [int(e) for e in experts]
    bank = torch.empty(len(ids) * rec, dtype=torch.uint8, device=device)
    view = bank.view(len(ids), rec)
    for x, e in enumerate(ids):
        gen = torch.Generator(device=device).manual_seed(seed * 1000003 + e)
        view[x, g:s] = torch.randint(0, 256, (s - g,), dtype=torch.uint8, device=device,
                                     generator=gen)
        sc = torch.rand((end - s) // 2, device=device, generator=gen) * 0.04 + 0.01
        view[x, s:end] = sc.half().view(torch.uint8)
        view[x, end:] = 0
    hdrs = np.frombuffer(b"".join(_header(layer, e, cb_base, hidden, inter) for e in ids),
                         np.uint8).reshape(len(ids), -1)
    view[:, :C.HDR.size] = torch.from_numpy(hdrs.copy()).to(device)
    cg = torch.Generator(device="cpu").manual_seed(seed ^ 0x5EED)
    books_f16 = (torch.rand(9, C.ENTRIES, C.VEC, generator=cg) * 0.6 - 0.3).half().view(torch.int16)
    return ExpertBank(bank, rec, books_f16, hidden, inter, n_experts, layer, cb_base, ids)


# ------------------------------------------------------------ the layer --

class SyntheticLayer:
    """Everything one MoE layer of a config needs, on the device."""

    def __init__(self, bank, router, shared=None, shared_gate=None):
        self.bank = bank
        self.router = router
        self.shared = shared
        self.shared_gate = shared_gate

    def packed_bytes(self, n_distinct_experts):
        """HBM bytes one token reads: routed records + shared Q4/Q8 + router."""
        b = n_distinct_experts * self.bank.packed_bytes_per_expert()
        if self.shared:
            for k in ("gate", "up", "down"):
                b += self.shared[k + "_w"].numel() + 2 * self.shared[k + "_s"].numel()
        b += 4 * self.router.numel()
        if self.shared_gate is not None:
            b += 4 * self.shared_gate.numel()
        return b

    def moe(self, top_k, renorm=True, max_tokens=1, tile_bank=True, ep_rank=0, ep_size=1,
            prefill_tokens=0, **router):
        """The device layer.  With tile_bank (default) the bank is re-tiled in
        place: take host_records() first if the container layout is needed.
        ep_rank/ep_size: the bank holds that rank's experts (random_bank's
        experts=ep.owned_experts(...))."""
        from .ops import MoELayer
        return MoELayer(self.bank.bank, self.bank.rec_bytes, self.bank.books,
                        self.bank.booksT, self.router, self.bank.hidden, self.bank.inter,
                        self.bank.E, top_k, renorm, self.shared, self.shared_gate,
                        max_tokens, tile_bank, ep_rank, ep_size, prefill_tokens, **router)

    def host_records(self):
        """The bank's records in container layout, as numpy arrays (host copy)."""
        raw = self.bank.bank.cpu().numpy()
        rb = self.bank.rec_bytes
        return [raw[x * rb:(x + 1) * rb].copy() for x in range(len(self.bank.ids))]


def shared_expert(hidden, inter, seed, std=0.02, group=32, bits=4, device="cuda"):
    """A Q4G/Q8G shared expert from N(0, std) weights."""
    gen = torch.Generator(device=device).manual_seed(seed)
    out = {"inter": inter, "group": group, "bits": bits}
    for k, (M, N) in (("gate", (inter, hidden)), ("up", (inter, hidden)),
                      ("down", (hidden, inter))):
        W = torch.randn(M, N, generator=gen, device=device) * std
        q, s = quantize_q(W, group, bits)
        out[k + "_w"], out[k + "_s"] = q, s
    return out


def router_matrix(n_experts, hidden, seed, std=0.02, device="cuda"):
    """fp32 [E][hidden] router drawn N(0, std)."""
    gen = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(n_experts, hidden, generator=gen, device=device) * std).contiguous()


# Routing skew.  Logit offsets b_e = -1.1 * ZIPF_KAPPA * sigma * ln(rank_e), sigma
# the std of a router logit (std * sqrt(hidden) for unit-variance tokens),
# make the expert a token ranks first follow Zipf(1.1) over a random
# popularity order: a simulation of 200k tokens at 256 experts / top-8
# fits exponent -1.09 over the 64 most popular experts at this kappa
# (offset 0.70 for sigma 1.69).
ZIPF_KAPPA = 0.4135
# u-component of a zipf_tokens token before RMSNorm, in units of sqrt(hidden)
ZIPF_A = 0.25


def zipf_direction(hidden, seed):
    """The unit vector u that carries the offsets (seeded, shared by every
    layer's router and every token)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    u = torch.randn(hidden, generator=g, dtype=torch.float64)
    return (u / u.norm()).float()


def zipf_router(n_experts, hidden, seed, u, a, s=1.1, std=0.02, device="cuda"):
    """fp32 [E][hidden] router whose logits on zipf_tokens are N(0, sigma^2)
    noise plus the offsets above: rows N(0, std) with their u-component
    removed, plus (b_e / a') u, where a' = a / rms(token) is the u-component
    a token has after RMSNorm.  Returns (router, popularity ranks)."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    W = torch.randn(n_experts, hidden, generator=gen) * std
    W -= torch.outer(W @ u, u)
    rank = torch.randperm(n_experts, generator=gen) + 1          # 1 = most popular
    sigma = std * math.sqrt(hidden)
    b = -s * ZIPF_KAPPA * sigma * torch.log(rank.double()).float()
    a_norm = a / math.sqrt((hidden - 1 + a * a) / hidden)
    W += torch.outer(b / a_norm, u)
    return W.to(device).contiguous(), rank


def zipf_tokens(n, T, hidden, u, a, seed, device="cuda"):
    """n steps of T decode tokens: N(0, 1) with the u-component replaced by a,
    [n][T][hidden] fp32."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    z = torch.randn(n, T, hidden, generator=gen)
    z -= (z @ u)[..., None] * u
    return (z + a * u).to(device)
