"""The WARP container pieces the expert path reads: WEXP expert records and
codebook records (docs/FORMAT.md, src/waste_format.h).

The layout is the reference's and must stay byte-compatible, so this module
states it once:

* expert record (waste_format.h:98-130): a 48-byte header ``<IHHBBHHHIIIIIIII``
  (magic 'WEXP', layer, expert_id, fmt=4 VQ3R, flags, codebook_id,
  lowrank_id=0, reserved, rec_4k_blocks, gate_off, up_off, down_off,
  chan_corr_off, crc32, 2 x reserved), then the gate, up and down index
  blocks, then the fp16 per-row scales of the three matrices, zero-padded to
  a multiple of 4 KiB (convert.py:942-977);
* index block (convert.py:777-792, FORMAT.md "Index layout is blocked by 64
  rows"): ``[ceil(M/64)][N/8][64][3]`` uint8, padding rows zero;
* codebook record (waste_format.h:139-150): a 16-byte header ``<IHBBII``
  (magic 'WCBK', codebook_id, fmt, vec_dim=8, n_entries=256, 0) and
  256 x 8 fp16.  A layer's nine books are gate, up, down x 3 stages from its
  codebook base (convert.py:1352-1357).
"""
import struct
import zlib

import numpy as np

MAGIC_EXPERT = 0x50584557
MAGIC_CODEBOOK = 0x4B424357
FMT_VQ3R = 4
ALIGN = 4096
VEC = 8
ENTRIES = 256
STAGES = 3
BLOCK = 64
HDR = struct.Struct("<IHHBBHHHIIIIIIII")
CBK = struct.Struct("<IHBBII")
assert HDR.size == 48 and CBK.size == 16


def index_bytes(M, N):
    """Bytes of one blocked VQ3R index matrix [M][N]."""
    return ((M + BLOCK - 1) // BLOCK) * (N // VEC) * BLOCK * STAGES


def record_layout(hidden, inter):
    """Offsets of one expert record with gate/up [inter][hidden] and down
    [hidden][inter]: (gate_off, up_off, down_off, scale_off, payload_end,
    rec_bytes)."""
    g = HDR.size
    u = g + index_bytes(inter, hidden)
    d = u + index_bytes(inter, hidden)
    s = d + index_bytes(hidden, inter)
    end = s + 2 * (2 * inter + hidden)
    rec = (end + ALIGN - 1) // ALIGN * ALIGN
    return g, u, d, s, end, rec


def packed_bytes_per_expert(hidden, inter):
    """Index bytes plus fp16 scales of one expert: 3*inter*hidden*3/8 +
    2*(2*inter + hidden) — what one routed (token, expert) reads."""
    return 3 * inter * hidden * 3 // 8 + 2 * (2 * inter + hidden)


def block_indices(codes, M, N):
    """codes [M*N/8][3] (vector v of row r at r*N/8 + v) -> blocked bytes."""
    nv = N // VEC
    t = np.asarray(codes, np.uint8).reshape(M, nv, STAGES)
    pad = (-M) % BLOCK
    if pad:
        t = np.concatenate([t, np.zeros((pad, nv, STAGES), np.uint8)], 0)
    nb = t.shape[0] // BLOCK
    return np.ascontiguousarray(t.reshape(nb, BLOCK, nv, STAGES).transpose(0, 2, 1, 3)).reshape(-1)


def unblock_indices(blocked, M, N):
    """Inverse of block_indices: -> codes [M*N/8][3]."""
    nv = N // VEC
    nb = (M + BLOCK - 1) // BLOCK
    t = np.asarray(blocked, np.uint8).reshape(nb, nv, BLOCK, STAGES).transpose(0, 2, 1, 3)
    return np.ascontiguousarray(t.reshape(nb * BLOCK, nv, STAGES)[:M]).reshape(-1, STAGES)


def write_record(layer, eid, cb_base, blocked, scales, hidden, inter):
    """One 4 KiB-aligned WEXP record from three blocked index arrays (gate, up,
    down) and three fp16 scale arrays (as uint16)."""
    g, u, d, s, end, rec = record_layout(hidden, inter)
    body = b"".join(np.asarray(b, np.uint8).tobytes() for b in blocked)
    assert len(body) == s - g, "index blocks do not match the geometry"
    body += b"".join(np.asarray(x, np.uint16).tobytes() for x in scales)
    assert HDR.size + len(body) == end
    crc = zlib.crc32(body) & 0xFFFFFFFF
    hdr = HDR.pack(MAGIC_EXPERT, layer, eid, FMT_VQ3R, 0, cb_base, 0, 0, rec // ALIGN,
                   g, u, d, s, crc, 0, 0)
    return hdr + body + b"\0" * (rec - end)


def parse_header(buf):
    f = HDR.unpack(bytes(buf[:HDR.size]))
    return dict(magic=f[0], layer=f[1], expert_id=f[2], fmt=f[3], flags=f[4],
                codebook_id=f[5], lowrank_id=f[6], rec_4k_blocks=f[8], gate_off=f[9],
                up_off=f[10], down_off=f[11], chan_corr_off=f[12], crc32=f[13])


def codebook_bytes(books_f16, cb_base=0):
    """books_f16: [n][256][8] fp16 (or uint16) -> codebooks.bin records."""
    h = np.asarray(books_f16).view(np.uint16).reshape(-1, ENTRIES * VEC)
    out = bytearray()
    for i, b in enumerate(h):
        out += CBK.pack(MAGIC_CODEBOOK, (cb_base + i) & 0xFFFF, FMT_VQ3R, VEC, ENTRIES, 0)
        out += b.tobytes()
    return bytes(out)


def parse_codebooks(data):
    """codebooks.bin bytes -> [n][256][8] uint16 (fp16 bits)."""
    rec = CBK.size + ENTRIES * VEC * 2
    n = len(data) // rec
    out = np.empty((n, ENTRIES, VEC), np.uint16)
    for i in range(n):
        out[i] = np.frombuffer(data, np.uint16, ENTRIES * VEC,
                               i * rec + CBK.size).reshape(ENTRIES, VEC)
    return out


def books_decode(books_f16):
    """fp16 codebooks -> (books [n][256][8], booksT [n][8][256]) fp32 with
    subnormals flushed to zero, as the engine's loader decodes them
    (model.c:2911-2941)."""
    h = np.asarray(books_f16).view(np.uint16).astype(np.uint32)
    sign = (h >> 15) << 31
    e = (h >> 10) & 0x1F
    man = h & 0x3FF
    bits = np.where(e != 0, sign | ((e + 112) << 23) | (man << 13), sign).astype(np.uint32)
    books = bits.view(np.float32).reshape(-1, ENTRIES, VEC)
    return np.ascontiguousarray(books), np.ascontiguousarray(books.transpose(0, 2, 1))
