"""Seeded synthetic inputs in the reference's on-disk formats.

Writes what the reference's converter writes, so the same bytes can be fed to
the reference CPU engine and to this backend:

* expert records — the 48-byte ``waste_expert_hdr`` then gate | up | down
  index streams in the blocked layout ``[M/64][N/8][64][stages]`` (rows
  zero-padded to whole blocks), then one f16 scale per output row of gate,
  up and down, padded to 4 KiB (sqliteai/warp src/waste_format.h:98-132,
  docs/FORMAT.md:194-208, tools/convert.py:297-312 block_indices,
  tools/convert.py:457 write_expert_record);
* codebooks — ``n_books`` books of 256 entries x 8 f16 (codebooks.bin
  payload, src/waste_format.h:139-150);
* VQ4P records (``stages=4``; src/waste_format.h:57) — four stages of
  64-entry books, the four 6-bit indices of a row and position packed
  little-endian into three bytes (tools/convert.py:315-337), so the index
  streams have the same size as VQ3R's; any three bytes are a valid
  packing, so uniform random bytes are uniform indices;
* Q8G trunk rows — int8 rows padded to whole groups of 128 plus one f16
  scale per group (src/model.c:265-320 layout).

Distributions follow the benchmark configs: codebook entries N(0, 0.02^2),
indices uniform, x N(0, 1) rounded to bf16 and held in fp32, router rows
N(0, 1/hidden) so logits are about N(0, 1).
"""
from __future__ import annotations

import struct
import zlib
from dataclasses import dataclass, field

import numpy as np

MAGIC_EXPERT = 0x50584557
FMT_VQ3R, FMT_VQ2R, FMT_VQ4P = 4, 5, 8
ALIGN = 4096
HDR_SIZE = 48
HDR_FMT = "<IHHBBHHHIIIIIIII"      # waste_expert_hdr, src/waste_format.h:98-132
VEC_DIM, ENTRIES, BLOCK = 8, 256, 64
ENTRIES_VQ4P = 64
GROUP = 128


def f16_bits(a: np.ndarray) -> np.ndarray:
    return np.asarray(a, dtype=np.float32).astype(np.float16).view(np.uint16)


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even), returned as fp32."""
    u = np.asarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def flush_f16(raw: np.ndarray) -> np.ndarray:
    """The engine's codebook decode (src/model.c:1278-1287): sign kept,
    exponent 0 flushed to zero, exponent 31 not special-cased."""
    h = np.asarray(raw, dtype=np.uint16).astype(np.uint32)
    sign = (h >> 15) << 31
    e = (h >> 10) & 0x1F
    man = h & 0x3FF
    bits = np.where(e != 0, sign | ((e + 112) << 23) | (man << 13), sign)
    return bits.astype(np.uint32).view(np.float32)


def codebooks(rng: np.random.Generator, n_books: int, std: float = 0.02,
              entries: int = ENTRIES) -> np.ndarray:
    """Raw f16 codebook entries [n_books][entries][8] as uint16."""
    return f16_bits(rng.normal(0.0, std, size=(n_books, entries, VEC_DIM)))


def row_bytes(stages: int) -> int:
    """Index bytes per row and vector position: one per stage, or three
    for VQ4P's four packed 6-bit indices."""
    return 3 if stages == 4 else stages


def fmt_of(stages: int) -> int:
    return {2: FMT_VQ2R, 3: FMT_VQ3R, 4: FMT_VQ4P}[stages]


def unpack_p6(b: np.ndarray) -> np.ndarray:
    """[..., 3] packed VQ4P bytes -> [..., 4] 6-bit indices."""
    b = np.asarray(b, dtype=np.uint32)
    p = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16)
    return np.stack([(p >> (6 * s)) & 63 for s in range(4)], axis=-1).astype(np.uint8)


def block_indices(idx: np.ndarray) -> np.ndarray:
    """[M][N/8][stages] uint8 -> blocked bytes [ceil(M/64)][N/8][64][stages]."""
    M, nv, st = idx.shape
    nb = (M + BLOCK - 1) // BLOCK
    pad = np.zeros((nb * BLOCK, nv, st), dtype=np.uint8)
    pad[:M] = idx
    return np.ascontiguousarray(pad.reshape(nb, BLOCK, nv, st).transpose(0, 2, 1, 3)).reshape(-1)


def unblock_indices(blob: np.ndarray, M: int, N: int, stages: int) -> np.ndarray:
    nv = N // VEC_DIM
    nb = (M + BLOCK - 1) // BLOCK
    rb = row_bytes(stages)
    a = np.asarray(blob, dtype=np.uint8)[: nb * nv * BLOCK * rb]
    return a.reshape(nb, nv, BLOCK, rb).transpose(0, 2, 1, 3).reshape(nb * BLOCK, nv, rb)[:M]


def random_matrix(rng: np.random.Generator, M: int, N: int, stages: int = 3,
                  scale_lo: float = 0.5, scale_hi: float = 1.5):
    """One VQ matrix: blocked index bytes and f16 row scales (uint16)."""
    rb = row_bytes(stages)
    idx = random_bytes(rng, M * (N // VEC_DIM) * rb).reshape(M, N // VEC_DIM, rb)
    scales = f16_bits(rng.uniform(scale_lo, scale_hi, size=M))
    return block_indices(idx), scales


def index_bytes(M: int, N: int, stages: int) -> int:
    return ((M + BLOCK - 1) // BLOCK) * (N // VEC_DIM) * BLOCK * row_bytes(stages)


def record_bytes(inter: int, lat: int, stages: int) -> int:
    body = 2 * index_bytes(inter, lat, stages) + index_bytes(lat, inter, stages)
    body += 2 * (2 * inter + lat)
    return ((HDR_SIZE + body + ALIGN - 1) // ALIGN) * ALIGN


def expert_record(rng: np.random.Generator, layer: int, eid: int, cb_base: int,
                  inter: int, lat: int, stages: int = 3,
                  scale_lo: float = 0.5, scale_hi: float = 1.5) -> bytes:
    """One expert record: header, gate | up | down indices, scales, padding."""
    parts, offsets, off = [], [], HDR_SIZE
    for (M, N) in ((inter, lat), (inter, lat), (lat, inter)):
        b = random_bytes(rng, index_bytes(M, N, stages))
        if M % BLOCK:      # padding rows stay zero, as block_indices writes them
            b = b.reshape((M + BLOCK - 1) // BLOCK, N // VEC_DIM, BLOCK, row_bytes(stages))
            b[-1, :, M % BLOCK:, :] = 0
            b = b.reshape(-1)
        offsets.append(off)
        parts.append(b.tobytes())
        off += b.size
    corr_off = off
    for M in (inter, inter, lat):
        s = f16_bits(rng.uniform(scale_lo, scale_hi, size=M)).tobytes()
        parts.append(s)
        off += len(s)
    body = b"".join(parts)
    total = HDR_SIZE + len(body)
    blocks = (total + ALIGN - 1) // ALIGN
    fmt = fmt_of(stages)
    hdr = struct.pack(HDR_FMT, MAGIC_EXPERT, layer, eid, fmt, 0, cb_base, 0, 0, blocks,
                      offsets[0], offsets[1], offsets[2], corr_off,
                      zlib.crc32(body) & 0xFFFFFFFF, 0, 0)
    return hdr + body + b"\0" * (blocks * ALIGN - total)


def parse_header(rec: bytes | np.ndarray) -> dict:
    h = struct.unpack(HDR_FMT, bytes(rec[:HDR_SIZE]))
    keys = ("magic", "layer", "expert_id", "fmt", "flags", "codebook_id", "lowrank_id",
            "reserved0", "rec_4k_blocks", "gate_off", "up_off", "down_off",
            "chan_corr_off", "crc32", "r1", "r2")
    return dict(zip(keys, h))


def q8g(rng: np.random.Generator, rows: int, cols: int, s_lo: float, s_hi: float):
    """Q8G rows (int8, padded to whole groups) and f16 group scales."""
    ng = (cols + GROUP - 1) // GROUP
    q = rng.integers(-127, 128, size=(rows, ng * GROUP), dtype=np.int8)
    if cols % GROUP:
        q[:, cols:] = 0
    s = f16_bits(rng.uniform(s_lo, s_hi, size=(rows, ng)))
    return q, s


def trunk_tensor(rng: np.random.Generator, rows: int, cols: int, bits: int, group: int = GROUP):
    """A quantised trunk tensor in the engine's layout (src/model.c:601-610):
    (raw row bytes [rows][rowbytes] uint8, f16 group scales [rows][ng],
    rowbytes). Q8G/Q4G rows are ng*group*bits/8 bytes, Q3G rows a 3-bit
    bitstream plus one guard byte. Padding past `cols` is zero."""
    ng = (cols + group - 1) // group
    if bits == 3:
        rowbytes = (ng * group * 3 + 7) // 8 + 1
    else:
        rowbytes = ng * group * bits // 8
    raw = rng.integers(0, 256, size=(rows, rowbytes), dtype=np.uint8)
    if bits == 8 and cols % group:
        raw[:, cols:] = 0
    s = f16_bits(rng.uniform(2e-4, 2e-3, size=(rows, ng)))
    return raw, s, rowbytes


@dataclass
class MoELayer:
    """One Kimi-Linear-shaped MoE layer, as the engine holds it after load."""
    layer: int
    hidden: int
    inter: int
    n_experts: int
    top_k: int
    renorm: int
    routed_scale: float
    stages: int
    cb_base: int
    books_raw: np.ndarray            # [n_books][256 (64 for VQ4P)][8] uint16
    router: np.ndarray               # [E][hidden] f32
    bias: np.ndarray | None          # [E] f32
    bank: np.ndarray                 # E * rec_bytes uint8
    rec_bytes: int
    shared_inter: int
    sh: dict = field(default_factory=dict)   # gate/up/down (q, s)
    act_situ: int = 0                # 1: K3's SiTU in place of SiLU(g)*u
    situ_beta: float = 0.0
    situ_lbeta: float = 0.0

    @property
    def books(self) -> np.ndarray:
        return flush_f16(self.books_raw)

    @property
    def n_books(self) -> int:
        return self.books_raw.shape[0]

    def record(self, e: int) -> np.ndarray:
        return self.bank[e * self.rec_bytes:(e + 1) * self.rec_bytes]

    def matrix(self, e: int, kind: int):
        """(blocked index bytes, f16 scales, M, N) of gate(0)/up(1)/down(2)."""
        rec = self.record(e)
        h = parse_header(rec)
        M, N = ((self.inter, self.hidden), (self.inter, self.hidden),
                (self.hidden, self.inter))[kind]
        off = (h["gate_off"], h["up_off"], h["down_off"])[kind]
        idx = rec[off:off + index_bytes(M, N, self.stages)]
        s0 = h["chan_corr_off"] + 2 * (0, self.inter, 2 * self.inter)[kind]
        sc = rec[s0:s0 + 2 * M].view(np.uint16)
        return idx, sc, M, N


def random_bytes(rng: np.random.Generator, n: int) -> np.ndarray:
    """n uniform bytes from the generator's raw 64-bit stream (the fastest
    path numpy offers; PCG64 output is stable across numpy versions)."""
    return rng.bit_generator.random_raw((n + 7) // 8).view(np.uint8)[:n].copy()


def _finish_bank(bank: np.ndarray, rng: np.random.Generator, layer: int, cb_base: int,
                 inter: int, lat: int, stages: int, scale_lo: float, scale_hi: float,
                 eid0: int = 0):
    """Turns E rows of random bytes into E valid records in place (expert ids
    eid0, eid0+1, ...): zero the index padding rows, write the f16 row
    scales, zero the 4 KiB tail and write each header with its crc32."""
    E, rb = bank.shape
    off = HDR_SIZE
    offs = []
    for (M, N) in ((inter, lat), (inter, lat), (lat, inter)):
        n = index_bytes(M, N, stages)
        offs.append(off)
        if M % BLOCK:
            v = bank[:, off:off + n].reshape(E, (M + BLOCK - 1) // BLOCK, N // VEC_DIM, BLOCK,
                                             row_bytes(stages))
            v[:, -1, :, M % BLOCK:, :] = 0
        off += n
    corr = off
    ns = 2 * inter + lat
    bank[:, corr:corr + 2 * ns] = f16_bits(rng.uniform(scale_lo, scale_hi, size=(E, ns))).view(np.uint8)
    end = corr + 2 * ns
    bank[:, end:] = 0
    fmt = fmt_of(stages)
    blocks = rb // ALIGN
    for e in range(E):
        crc = zlib.crc32(memoryview(bank[e, HDR_SIZE:end])) & 0xFFFFFFFF
        bank[e, :HDR_SIZE] = np.frombuffer(
            struct.pack(HDR_FMT, MAGIC_EXPERT, layer, eid0 + e, fmt, 0, cb_base, 0, 0, blocks,
                        offs[0], offs[1], offs[2], corr, crc, 0, 0), dtype=np.uint8)


def bank(rng: np.random.Generator, layer: int, n_experts: int, cb_base: int, inter: int,
         lat: int, stages: int = 3, scale_lo: float = 0.5, scale_hi: float = 1.5) -> np.ndarray:
    """A whole layer's bank: n_experts records, uniform random indices."""
    rb = record_bytes(inter, lat, stages)
    b = random_bytes(rng, n_experts * rb).reshape(n_experts, rb)
    _finish_bank(b, rng, layer, cb_base, inter, lat, stages, scale_lo, scale_hi)
    return b.reshape(-1)


def bank_range(seed: int, layer: int, first: int, count: int, cb_base: int, inter: int,
               lat: int, stages: int = 3, scale_lo: float = 0.5,
               scale_hi: float = 1.5) -> np.ndarray:
    """Records [first, first+count) of a layer's bank, each from its own
    generator seeded by (seed, expert id): a rank that holds part of the
    experts builds only those, and every split of the range gives the same
    bytes. Returned as [count][rec_bytes] uint8."""
    rb = record_bytes(inter, lat, stages)
    out = np.empty((count, rb), dtype=np.uint8)
    for k in range(count):
        rng = np.random.default_rng((seed, first + k))
        out[k] = random_bytes(rng, rb)
        _finish_bank(out[k:k + 1], rng, layer, cb_base, inter, lat, stages, scale_lo, scale_hi,
                     eid0=first + k)
    return out


def set_layer(records: np.ndarray, layer: int) -> None:
    """Rewrites the layer field of [n][rec_bytes] records in place (the
    crc32 covers the payload only), for benchmarks that load the same
    payloads as several resident layers."""
    records[:, 4:6] = np.frombuffer(struct.pack("<H", layer), dtype=np.uint8)


def trunk(seed: int, hidden: int, n_experts: int, shared_inter: int):
    """A seeded router [E][hidden] (rows N(0, 1/hidden), so logits are about
    N(0, 1)) and Q8G shared expert {gate, up, down: (q, s)}."""
    rng = np.random.default_rng(seed)
    router = (rng.standard_normal((n_experts, hidden), dtype=np.float32)
              / np.float32(np.sqrt(hidden))).astype(np.float32)
    sh = {}
    if shared_inter:
        sh["gate"] = q8g(rng, shared_inter, hidden, 2e-4, 5e-4)
        sh["up"] = q8g(rng, shared_inter, hidden, 2e-4, 5e-4)
        sh["down"] = q8g(rng, hidden, shared_inter, 2e-4, 5e-4)
    return router, sh


def derive_layer(base: "MoELayer", layer: int, seed: int) -> "MoELayer":
    """Another layer for benchmarks that need many resident layers: the base
    bank's index bytes and scales under this layer's headers (the layer
    field; the crc32 does not cover the header), plus a fresh router and
    shared expert, so routing differs from layer to layer. Loaded, it is a
    separate copy in HBM like any other layer."""
    rng = np.random.default_rng(seed)
    b = base.bank.copy().reshape(base.n_experts, base.rec_bytes)
    b[:, 4:6] = np.frombuffer(struct.pack("<H", layer), dtype=np.uint8)
    router = (rng.standard_normal(base.router.shape, dtype=np.float32)
              / np.float32(np.sqrt(base.hidden))).astype(np.float32)
    sh = {}
    if base.shared_inter:
        sh["gate"] = q8g(rng, base.shared_inter, base.hidden, 2e-4, 5e-4)
        sh["up"] = q8g(rng, base.shared_inter, base.hidden, 2e-4, 5e-4)
        sh["down"] = q8g(rng, base.hidden, base.shared_inter, 2e-4, 5e-4)
    return MoELayer(layer, base.hidden, base.inter, base.n_experts, base.top_k, base.renorm,
                    base.routed_scale, base.stages, base.cb_base, base.books_raw, router,
                    base.bias, b.reshape(-1), base.rec_bytes, base.shared_inter, sh,
                    base.act_situ, base.situ_beta, base.situ_lbeta)


def moe_layer(seed: int, hidden: int = 2304, inter: int = 1024, n_experts: int = 256,
              top_k: int = 8, shared_inter: int = 1024, layer: int = 1,
              routed_scale: float = 2.446, renorm: int = 1, stages: int = 3,
              with_bias: bool = False, cb_base: int | None = None, act_situ: int = 0,
              situ_beta: float = 4.0, situ_lbeta: float = 25.0) -> MoELayer:
    """Seeded layer at the Kimi-Linear-48B shape by default (hidden 2304,
    expert inter 1024, 256 experts, top-8, one shared expert, routed scale
    2.446 with renorm). stages 4 is a VQ4P layer (64-entry books)."""
    rng = np.random.default_rng(seed)
    if cb_base is None:
        cb_base = 3 * stages * (layer - 1) if layer >= 1 else 0
    n_books = cb_base + 3 * stages
    books_raw = codebooks(rng, n_books, entries=ENTRIES_VQ4P if stages == 4 else ENTRIES)
    router = (rng.standard_normal((n_experts, hidden), dtype=np.float32)
              / np.float32(np.sqrt(hidden))).astype(np.float32)
    bias = (rng.normal(0, 0.05, size=n_experts).astype(np.float32) if with_bias else None)
    rb = record_bytes(inter, hidden, stages)
    bk = bank(rng, layer, n_experts, cb_base, inter, hidden, stages)
    sh = {}
    if shared_inter:
        sh["gate"] = q8g(rng, shared_inter, hidden, 2e-4, 5e-4)
        sh["up"] = q8g(rng, shared_inter, hidden, 2e-4, 5e-4)
        sh["down"] = q8g(rng, hidden, shared_inter, 2e-4, 5e-4)
    return MoELayer(layer, hidden, inter, n_experts, top_k, renorm, routed_scale, stages,
                    cb_base, books_raw, router, bias, bk, rb, shared_inter, sh, act_situ,
                    situ_beta if act_situ else 0.0, situ_lbeta if act_situ else 0.0)


NORM_EPS = 1e-6      # rms_norm_eps of the synthetic decoder layers


def norm_weight(seed: int, hidden: int) -> np.ndarray:
    """A post-attention rmsnorm weight: N(1, 0.1^2) per channel, seeded."""
    rng = np.random.default_rng(seed)
    return (1.0 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)


def activations(seed: int, n: int, T: int = 1) -> np.ndarray:
    """x ~ N(0, 1) rounded to bf16, held in fp32, shape [T][n]."""
    rng = np.random.default_rng(seed)
    return bf16_round(rng.standard_normal((T, n), dtype=np.float32))


def zipf_routes(seed: int, T: int, E: int, K: int, s: float = 1.1) -> np.ndarray:
    """[T][K] distinct expert ids per token drawn from Zipf(s) over a seeded
    permutation of the E ids (prefill routing skew)."""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(E)
    p = 1.0 / np.arange(1, E + 1, dtype=np.float64) ** s
    p /= p.sum()
    out = np.empty((T, K), dtype=np.int32)
    for t in range(T):
        out[t] = perm[rng.choice(E, size=K, replace=False, p=p)]
    return out


# ---- a whole container ---------------------------------------------------------

#: Kimi-Linear-48B's shape for a full decode step: 27
#: layers, layer 0 dense (its intermediate width is not recorded in the
#: reference; 9216 is used), KDA layers of 32 heads x 128 and an MLA layer
#: every fourth (NoPE, latent 512), 256 experts top-8 of 1024, one shared
#: expert, vocab 163840. The trunk is Q4G but for the embedding, lm_head and
#: shared experts (Q8G) and the router, norms and small parameters (F32).
KIMI_LINEAR_48B = dict(hidden=2304, layers=27, first_dense=1, dense_inter=9216, moe_inter=1024,
                       experts=256, top_k=8, n_shared=1, routed_scale=2.446, kda_heads=32,
                       kda_dim=128, conv_k=4, mla_heads=32, qk_nope=128, qk_rope=64, v_head=128,
                       kv_lora=512, vocab=163840, full_attn=(4, 8, 12, 16, 20, 24), eps=1e-6)

FMT_F32, FMT_Q8G, FMT_Q4G = 0, 2, 3           # waste_fmt, src/waste_format.h:46-49
MAGIC_CODEBOOK = 0x4B424357                   # 'WCBK', src/waste_format.h


class _TrunkWriter:
    """trunk.bin written as it grows, with the manifest's tensor index:
    F32 tensors raw; Q8G/Q4G rows padded to whole groups of 128 (Q4G: two
    signed nibbles per byte, low first, biased by 8), then one f16 scale per
    (row, group) — the layout src/model.c reads (:265-320)."""

    def __init__(self, path, rng):
        self.f = open(path, "wb")
        self.rng = rng
        self.off = 0
        self.index = []

    def _put(self, b):
        self.f.write(b)
        self.off += len(b)

    def f32(self, name, a):
        a = np.ascontiguousarray(a, dtype=np.float32)
        off = self.off
        self._put(a.tobytes())
        self.index.append({"name": name, "fmt": FMT_F32, "off": off, "shape": list(a.shape),
                           "bytes": self.off - off})

    def quant(self, name, shape, bits):
        rows, n_in = int(np.prod(shape[:-1])), shape[-1]
        ng = (n_in + GROUP - 1) // GROUP
        off = self.off
        rb = ng * GROUP if bits == 8 else ng * GROUP // 2
        self._put(random_bytes(self.rng, rows * rb).tobytes())
        soff = self.off
        # weights uniform over the code range; scales that keep y = W x at
        # about the size of x (variance of a code: 127^2/3 or 21.25)
        var = 127.0 ** 2 / 3.0 if bits == 8 else 21.25
        s = self.rng.uniform(0.8, 1.2, size=(rows, ng)) / np.sqrt(n_in * var)
        self._put(f16_bits(s).tobytes())
        self.index.append({"name": name, "fmt": FMT_Q8G if bits == 8 else FMT_Q4G, "off": off,
                           "shape": list(shape), "group": GROUP, "scale_off": soff,
                           "bytes": self.off - off})

    def close(self):
        self.f.close()


def write_container(out: str, seed: int = 0, **over) -> dict:
    """A synthetic container the reference engine loads (manifest.json,
    trunk.bin, codebooks.bin, experts-L<n>.bin; the format of
    docs/FORMAT.md, src/waste_format.h), Kimi-Linear-48B-shaped by default
    (KIMI_LINEAR_48B; keyword arguments override). Seeded; weights random
    in their formats' code ranges, codebooks N(0, 0.02^2). Returns the
    config used. The record checksums are left 0 (the engine checks them
    only with WASTE_VERIFY)."""
    import json
    import os
    c = dict(KIMI_LINEAR_48B, **over)
    os.makedirs(out, exist_ok=True)
    rng = np.random.default_rng(seed)
    hid, H, D = c["hidden"], c["kda_heads"], c["kda_dim"]
    C = H * D
    full = set(c["full_attn"])
    kda_layers = [L + 1 for L in range(c["layers"]) if L + 1 not in full]
    t = _TrunkWriter(os.path.join(out, "trunk.bin"), rng)
    t.quant("model.embed_tokens.weight", [c["vocab"], hid], 8)
    ones = lambda n: (1.0 + rng.normal(0.0, 0.02, n)).astype(np.float32)
    for L in range(c["layers"]):
        p = f"model.layers.{L}."
        t.f32(p + "input_layernorm.weight", ones(hid))
        t.f32(p + "post_attention_layernorm.weight", ones(hid))
        a = p + "self_attn."
        if L + 1 in full:                               # MLA (NoPE)
            nh = c["mla_heads"]
            t.quant(a + "q_proj.weight", [nh * (c["qk_nope"] + c["qk_rope"]), hid], 4)
            t.quant(a + "kv_a_proj_with_mqa.weight", [c["kv_lora"] + c["qk_rope"], hid], 4)
            t.f32(a + "kv_a_layernorm.weight", ones(c["kv_lora"]))
            t.quant(a + "kv_b_proj.weight", [nh * (c["qk_nope"] + c["v_head"]), c["kv_lora"]], 4)
            t.quant(a + "o_proj.weight", [hid, nh * c["v_head"]], 4)
        else:                                           # KDA
            for w in ("q_proj", "k_proj", "v_proj"):
                t.quant(a + w + ".weight", [C, hid], 4)
            t.quant(a + "b_proj.weight", [H, hid], 4)
            t.quant(a + "f_a_proj.weight", [D, hid], 4)
            t.quant(a + "f_b_proj.weight", [C, D], 4)
            t.quant(a + "g_a_proj.weight", [D, hid], 4)
            t.quant(a + "g_b_proj.weight", [C, D], 4)
            t.quant(a + "o_proj.weight", [hid, C], 4)
            for w in ("q_conv1d", "k_conv1d", "v_conv1d"):
                t.f32(a + w + ".weight", rng.normal(0.0, 0.3, (C, 1, c["conv_k"])))
            t.f32(a + "A_log", np.log(rng.uniform(1.0, 16.0, (1, 1, H, 1))))
            t.f32(a + "dt_bias", rng.normal(0.0, 0.1, C))
            t.f32(a + "o_norm.weight", ones(D))
        if L < c["first_dense"]:
            m = p + "mlp."
            t.quant(m + "gate_proj.weight", [c["dense_inter"], hid], 4)
            t.quant(m + "up_proj.weight", [c["dense_inter"], hid], 4)
            t.quant(m + "down_proj.weight", [hid, c["dense_inter"]], 4)
        else:
            m = p + "block_sparse_moe."
            t.f32(m + "gate.weight", rng.standard_normal((c["experts"], hid), dtype=np.float32)
                  / np.float32(np.sqrt(hid)))
            t.f32(m + "gate.e_score_correction_bias", rng.normal(0.0, 0.05, c["experts"]))
            si = c["moe_inter"] * c["n_shared"]
            t.quant(m + "shared_experts.gate_proj.weight", [si, hid], 8)
            t.quant(m + "shared_experts.up_proj.weight", [si, hid], 8)
            t.quant(m + "shared_experts.down_proj.weight", [hid, si], 8)
    t.f32("model.norm.weight", ones(hid))
    t.quant("lm_head.weight", [c["vocab"], hid], 8)
    t.close()

    layers, cb_base = {}, 0
    with open(os.path.join(out, "codebooks.bin"), "wb") as cf:
        for L in range(c["first_dense"], c["layers"]):
            books = codebooks(rng, 3 * 3)
            for k in range(9):
                cf.write(struct.pack("<IHBBII", MAGIC_CODEBOOK, (cb_base + k) & 0xFFFF,
                                     FMT_VQ3R, VEC_DIM, ENTRIES, 0))
                cf.write(books[k].tobytes())
            name = f"experts-L{L}.bin"
            bk = bank(rng, L, c["experts"], cb_base, c["moe_inter"], hid)
            bk.tofile(os.path.join(out, name))
            layers[str(L)] = {"file": name, "experts": c["experts"], "bytes": int(bk.size),
                              "codebook_base": cb_base}
            cb_base += 9
    cfg = {"model_type": "kimi_linear", "architectures": ["KimiLinearForCausalLM"],
           "hidden_size": hid, "num_hidden_layers": c["layers"],
           "first_k_dense_replace": c["first_dense"], "intermediate_size": c["dense_inter"],
           "moe_intermediate_size": c["moe_inter"], "num_experts": c["experts"],
           "num_experts_per_token": c["top_k"], "num_shared_experts": c["n_shared"],
           "moe_renormalize": True, "moe_router_activation_func": "sigmoid",
           "routed_scaling_factor": c["routed_scale"], "num_attention_heads": c["mla_heads"],
           "qk_nope_head_dim": c["qk_nope"], "qk_rope_head_dim": c["qk_rope"],
           "v_head_dim": c["v_head"], "kv_lora_rank": c["kv_lora"], "q_lora_rank": None,
           "mla_use_nope": True, "rms_norm_eps": c["eps"], "vocab_size": c["vocab"],
           "tie_word_embeddings": False, "bos_token_id": 1, "eos_token_id": 2,
           "linear_attn_config": {"head_dim": D, "num_heads": H,
                                  "short_conv_kernel_size": c["conv_k"],
                                  "kda_layers": kda_layers,
                                  "full_attn_layers": sorted(full)}}
    manifest = {"format_version": 0, "arch": "kimi_linear", "tensor_prefix": "", "config": cfg,
                "expert_quant": {"fmt": "VQ3R", "stages": 3, "vec_dim": VEC_DIM,
                                 "entries": ENTRIES, "index_block": BLOCK, "bits_per_weight": 3},
                "layers": layers, "trunk": t.index}
    with open(os.path.join(out, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return c
