"""Seeded cases shared by the golden-vector tests (CPU) and the parity tests
(GPU). The fixtures themselves are written by tests/golden/make_golden.py."""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

MOE_CASES = {
    "moe_small": (5, dict(hidden=256, inter=128, n_experts=16, top_k=4, shared_inter=128,
                          with_bias=True, routed_scale=2.0), 7, 16),
    "moe_ragged": (11, dict(hidden=192, inter=96, n_experts=12, top_k=3, shared_inter=192,
                            with_bias=False, renorm=0, routed_scale=1.0), 13, 5),
    "moe_kimi": (1234, dict(), 4321, 0),
    # K3's activation (SiTU, beta 4, linear beta 25) at a small shape
    "moe_situ": (17, dict(hidden=256, inter=128, n_experts=16, top_k=4, shared_inter=128,
                          with_bias=True, routed_scale=2.827, act_situ=1), 19, 16),
}

MATVEC_CASES = ("matvec_ragged", "matvec_square", "matvec_vq2r")

# VQ4P (four stages of 64-entry books, 6-bit indices packed four to three
# bytes): matvec fixtures in vq4p.npz, name -> (M, N). Books 4..7 of 12;
# x is zero on positions [32, 64) where N allows, so one table block has
# scale 0.
VQ4P_CASES = {"p6_square": (256, 2304), "p6_ragged": (70, 1000), "p6_down": (2304, 1024),
              "p6_small": (64, 256)}

# VQ4P MoE layers (moe_vq4p*.npz), in the form of MOE_CASES
VQ4P_MOE_CASES = {
    "moe_vq4p": (31, dict(hidden=256, inter=128, n_experts=16, top_k=4, shared_inter=128,
                          with_bias=True, routed_scale=2.0, stages=4), 33, 16),
    "moe_vq4p_situ": (37, dict(hidden=256, inter=128, n_experts=16, top_k=4, shared_inter=128,
                               with_bias=True, routed_scale=2.827, act_situ=1, stages=4), 39, 16),
}


def vq4p_books():
    """The raw f16 books of the VQ4P matvec fixtures: 12 books of 64."""
    from warp_b200 import synth
    return synth.codebooks(np.random.default_rng(4040), 12, entries=synth.ENTRIES_VQ4P)


def vq4p_case(name):
    """(idx, scale, x, M, N) of a VQ4P matvec fixture, regenerated from its
    seed (the fixture pins them by a sha256)."""
    import zlib
    from warp_b200 import synth
    M, N = VQ4P_CASES[name]
    idx, sc = synth.random_matrix(np.random.default_rng(zlib.crc32(name.encode())), M, N,
                                  stages=4)
    x = synth.activations(len(name) + M, N)[0]
    if N >= 512:
        x[256:512] = 0
    return idx, sc, x, M, N


def sha(*arrays) -> str:
    import hashlib
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()

# the trunk matvec fixtures (mvq.npz): name -> (rows, in, bits)
MVQ_CASES = {
    "q8g": (96, 2304, 8), "q8g_ragged": (70, 1000, 8), "q4g": (96, 2304, 4),
    "q4g_ragged": (50, 520, 4), "q3g": (64, 2304, 3), "q3g_ragged": (33, 300, 3),
}

# the rmsnorm fixtures (norm.npz): widths
NORM_SIZES = (2304, 1024, 7168, 100)


def load(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# KDA decode-step fixtures (kda.npz): name -> (H, K, V, steps); the state
# starts at zero and runs `steps` tokens.
KDA_CASES = {"kda_kimi": (32, 128, 128, 4), "kda_small": (4, 64, 64, 3)}
CONV_C, CONV_KS = 4096, 4                     # one of q/k/v's short convs
NORM_HEADS, NORM_DIM = 32, 128                # the gated o-norm, per head


def kda_inputs(name):
    """Seeded per-step inputs (q, k, v, g_log, beta) of a KDA fixture:
    q, k, v N(0, 1); log decays -|N(0, 0.5)| (g <= 0, as the decay gate
    gives); beta uniform (0, 1)."""
    H, K, V, T = KDA_CASES[name]
    rng = np.random.default_rng(len(name) * 131 + H)
    steps = []
    for _ in range(T):
        q = rng.standard_normal(H * K, dtype=np.float32)
        k = rng.standard_normal(H * K, dtype=np.float32)
        v = rng.standard_normal(H * V, dtype=np.float32)
        g = (-np.abs(rng.normal(0.0, 0.5, H * K))).astype(np.float32)
        beta = rng.uniform(0.0, 1.0, H).astype(np.float32)
        steps.append((q, k, v, g, beta))
    return steps


def conv_inputs():
    rng = np.random.default_rng(808)
    w = rng.normal(0.0, 0.5, (CONV_C, CONV_KS)).astype(np.float32)
    xs = rng.standard_normal((3, CONV_C), dtype=np.float32)
    return w, xs


def norm_inputs():
    rng = np.random.default_rng(809)
    x = rng.standard_normal(NORM_HEADS * NORM_DIM, dtype=np.float32)
    gate = rng.standard_normal(NORM_HEADS * NORM_DIM, dtype=np.float32)
    w = rng.normal(1.0, 0.1, NORM_DIM).astype(np.float32)
    return x, gate, w, np.float32(1e-6)


# The converter's encoder (enc.npz): name -> (n vectors, stages, entries,
# dim). "enc_ties" repeats entries inside each book (the first index must
# win); "enc_dim12" is a dimension other than 8.
ENC_CASES = {"enc_kimi": (20000, 3, 256, 8), "enc_ties": (3000, 2, 64, 8),
             "enc_dim12": (2000, 2, 32, 12)}
# Lloyd iterations: name -> (n, entries, dim); "lloyd_sparse" has fewer
# vectors than clusters, so most clusters stay empty.
LLOYD_CASES = {"lloyd_kimi": (50000, 256, 8), "lloyd_sparse": (100, 256, 8)}


def enc_inputs(name):
    """Seeded (X, books) of an encoder case: X like the converter's W/scale
    rows (|x| <= 1), books N(0, 0.3^2) per stage (shrinking by stage)."""
    n, st, en, dim = ENC_CASES[name]
    rng = np.random.default_rng(len(name) * 977 + n)
    X = np.clip(rng.normal(0.0, 0.4, (n, dim)), -1, 1).astype(np.float32)
    books = np.stack([rng.normal(0.0, 0.3 / (s + 1), (en, dim)) for s in range(st)]
                     ).astype(np.float32)
    if name == "enc_ties":
        books[:, en // 2:] = books[:, :en // 2]       # every entry twice
    return X, books


def lloyd_inputs(name):
    n, en, dim = LLOYD_CASES[name]
    rng = np.random.default_rng(len(name) * 313 + n)
    X = rng.normal(0.0, 0.4, (n, dim)).astype(np.float32)
    C0 = X[rng.choice(n, size=en, replace=n < en)].copy()
    return X, C0
