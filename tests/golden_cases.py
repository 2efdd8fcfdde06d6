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
