"""The bench's algorithmic bytes per unit, pinned to the figures the
roofline fractions are stated against (record layout of the reference's
expert format, src/waste_format.h:98-132, at the benchmark shapes)."""
import bench
from warp_b200 import synth


def test_kimi_linear_expert_bytes():
    # gate/up [1024][2304] and down [2304][1024], three stage bytes per
    # 8-dim vector: 884,736 B each; f16 row scales 2 x (1024+1024+2304)
    assert synth.index_bytes(1024, 2304, 3) == 884_736
    assert synth.index_bytes(2304, 1024, 3) == 884_736
    assert synth.record_bytes(1024, 2304, 3) == 2_666_496
    # one gate/up launch at one token: 8 experts x 2 matrices + x + codebooks
    assert bench.gateup_bytes() == 2 * 8 * 884_736 + 2304 * 4 + 2 * 3 * 256 * 8 * 4


def test_k3_class_expert_bytes():
    # 5,505,024 B per matrix, 22,528 B of scales: 16,537,600 B per expert,
    # 8.47 GB per 512-expert layer
    assert synth.index_bytes(2048, 7168, 3) == 5_505_024
    assert synth.index_bytes(7168, 2048, 3) == 5_505_024
    assert bench.k3_expert_bytes() == 16_537_600
    assert abs(512 * bench.k3_expert_bytes() / 1e9 - 8.47) < 0.01
    router, shared = bench.k3_trunk_bytes()
    assert router == 512 * 7168 * 4
    # Q8G: gate/up [2048][7168] and down [7168][2048] int8 + one f16 per 128
    assert shared == 3 * 2048 * 7168 + 2 * 3 * 2048 * 7168 // 128


def test_matvec_launch_bytes():
    # config 1: 32 matrices of 4096 x 4096 per launch
    one = synth.index_bytes(4096, 4096, 3) + 2 * 4096 + 4 * 4096 + 4 * 4096
    assert synth.index_bytes(4096, 4096, 3) == 6_291_456
    assert 32 * one + 3 * 256 * 8 * 4 == 202_661_888
