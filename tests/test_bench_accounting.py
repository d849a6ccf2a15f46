"""The algorithmic byte counts the bench divides by (no GPU): packed bytes per expert, the
step's and the gate/up launch's bytes, the attention and stack per-slot bytes."""

import numpy as np


def test_packed_bytes_per_expert_are_the_gguf_bytes():
    import bench

    # gate || up: 1024 rows x 8 blocks, down: 2048 rows x 2 blocks (H = 2048, I = 512)
    assert bench.packed_bytes_per_expert("Q6_K") == (1024 * 8 + 2048 * 2) * 210 == 2_580_480
    assert bench.packed_bytes_per_expert("Q4_K") == (1024 * 8 + 2048 * 2) * 144 == 1_769_472


def test_step_and_gate_up_bytes_count_routed_experts_and_rows():
    import bench

    ids = np.array([[0], [0], [5], [9], [5]], np.int32)  # 3 distinct experts, 5 rows
    nbytes, active = bench.step_bytes("Q6_K", ids)
    assert active == 3
    assert nbytes == 3 * 2_580_480 + 5 * 2048 * 2 * 2  # x read + out written
    gate_up = bench.kernel_bytes("Q6_K", ids)
    assert gate_up == 3 * 1024 * 8 * 210 + 5 * (2048 + 512) * 2  # gate+up packed, x read, h written


def test_attention_slot_bytes():
    import bench

    # K + V codes (2 kv heads x 256) + BF16 scales (2 planes x 16 groups)
    assert bench.ATTN_SLOT_BYTES == 1088
