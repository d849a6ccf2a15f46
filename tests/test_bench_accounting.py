"""The bench's measurement arithmetic (no GPU): the algorithmic byte counts it divides by
(packed bytes per expert, the step's and the gate/up launch's bytes, the attention per-slot
bytes), the clock record's summary, the roofline's traffic and its peak."""

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


def test_clock_summary_reads_median_clock_and_active_reasons():
    import bench

    s = bench.ClockSampler(0)
    s.lines = [
        "0, 1965, 1965, 812.40, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
        "0, 1950, 1965, 990.10, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "0, 1965, 1965, 1001.3, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
        "garbage line",
        "0, [N/A], 1965, 1.0, 0x0, Not Active, Not Active, Not Active, Not Active",
    ]
    got = s.summary()
    assert got["sm_mhz"] == 1965.0 and got["sm_max_mhz"] == 1965.0
    assert got["reasons"] == ["sw_power_cap"] and got["samples"] == 3

    s.lines = ["0, 1200, 1965, 700.0, 0x0000000000000008, Active, Not Active, Active, Not Active"]
    assert s.summary()["reasons"] == ["hw_slowdown", "sw_thermal_slowdown"]


def test_roofline_traffic_is_read_from_the_committed_profile_and_matches_the_bytes():
    import bench

    traffic = bench.ncu_traffic("Q6_K", 16)
    assert traffic is not None
    algorithmic = bench.kernel_bytes("Q6_K", bench.workload_ids(16))
    # DRAM bytes of one gate/up launch within a few percent of the algorithmic bytes: no re-reads
    assert 1.0 <= traffic / algorithmic < 1.05
    assert bench.ncu_traffic("Q4_K", 3) is None  # no summary for that case


def test_hbm_peak_prefers_the_measured_file(tmp_path, monkeypatch):
    import json

    import bench

    monkeypatch.setattr(bench, "ROOT", tmp_path)
    assert bench.hbm_peak() == (bench.FALLBACK_HBM_GBS, "fallback")
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps({"hbm_gbs": 6550.1}))
    assert bench.hbm_peak() == (6550.1, "measured")
