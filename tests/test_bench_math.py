"""CPU checks of the bench's roofline and layer arithmetic (no GPU): the algorithmic bytes and
FLOPs it divides by, the fraction it reports, and the all-reduce split of a TP line."""
import pytest

import bench

H, I, K = bench.H, bench.INTER, bench.K_TOP


def test_decode_c1_gate_up_algorithmic_bytes():
    # 380 touched experts + the shared one, 64 tokens: weights (2 I H per expert + its fp32
    # 128x128 scales) plus the activations read (rows x (H + H/128 scales)) and written
    # (rows x (I + I/128 scales)); rows = 64 x (10 routed + 1 shared)
    rows = 64 * (K + 1)
    w = 381 * (2 * I * H + 2 * (I // 128) * (H // 128) * 4)
    act = rows * (H + (H // 128) * 4) + rows * (I + (I // 128) * 4)
    assert bench.kernel_bytes("gemm_gate_up", 380, rows, I, I, 64) == w + act == 3_200_557_056


def test_prefill_gate_up_flops():
    rows = 8192 * (K + 1)
    assert bench.kernel_flops("gemm_gate_up", rows, I) == 2 * rows * 2 * I * H
    assert bench.kernel_flops("gemm_down", rows, I) == 2 * rows * H * I


def _result(**stage):
    st = {"router_topk": 0.013, "dispatch": 0.015, "gather_quant": 0.003, "gemm_gate_up": 0.462,
          "gemm_down": 0.251, "combine": 0.011}
    st.update(stage)
    return {"stage_ms": st, "inter": I, "shared": I, "n_touched": 380, "ms_step": 0.741, "ar_ms": 0.0}


def test_decode_roofline_is_gate_up_bytes_over_its_event_time():
    r = _result()
    roof, dom = bench.roofline(r, 64, prefill=False)
    assert dom == "gemm_gate_up" and roof["bound"] == "hbm"
    expect = 3_200_557_056 / (0.462e-3) / 1e9
    assert roof["achieved"] == pytest.approx(expect)
    assert roof["frac"] == pytest.approx(expect / roof["peak"])


def test_prefill_roofline_reports_both_bounds():
    r = _result(gemm_gate_up=1.8, gemm_down=1.0)
    r["n_touched"] = 512
    roof, _ = bench.roofline(r, 8192, prefill=True)
    assert {roof["bound"], roof["other"]["bound"]} == {"hbm", "tensor"}
    assert roof["algorithmic_flops_per_launch"] == bench.kernel_flops("gemm_gate_up", 8192 * (K + 1), I)


def test_tp_layer_summary_splits_the_allreduce_from_the_fused_stage():
    class Comm:  # any non-None group marks the fused combine + all-reduce
        pass

    r = _result(combine=0.0387)
    r["ms_step"] = 0.216
    s = bench.layer_summary(r, 256, 8, Comm(), False, combine_alone_ms=0.0145)
    assert s["combine_allreduce_ms"] == pytest.approx(0.0387)
    assert s["allreduce_added_ms"] == pytest.approx(0.0387 - 0.0145)
    assert s["allreduce_added_share"] == pytest.approx((0.0387 - 0.0145) / 0.216)
    single = bench.layer_summary(_result(), 64, 1, None, False)
    assert single["allreduce_added_ms"] is None and single["allreduce_share"] == 0.0
