"""Display strings of the session surface (labels, Duration, NpuProfile)."""
from rustgears_b200.session import NpuPrecision, NpuProfile, OpRecord, _fmt_duration
from rustgears_b200.spec import Activation


def test_duration_debug_format():
    assert _fmt_duration(84_200) == "84.2µs"
    assert _fmt_duration(61_500) == "61.5µs"
    assert _fmt_duration(999) == "999ns"
    assert _fmt_duration(1_000) == "1µs"
    assert _fmt_duration(1_500_000) == "1.5ms"
    assert _fmt_duration(2_000_001_000) == "2.000001s"


def test_activation_display():
    assert [str(a) for a in (Activation.NONE, Activation.RELU, Activation.SIGMOID, Activation.TANH,
                             Activation.GELU)] == ["none", "ReLU", "Sigmoid", "Tanh", "GELU"]
    assert str(Activation.leaky_relu(0.01)) == "LeakyReLU(0.01)"
    assert str(Activation.leaky_relu(1.0)) == "LeakyReLU(1)"


def test_profile_display_matches_usage_doc_layout():
    # docs/USAGE.md:378-380 shape of the printout (byte counts per the current code: 1560 B)
    p = NpuProfile(NpuPrecision.Int8, 4, 2, 5392, 1560, 40960, 84_200,
                   [OpRecord("NPU::FusedGemmAct(16->64, ReLU)", 32768, 61_500),
                    OpRecord("NPU::Gemm(64->4)", 8192, 21_900)])
    s = str(p)
    assert s.splitlines()[0] == ("NPU Profile [INT8 | layers: 4 -> 2 fused | weights: 5392 B -> 1560 B (3.46x) | "
                                 "MACs: 40960 | time: 84.2µs (0.97 GOPS)]")
    # npu.rs:172 `"  - {:<42} {:>10} MACs   {:?}"` (the doc's sample has one more space)
    assert s.splitlines()[1] == "  - NPU::FusedGemmAct(16->64, ReLU)" + " " * 11 + " " + "     32768 MACs   61.5µs"
    assert s.splitlines()[2] == "  - NPU::Gemm(64->4)" + " " * 26 + " " + "      8192 MACs   21.9µs"
    assert abs(p.gops() - 0.9729) < 1e-3
