"""The oracle against the reference's own known answers for the Npu(Int8) path."""
import numpy as np

from oracle import configs, oracle


def test_usage_doc_report(oracle_lib):
    # docs/USAGE.md:376-380: 4 -> 2 fused ops, 5392 B fp32, 40960 MACs, these labels.
    # The doc prints 1552 B (3.47x); quantize.rs:43-45 adds 4 B per scale -> 1560 B (3.46x).
    layers, x = configs.usage_doc_model()
    p = oracle.Program(layers)
    assert p.summary(len(layers)) == (
        "InferenceSession [provider = NPU (INT8), layers: 4 -> 2 fused ops, weights: 5392 B -> 1560 B "
        "(3.46x compression)]\n  Pipeline: NPU::FusedGemmAct(16->64, ReLU) -> NPU::Gemm(64->4)")
    y, ns, macs = p.execute(x)
    assert y.shape == (32, 4)
    assert macs.tolist() == [32768, 8192] and macs.sum() == 40960
    assert (p.fp32_bytes, p.npu_bytes) == (5392, 1560)


def test_integration_structure(oracle_lib):
    # tests/integration.rs:128-164: 9 raw layers -> 5 fused ops, compression > 3.
    layers, x = configs.integration_model()
    p = oracle.Program(layers)
    assert p.original_layers == 9 and len(p.ops) == 5
    assert p.compression_ratio() > 3.0
    assert [o.label() for o in p.ops] == [
        "NPU::FusedConv2dAct(1->4, k=3, ReLU)", "NPU::MaxPool2d(k=2)", "NPU::Flatten",
        "NPU::FusedGemmAct(64->16, ReLU)", "NPU::Gemm(16->4)"]
    y, _, _ = p.execute(x)
    assert y.shape == (8, 4) and np.isfinite(y).all()


def test_quantizer_semantics(oracle_lib):
    # quantize.rs:18-24: absmax ignores NaN, round half away from zero, clamp, NaN -> 0.
    x = np.array([0.5, -1.5, 2.5, np.nan, 127.0, -127.0, 63.5, -63.5], np.float32)
    q, s = oracle.quantize(x)
    assert s == np.float32(127.0) / np.float32(127.0)
    assert q.tolist() == [1, -2, 3, 0, 127, -127, 64, -64]
    q, s = oracle.quantize(np.zeros(5, np.float32))
    assert s == 1.0 and (q == 0).all()
    q, s = oracle.quantize(np.array([np.inf, 1.0, -np.inf], np.float32))
    assert np.isinf(s) and q.tolist() == [0, 0, 0]


def test_maxpool_nan_and_ties(oracle_lib):
    # kernels.rs:187: `v > best || v.is_nan()` -> NaN propagates, -inf windows stay -inf.
    x = np.array([[[[1, np.nan, 3, 4], [0, 2, -np.inf, -np.inf],
                    [5, 5, -1, -2], [5, 5, -3, -4]]]], np.float32)
    y = oracle.maxpool2d(x, 2, 2)
    assert np.isnan(y[0, 0, 0, 0]) and y[0, 0, 0, 1] == 4
    assert y[0, 0, 1, 0] == 5 and y[0, 0, 1, 1] == -1
    y = oracle.maxpool2d(np.full((1, 1, 2, 2), -np.inf, np.float32), 2, 2)
    assert y[0, 0, 0, 0] == -np.inf


def test_oracle_thread_count_independent(oracle_lib):
    layers, x = configs.c2_cnn(8)
    p = oracle.Program(layers)
    y1, _, _ = p.execute(x, nthreads=1)
    y4, _, _ = p.execute(x, nthreads=4)
    assert np.array_equal(y1, y4)


def test_linear_rows_matches_full(oracle_lib):
    layers, x = configs.c3_linear(40, 64, 24)
    p = oracle.Program(layers)
    y, tr = p.run_traced(x)
    yr, acc, sa = oracle.linear_rows(p.ops[0], p, 0, x, 10, 25)
    assert sa == tr[0]["a_scale"]
    assert np.array_equal(acc, tr[0]["acc"][10:25])
    assert np.array_equal(yr, y[10:25])
