"""Generates the golden fixtures in this folder from the oracle (the CPU
restatement of the reference Npu(Int8) path).  Run from the repo root:

    python tests/golden/make_golden.py [case ...]

Each case's .npz holds the input, every op's activation scale(s), i8
activations, i32 accumulators and f32 output, the program summary and the
weight byte counts.  tests/test_golden.py re-runs the oracle against them;
the GPU parity tests compare the device path with them bit for bit.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import configs, oracle  # noqa: E402


def trace_case(name):
    layers, x = configs.CASES[name]()
    prog = oracle.Program(layers)
    y, trace = prog.run_traced(x)
    d = {"x": x, "y": y, "summary": np.array(prog.summary(len(layers))),
         "fp32_bytes": np.int64(prog.fp32_bytes), "npu_bytes": np.int64(prog.npu_bytes),
         "n_ops": np.int64(len(prog.ops))}
    for i, t in enumerate(trace):
        d[f"op{i}_label"] = np.array(t["label"])
        d[f"op{i}_y"] = t["y"]
        if "aq" in t:
            d[f"op{i}_scales"] = np.atleast_1d(np.asarray(t.get("a_scale", t.get("a_scales")), np.float32))
            d[f"op{i}_aq"] = t["aq"]
            d[f"op{i}_acc"] = t["acc"]
    return d


def main():
    oracle.build()
    names = sys.argv[1:] or list(configs.CASES)  # e.g. `make_golden.py resnet_mini`
    for name in names:
        d = trace_case(name)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **d)
        print(name, "ops:", int(d["n_ops"]), "out:", d["y"].shape)


if __name__ == "__main__":
    main()
