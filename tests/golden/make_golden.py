"""Generates the committed golden fixtures under tests/golden/.

    python -m tests.golden.make_golden

Config 1 of the benchmark plan: one head, N=1024, head_dim=64, Q/K/V iid
N(0,1) from numpy PCG64 seeds 101/102/103, scale 1/sqrt(64).  The expected
outputs are exact softmax attention evaluated in float64 with numpy (an
implementation independent of both the oracle and the CUDA kernels), stored
as float32 for 128 evenly spaced rows, for the causal mask (the reference's
only mode, rust_src/src/waller_operator.rs:24) and the non-causal one.
"""
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
N, D = 1024, 64
ROWS = np.linspace(0, N - 1, 128).round().astype(np.int64)


def config1_inputs():
    return tuple(np.random.default_rng(s).standard_normal((N, D)).astype(np.float32)
                 for s in (101, 102, 103))


def exact_attention_f64(q, k, v, scale, causal):
    s = (q.astype(np.float64) @ k.astype(np.float64).T) * scale
    if causal:
        s = np.where(np.tril(np.ones(s.shape, dtype=bool)), s, -np.inf)
    s -= s.max(axis=1, keepdims=True)
    p = np.exp(s)
    return (p / p.sum(axis=1, keepdims=True)) @ v.astype(np.float64)


def load_golden(name):
    z = np.load(os.path.join(HERE, name + ".npz"))
    return z["rows"], z["out"]


def main():
    q, k, v = config1_inputs()
    for causal in (True, False):
        out = exact_attention_f64(q, k, v, 1.0 / 8.0, causal)[ROWS].astype(np.float32)
        name = "config1_causal" if causal else "config1_noncausal"
        np.savez_compressed(os.path.join(HERE, name + ".npz"), rows=ROWS, out=out)
        print("wrote", name)


if __name__ == "__main__":
    main()
