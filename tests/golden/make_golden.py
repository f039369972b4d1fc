"""Writes tests/golden/moe_small.npz: oracle outputs of small MoE layers that
pin the CPU restatement against regressions (the reference itself, in Go,
cannot run here).  Every case is rebuilt from its seeds by qg_oracle.make_moe
and qg_oracle.randn, so the file holds only the expected results.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))
import qg_oracle as O  # noqa: E402

# (bits, router mode, shared width): H=64, E=8, k=3, I=32, 5 tokens, seed 40 + case
CASES = [(b, mode, Is) for b in (32, 16, 8, 4) for mode in (O.ROUTER_TOPK, O.ROUTER_PREFIX)
         for Is in (0, 64)]
H, E, K, I, T = 64, 8, 3, 32, 5


def case_arrays(i, bits, mode, Is):
    m = O.make_moe(H, E, K, I, Is, bits, seed=40 + i)
    x = O.randn(40 + i, 100, (T, H))
    return m, x


def main():
    out = {}
    for i, (bits, mode, Is) in enumerate(CASES):
        m, x = case_arrays(i, bits, mode, Is)
        y, idx, w, sg, probs = O.moe_forward(m, x, mode, want_probs=True)
        out[f"c{i}_out"], out[f"c{i}_idx"], out[f"c{i}_w"] = y, idx, w
        out[f"c{i}_probs"] = probs
    out["cases"] = np.array(CASES, np.int32)
    np.savez_compressed(os.path.join(HERE, "moe_small.npz"), **out)


if __name__ == "__main__":
    main()
