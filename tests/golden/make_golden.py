"""Writes tests/golden/config0.npz: the float64 oracle's output on BASELINE config 0.

Config 0: one memory layer, forward, B=2, H=4, D=32 (E=128), T=512, chunk 64,
Omega window 8, 5 Polar Express steps, inputs from oracle.make_inputs(seed=0)
(q,k,v ~ N(0,1) L2-normalised per head, alpha=sigmoid(N(3,.5)),
eta=sigmoid(N(-3,.5)), theta=sigmoid(N(1,.5)), gamma=1) and the LM-path initial
state (W1=0, W2=[I;0], S=0).  A second case uses the Xavier initial state and
random gamma.  Outputs are stored as float32.

The reference itself cannot run here (no JAX), so these vectors pin the CUDA
path to the oracle and guard the oracle against regressions; the oracle is in
turn pinned by the reference's own known-answer tests (tests/test_oracle.py).

Run: python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import atlas_oracle as O  # noqa: E402

CFG0 = dict(B=2, T=512, H=4, D=32, E=128, chunk=64, omega=8, ns_steps=5)


def main():
    c = CFG0
    out = {}
    for tag, gmode, init in (("lm", "ones", "lm"), ("xav", "random", "xav")):
        q, k, v, a, e, t, g = O.make_inputs(c["B"], c["T"], c["H"], c["D"], seed=0, gamma_mode=gmode)
        st = (O.lm_initial_state(c["B"], c["H"], c["D"], c["E"]) if init == "lm"
              else O.make_xavier_state(c["B"], c["H"], c["D"], c["E"], seed=1))
        y, fin = O.scan_forward(q, k, v, a, e, t, g, st, c["chunk"], c["omega"], c["ns_steps"],
                                dtype=np.float64)
        out[f"{tag}_y"] = y.astype(np.float32)
        for n, x in zip(("W1", "W2", "S1", "S2"), fin):
            out[f"{tag}_{n}"] = x.astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "config0.npz"), **out)


if __name__ == "__main__":
    main()
