"""Generate the golden dequantisation fixtures (tests/golden/kquant_golden.npz).

The expected values come from gguf-py 0.19.0 (`gguf.quants.dequantize`), llama.cpp's
Python implementation of the Q4_K / Q5_K / Q6_K formats, i.e. an implementation
independent of both the oracle and the CUDA kernels. The reference project (Rust) has no
golden vectors of its own and cannot be built in this image, so these fixtures and the
hand-derived known-answer tests pin the oracle. Inputs: seeded random blocks with the
benchmark distributions plus the hand-built edge blocks of tests/edge_blocks.py.

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))


def main():
    from gguf import GGMLQuantizationType as T
    from gguf import quants

    import oracle
    from edge_blocks import EDGE

    types = {12: T.Q4_K, 13: T.Q5_K, 14: T.Q6_K}
    out = {}
    rng = np.random.default_rng(20261201)
    for qt, tt in types.items():
        bb = oracle.BLOCK_BYTES[qt]
        raw = np.concatenate([oracle.random_blocks(qt, 24, rng), EDGE[qt]()])
        nb = raw.size // bb
        ref = quants.dequantize(raw.reshape(nb, bb), tt).reshape(-1).astype(np.float32)
        out[f"raw_{qt}"] = raw
        out[f"deq_{qt}"] = ref
        # a small GEMV case (K = 512, N = 6) with x ~ N(0,1): y from the gguf dequant and a
        # float64 dot (compared with tolerance)
        K, N = 512, 6
        w = oracle.random_blocks(qt, N * (K // 256), rng)
        x = rng.standard_normal(K).astype(np.float32)
        Wd = quants.dequantize(w.reshape(-1, bb), tt).reshape(N, K).astype(np.float64)
        out[f"gemv_w_{qt}"] = w
        out[f"gemv_x_{qt}"] = x
        out[f"gemv_y_{qt}"] = (Wd @ x.astype(np.float64)).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "kquant_golden.npz"), **out)
    print("wrote", os.path.join(HERE, "kquant_golden.npz"))


if __name__ == "__main__":
    main()
