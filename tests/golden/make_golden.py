"""Writes tests/golden/kquant_dequant.npz: Q4_K / Q6_K blocks and their f32 values as decoded by
gguf-py (gguf.quants.Q4_K/Q6_K.dequantize_blocks, the Python decoder that ships with llama.cpp,
the reference's pinned ggml dependency).  The blocks are random bytes with sane f16 scales plus
blocks from the oracle's own quantiser, so the oracle's and the kernels' block decoders are pinned
to an implementation that is not ours.

Run here (gguf-py is importable in this container):  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
import oracle as O  # noqa: E402


def main():
    rng = np.random.default_rng(20261201)
    out = {}
    for name, qt, cls, nbytes in (("q4_k", O.TYPE_Q4_K, quants.Q4_K, 144), ("q6_k", O.TYPE_Q6_K, quants.Q6_K, 210)):
        rand = rng.integers(0, 256, size=(48, nbytes), dtype=np.uint8)
        if qt == O.TYPE_Q4_K:
            rand[:, 0:2] = np.array([0.0123], dtype=np.float16).view(np.uint8)
            rand[:, 2:4] = np.array([-0.0031], dtype=np.float16).view(np.uint8)
            rand[5, 0:2] = np.array([0.0], dtype=np.float16).view(np.uint8)
        else:
            rand[:, 208:210] = np.array([0.00071], dtype=np.float16).view(np.uint8)
        w = (rng.standard_normal((16, 256)) * 0.02).astype(np.float32)
        w[3] = 0.0
        w[4] = np.abs(w[4]) + 0.01  # all-positive sub-blocks (min clamps to 0)
        ours = O.quantize(qt, w).reshape(16, nbytes)
        blocks = np.concatenate([rand, ours])
        vals = cls.dequantize_blocks(blocks).astype(np.float32)
        out[name + "_blocks"] = blocks
        out[name + "_values"] = vals
        out[name + "_source"] = w
    np.savez_compressed(os.path.join(HERE, "kquant_dequant.npz"), **out)
    print("wrote", os.path.join(HERE, "kquant_dequant.npz"))


if __name__ == "__main__":
    main()
