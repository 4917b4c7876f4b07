"""Writes tests/golden/tiny_qwen3moe_f16.json: the reference's own fixture model
(tests/fixtures/tiny-qwen3moe-f16.gguf of the tetraeder tree, 2 layers, 64 wide, 8 experts, F16
experts) as gguf-py's GGUFReader reads it -- every metadata value (arrays as their length), and
per tensor its type, shape, absolute data offset, byte count and sha256.  tests/test_gguf.py holds
this repository's GGUF reader to it whenever the fixture is at hand.

Run here (gguf-py is importable in this container):
    python tests/golden/make_gguf_golden.py /path/to/tetraeder/tests/fixtures/tiny-qwen3moe-f16.gguf
"""
import hashlib
import json
import os
import sys

import numpy as np
from gguf import GGUFReader, GGUFValueType

HERE = os.path.dirname(os.path.abspath(__file__))


def value(field):
    if field.types[0] == GGUFValueType.ARRAY:
        return {"array_len": len(field.data)}
    v = field.contents()
    if isinstance(v, (np.floating, float)):
        return float(v)
    if isinstance(v, (np.integer, int, bool)):
        return int(v)
    return v


def main(path):
    r = GGUFReader(path)
    kv = {k: value(f) for k, f in r.fields.items() if not k.startswith("GGUF.")}
    tensors = []
    raw = open(path, "rb").read()
    for t in r.tensors:
        off = int(t.data_offset)
        n = int(t.n_bytes)
        tensors.append({"name": t.name, "type": int(t.tensor_type), "shape": [int(x) for x in t.shape],
                        "offset": off, "nbytes": n, "sha256": hashlib.sha256(raw[off:off + n]).hexdigest()})
    out = {"file": os.path.basename(path), "bytes": len(raw), "kv": kv, "tensors": tensors}
    with open(os.path.join(HERE, "tiny_qwen3moe_f16.json"), "w") as f:
        json.dump(out, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main(sys.argv[1])
