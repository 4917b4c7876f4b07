"""Seeded synthetic inputs and checks shared by the tests.

The generators restate the reference's own test generators (paths relative to the tetraeder
project root) so the cases read like its tests:
  Rng / make_ids           crates/ggml-sys/tests/mul_mat_id_skip.rs:30-85 (xorshift64, ids with
                           distinct experts per token and a share of -1)
  routing                  crates/model/src/qwen3moe.rs:2930-2948 (LCG, skewed top-8 of 32)
"""
from __future__ import annotations

import numpy as np

import oracle as O

MASK64 = (1 << 64) - 1


class XorShift:
    """xorshift64 of mul_mat_id_skip.rs:30-45: f32 uniform in [-1, 1), below(n)."""

    def __init__(self, seed: int):
        self.s = seed & MASK64

    def next_u64(self) -> int:
        s = self.s
        s ^= (s << 13) & MASK64
        s ^= s >> 7
        s ^= (s << 17) & MASK64
        self.s = s
        return s

    def f32(self, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        for i in range(n):
            out[i] = np.float32((self.next_u64() >> 40) / float(1 << 23) - 1.0)
        return out

    def below(self, n: int) -> int:
        return self.next_u64() % n


def make_ids(rng: XorShift, experts: int, used: int, tokens: int, neg_pct: int) -> np.ndarray:
    """Distinct experts per token, `neg_pct` percent of the slots -1 (mul_mat_id_skip.rs:68-85)."""
    ids = []
    for _ in range(tokens):
        pool = list(range(experts))
        for j in range(used):
            pick = j + rng.below(len(pool) - j)
            pool[j], pool[pick] = pool[pick], pool[j]
            ids.append(-1 if rng.below(100) < neg_pct else pool[j])
    return np.array(ids, dtype=np.int32).reshape(tokens, used)


def routing():
    """The skewed top-8-of-32 routing of the reference's pair-group tests (qwen3moe.rs:2930-2948)."""
    n_expert, n_used, n_tokens = 32, 8, 24
    x = 12345
    chosen = []
    for _ in range(n_tokens):
        token = []
        while len(token) < n_used:
            x = (x * 6364136223846793005 + 1442695040888963407) & MASK64
            u = (x >> 33) / float(1 << 31)
            e = int(u * u * n_expert)
            if e not in token:
                token.append(e)
        chosen.extend(token)
    return np.array(chosen, dtype=np.int32), n_used


def group_pairs(chosen, n_used, experts):
    """Restatement of group_pairs (qwen3moe.rs:2126-2150): pairs of `experts`, in pair order."""
    pairs = [p for p, e in enumerate(chosen) if e in experts]
    return pairs


def random_kquant_bytes(rng: np.random.Generator, qtype: int, rows: int, ncols: int,
                        scale: float = 0.02) -> np.ndarray:
    """Valid random Q4_K / Q6_K rows (uniform nibbles/scales, f16 super-block scales near `scale`),
    fast enough for full-size expert tensors."""
    nb = ncols // 256
    if qtype == O.TYPE_Q4_K:
        blk = rng.integers(0, 256, size=(rows * nb, 144), dtype=np.uint8)
        d = (rng.uniform(0.5, 1.5, rows * nb) * scale / 63 / 4).astype(np.float16)
        dmin = (rng.uniform(0.5, 1.5, rows * nb) * scale / 63 / 8).astype(np.float16)
        blk[:, 0:2] = d.view(np.uint8).reshape(-1, 2)
        blk[:, 2:4] = dmin.view(np.uint8).reshape(-1, 2)
    else:
        blk = rng.integers(0, 256, size=(rows * nb, 210), dtype=np.uint8)
        sc = rng.integers(-127, 128, size=(rows * nb, 16)).astype(np.int8)
        blk[:, 192:208] = sc.view(np.uint8)
        d = (rng.uniform(0.5, 1.5, rows * nb) * scale / 127 / 16).astype(np.float16)
        blk[:, 208:210] = d.view(np.uint8).reshape(-1, 2)
    return blk.reshape(rows, nb * blk.shape[1])


def quantized_experts(rng: np.random.Generator, qtype: int, E: int, rows: int, ncols: int,
                      std: float = 0.02, exact: bool = True) -> np.ndarray:
    """[E, rows, row_size] bytes: N(0, std) quantised with the oracle's fit (exact=True) or
    random valid blocks (exact=False, for full-size tensors)."""
    if exact:
        w = (rng.standard_normal((E, rows, ncols)) * std).astype(np.float32)
        return O.quantize(qtype, w)
    return random_kquant_bytes(rng, qtype, E * rows, ncols, std).reshape(E, rows, -1)


def nrms(got: np.ndarray, want: np.ndarray) -> float:
    rms = float(np.sqrt(np.mean(np.square(want, dtype=np.float64))))
    return float(np.sqrt(np.mean(np.square(got.astype(np.float64) - want)))) / max(rms, 1e-30)


def maxabs_over_rms(got: np.ndarray, want: np.ndarray) -> float:
    rms = float(np.sqrt(np.mean(np.square(want, dtype=np.float64))))
    return float(np.max(np.abs(got.astype(np.float64) - want))) / max(rms, 1e-30)


# The north-star output tolerance: normalised RMS error <= 1e-2 and max-abs <= 5e-2 x output RMS.
NORTH_NRMS, NORTH_MAXABS = 1e-2, 5e-2


def q6r_pack(W: np.ndarray) -> np.ndarray:
    """Q6_K matrices uint8 [n, rows, nb * 210] in the 8-row fragment order of tmoe_prepack, restated
    from the layout's description with numpy reshapes: per 8-row group and super-block a unit of 1680
    bytes; half h of the block holds the ql bytes 64h + 16i + 4t4 + j of row g at 768h + 16(4g + t4)
    + 4i + j and the qh bytes 128 + 32h + 16i + 4t4 + j at 768h + 512 + 8(4g + t4) + 4i + j; then the
    rows' 16 scale bytes (1536 + 16g) and their d (1664 + 2g)."""
    n, rows, rb = W.shape
    nb = rb // 210
    blk = W.reshape(n, rows // 8, 8, nb, 210).transpose(0, 1, 3, 2, 4)  # [n, group, block, g, 210]
    lead = blk.shape[:3]
    unit = np.empty(lead + (1680,), np.uint8)
    for h in range(2):
        ql = blk[..., 64 * h:64 * h + 64].reshape(lead + (8, 4, 4, 4))  # g, i, t4, j
        unit[..., 768 * h:768 * h + 512] = ql.transpose(0, 1, 2, 3, 5, 4, 6).reshape(lead + (512,))
        qh = blk[..., 128 + 32 * h:160 + 32 * h].reshape(lead + (8, 2, 4, 4))  # g, i, t4, j
        unit[..., 768 * h + 512:768 * h + 768] = qh.transpose(0, 1, 2, 3, 5, 4, 6).reshape(lead + (256,))
    unit[..., 1536:1664] = blk[..., 192:208].reshape(lead + (128,))
    unit[..., 1664:1680] = blk[..., 208:210].reshape(lead + (16,))
    return np.ascontiguousarray(unit).reshape(n, rows, rb)


def q6r_unpack(P: np.ndarray) -> np.ndarray:
    """The inverse of q6r_pack: 8-row fragment-ordered Q6_K units back to ggml rows."""
    n, rows, rb = P.shape
    nb = rb // 210
    unit = P.reshape(n, rows // 8, nb, 1680)
    lead = unit.shape[:3]
    blk = np.empty(lead + (8, 210), np.uint8)
    for h in range(2):
        ql = unit[..., 768 * h:768 * h + 512].reshape(lead + (8, 4, 4, 4))  # g, t4, i, j
        blk[..., 64 * h:64 * h + 64] = ql.transpose(0, 1, 2, 3, 5, 4, 6).reshape(lead + (8, 64))
        qh = unit[..., 768 * h + 512:768 * h + 768].reshape(lead + (8, 4, 2, 4))  # g, t4, i, j
        blk[..., 128 + 32 * h:160 + 32 * h] = qh.transpose(0, 1, 2, 3, 5, 4, 6).reshape(lead + (8, 32))
    blk[..., 192:208] = unit[..., 1536:1664].reshape(lead + (8, 16))
    blk[..., 208:210] = unit[..., 1664:1680].reshape(lead + (8, 2))
    return np.ascontiguousarray(blk.transpose(0, 1, 3, 2, 4)).reshape(n, rows, rb)
