"""B200-native (sm_100a) Qwen3-MoE layer hot path of Tetraeder's `--engine moe` builder:
router -> token-to-expert dispatch -> Q4_K/Q6_K SwiGLU expert products -> weighted combine,
behind the C ABI of include/tmoe.h (libtmoe.so, built from csrc/ by build.py)."""
from ._lib import TYPE_Q4_K, TYPE_Q6_K, TmoeError, header_symbols, load  # noqa: F401

__all__ = ["TYPE_Q4_K", "TYPE_Q6_K", "TmoeError", "header_symbols", "load", "MoeLayer", "ExpertWeights",
           "SlotCache", "GgufFile"]


def __getattr__(name):
    if name in ("MoeLayer", "ExpertWeights", "SlotCache", "row_size"):
        from . import moe
        return getattr(moe, name)
    if name in ("GgufFile", "GgufError", "Hparams"):
        from . import gguf
        return getattr(gguf, name)
    raise AttributeError(name)
