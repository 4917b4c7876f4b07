"""Synthetic qwen3moe GGUF files for the GGUF reader's tests, written with gguf-py (the Python
GGUF writer that ships with llama.cpp; the reference writes its own fixtures with it,
xtask/tiny_moe.py).  Test infrastructure only.

write_moe_gguf: a Qwen3-MoE file with every tensor the MoE builder names (token embedding, output,
per layer attention, norms, router and the three stacked expert tensors).  Expert tensors are
Q4_K/Q6_K bytes from the oracle's quantiser (or, quantise=False, seeded random bytes, for load
timing) or F16; the metadata also carries one value of every GGUF kind, so that a reader's
handling of each is checked against gguf-py's."""
from __future__ import annotations

import numpy as np

QUANT_BYTES = {12: 144, 14: 210}


def _expert_bytes(rng, qtype, E, rows, cols, quantise):
    if quantise:
        import oracle as O
        w = (rng.standard_normal((E, rows, cols)) * 0.05).astype(np.float32)
        return np.ascontiguousarray(O.quantize(qtype, w)).reshape(E, rows, cols // 256 * QUANT_BYTES[qtype])
    return rng.integers(0, 256, (E, rows, cols // 256 * QUANT_BYTES[qtype]), dtype=np.uint8)


def write_moe_gguf(path, *, n_layer=2, n_embd=256, n_head=4, n_head_kv=2, head_dim=64, n_expert=4, n_used=2,
                   n_ff=256, n_vocab=300, gate_type=12, down_type=14, seed=7, quantise=True, tied=False,
                   split_max_tensors=0, extra_kv=True, attn_types=(1, 1, 1, 1), embd_type=1, out_type=1):
    """Writes the file(s) and returns {tensor name: (ggml type, numpy data as written)}."""
    import gguf
    rng = np.random.default_rng(seed)
    qt = gguf.GGMLQuantizationType
    w = gguf.GGUFWriter(str(path), "qwen3moe", split_max_tensors=split_max_tensors)
    w.add_name("synthetic-qwen3moe")
    w.add_block_count(n_layer)
    w.add_context_length(4096)
    w.add_embedding_length(n_embd)
    w.add_feed_forward_length(n_ff * n_used)
    w.add_head_count(n_head)
    w.add_head_count_kv(n_head_kv)
    w.add_key_length(head_dim)
    w.add_value_length(head_dim)
    w.add_rope_freq_base(1000000.0)
    w.add_layer_norm_rms_eps(1e-6)
    w.add_expert_count(n_expert)
    w.add_expert_used_count(n_used)
    w.add_expert_feed_forward_length(n_ff)
    if extra_kv:  # one value of every kind
        w.add_uint8("test.u8", 200)
        w.add_int8("test.i8", -100)
        w.add_uint16("test.u16", 60000)
        w.add_int16("test.i16", -30000)
        w.add_uint32("test.u32", 4000000000)
        w.add_int32("test.i32", -2000000000)
        w.add_float32("test.f32", 0.1)
        w.add_bool("test.bool", True)
        w.add_string("test.str", "Tetraeder ∆ test")
        w.add_array("test.arr_i32", [1, -2, 3])
        w.add_array("test.arr_str", ["a", "bc", ""])
        w.add_uint64("test.u64", 1 << 60)
        w.add_int64("test.i64", -(1 << 60))
        w.add_float64("test.f64", -2.5e-300)
    written = {}

    def add(name, arr, raw_dtype=None):
        if raw_dtype is None:
            w.add_tensor(name, arr)
            written[name] = (0 if arr.dtype == np.float32 else 1, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=raw_dtype)
            written[name] = (int(raw_dtype), arr)

    def f16(*shape, std=0.1):
        return (rng.standard_normal(shape) * std).astype(np.float16)

    def matrix(name, qtype, rows, cols, std=0.1):
        """F16, or Q4_K/Q6_K bytes of N(0, std) values (the oracle's quantiser)."""
        if qtype in QUANT_BYTES:
            import oracle as O
            w_ = (rng.standard_normal((rows, cols)) * std).astype(np.float32)
            add(name, np.ascontiguousarray(O.quantize(qtype, w_)).reshape(rows, -1), qt(qtype))
        else:
            add(name, f16(rows, cols, std=std))

    def f32(*shape):
        return (1.0 + 0.1 * rng.standard_normal(shape)).astype(np.float32)

    matrix("token_embd.weight", embd_type, n_vocab, n_embd, std=0.5)
    add("output_norm.weight", f32(n_embd))
    if not tied:
        matrix("output.weight", out_type, n_vocab, n_embd)
    for il in range(n_layer):
        p = f"blk.{il}."
        add(p + "attn_norm.weight", f32(n_embd))
        matrix(p + "attn_q.weight", attn_types[0], n_head * head_dim, n_embd)
        matrix(p + "attn_k.weight", attn_types[1], n_head_kv * head_dim, n_embd)
        matrix(p + "attn_v.weight", attn_types[2], n_head_kv * head_dim, n_embd)
        matrix(p + "attn_output.weight", attn_types[3], n_embd, n_head * head_dim)
        add(p + "attn_q_norm.weight", f32(head_dim))
        add(p + "attn_k_norm.weight", f32(head_dim))
        add(p + "ffn_norm.weight", f32(n_embd))
        add(p + "ffn_gate_inp.weight", (rng.standard_normal((n_expert, n_embd)) * 0.5).astype(np.float32))
        for name, qtype, rows, cols in (("ffn_gate_exps", gate_type, n_ff, n_embd),
                                        ("ffn_up_exps", gate_type, n_ff, n_embd),
                                        ("ffn_down_exps", down_type, n_embd, n_ff)):
            if qtype in QUANT_BYTES:
                add(p + name + ".weight", _expert_bytes(rng, qtype, n_expert, rows, cols, quantise), qt(qtype))
            else:
                add(p + name + ".weight", f16(n_expert, rows, cols))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return written
