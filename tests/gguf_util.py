"""Test helpers: GGUF files written by llama.cpp's own gguf-py writer (the
installed `gguf` package), so the loader is checked against an independent
writer rather than against itself."""

from __future__ import annotations

import struct

import numpy as np


def write_gguf(path, tensors: dict, metadata: dict | None = None, arch: str = "llama", alignment: int | None = None):
    """tensors: name -> (numpy array, ggml type name or None). A block or BF16
    type takes the stored bytes as uint8 [rows, row_bytes]; None takes a
    float32 / float16 array as is. metadata: key -> python value."""
    import gguf

    w = gguf.GGUFWriter(str(path), arch)
    if alignment is not None:
        w.add_custom_alignment(alignment)
    for key, value in (metadata or {}).items():
        if isinstance(value, bool):
            w.add_bool(key, value)
        elif isinstance(value, int):
            w.add_uint32(key, value)
        elif isinstance(value, float):
            w.add_float32(key, value)
        elif isinstance(value, str):
            w.add_string(key, value)
        else:
            w.add_array(key, list(value))
    for name, (arr, tname) in tensors.items():
        if tname is None:
            w.add_tensor(name, arr)
        else:
            w.add_tensor(name, arr, raw_dtype=getattr(gguf.GGMLQuantizationType, tname))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def llama_cpp_permute(rows: np.ndarray, n_head: int) -> np.ndarray:
    """convert_hf_to_gguf's q/k row order: HF row (h, p, d) is stored as row
    (h, d, p) (rows [n, ...], p the rotary half, d < n / n_head / 2)."""
    n = rows.shape[0]
    dim = n // n_head // 2
    return rows.reshape(n_head, 2, dim, *rows.shape[1:]).swapaxes(1, 2).reshape(rows.shape)


def decoder_to_gguf(dec, path):
    """A Q4LlamaDecoder's weights written as a llama GGUF in llama.cpp's
    layout: separate q/k/v (q/k rows permuted), gate/up, norms as F32,
    token_embd as BF16, output as Q4_0."""
    s = dec.s
    D, H, I = s.head_dim, s.hidden, s.inter
    rb = H // 32 * 18  # bytes per Q4_0 row of K = hidden

    def rows(blob, n):
        return blob.cpu().numpy().reshape(n, -1)

    def bf16_bytes(t):
        import torch

        return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint8).reshape(t.shape[0], -1)

    tensors = {}
    for li, lw in enumerate(dec.layers):
        b = f"blk.{li}."
        qkv = rows(lw["qkv"], s.qkv)
        q, k, v = qkv[:s.heads * D], qkv[s.heads * D:(s.heads + s.kv_heads) * D], qkv[(s.heads + s.kv_heads) * D:]
        tensors[b + "attn_q.weight"] = (llama_cpp_permute(q, s.heads), "Q4_0")
        tensors[b + "attn_k.weight"] = (llama_cpp_permute(k, s.kv_heads), "Q4_0")
        tensors[b + "attn_v.weight"] = (np.ascontiguousarray(v), "Q4_0")
        tensors[b + "attn_output.weight"] = (rows(lw["o"], H), "Q4_0")
        gu = rows(lw["gate_up"], 2 * I).reshape(I, 2, rb)
        tensors[b + "ffn_gate.weight"] = (np.ascontiguousarray(gu[:, 0]), "Q4_0")
        tensors[b + "ffn_up.weight"] = (np.ascontiguousarray(gu[:, 1]), "Q4_0")
        tensors[b + "ffn_down.weight"] = (rows(lw["down"], H), "Q4_0")
        tensors[b + "attn_norm.weight"] = (lw["attn_norm"].float().cpu().numpy(), None)
        tensors[b + "ffn_norm.weight"] = (lw["mlp_norm"].float().cpu().numpy(), None)
    tensors["token_embd.weight"] = (bf16_bytes(dec.embed), "BF16")
    tensors["output_norm.weight"] = (dec.final_norm.float().cpu().numpy(), None)
    tensors["output.weight"] = (rows(dec.lm_head, s.vocab), "Q4_0")
    md = {"llama.embedding_length": H, "llama.feed_forward_length": I, "llama.attention.head_count": s.heads,
          "llama.attention.head_count_kv": s.kv_heads, "llama.block_count": dec.n_layers,
          "llama.rope.freq_base": float(s.rope_theta), "llama.attention.layer_norm_rms_epsilon": float(s.eps)}
    write_gguf(path, tensors, md)


def raw_gguf(version=3, tensors=(), metadata=(), magic=b"GGUF", endian="<", data=b"", alignment=32) -> bytes:
    """A GGUF file assembled by hand, for the malformed and refused cases the
    real writer will not produce. tensors: (name, extents, type id, offset);
    metadata: (key, type id, packed value bytes)."""
    out = bytearray(magic)
    out += struct.pack(endian + "I", version)
    out += struct.pack(endian + "QQ", len(tensors), len(metadata))

    def s(x):
        b = x.encode()
        return struct.pack(endian + "Q", len(b)) + b

    for key, vt, packed in metadata:
        out += s(key) + struct.pack(endian + "I", vt) + packed
    for name, ne, gt, off in tensors:
        out += s(name) + struct.pack(endian + "I", len(ne)) + b"".join(struct.pack(endian + "Q", e) for e in ne)
        out += struct.pack(endian + "IQ", gt, off)
    out += b"\0" * ((-len(out)) % alignment)
    return bytes(out) + data
