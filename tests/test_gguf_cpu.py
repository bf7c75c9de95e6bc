"""The GGUF container reader (torchnative_b200.gguf.GGUFContainer) on the CPU,
against files written by llama.cpp's gguf-py and against hand-built
malformed ones: metadata values, torch-order shapes, aligned offsets and the
stored bytes equal the writer's; the reference's refusals hold by name."""

import struct

import numpy as np
import pytest

from tests import gguf_util
from torchnative_b200 import gguf as G

gguf = pytest.importorskip("gguf")


def test_type_table_sizes_equal_gguf_py():
    for tid, (name, block, size, handling, _) in G.GGML_TYPE_TABLE.items():
        try:
            qt = gguf.GGMLQuantizationType(tid)
        except ValueError:
            continue
        assert qt.name == name, tid
        if block is None or name == "Q8_1":  # gguf-py lists Q8_1 at its old 40-byte size
            continue
        assert gguf.GGML_QUANT_SIZES[qt] == (block, size), name


def test_reads_what_gguf_py_writes(tmp_path):
    rng = np.random.default_rng(0)
    f32 = rng.standard_normal((3, 64)).astype(np.float32)
    f16 = rng.standard_normal(96).astype(np.float16)
    q4 = rng.integers(0, 256, size=(5, 4 * 18), dtype=np.uint8)   # 5 rows of 128 elements
    q8 = rng.integers(0, 256, size=(2, 3 * 34), dtype=np.uint8)   # 2 rows of 96 elements
    bf = rng.integers(0, 256, size=(4, 2 * 32), dtype=np.uint8)   # 4 rows of 32 bf16
    path = tmp_path / "m.gguf"
    md = {"llama.block_count": 2, "llama.rope.freq_base": 500000.0, "general.name": "tiny", "flag.x": True,
          "tokenizer.ggml.scores": [0.5, 1.5, -2.0]}
    gguf_util.write_gguf(path, {"a": (f32, None), "b": (f16, None), "c": (q4, "Q4_0"), "d": (q8, "Q8_0"),
                                "e": (bf, "BF16")}, md)
    with G.GGUFContainer(path) as f:
        assert f.version == 3
        assert f.metadata["general.architecture"] == "llama"
        assert f.metadata["llama.block_count"] == 2 and f.metadata["general.name"] == "tiny"
        assert f.metadata["flag.x"] is True
        assert f.metadata["llama.rope.freq_base"] == np.float32(500000.0)
        assert list(f.metadata["tokenizer.ggml.scores"]) == [0.5, 1.5, -2.0]
        want = {"a": ((3, 64), "F32", f32.tobytes()), "b": ((96,), "F16", f16.tobytes()),
                "c": ((5, 128), "Q4_0", q4.tobytes()), "d": ((2, 96), "Q8_0", q8.tobytes()),
                "e": ((4, 32), "BF16", bf.tobytes())}
        for name, (shape, tname, raw) in want.items():
            info = f.slot(name)
            assert info.shape == shape and info.type_name == tname, name
            assert info.start % f.alignment == 0 and info.start >= f.data_start
            assert bytes(f.bytes_of(name)) == raw, name
        assert f.slot("c").block_format == "q4_0" and f.slot("d").block_format == "q8_0" and f.slot("a").block_format is None
        with pytest.raises(KeyError, match="no tensor 'zz' in this file"):
            f.slot("zz")


def test_custom_alignment(tmp_path):
    q4 = np.arange(2 * 18, dtype=np.uint8).reshape(1, 36)
    path = tmp_path / "a.gguf"
    gguf_util.write_gguf(path, {"x": (np.ones(7, np.float32), None), "w": (q4, "Q4_0")}, alignment=64)
    with G.GGUFContainer(path) as f:
        assert f.alignment == 64 and f.slot("w").start % 64 == 0
        assert bytes(f.bytes_of("w")) == q4.tobytes()


def _file(tmp_path, raw):
    p = tmp_path / "x.gguf"
    p.write_bytes(raw)
    return p


def test_malformed_files_are_refused_by_name(tmp_path):
    with pytest.raises(G.GGUFMalformed, match="a GGUF file starts with"):
        G.GGUFContainer(_file(tmp_path, gguf_util.raw_gguf(magic=b"GGML")))
    with pytest.raises(G.GGUFMalformed, match="zero bytes long"):
        G.GGUFContainer(_file(tmp_path, b""))
    with pytest.raises(G.GGUFUnsupported, match="big-endian"):
        G.GGUFContainer(_file(tmp_path, gguf_util.raw_gguf(endian=">")))
    with pytest.raises(G.GGUFUnsupported, match="version 1"):
        G.GGUFContainer(_file(tmp_path, gguf_util.raw_gguf(version=1)))
    # a Q4_0 tensor whose bytes are not all there
    with pytest.raises(G.GGUFMalformed, match="cut short"):
        G.GGUFContainer(_file(tmp_path, gguf_util.raw_gguf(tensors=[("w", (64, 2), 2, 0)], data=b"\0" * 40)))
    with pytest.raises(G.GGUFMalformed, match="the file ends inside"):
        G.GGUFContainer(_file(tmp_path, gguf_util.raw_gguf(metadata=[("k", 8, struct.pack("<Q", 99) + b"ab")])))
    with pytest.raises(G.GGUFMalformed, match="does not divide into blocks of 32"):
        G.GGUFContainer(_file(tmp_path, gguf_util.raw_gguf(tensors=[("w", (48, 1), 2, 0)], data=b"\0" * 64)))
    with pytest.raises(G.GGUFMalformed, match="off the 32-byte alignment"):
        G.GGUFContainer(_file(tmp_path, gguf_util.raw_gguf(tensors=[("w", (32, 1), 2, 8)], data=b"\0" * 64)))
    with pytest.raises(G.GGUFMalformed, match="defined more than once"):
        G.GGUFContainer(_file(tmp_path, gguf_util.raw_gguf(metadata=[("k", 4, struct.pack("<I", 1))] * 2)))


def test_refused_and_kernel_less_types(tmp_path):
    data = b"\0" * 1024
    p = _file(tmp_path, gguf_util.raw_gguf(
        tensors=[("q81", (32, 1), 9, 0), ("q6k", (256, 1), 14, 64), ("odd", (4, 1), 99, 320)], data=data))
    with G.GGUFContainer(p) as f:
        with pytest.raises(G.GGUFUnsupported, match="Q8_1.*activation"):
            f.bytes_of("q81")
        assert len(f.bytes_of("q6k")) == 210  # readable bytes, no kernel
        assert isinstance(G.why_refused(14, "q6k"), G.GGUFUnsupported) and "has no B200 kernel" in str(G.why_refused(14))
        assert G.why_refused(2) is None and G.why_refused(8) is None and G.why_refused(12) is None and G.why_refused(0) is None
        with pytest.raises(G.GGUFUnsupported, match="type id 99"):
            f.bytes_of("odd")
        with pytest.raises(G.GGUFUnsupported, match="has no B200 kernel"):
            G.load_tensor(f, "q6k")
