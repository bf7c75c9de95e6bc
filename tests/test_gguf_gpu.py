"""GGUF tensors straight to the device (torchnative_b200.gguf), against files
written by llama.cpp's gguf-py: blocks stay byte-identical in HBM, dense and
dequantised tensors are bit-exact, llama.cpp's q/k row order is undone by
rows, and a Llama decoder loaded from a GGUF file of another decoder's weights
holds the same bytes and decodes the same token with the same logits."""

import dataclasses

import numpy as np
import pytest
import torch

from oracle import oracle
from tests import gguf_util, q4_exact

pytestmark = pytest.mark.gpu
gguf = pytest.importorskip("gguf")


@pytest.fixture(scope="module")
def G(cuda_device):
    from torchnative_b200 import _native, build, gguf as g

    build.build()
    _native.lib()
    return g


def test_tensors_reach_the_device_byte_for_byte(G, cuda_device, tmp_path):
    rng = np.random.default_rng(41)
    q4 = np.frombuffer(q4_exact.random_q4_0_blob(rng, 6, 256), np.uint8).reshape(6, -1)
    q8 = np.frombuffer(q4_exact.random_q8_0_blob(rng, 3, 128), np.uint8).reshape(3, -1)
    f32 = rng.standard_normal((4, 33)).astype(np.float32)
    f16 = rng.standard_normal(40).astype(np.float16)
    bf = rng.integers(0, 256, size=(2, 64), dtype=np.uint8)
    bf[:, 1::2] &= 0x3F  # finite bf16 values
    path = tmp_path / "t.gguf"
    gguf_util.write_gguf(path, {"q4": (q4, "Q4_0"), "q8": (q8, "Q8_0"), "f32": (f32, None), "f16": (f16, None),
                                "bf": (bf, "BF16")})
    with G.GGUFContainer(path) as f:
        for name, arr, fmt, n in (("q4", q4, "q4_0", 6 * 256), ("q8", q8, "q8_0", 3 * 128)):
            q = G.load_tensor(f, name, keep_blocks=True, device=cuda_device)
            assert q.format == fmt and q.blob.device.type == "cuda"
            assert q.blob.cpu().numpy().tobytes() == arr.tobytes()
            deq = G.load_tensor(f, name, keep_blocks=False, device=cuda_device)
            want = (oracle.q4_0_dequantize if fmt == "q4_0" else oracle.q8_0_dequantize)(arr.tobytes(), n)
            assert deq.dtype == torch.float32 and deq.cpu().numpy().tobytes() == want.tobytes()
        assert G.load_tensor(f, "f32", device=cuda_device).cpu().numpy().tobytes() == f32.tobytes()
        t16 = G.load_tensor(f, "f16", device=cuda_device)
        assert t16.dtype == torch.float16 and t16.cpu().numpy().tobytes() == f16.tobytes()
        tb = G.load_tensor(f, "bf", device=cuda_device)
        assert tb.dtype == torch.bfloat16 and tb.shape == (2, 32)
        assert tb.view(torch.int16).cpu().numpy().tobytes() == bf.tobytes()


def test_quantized_linear_is_the_files_blocks(G, cuda_device, tmp_path):
    from torchnative_b200 import quant

    rng = np.random.default_rng(42)
    blob = q4_exact.random_q4_0_blob(rng, 48, 512)
    path = tmp_path / "l.gguf"
    gguf_util.write_gguf(path, {"w": (np.frombuffer(blob, np.uint8).reshape(48, -1), "Q4_0"),
                                "n": (np.ones(512, np.float32), None)})
    x = torch.randn(3, 512, device=cuda_device)
    with G.GGUFContainer(path) as f:
        mod = G.quantized_linear(f, "w", device=cuda_device)
        assert (mod.in_features, mod.out_features, mod.format) == (512, 48, "q4_0")
        want = quant._quantized_linear(x, quant._quantized_from_blob(blob, (48, 512), "q4_0", cuda_device))
        assert torch.equal(mod(x), want)
        with pytest.raises(G.GGUFUnsupported, match="not a block-quantised type"):
            G.quantized_linear(f, "n", device=cuda_device)


def test_llama_cpp_row_order_is_undone_by_rows(G, cuda_device, tmp_path):
    rng = np.random.default_rng(43)
    heads = 4
    hf = np.frombuffer(q4_exact.random_q4_0_blob(rng, 64, 128), np.uint8).reshape(64, -1)  # 4 heads x 16 rows
    dense = rng.standard_normal((64, 8)).astype(np.float32)
    path = tmp_path / "p.gguf"
    gguf_util.write_gguf(path, {"q": (gguf_util.llama_cpp_permute(hf, heads), "Q4_0"),
                                "d": (gguf_util.llama_cpp_permute(dense, heads), None)})
    with G.GGUFContainer(path) as f:
        q = G.load_tensor(f, "q", keep_blocks=True, permute_heads=heads, device=cuda_device)
        assert q.blob.cpu().numpy().tobytes() == hf.tobytes()
        d = G.load_tensor(f, "d", permute_heads=heads, device=cuda_device)
        assert d.cpu().numpy().tobytes() == dense.tobytes()
        with pytest.raises(G.GGUFUnsupported, match="q/k row order"):
            G.load_tensor(f, "q", keep_blocks=True, permute_heads=5, device=cuda_device)


def test_decoder_from_gguf_decodes_what_its_source_decodes(G, cuda_device, tmp_path):
    from torchnative_b200.llama_decode import LlamaShape, Q4LlamaDecoder

    shape = LlamaShape(256, 512, 4, 2, 64, 512, 2, 10000.0)
    a = Q4LlamaDecoder(shape, batch=1, capacity=64, device=cuda_device, seed=7)
    path = tmp_path / "llama.gguf"
    gguf_util.decoder_to_gguf(a, path)
    b = Q4LlamaDecoder.from_gguf(path, batch=1, capacity=64, device=cuda_device)
    # GGUF stores eps as float32; the kernels take float32 either way
    assert np.float32(b.s.eps) == np.float32(shape.eps)
    assert dataclasses.replace(b.s, eps=shape.eps) == shape
    for la, lb in zip(a.layers, b.layers):
        for key in ("attn_norm", "qkv", "o", "mlp_norm", "gate_up", "down"):
            assert torch.equal(la[key], lb[key]), key
    for key in ("final_norm", "lm_head", "embed"):
        assert torch.equal(getattr(a, key), getattr(b, key)), key
    tok = torch.tensor([17], dtype=torch.int32, device=cuda_device)
    outs = []
    for dec in (a, b):
        dec.fill_prompt_cache(20)
        dec.start(tok)
        dec.step()
        torch.cuda.synchronize()
        outs.append((dec.tokens.clone(), dec.logits.clone()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    from torchnative_b200 import _native
    _native.device_status(reset=True)
