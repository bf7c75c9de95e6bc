"""The tensor-parallel load point of QuantizedLinear: `pending_from_linear(...,
shard=(rank, world))` swaps a layer before its weight exists and `adopt()`
keeps this rank's output rows of whatever arrives -- the reference's
`_process_model_before_weight_loading` / `adopt` path
(torchnative/python/torchnative/quant/hf.py:340, quant/__init__.py:154-237)
with the column shard of a Q4_0 linear added. A pre-quantised weight (a GGUF
file's blocks) is sliced as bytes on any device; a dense weight is quantised
on the GPU after slicing."""

import numpy as np
import pytest
import torch

from tests import q4_exact
from torchnative_b200 import quant


def _meta_linear(n, k, bias=False):
    with torch.device("meta"):
        return torch.nn.Linear(k, n, bias=bias)


def test_pending_layer_keeps_the_loader_weight_entry_and_its_shard_size():
    lin = _meta_linear(256, 64)
    q = quant.QuantizedLinear.pending_from_linear(lin, "q4_0", shard=(1, 4))
    assert q.out_features == 64 and q.in_features == 64 and q.qweight is None
    assert "weight" in dict(q.named_parameters()) and q.weight.device.type == "meta"
    with pytest.raises(ValueError, match="cannot shard 256 output rows 3 ways"):
        quant.QuantizedLinear.pending_from_linear(lin, "q4_0", shard=(0, 3))
    with pytest.raises(ValueError, match="cannot shard"):
        quant.QuantizedLinear.pending_from_linear(lin, "q4_0", shard=(4, 4))


def test_adopt_slices_a_prequantised_blob_by_rows_for_every_rank():
    rng = np.random.default_rng(11)
    n, k, world = 96, 128, 4
    blob = np.frombuffer(q4_exact.random_q4_0_blob(rng, n, k), dtype=np.uint8)
    full = quant.QTensor(torch.from_numpy(blob.copy()), (n, k), "q4_0")
    parts = []
    for r in range(world):
        q = quant.QuantizedLinear.pending_from_linear(_meta_linear(n, k), "q4_0", shard=(r, world))
        q.adopt(full)
        assert q.qweight.shape == (n // world, k) and "weight" not in dict(q.named_parameters())
        parts.append(q.qweight.blob.numpy())
    assert np.array_equal(np.concatenate(parts), blob)
    # adopt runs once, and the arriving shape must be the unsharded one
    with pytest.raises(ValueError, match="runs once"):
        q.adopt(full)
    q2 = quant.QuantizedLinear.pending_from_linear(_meta_linear(n, k), "q4_0", shard=(0, world))
    with pytest.raises(ValueError, match="does not match"):
        q2.adopt(quant.QTensor(torch.from_numpy(blob[: n // 2 * k // 32 * 18].copy()), (n // 2, k), "q4_0"))


def test_adopt_without_a_shard_keeps_the_whole_blob():
    rng = np.random.default_rng(12)
    blob = np.frombuffer(q4_exact.random_q4_0_blob(rng, 64, 64), dtype=np.uint8)
    q = quant.QuantizedLinear.pending_from_linear(_meta_linear(64, 64), "q4_0")
    q.adopt(quant.QTensor(torch.from_numpy(blob.copy()), (64, 64), "q4_0"))
    assert np.array_equal(q.qweight.blob.numpy(), blob)


@pytest.mark.gpu
def test_dense_weight_is_sliced_then_quantised_and_the_shards_rebuild_the_output(cuda_device):
    from oracle import oracle
    from torchnative_b200 import build

    build.build()
    n, k, world = 256, 512, 4
    g = torch.Generator().manual_seed(13)
    w = torch.randn((n, k), generator=g)
    bias = torch.randn(n, generator=g)
    lin = torch.nn.Linear(k, n)
    with torch.no_grad():
        lin.weight.copy_(w)
        lin.bias.copy_(bias)
    whole = quant._quantize(w.to(cuda_device), "q4_0")
    x = torch.randn((3, k), generator=g).to(cuda_device)
    outs = []
    for r in range(world):
        q = quant.QuantizedLinear.pending_from_linear(lin, "q4_0", shard=(r, world))
        q.adopt(w.to(cuda_device))
        rows = slice(r * n // world, (r + 1) * n // world)
        # the shard's blocks are the unsharded quantisation's rows, byte for byte
        assert torch.equal(q.qweight.blob, whole.blob.view(n, -1)[rows].reshape(-1))
        assert torch.equal(q.bias.detach().cpu(), bias[rows])
        outs.append(q.to(cuda_device)(x))
    y = torch.cat(outs, dim=1).cpu().numpy().astype(np.float64)
    exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(oracle.q8_0_quantize(x.cpu().numpy()),
                                                         whole.blob.cpu().numpy().tobytes(), 3, n, k)
    exact = exact + bias.numpy().astype(np.float64)
    bound = q4_exact.linear_bound(k, abs_sum, ref_err) + np.abs(exact) * 2.0 ** -23
    assert float(np.max(np.abs(y - exact) / bound)) <= 1.0
