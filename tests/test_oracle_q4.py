"""The Q4_0 oracle against llama.cpp's own answers, and its linear against the
exact value of the quantised operands.

These pin the CPU restatement (oracle/tn_oracle.c) before any GPU result is
compared with it:

1. writer bytes and reader bits equal llama.cpp gguf-py's frozen answers in
   tests/golden/q4_gguf_golden.json (the reference's
   scripts/q4quality/golden_gguf_py.json), with no tolerance, as the
   reference's tests/numerics/test_q4ref.py:104-141 requires of candle;
2. the same codec equals the installed gguf-py on seeded inputs;
3. the linear is within the reference's counted float32 bound of its exact
   value (scripts/q4quality/q4_gguf_ref.py:398-465, 511; K = K_in/32 + 3),
   and the bound refuses a linear that skipped activation quantisation
   (test_q4ref.py:203-255);
4. lossless integer operands give the exact integer matmul
   (tests/numerics/test_qgemm.py:102-137 of the reference).
"""

import json
import os
import struct

import numpy as np
import pytest

from oracle import oracle
from tests import q4_exact

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "q4_gguf_golden.json")


def _golden():
    with open(GOLDEN) as fh:
        return json.load(fh)


def _f32(hexstr):
    raw = bytes.fromhex(hexstr)
    return np.array(struct.unpack(f"<{len(raw) // 4}f", raw), dtype=np.float32)


def test_golden_file_still_exercises_its_edges():
    doc = _golden()
    cases = {(c["format"], c["name"]): c for c in doc["cases"]}
    assert len(doc["provenance"]["gguf_quants_sha256"]) == 64
    d = lambda c: struct.unpack("<e", bytes.fromhex(c["blob"])[0:2])[0]  # noqa: E731
    assert d(cases[("q4_0", "pos_extreme")]) < 0 and d(cases[("q4_0", "neg_extreme")]) > 0
    zero = cases[("q4_0", "zero")]
    assert d(zero) == 0.0 and set(bytes.fromhex(zero["blob"])[2:]) == {0x88}
    raw = struct.unpack("<H", bytes.fromhex(cases[("q4_0", "subnormal_d")]["blob"])[0:2])[0]
    assert raw & 0x7C00 == 0 and raw & 0x3FF != 0
    ties = _f32(cases[("q8_0", "ties")]["input_f32"])
    assert np.max(np.abs(ties)) == 127.0 and 2.5 in ties and -126.5 in ties
    assert len(doc["cases"]) == 10


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_writer_bytes_equal_llama_cpp(fmt):
    quant = {"q4_0": oracle.q4_0_quantize, "q8_0": oracle.q8_0_quantize}[fmt]
    n = 0
    for c in _golden()["cases"]:
        if c["format"] != fmt or "input_f32" not in c:
            continue
        got = quant(_f32(c["input_f32"]))
        assert got == bytes.fromhex(c["blob"]), (fmt, c["name"])
        n += 1
    assert n == {"q4_0": 7, "q8_0": 2}[fmt]


@pytest.mark.parametrize("fmt", ["q4_0", "q8_0"])
def test_reader_bits_equal_llama_cpp(fmt):
    deq = {"q4_0": oracle.q4_0_dequantize, "q8_0": oracle.q8_0_dequantize}[fmt]
    for c in _golden()["cases"]:
        if c["format"] != fmt:
            continue
        n = int(np.prod(c["shape"]))
        got = deq(bytes.fromhex(c["blob"]), n)
        assert got.tobytes() == bytes.fromhex(c["dequant_f32"]), (fmt, c["name"])


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_codec_equals_installed_gguf_py(seed):
    gguf = pytest.importorskip("gguf")
    from gguf import quants

    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((8, 256)) * (0.01 + seed)).astype(np.float32)
    x[0, :32] = 0.0
    x[1, 5] = -np.abs(x[1]).max() * 1.5  # a negative signed maximum
    for fmt, qt, mine in (("q4_0", gguf.GGMLQuantizationType.Q4_0, oracle.q4_0_quantize),
                          ("q8_0", gguf.GGMLQuantizationType.Q8_0, oracle.q8_0_quantize)):
        want = quants.quantize(x, qt).tobytes()
        assert mine(x) == want, fmt
        deq = {"q4_0": oracle.q4_0_dequantize, "q8_0": oracle.q8_0_dequantize}[fmt]
        assert deq(want, x.size).tobytes() == quants.dequantize(np.frombuffer(want, np.uint8).reshape(8, -1),
                                                                 qt).astype(np.float32).tobytes()


@pytest.mark.parametrize("rows,out_f,in_f,seed", [(1, 8, 64, 11), (3, 12, 512, 12), (2, 5, 1024, 13),
                                                  (4, 37, 4096, 14)])
def test_linear_within_counted_bound_of_exact_value(rows, out_f, in_f, seed):
    w = (np.random.default_rng(seed + 1).standard_normal((out_f, in_f)) * 0.05).astype(np.float32)
    x = q4_exact.tie_free_gauss(rows, in_f, seed)
    blob = oracle.q4_0_quantize(w)
    got = oracle.q4_0_linear(x, blob, out_f, threads=3)
    xq = oracle.q8_0_quantize(x)
    exact, abs_sum, ref_err = q4_exact.exact_linear_q4_0(xq, blob, rows, out_f, in_f)
    bound = q4_exact.linear_bound(in_f, abs_sum, ref_err)
    assert float(np.max(np.abs(got - exact) / bound)) <= 1.0
    # The bound must refuse the nearest wrong linear: no activation quantisation.
    wdq = oracle.q4_0_dequantize(blob, out_f * in_f).astype(np.float64).reshape(out_f, in_f)
    assert float(np.max(np.abs(x.astype(np.float64) @ wdq.T - exact) / bound)) > 1.0


def test_linear_is_the_row_dot_and_bias_is_one_add():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, 256)).astype(np.float32)
    w = rng.standard_normal((9, 256)).astype(np.float32)
    bias = rng.standard_normal(9).astype(np.float32)
    blob = oracle.q4_0_quantize(w)
    y = oracle.q4_0_linear(x, blob, 9, threads=4)
    yb = oracle.q4_0_linear(x, blob, 9, bias=bias, threads=2)
    assert (yb == (y + bias).astype(np.float32)).all()
    xq = oracle.q8_0_quantize(x)
    nb = 256 // 32
    for r in range(3):
        for c in range(9):
            one = oracle.lib().tno_q4_0_q8_0_dot(np.frombuffer(blob, np.uint8)[c * nb * 18:].ctypes.data,
                                                 np.frombuffer(xq, np.uint8)[r * nb * 34:].ctypes.data, nb)
            assert np.float32(one) == y[r, c]


def test_lossless_integer_operands_give_the_exact_integer_matmul():
    # scale 1 (f16 1.0), codes in [-8, 7]; activations integers with block absmax 127
    rng = np.random.default_rng(7)
    M, N, K = 3, 10, 256
    codes = rng.integers(-8, 8, size=(N, K))
    blob = q4_exact.q4_0_blob_from_codes(codes, np.ones((N, K // 32), dtype=np.float16))
    x = rng.integers(-127, 128, size=(M, K)).astype(np.float32)
    x[:, ::32] = 127.0  # every block's absmax is 127 -> d = 1, codes = x
    y = oracle.q4_0_linear(x, blob, N)
    assert (y.astype(np.float64) == x.astype(np.float64) @ codes.T.astype(np.float64)).all()


# ---- Q8_0 weights (BlockQ8_0::vec_dot_unopt, k_quants.rs:737-756) ----------


@pytest.mark.parametrize("rows,out_f,in_f,seed", [(1, 8, 64, 21), (3, 12, 512, 22), (4, 37, 4096, 23)])
def test_q8_0_weight_linear_within_counted_bound_of_exact_value(rows, out_f, in_f, seed):
    """The Q8_0-weight linear: the weight written by BlockQ8_0::from_float
    (pinned to gguf-py above), the activations quantised the same way, and the
    result within the reference's counted bound of the exact value; the bound
    refuses the unquantised-activation answer."""
    w = (np.random.default_rng(seed + 1).standard_normal((out_f, in_f)) * 0.05).astype(np.float32)
    x = q4_exact.tie_free_gauss(rows, in_f, seed)
    blob = oracle.q8_0_quantize(w)
    got = oracle.q8_0_linear(x, blob, out_f, threads=3)
    xq = oracle.q8_0_quantize(x)
    exact, abs_sum, ref_err = q4_exact.exact_linear_q8_0(xq, blob, rows, out_f, in_f)
    bound = q4_exact.linear_bound(in_f, abs_sum, ref_err)
    assert float(np.max(np.abs(got - exact) / bound)) <= 1.0
    wdq = oracle.q8_0_dequantize(blob, out_f * in_f).astype(np.float64).reshape(out_f, in_f)
    assert float(np.max(np.abs(x.astype(np.float64) @ wdq.T - exact) / bound)) > 1.0


def test_q8_0_weight_linear_is_the_row_dot_and_lossless_operands_are_exact():
    rng = np.random.default_rng(25)
    M, N, K = 3, 10, 256
    codes = rng.integers(-127, 128, size=(N, K))
    blob = q4_exact.q8_0_blob_from_codes(codes, np.ones((N, K // 32), dtype=np.float16))
    x = rng.integers(-127, 128, size=(M, K)).astype(np.float32)
    x[:, ::32] = 127.0  # every block's absmax is 127 -> d = 1, codes = x
    y = oracle.q8_0_linear(x, blob, N, threads=2)
    assert (y.astype(np.float64) == x.astype(np.float64) @ codes.T.astype(np.float64)).all()
    xq = oracle.q8_0_quantize(x)
    nb = K // 32
    for r in range(M):
        for c in range(N):
            one = oracle.lib().tno_q8_0_q8_0_dot(np.frombuffer(blob, np.uint8)[c * nb * 34:].ctypes.data,
                                                 np.frombuffer(xq, np.uint8)[r * nb * 34:].ctypes.data, nb)
            assert np.float32(one) == y[r, c]


# ---- Q4_K weights with Q8_K activations (k_quants.rs:153-190, 1478-1544) ----


def test_q4_k_reader_bits_equal_llama_cpp():
    cases = [c for c in _golden()["cases"] if c["format"] == "q4_k"]
    assert len(cases) == 1 and cases[0]["name"] == "foreign"
    c = cases[0]
    n = int(np.prod(c["shape"]))
    assert oracle.q4_k_dequantize(bytes.fromhex(c["blob"]), n).tobytes() == bytes.fromhex(c["dequant_f32"])


@pytest.mark.parametrize("seed", [0, 1])
def test_q4_k_reader_equals_installed_gguf_py(seed):
    gguf = pytest.importorskip("gguf")
    from gguf import quants

    rng = np.random.default_rng(seed + 60)
    blob = q4_exact.q4_k_blob(rng, 3, 512)
    want = quants.dequantize(np.frombuffer(blob, np.uint8).reshape(3, -1), gguf.GGMLQuantizationType.Q4_K)
    assert oracle.q4_k_dequantize(blob, 3 * 512).tobytes() == want.astype(np.float32).tobytes()


def test_q8_k_activation_writer_follows_its_rules():
    rng = np.random.default_rng(61)
    x = (rng.standard_normal((2, 512)) * 3).astype(np.float32)
    x[0, 300] = -20.0  # negative signed maximum of the second super-block of row 0 (-> code -127)
    x[1, :256] = 0.0   # an all-zero super-block
    raw = np.frombuffer(oracle.q8_k_quantize(x), np.uint8).reshape(2, 2, 292)
    d = raw[:, :, 0:4].copy().view(np.float32)[..., 0]
    q = raw[:, :, 4:260].copy().view(np.int8).astype(np.int64)
    bs = raw[:, :, 260:].copy().view(np.int16).astype(np.int64)
    assert d[1, 0] == 0.0 and not q[1, 0].any() and not bs[1, 0].any()
    assert q[0, 1, 300 - 256] == -127 and np.float32(d[0, 1]) == np.float32(1.0) / (np.float32(-127.0) / np.float32(-20.0))
    assert (bs == q.reshape(2, 2, 16, 16).sum(axis=3)).all()
    for r in range(2):
        for b in range(2):
            if d[r, b] == 0:
                continue
            xb = x[r, 256 * b:256 * (b + 1)]
            mx = xb[np.argmax(np.abs(xb))]
            iscale = np.float32(-127.0) / np.float32(mx)
            v = (iscale * xb).astype(np.float32)
            want = np.clip(np.where(v >= 0, np.floor(v + 0.5), np.ceil(v - 0.5)), -128, 127)
            assert (q[r, b] == want).all()


@pytest.mark.parametrize("rows,out_f,in_f,seed", [(1, 8, 256, 62), (3, 12, 1024, 63), (2, 37, 4096, 64)])
def test_q4_k_linear_within_counted_bound_of_exact_value(rows, out_f, in_f, seed):
    rng = np.random.default_rng(seed)
    blob = q4_exact.q4_k_blob(rng, out_f, in_f)
    x = (rng.standard_normal((rows, in_f)) * 1.3).astype(np.float32)
    got = oracle.q4_k_linear(x, blob, out_f)
    xq = oracle.q8_k_quantize(x)
    exact, abs_sum, ref_err = q4_exact.exact_linear_q4_k(xq, blob, rows, out_f, in_f)
    bound = q4_exact.linear_bound_q4_k(in_f, abs_sum, ref_err)
    assert float(np.max(np.abs(got - exact) / bound)) <= 1.0
    wdq = oracle.q4_k_dequantize(blob, out_f * in_f).astype(np.float64).reshape(out_f, in_f)
    assert float(np.max(np.abs(x.astype(np.float64) @ wdq.T - exact) / bound)) > 1.0
    # one element is one row dot
    xb = np.frombuffer(xq, np.uint8)
    one = oracle.lib().tno_q4_k_q8_k_dot(np.frombuffer(blob, np.uint8)[(out_f - 1) * (in_f // 256) * 144:].ctypes.data,
                                        xb[(rows - 1) * (in_f // 256) * 292:].ctypes.data, in_f // 256)
    assert np.float32(one) == got[rows - 1, out_f - 1]


def test_q4_k_lossless_operands_give_the_exact_integer_matmul():
    rng = np.random.default_rng(65)
    M, N, K = 3, 10, 512
    blob = q4_exact.q4_k_blob(rng, N, K, lossless=True)
    codes = oracle.q4_k_dequantize(blob, N * K).reshape(N, K).astype(np.float64)  # the nibbles themselves
    assert codes.min() >= 0 and codes.max() <= 15 and (codes == np.round(codes)).all()
    x = rng.integers(-127, 128, size=(M, K)).astype(np.float32)
    x[:, ::256] = 127.0  # every super-block's signed maximum is +127 -> d = -1, codes = -x
    y = oracle.q4_k_linear(x, blob, N)
    assert (y.astype(np.float64) == x.astype(np.float64) @ codes.T).all()
