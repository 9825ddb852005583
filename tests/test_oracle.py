"""The CPU oracle and the host quantiser against the reference's golden
vectors (tests/golden, generated from the unmodified reference by
tests/golden/make_golden.py) and the reference's own known-answer tests.
No GPU needed."""
import numpy as np
import pytest

import nutllm_b200 as nb
from nutllm_b200 import synthetic as syn
from tests.conftest import golden_path

QUANT = np.load(golden_path("quant_golden.npz"))
QMV = np.load(golden_path("qmatvec_golden.npz"))
CASES = sorted({k.rsplit("_", 1)[0] for k in QUANT.files if k.endswith("_input")})


def _dequant(data, scales, rows, cols, qtype):
    n = rows * cols
    if qtype == nb.INT8:
        q = data.view(np.int8).astype(np.float32)
    else:
        v = np.empty(data.size * 2, np.int16)
        v[0::2], v[1::2] = data & 0x0F, data >> 4
        q = np.where(v >= 8, v - 16, v)[:n].astype(np.float32)
    s = scales.view(np.float16).astype(np.float32)
    return (q * np.repeat(s, 32)[:n]).reshape(rows, cols)


@pytest.mark.parametrize("case", CASES)
def test_quantisers_bit_exact_with_reference(orc, case):
    w = QUANT[f"{case}_input"]
    qtype = nb.INT8 if case.endswith("int8") else nb.INT4
    want_d, want_s = QUANT[f"{case}_data"], QUANT[f"{case}_scales"]
    for impl in (orc.quantize, nb.quantize):
        d, s = impl(w, qtype)
        assert np.array_equal(d, want_d)
        assert np.array_equal(s, want_s)
    # QuantizedMatrix::value and storage_bytes (src/quant.cpp:217-240)
    values = _dequant(want_d, want_s, *w.shape, qtype)
    assert np.array_equal(values, QUANT[f"{case}_values"])
    assert int(QUANT[f"{case}_storage"][0]) == want_d.nbytes + want_s.nbytes
    # round trip within the reference's error bound (src/quant_selftest.cpp:23-41)
    assert np.all(np.abs(w - values) <= QUANT[f"{case}_bounds"] + 1e-7)


def test_int4_packing_known_answer(orc):
    """src/quant_selftest.cpp:92-101: [-7, -1, 2, 7] packs to f9 72."""
    w = np.array([[-7.0, -1.0, 2.0, 7.0]], np.float32)
    for impl in (orc.quantize, nb.quantize):
        d, _ = impl(w, nb.INT4)
        assert d.tolist() == [0xF9, 0x72]


def test_storage_accounting():
    """src/quant_selftest.cpp:155-159: int8 n + 2 blocks, int4 ceil(n/2) + 2 blocks."""
    w = np.random.default_rng(1).uniform(-1, 1, (5, 37)).astype(np.float32)
    blocks = (w.size + 31) // 32
    d8, s8 = nb.quantize(w, nb.INT8)
    d4, s4 = nb.quantize(w, nb.INT4)
    assert d8.nbytes + s8.nbytes == w.size + 2 * blocks
    assert d4.nbytes + s4.nbytes == (w.size + 1) // 2 + 2 * blocks


def test_fp16_scale_encoder_sweep(orc):
    """Scales over the whole fp16 range (normals, subnormals, rounding
    boundaries) encode identically in the host quantiser and the oracle."""
    rng = np.random.default_rng(7)
    vals = np.exp(rng.uniform(np.log(1e-9), np.log(65504.0), 20000)).astype(np.float32)
    edges = [2.0 ** -24, 2.0 ** -14, 2.0 ** -14 * (1 - 2 ** -12), 65504.0, 1.0,
             1.0 + 2 ** -11, 1.0 + 3 * 2 ** -11, 2.0 ** -25, 1e-30]
    for v in np.concatenate([vals, np.array(edges, np.float32)]):
        assert nb.scale_to_half(float(v)) == orc.half_from_float(float(v))


def test_quantiser_rejects_what_the_reference_rejects():
    bad = np.array([[1.0, np.nan]], np.float32)
    with pytest.raises(ValueError, match="non-finite"):
        nb.quantize(bad, nb.INT8)
    with pytest.raises(nb.RangeError, match="exceeds fp16"):
        nb.quantize(np.full((1, 32), 1e6, np.float32), nb.INT4)
    with pytest.raises(ValueError):
        nb.quantize(np.zeros((0, 4), np.float32), nb.INT8)


@pytest.mark.parametrize("key", sorted({k.rsplit("_", 1)[0] for k in QMV.files if k.endswith("_y")}))
def test_oracle_qmatvec_bit_exact_with_reference(orc, key):
    rows, cols = (int(v) for v in key.split("_")[0].split("x"))
    qtype = nb.INT8 if key.endswith("int8") else nb.INT4
    y = orc.qmatvec(qtype, rows, cols, QMV[f"{key}_data"], QMV[f"{key}_scales"], QMV[f"{key}_x"])
    assert np.array_equal(y, QMV[f"{key}_y"])


def test_oracle_token_loop_bit_exact_tiny_int8(orc):
    g = np.load(golden_path("tiny_int8_golden.npz"))
    wl = syn.WORKLOADS["tiny-int8"]
    c = wl.model_config()
    w = syn.build_model(c, wl.qtype, 1234)
    assert w.storage_bytes() == int(g["storage"][0])
    prompt = syn.prompt_ids(c, 1234, wl.prompt)
    assert np.array_equal(prompt, g["prompt"])
    ids, logits, hidden = orc.model(w).generate(prompt, wl.steps)
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(logits, g["logits"])
    assert np.array_equal(hidden, g["prefill_hidden"])


@pytest.mark.slow
def test_oracle_token_loop_tinyllama_int4(orc):
    g = np.load(golden_path("tinyllama_int4_golden.npz"))
    wl = syn.WORKLOADS["tinyllama-int4"]
    c = wl.model_config()
    w = syn.build_model(c, wl.qtype, 1234)
    assert w.storage_bytes() == int(g["storage"][0])
    prompt = syn.prompt_ids(c, 1234, wl.prompt)
    ids, logits, hidden = orc.model(w).generate(prompt, wl.steps)
    assert np.array_equal(ids, g["ids"])
    assert np.array_equal(hidden, g["prefill_hidden"])
    assert np.array_equal(np.take_along_axis(logits, g["top_ids"].astype(np.int64), axis=1),
                          g["top_logits"])


def test_synthetic_generator_is_deterministic():
    a = nb.synth_normal(99, 5, 1001, 0.02)
    b = nb.synth_normal(99, 5, 1001, 0.02)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, nb.synth_normal(99, 6, 1001, 0.02))
    assert abs(float(a.std()) - 0.02) < 0.002
    # element i depends only on (seed, stream, i): prefixes agree
    assert np.array_equal(nb.synth_normal(99, 5, 10, 0.02), a[:10])
    t = nb.synth_tokens(3, 3, 1000, 1, 511)
    assert t.min() >= 1 and t.max() <= 511


def _dequantize(orc, w, qtype):
    """dequantize() and error_bound() (src/quant.cpp:199-233) of the host
    quantiser's output for w."""
    d, s = nb.quantize(w, qtype)
    n = w.size
    scale = np.array([orc.half_to_float(int(h)) for h in s], np.float32)
    if qtype == nb.INT8:
        q = d.view(np.int8).astype(np.float32)
    else:
        nib = np.stack([d & 0xF, d >> 4], axis=1).reshape(-1).astype(np.int8)
        q = np.where(nib > 7, nib - 16, nib).astype(np.float32)[:n]
    blk = np.arange(n) // 32
    values = (q * scale[blk]).astype(np.float32).reshape(w.shape)
    half_rounding = np.maximum(scale / np.float32(2047.0), np.float32(2.0 ** -25))
    limit = np.float32(127.0 if qtype == nb.INT8 else 7.0)
    bound = (scale * np.float32(0.5) + (limit + np.float32(0.5)) * half_rounding)[blk]
    return values, bound.reshape(w.shape)


def _matmul_f32(a, b):
    """matmul_naive / matmul_quantized order: each output an in-order float
    sum over the inner index."""
    out = np.zeros((a.shape[0], b.shape[1]), np.float32)
    for k in range(a.shape[1]):
        out = (out + a[:, k:k + 1] * b[k:k + 1, :]).astype(np.float32)
    return out


def _perplexity(logits, targets):
    """perplexity() (src/perplexity.cpp): max-shifted double log-sum-exp."""
    nll = 0.0
    for r in range(logits.shape[0]):
        m = logits[r].max()
        nll += np.log(np.exp((logits[r] - m).astype(np.float64)).sum()) + \
            float(m - logits[r, targets[r]])
    return float(np.exp(nll / logits.shape[0]))


def test_quant_selftest_known_answers(orc):
    """The reference's quantisation self-test on its own seeded inputs
    (src/quant_selftest.cpp:71-184; values printed by the reference and
    recorded in docs/08-quantisation.md:89-99): the host quantiser's
    round-trip worst error/bound ratios 0.879 (INT8) and 0.993 (INT4), the
    quantised-matmul ratios 0.726 and 0.756, and the synthetic perplexities
    11.598 (fp32), 11.608 (INT8), 11.715 (INT4).  Inputs come from the
    oracle's restatement of std::uniform_real_distribution<float> over
    std::mt19937 (seeds 505, 606, 707)."""
    w = orc.uniform_floats(505, -1.0, 1.0, (5, 37))
    left = orc.uniform_floats(606, -1.0, 1.0, (3, 5))
    acts = orc.uniform_floats(707, -1.0, 1.0, (12, 5))
    want_rt = {nb.INT8: 0.879, nb.INT4: 0.993}
    want_mm = {nb.INT8: 0.726, nb.INT4: 0.756}
    ref = _matmul_f32(left, w)
    for qtype in (nb.INT8, nb.INT4):
        values, bound = _dequantize(orc, w, qtype)
        err = np.abs(w - values)
        assert np.all(err <= bound + 1e-7)
        assert round(float((err / bound).max()), 3) == want_rt[qtype]
        mm_bound = np.abs(left.astype(np.float64)) @ bound.astype(np.float64)
        mm_err = np.abs(ref.astype(np.float64) - _matmul_f32(left, values))
        assert np.all(mm_err <= mm_bound + 1e-5)
        assert round(float((mm_err / mm_bound).max()), 3) == want_mm[qtype]
    fp32 = _matmul_f32(acts, w)
    targets = np.argmax(fp32, axis=1)
    got = [_perplexity(fp32, targets)] + [
        _perplexity(_matmul_f32(acts, _dequantize(orc, w, q)[0]), targets)
        for q in (nb.INT8, nb.INT4)]
    assert [round(v, 3) for v in got] == [11.598, 11.608, 11.715]


def test_oracle_synthetic_generator_bit_identical_to_host_library(orc):
    """The reference's CPU baseline draws its weights and prompt through the
    oracle's own restatement of the seeded generator; it must give the host
    library's bytes exactly (odd lengths and several streams included)."""
    import oracle
    for seed, stream, n, sigma in ((1234, 1, 4097, 0.02), (7, 1003, 1 << 16, 0.02),
                                   (99, 8, 33, 1.0), (1234, 2, 1, 0.02)):
        a = orc.synth_normal(seed, stream, n, sigma)
        b = nb.synth_normal(seed, stream, n, sigma)
        assert a.tobytes() == b.tobytes()
    for seed, stream, n, lo, hi in ((1234, 3, 512, 1, 31999), (5, 9, 100, 1, 511)):
        assert np.array_equal(orc.synth_tokens(seed, stream, n, lo, hi),
                              nb.synth_tokens(seed, stream, n, lo, hi))
    c = syn.WORKLOADS["tiny-int8"].model_config()
    assert np.array_equal(oracle.projection_fp32(c, 1234, 2, 6),
                          syn.projection_fp32(c, 1234, 2, 6))
    assert np.array_equal(oracle.prompt_ids(c, 1234, 5), syn.prompt_ids(c, 1234, 5))
