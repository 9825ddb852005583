"""llama2.c checkpoints end to end: the host loaders (load_llama2c_quantized_model
and the fp32 load_llama2c_model, reference src/llama2.cpp:199-412), the
generation sampler (choose_token, src/generate.cpp:25-73) and both overloads
of generate_tokens_cached (src/generate.cpp:128-216) through the C++ host API.

Checkpoints are rebuilt from seeds by tests/golden/make_llama2c_fixture.py;
the goldens in tests/golden/llama2c_golden.npz were produced by the
unmodified reference from the same bytes.  CPU tests pin the oracle's
restatement and the host loader/sampler; GPU tests run the product path.
"""
import hashlib
import os

import numpy as np
import pytest

import nutllm_b200 as nb
import oracle
from tests.conftest import golden_path
from tests.golden import make_llama2c_fixture as fx

G = np.load(golden_path("llama2c_golden.npz"))
QTYPES = ((0, "int8"), (1, "int4"), (2, "fp32"))
REF_FIXTURES = os.path.join(oracle.reference_dir() or os.devnull, "tests", "fixtures")


@pytest.fixture(scope="module")
def checkpoints(tmp_path_factory):
    d = tmp_path_factory.mktemp("llama2c")
    return {name: fx.write_checkpoint(str(d / f"{name}.bin"), name) for name in fx.CONFIGS}


def _oracle_model(orc, path, qtype):
    """A host image of the checkpoint quantised by the oracle's quantiser."""
    t = oracle.read_llama2c(path)
    c = nb.Config(**t["config"])

    def q(w):
        data, scales = orc.quantize(w, qtype)
        return nb.QuantizedMatrix(data, scales, w.shape[0], w.shape[1], qtype)

    layers = []
    for l in range(c.layers):
        layers.append(nb.LayerWeights(
            q(t["wq"][l]), q(t["wk"][l]), q(t["wv"][l]), q(t["wo"][l]), q(t["w1"][l]),
            q(t["w3"][l]), q(t["w2"][l]),
            attention_norm=np.ascontiguousarray(t["attention_norm"][l]),
            ffn_norm=np.ascontiguousarray(t["ffn_norm"][l])))
    return nb.ModelWeights(
        config=c, qtype=qtype, embeddings=np.ascontiguousarray(t["embeddings"]),
        layers=layers, final_norm=np.ascontiguousarray(t["final_norm"]),
        lm_head=None if t["tied"] else np.ascontiguousarray(t["classifier"]),
        tied_embeddings=t["tied"])


# ------------------------------------------------------------------ CPU


@pytest.mark.parametrize("name", list(fx.CONFIGS))
def test_fixture_bytes_match_golden(checkpoints, name):
    digest = hashlib.sha256(open(checkpoints[name], "rb").read()).digest()
    assert np.array_equal(np.frombuffer(digest, np.uint8), G[f"{name}/sha256"])


@pytest.mark.parametrize("qtype,qname", QTYPES)
@pytest.mark.parametrize("name", list(fx.CONFIGS))
def test_host_loader_matches_reference_bytes(checkpoints, name, qtype, qname):
    """Config, tied flag, storage_bytes() and every loaded byte (quantised
    data, fp16 scales, fp32 norms/embeddings/classifier) equal the reference
    loader's."""
    cfg, tied, nbytes, digest = nb.llama2c_inspect(checkpoints[name], qtype)
    key = f"{name}/{qname}"
    assert cfg == G[f"{key}/config"].tolist()
    assert tied == bool(G[f"{key}/tied"])
    assert nbytes == int(G[f"{key}/storage_bytes"])
    assert digest == int(G[f"{key}/digest"])


@pytest.mark.parametrize("qtype,qname", QTYPES)
@pytest.mark.parametrize("name", list(fx.CONFIGS))
def test_oracle_generation_matches_reference(orc, checkpoints, name, qtype, qname):
    """The oracle's generate_tokens_cached (eos stop, context limit, greedy
    and seeded top-p) gives the reference's ids on the reference's bytes."""
    c = fx.config_of(name)
    prompt = G[f"{name}/prompt"]
    key = f"{name}/{qname}"
    if qtype == nb.FP32:
        m = orc.fp32_model(oracle.read_llama2c(checkpoints[name]))
        gen = lambda *a, **k: m.generate_cached(*a, **k)[0]  # noqa: E731
    else:
        m = orc.model(_oracle_model(orc, checkpoints[name], qtype))
        gen = m.generate_cached
    assert gen(prompt, c["max_tokens"]).tolist() == G[f"{key}/greedy"].tolist()
    assert (gen(prompt, c["max_tokens"], **fx.SAMPLING).tolist()
            == G[f"{key}/sampled"].tolist())


def _logit_rows(seed):
    rng = np.random.default_rng(seed)
    rows = [rng.standard_normal(300).astype(np.float32) * 3,
            np.zeros(17, np.float32),                                   # all ties
            np.repeat(rng.standard_normal(8), 5).astype(np.float32),    # tied pairs
            np.array([5.0], np.float32),
            (rng.standard_normal(2000) * 0.01).astype(np.float32)]
    return rows


@pytest.mark.parametrize("temperature,top_p", [(0.0, 1.0), (0.7, 0.9), (1.0, 1.0),
                                               (2.5, 0.5), (0.3, 1e-6), (1.3, 0.999)])
def test_sampler_matches_oracle(orc, temperature, top_p):
    for seed in (1, 7, 4242):
        for i, row in enumerate(_logit_rows(seed)):
            steps = np.tile(row, (6, 1))  # six draws from one generator
            want = orc.choose_tokens(steps, temperature, top_p, seed + i)
            got = nb.choose_tokens(steps, temperature, top_p, seed + i)
            assert got.tolist() == want.tolist(), (seed, i)


@pytest.mark.parametrize("temperature,top_p", [(0.5, 0.0), (0.5, 1.5), (float("inf"), 0.9),
                                               (float("nan"), 0.9)])
def test_sampler_rejects_bad_settings(temperature, top_p):
    with pytest.raises(ValueError, match="sampling: invalid temperature or top-p"):
        nb.choose_tokens(np.zeros((1, 4), np.float32), temperature, top_p, 1)


def _write_header(path, header, floats=0):
    with open(path, "wb") as f:
        f.write(np.array(header, np.int32).tobytes())
        f.write(np.zeros(floats, np.float32).tobytes())
    return str(path)


@pytest.mark.parametrize("header,floats,error,message", [
    ([4, 4], 0, RuntimeError, "llama2 checkpoint: truncated header"),
    ([0, 4, 1, 1, 1, 6, 8], 0, RuntimeError, "llama2 checkpoint: invalid dimension"),
    ([4, 4, 1, 1, 1, 0, 8], 0, RuntimeError, "llama2 checkpoint: invalid vocabulary"),
    ([6, 4, 1, 4, 4, 6, 8], 0, RuntimeError, "heads do not divide dimension"),
    ([4, 4, 1, 1, 1, 6, 8], 10, RuntimeError, "size does not match configuration"),
    ([4, 4, 1, 1, 2, 6, 8], 0, ValueError, "model config: invalid dimensions"),
])
def test_loader_errors_match_reference(tmp_path, header, floats, error, message):
    path = _write_header(tmp_path / "bad.bin", header, floats)
    with pytest.raises(error, match=message):
        nb.llama2c_inspect(path, 1)
    if oracle.reference_available():
        with pytest.raises(RuntimeError, match=message):
            oracle.Reference().llama2c_inspect(path, 1)


def test_loader_missing_file(tmp_path):
    with pytest.raises(RuntimeError, match="llama2 checkpoint: cannot open"):
        nb.llama2c_inspect(str(tmp_path / "absent.bin"), 0)


@pytest.mark.skipif(not os.path.isdir(REF_FIXTURES) or not oracle.reference_available(),
                    reason="reference fixtures are only present where the reference is")
@pytest.mark.parametrize("fname", ["tiny-llama2.bin", "tiny-llama2-shared.bin"])
@pytest.mark.parametrize("qtype,qname", QTYPES)
def test_reference_fixtures(orc, ref, fname, qtype, qname):
    """The reference's own llama2.c fixtures: the host loader reads the same
    bytes as the reference loader, and the oracle reproduces the reference's
    known answer (greedy ids {4, 5} after the prompt "H", fp32 and both
    quantisations, src/loader_selftest.cpp:84-116)."""
    path = os.path.join(REF_FIXTURES, fname)
    assert nb.llama2c_inspect(path, qtype) == ref.llama2c_inspect(path, qtype)
    if fname == "tiny-llama2.bin":
        prompt = ref.llama2c_encode(os.path.join(REF_FIXTURES, "tiny-llama2.tokenizer"),
                                    6, "H")
        want = ref.llama2c_generate(path, qtype, prompt, 32)
        assert want.tolist() == [4, 5]
        if qtype == nb.FP32:
            ids = orc.fp32_model(oracle.read_llama2c(path)).generate_cached(prompt, 32)[0]
        else:
            ids = orc.model(_oracle_model(orc, path, qtype)).generate_cached(prompt, 32)
        assert ids.tolist() == [4, 5]


# ------------------------------------------------------------------ GPU


@pytest.mark.gpu
@pytest.mark.parametrize("qtype,qname", QTYPES)
@pytest.mark.parametrize("name", list(fx.CONFIGS))
def test_llama2c_generation_matches_reference(gpu, checkpoints, name, qtype, qname):
    """Loader + generate_tokens_cached through the C++ host API on the
    device: greedy and seeded top-p ids equal the reference's."""
    c = fx.config_of(name)
    prompt = G[f"{name}/prompt"]
    key = f"{name}/{qname}"
    ids, st = nb.llama2c_generate(checkpoints[name], qtype, prompt, c["max_tokens"])
    assert ids.tolist() == G[f"{key}/greedy"].tolist()
    assert st.prefill_tokens == len(prompt) and st.generated_tokens == len(ids)
    ids, st = nb.llama2c_generate(checkpoints[name], qtype, prompt, c["max_tokens"],
                                  **fx.SAMPLING)
    assert ids.tolist() == G[f"{key}/sampled"].tolist()
    assert st.generated_tokens == len(ids)


@pytest.mark.gpu
def test_llama2c_generation_errors(gpu, checkpoints):
    path = checkpoints["gqa_separate"]
    with pytest.raises(ValueError, match="generation: invalid prompt length"):
        nb.llama2c_generate(path, 1, np.zeros(0, np.int32), 4)
    with pytest.raises(ValueError, match="generation: invalid prompt length"):
        nb.llama2c_generate(path, 1, np.full(49, 2, np.int32), 4)
    with pytest.raises(IndexError, match="token out of range"):
        nb.llama2c_generate(path, 1, np.array([2, 300], np.int32), 4)
    with pytest.raises(ValueError, match="sampling: invalid temperature or top-p"):
        nb.llama2c_generate(path, 1, np.array([2, 3], np.int32), 4, temperature=0.5,
                            top_p=0.0)
    ids, _ = nb.llama2c_generate(path, 1, np.array([2, 3], np.int32), 0)
    assert ids.size == 0
    # the fp32 path keeps prefill_tokens' messages
    with pytest.raises(IndexError, match="kv cache: token id out of range"):
        nb.llama2c_generate(path, nb.FP32, np.array([2, 300], np.int32), 4)
    with pytest.raises(ValueError, match="generation: invalid prompt length"):
        nb.llama2c_generate(path, nb.FP32, np.zeros(0, np.int32), 4)


def _fp32_device_model(t):
    layers = [dict(query=t["wq"][l], key=t["wk"][l], value=t["wv"][l], output=t["wo"][l],
                   gate=t["w1"][l], up=t["w3"][l], down=t["w2"][l],
                   attention_norm=t["attention_norm"][l], ffn_norm=t["ffn_norm"][l])
              for l in range(t["config"]["layers"])]
    return nb.DeviceModel.fp32(nb.Config(**t["config"]), t["embeddings"], layers,
                               t["final_norm"], None if t["tied"] else t["classifier"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(fx.CONFIGS))
def test_fp32_decode_matches_oracle(gpu, orc, checkpoints, name):
    """decode_token over fp32 weights (src/kvcache.cpp:265-284) on the
    device: hidden rows and logits of every prompt position and greedy step
    within 2e-3 absolute + 1e-3 relative of the oracle's restatement (fp32
    projections summed in a different order than linear_threaded), the same
    ids, and the cache holding the oracle's keys and values."""
    t = oracle.read_llama2c(checkpoints[name])
    want = orc.fp32_model(t)
    dm = _fp32_device_model(t)
    cache = nb.KVCache(dm)
    c = fx.config_of(name)
    prompt = [int(v) for v in G[f"{name}/prompt"]]
    tok = prompt[0]
    for step in range(min(len(prompt) + c["max_tokens"] // 2, t["config"]["max_seq"])):
        h = nb.decode_quantized_token(dm, tok, cache)
        hw = want.decode(tok)
        assert np.allclose(h, hw, atol=2e-3, rtol=1e-3), float(np.abs(h - hw).max())
        lg, best = nb.logits(dm, cache)
        lw = want.logits(hw)
        assert np.allclose(lg, lw, atol=2e-3, rtol=1e-3), float(np.abs(lg - lw).max())
        if step + 1 < len(prompt):
            tok = prompt[step + 1]
        else:
            assert best == int(np.argmax(lw))
            tok = best
    assert cache.length() == want.length
    kvh = t["config"]["kv_heads"]
    for l in range(t["config"]["layers"]):
        for hh in range(kvh):
            for pos in (0, want.length - 1):
                assert np.allclose(cache.key(l, hh, pos), want.keys[l, hh, pos], atol=2e-3,
                                   rtol=1e-3)
                assert np.allclose(cache.value(l, hh, pos), want.values[l, hh, pos],
                                   atol=2e-3, rtol=1e-3)
    with pytest.raises(IndexError, match="kv cache: token id out of range"):
        nb.decode_quantized_token(dm, t["config"]["vocab_size"], cache)
    cache.close()
    dm.close()


SELFTEST = os.path.join(os.path.dirname(nb.HOST_LIB), "..", "bin", "nutllm_selftest")


def test_host_selftest_binary_built():
    import subprocess
    r = subprocess.run([SELFTEST], capture_output=True, text=True)
    assert r.returncode == 2 and "usage" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("qname", ["int8", "int4"])
@pytest.mark.parametrize("name", list(fx.CONFIGS))
def test_host_api_selftest(gpu, checkpoints, name, qname):
    """The C++ API a reference caller uses (KVCache, prefill_quantized,
    decode_quantized_token, generate_tokens_cached, loader) and its
    exception classes, exercised by nutllm_selftest on the device."""
    import subprocess
    prompt = [str(int(t)) for t in G[f"{name}/prompt"]]
    r = subprocess.run([SELFTEST, checkpoints[name], qname, *prompt], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout and "all host API checks passed" in r.stdout


# ------------------------------------------------------------------ tokenizer

TG = np.load(golden_path("tokenizer_golden.npz"))


@pytest.fixture(scope="module")
def tokenizer_file(tmp_path_factory):
    path, vocab = fx.write_tokenizer(str(tmp_path_factory.mktemp("tok") / "tok.bin"))
    assert np.array_equal(np.frombuffer(hashlib.sha256(open(path, "rb").read()).digest(),
                                        np.uint8), TG["sha256"])
    return path, vocab


@pytest.mark.parametrize("i", range(len(fx.TOKENIZER_TEXTS)))
def test_tokenizer_matches_reference(tokenizer_file, i):
    """Llama2Tokenizer encode (BOS / no BOS / BOS+EOS) and decode give the
    reference's ids and bytes: merges by score with first-position ties, the
    first id of a duplicated piece, byte fallback for characters without a
    token, the dummy-prefix space and its removal after BOS."""
    path, vocab = tokenizer_file
    text = fx.TOKENIZER_TEXTS[i]
    for bos, eos in ((1, 0), (0, 0), (1, 1)):
        ids = nb.tokenizer_encode(path, vocab, text, bool(bos), bool(eos))
        assert ids == TG[f"t{i}/ids{bos}{eos}"].tolist()
        back = nb.tokenizer_decode(path, vocab, ids if not eos else ids[:-1])
        assert back == bytes(TG[f"t{i}/text{bos}{eos}"])


def test_tokenizer_errors(tmp_path, tokenizer_file):
    path, vocab = tokenizer_file
    with pytest.raises(RuntimeError, match="llama2 tokenizer: cannot open"):
        nb.tokenizer_encode(str(tmp_path / "absent.bin"), vocab, "a")
    with pytest.raises(RuntimeError, match="llama2 tokenizer: trailing data"):
        nb.tokenizer_encode(path, vocab - 1, "a")
    with pytest.raises(RuntimeError, match="malformed vocabulary entry|truncated token"):
        nb.tokenizer_encode(path, vocab + 1, "a")
    with pytest.raises(ValueError, match="llama2 tokenizer: invalid vocabulary"):
        nb.tokenizer_encode(path, 0, "a")
    with pytest.raises(IndexError, match="llama2 tokenizer: token id out of range"):
        nb.tokenizer_decode(path, vocab, [5, vocab])


@pytest.mark.skipif(not os.path.isdir(REF_FIXTURES),
                    reason="reference fixtures are only present where the reference is")
def test_tokenizer_reference_fixture():
    """The reference's known answer: "H" encodes to the prompt whose greedy
    continuation {4, 5} decodes to "Hi!" (src/loader_selftest.cpp:82-116)."""
    tok = os.path.join(REF_FIXTURES, "tiny-llama2.tokenizer")
    ids = nb.tokenizer_encode(tok, 6, "H")
    if oracle.reference_available():
        assert ids == oracle.Reference().llama2c_encode(tok, 6, "H").tolist()
    assert nb.tokenizer_decode(tok, 6, ids + [4, 5]) == b"Hi!"


def _write_tinyllama_shape(path, layers=2, seed=77):
    """A seeded llama2.c checkpoint of TinyLlama's layer shape (dim 2048,
    FFN 5632, 32 heads over 4 kv heads, vocabulary 32000, tied classifier)
    with `layers` layers, written tensor by tensor."""
    dim, ffn, heads, kv, vocab, max_seq = 2048, 5632, 32, 4, 32000, 256
    hd = dim // heads
    kvd = kv * hd
    stream = [1000]

    def normal(n, sigma=0.02):
        stream[0] += 1
        return nb.synth_normal(seed, stream[0], n, sigma)

    with open(path, "wb") as f:
        f.write(np.array([dim, ffn, layers, heads, kv, vocab, max_seq], np.int32).tobytes())
        f.write(normal(vocab * dim).tobytes())                         # embeddings
        f.write(np.ones(layers * dim, np.float32).tobytes())           # attention norms
        for rows, cols in ((dim, dim), (kvd, dim), (kvd, dim), (dim, dim)):
            f.write(normal(layers * rows * cols).tobytes())            # wq wk wv wo
        f.write(np.ones(layers * dim, np.float32).tobytes())           # ffn norms
        for rows, cols in ((ffn, dim), (dim, ffn), (ffn, dim)):
            f.write(normal(layers * rows * cols).tobytes())            # w1 w2 w3
        f.write(np.ones(dim, np.float32).tobytes())                    # final norm
        f.write(np.zeros(max_seq * hd, np.float32).tobytes())          # RoPE (unused)
    return path


@pytest.mark.gpu
@pytest.mark.slow
def test_streaming_loader_tinyllama_shape(gpu, orc, tmp_path):
    """load_llama2c_quantized_model streams to the device: layer l + 1 is
    read and quantised on the host while layer l is packed and uploaded,
    and the returned weights carry that device image.  On a two-layer
    TinyLlama-shape INT4 checkpoint, the host bytes equal the oracle
    quantiser's (storage size), the generated ids equal the oracle's greedy
    ids at every step whose top-2 gap is clear, and the load is timed."""
    import time
    path = _write_tinyllama_shape(str(tmp_path / "tl2.bin"))
    prompt = np.array([1, 3407, 20, 9011, 17], np.int32)
    steps = 6
    t0 = time.perf_counter()
    ids, st = nb.llama2c_generate(path, nb.INT4, prompt, steps)
    total = time.perf_counter() - t0
    work = st.prefill_seconds + st.decode_seconds
    m = _oracle_model(orc, path, nb.INT4)
    cfg, tied, nbytes, _ = nb.llama2c_inspect(path, nb.INT4)
    assert tied and nbytes == m.storage_bytes()
    om = orc.model(m)
    ids_o, lg_o, _ = om.generate(prompt, steps)
    assert len(ids) == steps
    s = np.sort(lg_o, axis=1)
    clear = (s[:, -1] - s[:, -2]) > 4e-3
    print(f"streaming load + generate of a 2-layer TinyLlama-shape INT4 checkpoint "
          f"({os.path.getsize(path) / 1e6:.0f} MB): {total:.2f} s, of which "
          f"{work * 1e3:.1f} ms on the device; ids compared at {int(clear.sum())} of {steps}")
    first = next((i for i, c in enumerate(clear) if not c), steps)
    assert first > 0
    assert ids[:first].tolist() == ids_o[:first].tolist()
