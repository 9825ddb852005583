"""fp32 safetensors checkpoints and the byte-level BPE tokenizer: the host
loader (SafeTensorFile / load_model, reference src/loader.cpp:24-498), the
Tokenizer (src/tokenizer.cpp) and generate_tokens / generate_tokens_cached
over fp32 weights (src/generate.cpp:101-172) through the C++ host API.

Checkpoints and tokenizer files are rebuilt from seeds by
tests/golden/make_safetensors_fixture.py; tests/golden/safetensors_golden.npz
holds the unmodified reference's results on the same bytes: configs,
storage sizes and byte digests, generated ids, and the class and message of
every malformed file.  CPU tests pin the host loader, the tokenizer and the
oracle; GPU tests run generation on the device.
"""
import hashlib
import os

import numpy as np
import pytest

import nutllm_b200 as nb
import oracle
from tests.conftest import golden_path
from tests.golden import make_safetensors_fixture as fx

G = np.load(golden_path("safetensors_golden.npz"))
REF_FIXTURES = os.path.join(oracle.reference_dir() or os.devnull, "tests", "fixtures")
HAVE_REF_FIXTURES = os.path.exists(os.path.join(REF_FIXTURES, "tiny.safetensors"))
STATUS = {ValueError: 1, IndexError: 2, nb.LengthError: 3, RuntimeError: 4,
          nb.RangeError: 5}


def _status(exc) -> int:
    for cls, code in STATUS.items():
        if type(exc) is cls:
            return code
    raise AssertionError(f"unexpected exception class {type(exc)}")


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    d = tmp_path_factory.mktemp("safetensors")
    out = {}
    for name in fx.CONFIGS:
        p = d / f"{name}.safetensors"
        p.write_bytes(fx.safetensors_bytes(name))
        out[name] = str(p)
    return out


@pytest.fixture(scope="module")
def bpe(tmp_path_factory):
    d = tmp_path_factory.mktemp("bpe")
    v, m = fx.bpe_files()
    (d / "v.txt").write_text(v)
    (d / "m.txt").write_text(m)
    return str(d / "v.txt"), str(d / "m.txt")


# ------------------------------------------------------------------ CPU


@pytest.mark.parametrize("name", list(fx.CONFIGS))
def test_fixture_bytes_match_golden(files, name):
    digest = hashlib.sha256(open(files[name], "rb").read()).digest()
    assert np.array_equal(np.frombuffer(digest, np.uint8), G[f"{name}/sha256"])


@pytest.mark.parametrize("name", list(fx.CONFIGS))
def test_loader_matches_reference_bytes(files, name):
    """Config, storage_bytes() and every loaded byte (the [in][out]
    matrices after the transpose, norms, embeddings, lm_head) equal the
    reference loader's."""
    cfg, nbytes, digest = nb.safetensors_inspect(files[name])
    assert cfg == G[f"{name}/config"].tolist()
    assert nbytes == int(G[f"{name}/storage_bytes"])
    assert digest == int(G[f"{name}/digest"])


@pytest.mark.parametrize("label", list(fx.malformed_cases()))
def test_malformed_file_errors_match_reference(tmp_path, label):
    """Every damaged file fails with the reference's class and message."""
    data = fx.malformed_cases()[label]
    assert np.array_equal(np.frombuffer(hashlib.sha256(data).digest(), np.uint8),
                          G[f"bad/{label}/sha256"])
    p = tmp_path / "bad.safetensors"
    p.write_bytes(data)
    with pytest.raises(Exception) as e:
        nb.safetensors_inspect(str(p))
    assert _status(e.value) == int(G[f"bad/{label}/status"])
    assert str(e.value) == bytes(G[f"bad/{label}/message"]).decode()


def test_missing_file(tmp_path):
    p = str(tmp_path / "absent.safetensors")
    with pytest.raises(RuntimeError, match=f"safetensors: cannot open {p}: No such file"):
        nb.safetensors_inspect(p)


@pytest.mark.parametrize("name", list(fx.CONFIGS))
def test_oracle_generation_matches_reference(orc, files, name):
    """The oracle's fp32 decoder over load_model's tensors gives the
    reference's ids (greedy and seeded top-p; the reference's cached and
    uncached loops agree on these)."""
    c = fx.config_of(name)
    m = orc.fp32_model(oracle.read_safetensors_model(files[name]))
    prompt = G[f"{name}/prompt"]
    for cached in (0, 1):
        assert (m.generate_cached(prompt, c["max_tokens"])[0].tolist()
                == G[f"{name}/greedy{cached}"].tolist())
        assert (m.generate_cached(prompt, c["max_tokens"], **fx.SAMPLING)[0].tolist()
                == G[f"{name}/sampled{cached}"].tolist())


def test_bpe_files_match_golden(bpe):
    v, m = fx.bpe_files()
    assert np.array_equal(
        np.frombuffer(hashlib.sha256((v + "\0" + m).encode()).digest(), np.uint8),
        G["bpe/sha256"])


@pytest.mark.parametrize("i", range(len(fx.BPE_TEXTS)))
def test_bpe_matches_reference(bpe, i):
    ids = nb.bpe_encode(*bpe, fx.BPE_TEXTS[i])
    assert ids == G[f"bpe/t{i}/ids"].tolist()
    assert nb.bpe_decode(*bpe, ids) == fx.BPE_TEXTS[i]


@pytest.mark.parametrize("label", list(fx.bpe_malformed()))
def test_bpe_malformed_errors_match_reference(tmp_path, label):
    v, m = fx.bpe_malformed()[label]
    (tmp_path / "v.txt").write_text(v)
    (tmp_path / "m.txt").write_text(m)
    with pytest.raises(Exception) as e:
        nb.bpe_encode(str(tmp_path / "v.txt"), str(tmp_path / "m.txt"), b"a")
    assert _status(e.value) == int(G[f"bpebad/{label}/status"])
    assert str(e.value) == bytes(G[f"bpebad/{label}/message"]).decode()


def test_bpe_errors(bpe, tmp_path):
    with pytest.raises(IndexError, match="tokenizer: token id out of range"):
        nb.bpe_decode(*bpe, [10 ** 6])
    with pytest.raises(RuntimeError, match="tokenizer: cannot open vocabulary"):
        nb.bpe_encode(str(tmp_path / "none"), bpe[1], b"a")
    with pytest.raises(RuntimeError, match="tokenizer: cannot open merges"):
        nb.bpe_encode(bpe[0], str(tmp_path / "none"), b"a")
    # a byte without a token
    (tmp_path / "v.txt").write_text("0 61\n1 62\n")
    (tmp_path / "m.txt").write_text("")
    with pytest.raises(RuntimeError, match="tokenizer: input byte absent from vocabulary"):
        nb.bpe_encode(str(tmp_path / "v.txt"), str(tmp_path / "m.txt"), b"abc")
    # a signed id is read as the reference's formatted read takes it
    (tmp_path / "v.txt").write_text("+0 61\n1 62\n")
    assert nb.bpe_encode(str(tmp_path / "v.txt"), str(tmp_path / "m.txt"), b"ba") == [1, 0]


@pytest.mark.skipif(not HAVE_REF_FIXTURES,
                    reason="reference fixtures are only present where the reference is")
def test_reference_fixture_known_answer(orc):
    """The reference's own tiny.safetensors + tiny.vocab/merges: encode("H")
    is [0], greedy generation gives [1, 2] and the whole decodes to "Hi!"
    (src/loader_selftest.cpp:48-78)."""
    v, m = (os.path.join(REF_FIXTURES, f) for f in ("tiny.vocab", "tiny.merges"))
    prompt = nb.bpe_encode(v, m, b"H")
    assert prompt == [0]
    t = oracle.read_safetensors_model(os.path.join(REF_FIXTURES, "tiny.safetensors"))
    ids = orc.fp32_model(t).generate_cached(prompt, 8)[0].tolist()
    assert ids == [1, 2]
    assert nb.bpe_decode(v, m, prompt + ids) == b"Hi!"
    cfg, _, _ = nb.safetensors_inspect(os.path.join(REF_FIXTURES, "tiny.safetensors"))
    assert cfg[0] == 2 and cfg[7] == 3


# ------------------------------------------------------------------ GPU


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(fx.CONFIGS))
def test_generation_matches_reference(gpu, files, name):
    """load_model + generate_tokens / generate_tokens_cached on the device:
    greedy and seeded top-p ids equal the reference's."""
    c = fx.config_of(name)
    prompt = G[f"{name}/prompt"]
    for cached in (0, 1):
        ids = nb.safetensors_generate(files[name], prompt, c["max_tokens"],
                                      cached=bool(cached))
        assert ids.tolist() == G[f"{name}/greedy{cached}"].tolist()
        ids = nb.safetensors_generate(files[name], prompt, c["max_tokens"],
                                      cached=bool(cached), **fx.SAMPLING)
        assert ids.tolist() == G[f"{name}/sampled{cached}"].tolist()


@pytest.mark.gpu
def test_generation_errors(gpu, files):
    p = files["odd_context"]
    with pytest.raises(ValueError, match="generation: prompt cannot be empty"):
        nb.safetensors_generate(p, np.zeros(0, np.int32), 4, cached=False)
    with pytest.raises(nb.LengthError, match="generation: prompt exceeds context"):
        nb.safetensors_generate(p, np.zeros(17, np.int32), 4, cached=False)
    with pytest.raises(ValueError, match="generation: invalid prompt length"):
        nb.safetensors_generate(p, np.zeros(17, np.int32), 4)
    # a full context generates nothing
    assert nb.safetensors_generate(p, np.zeros(16, np.int32), 4, cached=False).size == 0


@pytest.mark.gpu
@pytest.mark.skipif(not HAVE_REF_FIXTURES,
                    reason="reference fixtures are only present where the reference is")
def test_reference_fixture_on_device(gpu):
    ids = nb.safetensors_generate(os.path.join(REF_FIXTURES, "tiny.safetensors"), [0], 8,
                                  cached=False)
    assert ids.tolist() == [1, 2]
