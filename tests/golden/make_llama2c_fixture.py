"""Seeded llama2.c checkpoints and their golden outputs from the reference.

Test infrastructure.  ``write_checkpoint(path, name)`` writes a small
checkpoint in the llama2.c "legacy" format that the reference's
load_llama2c_quantized_model reads (src/llama2.cpp:199-298): seven int32
(dim, ffn_dim, layers, heads, kv_heads, vocab — negative when a separate
classifier follows — and max_seq), then fp32 embeddings, attention norms,
wq, wk, wv, wo, ffn norms, w1 (gate), w2 (down), w3 (up), final norm, RoPE
tables (never read) and the optional classifier.  Weights come from
numpy's seeded generator, so the tests rebuild the same bytes on any machine
(the file's SHA-256 is stored beside the goldens and checked).

Run here, where the reference builds (``make -C oracle ref``), to refresh
``llama2c_golden.npz``:

    python tests/golden/make_llama2c_fixture.py

For each checkpoint and loader type (INT8, INT4 through
load_llama2c_quantized_model; fp32 through load_llama2c_model) it records the
reference loader's config, tied flag, storage_bytes() and byte digest, and
the ids of the reference's generate_tokens_cached: greedy, and top-p sampled
with a fixed seed, both with the reference's eos stop (token 1) and context
limit.
"""
from __future__ import annotations

import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "llama2c_golden.npz")

# name: (dim, ffn, layers, heads, kv_heads, vocab (negative = separate
# classifier), max_seq, seed, prompt length, max_tokens, projection gain)
CONFIGS = {
    # GQA with a separate classifier; widths multiple of 32 (tiled device path)
    "gqa_separate": (128, 352, 2, 4, 2, -300, 48, 11, 7, 12, 1.0),
    # shared classifier, widths not multiples of 32 (blocks span rows); the
    # context fills before max_tokens, so generation stops at capacity.  The
    # larger gain keeps the layers from being swamped by the input token's
    # own embedding (which a tied classifier would otherwise echo back).
    "unaligned_shared": (24, 40, 2, 2, 2, 40, 24, 12, 6, 40, 4.0),
}

SAMPLING = dict(temperature=1.1, top_p=0.9, seed=7)


def config_of(name: str) -> dict:
    dim, ffn, layers, heads, kv, vocab, max_seq, seed, n_prompt, max_tokens, gain = CONFIGS[name]
    return dict(dim=dim, ffn=ffn, layers=layers, heads=heads, kv_heads=kv, vocab=vocab,
                max_seq=max_seq, seed=seed, n_prompt=n_prompt, max_tokens=max_tokens,
                gain=gain)


def checkpoint_bytes(name: str) -> bytes:
    c = config_of(name)
    dim, ffn, layers, heads, kv = c["dim"], c["ffn"], c["layers"], c["heads"], c["kv_heads"]
    vocab = abs(c["vocab"])
    hd = dim // heads
    kvd = kv * hd
    rng = np.random.default_rng(c["seed"])

    def mat(rows, cols, count=1):
        return (c["gain"] * rng.standard_normal((count, rows, cols)) /
                np.sqrt(cols)).astype(np.float32)

    def gains(count):
        return (1.0 + 0.1 * rng.standard_normal((count, dim))).astype(np.float32)

    parts = [np.array([dim, ffn, layers, heads, kv, c["vocab"], c["max_seq"]], np.int32)]
    parts.append(rng.standard_normal((vocab, dim)).astype(np.float32))  # embeddings
    parts.append(gains(layers))                                          # attention norms
    parts.append(mat(dim, dim, layers))                                  # wq
    parts.append(mat(kvd, dim, layers))                                  # wk
    parts.append(mat(kvd, dim, layers))                                  # wv
    parts.append(mat(dim, dim, layers))                                  # wo
    parts.append(gains(layers))                                          # ffn norms
    parts.append(mat(ffn, dim, layers))                                  # w1 gate
    parts.append(mat(dim, ffn, layers))                                  # w2 down
    parts.append(mat(ffn, dim, layers))                                  # w3 up
    parts.append(gains(1))                                               # final norm
    parts.append(rng.standard_normal((c["max_seq"], hd)).astype(np.float32))  # RoPE (unused)
    if c["vocab"] < 0:
        parts.append((rng.standard_normal((vocab, dim)) / np.sqrt(dim)).astype(np.float32))
    return b"".join(p.tobytes() for p in parts)


def write_checkpoint(path: str, name: str) -> str:
    with open(path, "wb") as f:
        f.write(checkpoint_bytes(name))
    return path


def prompt_of(name: str) -> np.ndarray:
    c = config_of(name)
    rng = np.random.default_rng(1000 + c["seed"])
    return rng.integers(2, abs(c["vocab"]), size=c["n_prompt"]).astype(np.int32)


TOKENIZER_GOLDEN = os.path.join(HERE, "tokenizer_golden.npz")

# texts the tokenizer goldens cover (utf-8): merges, ties, byte fallback for
# characters without a token (2-, 3- and 4-byte sequences), empty text
TOKENIZER_TEXTS = ["the cat", "Hi!", "caf\u00e9 au lait", "thing and then", "",
                   "\u017e\u20ac\U0001d11e", "  spaces  ", "the the the", "ATHENA"]


def tokenizer_bytes(seed: int = 5) -> tuple[bytes, int]:
    """A llama2.c tokenizer file (the layout Llama2Tokenizer::load reads,
    src/llama2.cpp:414-453): ids 0-2 special, 3-258 the byte pieces
    <0x00>..<0xFF>, then single characters and seeded merge pieces with
    seeded scores, one duplicated piece (the first id must win) and two
    pieces with equal scores (the first position must win)."""
    rng = np.random.default_rng(seed)
    pieces = ["<unk>", "\n<s>\n", "\n</s>\n"] + [f"<0x{b:02X}>" for b in range(256)]
    chars = [" "] + list("abcdefghijklmnopqrstuvwxyz") + list("ATHEN") + list("!.,") + ["\u00e9"]
    merges = ["th", "he", "the", " t", " th", " the", "in", "ing", "an", "and", " a", "ca",
              "caf", "caf\u00e9", "at", " c", " ca", " cat", "en", "then", " l", "la",
              "lait", "ai", "it", "  ", "ATH", "EN", "ENA", "th"]  # "th" twice
    pieces += chars + merges
    scores = [0.0] * 259 + list(rng.uniform(-10, -5, len(chars))) + \
        list(rng.uniform(-5, 0, len(merges)))
    scores[pieces.index("en")] = scores[pieces.index("an")]  # a tie
    out = [np.array([max(len(p.encode()) for p in pieces)], np.uint32).tobytes()]
    for p, sc in zip(pieces, scores):
        b = p.encode()
        out.append(np.array([sc], np.float32).tobytes())
        out.append(np.array([len(b)], np.int32).tobytes())
        out.append(b)
    return b"".join(out), len(pieces)


def write_tokenizer(path: str) -> tuple[str, int]:
    data, vocab = tokenizer_bytes()
    with open(path, "wb") as f:
        f.write(data)
    return path, vocab


def make_tokenizer_goldens(ref) -> None:
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        path, vocab = write_tokenizer(os.path.join(tmp, "tok.bin"))
        out["sha256"] = np.frombuffer(hashlib.sha256(open(path, "rb").read()).digest(), np.uint8)
        out["vocab"] = np.array(vocab)
        for i, text in enumerate(TOKENIZER_TEXTS):
            raw = text.encode("utf-8")
            for bos, eos in ((1, 0), (0, 0), (1, 1)):
                ids = ref.tokenizer_encode(path, vocab, raw, bool(bos), bool(eos))
                out[f"t{i}/ids{bos}{eos}"] = np.array(ids, np.int32)
                back = ref.tokenizer_decode(path, vocab, ids if not eos else ids[:-1])
                out[f"t{i}/text{bos}{eos}"] = np.frombuffer(back, np.uint8)
    np.savez_compressed(TOKENIZER_GOLDEN, **out)
    print("wrote", TOKENIZER_GOLDEN)


def main() -> None:
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle import Reference

    ref = Reference()
    make_tokenizer_goldens(ref)
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        for name in CONFIGS:
            c = config_of(name)
            path = write_checkpoint(os.path.join(tmp, name + ".bin"), name)
            out[f"{name}/sha256"] = np.frombuffer(
                hashlib.sha256(open(path, "rb").read()).digest(), np.uint8)
            prompt = prompt_of(name)
            out[f"{name}/prompt"] = prompt
            for qtype, qname in ((0, "int8"), (1, "int4"), (2, "fp32")):
                cfg, tied, nbytes, digest = ref.llama2c_inspect(path, qtype)
                key = f"{name}/{qname}"
                out[f"{key}/config"] = np.array(cfg, np.int64)
                out[f"{key}/tied"] = np.array(tied)
                out[f"{key}/storage_bytes"] = np.array(nbytes, np.uint64)
                out[f"{key}/digest"] = np.array(digest, np.uint64)
                out[f"{key}/greedy"] = ref.llama2c_generate(path, qtype, prompt,
                                                            c["max_tokens"])
                out[f"{key}/sampled"] = ref.llama2c_generate(path, qtype, prompt,
                                                             c["max_tokens"], **SAMPLING)
                print(key, "greedy", out[f"{key}/greedy"].tolist(), "sampled",
                      out[f"{key}/sampled"].tolist(), "storage", nbytes)
    np.savez_compressed(GOLDEN, **out)
    print("wrote", GOLDEN)


if __name__ == "__main__":
    main()
