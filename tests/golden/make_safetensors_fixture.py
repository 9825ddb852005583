"""Seeded safetensors checkpoints, BPE tokenizer files and their golden
outputs from the reference.

Test infrastructure.  ``safetensors_bytes(name)`` builds a small fp32
Llama-style checkpoint in the layout the reference's load_model reads
(src/loader.cpp:286-498): a little-endian uint64 header length, a JSON
header (``__metadata__`` with the nutllm.* config strings, then one F32
tensor entry per weight with its byte offsets) padded with spaces, then the
tensors.  ``malformed_cases()`` derives damaged files from it (truncations,
JSON the reference rejects, bad tensor entries, bad metadata, missing or
mis-shaped weights); ``bpe_files()`` writes a byte-level BPE vocabulary and
merge list (src/tokenizer.cpp) and ``bpe_malformed()`` damaged variants.
Weights and merges come from numpy's seeded generator, so the tests rebuild
the same bytes on any machine (SHA-256 stored beside the goldens).

Run here, where the reference builds (``make -C oracle ref``), to refresh
``safetensors_golden.npz``:

    python tests/golden/make_safetensors_fixture.py

It records the reference loader's config, storage_bytes() and byte digest,
the ids of generate_tokens and generate_tokens_cached (greedy and seeded
top-p), the (status, message) each malformed file raises, and the BPE
encode/decode results and errors.  The reference library is loaded before
numpy: with numpy's bundled libraries loaded first, the reference's
formatted stream reads (the vocabulary ids) misparse in this process.
"""
from __future__ import annotations

import ctypes
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
if __name__ == "__main__":
    # load the reference and run one tokenizer read before numpy is imported
    _ref_so = os.path.join(ROOT, "oracle", "_ref", "libnutref.so")
    if os.path.exists(_ref_so):
        import tempfile as _tf
        _lib = ctypes.CDLL(_ref_so)
        with _tf.TemporaryDirectory() as _d:
            _v, _m = os.path.join(_d, "v"), os.path.join(_d, "m")
            open(_v, "w").write("0 61\n")
            open(_m, "w").write("")
            _ids, _n = (ctypes.c_int * 4)(), ctypes.c_size_t(0)
            _lib.ref_bpe_encode.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p,
                                            ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
                                            ctypes.c_void_p]
            assert _lib.ref_bpe_encode(_v.encode(), _m.encode(), b"a", 1, _ids, 4,
                                       ctypes.byref(_n)) == 0

import hashlib  # noqa: E402
import json  # noqa: E402
import struct  # noqa: E402
import tempfile  # noqa: E402

import numpy as np  # noqa: E402

GOLDEN = os.path.join(HERE, "safetensors_golden.npz")

# name: (layers, heads, dim, ffn, vocab, max_seq, eos, seed, prompt length,
# max_tokens, projection gain)
CONFIGS = {
    "mha_small": (2, 4, 64, 176, 120, 40, 3, 21, 5, 12, 1.5),
    # generation runs into the context limit
    "odd_context": (1, 3, 24, 40, 50, 16, 5, 22, 4, 20, 3.0),
}
SAMPLING = dict(temperature=0.8, top_p=0.9, seed=42)


def config_of(name: str) -> dict:
    layers, heads, dim, ffn, vocab, max_seq, eos, seed, n_prompt, max_tokens, gain = \
        CONFIGS[name]
    return dict(layers=layers, heads=heads, dim=dim, head_dim=dim // heads, ffn=ffn,
                vocab=vocab, max_seq=max_seq, eos=eos, seed=seed, n_prompt=n_prompt,
                max_tokens=max_tokens, gain=gain)


def tensors_of(name: str) -> dict:
    """name -> float32 array, [out][in] projections (HF naming)."""
    c = config_of(name)
    rng = np.random.default_rng(c["seed"])
    dim, ffn = c["dim"], c["ffn"]

    def mat(rows, cols):
        return (c["gain"] * rng.standard_normal((rows, cols)) / np.sqrt(cols)).astype(
            np.float32)

    def gains():
        return (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)

    t = {"model.embed_tokens.weight": rng.standard_normal((c["vocab"], dim)).astype(
        np.float32)}
    for l in range(c["layers"]):
        p = f"model.layers.{l}"
        t[f"{p}.self_attn.q_proj.weight"] = mat(dim, dim)
        t[f"{p}.self_attn.k_proj.weight"] = mat(dim, dim)
        t[f"{p}.self_attn.v_proj.weight"] = mat(dim, dim)
        t[f"{p}.self_attn.o_proj.weight"] = mat(dim, dim)
        t[f"{p}.mlp.gate_proj.weight"] = mat(ffn, dim)
        t[f"{p}.mlp.up_proj.weight"] = mat(ffn, dim)
        t[f"{p}.mlp.down_proj.weight"] = mat(dim, ffn)
        t[f"{p}.input_layernorm.weight"] = gains()
        t[f"{p}.post_attention_layernorm.weight"] = gains()
    t["model.norm.weight"] = gains()
    t["lm_head.weight"] = (rng.standard_normal((c["vocab"], dim)) / np.sqrt(dim)).astype(
        np.float32)
    return t


def metadata_of(name: str) -> dict:
    c = config_of(name)
    return {f"nutllm.{k}": str(v) for k, v in (
        ("layers", c["layers"]), ("heads", c["heads"]), ("dim", c["dim"]),
        ("head_dim", c["head_dim"]), ("ffn_dim", c["ffn"]), ("vocab_size", c["vocab"]),
        ("max_seq", c["max_seq"]), ("eos_token", c["eos"]))}


def pack(header: dict, payload: bytes, pad: int = 8) -> bytes:
    h = json.dumps(header).encode()
    h += b" " * ((-len(h)) % pad)
    return struct.pack("<Q", len(h)) + h + payload


def layout(tensors: dict, metadata: dict | None):
    header = {} if metadata is None else {"__metadata__": metadata}
    chunks, at = [], 0
    for k, a in tensors.items():
        b = np.ascontiguousarray(a, np.float32).tobytes()
        header[k] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [at, at + len(b)]}
        chunks.append(b)
        at += len(b)
    return header, b"".join(chunks)


def safetensors_bytes(name: str) -> bytes:
    header, payload = layout(tensors_of(name), metadata_of(name))
    return pack(header, payload)


def prompt_of(name: str) -> np.ndarray:
    c = config_of(name)
    rng = np.random.default_rng(500 + c["seed"])
    return rng.integers(0, c["vocab"], size=c["n_prompt"]).astype(np.int32)


def malformed_cases() -> dict:
    """label -> file bytes; every one is rejected by load_model."""
    name = "odd_context"
    t, md = tensors_of(name), metadata_of(name)
    good = safetensors_bytes(name)
    header, payload = layout(t, md)
    out = {
        "empty": b"",
        "short_prefix": good[:5],
        "truncated_12": good[:12],
        "zero_header": struct.pack("<Q", 0) + b"{}",
        "header_past_end": struct.pack("<Q", 1 << 40) + b"{}",
    }

    def raw(text: str) -> bytes:
        h = text.encode()
        return struct.pack("<Q", len(h)) + h + payload

    out.update({
        "json_trailing": raw('{"a": 1} x'),
        "json_true": raw('{"a": true}'),
        "json_negative": raw('{"a": -1}'),
        "json_escape_u": raw('{"a\\u0041": 1}'),
        "json_duplicate": raw('{"a": 1, "a": 2}'),
        "json_control": raw('{"a\tb": 1}'),
        "json_unterminated": raw('{"abc'),
        "json_bad_delim": raw('{"a": 1; "b": 2}'),
        "json_no_colon": raw('{"a" 1}'),
        "json_key": raw('{1: 2}'),
        "json_array_delim": raw('{"a": [1 2]}'),
        "json_overflow": raw('{"a": 99999999999999999999999}'),
        "json_missing": raw('{"a": }'),
        "root_array": raw('[1, 2]'),
        "metadata_not_object": raw('{"__metadata__": [1]}'),
        "metadata_number": raw('{"__metadata__": {"a": 1}}'),
        "no_tensors": raw('{"__metadata__": {"a": "1"}}'),
    })

    def edit(key, field, value):
        h = json.loads(json.dumps(header))
        if value is None:
            del h[key][field]
        else:
            h[key][field] = value
        return pack(h, payload)

    first = "model.embed_tokens.weight"
    n = t[first].nbytes
    out.update({
        "tensor_not_object": pack({**header, first: [1]}, payload),
        "dtype_f16": edit(first, "dtype", "F16"),
        "dtype_missing": edit(first, "dtype", None),
        "shape_string": edit(first, "shape", ["50", 24]),
        "shape_scalar": edit(first, "shape", []),
        "shape_zero": edit(first, "shape", [0, 24]),
        "offsets_one": edit(first, "data_offsets", [0]),
        "offsets_string": edit(first, "data_offsets", ["0", n]),
        "extent_short": edit(first, "data_offsets", [0, n - 4]),
        "extent_past_end": edit(first, "data_offsets", [len(payload), len(payload) + n]),
        "misaligned": edit(first, "data_offsets", [2, n + 2]),
    })

    def with_md(**changes):
        m = dict(md)
        for k, v in changes.items():
            if v is None:
                m.pop(f"nutllm.{k}")
            else:
                m[f"nutllm.{k}"] = v
        h, p = layout(t, m)
        return pack(h, p)

    out.update({
        "md_missing_layers": with_md(layers=None),
        "md_empty_dim": with_md(dim=""),
        "md_invalid_heads": with_md(heads="3x"),
        "md_overflow": with_md(max_seq="99999999999999999999999"),
        "md_bad_config": with_md(head_dim="9"),
        "md_eos_outside": with_md(eos_token="50"),
    })

    def with_tensors(drop=None, reshape=None):
        tt = dict(t)
        if drop:
            tt.pop(drop)
        if reshape:
            k, shape = reshape
            tt[k] = np.zeros(shape, np.float32)
        h, p = layout(tt, md)
        return pack(h, p)

    out.update({
        "missing_q": with_tensors(drop="model.layers.0.self_attn.q_proj.weight"),
        "missing_lm_head": with_tensors(drop="lm_head.weight"),
        "wrong_gate": with_tensors(reshape=("model.layers.0.mlp.gate_proj.weight", (24, 40))),
        "wrong_norm": with_tensors(reshape=("model.norm.weight", (25,))),
        "wrong_embed": with_tensors(reshape=("model.embed_tokens.weight", (24, 50))),
    })
    return out


# --------------------------------------------------------------- BPE files

BPE_TEXTS = [b"the theme then", b"aaaa", b"", b"\x00\xff\n\t", b"banana bandana",
             b"hello, world!"]


def bpe_files(seed: int = 9) -> tuple[str, str]:
    """(vocabulary text, merges text): the 256 single bytes in a seeded order,
    then merges built by joining seeded adjacent pairs of a corpus."""
    rng = np.random.default_rng(seed)
    order = rng.permutation(256)
    vocab = [bytes([int(b)]) for b in order]
    corpus = b" ".join(BPE_TEXTS) * 2
    merges = []
    known = set(vocab)
    for _ in range(24):
        i = int(rng.integers(0, len(corpus) - 3))
        left = corpus[i:i + 1 + int(rng.integers(0, 2))]
        right = corpus[i + len(left):i + len(left) + 1]
        if not right or (left, right) in merges:
            continue
        for piece in (left, right):
            if piece not in known:
                known.add(piece)
                vocab.append(piece)
        if left + right not in known:
            known.add(left + right)
            vocab.append(left + right)
        merges.append((left, right))
    vtext = "".join(f"{i} {p.hex()}\n" for i, p in enumerate(vocab))
    mtext = "".join(f"{a.hex()} {b.hex()}\n" + ("\n" if k == 3 else "")
                    for k, (a, b) in enumerate(merges))
    return vtext, mtext


def bpe_malformed() -> dict:
    """label -> (vocabulary text, merges text), each rejected by load."""
    v, m = bpe_files()
    lines = v.splitlines(keepends=True)
    mlines = m.splitlines(keepends=True)
    first_merge = mlines[0].split()
    return {
        "gap_in_ids": (lines[0] + "".join(lines[2:]), m),
        "odd_hex": (lines[0].replace(lines[0].split()[1], "abc", 1) + "".join(lines[1:]), m),
        "bad_hex_digit": ("0 zz\n" + "".join(lines[1:]), m),
        "missing_token": ("0\n" + "".join(lines[1:]), m),
        "negative_id": ("-1 " + lines[0].split()[1] + "\n" + "".join(lines[1:]), m),
        "duplicate_token": (v + f"{len(lines)} {lines[0].split()[1]}\n", m),
        "empty_vocab": ("", m),
        "merge_three_words": (v, mlines[0].rstrip("\n") + " 61\n" + "".join(mlines[1:])),
        "merge_one_word": (v, first_merge[0] + "\n" + m),
        "merge_duplicate": (v, m + mlines[0]),
        "merge_not_in_vocab": (v, m + "00 00\n"),
        "merge_bad_hex": (v, m + "0g 61\n"),
    }


def sha(b: bytes) -> np.ndarray:
    return np.frombuffer(hashlib.sha256(b).digest(), np.uint8)


def main() -> None:
    sys.path.insert(0, ROOT)
    from oracle import RefError, Reference

    ref = Reference()
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        for name in CONFIGS:
            c = config_of(name)
            data = safetensors_bytes(name)
            path = os.path.join(tmp, name + ".safetensors")
            open(path, "wb").write(data)
            out[f"{name}/sha256"] = sha(data)
            cfg, nbytes, digest = ref.safetensors_inspect(path)
            out[f"{name}/config"] = np.array(cfg, np.int64)
            out[f"{name}/storage_bytes"] = np.array(nbytes, np.uint64)
            out[f"{name}/digest"] = np.array(digest, np.uint64)
            prompt = prompt_of(name)
            out[f"{name}/prompt"] = prompt
            for cached in (0, 1):
                g = ref.safetensors_generate(path, prompt, c["max_tokens"], cached=bool(cached))
                s = ref.safetensors_generate(path, prompt, c["max_tokens"], cached=bool(cached),
                                             **SAMPLING)
                out[f"{name}/greedy{cached}"] = g
                out[f"{name}/sampled{cached}"] = s
                print(name, "cached" if cached else "uncached", g.tolist(), s.tolist())
        for label, data in malformed_cases().items():
            path = os.path.join(tmp, "bad.safetensors")
            open(path, "wb").write(data)
            out[f"bad/{label}/sha256"] = sha(data)
            try:
                ref.safetensors_inspect(path)
                raise SystemExit(f"{label}: the reference accepted it")
            except RefError as e:
                out[f"bad/{label}/status"] = np.array(e.status)
                out[f"bad/{label}/message"] = np.frombuffer(e.message.encode(), np.uint8)
                print(label, e.status, e.message)
        vtext, mtext = bpe_files()
        vp, mp = os.path.join(tmp, "v.txt"), os.path.join(tmp, "m.txt")
        open(vp, "w").write(vtext)
        open(mp, "w").write(mtext)
        out["bpe/sha256"] = sha((vtext + "\0" + mtext).encode())
        for i, text in enumerate(BPE_TEXTS):
            ids = ref.bpe_encode(vp, mp, text)
            out[f"bpe/t{i}/ids"] = ids
            assert ref.bpe_decode(vp, mp, ids) == text
            print("bpe", text, ids.tolist())
        for label, (vt, mt) in bpe_malformed().items():
            open(vp, "w").write(vt)
            open(mp, "w").write(mt)
            try:
                ref.bpe_encode(vp, mp, b"a")
                raise SystemExit(f"bpe {label}: the reference accepted it")
            except RefError as e:
                out[f"bpebad/{label}/status"] = np.array(e.status)
                out[f"bpebad/{label}/message"] = np.frombuffer(e.message.encode(), np.uint8)
                print("bpe", label, e.status, e.message)
    np.savez_compressed(GOLDEN, **out)
    print("wrote", GOLDEN)


if __name__ == "__main__":
    main()
