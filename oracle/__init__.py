"""Test infrastructure only: CPU checkers for the nutllm token loop.

* ``Oracle``    — ctypes binding of ``_build/liboracle.so``, the plain-C
  restatement of the reference algorithm (nut_oracle.c).
* ``Reference`` — ctypes binding of ``_ref/libnutref.so``, the unmodified
  reference sources compiled by this directory's Makefile (present only
  where the reference was available at build time).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline and
reference legs may import this package, and only as the checker or the
timed CPU baseline — never as the product path.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "_build", "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libnutref.so")

_P = C.c_void_p
_I64 = C.c_int64


def _ptr(a):
    return None if a is None else a.ctypes.data


def reference_dir() -> Optional[str]:
    """Where the reference's sources lie, if anywhere: $NUTLLM_REFERENCE, else
    the "reference_path" of the repository's BASELINE.json; None when
    neither names an existing directory (e.g. on a GPU box)."""
    import json
    path = os.environ.get("NUTLLM_REFERENCE")
    if not path:
        try:
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                path = json.load(f).get("reference_path")
        except (OSError, ValueError):
            path = None
    return path if path and os.path.isdir(path) else None


def build_oracle() -> str:
    """Builds liboracle.so with gcc if it is missing (it is plain C)."""
    if not os.path.exists(ORACLE_LIB):
        subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    return ORACLE_LIB


# ---------------------------------------------------------------- oracle


class _Config(C.Structure):
    _fields_ = [(n, C.c_int64) for n in (
        "layers", "heads", "dim", "head_dim", "ffn_dim", "vocab_size",
        "max_seq", "eos_token", "kv_heads")]


class _QM(C.Structure):
    _fields_ = [("data", _P), ("scales", _P), ("rows", _I64), ("cols", _I64)]


class _Layer(C.Structure):
    _fields_ = [(n, _QM) for n in ("q", "k", "v", "o", "gate", "up", "down")] + [
        ("attention_norm", _P), ("ffn_norm", _P)]


class _Model(C.Structure):
    _fields_ = [("config", _Config), ("type", C.c_int), ("embeddings", _P),
                ("final_norm", _P), ("lm_head", _P), ("layers", C.POINTER(_Layer))]


class _KV(C.Structure):
    _fields_ = [("keys", _P), ("values", _P), ("length", _I64)]


class Oracle:
    def __init__(self):
        lib = C.CDLL(build_oracle())
        lib.orc_last_error.restype = C.c_char_p
        lib.orc_half_from_float.argtypes = [C.c_float, C.POINTER(C.c_int)]
        lib.orc_half_from_float.restype = C.c_uint16
        lib.orc_half_to_float.argtypes = [C.c_uint16]
        lib.orc_half_to_float.restype = C.c_float
        lib.orc_quantize.argtypes = [_P, _I64, _I64, C.c_int, _P, _P]
        lib.orc_qmatvec.argtypes = [C.c_int, _I64, _I64, _P, _P, _P, _P]
        lib.orc_set_threads.argtypes = [C.c_int]
        lib.orc_set_threads.restype = None
        lib.orc_rmsnorm.argtypes = [_P, _P, _P, _I64, C.c_float]
        lib.orc_rmsnorm.restype = None
        lib.orc_uniform_floats.argtypes = [C.c_uint32, C.c_float, C.c_float, _I64, _P]
        lib.orc_uniform_floats.restype = None
        lib.orc_rope.argtypes = [_P, _I64, _I64]
        lib.orc_rope.restype = None
        lib.orc_matvec_f32.argtypes = [_P, _I64, _I64, _P, _P]
        lib.orc_matvec_f32.restype = None
        lib.orc_matmul_f32.argtypes = [_P, _P, _I64, _I64, _I64, _P]
        lib.orc_matmul_f32.restype = None
        lib.orc_argmax.argtypes = [_P, _I64]
        lib.orc_argmax.restype = _I64
        lib.orc_decode_token.argtypes = [C.POINTER(_Model), C.POINTER(_KV),
                                         C.c_int, _P]
        lib.orc_logits.argtypes = [C.POINTER(_Model), _P, _P, C.POINTER(_I64)]
        lib.orc_generate.argtypes = [C.POINTER(_Model), C.POINTER(_KV), _P,
                                     _I64, _I64, _P, _P, _P]
        lib.orc_choose_tokens.argtypes = [_P, _I64, _I64, C.c_float, C.c_float,
                                          C.c_uint32, _P]
        lib.orc_generate_sampled.argtypes = [C.POINTER(_Model), C.POINTER(_KV), _P,
                                             _I64, _I64, C.c_float, C.c_float,
                                             C.c_uint32, _P, C.POINTER(_I64)]
        lib.orc_synth_normal.argtypes = [C.c_uint64, C.c_uint64, C.c_float, _P, _I64]
        lib.orc_synth_normal.restype = None
        lib.orc_synth_tokens.argtypes = [C.c_uint64, C.c_uint64, C.c_int, C.c_int, _P, _I64]
        lib.orc_synth_tokens.restype = None
        self.lib = lib

    def _check(self, status):
        if status != 0:
            raise RuntimeError(f"oracle status {status}: "
                               f"{self.lib.orc_last_error().decode()}")

    def set_threads(self, n: int) -> None:
        self.lib.orc_set_threads(n)

    def half_from_float(self, v: float) -> int:
        st = C.c_int(0)
        h = self.lib.orc_half_from_float(v, C.byref(st))
        self._check(st.value)
        return h

    def half_to_float(self, h: int) -> float:
        return self.lib.orc_half_to_float(h)

    def quantize(self, w: np.ndarray, qtype: int):
        w = np.ascontiguousarray(w, np.float32)
        rows, cols = w.shape
        n = rows * cols
        data = np.zeros(n if qtype == 0 else (n + 1) // 2, np.uint8)
        scales = np.zeros((n + 31) // 32, np.uint16)
        self._check(self.lib.orc_quantize(_ptr(w), rows, cols, qtype,
                                          _ptr(data), _ptr(scales)))
        return data, scales

    def qmatvec(self, qtype, rows, cols, data, scales, x):
        y = np.empty(rows, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        self._check(self.lib.orc_qmatvec(qtype, rows, cols, _ptr(data),
                                         _ptr(scales), _ptr(x), _ptr(y)))
        return y

    def rmsnorm(self, x, w, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.empty_like(x)
        self.lib.orc_rmsnorm(_ptr(x), _ptr(w), _ptr(out), x.size, eps)
        return out

    def matmul_f32(self, a, b):
        """matmul_threaded: a [m][k] @ b [k][n], the reference's fused order."""
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        c = np.empty((a.shape[0], b.shape[1]), np.float32)
        self.lib.orc_matmul_f32(_ptr(a), _ptr(b), a.shape[0], a.shape[1], b.shape[1], _ptr(c))
        return c

    def matvec_f32(self, w, x):
        w = np.ascontiguousarray(w, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(w.shape[0], np.float32)
        self.lib.orc_matvec_f32(_ptr(w), w.shape[0], w.shape[1], _ptr(x), _ptr(y))
        return y

    def choose_tokens(self, logits: np.ndarray, temperature: float, top_p: float,
                      seed: int) -> np.ndarray:
        """choose_token over rows of logits with one seeded mt19937
        (src/generate.cpp:25-73)."""
        lg = np.ascontiguousarray(np.atleast_2d(logits), np.float32)
        out = np.zeros(lg.shape[0], np.int64)
        self._check(self.lib.orc_choose_tokens(_ptr(lg), lg.shape[0], lg.shape[1],
                                               temperature, top_p, seed, _ptr(out)))
        return out

    def uniform_floats(self, seed: int, lo: float, hi: float, shape) -> np.ndarray:
        """std::uniform_real_distribution<float>(lo, hi) over
        std::mt19937(seed), row-major into `shape`."""
        out = np.empty(shape, np.float32)
        self.lib.orc_uniform_floats(seed, lo, hi, out.size, _ptr(out))
        return out

    def rope(self, values: np.ndarray, position: int) -> np.ndarray:
        """rotate_vector of one head (src/kvcache.cpp:48-59), in place."""
        assert values.dtype == np.float32 and values.flags.c_contiguous
        self.lib.orc_rope(_ptr(values), values.size, position)
        return values

    def synth_normal(self, seed: int, stream: int, n: int, sigma: float) -> np.ndarray:
        """The benchmark's seeded N(0, sigma^2) stream (orc_synth_normal)."""
        out = np.empty(n, np.float32)
        self.lib.orc_synth_normal(seed, stream, sigma, _ptr(out), n)
        return out

    def synth_tokens(self, seed: int, stream: int, n: int, lo: int, hi: int) -> np.ndarray:
        out = np.empty(n, np.int32)
        self.lib.orc_synth_tokens(seed, stream, lo, hi, _ptr(out), n)
        return out

    def model(self, weights) -> "OracleModel":
        return OracleModel(self, weights)

    def fp32_model(self, tensors: dict) -> "Fp32Model":
        return Fp32Model(self, tensors)


# ------------------------------------------------- seeded workload tensors
#
# The benchmark's synthetic tensors drawn by the oracle's own restatement of
# the generator, so the reference's CPU baseline loads no library of this
# repository: embeddings stream 1, classifier stream 2, prompt ids token
# stream 3, projection j of layer l stream 1000 + 8 l + j, N(0, 0.02).

SIGMA = 0.02
_shared_oracle = None


def _orc() -> "Oracle":
    global _shared_oracle
    if _shared_oracle is None:
        _shared_oracle = Oracle()
    return _shared_oracle


def projection_shapes(c):
    kv = int(c.kv_heads or c.heads) * int(c.head_dim)
    d, f = int(c.dim), int(c.ffn_dim)
    return [(d, d), (kv, d), (kv, d), (d, d), (f, d), (f, d), (d, f)]


def embeddings_fp32(c, seed: int) -> np.ndarray:
    V, d = int(c.vocab_size), int(c.dim)
    return _orc().synth_normal(seed, 1, V * d, SIGMA).reshape(V, d)


def lm_head_fp32(c, seed: int) -> np.ndarray:
    V, d = int(c.vocab_size), int(c.dim)
    return _orc().synth_normal(seed, 2, V * d, SIGMA).reshape(V, d)


def projection_fp32(c, seed: int, layer: int, j: int) -> np.ndarray:
    rows, cols = projection_shapes(c)[j]
    return _orc().synth_normal(seed, 1000 + 8 * layer + j, rows * cols,
                               SIGMA).reshape(rows, cols)


def prompt_ids(c, seed: int, n: int, stream: int = 3) -> np.ndarray:
    return _orc().synth_tokens(seed, stream, n, 1, int(c.vocab_size) - 1)


class OracleModel:
    """Oracle view of an nutllm_b200.ModelWeights host image (same bytes)."""

    def __init__(self, oracle: Oracle, w):
        self.o = oracle
        self.w = w
        c = w.config
        self.config = c
        layers = (_Layer * int(c.layers))()
        for i, lw in enumerate(w.layers):
            for name, m in zip(("q", "k", "v", "o", "gate", "up", "down"),
                               lw.projections()):
                setattr(layers[i], name, _QM(m.data.ctypes.data,
                                             m.scales.ctypes.data, m.rows, m.cols))
            layers[i].attention_norm = lw.attention_norm.ctypes.data
            layers[i].ffn_norm = lw.ffn_norm.ctypes.data
        self._layers = layers
        m = _Model()
        m.config = _Config(*[int(getattr(c, n)) for n, _ in _Config._fields_])
        m.config.kv_heads = c.kv_heads or c.heads
        m.type = w.qtype
        m.embeddings = w.embeddings.ctypes.data
        m.final_norm = w.final_norm.ctypes.data
        m.lm_head = w.output_weights().ctypes.data
        m.layers = C.cast(layers, C.POINTER(_Layer))
        self._model = m
        kvh = c.kv_heads or c.heads
        n = int(c.layers * kvh * c.max_seq * c.head_dim)
        self.keys = np.zeros(n, np.float32)
        self.values = np.zeros(n, np.float32)
        self.kv = _KV(self.keys.ctypes.data, self.values.ctypes.data, 0)

    def reset(self):
        self.kv.length = 0

    def decode(self, token: int) -> np.ndarray:
        h = np.empty(self.config.dim, np.float32)
        self.o._check(self.o.lib.orc_decode_token(C.byref(self._model),
                                                  C.byref(self.kv), token, _ptr(h)))
        return h

    def logits(self, hidden: np.ndarray):
        out = np.empty(self.config.vocab_size, np.float32)
        best = _I64(0)
        self.o._check(self.o.lib.orc_logits(C.byref(self._model), _ptr(hidden),
                                            _ptr(out), C.byref(best)))
        return out, best.value

    def generate(self, prompt: Sequence[int], steps: int):
        """prefill + `steps` greedy tokens; returns (ids, logits, prefill hidden)."""
        p = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(max(steps, 1), np.int32)
        lg = np.empty((max(steps, 1), self.config.vocab_size), np.float32)
        hid = np.empty(self.config.dim, np.float32)
        self.o._check(self.o.lib.orc_generate(C.byref(self._model), C.byref(self.kv),
                                              _ptr(p), p.size, steps, _ptr(ids),
                                              _ptr(lg), _ptr(hid)))
        return ids[:steps], lg[:steps], hid

    def generate_cached(self, prompt: Sequence[int], max_tokens: int,
                        temperature: float = 0.0, top_p: float = 1.0,
                        seed: int = 1) -> np.ndarray:
        """generate_tokens_cached (src/generate.cpp:174-216): eos stop and
        context limit, greedy or top-p sampled."""
        p = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(max(max_tokens, 1), np.int32)
        n = _I64(0)
        self.o._check(self.o.lib.orc_generate_sampled(
            C.byref(self._model), C.byref(self.kv), _ptr(p), p.size, max_tokens,
            temperature, top_p, seed, _ptr(ids), C.byref(n)))
        return ids[:n.value]


class Fp32Model:
    """The fp32-weight decoder (ModelWeights) of a llama2.c checkpoint,
    restated from decode_token / decoder_layer_step / attention_step
    (src/kvcache.cpp:35-171,265-284) and generate_tokens_cached
    (src/generate.cpp:128-172) over read_llama2c's tensors.

    Projections follow linear_threaded (src/threading.cpp:200-214: for an
    [in][out] matrix, each output is an in-order chain of multiply-adds),
    which is matmul_threaded of one row, so they run through orc_matmul_f32
    on the transposed ([in][out]) matrices; the classifier follows
    matvec_threaded.  Attention keeps the reference's double dot products and
    weighted sums.  The prompt runs one position at a time (the reference's
    prefill_tokens computes the same rows as whole-matrix products, equal up
    to rounding order); ids are pinned against the reference's goldens."""

    def __init__(self, oracle: Oracle, t: dict):
        self.o = oracle
        c = t["config"]
        self.c = c
        self.kvh = c["kv_heads"] or c["heads"]
        T = lambda a: np.ascontiguousarray(np.swapaxes(a, -1, -2))  # noqa: E731
        self.wq, self.wk, self.wv, self.wo = T(t["wq"]), T(t["wk"]), T(t["wv"]), T(t["wo"])
        self.gate, self.down, self.up = T(t["w1"]), T(t["w2"]), T(t["w3"])
        self.att_norm, self.ffn_norm = t["attention_norm"], t["ffn_norm"]
        self.emb = np.ascontiguousarray(t["embeddings"])
        self.final_norm = np.ascontiguousarray(t["final_norm"])
        self.cls = self.emb if t["tied"] else np.ascontiguousarray(t["classifier"])
        hd, S = c["head_dim"], c["max_seq"]
        self.keys = np.zeros((c["layers"], self.kvh, S, hd), np.float32)
        self.values = np.zeros_like(self.keys)
        self.length = 0

    def _linear(self, x, w):
        return self.o.matmul_f32(x[None, :], w)[0]

    def decode(self, token: int) -> np.ndarray:
        c, o = self.c, self.o
        if not 0 <= token < c["vocab_size"]:
            raise IndexError("kv cache: token id out of range")
        if self.length >= c["max_seq"]:
            raise OverflowError("kv cache: context is full")
        pos, hd, H = self.length, c["head_dim"], c["heads"]
        h = self.emb[token].copy()
        scale = np.float32(1.0) / np.sqrt(np.float32(hd))
        group = H // self.kvh
        for l in range(c["layers"]):
            x = o.rmsnorm(h, self.att_norm[l])
            q = self._linear(x, self.wq[l])
            k = self._linear(x, self.wk[l])
            v = self._linear(x, self.wv[l])
            for hh in range(H):
                seg = np.ascontiguousarray(q[hh * hd:(hh + 1) * hd])
                q[hh * hd:(hh + 1) * hd] = o.rope(seg, pos)
            for hh in range(self.kvh):
                seg = np.ascontiguousarray(k[hh * hd:(hh + 1) * hd])
                self.keys[l, hh, pos] = o.rope(seg, pos)
                self.values[l, hh, pos] = v[hh * hd:(hh + 1) * hd]
            ctx = np.zeros(c["dim"], np.float32)
            for hh in range(H):
                K = self.keys[l, hh // group, :pos + 1].astype(np.float64)
                V = self.values[l, hh // group, :pos + 1].astype(np.float64)
                qh = q[hh * hd:(hh + 1) * hd].astype(np.float64)
                sc = (K @ qh).astype(np.float32) * scale
                e = np.exp(sc - sc.max()).astype(np.float32)
                total = np.float32(e.astype(np.float64).sum())
                wts = (e / total).astype(np.float64)
                ctx[hh * hd:(hh + 1) * hd] = (wts @ V).astype(np.float32)
            h = (h + self._linear(ctx, self.wo[l])).astype(np.float32)
            x = o.rmsnorm(h, self.ffn_norm[l])
            g = self._linear(x, self.gate[l])
            u = self._linear(x, self.up[l])
            act = (g / (np.float32(1) + np.exp(-g)) * u).astype(np.float32)
            h = (h + self._linear(act, self.down[l])).astype(np.float32)
        self.length += 1
        return h

    def logits(self, hidden: np.ndarray) -> np.ndarray:
        return self.o.matvec_f32(self.cls, self.o.rmsnorm(hidden, self.final_norm))

    def generate_cached(self, prompt, max_tokens: int, temperature: float = 0.0,
                        top_p: float = 1.0, seed: int = 1):
        """(ids, logits per step): eos stop (token 1) and context limit; a
        sampled run replays one seeded generator over the rows so far."""
        c = self.c
        if len(prompt) == 0 or len(prompt) > c["max_seq"]:
            raise ValueError("generation: invalid prompt length")
        self.length = 0
        for t in prompt:
            h = self.decode(int(t))
        ids, rows = [], []
        while len(ids) < max_tokens and self.length < c["max_seq"]:
            rows.append(self.logits(h))
            if temperature <= 0:
                tok = int(np.argmax(rows[-1]))
            else:
                tok = int(self.o.choose_tokens(np.stack(rows), temperature, top_p, seed)[-1])
            if tok == c["eos_token"]:
                break
            ids.append(tok)
            h = self.decode(tok)
        return np.array(ids, np.int32), rows


# ------------------------------------------------------------- reference


class RefError(RuntimeError):
    """A reference call that threw: status 1 invalid_argument, 2
    out_of_range, 3 length_error, 4 other runtime errors, 5 range_error."""

    def __init__(self, status: int, message: str):
        super().__init__(f"reference status {status}: {message}")
        self.status = status
        self.message = message


def reference_available() -> bool:
    return os.path.exists(REF_LIB)


class Reference:
    """The unmodified reference (oracle/_ref/libnutref.so)."""

    def __init__(self):
        if not reference_available():
            raise RuntimeError("reference build missing: make -C oracle ref")
        lib = C.CDLL(REF_LIB)
        lib.ref_last_error.restype = C.c_char_p
        S = C.c_size_t
        lib.ref_quantize.argtypes = [_P, S, S, C.c_int, _P, S, _P, S]
        lib.ref_qmatrix_info.argtypes = [_P, S, S, C.c_int, C.POINTER(S), _P, _P]
        lib.ref_qmatvec.argtypes = [C.c_int, S, S, _P, _P, _P, _P, S]
        lib.ref_qmatvec_time.argtypes = [C.c_int, S, S, _P, _P, _P, _P, S, S,
                                         C.POINTER(C.c_double)]
        lib.ref_rmsnorm.argtypes = [_P, _P, _P, S, C.c_float]
        lib.ref_matvec_threaded.argtypes = [_P, S, S, _P, _P, S]
        lib.ref_matvec_time.argtypes = [_P, S, S, _P, _P, S, S, C.POINTER(C.c_double)]
        lib.ref_matmul_threaded.argtypes = [_P, _P, _P, S, S, S, S, S,
                                            C.POINTER(C.c_double)]
        lib.ref_model_new.argtypes = [C.POINTER(_I64), C.c_int, C.c_int, C.POINTER(_P)]
        lib.ref_model_free.argtypes = [_P]
        lib.ref_model_free.restype = None
        lib.ref_model_set_embeddings.argtypes = [_P, _P]
        lib.ref_model_set_final.argtypes = [_P, _P, _P]
        lib.ref_model_add_layer.argtypes = [_P, C.POINTER(_P), _P, _P]
        lib.ref_model_storage_bytes.argtypes = [_P, C.POINTER(S)]
        lib.ref_model_layer_bytes.argtypes = [_P, S, C.c_int, _P, S, _P, S]
        lib.ref_generate.argtypes = [_P, _P, S, S, S, _P, _P, _P,
                                     C.POINTER(C.c_double), C.POINTER(C.c_double)]
        lib.ref_trace.argtypes = [_P, _P, S, S, S, _P]
        lib.ref_llama2c_generate.argtypes = [C.c_char_p, C.c_int, _P, S, S, C.c_float,
                                             C.c_float, C.c_uint, _P, C.POINTER(S)]
        lib.ref_llama2c_inspect.argtypes = [C.c_char_p, C.c_int, C.POINTER(_I64),
                                            C.POINTER(C.c_int), C.POINTER(C.c_uint64),
                                            C.POINTER(C.c_uint64)]
        lib.ref_llama2c_encode.argtypes = [C.c_char_p, S, C.c_char_p, C.c_int, _P, S,
                                           C.POINTER(S)]
        lib.ref_llama2c_encode2.argtypes = [C.c_char_p, S, C.c_char_p, S, C.c_int, C.c_int,
                                            _P, S, C.POINTER(S)]
        lib.ref_llama2c_decode.argtypes = [C.c_char_p, S, _P, S, C.c_char_p, S,
                                           C.POINTER(S)]
        lib.ref_safetensors_inspect.argtypes = [C.c_char_p, C.POINTER(_I64),
                                                C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]
        lib.ref_safetensors_generate.argtypes = [C.c_char_p, _P, S, S, C.c_float, C.c_float,
                                                 C.c_uint, C.c_int, _P, C.POINTER(S)]
        lib.ref_bpe_encode.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p, S, _P, S,
                                       C.POINTER(S)]
        lib.ref_bpe_decode.argtypes = [C.c_char_p, C.c_char_p, _P, S, C.c_char_p, S,
                                       C.POINTER(S)]
        self.lib = lib

    def _check(self, status):
        if status != 0:
            raise RefError(status, self.lib.ref_last_error().decode())

    def quantize(self, w: np.ndarray, qtype: int):
        w = np.ascontiguousarray(w, np.float32)
        rows, cols = w.shape
        n = rows * cols
        data = np.zeros(n if qtype == 0 else (n + 1) // 2, np.uint8)
        scales = np.zeros((n + 31) // 32, np.uint16)
        self._check(self.lib.ref_quantize(_ptr(w), rows, cols, qtype, _ptr(data),
                                          data.size, _ptr(scales), scales.size))
        return data, scales

    def quantized_values(self, w: np.ndarray, qtype: int):
        w = np.ascontiguousarray(w, np.float32)
        rows, cols = w.shape
        values = np.empty_like(w)
        bounds = np.empty_like(w)
        nbytes = C.c_size_t(0)
        self._check(self.lib.ref_qmatrix_info(_ptr(w), rows, cols, qtype,
                                              C.byref(nbytes), _ptr(values),
                                              _ptr(bounds)))
        return values, bounds, nbytes.value

    def qmatvec(self, qtype, rows, cols, data, scales, x, threads=1):
        y = np.empty(rows, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        self._check(self.lib.ref_qmatvec(qtype, rows, cols, _ptr(data), _ptr(scales),
                                         _ptr(x), _ptr(y), threads))
        return y

    def qmatvec_time(self, qtype, rows, cols, data, scales, x, threads, reps):
        y = np.empty(rows, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        sec = C.c_double(0)
        self._check(self.lib.ref_qmatvec_time(qtype, rows, cols, _ptr(data),
                                              _ptr(scales), _ptr(x), _ptr(y),
                                              threads, reps, C.byref(sec)))
        return sec.value, y

    def rmsnorm(self, x, w, eps=1e-5):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self._check(self.lib.ref_rmsnorm(_ptr(x), _ptr(np.ascontiguousarray(w, np.float32)),
                                         _ptr(out), x.size, eps))
        return out

    def matmul_f32(self, a, b, threads=1):
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        c = np.empty((a.shape[0], b.shape[1]), np.float32)
        self._check(self.lib.ref_matmul_threaded(_ptr(a), _ptr(b), _ptr(c), a.shape[0],
                                                 a.shape[1], b.shape[1], threads, 0, None))
        return c

    def matmul_time(self, a, b, threads, reps):
        """Seconds per matmul_threaded call (median-free mean over reps)."""
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        c = np.empty((a.shape[0], b.shape[1]), np.float32)
        t = C.c_double(0.0)
        self._check(self.lib.ref_matmul_threaded(_ptr(a), _ptr(b), _ptr(c), a.shape[0],
                                                 a.shape[1], b.shape[1], threads, reps,
                                                 C.byref(t)))
        return t.value

    def matvec_time(self, w, x, threads, reps):
        """Seconds per matvec_threaded call."""
        w = np.ascontiguousarray(w, np.float32)
        x = np.ascontiguousarray(x, np.float32)
        y = np.empty(w.shape[0], np.float32)
        t = C.c_double(0.0)
        self._check(self.lib.ref_matvec_time(_ptr(w), w.shape[0], w.shape[1], _ptr(x),
                                             _ptr(y), threads, reps, C.byref(t)))
        return t.value

    def matvec_f32(self, w, x, threads=1):
        w = np.ascontiguousarray(w, np.float32)
        y = np.empty(w.shape[0], np.float32)
        self._check(self.lib.ref_matvec_threaded(_ptr(w), w.shape[0], w.shape[1],
                                                 _ptr(np.ascontiguousarray(x, np.float32)),
                                                 _ptr(y), threads))
        return y

    def model(self, config, qtype: int, seed: int, tied: bool = False,
              layer_fp32=None, embeddings=None, lm_head=None) -> "RefModel":
        return RefModel(self, config, qtype, seed, tied, layer_fp32, embeddings,
                        lm_head)

    def llama2c_generate(self, path: str, qtype: int, prompt, max_tokens: int,
                         temperature: float = 0.0, top_p: float = 1.0, seed: int = 1):
        """load_llama2c_quantized_model (qtype 0 / 1) or load_llama2c_model
        (qtype 2) + generate_tokens_cached (eos stop)."""
        p = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(max(max_tokens, 1), np.int32)
        n = C.c_size_t(0)
        self._check(self.lib.ref_llama2c_generate(path.encode(), qtype, _ptr(p),
                                                  p.size, max_tokens, temperature, top_p,
                                                  seed, _ptr(ids), C.byref(n)))
        return ids[:n.value]

    def llama2c_inspect(self, path: str, qtype: int):
        """(config[9], tied, storage_bytes, fnv1a digest) of the reference loader."""
        cfg = (_I64 * 9)()
        tied = C.c_int(0)
        nbytes = C.c_uint64(0)
        digest = C.c_uint64(0)
        self._check(self.lib.ref_llama2c_inspect(path.encode(), qtype, cfg, C.byref(tied),
                                                 C.byref(nbytes), C.byref(digest)))
        return list(cfg), bool(tied.value), nbytes.value, digest.value

    def tokenizer_encode(self, path: str, vocab: int, text: bytes, bos: bool, eos: bool):
        ids = np.zeros(len(text) + 3, np.int32)
        n = C.c_size_t(0)
        self._check(self.lib.ref_llama2c_encode2(path.encode(), vocab, text, len(text),
                                                 int(bos), int(eos), _ptr(ids), ids.size,
                                                 C.byref(n)))
        return ids[:n.value].tolist()

    def tokenizer_decode(self, path: str, vocab: int, ids) -> bytes:
        a = np.ascontiguousarray(ids, np.int32)
        cap = 64 * max(len(a), 1)
        buf = C.create_string_buffer(cap)
        n = C.c_size_t(0)
        self._check(self.lib.ref_llama2c_decode(path.encode(), vocab, _ptr(a), len(a), buf,
                                                cap, C.byref(n)))
        return buf.raw[:n.value]

    def safetensors_inspect(self, path: str):
        """(config[9], storage_bytes, fnv1a digest) of load_model(path)."""
        cfg = (_I64 * 9)()
        nbytes = C.c_uint64(0)
        digest = C.c_uint64(0)
        self._check(self.lib.ref_safetensors_inspect(path.encode(), cfg, C.byref(nbytes),
                                                     C.byref(digest)))
        return list(cfg), nbytes.value, digest.value

    def safetensors_generate(self, path: str, prompt, max_tokens: int, temperature=0.0,
                             top_p=1.0, seed=1, cached=True):
        """load_model + generate_tokens_cached (or generate_tokens)."""
        p = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(max(max_tokens, 1), np.int32)
        n = C.c_size_t(0)
        self._check(self.lib.ref_safetensors_generate(path.encode(), _ptr(p), p.size,
                                                      max_tokens, temperature, top_p, seed,
                                                      int(cached), _ptr(ids), C.byref(n)))
        return ids[:n.value]

    def bpe_encode(self, vocab_path: str, merges_path: str, text: bytes):
        ids = np.zeros(len(text) + 1, np.int32)
        n = C.c_size_t(0)
        self._check(self.lib.ref_bpe_encode(vocab_path.encode(), merges_path.encode(), text,
                                            len(text), _ptr(ids), ids.size, C.byref(n)))
        return ids[:n.value]

    def bpe_decode(self, vocab_path: str, merges_path: str, ids) -> bytes:
        a = np.ascontiguousarray(ids, np.int32)
        cap = 1 << 16
        buf = C.create_string_buffer(cap)
        n = C.c_size_t(0)
        self._check(self.lib.ref_bpe_decode(vocab_path.encode(), merges_path.encode(),
                                            _ptr(a), len(a), buf, cap, C.byref(n)))
        return buf.raw[:n.value]

    def llama2c_encode(self, tokenizer_path: str, vocab: int, text: str, bos: bool = True):
        ids = np.zeros(4 * len(text.encode()) + 8, np.int32)
        n = C.c_size_t(0)
        self._check(self.lib.ref_llama2c_encode(tokenizer_path.encode(), vocab, text.encode(),
                                                int(bos), _ptr(ids), ids.size, C.byref(n)))
        return ids[:n.value]


class RefModel:
    """A QuantizedModelWeights built inside the reference from seeded fp32
    weights, quantised by the reference's own quantiser."""

    def __init__(self, ref: Reference, c, qtype, seed, tied, layer_fp32=None,
                 embeddings=None, lm_head=None):
        self.r = ref
        self.config = c
        cfg = (_I64 * 9)(*[int(getattr(c, n)) for n, _ in _Config._fields_])
        h = _P()
        ref._check(ref.lib.ref_model_new(cfg, qtype, int(tied), C.byref(h)))
        self.h = h
        emb = embeddings if embeddings is not None else embeddings_fp32(c, seed)
        ref._check(ref.lib.ref_model_set_embeddings(h, _ptr(emb)))
        ones = np.ones(c.dim, np.float32)
        lm = None if tied else (lm_head if lm_head is not None else lm_head_fp32(c, seed))
        ref._check(ref.lib.ref_model_set_final(h, _ptr(ones), _ptr(lm)))
        for layer in range(c.layers):
            mats = ([layer_fp32(layer, j) for j in range(7)] if layer_fp32
                    else [projection_fp32(c, seed, layer, j) for j in range(7)])
            arr = (_P * 7)(*[m.ctypes.data for m in mats])
            ref._check(ref.lib.ref_model_add_layer(h, arr, _ptr(ones), _ptr(ones)))

    def storage_bytes(self) -> int:
        n = C.c_size_t(0)
        self.r._check(self.r.lib.ref_model_storage_bytes(self.h, C.byref(n)))
        return n.value

    def layer_bytes(self, layer: int, which: int, rows: int, cols: int, qtype: int):
        n = rows * cols
        data = np.zeros(n if qtype == 0 else (n + 1) // 2, np.uint8)
        scales = np.zeros((n + 31) // 32, np.uint16)
        self.r._check(self.r.lib.ref_model_layer_bytes(self.h, layer, which, _ptr(data),
                                                       data.size, _ptr(scales), scales.size))
        return data, scales

    def generate(self, prompt, steps, threads=1, want_logits=True):
        p = np.ascontiguousarray(prompt, np.int32)
        ids = np.zeros(max(steps, 1), np.int32)
        lg = (np.empty((max(steps, 1), self.config.vocab_size), np.float32)
              if want_logits else None)
        hid = np.empty(self.config.dim, np.float32)
        ps, ds = C.c_double(0), C.c_double(0)
        self.r._check(self.r.lib.ref_generate(self.h, _ptr(p), p.size, steps, threads,
                                              _ptr(ids), _ptr(lg), _ptr(hid),
                                              C.byref(ps), C.byref(ds)))
        return ids[:steps], (lg[:steps] if lg is not None else None), hid, ps.value, ds.value

    def trace(self, prompt, steps, threads=1):
        p = np.ascontiguousarray(prompt, np.int32)
        out = np.empty((p.size + steps, self.config.dim), np.float32)
        self.r._check(self.r.lib.ref_trace(self.h, _ptr(p), p.size, steps, threads,
                                           _ptr(out)))
        return out

    def __del__(self):
        try:
            self.r.lib.ref_model_free(self.h)
        except Exception:
            pass


# ------------------------------------------------------------- llama2.c


def read_safetensors_model(path: str) -> dict:
    """The tensors of an fp32 safetensors checkpoint in read_llama2c's form
    (load_model's names and metadata, src/loader.cpp:440-498): projections
    [out][in] as stored, kv_heads 0, a separate classifier.  A checker for
    well-formed files only (no validation beyond the shapes it reshapes)."""
    import json
    raw = np.fromfile(path, dtype=np.uint8)
    n = int(raw[:8].view(np.uint64)[0])
    header = json.loads(bytes(raw[8:8 + n]).decode())
    md = header.pop("__metadata__")
    base = 8 + n

    def t(name):
        e = header[name]
        b, end = e["data_offsets"]
        return raw[base + b:base + end].view(np.float32).reshape(e["shape"])

    cfg = {k: int(md[f"nutllm.{k}"]) for k in ("layers", "heads", "dim", "head_dim",
                                                "ffn_dim", "vocab_size", "max_seq",
                                                "eos_token")}
    cfg["kv_heads"] = 0
    L = cfg["layers"]
    stack = lambda suffix: np.stack([t(f"model.layers.{l}.{suffix}")  # noqa: E731
                                     for l in range(L)])
    return {"config": cfg, "tied": False, "embeddings": t("model.embed_tokens.weight"),
            "wq": stack("self_attn.q_proj.weight"), "wk": stack("self_attn.k_proj.weight"),
            "wv": stack("self_attn.v_proj.weight"), "wo": stack("self_attn.o_proj.weight"),
            "w1": stack("mlp.gate_proj.weight"), "w3": stack("mlp.up_proj.weight"),
            "w2": stack("mlp.down_proj.weight"),
            "attention_norm": stack("input_layernorm.weight"),
            "ffn_norm": stack("post_attention_layernorm.weight"),
            "final_norm": t("model.norm.weight"), "classifier": t("lm_head.weight")}


def read_llama2c(path: str) -> dict:
    """The fp32 tensors of a llama2.c checkpoint, sectioned as the
    reference's parse_layout does (src/llama2.cpp:199-298): header of seven
    int32, then embeddings, attention norms, wq, wk, wv, wo, ffn norms, w1,
    w2, w3, final norm, RoPE tables (skipped), classifier if vocab < 0.
    eos is token 1.  Raises ValueError if the size does not match."""
    raw = np.fromfile(path, dtype=np.uint8)
    head = raw[:28].view(np.int32)
    dim, ffn, layers, heads, kv, vocab_s, max_seq = (int(v) for v in head)
    vocab = abs(vocab_s)
    hd = dim // heads
    kvd = kv * hd
    f = raw[28:].view(np.float32)
    sizes = [("embeddings", (vocab, dim)), ("attention_norm", (layers, dim)),
             ("wq", (layers, dim, dim)), ("wk", (layers, kvd, dim)),
             ("wv", (layers, kvd, dim)), ("wo", (layers, dim, dim)),
             ("ffn_norm", (layers, dim)), ("w1", (layers, ffn, dim)),
             ("w2", (layers, dim, ffn)), ("w3", (layers, ffn, dim)),
             ("final_norm", (dim,)), ("rope", (max_seq, hd))]
    if vocab_s < 0:
        sizes.append(("classifier", (vocab, dim)))
    out, at = {}, 0
    for name, shape in sizes:
        n = int(np.prod(shape))
        out[name] = f[at:at + n].reshape(shape)
        at += n
    if at != f.size:
        raise ValueError("llama2 checkpoint: size does not match configuration")
    out["config"] = dict(layers=layers, heads=heads, dim=dim, head_dim=hd, ffn_dim=ffn,
                         vocab_size=vocab, max_seq=max_seq, eos_token=1, kv_heads=kv)
    out["tied"] = vocab_s > 0
    return out
