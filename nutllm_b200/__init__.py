"""nutllm_b200 — the nutllm token loop on B200 (sm_100a).

Python mirror of the reference's C++ host API for the quantised token loop
(MokiMeow/nutllm include/quant.hpp, quant_model.hpp, kvcache.hpp,
generate.hpp), bound through ctypes to the C ABI of the in-tree
``lib/libnutcuda.so`` (include/nutllm_cuda.h) and the host library
``lib/libnutllm.so`` (include/nutllm_host.h).  There is no CPU fallback: if
the CUDA library is missing, loading fails loudly.

Errors are raised as the Python counterparts of the exception classes the
reference throws for the same condition: ``ValueError`` for
``std::invalid_argument``, ``IndexError`` for ``std::out_of_range``,
``OverflowError`` for ``std::length_error`` and ``std::range_error``,
``RuntimeError`` otherwise.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(HERE, "lib")
CUDA_LIB = os.path.join(LIB_DIR, "libnutcuda.so")
HOST_LIB = os.path.join(LIB_DIR, "libnutllm.so")

INT8 = 0
INT4 = 1
# loader type of the llama2.c entries that keeps fp32 weights
# (load_llama2c_model and the ModelWeights overload of generation)
FP32 = 2

NUT_OK = 0
NUT_INVALID_ARGUMENT = 1
NUT_OUT_OF_RANGE = 2
NUT_LENGTH_ERROR = 3
NUT_RUNTIME_ERROR = 4
NUT_RANGE_ERROR = 5
NUT_DEVICE_TIMEOUT = 6


class LengthError(OverflowError):
    """std::length_error."""


class RangeError(OverflowError):
    """std::range_error."""


class DeviceTimeout(RuntimeError):
    """A bounded device-side wait gave up (NUT_DEVICE_TIMEOUT)."""


_EXC = {
    NUT_INVALID_ARGUMENT: ValueError,
    NUT_OUT_OF_RANGE: IndexError,
    NUT_LENGTH_ERROR: LengthError,
    NUT_RANGE_ERROR: RangeError,
    NUT_RUNTIME_ERROR: RuntimeError,
    NUT_DEVICE_TIMEOUT: DeviceTimeout,
}


# --------------------------------------------------------------------------
# C structures (include/nutllm_cuda.h)


class Config(C.Structure):
    """ModelConfig (reference include/model.hpp:8-24)."""

    _fields_ = [(n, C.c_int64) for n in (
        "layers", "heads", "dim", "head_dim", "ffn_dim", "vocab_size",
        "max_seq", "eos_token", "kv_heads")]

    @property
    def effective_kv_heads(self) -> int:
        return self.kv_heads or self.heads

    @property
    def kv_dim(self) -> int:
        return self.effective_kv_heads * self.head_dim

    def as_dict(self) -> dict:
        return {n: int(getattr(self, n)) for n, _ in self._fields_}


class QMatrixView(C.Structure):
    _fields_ = [("data", C.c_void_p), ("scales", C.c_void_p),
                ("rows", C.c_int64), ("cols", C.c_int64),
                ("block_size", C.c_int64), ("type", C.c_int32)]


class LayerView(C.Structure):
    _fields_ = [(n, QMatrixView) for n in (
        "query", "key", "value", "output", "gate", "up", "down")] + [
        ("attention_norm", C.c_void_p), ("ffn_norm", C.c_void_p)]


class ModelView(C.Structure):
    _fields_ = [("config", Config), ("quant_type", C.c_int32),
                ("tied_embeddings", C.c_int32), ("embeddings", C.c_void_p),
                ("final_norm", C.c_void_p), ("lm_head", C.c_void_p),
                ("layers", C.POINTER(LayerView)), ("n_layers", C.c_int64)]


class LayerF32View(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "query", "key", "value", "output", "gate", "up", "down", "attention_norm",
        "ffn_norm")]


class ModelF32View(C.Structure):
    _fields_ = [("config", Config), ("tied_embeddings", C.c_int32),
                ("embeddings", C.c_void_p), ("final_norm", C.c_void_p),
                ("lm_head", C.c_void_p), ("layers", C.POINTER(LayerF32View)),
                ("n_layers", C.c_int64)]


class GenerationStats(C.Structure):
    """GenerationStats (reference include/generate.hpp:19-24)."""

    _fields_ = [("prefill_tokens", C.c_int64), ("generated_tokens", C.c_int64),
                ("prefill_seconds", C.c_double), ("decode_seconds", C.c_double)]


# --------------------------------------------------------------------------
# library loading


_cuda = None
_host = None

_P = C.c_void_p
_I64 = C.c_int64
_PI64 = C.POINTER(C.c_int64)


def _declare(lib, name, args, res=C.c_int):
    f = getattr(lib, name)
    f.argtypes = args
    f.restype = res


def cuda_lib() -> C.CDLL:
    """The C ABI library; raises if it has not been built."""
    global _cuda
    if _cuda is None:
        if not os.path.exists(CUDA_LIB):
            raise RuntimeError(
                f"nutllm_b200: {CUDA_LIB} is missing; build it with "
                "`make -C nutllm_b200` (there is no CPU fallback)")
        lib = C.CDLL(CUDA_LIB)
        _declare(lib, "nut_last_error", [], C.c_char_p)
        _declare(lib, "nut_device_count", [C.POINTER(C.c_int)])
        _declare(lib, "nut_qmatrix_create", [C.POINTER(QMatrixView), C.c_int,
                                             C.POINTER(_P)])
        _declare(lib, "nut_qmatrix_destroy", [_P])
        _declare(lib, "nut_qmatrix_download", [_P, _P, _P])
        _declare(lib, "nut_qmatvec", [_P, _P, _P])
        _declare(lib, "nut_qmatvec_async", [_P, _P, _P, _P])
        _declare(lib, "nut_qmatrix_gemm", [_P, _P, _I64, _P, _P])
        _declare(lib, "nut_qmatrix_error", [_P])
        _declare(lib, "nut_matmul_f32", [_P, _P, _P, _I64, _I64, _I64, _P])
        _declare(lib, "nut_matvec_f32", [_P, _P, _P, _I64, _I64, _P])
        _declare(lib, "nut_model_create", [C.POINTER(ModelView), C.c_int,
                                           C.POINTER(_P)])
        _declare(lib, "nut_model_create_f32", [C.POINTER(ModelF32View), C.c_int,
                                               C.POINTER(_P)])
        _declare(lib, "nut_model_destroy", [_P])
        _declare(lib, "nut_model_storage_bytes", [_P, C.POINTER(C.c_uint64)])
        _declare(lib, "nut_model_stream", [_P, C.POINTER(_P)])
        _declare(lib, "nut_model_set_prefill_threshold", [_P, _I64])
        _declare(lib, "nut_launch_count", [C.POINTER(C.c_uint64)])
        _declare(lib, "nut_kv_create", [_P, C.POINTER(_P)])
        _declare(lib, "nut_kv_destroy", [_P])
        _declare(lib, "nut_kv_reset", [_P])
        _declare(lib, "nut_kv_length", [_P, _PI64])
        _declare(lib, "nut_kv_set_length", [_P, _I64])
        _declare(lib, "nut_kv_memory_bytes", [_P, C.POINTER(C.c_uint64)])
        _declare(lib, "nut_kv_read", [_P, _I64, _I64, _I64, _P, _P])
        _declare(lib, "nut_decode_token", [_P, _P, C.c_int32, _P])
        _declare(lib, "nut_prefill", [_P, _P, _P, _I64, _P])
        _declare(lib, "nut_logits", [_P, _P, _P, C.POINTER(C.c_int32)])
        _declare(lib, "nut_generate_greedy", [
            _P, _P, _P, _I64, _I64, C.c_int32, _P, _PI64, _P,
            C.POINTER(GenerationStats)])
        _declare(lib, "nut_tp_unique_id", [_P, _I64])
        _declare(lib, "nut_batch_create", [C.POINTER(ModelView), C.c_int, _I64, C.c_int,
                                           C.c_int, _P, C.POINTER(_P)])
        _declare(lib, "nut_batch_create_synthetic", [C.POINTER(Config), C.c_uint64, C.c_int,
                                                     _I64, C.c_int, C.c_int, _P,
                                                     C.POINTER(_P)])
        _declare(lib, "nut_batch_destroy", [_P], None)
        _declare(lib, "nut_batch_info", [_P, _PI64])
        _declare(lib, "nut_tp_shard", [C.POINTER(Config), C.c_int, C.c_int, _PI64])
        _declare(lib, "nut_batch_ipc_handle", [_P, _P, _I64])
        _declare(lib, "nut_batch_set_prefill_threshold", [_P, _I64])
        _declare(lib, "nut_batch_open_peers", [_P, _P, _I64])
        _declare(lib, "nut_batch_stream", [_P, C.POINTER(_P)])
        _declare(lib, "nut_peer_all_reduce", [_P, _P, _I64, _P, _P, C.c_int, C.c_int, _P, _P,
                                              _I64, _P])
        _declare(lib, "nut_batch_generate", [_P, _P, _I64, _I64, _P, _P,
                                             C.POINTER(GenerationStats)])
        _cuda = lib
    return _cuda


def host_lib() -> C.CDLL:
    global _host
    if _host is None:
        if not os.path.exists(HOST_LIB):
            raise RuntimeError(
                f"nutllm_b200: {HOST_LIB} is missing; build it with "
                "`make -C nutllm_b200`")
        lib = C.CDLL(HOST_LIB)
        _declare(lib, "nut_host_last_error", [], C.c_char_p)
        _declare(lib, "nut_host_quantize", [_P, _I64, _I64, C.c_int32, _P, _P])
        _declare(lib, "nut_host_scale_to_half", [C.c_float,
                                                 C.POINTER(C.c_uint16)])
        _declare(lib, "nut_synth_normal", [C.c_uint64, C.c_uint64, C.c_float,
                                           _P, C.c_size_t], None)
        _declare(lib, "nut_synth_tokens", [C.c_uint64, C.c_uint64, C.c_int,
                                           C.c_int, _P, C.c_size_t], None)
        _declare(lib, "nut_host_llama2c_generate",
                 [C.c_char_p, C.c_int32, _P, _I64, _I64, C.c_float, C.c_float,
                  C.c_uint32, _P, _PI64, C.POINTER(GenerationStats)])
        _declare(lib, "nut_host_llama2c_inspect",
                 [C.c_char_p, C.c_int32, _PI64, C.POINTER(C.c_int32),
                  C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)])
        _declare(lib, "nut_host_choose_tokens",
                 [_P, _I64, _I64, C.c_float, C.c_float, C.c_uint32, _P])
        _declare(lib, "nut_host_tokenizer_encode",
                 [C.c_char_p, _I64, C.c_char_p, _I64, C.c_int32, C.c_int32, _P, _I64, _PI64])
        _declare(lib, "nut_host_tokenizer_decode",
                 [C.c_char_p, _I64, _P, _I64, C.c_char_p, _I64, _PI64])
        _declare(lib, "nut_host_safetensors_inspect",
                 [C.c_char_p, _PI64, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)])
        _declare(lib, "nut_host_safetensors_generate",
                 [C.c_char_p, _P, _I64, _I64, C.c_float, C.c_float, C.c_uint32, C.c_int32,
                  _P, _PI64])
        _declare(lib, "nut_host_bpe_encode",
                 [C.c_char_p, C.c_char_p, C.c_char_p, _I64, _P, _I64, _PI64])
        _declare(lib, "nut_host_bpe_decode",
                 [C.c_char_p, C.c_char_p, _P, _I64, C.c_char_p, _I64, _PI64])
        _host = lib
    return _host


def _check(status: int, lib=None) -> None:
    if status == NUT_OK:
        return
    if lib is None:
        msg = cuda_lib().nut_last_error()
    else:
        msg = lib.nut_host_last_error()
    raise _EXC.get(status, RuntimeError)(msg.decode() if msg else "nutllm error")


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


def device_count() -> int:
    n = C.c_int(0)
    _check(cuda_lib().nut_device_count(C.byref(n)))
    return n.value


# --------------------------------------------------------------------------
# host quantiser and synthetic inputs


def storage_sizes(rows: int, cols: int, qtype: int) -> tuple[int, int]:
    n = rows * cols
    return (n if qtype == INT8 else (n + 1) // 2), (n + 31) // 32



def launch_count() -> int:
    """Kernels the library has launched in this process so far."""
    out = C.c_uint64()
    _check(cuda_lib().nut_launch_count(C.byref(out)))
    return out.value


def matmul_f32_async(a_dev: int, b_dev: int, c_dev: int, m: int, k: int, n: int,
                     stream: int = 0) -> None:
    """matmul_threaded on device buffers (bit-identical to the reference)."""
    _check(cuda_lib().nut_matmul_f32(a_dev, b_dev, c_dev, m, k, n, stream or None))


def matvec_f32_async(w_dev: int, x_dev: int, y_dev: int, rows: int, cols: int,
                     stream: int = 0) -> None:
    """matvec_threaded on device buffers (bit-identical to the reference)."""
    _check(cuda_lib().nut_matvec_f32(w_dev, x_dev, y_dev, rows, cols, stream or None))

def quantize(weights: np.ndarray, qtype: int) -> tuple[np.ndarray, np.ndarray]:
    """QuantizedMatrix::quantize (reference src/quant.cpp:154-197): returns
    (packed bytes, fp16 scale bits) in the reference storage layout."""
    w = np.ascontiguousarray(weights, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("quantize: expected a 2-D matrix")
    rows, cols = w.shape
    nd, ns = storage_sizes(rows, cols, qtype)
    data = np.zeros(nd, np.uint8)
    scales = np.zeros(ns, np.uint16)
    lib = host_lib()
    _check(lib.nut_host_quantize(_ptr(w), rows, cols, qtype, _ptr(data),
                                 _ptr(scales)), lib)
    return data, scales


def scale_to_half(value: float) -> int:
    lib = host_lib()
    out = C.c_uint16(0)
    _check(lib.nut_host_scale_to_half(C.c_float(value), C.byref(out)), lib)
    return out.value


def synth_normal(seed: int, stream: int, n: int, sigma: float = 0.02) -> np.ndarray:
    out = np.empty(n, np.float32)
    host_lib().nut_synth_normal(seed, stream, sigma, _ptr(out), n)
    return out


def synth_tokens(seed: int, stream: int, n: int, lo: int, hi: int) -> np.ndarray:
    out = np.empty(n, np.int32)
    host_lib().nut_synth_tokens(seed, stream, lo, hi, _ptr(out), n)
    return out


def llama2c_generate(path: str, qtype: int, prompt, max_tokens: int,
                     temperature: float = 0.0, top_p: float = 1.0,
                     seed: int = 1) -> tuple[np.ndarray, GenerationStats]:
    """load_llama2c_quantized_model (qtype INT8 / INT4) or load_llama2c_model
    (qtype FP32) + generate_tokens_cached through the C++ host API (reference
    include/llama2.hpp:27-29, include/generate.hpp:29-36): stops at eos
    (token 1) or a full context like the reference."""
    lib = host_lib()
    p = np.ascontiguousarray(prompt, np.int32)
    ids = np.zeros(max(max_tokens, 1), np.int32)
    n = C.c_int64(0)
    st = GenerationStats()
    _check(lib.nut_host_llama2c_generate(os.fsencode(path), qtype, _ptr(p), p.size,
                                         max_tokens, temperature, top_p, seed, _ptr(ids),
                                         C.byref(n), C.byref(st)), lib)
    return ids[:n.value], st


def llama2c_inspect(path: str, qtype: int) -> tuple[list, bool, int, int]:
    """(config[9], tied classifier, storage_bytes, FNV-1a digest of the
    loaded bytes) of the host loader; no device involved."""
    lib = host_lib()
    cfg = (C.c_int64 * 9)()
    tied = C.c_int32(0)
    nbytes = C.c_uint64(0)
    digest = C.c_uint64(0)
    _check(lib.nut_host_llama2c_inspect(os.fsencode(path), qtype, cfg, C.byref(tied),
                                        C.byref(nbytes), C.byref(digest)), lib)
    return list(cfg), bool(tied.value), nbytes.value, digest.value


def safetensors_inspect(path: str) -> tuple[list, int, int]:
    """(config[9], storage_bytes, FNV-1a digest) of load_model(path) (the
    fp32 safetensors loader, reference src/loader.cpp:440-498)."""
    lib = host_lib()
    cfg = (C.c_int64 * 9)()
    nbytes = C.c_uint64(0)
    digest = C.c_uint64(0)
    _check(lib.nut_host_safetensors_inspect(os.fsencode(path), cfg, C.byref(nbytes),
                                            C.byref(digest)), lib)
    return list(cfg), nbytes.value, digest.value


def safetensors_generate(path: str, prompt, max_tokens: int, temperature: float = 0.0,
                         top_p: float = 1.0, seed: int = 1, cached: bool = True) -> np.ndarray:
    """load_model + generate_tokens_cached (cached) or generate_tokens on the
    current device through the C++ host API."""
    lib = host_lib()
    p = np.ascontiguousarray(prompt, np.int32)
    ids = np.zeros(max(max_tokens, 1), np.int32)
    n = C.c_int64(0)
    _check(lib.nut_host_safetensors_generate(os.fsencode(path), _ptr(p) if p.size else None,
                                             p.size, max_tokens, temperature, top_p, seed,
                                             int(cached), _ptr(ids), C.byref(n)), lib)
    return ids[:n.value]


def bpe_encode(vocab_path: str, merges_path: str, text: bytes) -> list:
    """Tokenizer::load(vocab_path, merges_path).encode(text) (byte-level BPE)."""
    lib = host_lib()
    ids = np.zeros(len(text) + 1, np.int32)
    n = C.c_int64(0)
    _check(lib.nut_host_bpe_encode(os.fsencode(vocab_path), os.fsencode(merges_path), text,
                                   len(text), _ptr(ids), ids.size, C.byref(n)), lib)
    return ids[:n.value].tolist()


def bpe_decode(vocab_path: str, merges_path: str, ids) -> bytes:
    """Tokenizer::load(vocab_path, merges_path).decode(ids)."""
    lib = host_lib()
    a = np.ascontiguousarray(ids, np.int32)
    cap = 1 << 16
    buf = C.create_string_buffer(cap)
    n = C.c_int64(0)
    _check(lib.nut_host_bpe_decode(os.fsencode(vocab_path), os.fsencode(merges_path),
                                   _ptr(a) if a.size else None, a.size, buf, cap,
                                   C.byref(n)), lib)
    return buf.raw[:n.value]


def tokenizer_encode(path: str, vocab: int, text: str, bos: bool = True,
                     eos: bool = False) -> list:
    """Llama2Tokenizer::load(path, vocab).encode(text, bos, eos)."""
    lib = host_lib()
    raw = text.encode("utf-8")
    cap = len(raw) + 3
    ids = np.zeros(cap, np.int32)
    n = C.c_int64(0)
    _check(lib.nut_host_tokenizer_encode(os.fsencode(path), vocab, raw, len(raw), int(bos),
                                         int(eos), _ptr(ids), cap, C.byref(n)), lib)
    return ids[:n.value].tolist()


def tokenizer_decode(path: str, vocab: int, ids) -> bytes:
    """Llama2Tokenizer::load(path, vocab).decode(ids), as raw bytes."""
    lib = host_lib()
    a = np.ascontiguousarray(ids, np.int32)
    cap = 64 * max(len(a), 1)
    buf = C.create_string_buffer(cap)
    n = C.c_int64(0)
    _check(lib.nut_host_tokenizer_decode(os.fsencode(path), vocab, _ptr(a), len(a), buf, cap,
                                         C.byref(n)), lib)
    return buf.raw[:n.value]


def choose_tokens(logits: np.ndarray, temperature: float, top_p: float,
                  seed: int) -> np.ndarray:
    """The generation token choice over rows of logits with one seeded
    std::mt19937 (reference src/generate.cpp:25-73)."""
    lib = host_lib()
    lg = np.ascontiguousarray(np.atleast_2d(logits), np.float32)
    out = np.zeros(lg.shape[0], np.int64)
    _check(lib.nut_host_choose_tokens(_ptr(lg), lg.shape[0], lg.shape[1], temperature,
                                      top_p, seed, _ptr(out)), lib)
    return out


# --------------------------------------------------------------------------
# quantised matrices and models (host images)


@dataclass
class QuantizedMatrix:
    """Host storage of one quantised matrix (reference include/quant.hpp)."""

    data: np.ndarray
    scales: np.ndarray
    rows: int
    cols: int
    qtype: int

    @classmethod
    def quantize(cls, weights: np.ndarray, qtype: int) -> "QuantizedMatrix":
        data, scales = quantize(weights, qtype)
        return cls(data, scales, int(weights.shape[0]), int(weights.shape[1]),
                   qtype)

    def view(self) -> QMatrixView:
        return QMatrixView(self.data.ctypes.data, self.scales.ctypes.data,
                           self.rows, self.cols, 32, self.qtype)

    def storage_bytes(self) -> int:
        return int(self.data.nbytes + self.scales.nbytes)


PROJECTIONS = ("query", "key", "value", "output", "gate", "up", "down")


@dataclass
class LayerWeights:
    """QuantizedLayerWeights (reference include/quant_model.hpp:9-29)."""

    query: QuantizedMatrix
    key: QuantizedMatrix
    value: QuantizedMatrix
    output: QuantizedMatrix
    gate: QuantizedMatrix
    up: QuantizedMatrix
    down: QuantizedMatrix
    attention_norm: np.ndarray
    ffn_norm: np.ndarray

    def projections(self) -> list[QuantizedMatrix]:
        return [getattr(self, p) for p in PROJECTIONS]


@dataclass
class ModelWeights:
    """QuantizedModelWeights (reference include/quant_model.hpp:31-46)."""

    config: Config
    qtype: int
    embeddings: np.ndarray  # [vocab, dim] fp32
    layers: list
    final_norm: np.ndarray
    lm_head: Optional[np.ndarray]  # None when tied
    tied_embeddings: bool = False

    def output_weights(self) -> np.ndarray:
        return self.embeddings if self.tied_embeddings else self.lm_head

    def storage_bytes(self) -> int:
        """QuantizedModelWeights::storage_bytes (src/quant_model.cpp:140-156)."""
        total = self.embeddings.nbytes + self.final_norm.nbytes
        if not self.tied_embeddings:
            total += self.lm_head.nbytes
        for layer in self.layers:
            total += sum(m.storage_bytes() for m in layer.projections())
            total += layer.attention_norm.nbytes + layer.ffn_norm.nbytes
        return total

    def view(self) -> tuple[ModelView, object]:
        """C view; the second value keeps the layer array alive."""
        layers = (LayerView * len(self.layers))()
        for i, layer in enumerate(self.layers):
            lv = layers[i]
            for p in PROJECTIONS:
                setattr(lv, p, getattr(layer, p).view())
            lv.attention_norm = layer.attention_norm.ctypes.data
            lv.ffn_norm = layer.ffn_norm.ctypes.data
        v = ModelView()
        v.config = self.config
        v.quant_type = self.qtype
        v.tied_embeddings = int(self.tied_embeddings)
        v.embeddings = self.embeddings.ctypes.data
        v.final_norm = self.final_norm.ctypes.data
        v.lm_head = None if self.tied_embeddings else self.lm_head.ctypes.data
        v.layers = C.cast(layers, C.POINTER(LayerView))
        v.n_layers = len(self.layers)
        return v, layers


# --------------------------------------------------------------------------
# device objects


class DeviceQMatrix:
    """Device mirror of one quantised matrix (nut_qmatrix)."""

    def __init__(self, m: QuantizedMatrix, device: int = 0):
        self.rows, self.cols, self.qtype = m.rows, m.cols, m.qtype
        h = C.c_void_p()
        _check(cuda_lib().nut_qmatrix_create(C.byref(m.view()), device,
                                             C.byref(h)))
        self.handle = h

    def matvec(self, x: np.ndarray) -> np.ndarray:
        """matvec_quantized_threaded with host buffers."""
        x = np.ascontiguousarray(x, np.float32)
        if x.shape != (self.cols,):
            raise ValueError("quantized matvec: vector length mismatch")
        y = np.empty(self.rows, np.float32)
        _check(cuda_lib().nut_qmatvec(self.handle, _ptr(x), _ptr(y)))
        return y

    def matvec_async(self, x_dev: int, y_dev: int, stream: int = 0) -> None:
        _check(cuda_lib().nut_qmatvec_async(self.handle, x_dev, y_dev,
                                            stream or None))

    def gemm_async(self, x_dev: int, tokens: int, y_dev: int, stream: int = 0) -> None:
        """Y[tokens][rows] = X[tokens][cols] Q^T on the tensor cores (fp16
        operands, fp32 accumulation), device buffers."""
        _check(cuda_lib().nut_qmatrix_gemm(self.handle, x_dev, int(tokens), y_dev,
                                           stream or None))

    def check(self) -> None:
        """Raises DeviceTimeout if an earlier asynchronous call gave up."""
        _check(cuda_lib().nut_qmatrix_error(self.handle))

    def download(self) -> tuple[np.ndarray, np.ndarray]:
        nd, ns = storage_sizes(self.rows, self.cols, self.qtype)
        data = np.empty(nd, np.uint8)
        scales = np.empty(ns, np.uint16)
        _check(cuda_lib().nut_qmatrix_download(self.handle, _ptr(data),
                                               _ptr(scales)))
        return data, scales

    def close(self) -> None:
        if getattr(self, "handle", None):
            cuda_lib().nut_qmatrix_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def tp_shard(config: Config, rank: int, world: int) -> dict:
    """This rank's slice of heads, kv heads, FFN units and classifier rows
    (host only; raises ValueError when the split is not even)."""
    v = (C.c_int64 * 8)()
    _check(cuda_lib().nut_tp_shard(C.byref(config), rank, world, v))
    keys = ("head0", "heads", "kv0", "kv_heads", "ffn0", "ffn", "vocab0", "vocab_rows")
    return dict(zip(keys, [int(x) for x in v]))


PEER_AR_CHUNKS = 128


def peer_all_reduce(x: int, out: int, n: int, recv: Sequence[int], flags: Sequence[int],
                    rank: int, world: int, epochs: int, error: int, limit_ns: int,
                    stream: int = 0) -> None:
    """nut_peer_all_reduce on device pointers (ints): raises DeviceTimeout if
    a wait for a peer's chunk gave up after limit_ns."""
    r = (C.c_void_p * world)(*recv)
    f = (C.c_void_p * world)(*flags)
    _check(cuda_lib().nut_peer_all_reduce(x, out, n, r, f, rank, world, epochs, error,
                                          int(limit_ns), stream or None))


def tp_unique_id() -> bytes:
    """ncclGetUniqueId, for rank 0 to broadcast to the other ranks."""
    buf = (C.c_uint8 * 128)()
    _check(cuda_lib().nut_tp_unique_id(buf, 128))
    return bytes(buf)


class TPBatch:
    """One rank's shard of the tensor-parallel batched decoder (nut_batch):
    `batch` sequences generated in lockstep, heads / FFN units / classifier
    rows split over `world` ranks with NCCL all-reduces.  Build it from host
    weights (`weights`, every rank passes the whole model) or, for shapes too
    large for the host, from seeded synthetic weights (`config`, `seed`)."""

    def __init__(self, batch: int, rank: int = 0, world: int = 1, nccl_id: bytes = None,
                 weights: "ModelWeights" = None, config: Config = None, seed: int = 0,
                 device: int = 0):
        if world > 1 and (nccl_id is None or len(nccl_id) < 128):
            raise ValueError("TPBatch: world > 1 needs the 128-byte NCCL id")
        idbuf = (C.c_uint8 * 128).from_buffer_copy(nccl_id[:128]) if nccl_id else None
        h = C.c_void_p()
        lib = cuda_lib()
        if weights is not None:
            view, keep = weights.view()
            _check(lib.nut_batch_create(C.byref(view), device, batch, rank, world, idbuf,
                                        C.byref(h)))
            del keep
            self.config = Config(**weights.config.as_dict())
        else:
            if config is None:
                raise ValueError("TPBatch: weights or config required")
            _check(lib.nut_batch_create_synthetic(C.byref(config), seed, device, batch, rank,
                                                  world, idbuf, C.byref(h)))
            self.config = Config(**config.as_dict())
        self.handle = h
        self.batch, self.rank, self.world = batch, rank, world

    def set_prefill_threshold(self, min_tokens: int) -> None:
        """Prompts of at least min_tokens tokens (0 = never) are prefilled as
        GEMMs over whole sequences rather than one position per pass."""
        _check(cuda_lib().nut_batch_set_prefill_threshold(self.handle, int(min_tokens)))

    def ipc_handle(self) -> bytes:
        """This rank's receive-area handle for the peer-memory all-reduce."""
        buf = (C.c_uint8 * 64)()
        _check(cuda_lib().nut_batch_ipc_handle(self.handle, buf, 64))
        return bytes(buf)

    def open_peers(self, handles: list) -> None:
        """Switches the Wo/Wdown sums from NCCL to the peer-memory all-reduce
        (handles: every rank's ipc_handle(), in rank order).  Collective."""
        blob = b"".join(h[:64].ljust(64, b"\0") for h in handles)
        buf = (C.c_uint8 * len(blob)).from_buffer_copy(blob)
        _check(cuda_lib().nut_batch_open_peers(self.handle, buf, 64))

    def info(self) -> dict:
        v = (C.c_int64 * 8)()
        _check(cuda_lib().nut_batch_info(self.handle, v))
        keys = ("batch", "heads", "kv_heads", "ffn", "vocab0", "vocab_rows",
                "weight_bytes", "world")
        return dict(zip(keys, [int(x) for x in v]))

    @property
    def stream(self) -> int:
        out = _P()
        _check(cuda_lib().nut_batch_stream(self.handle, C.byref(out)))
        return int(out.value or 0)

    def generate(self, prompts: np.ndarray, steps: int, want_logits: bool = False):
        """prompts [batch][n] -> (ids [batch][steps], logits [steps][batch][this
        rank's vocabulary rows] or None, GenerationStats).  Collective over
        the ranks."""
        p = np.ascontiguousarray(prompts, np.int32)
        if p.ndim != 2 or p.shape[0] != self.batch:
            raise ValueError("TPBatch.generate: prompts must be [batch][n]")
        ids = np.zeros((self.batch, max(steps, 1)), np.int32)
        rows = self.info()["vocab_rows"] if want_logits else 0
        lg = np.zeros((max(steps, 1), self.batch, rows), np.float32) if want_logits else None
        st = GenerationStats()
        _check(cuda_lib().nut_batch_generate(self.handle, _ptr(p), p.shape[1], steps,
                                             _ptr(ids), _ptr(lg), C.byref(st)))
        return ids[:, :steps], (lg[:steps] if lg is not None else None), st

    def close(self) -> None:
        if getattr(self, "handle", None):
            cuda_lib().nut_batch_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DeviceModel:
    """A QuantizedModelWeights image (or, through DeviceModel.fp32, a
    ModelWeights image) on one GPU (nut_model)."""

    def __init__(self, weights: ModelWeights, device: int = 0):
        self.config = Config(**weights.config.as_dict())
        self.device = device
        view, keep = weights.view()
        h = C.c_void_p()
        _check(cuda_lib().nut_model_create(C.byref(view), device, C.byref(h)))
        del keep
        self.handle = h

    @classmethod
    def fp32(cls, config: Config, embeddings: np.ndarray, layers: Sequence[dict],
             final_norm: np.ndarray, lm_head: np.ndarray = None,
             device: int = 0) -> "DeviceModel":
        """An fp32-weight model (the reference's ModelWeights) on one GPU
        (nut_model_create_f32).  Each layer is a dict of fp32 arrays: query,
        key, value, output, gate, up, down as [out][in] (the llama2.c
        storage), attention_norm and ffn_norm; lm_head None ties the
        classifier to the embeddings."""
        self = cls.__new__(cls)
        self.config = Config(**config.as_dict())
        self.device = device
        keep = []

        def arr(a):
            a = np.ascontiguousarray(a, np.float32)
            keep.append(a)
            return a.ctypes.data

        lv = (LayerF32View * len(layers))()
        for i, lw in enumerate(layers):
            for name in ("query", "key", "value", "output", "gate", "up", "down",
                         "attention_norm", "ffn_norm"):
                setattr(lv[i], name, arr(lw[name]))
        view = ModelF32View()
        view.config = self.config
        view.tied_embeddings = int(lm_head is None)
        view.embeddings = arr(embeddings)
        view.final_norm = arr(final_norm)
        view.lm_head = None if lm_head is None else arr(lm_head)
        view.layers = C.cast(lv, C.POINTER(LayerF32View))
        view.n_layers = len(layers)
        h = C.c_void_p()
        _check(cuda_lib().nut_model_create_f32(C.byref(view), device, C.byref(h)))
        self.handle = h
        return self

    def storage_bytes(self) -> int:
        out = C.c_uint64(0)
        _check(cuda_lib().nut_model_storage_bytes(self.handle, C.byref(out)))
        return out.value

    def set_prefill_threshold(self, min_tokens: int) -> None:
        """Prompts of at least min_tokens tokens (0 = never) are prefilled as
        one batch of tensor-core GEMMs (fp16 operands)."""
        _check(cuda_lib().nut_model_set_prefill_threshold(self.handle, int(min_tokens)))

    @property
    def stream(self) -> int:
        """The cudaStream_t (as an integer) all work on this model runs on."""
        out = _P()
        _check(cuda_lib().nut_model_stream(self.handle, C.byref(out)))
        return int(out.value or 0)

    def close(self) -> None:
        if getattr(self, "handle", None):
            cuda_lib().nut_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KVCache:
    """Device KV cache and decode state of one sequence (nut_kv)."""

    def __init__(self, model: DeviceModel):
        self.model = model
        h = C.c_void_p()
        _check(cuda_lib().nut_kv_create(model.handle, C.byref(h)))
        self.handle = h

    def length(self) -> int:
        out = C.c_int64(0)
        _check(cuda_lib().nut_kv_length(self.handle, C.byref(out)))
        return out.value

    def capacity(self) -> int:
        return int(self.model.config.max_seq)

    def reset(self) -> None:
        _check(cuda_lib().nut_kv_reset(self.handle))

    def set_length(self, n: int) -> None:
        _check(cuda_lib().nut_kv_set_length(self.handle, n))

    def memory_bytes(self) -> int:
        out = C.c_uint64(0)
        _check(cuda_lib().nut_kv_memory_bytes(self.handle, C.byref(out)))
        return out.value

    def key(self, layer: int, head: int, position: int) -> np.ndarray:
        out = np.empty(self.model.config.head_dim, np.float32)
        _check(cuda_lib().nut_kv_read(self.handle, layer, head, position,
                                      _ptr(out), None))
        return out

    def value(self, layer: int, head: int, position: int) -> np.ndarray:
        out = np.empty(self.model.config.head_dim, np.float32)
        _check(cuda_lib().nut_kv_read(self.handle, layer, head, position,
                                      None, _ptr(out)))
        return out

    def close(self) -> None:
        if getattr(self, "handle", None):
            cuda_lib().nut_kv_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def decode_quantized_token(model: DeviceModel, token: int, cache: KVCache,
                           thread_count: int = 1) -> np.ndarray:
    """decode_quantized_token (reference src/quant_model.cpp:158-206)."""
    if thread_count == 0:
        raise ValueError("quantized decode: zero threads")
    hidden = np.empty(model.config.dim, np.float32)
    _check(cuda_lib().nut_decode_token(model.handle, cache.handle, int(token),
                                       _ptr(hidden)))
    return hidden


def prefill_quantized(model: DeviceModel, tokens: Sequence[int], cache: KVCache,
                      thread_count: int = 1) -> np.ndarray:
    """prefill_quantized (reference src/quant_model.cpp:208-220)."""
    if thread_count == 0:
        raise ValueError("quantized decode: zero threads")
    t = np.ascontiguousarray(tokens, np.int32)
    hidden = np.empty(model.config.dim, np.float32)
    _check(cuda_lib().nut_prefill(model.handle, cache.handle,
                                  _ptr(t) if t.size else None, t.size,
                                  _ptr(hidden)))
    return hidden


def logits(model: DeviceModel, cache: KVCache) -> tuple[np.ndarray, int]:
    """Final rmsnorm + lm_head + argmax of the last hidden vector."""
    out = np.empty(model.config.vocab_size, np.float32)
    best = C.c_int32(0)
    _check(cuda_lib().nut_logits(model.handle, cache.handle, _ptr(out),
                                 C.byref(best)))
    return out, best.value


def generate_greedy(model: DeviceModel, cache: KVCache, prompt: Sequence[int],
                    max_tokens: int, stop_at_eos: bool = True,
                    want_logits: bool = False):
    """Greedy generate_tokens_cached (reference src/generate.cpp:174-216).

    Returns (ids, logits or None, GenerationStats)."""
    p = np.ascontiguousarray(prompt, np.int32)
    ids = np.zeros(max(max_tokens, 1), np.int32)
    lg = (np.empty((max_tokens, model.config.vocab_size), np.float32)
          if want_logits and max_tokens > 0 else None)
    n = C.c_int64(0)
    stats = GenerationStats()
    _check(cuda_lib().nut_generate_greedy(
        model.handle, cache.handle, _ptr(p) if p.size else None, p.size,
        max_tokens, int(stop_at_eos), _ptr(ids), C.byref(n), _ptr(lg),
        C.byref(stats)))
    return ids[:n.value].copy(), (lg[:n.value] if lg is not None else None), stats
