"""nut_greedy_head_static: the greedy head that allocates nothing.

Callers that cannot call cudaMalloc / cudaFree (their device memory comes
from a host runtime's own arena, or they issue work where allocating is not
allowed) pass every input and output as device memory; the kernels' only
scratch is a fixed device array inside the library.  This test gives the
entry point device buffers holding the same hidden vectors, final norm and
classifier as a model handle, and checks its logits and argmax against the
model-handle entry point nut_logits, within the suite's logit tolerance, on
two calls in a row (the second call must not see the first call's scratch).
The file sorts last so a run that stops at the first failure has already
run every other test.
"""
import ctypes

import numpy as np
import pytest

import nutllm_b200 as nb
from nutllm_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-3
LOGIT_RTOL = 1e-3


def _entry():
    f = nb.cuda_lib().nut_greedy_head_static
    f.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 3 + [ctypes.c_void_p] * 3
    f.restype = ctypes.c_int
    return f


def _close(got, want):
    return np.all(np.abs(got - want) <= LOGIT_ATOL + LOGIT_RTOL * np.abs(want))


def test_static_head_matches_model_head_on_consecutive_calls(gpu):
    import torch

    wl = syn.WORKLOADS["tiny-int8"]
    c = wl.model_config()
    w = syn.build_model(c, wl.qtype, 1234)
    model = nb.DeviceModel(w, gpu)
    kv = nb.KVCache(model)
    prompt = syn.prompt_ids(c, 1234, wl.prompt)
    h1 = nb.prefill_quantized(model, prompt, kv)
    ref1, arg1 = nb.logits(model, kv)
    h2 = nb.decode_quantized_token(model, arg1, kv)
    ref2, arg2 = nb.logits(model, kv)

    dev = torch.device("cuda", gpu)
    torch.cuda.set_device(dev)
    norm = torch.from_numpy(w.final_norm).to(dev)
    weights = torch.from_numpy(np.ascontiguousarray(w.output_weights())).to(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    V, D = int(c.vocab_size), int(c.dim)
    f = _entry()

    for hidden, ref, arg in ((h1, ref1, arg1), (h2, ref2, arg2)):
        x = torch.from_numpy(hidden).to(dev).reshape(1, D)
        logits = torch.full((1, V), float("nan"), device=dev)
        argmax = torch.full((1,), -1, dtype=torch.int32, device=dev)
        status = f(x.data_ptr(), norm.data_ptr(), weights.data_ptr(), 1, V, D,
                   logits.data_ptr(), argmax.data_ptr(), stream)
        assert status == nb.NUT_OK, nb.cuda_lib().nut_last_error()
        torch.cuda.synchronize(dev)
        assert _close(logits.cpu().numpy()[0], ref)
        assert int(argmax.cpu()[0]) == arg

    # both rows in one call, then without the logits output
    x = torch.from_numpy(np.stack([h1, h2])).to(dev)
    logits = torch.empty((2, V), device=dev)
    argmax = torch.empty((2,), dtype=torch.int32, device=dev)
    for out in (logits.data_ptr(), None):
        status = f(x.data_ptr(), norm.data_ptr(), weights.data_ptr(), 2, V, D, out,
                   argmax.data_ptr(), stream)
        assert status == nb.NUT_OK, nb.cuda_lib().nut_last_error()
        torch.cuda.synchronize(dev)
        assert argmax.cpu().tolist() == [arg1, arg2]
    assert _close(logits.cpu().numpy()[0], ref1) and _close(logits.cpu().numpy()[1], ref2)


def test_static_head_rejects_batch_beyond_its_scratch(gpu):
    f = _entry()
    dummy = ctypes.c_void_p(16)  # never dereferenced: the size check comes first
    status = f(dummy, dummy, dummy, 65, 512, 288, None, dummy, None)
    assert status == nb.NUT_LENGTH_ERROR
    assert b"exceeds the static scratch limit of 64" in nb.cuda_lib().nut_last_error()
