"""nut_greedy_head_static: the greedy head that allocates nothing.

Callers that cannot call cudaMalloc / cudaFree (their device memory comes
from a host runtime's own arena, or they issue work where allocating is not
allowed) pass every input and output as device memory; the kernels' only
scratch is a fixed device array inside the library.  These tests give the
entry point device buffers and check its logits and argmax against the CPU
oracle (the reference's final rmsnorm + fp32 classifier + first-index
argmax, src/generate.cpp:197-201) and against the model-handle entry point
nut_logits, within the suite's logit tolerance, on two calls in a row (the
second call must not see the first call's scratch).  They also cover the
scalar path (dim % 4 != 0), an arena pointer that is only 4-byte aligned,
and that a call leaves the device's free memory unchanged.
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


def _oracle_head(orc, hidden, norm, weights):
    """rmsnorm + matvec_threaded + first-index argmax on the CPU."""
    x = orc.rmsnorm(hidden, norm)
    logits = orc.matvec_f32(weights, x)
    return logits, int(np.argmax(logits))


def test_static_head_matches_oracle_on_consecutive_calls(gpu, orc):
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
    om = orc.model(w)
    o1, oa1 = om.logits(h1)
    o2, oa2 = om.logits(h2)
    assert (oa1, oa2) == (arg1, arg2)

    dev = torch.device("cuda", gpu)
    torch.cuda.set_device(dev)
    norm = torch.from_numpy(w.final_norm).to(dev)
    weights = torch.from_numpy(np.ascontiguousarray(w.output_weights())).to(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    V, D = int(c.vocab_size), int(c.dim)
    f = _entry()

    for hidden, ref, want, arg in ((h1, ref1, o1, arg1), (h2, ref2, o2, arg2)):
        x = torch.from_numpy(hidden).to(dev).reshape(1, D)
        logits = torch.full((1, V), float("nan"), device=dev)
        argmax = torch.full((1,), -1, dtype=torch.int32, device=dev)
        status = f(x.data_ptr(), norm.data_ptr(), weights.data_ptr(), 1, V, D,
                   logits.data_ptr(), argmax.data_ptr(), stream)
        assert status == nb.NUT_OK, nb.cuda_lib().nut_last_error()
        torch.cuda.synchronize(dev)
        got = logits.cpu().numpy()[0]
        assert _close(got, want)
        assert _close(got, ref)
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
    assert _close(logits.cpu().numpy()[0], o1) and _close(logits.cpu().numpy()[1], o2)


@pytest.mark.parametrize("dim,offset", [(290, 0), (288, 1), (291, 1)])
def test_static_head_scalar_path_and_unaligned_arena(gpu, orc, dim, offset):
    """dim % 4 != 0, and/or a weights pointer 4 bytes past a 16-byte
    boundary (an arena slice): both must take the scalar loop."""
    import torch

    rng = np.random.default_rng(dim * 7 + offset)
    V, B = 777, 3
    hidden = rng.standard_normal((B, dim)).astype(np.float32)
    norm = (1.0 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    weights = (0.02 * rng.standard_normal((V, dim))).astype(np.float32)
    dev = torch.device("cuda", gpu)
    torch.cuda.set_device(dev)
    arena = torch.zeros(V * dim + 8, device=dev)  # the caller's own buffer
    arena[offset:offset + V * dim] = torch.from_numpy(weights.ravel()).to(dev)
    wptr = arena.data_ptr() + 4 * offset
    assert (wptr % 16 == 0) == (offset == 0)
    x = torch.from_numpy(hidden).to(dev)
    nd = torch.from_numpy(norm).to(dev)
    logits = torch.empty((B, V), device=dev)
    argmax = torch.empty((B,), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    f = _entry()
    for _ in range(2):
        logits.fill_(float("nan"))
        argmax.fill_(-1)
        status = f(x.data_ptr(), nd.data_ptr(), wptr, B, V, dim, logits.data_ptr(),
                   argmax.data_ptr(), stream)
        assert status == nb.NUT_OK, nb.cuda_lib().nut_last_error()
        torch.cuda.synchronize(dev)
        got, ids = logits.cpu().numpy(), argmax.cpu().numpy()
        for b in range(B):
            want, arg = _oracle_head(orc, hidden[b], norm, weights)
            assert _close(got[b], want)
            top2 = np.sort(want)[-2:]
            if top2[1] - top2[0] > 1e-4:  # no near-tie: ids must agree
                assert int(ids[b]) == arg


def test_static_head_allocates_nothing(gpu):
    """After the first call on the device, further calls leave the device's
    free memory unchanged (nothing allocated, nothing freed)."""
    import torch

    dev = torch.device("cuda", gpu)
    torch.cuda.set_device(dev)
    V, D, B = 4096, 256, 8
    x = torch.randn(B, D, device=dev)
    nd = torch.ones(D, device=dev)
    wd = torch.randn(V, D, device=dev) * 0.02
    logits = torch.empty((B, V), device=dev)
    argmax = torch.empty((B,), dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    f = _entry()

    def call():
        status = f(x.data_ptr(), nd.data_ptr(), wd.data_ptr(), B, V, D,
                   logits.data_ptr(), argmax.data_ptr(), stream)
        assert status == nb.NUT_OK, nb.cuda_lib().nut_last_error()
        torch.cuda.synchronize(dev)

    call()  # first call on the device: resolves the scratch address
    free0, _ = torch.cuda.mem_get_info(dev)
    for _ in range(3):
        call()
    free1, _ = torch.cuda.mem_get_info(dev)
    assert free1 == free0
    xs = x.cpu().double()
    xs = xs / torch.sqrt((xs * xs).mean(dim=1, keepdim=True) + 1e-5)
    want = (xs @ wd.cpu().double().T).numpy()
    assert _close(logits.cpu().numpy(), want)


def test_static_head_rejects_batch_beyond_its_scratch(gpu):
    f = _entry()
    dummy = ctypes.c_void_p(16)  # never dereferenced: the size check comes first
    status = f(dummy, dummy, dummy, 65, 512, 288, None, dummy, None)
    assert status == nb.NUT_LENGTH_ERROR
    assert b"exceeds the static scratch limit of 64" in nb.cuda_lib().nut_last_error()


def test_static_head_rejects_pointer_not_aligned_to_its_element(gpu):
    f = _entry()
    dummy = ctypes.c_void_p(16)  # never dereferenced: the alignment check comes first
    odd = ctypes.c_void_p(18)
    status = f(dummy, dummy, odd, 1, 512, 288, None, dummy, None)
    assert status == nb.NUT_INVALID_ARGUMENT
    assert b"not aligned" in nb.cuda_lib().nut_last_error()
