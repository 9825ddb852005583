"""fp32 products of the reference's own kernel benches (matmul_threaded,
matvec_threaded, src/threading.cpp:163-198): the CUDA kernels follow the
reference build's arithmetic order, so results are compared bit for bit.

CPU: the oracle's restatement against the reference compiled here.
GPU: the CUDA kernels (through the C ABI) against the oracle.
"""
import numpy as np
import pytest

import oracle

SHAPES_MM = [(7, 13, 19), (64, 96, 80), (100, 1000, 33), (768, 768, 768)]
SHAPES_MV = [(4096, 4096), (1000, 77), (33, 64), (5, 4096), (40, 13), (40, 9), (40, 6)]


def _data(seed, *shape):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


def _same(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32),
                          np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.skipif(not oracle.reference_available(), reason="reference build missing")
@pytest.mark.parametrize("shape", SHAPES_MM[:3], ids=str)
def test_oracle_matmul_is_the_reference(orc, ref, shape):
    m, k, n = shape
    a, b = _data(1, m, k), _data(2, k, n)
    assert _same(orc.matmul_f32(a, b), ref.matmul_f32(a, b, threads=4))


@pytest.mark.skipif(not oracle.reference_available(), reason="reference build missing")
@pytest.mark.parametrize("shape", SHAPES_MV[1:], ids=str)
def test_oracle_matvec_is_the_reference(orc, ref, shape):
    w, x = _data(3, *shape), _data(4, shape[1])
    assert _same(orc.matvec_f32(w, x), ref.matvec_f32(w, x, threads=4))


@pytest.mark.gpu
@pytest.mark.parametrize("shape", SHAPES_MM, ids=str)
def test_cuda_matmul_bit_exact(gpu, orc, shape):
    import torch
    import nutllm_b200 as nb
    m, k, n = shape
    a, b = _data(1, m, k), _data(2, k, n)
    dev = torch.device("cuda", gpu)
    ad, bd = torch.from_numpy(a).to(dev), torch.from_numpy(b).to(dev)
    cd = torch.full((m, n), float("nan"), device=dev)
    nb.matmul_f32_async(ad.data_ptr(), bd.data_ptr(), cd.data_ptr(), m, k, n,
                        torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    assert _same(cd.cpu().numpy(), orc.matmul_f32(a, b))


@pytest.mark.gpu
@pytest.mark.parametrize("shape", SHAPES_MV, ids=str)
def test_cuda_matvec_bit_exact(gpu, orc, shape):
    import torch
    import nutllm_b200 as nb
    w, x = _data(3, *shape), _data(4, shape[1])
    dev = torch.device("cuda", gpu)
    wd, xd = torch.from_numpy(w).to(dev), torch.from_numpy(x).to(dev)
    yd = torch.full((shape[0],), float("nan"), device=dev)
    nb.matvec_f32_async(wd.data_ptr(), xd.data_ptr(), yd.data_ptr(), shape[0], shape[1],
                        torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    assert _same(yd.cpu().numpy(), orc.matvec_f32(w, x))
