"""The prefill GEMM (nut_qmatrix_gemm) on the tensor cores.

Y[tokens][rows] = X[tokens][cols] Q^T with fp16 operands and fp32
accumulation.  Rounding both operands to fp16 perturbs each product by a
relative 2^-11 + 2^-11 at most (plus fp32 accumulation, far smaller; the
activations here are N(0, 1), so fp16's subnormal range only adds an
absolute error far below 1e-6), so every element must satisfy
|y - exact| <= 2^-10 sum_k |x_k w_k| + 1e-6; "exact" is the float64
product of X and the exactly dequantised weights (q * scale).
"""
import numpy as np
import pytest

import nutllm_b200 as nb

pytestmark = pytest.mark.gpu

SEED = 1234


def dequantize(q: nb.QuantizedMatrix) -> np.ndarray:
    n = q.rows * q.cols
    if q.qtype == nb.INT8:
        vals = q.data.view(np.int8)[:n].astype(np.float64)
    else:
        b = q.data.astype(np.int16)
        nib = np.empty(2 * b.size, np.int16)
        nib[0::2] = b & 0xF
        nib[1::2] = b >> 4
        nib = nib[:n]
        vals = np.where(nib >= 8, nib - 16, nib).astype(np.float64)
    s = q.scales.view(np.float16).astype(np.float64)
    return (vals * np.repeat(s, 32)[:n]).reshape(q.rows, q.cols)


def run_gemm(gpu, rows, cols, tokens, qtype):
    import torch
    w = nb.synth_normal(SEED, 7, rows * cols, 0.02).reshape(rows, cols)
    q = nb.QuantizedMatrix.quantize(w, qtype)
    x = nb.synth_normal(SEED, 9, tokens * cols, 1.0).reshape(tokens, cols)
    dev = torch.device("cuda", gpu)
    m = nb.DeviceQMatrix(q, gpu)
    xd = torch.from_numpy(x).to(dev)
    yd = torch.full((tokens, rows), float("nan"), device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    for _ in range(2):  # the second call reuses the cached fp16 weights
        m.gemm_async(xd.data_ptr(), tokens, yd.data_ptr(), stream)
    torch.cuda.synchronize(dev)
    m.check()
    wd = dequantize(q)
    exact = x.astype(np.float64) @ wd.T
    bound = 2.0 ** -10 * (np.abs(x).astype(np.float64) @ np.abs(wd).T) + 1e-6
    return yd.cpu().numpy().astype(np.float64), exact, bound


SHAPES = [(2048, 2048, 512), (5632, 2048, 512), (2048, 5632, 512)]


@pytest.mark.parametrize("qtype", [nb.INT4, nb.INT8], ids=["int4", "int8"])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: f"{s[0]}x{s[1]}xM{s[2]}")
def test_gemm_within_f16_bound(gpu, qtype, shape):
    y, exact, bound = run_gemm(gpu, *shape, qtype)
    err = np.abs(y - exact)
    assert np.all(np.isfinite(y))
    assert np.all(err <= bound), f"max excess {float((err - bound).max()):.3e}"


@pytest.mark.parametrize("shape", [(1000, 64, 200), (2100, 96, 129), (128, 2048, 1),
                                   (32000, 2048, 64)],
                         ids=lambda s: f"{s[0]}x{s[1]}xM{s[2]}")
def test_gemm_edge_shapes(gpu, shape):
    """Partial output tiles in both dimensions, a single token, K = 64."""
    y, exact, bound = run_gemm(gpu, *shape, nb.INT4)
    assert np.all(np.abs(y - exact) <= bound)


@pytest.mark.parametrize("shape", [(32000, 2048, 512), (20000, 2048, 300)],
                         ids=lambda s: f"{s[0]}x{s[1]}xM{s[2]}")
def test_gemm_sm_pairs(gpu, shape):
    """Several waves of 256-column tiles with more than 128 tokens: the
    SM-pair form (256 x 256 tiles over two CTAs).  The second shape has a
    partial 256-row tile (rows 256..299 of 512) and a partial last column
    tile (20000 = 78 x 256 + 32)."""
    y, exact, bound = run_gemm(gpu, *shape, nb.INT4)
    assert np.all(np.isfinite(y))
    err = np.abs(y - exact)
    assert np.all(err <= bound), f"max excess {float((err - bound).max()):.3e}"
