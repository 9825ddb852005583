"""Generates the golden vectors in this directory from the unmodified
reference (oracle/_ref/libnutref.so, built from the reference sources by
oracle/Makefile).  Run from the repository root:

    make -C oracle ref REF=<reference source tree> && python tests/golden/make_golden.py

quant_golden.npz   seeded and edge-case fp32 matrices with the reference
                   quantiser's bytes, fp16 scales, dequantised values,
                   error bounds and storage size (QuantizedMatrix::quantize,
                   src/quant.cpp:154-197).
qmatvec_golden.npz quantised matvec outputs of the reference
                   (matvec_quantized_threaded, src/quant.cpp:262-321).
tiny_int8_golden.npz  the reference token loop on the seeded tiny INT8 model:
                   prompt, 16 greedy ids, their logits, the prefill hidden.
tinyllama_int4_golden.npz  the same loop at TinyLlama shape (INT4): ids and
                   the top-8 logits of every step.
tinyllama_int8_long_golden.npz  BASELINE config 3 at its stated size:
                   TinyLlama shape INT8, a 512-token prompt and 256 greedy
                   steps (KV cache at 768 positions): ids, the top-16 logits
                   of every step and the whole logit rows of five steps.
                   Written alone by `python tests/golden/make_golden.py long`.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from nutllm_b200 import synthetic as syn  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
SEED = 1234


def quant_cases():
    rng = np.random.default_rng(505)
    cases = {
        "uniform_5x37": rng.uniform(-1, 1, (5, 37)),
        "uniform_7x64": rng.uniform(-1, 1, (7, 64)),
        "zeros_1x33": np.zeros((1, 33)),
        "kat_1x4": np.array([[-7.0, -1.0, 2.0, 7.0]]),
        "normal_16x96": rng.normal(0, 0.02, (16, 96)),
        "tiny_values_3x64": rng.normal(0, 1e-6, (3, 64)),
        "subnormal_scales_2x32": rng.normal(0, 1e-9, (2, 32)),
        "large_values_2x64": rng.uniform(-4.0e5, 4.0e5, (2, 64)),
        "ties_1x32": np.array([[7.0] + [0.5 * k for k in range(-15, 16)]]),
        "single_1x1": np.array([[0.3]]),
    }
    return {k: v.astype(np.float32) for k, v in cases.items()}


def main():
    ref = oracle.Reference()
    out = {}
    for name, w in quant_cases().items():
        for qt, tname in ((0, "int8"), (1, "int4")):
            data, scales = ref.quantize(w, qt)
            values, bounds, nbytes = ref.quantized_values(w, qt)
            key = f"{name}_{tname}"
            out[f"{key}_input"] = w
            out[f"{key}_data"] = data
            out[f"{key}_scales"] = scales
            out[f"{key}_values"] = values
            out[f"{key}_bounds"] = bounds
            out[f"{key}_storage"] = np.array([nbytes])
    np.savez_compressed(os.path.join(OUT, "quant_golden.npz"), **out)

    import nutllm_b200 as nb
    mv = {}
    for rows, cols in [(48, 2048), (33, 5632), (7, 64), (5, 37)]:
        w = nb.synth_normal(SEED, 21, rows * cols, 0.02).reshape(rows, cols)
        x = nb.synth_normal(SEED, 22, cols, 1.0)
        for qt, tname in ((0, "int8"), (1, "int4")):
            data, scales = ref.quantize(w, qt)
            key = f"{rows}x{cols}_{tname}"
            mv[f"{key}_data"] = data
            mv[f"{key}_scales"] = scales
            mv[f"{key}_x"] = x
            mv[f"{key}_y"] = ref.qmatvec(qt, rows, cols, data, scales, x, threads=1)
    np.savez_compressed(os.path.join(OUT, "qmatvec_golden.npz"), **mv)

    wl = syn.WORKLOADS["tiny-int8"]
    c = wl.model_config()
    rm = ref.model(c, wl.qtype, SEED)
    prompt = syn.prompt_ids(c, SEED, wl.prompt)
    ids, logits, hidden, _, _ = rm.generate(prompt, wl.steps, threads=1)
    w = syn.build_model(c, wl.qtype, SEED)
    digest = np.array([int(np.bitwise_xor.reduce(np.concatenate(
        [m.data for layer in w.layers for m in layer.projections()]).view(np.uint8)))])
    np.savez_compressed(os.path.join(OUT, "tiny_int8_golden.npz"), prompt=prompt, ids=ids,
                        logits=logits, prefill_hidden=hidden,
                        storage=np.array([rm.storage_bytes()]), byte_xor=digest)

    wl = syn.WORKLOADS["tinyllama-int4"]
    c = wl.model_config()
    rm = ref.model(c, wl.qtype, SEED)
    prompt = syn.prompt_ids(c, SEED, wl.prompt)
    ids, logits, hidden, _, _ = rm.generate(prompt, wl.steps, threads=os.cpu_count())
    top = np.argsort(-logits, axis=1, kind="stable")[:, :8]
    np.savez_compressed(os.path.join(OUT, "tinyllama_int4_golden.npz"), prompt=prompt,
                        ids=ids, top_ids=top.astype(np.int32),
                        top_logits=np.take_along_axis(logits, top, axis=1),
                        prefill_hidden=hidden, storage=np.array([rm.storage_bytes()]))
    print("golden vectors written to", OUT)


LONG_FULL_STEPS = (0, 64, 128, 192, 255)


def long_golden(ref=None):
    """BASELINE config 3 through the reference's own loop (all host threads):
    prefill_quantized of 512 tokens, then 256 greedy steps."""
    ref = ref or oracle.Reference()
    wl = syn.WORKLOADS["tinyllama-int8-long"]
    c = wl.model_config()
    rm = ref.model(c, wl.qtype, SEED)
    prompt = syn.prompt_ids(c, SEED, wl.prompt)
    ids, logits, hidden, _, _ = rm.generate(prompt, wl.steps, threads=os.cpu_count())
    top = np.argsort(-logits, axis=1, kind="stable")[:, :16]
    np.savez_compressed(os.path.join(OUT, "tinyllama_int8_long_golden.npz"), prompt=prompt,
                        ids=ids, top_ids=top.astype(np.int32),
                        top_logits=np.take_along_axis(logits, top, axis=1),
                        full_steps=np.array(LONG_FULL_STEPS, np.int32),
                        full_logits=logits[list(LONG_FULL_STEPS)],
                        prefill_hidden=hidden)
    print("long golden written to", OUT)


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "long":
        long_golden()
    else:
        main()
        long_golden()
