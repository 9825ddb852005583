"""The algorithmic byte counts behind bench.py's roofline line (CPU).

A batch-1 decode pass moves every quantised weight and fp16 scale once, the
embedding row, the norms, the KV history and, when it produces logits, the
fp32 classifier (the reference's decode_quantized_token plus the greedy
head, src/quant_model.cpp:158-206, src/generate.cpp:197-201).  Prompts of
GEMM_PREFILL_MIN tokens or more go through the GEMM prefill, so the
persistent launch then covers only the decode part of the generation."""
from nutllm_b200 import synthetic as syn


def test_tinyllama_int4_pass_bytes_match_the_stated_unit():
    wl = syn.WORKLOADS["tinyllama-int4"]
    c = wl.model_config()
    # 544,997,376 B of INT4 tiles and scales + 8,192 embedding row + 360,448
    # norms + 45,056 (pos + 1) of KV; + 262,152,192 with the classifier
    assert syn.algorithmic_decode_bytes(c, wl.qtype, 0, False) == (
        544_997_376 + 8_192 + 360_448 + 45_056)
    assert (syn.algorithmic_decode_bytes(c, wl.qtype, 0, True)
            - syn.algorithmic_decode_bytes(c, wl.qtype, 0, False)) == 262_144_000 + 8_192


def test_short_prompt_launch_is_the_whole_generation():
    wl = syn.WORKLOADS["tinyllama-int4"]
    c = wl.model_config()
    assert wl.prompt < syn.GEMM_PREFILL_MIN
    whole = syn.algorithmic_generation_bytes(c, wl.qtype, wl.prompt, wl.steps)
    assert syn.algorithmic_decode_launch_bytes(c, wl.qtype, wl.prompt, wl.steps) == whole
    assert whole == 15_657_529_344


def test_gemm_prefilled_prompt_counts_only_the_decode_part():
    wl = syn.WORKLOADS["tinyllama-int8-long"]
    c = wl.model_config()
    n, steps = wl.prompt, wl.steps
    assert n >= syn.GEMM_PREFILL_MIN
    launch = syn.algorithmic_decode_launch_bytes(c, wl.qtype, n, steps)
    whole = syn.algorithmic_generation_bytes(c, wl.qtype, n, steps)
    prompt_passes = sum(syn.algorithmic_decode_bytes(c, wl.qtype, pos, False)
                        for pos in range(n))
    # the whole generation less the prompt's passes (their classifier read
    # after the last prompt token stays: the first generated token needs it)
    assert launch == whole - prompt_passes
    # steps passes, steps classifier reads in all
    classifier = (syn.algorithmic_decode_bytes(c, wl.qtype, 0, True)
                  - syn.algorithmic_decode_bytes(c, wl.qtype, 0, False))
    passes = sum(syn.algorithmic_decode_bytes(c, wl.qtype, pos, False)
                 for pos in range(n, n + steps))
    assert launch == passes + steps * classifier
