"""Reader of the persistent decode kernel's phase trace.

Setting NUTLLM_TRACE_FILE makes every persistent launch append its trace to
that file: a header of four int32 (CTAs, records per CTA, tokens, layers |
words per record << 16), then one record of `words` uint64 per (CTA, phase
occurrence), CTA-major.  Every CTA opens the same sequence of occurrences:
per token, per layer the steps QKV (id 0), ATTWO (1) and GUDOWN (2), then
the classifier (5) when the token's logits are produced.  Record words:
0 phase id, 1 global timer at entry (ns), 6 SM clock at entry, 2 inputs
staged, 3 cycles warp 0 waited for weight stages, 4 digits ready, 5 weights
consumed, 7 exit, 8 finish red.adds issued, 9 finish fence passed, 11
gate/up consumed, 12 SwiGLU outputs complete, 13 key/value fence passed
(slots 2-13 in SM clock cycles; unused slots are 0).

    python -m nutllm_b200.trace FILE [--mhz 1965]

prints, per phase, the median critical path of a step (the last CTA out of
the step after the previous step's last CTA out; exits placed on the global
timer through the SM clock) and the median per-CTA cycles of its sub-steps.
"""
from __future__ import annotations

import argparse
import sys
from dataclasses import dataclass

import numpy as np

PHASES = {0: "QKV", 1: "ATTWO", 2: "GUDOWN", 5: "LMHEAD"}


@dataclass
class Launch:
    ctas: int
    stride: int
    tokens: int
    layers: int
    rec: np.ndarray  # [ctas][stride][words] uint64


def read(path: str) -> list[Launch]:
    """Every launch appended to the trace file."""
    raw = open(path, "rb").read()
    out, off = [], 0
    while off + 16 <= len(raw):
        ctas, stride, tokens, lw = np.frombuffer(raw, np.int32, 4, off)
        layers, words = int(lw) & 0xFFFF, int(lw) >> 16
        n = int(ctas) * int(stride) * words
        off += 16
        if ctas <= 0 or stride <= 0 or words <= 0 or off + 8 * n > len(raw):
            raise ValueError(f"trace: truncated or malformed launch at byte {off - 16}")
        rec = np.frombuffer(raw, np.uint64, n, off).reshape(int(ctas), int(stride), words)
        out.append(Launch(int(ctas), int(stride), int(tokens), layers, rec))
        off += 8 * n
    if off != len(raw):
        raise ValueError(f"trace: {len(raw) - off} trailing bytes")
    return out


def steps(launch: Launch, mhz: float) -> list[dict]:
    """Per occurrence: phase, the critical path (ns) and the per-CTA
    sub-step cycles (medians over CTAs that did work in it)."""
    r = launch.rec.astype(np.int64)
    used = r[:, :, 1].max(axis=0) > 0  # occurrences some CTA opened
    result, prev_out = [], None
    for k in np.nonzero(used)[0]:
        e = r[:, k, :]
        live = e[:, 1] > 0
        entry_ns = e[live, 1]
        exit_ns = entry_ns + (e[live, 7] - e[live, 6]) * 1e3 / mhz
        last_out = float(exit_ns.max())
        first_in = float(entry_ns.min())
        wall = last_out - (prev_out if prev_out is not None else first_in)
        prev_out = last_out
        phase = int(np.bincount(e[live, 0].astype(np.int64)).argmax())
        cyc = e[live]

        def span(a, b):
            ok = (cyc[:, a] > 0) & (cyc[:, b] >= cyc[:, a])
            return float(np.median(cyc[ok, b] - cyc[ok, a])) if ok.any() else None

        result.append({"occurrence": int(k), "phase": phase, "wall_ns": wall,
                       "stage": span(6, 2), "work": span(2, 5), "finish": span(5, 7),
                       "total": span(6, 7)})
    return result


def summary(launches: list[Launch], mhz: float) -> dict[str, dict]:
    """Medians per phase over every occurrence of every launch."""
    acc: dict[int, dict[str, list]] = {}
    for ln in launches:
        for s in steps(ln, mhz):
            d = acc.setdefault(s["phase"], {"wall_ns": [], "stage": [], "work": [],
                                             "finish": [], "total": []})
            for key in d:
                if s[key] is not None:
                    d[key].append(s[key])
    out = {}
    for ph, d in sorted(acc.items()):
        out[PHASES.get(ph, str(ph))] = {
            "steps": len(d["wall_ns"]),
            **{key: (float(np.median(v)) if v else None) for key, v in d.items()}}
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("file")
    ap.add_argument("--mhz", type=float, default=1965.0,
                    help="SM clock used to place exits on the global timer")
    a = ap.parse_args(argv)
    launches = read(a.file)
    print(f"{len(launches)} launch(es), {launches[0].ctas} CTAs" if launches else "empty")
    print(f"{'phase':8s} {'steps':>6s} {'critical path us':>17s} {'stage cyc':>10s} "
          f"{'work cyc':>9s} {'finish cyc':>11s} {'CTA total cyc':>14s}")
    for name, d in summary(launches, a.mhz).items():
        def f(v, scale=1.0):
            return "-" if v is None else f"{v * scale:.1f}"
        print(f"{name:8s} {d['steps']:6d} {f(d['wall_ns'], 1e-3):>17s} {f(d['stage']):>10s} "
              f"{f(d['work']):>9s} {f(d['finish']):>11s} {f(d['total']):>14s}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
