"""The phase-trace reader (nutllm_b200/trace.py) on a synthetic trace file
written in the kernel's format (CPU): header, record layout, critical path
per step and per-CTA sub-step cycles."""
import numpy as np
import pytest

from nutllm_b200 import trace

WORDS = 16


def _launch(ctas, tokens, layers, fill):
    stride = tokens * (3 * layers + 1)
    rec = np.zeros((ctas, stride, WORDS), np.uint64)
    fill(rec)
    hdr = np.array([ctas, stride, tokens, layers | (WORDS << 16)], np.int32)
    return hdr.tobytes() + rec.tobytes()


def _fill(rec):
    # one token, one layer: QKV, ATTWO, GUDOWN, LMHEAD; at 1000 MHz one
    # cycle is one ns.  CTA c enters occurrence k at 1000 k + 10 c ns and
    # stays 100 (c + 1) cycles: staged after 10, work 50, the rest finish.
    for c in range(rec.shape[0]):
        for k, ph in enumerate((0, 1, 2, 5)):
            clk0 = 5000 + 7 * c
            total = 100 * (c + 1)
            rec[c, k, 0] = ph
            rec[c, k, 1] = 1000 * k + 10 * c + 1
            rec[c, k, 6] = clk0
            rec[c, k, 2] = clk0 + 10
            rec[c, k, 5] = clk0 + 60
            rec[c, k, 7] = clk0 + total


def test_reader_critical_path_and_substeps(tmp_path):
    f = tmp_path / "trace.bin"
    f.write_bytes(_launch(2, 1, 1, _fill) * 2)  # two launches appended
    launches = trace.read(str(f))
    assert len(launches) == 2 and launches[0].ctas == 2 and launches[0].stride == 4
    st = trace.steps(launches[0], mhz=1000.0)
    assert [s["phase"] for s in st] == [0, 1, 2, 5]
    # last CTA out of step k: CTA 1 at 1000 k + 11 + 200 ns
    outs = [1000 * k + 11 + 200 for k in range(4)]
    assert st[0]["wall_ns"] == pytest.approx(outs[0] - 1)  # from the first entry
    for k in range(1, 4):
        assert st[k]["wall_ns"] == pytest.approx(outs[k] - outs[k - 1])
    assert st[0]["stage"] == 10 and st[0]["work"] == 50
    assert st[0]["finish"] == pytest.approx(np.median([40, 140]))
    summ = trace.summary(launches, mhz=1000.0)
    assert list(summ) == ["QKV", "ATTWO", "GUDOWN", "LMHEAD"]
    assert summ["ATTWO"]["steps"] == 2 and summ["ATTWO"]["wall_ns"] == pytest.approx(1000.0)


def test_reader_rejects_truncated_file(tmp_path):
    f = tmp_path / "trace.bin"
    f.write_bytes(_launch(2, 1, 1, _fill)[:-8])
    with pytest.raises(ValueError, match="truncated"):
        trace.read(str(f))


def test_reader_command_line(tmp_path, capsys):
    f = tmp_path / "trace.bin"
    f.write_bytes(_launch(2, 1, 1, _fill))
    assert trace.main([str(f), "--mhz", "1000"]) == 0
    out = capsys.readouterr().out
    assert "QKV" in out and "LMHEAD" in out and "1 launch(es), 2 CTAs" in out
