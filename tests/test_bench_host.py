"""bench.py's SP parity machinery on CPU, at a reduced sequence length:
the global inputs do not depend on how a span is cut (so every SP degree
sees the same tensors), and the torch restatement of the reference's
quantised path that rank 0 runs equals the oracle — bit for bit on the Sage
paths, within one bf16 ulp on BF16 (fp64 vs fp32 softmax)."""
import numpy as np
import pytest
import torch

import bench
from oracle import attention as oa
from oracle import elementwise as ew
from oracle import fp8 as of
from oracle.numerics import bf16_round


@pytest.fixture
def small(monkeypatch):
    monkeypatch.setattr(bench, "SEQ", 900)
    monkeypatch.setattr(bench, "HEADS", 2)
    monkeypatch.setattr(bench, "WIDTH", 256)
    monkeypatch.setattr(bench, "INPUT_BLOCK", 128)


def test_global_rows_do_not_depend_on_the_split(small):
    dev = torch.device("cpu")
    whole = {w: bench.global_rows(w, 0, 912, dev) for w in "qkv"}
    assert not whole["q"][900:].any() and not whole["k"][900:].any()  # padding rows are zero
    for peers in (2, 3, 8):
        span = -(-912 // peers)
        for w in "qkv":
            parts = [bench.global_rows(w, r * span, min((r + 1) * span, 912), dev) for r in range(peers)]
            assert torch.equal(torch.cat(parts), whole[w])
    assert not torch.equal(whole["q"], whole["v"])


def _oracle_rows(prec, wire, cos, sin):
    dev = torch.device("cpu")
    q, k, v = (bench.global_rows(w, 0, 900, dev).float().numpy().reshape(1, 900, 2, 128) for w in "qkv")
    qr, kr = ew.partial_rope(q, k, cos.numpy(), sin.numpy())
    qh, kh, vh = (x.transpose(0, 2, 1, 3) for x in (qr, kr, v))
    rows = bench.parity_rows().numpy()

    def rt(x):
        w = of.wire_encode([x.reshape(-1, 128)], 1)
        return of.wire_decode(w, 1, x.size // 128, 1, 128)[0].reshape(x.shape)

    if wire == "fp8":
        qh, kh, vh = rt(qh), rt(kh), rt(vh)
    o = oa.sage_attention(qh, kh, vh, rows=rows) if prec == "sage" else oa.dense_attention(qh, kh, vh)[:, :, rows]
    o = bf16_round(o)
    pre = o.transpose(0, 2, 1, 3).reshape(len(rows), 256)
    if wire == "fp8":
        o = rt(o)
    return o.transpose(0, 2, 1, 3).reshape(len(rows), 256), pre


@pytest.mark.parametrize("prec,wire", [("sage", None), ("sage", "fp8"), ("bf16", None)])
def test_restatement_equals_oracle(small, prec, wire):
    from xgen_b200.h3.rope import rope_partial

    cos, sin = rope_partial(900, 128)
    ref, exact, pre = bench.reference_rows(prec, wire, torch.device("cpu"), cos, sin)
    want, want_pre = _oracle_rows(prec, wire, cos, sin)
    tol = 0.0 if prec == "sage" else 2.0 ** -8 * np.abs(want).max()
    assert np.abs(ref.numpy() - want).max() <= tol
    assert np.abs(pre.numpy() - want_pre).max() <= tol
    assert oa.cosine(exact.numpy(), want) > 0.99


def test_return_wire_is_per_row(small):
    x = torch.randn(64, 256).bfloat16().float()
    rt = bench._wire_round_trip(x.view(-1, 128)).view(64, 256)
    w = of.wire_encode([x.numpy().reshape(-1, 128)], 1)
    want = of.wire_decode(w, 1, 128, 1, 128)[0].reshape(64, 256)
    assert np.array_equal(rt.numpy(), want)


def test_launch_accounting():
    assert bench.kernels_per_step("sage", 1, 1) == 2
    assert bench.kernels_per_step("bf16", 1, 1) == 2
    assert bench.kernels_per_step("sage", 8, 1) == 5
    assert bench.kernels_per_step("sage", 8, 3) == 15
    assert bench.kernels_per_step("sage", 8, 1, "fp8", "peer") == 9
    assert bench.kernels_per_step("sage", 1, 1, "fp8", "peer") == 2
    assert bench.kernels_per_step("sage", 2, 1, "int8") == 6
    assert bench.kernels_per_step("bf16", 4, 2) == 3


def test_reference_arm_reports_the_b200_arm_config(monkeypatch, capsys):
    """The reference arm's JSON line carries the same workload config as the
    B200 arm's (the driver compares the two lines), with its CPU path named
    on its own key."""
    monkeypatch.setattr(bench, "cpu_attention_sample", lambda seconds, threads=None: (2.0, 1.0, 0.5, 4))
    monkeypatch.delenv("RANK", raising=False)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    monkeypatch.setattr("sys.argv", ["bench.py", "--impl", "reference", "--steps", "2", "--warmup", "1"])
    bench.main()
    import json

    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["config"] == bench.workload_config(1, "sage", "fp8")
    assert "reference_path" in line and line["value"] == 2.0


def test_trace_stage_times_are_differences_of_consecutive_marks():
    """xgen_b200.trace: each stage's time is the gap from the previous mark;
    repeated names add up; with no timeline open, mark() records nothing."""
    from xgen_b200 import trace

    class Ev:
        def __init__(self, t):
            self.t = t

        def elapsed_time(self, other):
            return other.t - self.t

    events = [("start", Ev(0.0)), ("gathered", Ev(1.5)), ("attended", Ev(11.5)), ("gathered", Ev(12.0))]
    assert trace.stage_ms(events) == {"gathered": 2.0, "attended": 10.0}
    assert trace.stop() == []
    trace.mark("start")  # no timeline open: no CUDA call, nothing kept
    assert trace.stop() == []
