"""Benchmark: Ulysses-SP H3 self-attention at the 768P-5s shape on B200.

One step = one SP self-attention layer of the MiniMax-H3 DiT (BASELINE
config 2/3 shape: 31x48x84 video + 512 text + 1,250 audio = 126,754 tokens,
24 heads x 128): RoPE on Q/K, the seq->head redistribution, Sage-FP8 (or
BF16) attention on tcgen05, and the head->seq return, per rank on
S_loc = S_pad / N tokens. At N > 1 the redistribution is PHAA over NCCL with
the FP8 wire (RoPE fused into the encode, attention epilogue writing the
return send buffer). Inputs are synthetic (seeded N(0,1) Q/V, K with a
per-head channel bias of std 2), resident in HBM before timing and larger
than L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--precision sage|bf16]
    torchrun --nproc-per-node N bench.py --gpus N ...
    python bench.py --impl reference   # the reference's CPU attention path

Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from datetime import datetime, timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "SP attention TFLOP/s/GPU and DiT block ms at 768P-5s, 1/2/4/8 B200"
GRID = (31, 48, 84)
TEXT, AUDIO = 512, 1250
HEADS, HEAD_DIM = 24, 128
SEQ = GRID[0] * GRID[1] * GRID[2] + TEXT + AUDIO  # 126,754
FLOPS_PER_LAYER = 4.0 * SEQ * SEQ * HEAD_DIM * HEADS  # non-causal QK^T + PV


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--precision", choices=("sage", "bf16"), default="sage")
    # One head chunk: measured on B200 (768P-5s, Sage), a single FP8 exchange
    # per direction beats PHAA's chunked overlap at SP2 (71.7 vs 75.4 ms per
    # layer) and SP8 (19.3 vs 19.5 ms): the NCCL kernels overlapping the
    # one-CTA-per-SM attention kernel slow it more than they hide, and
    # chunks of 3 heads quantize to 10.05 waves of 148 SMs.
    ap.add_argument("--phaa-num", type=int, default=1)
    ap.add_argument("--wire", choices=("fp8", "int8"), default="fp8",
                    help="SP gather transport (Sage): the FP8 wire, or Sage-quantised INT8")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-block", action="store_true", help="skip the full DiT block timing")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--kernel-only", action="store_true",
                    help="time only the attention kernel on --seq/--heads (profiling case)")
    ap.add_argument("--seq", type=int, default=SEQ)
    ap.add_argument("--heads", type=int, default=HEADS)
    ap.add_argument("--linear-only", action="store_true",
                    help="time the FP8 Linear stack of one block (BASELINE config 4)")
    ap.add_argument("--sp", type=int, default=8, help="SP degree that sets the linear-stack M")
    ap.add_argument("--hbm-kernels", action="store_true",
                    help="time the HBM-bound kernels at one SP rank's shapes (--sp) against the measured HBM copy bandwidth")
    return ap.parse_args()


def linear_stack(args, dev=None, quiet=False):
    """the block's FP8 Linear stack (QKV hid->3*hid, O,
    FFN up hid->F, down F->hid) at M = ceil(126,754 / sp) tokens, per-token
    e4m3 activations and per-channel e4m3 weights; times each projection
    (activation quantisation + tcgen05 GEMM) with CUDA events."""
    import torch

    from xgen_b200.fp8_linear import H3FP8Linear

    dev = dev or torch.device("cuda", 0)
    hid, ffn = 3072, 12288
    m = -(-SEQ // max(1, args.sp))
    g = torch.Generator(device=dev).manual_seed(3)
    shapes = {"to_qkv": (3 * hid, hid), "to_out": (hid, hid), "ff_up": (ffn, hid), "ff_down": (hid, ffn)}
    res, total_flops, total_ms = {}, 0.0, 0.0
    for name, (n, k) in shapes.items():
        w = (torch.randn(n, k, device=dev, generator=g) * 0.02).bfloat16()
        layer = H3FP8Linear(w, torch.zeros(n, device=dev, dtype=torch.bfloat16), scaling="per_token")
        x = torch.randn(m, k, device=dev, generator=g).bfloat16()
        for _ in range(max(1, args.warmup)):
            layer(x)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.steps):
            layer(x)
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / args.steps
        flops = 2.0 * m * n * k
        res[name] = {"ms": ms, "tflops": flops / ms / 1e9}
        total_flops += flops
        total_ms += ms
    out = {"linear_stack": res, "m": m, "total_ms": total_ms, "tflops": total_flops / total_ms / 1e9}
    if not quiet:
        print(json.dumps(out), flush=True)
    return out


def kernel_only(args):
    """Prepare once, then run the attention kernel W + K times on a
    [1, heads, seq, 128] problem; prints its mean time (the ncu case)."""
    import torch

    from xgen_b200.attention import dense_attention, kernel_errors, sage_attention_prepared, sage_prepare

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    shape = (1, args.heads, args.seq, HEAD_DIM)
    q = torch.randn(shape, device=dev, generator=g).bfloat16()
    k = (torch.randn(shape, device=dev, generator=g) + 2 * torch.randn(1, args.heads, 1, HEAD_DIM, device=dev, generator=g)).bfloat16()
    v = torch.randn(shape, device=dev, generator=g).bfloat16()
    out = torch.empty_like(q)
    if args.precision == "sage":
        ws = sage_prepare(q, k, v)
        run = lambda: sage_attention_prepared(ws, out)  # noqa: E731
    else:
        run = lambda: dense_attention(q, k, v, out=out)  # noqa: E731
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        run()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    flops = 4.0 * args.seq * args.seq * HEAD_DIM * args.heads
    assert kernel_errors(dev) == 0
    print(json.dumps({"kernel": f"attention_{args.precision}", "seq": args.seq, "heads": args.heads,
                      "ms": ms, "tflops": flops / ms / 1e9}), flush=True)


def hbm_kernels(args):
    """The HBM-bound kernels of one SP rank at 768P-5s (--sp, default 8),
    each timed alone with CUDA events around every launch and a 512 MB
    write between launches, so no input is still in L2. Algorithmic bytes
    are each kernel's compulsory reads and writes (every input read once,
    every output written once); GB/s is compared with MEASURED_PEAKS.json's
    copy bandwidth. Prints one JSON line."""
    import torch

    from xgen_b200 import ops
    from xgen_b200.attention import SageWorkspace, kernel_errors, sage_prepare, sage_prepare_wire
    from xgen_b200.h3.rope import rope_3d
    from xgen_b200.phaa import fp8_transport as wire

    dev = torch.device("cuda", 0)
    sp = max(1, args.sp)
    s_pad = -(-SEQ // (16 * sp)) * (16 * sp)
    s_loc, hl, width = s_pad // sp, HEADS // sp, HEADS * HEAD_DIM
    m = -(-SEQ // sp)  # linear-stack rows
    hid, ffn = 3072, 12288
    g = torch.Generator(device=dev).manual_seed(11)
    rnd = lambda *shape: torch.randn(*shape, device=dev, generator=g).bfloat16()  # noqa: E731
    cos, sin = (t[:s_loc].contiguous().to(dev) for t in rope_3d(GRID, TEXT + AUDIO))
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)

    def timed(run):
        for _ in range(max(3, args.warmup)):
            run()
        total = 0.0
        for _ in range(max(1, args.steps)):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            run()
            e.record()
            torch.cuda.synchronize()
            total += s.elapsed_time(e)
        return total / max(1, args.steps)

    rows = {}

    def record(name, nbytes, ms, shape):
        rows[name] = {"ms": ms, "bytes": int(nbytes), "gbs": nbytes / ms / 1e6, "shape": shape}

    # PHAA FP8 wire: encode with fused RoPE (3 streams, 8 peers), decode
    # the [peer, S_loc, B, H_loc, D] views PHAA hands the codec (one head chunk)
    qkv = [rnd(1, s_loc, width).unflatten(-1, (HEADS, HEAD_DIM)).unflatten(2, (sp, hl)).permute(2, 1, 0, 3, 4)
           for _ in range(3)]
    payload = 3 * s_loc * HEADS * (HEAD_DIM + 4)
    buf = wire.encode(qkv, HEAD_DIM, sp, rotary_emb=(cos, sin))
    ms = timed(lambda: wire.encode(qkv, HEAD_DIM, sp, rotary_emb=(cos, sin), out=buf))
    record("fp8_wire_encode_rope", 3 * s_loc * width * 2 + 2 * cos.numel() * 4 + payload, ms,
           f"3 x [1, {s_loc}, {width}] bf16 -> {sp} peers")
    gathered = [torch.empty(sp, s_loc, 1, hl, HEAD_DIM, device=dev, dtype=torch.bfloat16) for _ in range(3)]
    ms = timed(lambda: wire.decode(buf, gathered, HEAD_DIM, sp))
    record("fp8_wire_decode", payload + 3 * s_loc * width * 2, ms, f"-> 3 x [{sp}, {s_loc}, 1, {hl}, 128] bf16")
    # the PHAA Sage path: Sage preparation reading the received wire itself
    ws_wire = SageWorkspace(1, hl, SEQ, dev)
    ms = timed(lambda: sage_prepare_wire(buf, peers=sp, seq=s_loc, batch=1, heads=hl, valid_seq=SEQ, ws=ws_wire))
    n = hl * SEQ * HEAD_DIM
    record("sage_prep_from_wire", payload + 3 * n + (2 * ws_wire.q_scale.numel() + ws_wire.v_scale.numel()) * 4,
           ms, f"wire of 3 x [{sp}, {s_loc}, 1, {hl}] rows -> Sage operands (replaces decode + sage_prep)")
    del qkv, buf, ws_wire

    # Sage preparation on the gathered layout (strided [B, H, S_real, D] views)
    views = [t.permute(2, 3, 0, 1, 4).flatten(2, 3)[:, :, :SEQ] for t in gathered]
    ws = SageWorkspace(1, hl, SEQ, dev)
    ms = timed(lambda: sage_prepare(*views, ws=ws))
    n = hl * SEQ * HEAD_DIM
    record("sage_prep", 3 * n * 2 + 3 * n + (2 * ws.q_scale.numel() + ws.v_scale.numel()) * 4, ms,
           f"3 x [1, {hl}, {SEQ}, 128] bf16 (gathered views)")
    del views, ws, gathered

    # standalone partial RoPE and Q/K RMSNorm + RoPE on [1, S_loc, H, D]
    q4, k4 = rnd(1, s_loc, HEADS, HEAD_DIM), rnd(1, s_loc, HEADS, HEAD_DIM)
    with torch.no_grad():
        ms = timed(lambda: ops.try_h3_partial_rope(q4, k4, cos, sin))
        record("partial_rope", 4 * q4.numel() * 2 + 2 * cos.numel() * 4, ms, f"2 x [1, {s_loc}, 24, 128] bf16")
        nq = torch.nn.RMSNorm(HEAD_DIM, eps=1e-6).to(dev, torch.bfloat16)
        nk = torch.nn.RMSNorm(HEAD_DIM, eps=1e-6).to(dev, torch.bfloat16)
        ms = timed(lambda: ops.try_h3_qk_rms(q4, k4, nq, nk, rotary_emb=(cos, sin)))
        record("qk_rms_rope", 4 * q4.numel() * 2 + 2 * cos.numel() * 4, ms, f"2 x [1, {s_loc}, 24, 128] bf16")
    del q4, k4

    # block elementwise: fused norm/modulate/quant, gated residual, FFN quant, SwiGLU
    x = rnd(1, m, hid)
    table = rnd(3, 6 * hid)
    idx = torch.randint(0, 3, (m,), device=dev, generator=g)
    ms = timed(lambda: ops.norm_modulate_quant(x, "layernorm", None, 1e-6, table[:, hid:2 * hid],
                                               table[:, :hid], idx))
    record("norm_modulate_quant", x.numel() * 2 + x.numel() + m * 4 + m * 8, ms, f"[1, {m}, {hid}] bf16 -> e4m3")
    res = rnd(1, m, hid)
    ms = timed(lambda: ops.indexed_affine(x, table[:, 2 * hid:3 * hid], res, idx, modulation=False))
    record("indexed_affine_gate", 3 * x.numel() * 2 + m * 8, ms, f"[1, {m}, {hid}] bf16")
    del x, res
    hmat = rnd(m, ffn)
    ms = timed(lambda: ops.quantize_per_token(hmat))
    record("fp8_quantize_per_token", hmat.numel() * 3 + m * 4, ms, f"[{m}, {ffn}] bf16 -> e4m3")
    del hmat
    up = rnd(m, 2 * ffn)
    ms = timed(lambda: ops.gate_first_swiglu(up))
    record("swiglu", up.numel() * 2 + up.numel(), ms, f"[{m}, {2 * ffn}] -> [{m}, {ffn}] bf16")
    del up
    torch.cuda.synchronize()
    assert kernel_errors(dev) == 0
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs", 6650.0)
    for r in rows.values():
        r["frac"] = r["gbs"] / peak
    print(json.dumps({"hbm_kernels": rows, "sp": sp, "peak_gbs": peak,
                      "peak_source": "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback 6650 GB/s",
                      "l2": "512 MB write between launches"}), flush=True)


# ------------------------------------------------------------------ helpers
def dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region.

    The sampler starts (and is waited for until its first sample) before the
    region; `mark_start()` / `mark_end()` bracket the region and only samples
    time-stamped inside it count. The interval is 20 ms, so even the ~90 ms
    regions of an 8-GPU run get several samples."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            deadline = time.time() + 5.0
            while time.time() < deadline and not Path(self.path).read_text().strip():
                time.sleep(0.02)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.05)  # let the sample covering the region's end land
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    @staticmethod
    def _when(stamp: str) -> float | None:
        try:
            return datetime.strptime(stamp.strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return None

    def summary(self):
        if self.proc is None or not self.path:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 10 and parts[2].isdigit():
                rows.append(parts)
        os.unlink(self.path)
        if self.t0 is not None and self.t1 is not None:
            inside = [r for r in rows if (w := self._when(r[0])) is not None
                      and self.t0 - 0.02 <= w <= self.t1 + 0.02]
            rows = inside or rows
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [int(r[2]) for r in rows]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[6:10]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": int(rows[0][3]),
                "power_w_max": max(float(r[4]) for r in rows if r[4].replace(".", "").isdigit()),
                "samples": len(rows), "reasons": reasons}


def cpu_attention_sample(seconds: float, threads: int | None = None):
    """The reference's CPU attention path (fp32 SDPA, x_base/x_base/operator/
    attention.py:29-34) on one head of the full 126,754-token sequence with a
    sample of query rows, sized to ~`seconds` of work; returns TFLOP/s."""
    import torch

    from oracle.attention import dense_attention  # the oracle port of that path

    if threads:
        torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    k = torch.randn(1, 1, SEQ, HEAD_DIM, generator=g).numpy()
    v = torch.randn(1, 1, SEQ, HEAD_DIM, generator=g).numpy()
    rows = 256
    total_flops, total_time = 0.0, 0.0
    while total_time < seconds:
        q = torch.randn(1, 1, rows, HEAD_DIM, generator=g).numpy()
        t0 = time.perf_counter()
        dense_attention(q, k, v)
        dt = time.perf_counter() - t0
        total_flops += 4.0 * rows * SEQ * HEAD_DIM
        total_time += dt
        if dt < seconds / 8:
            rows *= 2
    return total_flops / total_time / 1e12, total_flops, total_time, torch.get_num_threads()


# ------------------------------------------------------------------ reference arm
def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    import torch

    threads = os.cpu_count() or 1
    per_step = []
    for i in range(args.warmup + args.steps):
        tflops, flops, secs, used = cpu_attention_sample(max(2.0, args.cpu_seconds / 4), threads)
        if i >= args.warmup:
            per_step.append((tflops, flops, secs))
    value = statistics.median(t for t, _, _ in per_step)
    sample = (f"fp32 SDPA on CPU: 1 head, growing query-row samples x {SEQ} keys, "
              f"~{per_step[0][2]:.1f}s per step")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": FLOPS_PER_LAYER / (value * 1e12) * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(world, "reference-cpu"),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": used, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(world, precision, wire="fp8"):
    cfg = {"workload": "h3-sp-self-attention-768p5s", "seq_real": SEQ, "grid": list(GRID),
           "text_tokens": TEXT, "audio_tokens": AUDIO, "heads": HEADS, "head_dim": HEAD_DIM,
           "sp": world, "precision": precision, "parallelism": f"sp{world}",
           "l2": "inputs larger than L2 (3 x S_loc x 3072 bf16 per rank)"}
    if world > 1 and precision == "sage":
        cfg["wire"] = wire
    return cfg


# ------------------------------------------------------------------ B200 arm
def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.kernel_only:
        return kernel_only(args)
    if args.hbm_kernels:
        return hbm_kernels(args)
    if args.linear_only:
        return linear_stack(args)

    import torch
    import torch.distributed as dist

    from xgen_b200 import _lib
    from xgen_b200.attention import H3AttentionBackendB200, kernel_errors
    from xgen_b200.h3.rope import rope_3d
    from xgen_b200.h3.sp_attention import sp_self_attention
    from xgen_b200.sp.mesh import ParallelManager
    from xgen_b200.sp.padding import get_pad_manager

    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
        # the H3 enable_parallel mesh: every GPU of the job in one SP group
        group = ParallelManager(1, 1, world, 1).sp_group
    _lib.lib()

    # Workload: pad the packed sequence to a multiple of 16*SP.
    s_pad = -(-SEQ // (16 * world)) * (16 * world)
    s_loc = s_pad // world
    get_pad_manager()._pads["mmh3_seq"] = s_pad - SEQ
    cos_full, sin_full = rope_3d(GRID, TEXT + AUDIO)
    pad_rows = torch.zeros(s_pad - SEQ, HEAD_DIM)
    cos_full = torch.cat([cos_full, pad_rows + 1.0])
    sin_full = torch.cat([sin_full, pad_rows])
    cos = cos_full[rank * s_loc:(rank + 1) * s_loc].contiguous().to(dev)
    sin = sin_full[rank * s_loc:(rank + 1) * s_loc].contiguous().to(dev)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    width = HEADS * HEAD_DIM
    q = torch.randn(1, s_loc, width, device=dev, generator=g).bfloat16()
    k_bias = torch.randn(1, 1, width, device=dev, generator=torch.Generator(device=dev).manual_seed(7)) * 2.0
    k = (torch.randn(1, s_loc, width, device=dev, generator=g) + k_bias).bfloat16()
    v = torch.randn(1, s_loc, width, device=dev, generator=g).bfloat16()
    if world > 1 and rank == world - 1 and s_pad > SEQ:
        for t in (q, k, v):  # the tail padding rows are zeros, as split_sequence makes them
            t[:, s_loc - (s_pad - SEQ):].zero_()

    backend = H3AttentionBackendB200(args.precision)
    comm_stream = torch.cuda.Stream(device=dev) if world > 1 else None
    fp8_wire = args.precision == "sage"

    def step(qq, kk, vv):
        return sp_self_attention(qq, kk, vv, (cos, sin), backend=backend, heads=HEADS,
                                 head_dim=HEAD_DIM, sp_group=group, sp_size=world,
                                 phaa_num=min(args.phaa_num, HEADS // world),
                                 fp8_transport=fp8_wire, comm_stream=comm_stream,
                                 int8_transport=fp8_wire and args.wire == "int8")

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-resident timing
    for _ in range(args.warmup):
        out = step(q, k, v)
    barrier()
    launches_before = backend.kernel_calls
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        clocks.mark_start()
        start.record()
        for _ in range(args.steps):
            out = step(q, k, v)
        end.record()
        barrier()
        clocks.mark_end()
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    attn_calls = (backend.kernel_calls - launches_before) // args.steps
    assert kernel_errors(dev) == 0, "a tcgen05 kernel reported a timed-out wait"
    value = FLOPS_PER_LAYER / (ms * 1e-3) / 1e12  # aggregate over all ranks

    # ---- dominant kernel alone: the attention kernel on prepared inputs
    roof = attention_roofline(args.precision, world, dev, s_pad)

    # ---- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        e2e = end_to_end(step, q, k, v, args, world, dev, barrier, max_over_ranks)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tflops, flops, secs, used = cpu_attention_sample(args.cpu_seconds)
        cpu = {"value": tflops, "unit": "TFLOP/s", "cores": used, "kind": "port",
               "sample": f"fp32 SDPA (oracle port of attention.py:29-34) on 1 head: "
                         f"{flops / 4 / SEQ / HEAD_DIM:.0f} query rows x {SEQ} keys in {secs:.1f}s"}

    block = None
    if not args.no_block:
        block = block_timing(args, world, rank, dev, group, s_loc, cos, sin, comm_stream, barrier,
                             max_over_ranks)

    kernels_per_layer = kernels_per_step(args.precision, world, min(args.phaa_num, HEADS // world),
                                         args.wire)
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8/e4m3 (fp32 accumulate)" if args.precision == "sage" else "bf16",
        "data": "synthetic", "config": workload_config(world, args.precision, args.wire),
        "per_gpu_tflops": value / world, "attention_calls_per_step": attn_calls,
        "gpu_launches": kernels_per_layer * args.steps,
        "clocks": clocks.summary(), "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
        "block": block,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    del out
    if world > 1:
        dist.destroy_process_group()


def block_timing(args, world, rank, dev, group, s_loc, cos, sin, comm_stream, barrier,
                 max_over_ranks):
    """The metric's "DiT block ms": one full H3 DiT block (BASELINE config 4/5
    dimensions: hidden 3072, 24 x 128 heads, GELU FFN 12288, AdaLN LayerNorm
    from a cached random 6 x 3072 table per modality) at 768P-5s on this
    rank's S_loc tokens: fused norm/modulate/quant, FP8 QKV, SP attention
    (PHAA FP8 wire at N > 1), FP8 to_out + gated residual, FP8 FFN with the
    GELU epilogue and gated residual. Random-init weights N(0, 0.02)."""
    import torch

    from xgen_b200.h3.block import H3BlockConfig, H3DiTBlockB200

    cfg = H3BlockConfig(hidden=3072, heads=HEADS, head_dim=HEAD_DIM, ffn=12288,
                        activation="gelu", norm="layernorm", precision=args.precision)
    blk = H3DiTBlockB200(H3DiTBlockB200.random_weights(cfg, seed=0), cfg, dev)
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    x = torch.randn(1, s_loc, cfg.hidden, device=dev, generator=g).bfloat16()
    table = (0.1 * torch.randn(3, 6 * cfg.hidden, device=dev,
                               generator=torch.Generator(device=dev).manual_seed(5))).bfloat16()
    # modality tag per token (video 0, text 1, audio 2) of this rank's span
    tags = torch.zeros(SEQ + world * 16, dtype=torch.int64)
    video = GRID[0] * GRID[1] * GRID[2]
    tags[video:video + TEXT] = 1
    tags[video + TEXT:SEQ] = 2
    idx = tags[rank * s_loc:(rank + 1) * s_loc].to(dev)

    def run():
        return blk.forward(x, table, idx, (cos, sin), sp_group=group, sp_size=world,
                           phaa_num=min(args.phaa_num, HEADS // world),
                           fp8_transport=args.precision == "sage", comm_stream=comm_stream)

    for _ in range(max(3, args.warmup)):
        run()
    barrier()
    steps = max(2, min(args.steps, 5))
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        run()
    e.record()
    barrier()
    ms = max_over_ranks(s.elapsed_time(e) / steps)
    gemm_flops = blk.flops(s_loc, SEQ) * world
    total = gemm_flops + FLOPS_PER_LAYER
    return {"ms": ms, "steps": steps, "tflops_aggregate": total / ms / 1e9,
            "tflops_per_gpu": total / ms / 1e9 / world, "gemm_flops": gemm_flops,
            "attention_flops": FLOPS_PER_LAYER,
            "config": "hidden 3072, 24x128 heads, FFN 12288 GELU, AdaLN LayerNorm, FP8 per-token linears"}


def kernels_per_step(precision, world, phaa, wire="fp8"):
    """Our kernel launches per layer: SP=1: RoPE + (Sage: 3 prepare + 1 attention).
    SP>1 per PHAA chunk: QKV encode, decode, (Sage: 3 prepare) + attention,
    return encode, decode. INT8 wire (one chunk): stats, stats finalize,
    encode, attention, return encode, decode."""
    attn = 4 if precision == "sage" else 1
    if world == 1:
        return 1 + attn
    if precision == "sage" and wire == "int8":
        return 6
    per_chunk = attn + (4 if precision == "sage" else 0)
    return phaa * per_chunk + (1 if precision != "sage" else 0)


def attention_roofline(precision, world, dev, s_pad):
    """Time the attention kernel alone (CUDA events on its stream) on this
    rank's head shard of the full sequence; achieved = algorithmic FLOPs per
    launch / mean launch time; peak = in-run cuBLAS FP8 (or BF16) GEMM."""
    import torch

    from xgen_b200.attention import SageWorkspace, dense_attention, sage_attention_prepared, sage_prepare

    heads = HEADS // world
    g = torch.Generator(device=dev).manual_seed(99)
    q = torch.randn(1, heads, SEQ, HEAD_DIM, device=dev, generator=g).bfloat16()
    k = torch.randn(1, heads, SEQ, HEAD_DIM, device=dev, generator=g).bfloat16()
    v = torch.randn(1, heads, SEQ, HEAD_DIM, device=dev, generator=g).bfloat16()
    out = torch.empty_like(q)
    if precision == "sage":
        ws = sage_prepare(q, k, v)
        run = lambda: sage_attention_prepared(ws, out)  # noqa: E731
    else:
        run = lambda: dense_attention(q, k, v, out=out)  # noqa: E731
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    reps = 5
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        run()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / reps
    flops = 4.0 * SEQ * SEQ * HEAD_DIM * heads
    achieved = flops / (ms * 1e-3) / 1e12
    peak, peak_src = gemm_peak(dev, precision)
    traffic = profile_traffic(precision, heads)
    return {"bound": "tensor", "kernel": f"attention_kernel<{'sage' if precision == 'sage' else 'bf16'}>",
            "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_source": peak_src, "kernel_ms": ms, "flops_per_launch": flops,
            "traffic": traffic}


def gemm_peak(dev, precision):
    """Dense tensor peak measured in-run: torch._scaled_mm e4m3 8192^3 (cuBLASLt)
    for the Sage kernel, else MEASURED_PEAKS.json's bf16 burst figure."""
    import torch

    if precision != "sage":
        peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
        if "bf16_tflops" in peaks:
            return peaks["bf16_tflops"], "MEASURED_PEAKS.json bf16_tflops (burst, cuBLAS)"
        return 1590.0, "fallback 1.59 PFLOP/s bf16"
    n = 8192
    a = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn)
    b = torch.randn(n, n, device=dev).to(torch.float8_e4m3fn).t()
    one = torch.ones((), device=dev)
    for _ in range(3):
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch._scaled_mm(a, b, scale_a=one, scale_b=one, out_dtype=torch.bfloat16)
        e.record()
        torch.cuda.synchronize()
        best = min(best, s.elapsed_time(e))
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12, "in-run cuBLASLt e4m3 GEMM 8192^3, best of 10 (burst)"


def profile_traffic(precision, heads):
    """DRAM bytes per launch from the committed ncu summary, scaled to this
    launch's heads (traffic grows in proportion to heads at fixed S)."""
    path = ROOT / "profiles" / f"attention_{precision}_traffic.json"
    if not path.exists():
        return None
    rec = json.loads(path.read_text())
    return rec["dram_bytes_per_head"] * heads


def end_to_end(step, q, k, v, args, world, dev, barrier, max_over_ranks):
    """Same layer through the public API with pinned host buffers: every
    step's Q/K/V shard is copied host->device and its output device->host
    inside the timed region. The copies run on a side stream with two device
    buffer sets, so step i+1's upload and step i-1's download overlap step
    i's compute (the way a serving loop would feed the layer)."""
    import torch

    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    houts = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(2)]
    # the same step count as the device-timed value: the first upload and the
    # last download are the only copies not hidden under a step's compute
    steps = max(2, min(args.steps, 20))
    bufs = [tuple(torch.empty_like(t) for t in (q, k, v)) for _ in range(2)]
    cs = torch.cuda.current_stream(dev)
    xs = torch.cuda.Stream(device=dev)
    loaded = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        with torch.cuda.stream(xs):
            if i >= 2:
                xs.wait_event(computed[i % 2])  # step i-2 has finished reading this set
            for d, h in zip(bufs[i % 2], (hq, hk, hv)):
                d.copy_(h, non_blocking=True)
            loaded[i % 2].record(xs)

    def run(n):
        upload(0)
        for i in range(n):
            if i + 1 < n:
                upload(i + 1)
            cs.wait_event(loaded[i % 2])
            out = step(*bufs[i % 2])
            computed[i % 2].record(cs)
            with torch.cuda.stream(xs):
                xs.wait_event(computed[i % 2])
                houts[i % 2].copy_(out, non_blocking=True)
                out.record_stream(xs)
        cs.wait_stream(xs)

    run(2)
    barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(cs)
    xs.wait_event(s)
    run(steps)
    e.record(cs)
    barrier()
    ms = max_over_ranks(s.elapsed_time(e) / steps)
    hout = houts[0]
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv))
    d2h = hout.numel() * hout.element_size()
    return {"value": FLOPS_PER_LAYER / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps}


if __name__ == "__main__":
    main()
