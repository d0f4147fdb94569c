"""numpy restatements of the reference's FP8 formats (test infrastructure).

- PHAA wire codec: x_base/x_base/phaa/fp8_transport.py:26-144
- per-tensor activation/weight quantisation: x_base/x_base/operator/h3_fp8.py:9-12,
  h3_fp8_quant.py:9-25 (bit-identical to each other by the reference's test
  x_base/tests/test_h3_cuda_precision_ops.py:51-58)
- per-token activation quantisation (the B200 FP8 Linear's target scheme)
- FP8 linear forward as torch._scaled_mm computes it: fp32 accumulation of
  exact e4m3 products, times both scales, plus bias, rounded once to bf16.
"""
from __future__ import annotations

import numpy as np

from .numerics import (E4M3_MAX, FLT_MIN, bf16_round, e4m3_from_f32, e4m3_to_f32, fdiv,
                       f16_round)

f32 = np.float32


def row_scale(x: np.ndarray) -> np.ndarray:
    """Wire scale of each row (last axis): max(max|x|/448, 1e-12)."""
    amax = np.abs(x.astype(f32)).max(axis=-1)
    return np.maximum(fdiv(amax, f32(448.0)), f32(1.0e-12)).astype(f32)


def wire_encode(sources, peers: int, peer_padding: int = 0) -> np.ndarray:
    """Encode 1 or 3 tensors whose flattened rows (last axis = width) are in
    [peer, seq, batch, head] order into the PHAA byte wire."""
    streams = len(sources)
    width = sources[0].shape[-1]
    rows = [s.reshape(-1, width).astype(f32) for s in sources]
    nrows = rows[0].shape[0]
    peer_rows = nrows // peers
    row_bytes = width + 4
    packet = peer_rows * streams * row_bytes
    wire = np.zeros(peers * (packet + peer_padding), dtype=np.uint8)
    for p in range(peers):
        base = p * (packet + peer_padding)
        for slot, r in enumerate(rows):
            block = r[p * peer_rows:(p + 1) * peer_rows]
            scale = row_scale(block)
            codes = e4m3_from_f32(np.clip(fdiv(block, scale[:, None]), -E4M3_MAX, E4M3_MAX))
            seg = np.zeros((peer_rows, row_bytes), dtype=np.uint8)
            seg[:, :width] = codes
            seg[:, width:] = scale.view(np.uint8).reshape(peer_rows, 4)
            start = base + slot * peer_rows * row_bytes
            wire[start:start + peer_rows * row_bytes] = seg.reshape(-1)
    return wire


def wire_decode(wire: np.ndarray, streams: int, rows: int, peers: int, width: int,
                peer_padding: int = 0, out_round=bf16_round):
    """Inverse of wire_encode: list of `streams` arrays [rows, width] holding
    e4m3 * scale rounded to the output dtype."""
    peer_rows = rows // peers
    row_bytes = width + 4
    packet = peer_rows * streams * row_bytes
    outs = [np.empty((rows, width), dtype=f32) for _ in range(streams)]
    for p in range(peers):
        base = p * (packet + peer_padding)
        for slot in range(streams):
            start = base + slot * peer_rows * row_bytes
            seg = wire[start:start + peer_rows * row_bytes].reshape(peer_rows, row_bytes)
            scale = np.ascontiguousarray(seg[:, width:]).view(f32).reshape(peer_rows)
            vals = e4m3_to_f32(seg[:, :width]) * scale[:, None]
            outs[slot][p * peer_rows:(p + 1) * peer_rows] = out_round(vals.astype(f32))
    return outs


def peer_padding(peer_rows: int, streams: int, width: int) -> int:
    """Align16 padding of one peer packet (fp8_transport.py:103-105)."""
    return (-(peer_rows * streams * (width + 4))) % 16


def quantize_per_tensor(x: np.ndarray, scalar_div: str = "cuda"):
    """scale = max(amax/448, FLT_MIN); codes = e4m3(clamp(x/scale, +-448)).

    `amax / 448.0` is a torch tensor-by-Python-scalar division. On CUDA
    tensors torch computes it as amax * fp32(1/448) (the divisor becomes a
    reciprocal multiply); on CPU tensors as an IEEE division. The reference
    runs on CUDA, so "cuda" is the default; "ieee" reproduces a CPU run."""
    x = x.astype(f32)
    amax = f32(np.abs(x).max()) if x.size else f32(0.0)
    if scalar_div == "cuda":
        raw = f32(amax * (f32(1.0) / f32(448.0)))
    else:
        raw = fdiv(amax, f32(448.0))
    scale = f32(max(raw, FLT_MIN))
    codes = e4m3_from_f32(np.clip(fdiv(x, scale), -E4M3_MAX, E4M3_MAX))
    return codes, scale


def quantize_per_token(x: np.ndarray):
    """Per-row dynamic e4m3 of x [rows, cols]: (codes, scales[rows])."""
    x = x.astype(f32)
    amax = np.abs(x).max(axis=-1)
    scales = np.maximum(fdiv(amax, f32(448.0)), FLT_MIN).astype(f32)
    codes = e4m3_from_f32(np.clip(fdiv(x, scales[:, None]), -E4M3_MAX, E4M3_MAX))
    return codes, scales


def quantize_weight_per_channel(w: np.ndarray):
    """Per-output-channel e4m3 of w [out, in]: (codes, scales[out])."""
    return quantize_per_token(w)


def scaled_mm(a_codes, b_codes, scale_a, scale_b, bias=None, out_round=bf16_round):
    """torch._scaled_mm(A, B^T): fp32 sum of exact e4m3 products times
    scale_a (per-tensor scalar or per-row [M]) and scale_b (scalar or per
    output channel [N]), plus bias, rounded to the output dtype once.
    a_codes [M, K], b_codes [N, K] (the weight as stored, [out, in])."""
    a = e4m3_to_f32(a_codes).astype(np.float64)
    b = e4m3_to_f32(b_codes).astype(np.float64)
    acc = (a @ b.T).astype(f32)  # exact products; fp64 sum stands in for fp32 accumulation
    sa = np.asarray(scale_a, dtype=f32).reshape(-1, 1) if np.ndim(scale_a) else f32(scale_a)
    sb = np.asarray(scale_b, dtype=f32).reshape(1, -1) if np.ndim(scale_b) else f32(scale_b)
    out = (acc * sa * sb).astype(f32)
    if bias is not None:
        out = out + bias.astype(f32)[None, :]
    return out_round(out.astype(f32))


__all__ = ["row_scale", "wire_encode", "wire_decode", "peer_padding", "quantize_per_tensor",
           "quantize_per_token", "quantize_weight_per_channel", "scaled_mm", "f16_round"]
