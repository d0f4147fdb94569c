"""CPU attention oracles (test infrastructure only).

dense_attention: fp32 scaled-dot-product attention — the reference's own
CPU path `base_attention_infer` (x_base/x_base/operator/attention.py:29-34).

sage_attention: a restatement of the Sage-style quantised attention the
reference reaches through the third-party `sageattention` 2.2.0 package
(call site x_base/x_base/operator/attention.py:150,363-375; package pinned
in docs/H3-SHARED-TP-CP.md:77, not vendored, not installed). Parity with the
package itself is unpinned; this follows the published SageAttention2
algorithm (Zhang et al., 2024) with BASELINE config 3's granularity:

  K~ = K - mean_tokens(K)                     (per head, per channel)
  Q~ = Q * sm_scale * log2(e)
  int8 per 64-token block: s = amax/127, x8 = rint(x / s)   (Q~ and K~)
  V  per channel e4m3: sv = max(amax_tokens|V|/448, FLT_MIN), v8 = e4m3(V/sv)
  S  = (q8 . k8^T) * s_q[blk] * s_k[blk]      (log2 domain, exact int32 sum)
  P  = exp2(S - rowmax(S)), l = sum(P)        (fp32)
  O  = (e4m3(P*448) . v8) * sv / (448 * l)     (fp32 accumulation)
"""
from __future__ import annotations

import math

import numpy as np

from .numerics import FLT_MIN, e4m3_from_f32, e4m3_to_f32, fdiv

f32 = np.float32
LOG2E = f32(1.4426950408889634)


def dense_attention(q, k, v, sm_scale=None):
    """fp32 SDPA of [B, H, S, D] arrays (numpy in, numpy out)."""
    import torch
    import torch.nn.functional as F

    t = [torch.from_numpy(np.ascontiguousarray(x, dtype=f32)) for x in (q, k, v)]
    return F.scaled_dot_product_attention(*t, scale=sm_scale).numpy()


def _block_int8(x: np.ndarray, block: int = 64):
    """x [..., S, D] fp32 -> (int8 codes, scales [..., ceil(S/block)])."""
    s, d = x.shape[-2:]
    nb = (s + block - 1) // block
    pad = nb * block - s
    xp = np.concatenate([x, np.zeros((*x.shape[:-2], pad, d), f32)], axis=-2) if pad else x
    xb = xp.reshape(*x.shape[:-2], nb, block, d)
    amax = np.abs(xb).max(axis=(-2, -1))
    scale = np.where(amax > 0, fdiv(amax, f32(127.0)), f32(1.0)).astype(f32)
    codes = np.clip(np.rint(fdiv(xb, scale[..., None, None])), -127, 127).astype(np.int8)
    return codes.reshape(*x.shape[:-2], nb * block, d)[..., :s, :], scale


def sage_quantize(q, k, v, sm_scale=None, block: int = 64):
    """Quantise fp32 [B, H, S, D] Q/K/V as the Sage prepare step does."""
    d = q.shape[-1]
    sm_scale = f32(sm_scale if sm_scale is not None else 1.0 / math.sqrt(d))
    qs_in = (q.astype(f32) * f32(sm_scale * LOG2E)).astype(f32)
    kmean = k.astype(np.float64).mean(axis=-2, keepdims=True).astype(f32)
    ks_in = (k.astype(f32) - kmean).astype(f32)
    q8, sq = _block_int8(qs_in, block)
    k8, sk = _block_int8(ks_in, block)
    vmax = np.abs(v.astype(f32)).max(axis=-2)
    sv = np.maximum(fdiv(vmax, f32(448.0)), FLT_MIN).astype(f32)
    v8 = e4m3_from_f32(fdiv(v.astype(f32), sv[..., None, :]))
    return dict(q8=q8, q_scale=sq, k8=k8, k_scale=sk, v8=v8, v_scale=sv, k_mean=kmean)


def sage_attention(q, k, v, sm_scale=None, rows=None, block: int = 64, quant=None):
    """Quantised attention output [B, H, len(rows) or S, D] (fp32).

    `rows` selects query rows (the oracle then costs O(len(rows) * S)), so
    full-length sequences can be checked on a sample of rows."""
    qd = quant or sage_quantize(q, k, v, sm_scale, block)
    b, h, s, d = q.shape
    rows = np.arange(s) if rows is None else np.asarray(rows)
    out = np.empty((b, h, len(rows), d), f32)
    kb = np.arange(s) // block
    for bi in range(b):
        for hi in range(h):
            q8 = qd["q8"][bi, hi, rows].astype(np.float64)
            k8 = qd["k8"][bi, hi].astype(np.float64)
            sc = (q8 @ k8.T).astype(f32)  # exact int32 sums
            sc = sc * qd["q_scale"][bi, hi, rows // block][:, None] * qd["k_scale"][bi, hi, kb][None, :]
            m = sc.max(axis=-1, keepdims=True)
            p = np.exp2((sc - m).astype(f32)).astype(f32)
            l = p.sum(axis=-1, dtype=np.float64).astype(f32)
            p8 = e4m3_to_f32(e4m3_from_f32(p * f32(448.0))).astype(np.float64)
            v8 = e4m3_to_f32(qd["v8"][bi, hi]).astype(np.float64)
            o = (p8 @ v8).astype(f32) * qd["v_scale"][bi, hi][None, :] / (f32(448.0) * l[:, None])
            out[bi, hi] = o.astype(f32)
    return out


def cosine(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))
