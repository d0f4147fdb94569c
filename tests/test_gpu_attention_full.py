"""Full-size 768P-5s attention (126,754 tokens, BASELINE configs 2/3) on the
SP8 shard's 3 heads, checked on sampled query rows (the oracles cost
O(rows x S)) and through a size-independent property:

- Sage kernel vs the oracle's SageAttention2 restatement: cosine >= 0.999
  per head (the north-star Sage bound);
- BF16 kernel vs exact fp64 attention: cosine >= 0.9999 and max-abs <= 2e-2
  (the north-star BF16 bound);
- key permutation invariance of the BF16 kernel: permuting K and V rows
  together changes only the fp32 summation order (cosine >= 0.99999,
  max-abs <= 1e-2 over every row).

Inputs follow BASELINE config 2: Q, V ~ N(0,1), K ~ N(0,1) plus a per-head
channel bias of std 2, seeded."""
import numpy as np
import pytest
import torch

from oracle import attention as oa

pytestmark = pytest.mark.gpu

S, H = 126754, 3
ROWS = np.unique(np.concatenate([np.linspace(0, S - 1, 40).astype(int), [0, 1, 63, 64, S - 65, S - 1]]))


@pytest.fixture(scope="module")
def qkv():
    g = torch.Generator().manual_seed(768)
    q = torch.randn(1, H, S, 128, generator=g)
    k = torch.randn(1, H, S, 128, generator=g) + 2.0 * torch.randn(1, H, 1, 128, generator=g)
    v = torch.randn(1, H, S, 128, generator=g)
    return q.bfloat16(), k.bfloat16(), v.bfloat16()


def _np(t):
    return t.float().cpu().numpy()


def test_full_size_sage_vs_oracle(cuda_device, qkv):
    from xgen_b200.attention import kernel_errors, sage_attention

    q, k, v = qkv
    out = sage_attention(*(t.to(cuda_device) for t in (q, k, v)))
    torch.cuda.synchronize()
    assert kernel_errors() == 0
    got = _np(out[:, :, ROWS])
    want = oa.sage_attention(_np(q), _np(k), _np(v), rows=ROWS)
    for h in range(H):
        assert oa.cosine(got[:, h], want[:, h]) >= 0.999, h


def test_full_size_bf16_vs_exact(cuda_device, qkv):
    from xgen_b200.attention import dense_attention, kernel_errors

    q, k, v = (t.to(cuda_device) for t in qkv)
    out = dense_attention(q, k, v)
    torch.cuda.synchronize()
    assert kernel_errors() == 0
    rows = torch.from_numpy(ROWS).to(cuda_device)
    qs = q[:, :, rows].double()
    p = torch.softmax((qs @ k.double().transpose(-1, -2)) / np.sqrt(128.0), dim=-1)
    want = (p @ v.double()).float().cpu().numpy()
    got = _np(out[:, :, rows])
    for h in range(H):
        assert oa.cosine(got[:, h], want[:, h]) >= 0.9999, h
    assert np.abs(got - want).max() <= 2e-2


def test_full_size_key_permutation_invariance(cuda_device, qkv):
    from xgen_b200.attention import dense_attention

    q, k, v = (t.to(cuda_device) for t in qkv)
    perm = torch.randperm(S, generator=torch.Generator().manual_seed(5)).to(cuda_device)
    a = dense_attention(q, k, v).float()
    b = dense_attention(q, k[:, :, perm], v[:, :, perm]).float()
    cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
    assert cos >= 0.99999 and (a - b).abs().max().item() <= 1e-2, cos
