"""CPU oracle for the xgen_b200 hot path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference (lightnateriver/xGen)
algorithms that the B200 kernels replace, so tests can check the CUDA path
against them. It is the checker, never the product: only `tests/`,
`__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg may import it,
and the `xgen_b200` package never does (its ops fail loudly when the CUDA
library is missing instead of falling back here).

Pinning. The elementwise restatements (RoPE, Q/K RMSNorm, indexed affine,
SwiGLU, FP8 wire codec, per-tensor FP8 quantisation) are checked bit-exactly
against golden fixtures produced by the reference's own Triton kernels
(tests/golden/make_golden.py). The PHAA layout restatement is checked
against the reference's run_phaa_attention on the same fixtures. The dense
attention oracle is fp32 scaled-dot-product attention, the reference's own
CPU path (x_base/x_base/operator/attention.py:29-34).

Parity unpinned: the Sage-style quantised attention. The reference calls the
third-party `sageattention` 2.2.0 (x_base/x_base/operator/attention.py:150,
363-375), which is neither vendored nor installed, and the reference's tests
mock it (x_base/tests/test_h3_sage_cuda.py:12-35), so no golden vector pins
its numerics. `oracle.attention.sage_attention` restates the published
SageAttention2 algorithm (Zhang et al., 2024: K mean-smoothing, per-block
INT8 Q/K, per-channel FP8 V, FP8 P, fp32 accumulation) with the block sizes
BASELINE config 3 names.
"""
