"""SP=2 over NCCL on two GPUs: the PHAA FP8-wire path (RoPE fused into the
encode, Sage attention, FP8 return) equals the same kernels run on one GPU.

Every wire operation is per row (one head of one token), so the SP=2 result
must match, bit for bit, a single-GPU pass that RoPEs, FP8-round-trips
Q/K/V, runs Sage attention over the full sequence and FP8-round-trips the
output. Skips when fewer than two GPUs are visible."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

HEADS, D = 4, 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(s):
    from xgen_b200.h3.rope import rope_partial

    g = torch.Generator().manual_seed(s)
    q = torch.randn(1, s, HEADS * D, generator=g).bfloat16()
    k = (torch.randn(1, s, HEADS * D, generator=g) + 2 * torch.randn(1, 1, HEADS * D, generator=g)).bfloat16()
    v = torch.randn(1, s, HEADS * D, generator=g).bfloat16()
    cos, sin = rope_partial(s, 96)
    return q, k, v, cos, sin


def _single_gpu_reference(q, k, v, cos, sin):
    from xgen_b200.attention import H3AttentionBackendB200
    from xgen_b200.ops import try_h3_partial_rope
    from xgen_b200.phaa import fp8_transport as fp8

    dev = torch.device("cuda", 0)
    s = q.shape[1]
    q, k, v = (t.to(dev).unflatten(-1, (HEADS, D)) for t in (q, k, v))
    with torch.no_grad():
        q, k = try_h3_partial_rope(q.contiguous(), k.contiguous(), cos.to(dev), sin.to(dev))
    rt = []
    for t in (q, k, v):  # one peer: wire encode + decode of every row
        out = torch.empty_like(t)
        fp8.decode(fp8.encode([t], D, 1), [out], D, 1)
        rt.append(out)
    att = H3AttentionBackendB200("sage")(*(t.transpose(1, 2) for t in rt))
    att = att.transpose(1, 2).contiguous()
    back = torch.empty_like(att)
    fp8.decode(fp8.encode([att], D, 1), [back], D, 1)
    return back.flatten(2).cpu()


def _worker(rank, world, port, q, k, v, cos, sin, results):
    import torch.distributed as dist
    from datetime import timedelta

    from xgen_b200.attention import H3AttentionBackendB200
    from xgen_b200.h3.sp_attention import sp_self_attention
    from xgen_b200.sp import comm
    from xgen_b200.sp.padding import get_pad_manager

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        s = q.shape[1]
        pad = get_pad_manager().set("mmh3_seq", s, world)
        shard = [comm.split_sequence(t, dist.group.WORLD, dim=1, pad=pad).to(dev) for t in (q, k, v)]
        cs = [comm.split_sequence(t, dist.group.WORLD, dim=0, pad=pad).to(dev) for t in (cos, sin)]
        out = sp_self_attention(*shard, tuple(cs), backend=H3AttentionBackendB200("sage"),
                                heads=HEADS, head_dim=D, sp_group=dist.group.WORLD, sp_size=world,
                                phaa_num=2, fp8_transport=True,
                                comm_stream=torch.cuda.Stream(device=dev))
        full = comm.gather_sequence(out, dist.group.WORLD, dim=1, pad=pad)
        torch.cuda.synchronize()
        results[rank] = full.cpu()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("s", [1022, 1024])
def test_sp2_fp8_phaa_matches_single_gpu(cuda_device, monkeypatch, s):
    """SP2 over NCCL equals one GPU bit for bit. The attention tail split is
    off on both sides (XGB_ATTN_TAIL_SPLIT=0, inherited by the spawned
    ranks): with it, a launch's split plan depends on how many heads it
    holds, and Sage split parts quantise P against their own running max."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    monkeypatch.setenv("XGB_ATTN_TAIL_SPLIT", "0")
    q, k, v, cos, sin = _inputs(s)
    expect = _single_gpu_reference(q, k, v, cos, sin)
    ctx = mp.get_context("spawn")
    results = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, k, v, cos, sin, results))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for r in range(2):
        assert torch.equal(results[r], expect), r
