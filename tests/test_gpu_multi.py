"""Token sharding on two GPUs over NCCL: each rank runs the library's kernels on its own
contiguous slice of tokens (shard.token_range; weights and modulation replicated), checks
its slice against the oracle, and the all-gathered slices equal the one-GPU result bit for
bit.  Covers the int8 GEMM (per-token quantisation in front of it) and the config-3 style
norm/mod/quant with a slice that straddles the boundary between two batch elements.
Skipped with fewer than two GPUs.  NVLink SHARP is off (NCCL_NVLS_ENABLE=0): nothing here
needs it, and a rank that fails an assertion then leaves no switch-side state behind."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_rows(dist, t, counts, dev):
    """all_gather_into_tensor of row slices of different lengths (padded to the longest)."""
    cap = max(counts)
    buf = torch.zeros((cap,) + tuple(t.shape[1:]), dtype=t.dtype, device=dev)
    buf[: t.shape[0]] = t
    out = torch.empty((len(counts) * cap,) + tuple(t.shape[1:]), dtype=t.dtype, device=dev)
    dist.all_gather_into_tensor(out, buf)
    return torch.cat([out[r * cap: r * cap + n] for r, n in enumerate(counts)])


def _worker(rank, world, port):
    import torch.distributed as dist

    from __graft_entry__ import load_package
    from oracle import oracle as O
    load_package()
    from thor_int8_gemm_b200 import ops, shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        # ---------------- int8 GEMM: 8191 x 3072 x 3072 (uneven slices), 1 % outlier channels
        M, N, K = 8191, 3072, 3072
        g = torch.Generator().manual_seed(5)
        x = torch.randn(M, K, generator=g)
        x[:, torch.randperm(K, generator=g)[: K // 100]] *= 20.0
        x = x.to(torch.bfloat16)
        w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
        bias = (torch.randn(N, generator=g) * 0.01).to(torch.bfloat16)
        a, b = shard.token_range(M, rank, world)
        counts = [hi - lo for lo, hi in (shard.token_range(M, r, world) for r in range(world))]
        wq, ws = ops.quant_rows(w.to(dev), "int8")
        xq, xs = ops.quant_rows(x[a:b].to(dev), "int8")
        out = ops.gemm_dequant(xq, wq, xs, ws, bias.to(dev))
        rows = np.unique(np.array([0, 1, (b - a) // 2, b - a - 1]))
        ridx = torch.from_numpy(rows).to(dev)
        q_ref, s_ref = O.quant_rows(x[a:b][torch.from_numpy(rows)].float().numpy(), O.QUANT_INT8)
        np.testing.assert_array_equal(xq[ridx].cpu().numpy(), q_ref)
        ref = O.gemm_i8_dequant(q_ref, wq.cpu().numpy(), s_ref, ws.cpu().numpy(), bias.float().numpy(), "bf16")
        np.testing.assert_array_equal(out[ridx].cpu().view(torch.int16).numpy().view(np.uint16), ref)
        full = _gather_rows(dist, out, counts, dev)
        if rank == 0:
            xq1, xs1 = ops.quant_rows(x.to(dev), "int8")
            one = ops.gemm_dequant(xq1, wq, xs1, ws, bias.to(dev))
            assert torch.equal(full, one), "gathered GEMM slices differ from the one-GPU result"

        # ---------------- norm/mod/quant: 3 batch elements of 700 tokens, D = 3072
        B, T, D = 3, 700, 3072
        x = torch.randn(B * T, D, generator=g).to(torch.bfloat16)
        shift = (torch.randn(B, D, generator=g) * 0.1).to(torch.bfloat16)
        scale = (torch.randn(B, D, generator=g) * 0.1).to(torch.bfloat16)
        a, b = shard.token_range(B * T, rank, world)
        counts = [hi - lo for lo, hi in (shard.token_range(B * T, r, world) for r in range(world))]
        idx = shard.mod_rows(a, b, rows_per_mod=T)
        assert len(np.unique(idx)) == 2, "each slice straddles a batch boundary"
        for kind, okind in (("fp8_e4m3", O.QUANT_FP8), ("int8", O.QUANT_INT8)):
            q, qs = ops.rms_mod_quant(x[a:b].to(dev), shift.to(dev), scale.to(dev),
                                      mod_index=torch.from_numpy(idx).to(dev), eps=1e-6, kind=kind)
            q_ref, qs_ref, _, _ = O.rms_mod_quant_per_token(x[a:b].float().numpy(), shift.float().numpy(),
                                                            scale.float().numpy(), mod_index=idx, eps=1e-6, kind=okind)
            codes = q.cpu().view(torch.uint8).numpy() if kind == "fp8_e4m3" else q.cpu().numpy()
            np.testing.assert_array_equal(codes, q_ref)
            np.testing.assert_array_equal(qs.cpu().numpy(), qs_ref)
            q_all = _gather_rows(dist, q.view(torch.uint8), counts, dev)
            s_all = _gather_rows(dist, qs.view(-1, 1), counts, dev)
            if rank == 0:
                q1, s1 = ops.rms_mod_quant(x.to(dev), shift.to(dev), scale.to(dev), rows_per_mod=T, eps=1e-6,
                                           kind=kind)
                assert torch.equal(q_all, q1.view(torch.uint8)) and torch.equal(s_all.view(-1), s1)
        assert ops.device_status(dev) == 0
        dist.barrier(device_ids=[rank])
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_two_gpu_token_sharding_nccl():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)
