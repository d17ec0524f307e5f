"""Token sharding across ranks, on CPU with the gloo backend (world size 2 and 3).

Each rank quantises its own token slice with the oracle (the same per-row
arithmetic the kernels implement) using its slice's modulation-row map; the
gathered slices must equal the unsharded result bit for bit, including a slice
that straddles the boundary between two batch elements.  The timing reduction
(max over ranks) is checked too.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O


def _shard():
    """The package's shard module (registers the package in spawned children too)."""
    from __graft_entry__ import load_package
    load_package()
    from thor_int8_gemm_b200 import shard
    return shard


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem():
    rng = np.random.default_rng(7)
    B, T, D = 2, 37, 256                     # 74 tokens: shards of 37 / 25 do not align to batch rows
    x = O.round_bf16(rng.standard_normal((B * T, D)).astype(np.float32))
    shift = O.round_bf16((rng.standard_normal((B, D)) * 0.1).astype(np.float32))
    scale = O.round_bf16((rng.standard_normal((B, D)) * 0.1).astype(np.float32))
    return x, shift, scale, T


def _worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    shard = _shard()
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, shift, scale, T = _problem()
        start, stop = shard.token_range(x.shape[0], rank, world)
        idx = shard.mod_rows(start, stop, rows_per_mod=T)
        q, qs, h, _ = O.rms_mod_quant_per_token(x[start:stop], shift, scale, mod_index=idx, eps=1e-6,
                                                kind=O.QUANT_FP8)
        # variable-size shards: pad to the largest, gather, trim
        n = torch.tensor([stop - start])
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, n)
        cap = int(max(s.item() for s in sizes))
        buf = torch.zeros(cap, x.shape[1] + 4, dtype=torch.uint8)
        buf[: stop - start, : x.shape[1]] = torch.from_numpy(q)
        buf[: stop - start, x.shape[1]:] = torch.from_numpy(qs.view(np.uint8).reshape(-1, 4))
        parts = [torch.zeros_like(buf) for _ in range(world)]
        dist.all_gather(parts, buf)
        t = shard.max_over_ranks(float(rank) + 0.5)
        if rank == 0:
            rows = torch.cat([p[: int(s.item())] for p, s in zip(parts, sizes)]).numpy()
            out_q.put((rows, t))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_token_shards_reassemble_bit_exact(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    import queue
    rows = None
    for _ in range(120):
        try:
            rows, t = q.get(timeout=1)
            break
        except queue.Empty:
            assert all(p.exitcode in (None, 0) for p in procs), [p.exitcode for p in procs]
    assert rows is not None, "no result from rank 0"
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    x, shift, scale, T = _problem()
    q_ref, qs_ref, _, _ = O.rms_mod_quant_per_token(x, shift, scale, rows_per_mod=T, eps=1e-6, kind=O.QUANT_FP8)
    D = x.shape[1]
    np.testing.assert_array_equal(rows[:, :D], q_ref)
    np.testing.assert_array_equal(rows[:, D:].copy().view(np.float32).reshape(-1), qs_ref)
    assert t == world - 1 + 0.5


def test_token_range_partitions():
    shard = _shard()
    for M in (0, 1, 7, 112640, 112641):
        for world in (1, 2, 3, 8):
            spans = [shard.token_range(M, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == M
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.token_range(10, 2, 2)


def test_mod_rows():
    shard = _shard()
    np.testing.assert_array_equal(shard.mod_rows(50, 60, rows_per_mod=56), [0] * 6 + [1] * 4)
    full = np.array([3, 1, 4, 1, 5, 9], np.int32)
    np.testing.assert_array_equal(shard.mod_rows(2, 5, mod_index=full), [4, 1, 5])
    with pytest.raises(ValueError):
        shard.mod_rows(0, 4)
